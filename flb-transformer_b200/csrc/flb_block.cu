// FLB block cells of the wavefront grid, forward (inference), bf16 storage, fp32 accumulation.
//
// The FLB model's grid (layers L x positions S, dependencies top (-1,0) -> port 0, left (0,-1)
// -> port 1, bottom-left (1,-1) -> port 2, four ports) is evaluated tick by tick on the host's
// launch stream: cell (l, t) runs at tick T = l + 2t, so a tick's cells are l = l0, l0+2, ...
// with t = (T - l) / 2, and their flat grid rows l*S + t form an arithmetic progression of step
// 2S - 1. Per tick, for all its cells at once:
//   1. LayerNorm (fp32 statistics) of the left and bottom-left neighbours   [own kernel]
//   2. lat_prior = P_lat LN(left), fdbk_prior = P_fb LN(diag)              [strided GEMMs]
//   3. lat' = lat_prior * sigmoid(G_L fdbk_prior + b_L)                    [GEMM + own kernel]
//   4. x'   = top * sigmoid(G_X lat' + b_X)                                [GEMM + own kernel]
//   5. q|k|v of the three tokens [x', lat', fdbk_prior]                    [one GEMM, N = 3D]
//   6. additive attention over the 3 tokens per head                       [own kernel]
//   7. o = W_o att                                                          [GEMM]
//   8. h_x = o0 + top, h_lat = o1 + lat_prior, h_fdbk = o2 + fdbk_prior,
//      aux = (lat_prior - h_lat)^2 + (fdbk_prior - h_fdbk)^2, written into the four port grids
//                                                                            [own kernel]
// The layers of a tick are two apart, so each GEMM is one cuBLAS strided-batched call over the
// tick's cells with the weights read in place from [L, N, K] stacks (stride two layers).
// Math as models/FLB_Model.py:32-96 (FLB_Attention_Layer, FLB_Block) with the reference's
// attention (kernels/additive_attention.py: s = sum_d v_a tanh(q + k) / sqrt(d_h), softmax,
// P @ V) over the 3 tokens.
#include <cuda_bf16.h>

#include "blas.cuh"
#include "common.cuh"

namespace flb {

namespace {

using bf16 = __nv_bfloat16;

struct Tick {
  int T, l0, n;  // tick, first layer, cells
};

__host__ __device__ inline Tick tick_of(int T, int L, int S) {
  int l0 = T - 2 * (S - 1);
  if (l0 < (T & 1)) l0 = T & 1;
  int l1 = T < L - 1 ? T : L - 1;
  if (((l1 - T) & 1) != 0) --l1;
  return Tick{T, l0, l1 >= l0 ? (l1 - l0) / 2 + 1 : 0};
}

__device__ __forceinline__ int64_t cell_row(int l, int t, int S) { return (int64_t)l * S + t; }

// 1. LayerNorm of the left (which 0) and bottom-left (which 1) neighbours; zero boundary rows
//    (t = 0, or l = L-1 for the bottom-left) normalise to the LayerNorm bias as in torch.
//    One warp per row, the row held in registers as 16-byte chunks (D <= 1024).
constexpr int kMaxChunks = 4;  // per lane: 4 x 8 bf16 -> D <= 32 * 32 = 1024

__global__ void blk_ln_kernel(const bf16* __restrict__ g_left, const bf16* __restrict__ g_diag,
                              const float* __restrict__ lw0, const float* __restrict__ lb0,
                              const float* __restrict__ lw1, const float* __restrict__ lb1,
                              bf16* __restrict__ out, int T, int l0, int n, int L, int S, int B,
                              int D, float eps) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  if (row >= 2 * n * B) return;
  const int which = row / (n * B), i = (row / B) % n, b = row % B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const bf16* src = nullptr;
  if (which == 0 && t > 0) src = g_left + (cell_row(l, t - 1, S) * B + b) * D;
  if (which == 1 && t > 0 && l + 1 < L) src = g_diag + (cell_row(l + 1, t - 1, S) * B + b) * D;
  const int nch = D / 8;
  float v[kMaxChunks][8];
  float s = 0.f, ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (src && c < nch) raw = reinterpret_cast<const uint4*>(src)[c];
    const uint32_t* r = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[e]));
      v[k][2 * e] = f.x;
      v[k][2 * e + 1] = f.y;
      s += f.x + f.y;
      ss += f.x * f.x + f.y * f.y;
    }
  }
  s = warp_sum(s);
  ss = warp_sum(ss);
  const float mean = s / D;
  const float rstd = rsqrtf(fmaxf(ss / D - mean * mean, 0.f) + eps);
  const float4* w4 = reinterpret_cast<const float4*>((which ? lw1 : lw0) + (int64_t)l * D);
  const float4* b4 = reinterpret_cast<const float4*>((which ? lb1 : lb0) + (int64_t)l * D);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)row * D);
#pragma unroll
  for (int k = 0; k < kMaxChunks; ++k) {
    const int c = lane + 32 * k;
    if (c >= nch) break;
    const float4 wa = w4[2 * c], wb = w4[2 * c + 1], ba = b4[2 * c], bb = b4[2 * c + 1];
    const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    const float bv[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __nv_bfloat162 h = __floats2bfloat162_rn((v[k][2 * e] - mean) * rstd * wv[2 * e] + bv[2 * e],
                                                     (v[k][2 * e + 1] - mean) * rstd * wv[2 * e + 1] + bv[2 * e + 1]);
      o[e] = *reinterpret_cast<const uint32_t*>(&h);
    }
    dst[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// the top neighbour of cell (l, t), batch row b: port 0 of row l-1, or x at position t for l = 0
__device__ __forceinline__ const bf16* top_row(const bf16* g0, const bf16* x, int l, int t, int b,
                                               int S, int B, int D) {
  return l > 0 ? g0 + (cell_row(l - 1, t, S) * B + b) * D : x + ((int64_t)b * S + t) * D;
}

// 3./4. gates: dst = m * sigmoid(z + bias[l]) with m = lat_prior (mode 0) or the top neighbour
//    (mode 1); dst rows have a pitch of 3D (a token slot of the [cells, B, 3, D] token tensor).
//    Grid: x over bf16 pairs of a row, y over the tick's (cell, batch) rows.
__global__ void blk_gate_kernel(const bf16* __restrict__ z, const float* __restrict__ bias,
                                const bf16* __restrict__ m, const bf16* __restrict__ g0,
                                const bf16* __restrict__ x, int mode, bf16* __restrict__ dst,
                                int T, int l0, int S, int B, int D) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= D / 2) return;
  const int rb = blockIdx.y;  // i * B + b
  const int i = rb / B, b = rb - i * B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const float2 zz = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(z + (int64_t)rb * D)[j]);
  const bf16* mrow = mode == 0 ? m + (int64_t)rb * D : top_row(g0, x, l, t, b, S, B, D);
  const float2 mm = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(mrow)[j]);
  const float2 bl = reinterpret_cast<const float2*>(bias + (int64_t)l * D)[j];
  const float s0 = 1.f / (1.f + __expf(-(zz.x + bl.x)));
  const float s1 = 1.f / (1.f + __expf(-(zz.y + bl.y)));
  reinterpret_cast<__nv_bfloat162*>(dst + (int64_t)rb * 3 * D)[j] =
      __floats2bfloat162_rn(mm.x * s0, mm.y * s1);
}

// 6. additive attention over the 3 tokens, one warp per (cell, batch row, head). qkv rows are
//    [cells, B, 3 tokens] of [q | k | v] (3D wide); att rows [cells, B, 3 tokens] of D with the
//    heads side by side (the reference's transpose(1, 2).view(B, 3, D)).
__global__ void blk_attn3_kernel(const bf16* __restrict__ qkv, const float* __restrict__ v_a,
                                 bf16* __restrict__ att, int l0, int n, int B, int D, int H) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.x * warps + (threadIdx.x >> 5);
  if (task >= n * B * H) return;
  const int h = task % H;
  const int64_t rb = task / H;  // i * B + b
  const int i = (int)(rb / B);
  const int dh = D / H;
  const float* w = v_a + ((int64_t)(l0 + 2 * i) * H + h) * dh;
  const bf16* base = qkv + rb * 3 * (3 * D) + h * dh;  // token r row: base + r * 3D
  float s[3][3];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int c = 0; c < 3; ++c) s[a][c] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {  // dh <= 128
    const int d = lane + 32 * kk;
    if (d >= dh) break;
    float q[3], k[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      q[r] = __bfloat162float(base[r * 3 * D + d]);
      k[r] = __bfloat162float(base[r * 3 * D + D + d]);
    }
    const float wd = w[d];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int c = 0; c < 3; ++c) s[a][c] = fmaf(wd, tanh_approx(q[a] + k[c]), s[a][c]);
  }
  const float scale = rsqrtf((float)dh);
  float p[3][3];
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      s[a][c] = warp_sum(s[a][c]) * scale;
      m = fmaxf(m, s[a][c]);
    }
    float l = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      p[a][c] = __expf(s[a][c] - m);
      l += p[a][c];
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) p[a][c] /= l;
  }
  bf16* out = att + rb * 3 * D + h * dh;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int d = lane + 32 * kk;
    if (d >= dh) break;
    float v[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) v[r] = __bfloat162float(base[r * 3 * D + 2 * D + d]);
#pragma unroll
    for (int a = 0; a < 3; ++a)
      out[a * D + d] = __float2bfloat16_rn(p[a][0] * v[0] + p[a][1] * v[1] + p[a][2] * v[2]);
  }
}

// 8. residuals and the auxiliary loss, written into the four port grids at the tick's cells.
//    Grid: x over bf16 pairs of a row, y over the tick's (cell, batch) rows.
__global__ void blk_out_kernel(const bf16* __restrict__ o, const bf16* __restrict__ lat_prior,
                               const bf16* __restrict__ tok, const bf16* __restrict__ x,
                               bf16* __restrict__ grids, int64_t port_stride, int T, int l0,
                               int S, int B, int D) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= D / 2) return;
  const int rb = blockIdx.y;
  const int i = rb / B, b = rb - i * B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  auto ld2 = [&](const bf16* p) {
    return __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(p)[j]);
  };
  const int64_t r3 = (int64_t)rb * 3;
  const float2 o0 = ld2(o + r3 * D), o1 = ld2(o + (r3 + 1) * D), o2 = ld2(o + (r3 + 2) * D);
  const float2 top = ld2(top_row(grids, x, l, t, b, S, B, D));
  const float2 lp = ld2(lat_prior + (int64_t)rb * D), fp = ld2(tok + (r3 + 2) * D);
  // the outputs as stored (bf16), as the aux term sees them
  const __nv_bfloat162 hx = __floats2bfloat162_rn(o0.x + top.x, o0.y + top.y);
  const __nv_bfloat162 hl = __floats2bfloat162_rn(o1.x + lp.x, o1.y + lp.y);
  const __nv_bfloat162 hf = __floats2bfloat162_rn(o2.x + fp.x, o2.y + fp.y);
  const float2 hlf = __bfloat1622float2(hl), hff = __bfloat1622float2(hf);
  const float ax = (lp.x - hlf.x) * (lp.x - hlf.x) + (fp.x - hff.x) * (fp.x - hff.x);
  const float ay = (lp.y - hlf.y) * (lp.y - hlf.y) + (fp.y - hff.y) * (fp.y - hff.y);
  const int64_t off = (cell_row(l, t, S) * B + b) * D;
  reinterpret_cast<__nv_bfloat162*>(grids + off)[j] = hx;
  reinterpret_cast<__nv_bfloat162*>(grids + port_stride + off)[j] = hl;
  reinterpret_cast<__nv_bfloat162*>(grids + 2 * port_stride + off)[j] = hf;
  reinterpret_cast<__nv_bfloat162*>(grids + 3 * port_stride + off)[j] = __floats2bfloat162_rn(ax, ay);
}

constexpr size_t kBlkBlasWs = 32u << 20;

struct BlockWs {
  bf16 *ln, *lat, *tok, *z, *qkv, *att, *o;
  void* blas;
};

size_t block_ws_layout(int64_t nmax, int64_t B, int64_t D, BlockWs* w, void* base) {
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t rowb = (size_t)nmax * B * D * sizeof(bf16);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += al(bytes);
    return o;
  };
  const size_t o_ln = take(2 * rowb), o_lat = take(rowb), o_tok = take(3 * rowb), o_z = take(rowb),
               o_qkv = take(9 * rowb), o_att = take(3 * rowb), o_o = take(3 * rowb),
               o_blas = take(kBlkBlasWs);
  if (w && base) {
    uint8_t* p = reinterpret_cast<uint8_t*>(base);
    w->ln = (bf16*)(p + o_ln);
    w->lat = (bf16*)(p + o_lat);
    w->tok = (bf16*)(p + o_tok);
    w->z = (bf16*)(p + o_z);
    w->qkv = (bf16*)(p + o_qkv);
    w->att = (bf16*)(p + o_att);
    w->o = (bf16*)(p + o_o);
    w->blas = p + o_blas;
  }
  return off;
}

int64_t max_cells_per_tick(int64_t L, int64_t S) {
  const int64_t a = (L + 1) / 2;
  return a < S ? a : S;
}

}  // namespace

size_t block_grid_workspace_bytes(int64_t L, int64_t S, int64_t B, int64_t D) {
  return block_ws_layout(max_cells_per_tick(L, S), B, D, nullptr, nullptr);
}

int block_grid_fwd(const flb_block_weights* W, const void* x, void* grids, int64_t L, int64_t S,
                   int64_t B, int64_t D, int64_t H, float eps, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
  BlockWs w;
  block_ws_layout(max_cells_per_tick(L, S), B, D, &w, ws);
  cublasHandle_t hb;
  int st = blas(s, w.blas, kBlkBlasWs, &hb);
  if (st != FLB_OK) return st;
  const bf16* xb = reinterpret_cast<const bf16*>(x);
  bf16* g = reinterpret_cast<bf16*>(grids);
  const int64_t port_stride = (L * S + L) * B * D;  // the engine's grids keep L dock rows
  const long long DD = D * D, BD = B * D;
  const int Li = (int)L, Si = (int)S, Bi = (int)B, Di = (int)D, Hi = (int)H;
  const int ticks = (int)(L + 2 * S - 2);
  int launches = 0;
  for (int T = 0; T < ticks; ++T) {
    const Tick tk = tick_of(T, Li, Si);
    const int n = tk.n, l0 = tk.l0;
    if (n == 0) continue;
    const int rows_ln = 2 * n * Bi;
    blk_ln_kernel<<<(rows_ln + 7) / 8, 256, 0, s>>>(g + port_stride, g + 2 * port_stride,
                                                    W->ln_lat_w, W->ln_lat_b, W->ln_fdbk_w,
                                                    W->ln_fdbk_b, w.ln, T, l0, n, Li, Si, Bi, Di,
                                                    eps);
    // priors: lat_prior -> w.lat [n, B, D]; fdbk_prior -> token slot 2 (row pitch 3D)
    const bf16* Wpl = reinterpret_cast<const bf16*>(W->w_prior_lat) + (int64_t)l0 * DD;
    const bf16* Wpf = reinterpret_cast<const bf16*>(W->w_prior_fdbk) + (int64_t)l0 * DD;
    const bf16* Wgl = reinterpret_cast<const bf16*>(W->w_gate_l) + (int64_t)l0 * DD;
    const bf16* Wgx = reinterpret_cast<const bf16*>(W->w_gate_x) + (int64_t)l0 * DD;
    const bf16* Wqkv = reinterpret_cast<const bf16*>(W->w_qkv) + (int64_t)l0 * 3 * DD;
    const bf16* Wo = reinterpret_cast<const bf16*>(W->w_o) + (int64_t)l0 * DD;
    if ((st = gemm_rm(hb, false, true, Bi, Di, Di, w.ln, Di, BD, Wpl, Di, 2 * DD, w.lat, Di, BD, n,
                      0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    if ((st = gemm_rm(hb, false, true, Bi, Di, Di, w.ln + n * BD, Di, BD, Wpf, Di, 2 * DD,
                      w.tok + 2 * D, 3 * Di, 3 * BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    // lateral gate
    if ((st = gemm_rm(hb, false, true, Bi, Di, Di, w.tok + 2 * D, 3 * Di, 3 * BD, Wgl, Di, 2 * DD,
                      w.z, Di, BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    const dim3 ew_grid((unsigned)((D / 2 + 127) / 128), (unsigned)(n * Bi));
    blk_gate_kernel<<<ew_grid, 128, 0, s>>>(w.z, W->b_gate_l, w.lat, g, xb, 0, w.tok + D, T, l0,
                                            Si, Bi, Di);
    // sensory gate
    if ((st = gemm_rm(hb, false, true, Bi, Di, Di, w.tok + D, 3 * Di, 3 * BD, Wgx, Di, 2 * DD, w.z,
                      Di, BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    blk_gate_kernel<<<ew_grid, 128, 0, s>>>(w.z, W->b_gate_x, nullptr, g, xb, 1, w.tok, T, l0, Si,
                                            Bi, Di);
    // q | k | v of the 3 tokens: [n, 3B, D] x [3D, D]^T
    if ((st = gemm_rm(hb, false, true, 3 * Bi, 3 * Di, Di, w.tok, Di, 3 * BD, Wqkv, Di, 6 * DD,
                      w.qkv, 3 * Di, 9 * BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    const int tasks = n * Bi * Hi;
    blk_attn3_kernel<<<(tasks + 7) / 8, 256, 0, s>>>(w.qkv, W->v_a, w.att, l0, n, Bi, Di, Hi);
    if ((st = gemm_rm(hb, false, true, 3 * Bi, Di, Di, w.att, Di, 3 * BD, Wo, Di, 2 * DD, w.o, Di,
                      3 * BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    blk_out_kernel<<<ew_grid, 128, 0, s>>>(w.o, w.lat, w.tok, xb, g, port_stride, T, l0, Si, Bi,
                                           Di);
    launches += 6;  // own kernels (the GEMMs are cuBLAS's)
  }
  count_launches(launches);
  return check_cuda(cudaGetLastError(), "flb block grid launch");
}

}  // namespace flb
