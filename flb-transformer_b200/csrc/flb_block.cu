// FLB block cells of the wavefront grid, forward (inference), bf16 storage, fp32 accumulation.
//
// The FLB model's grid (layers L x positions S, dependencies top (-1,0) -> port 0, left (0,-1)
// -> port 1, bottom-left (1,-1) -> port 2, four ports) is evaluated tick by tick on the host's
// launch stream: cell (l, t) runs at tick T = l + 2t, so a tick's cells are l = l0, l0+2, ...
// with t = (T - l) / 2, and their flat grid rows l*S + t form an arithmetic progression of step
// 2S - 1. Per tick, for all its cells at once:
//   1. LayerNorm (fp32 statistics) of the left and bottom-left neighbours   [fused into the
//      output kernel (8.) of the ticks that produce them; own kernel in the backward's recompute]
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

#include <algorithm>
#include <utility>
#include <mutex>

#include "blas.cuh"
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace flb {

namespace {

using bf16 = __nv_bfloat16;

// Programmatic dependent launch: a kernel launched with launch_pdl may be scheduled while its
// predecessor in the stream is still draining (its launch latency hides behind the predecessor's
// tail); it waits in pdl_wait, before touching the predecessor's outputs, until that grid has
// completed and its memory is visible. Without the launch attribute pdl_wait returns at once.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

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

// LayerNorm of one row by one warp (fp32 statistics over the bf16 values; src null = a zero
// row, which normalises to beta), the row held in registers as 16-byte chunks (D <= 1024).
__device__ __forceinline__ void ln_warp_row(const bf16* __restrict__ src,
                                            const float* __restrict__ gamma,
                                            const float* __restrict__ beta,
                                            bf16* __restrict__ out, int lane, int D, float eps) {
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
  const float4* w4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  uint4* dst = reinterpret_cast<uint4*>(out);
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

__global__ void blk_ln_kernel(const bf16* __restrict__ g_left, const bf16* __restrict__ g_diag,
                              const float* __restrict__ lw0, const float* __restrict__ lb0,
                              const float* __restrict__ lw1, const float* __restrict__ lb1,
                              bf16* __restrict__ out, int T, int l0, int n, int L, int S, int B,
                              int D, float eps) {
  pdl_wait();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  if (row >= 2 * n * B) return;
  const int which = row / (n * B), i = (row / B) % n, b = row % B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const bf16* src = nullptr;
  if (which == 0 && t > 0) src = g_left + (cell_row(l, t - 1, S) * B + b) * D;
  if (which == 1 && t > 0 && l + 1 < L) src = g_diag + (cell_row(l + 1, t - 1, S) * B + b) * D;
  ln_warp_row(src, (which ? lw1 : lw0) + (int64_t)l * D, (which ? lb1 : lb0) + (int64_t)l * D,
              out + (int64_t)row * D, lane, D, eps);
}

// The training forward's LayerNorm planes (PL_LN_LEFT, PL_LN_DIAG: [which][cell][B][D], rows in
// that order), all cells at once after the tick loop, from the port grids the forward wrote: the
// same LayerNorms of the same bf16 values that the output kernels put in the ring for the
// consumer ticks. One warp per row.
__global__ void blk_ln_planes_kernel(const bf16* __restrict__ g_left, const bf16* __restrict__ g_diag,
                                     const float* __restrict__ lw0, const float* __restrict__ lb0,
                                     const float* __restrict__ lw1, const float* __restrict__ lb1,
                                     bf16* __restrict__ out, int L, int S, int B, int D, float eps) {
  pdl_wait();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  const int64_t per = (int64_t)L * S * B;
  if (row >= 2 * per) return;
  const int which = (int)(row / per);
  const int64_t cell = (row - which * per) / B;
  const int b = (int)(row % B);
  const int l = (int)(cell / S), t = (int)(cell % S);
  const bf16* src = nullptr;
  if (which == 0 && t > 0) src = g_left + (cell_row(l, t - 1, S) * B + b) * D;
  if (which == 1 && t > 0 && l + 1 < L) src = g_diag + (cell_row(l + 1, t - 1, S) * B + b) * D;
  ln_warp_row(src, (which ? lw1 : lw0) + (int64_t)l * D, (which ? lb1 : lb0) + (int64_t)l * D,
              out + row * D, lane, D, eps);
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
                                int64_t cs, int T, int l0, int S, int B, int D) {
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= D / 2) return;
  const int rb = blockIdx.y;  // i * B + b
  const int i = rb / B, b = rb - i * B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const int64_t cr = (int64_t)i * cs + (int64_t)b * D;  // row of a one-unit cell array
  const float2 zz = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(z + cr)[j]);
  const bf16* mrow = mode == 0 ? m + cr : top_row(g0, x, l, t, b, S, B, D);
  const float2 mm = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(mrow)[j]);
  const float2 bl = reinterpret_cast<const float2*>(bias + (int64_t)l * D)[j];
  const float s0 = 1.f / (1.f + __expf(-(zz.x + bl.x)));
  const float s1 = 1.f / (1.f + __expf(-(zz.y + bl.y)));
  reinterpret_cast<__nv_bfloat162*>(dst + 3 * cr)[j] = __floats2bfloat162_rn(mm.x * s0, mm.y * s1);
}

// 6. additive attention over the 3 tokens, one warp per (cell, batch row, head). qkv rows are
//    [cells, B, 3 tokens] of [q | k | v] (3D wide); att rows [cells, B, 3 tokens] of D with the
//    heads side by side (the reference's transpose(1, 2).view(B, 3, D)). qkv is read through L2
//    (ld.global.cg): in the persistent forward other CTAs of the same launch wrote it.
__device__ __forceinline__ float ld_bf16_cg(const bf16* p) {
  return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(p))));
}

__device__ __forceinline__ void attn3_task(const bf16* __restrict__ qkv, const float* __restrict__ v_a,
                                           bf16* __restrict__ att, int64_t cs, int l0, int B,
                                           int D, int H, int task, int lane) {
  const int h = task % H;
  const int64_t rb = task / H;  // i * B + b
  const int i = (int)(rb / B);
  const int dh = D / H;
  const float* w = v_a + ((int64_t)(l0 + 2 * i) * H + h) * dh;
  const int64_t cr = (int64_t)i * cs + (rb - (int64_t)i * B) * D;  // one-unit row of (cell, b)
  const bf16* base = qkv + 9 * cr + h * dh;  // token r row: base + r * 3D
  float s[3][3], vv[4][3];
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
      q[r] = ld_bf16_cg(base + r * 3 * D + d);
      k[r] = ld_bf16_cg(base + r * 3 * D + D + d);
      vv[kk][r] = ld_bf16_cg(base + r * 3 * D + 2 * D + d);  // V with Q, K: one round trip
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
  bf16* out = att + 3 * cr + h * dh;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int d = lane + 32 * kk;
    if (d >= dh) break;
    const float* v = vv[kk];
#pragma unroll
    for (int a = 0; a < 3; ++a)
      out[a * D + d] = __float2bfloat16_rn(p[a][0] * v[0] + p[a][1] * v[1] + p[a][2] * v[2]);
  }
}

__global__ void blk_attn3_kernel(const bf16* __restrict__ qkv, const float* __restrict__ v_a,
                                 bf16* __restrict__ att, int64_t cs, int l0, int n, int B, int D,
                                 int H) {
  pdl_wait();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.x * warps + (threadIdx.x >> 5);
  if (task >= n * B * H) return;
  attn3_task(qkv, v_a, att, cs, l0, B, D, H, task, lane);
}

// 8. residuals and the auxiliary loss into the four port grids, with the next ticks'
//    LayerNorms fused in: a block per (cell, batch row) writes the four port outputs of the
//    row and normalises the two it has just produced for their consumers, so that no LayerNorm
//    launch opens a forward tick:
//    h_lat of cell (l, t) is the left input of (l, t+1) at tick T+2 (norm_lat of layer l),
//    h_fdbk the bottom-left input of (l-1, t+1) at tick T+1 (norm_fdbk of layer l-1). They go
//    to a ring of three LayerNorm buffers [slot = consumer tick % 3][left | diag][layer][B][D],
//    which blk_ln_init_kernel fills with the LayerNorm biases (the normalised zero boundary rows,
//    which no producer overwrites before their consumer's tick). Statistics over the bf16
//    values the port grids hold.
// One (cell, batch row) per block, one 16-byte chunk (8 features) per thread; LayerNorm
// statistics by warp sums and a fixed-order sum over the block's warps.
constexpr int kOutLnMaxWarps = 4;  // D <= 1024: 128 chunks

__device__ __forceinline__ void ln_chunk_store(const float (&v)[8], float mean, float rstd,
                                               const float4 (&w)[2], const float4 (&bb)[2],
                                               bf16* dst, int c) {
  const float wv[8] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w};
  const float bv[8] = {bb[0].x, bb[0].y, bb[0].z, bb[0].w, bb[1].x, bb[1].y, bb[1].z, bb[1].w};
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 h = __floats2bfloat162_rn((v[2 * e] - mean) * rstd * wv[2 * e] + bv[2 * e],
                                                   (v[2 * e + 1] - mean) * rstd * wv[2 * e + 1] + bv[2 * e + 1]);
    o[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  reinterpret_cast<uint4*>(dst)[c] = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void blk_out_ln_kernel(const bf16* __restrict__ o, const bf16* __restrict__ lat_prior,
                                  const bf16* __restrict__ tok, int64_t cs, const bf16* __restrict__ x,
                                  bf16* __restrict__ grids, int64_t port_stride,
                                  bf16* __restrict__ lnr, const float* __restrict__ lw0,
                                  const float* __restrict__ lb0, const float* __restrict__ lw1,
                                  const float* __restrict__ lb1, float eps, int T, int l0, int n,
                                  int L, int S, int B, int D) {
  __shared__ float red[4][kOutLnMaxWarps];  // per warp: sum and sum of squares of h_lat, h_fdbk
  const int row = blockIdx.x;               // i * B + b
  const int c = threadIdx.x, warp = c >> 5, lane = c & 31, nw = blockDim.x >> 5;
  const int i = row / B, b = row - i * B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const int nch = D / 8;
  const bool act = c < nch;
  // the LayerNorm parameters do not depend on the previous kernel: load them before the wait
  float4 wl[2], bl[2], wf[2], bf[2];
  if (act) {
    const float4* p0 = reinterpret_cast<const float4*>(lw0 + (int64_t)l * D) + 2 * c;
    const float4* p1 = reinterpret_cast<const float4*>(lb0 + (int64_t)l * D) + 2 * c;
    wl[0] = __ldg(p0); wl[1] = __ldg(p0 + 1); bl[0] = __ldg(p1); bl[1] = __ldg(p1 + 1);
    if (l >= 1) {
      const float4* p2 = reinterpret_cast<const float4*>(lw1 + (int64_t)(l - 1) * D) + 2 * c;
      const float4* p3 = reinterpret_cast<const float4*>(lb1 + (int64_t)(l - 1) * D) + 2 * c;
      wf[0] = __ldg(p2); wf[1] = __ldg(p2 + 1); bf[0] = __ldg(p3); bf[1] = __ldg(p3 + 1);
    }
  }
  pdl_wait();
  const int64_t r3 = (int64_t)row * 3;
  const int64_t off = (cell_row(l, t, S) * B + b) * D;
  float hl[8], hf[8];
  float sl = 0.f, ssl = 0.f, sf = 0.f, ssf = 0.f;
  if (act) {
    auto ld8 = [&](const bf16* p, float (&f)[8]) {
      const uint4 u = reinterpret_cast<const uint4*>(p)[c];
      const uint32_t* r = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[e]));
        f[2 * e] = v.x;
        f[2 * e + 1] = v.y;
      }
    };
    float o0[8], o1[8], o2[8], tp[8], lp[8], fp[8];
    ld8(o + r3 * D, o0);
    ld8(o + (r3 + 1) * D, o1);
    ld8(o + (r3 + 2) * D, o2);
    ld8(top_row(grids, x, l, t, b, S, B, D), tp);
    const int64_t cr = (int64_t)i * cs + (int64_t)b * D;  // row of a one-unit cell array
    ld8(lat_prior + cr, lp);
    ld8(tok + 3 * cr + 2 * D, fp);
    uint32_t px[4], pl[4], pf[4], pa[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      // the outputs as stored (bf16), as the aux term and the next LayerNorms see them
      const __nv_bfloat162 hx = __floats2bfloat162_rn(o0[2 * e] + tp[2 * e], o0[2 * e + 1] + tp[2 * e + 1]);
      const __nv_bfloat162 hl2 = __floats2bfloat162_rn(o1[2 * e] + lp[2 * e], o1[2 * e + 1] + lp[2 * e + 1]);
      const __nv_bfloat162 hf2 = __floats2bfloat162_rn(o2[2 * e] + fp[2 * e], o2[2 * e + 1] + fp[2 * e + 1]);
      const float2 hlf = __bfloat1622float2(hl2), hff = __bfloat1622float2(hf2);
      const float ax = (lp[2 * e] - hlf.x) * (lp[2 * e] - hlf.x) + (fp[2 * e] - hff.x) * (fp[2 * e] - hff.x);
      const float ay = (lp[2 * e + 1] - hlf.y) * (lp[2 * e + 1] - hlf.y) +
                       (fp[2 * e + 1] - hff.y) * (fp[2 * e + 1] - hff.y);
      const __nv_bfloat162 a2 = __floats2bfloat162_rn(ax, ay);
      px[e] = *reinterpret_cast<const uint32_t*>(&hx);
      pl[e] = *reinterpret_cast<const uint32_t*>(&hl2);
      pf[e] = *reinterpret_cast<const uint32_t*>(&hf2);
      pa[e] = *reinterpret_cast<const uint32_t*>(&a2);
      hl[2 * e] = hlf.x;
      hl[2 * e + 1] = hlf.y;
      hf[2 * e] = hff.x;
      hf[2 * e + 1] = hff.y;
      sl += hlf.x + hlf.y;
      ssl += hlf.x * hlf.x + hlf.y * hlf.y;
      sf += hff.x + hff.y;
      ssf += hff.x * hff.x + hff.y * hff.y;
    }
    reinterpret_cast<uint4*>(grids + off)[c] = make_uint4(px[0], px[1], px[2], px[3]);
    reinterpret_cast<uint4*>(grids + port_stride + off)[c] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
    reinterpret_cast<uint4*>(grids + 2 * port_stride + off)[c] = make_uint4(pf[0], pf[1], pf[2], pf[3]);
    reinterpret_cast<uint4*>(grids + 3 * port_stride + off)[c] = make_uint4(pa[0], pa[1], pa[2], pa[3]);
  }
  if (t + 1 >= S) return;  // the last column has no consumers (block-uniform)
  sl = warp_sum(sl);
  ssl = warp_sum(ssl);
  sf = warp_sum(sf);
  ssf = warp_sum(ssf);
  if (lane == 0) {
    red[0][warp] = sl;
    red[1][warp] = ssl;
    red[2][warp] = sf;
    red[3][warp] = ssf;
  }
  __syncthreads();
  if (!act) return;
  float tot[4] = {0.f, 0.f, 0.f, 0.f};
  for (int w = 0; w < nw; ++w)
#pragma unroll
    for (int q = 0; q < 4; ++q) tot[q] += red[q][w];
  const int64_t LBD = (int64_t)L * B * D;
  {
    const float mean = tot[0] / D;
    const float rstd = rsqrtf(fmaxf(tot[1] / D - mean * mean, 0.f) + eps);
    ln_chunk_store(hl, mean, rstd, wl, bl,
                   lnr + (int64_t)((T + 2) % 3) * 2 * LBD + ((int64_t)l * B + b) * D, c);
  }
  if (l >= 1) {
    const float mean = tot[2] / D;
    const float rstd = rsqrtf(fmaxf(tot[3] / D - mean * mean, 0.f) + eps);
    ln_chunk_store(hf, mean, rstd, wf, bf,
                   lnr + (int64_t)((T + 1) % 3) * 2 * LBD + LBD + ((int64_t)(l - 1) * B + b) * D, c);
  }
}

// The LayerNorm ring's initial contents: every row the LayerNorm bias of its layer (the
// normalised zero row). Grid: x over bf16 pairs, y over [slot][left | diag][layer][batch] rows.
__global__ void blk_ln_init_kernel(bf16* __restrict__ lnr, const float* __restrict__ lb0,
                                   const float* __restrict__ lb1, int L, int B, int D) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= D / 2) return;
  const int rowi = blockIdx.y;  // ((slot * 2 + which) * L + l) * B + b
  const int l = (rowi / B) % L, which = (rowi / (B * L)) % 2;
  const float2 bv = reinterpret_cast<const float2*>((which ? lb1 : lb0) + (int64_t)l * D)[j];
  reinterpret_cast<__nv_bfloat162*>(lnr + (int64_t)rowi * D)[j] = __floats2bfloat162_rn(bv.x, bv.y);
}

// Planes of a training step's per-cell tensors, kept in one buffer (flb_block_grid_saved_bytes):
// plane p holds, for every grid cell (l*S + t) in order, plane_units(p) units of B x D bf16. The forward
// fills planes 0-7 with its intermediates [ln_left | ln_diag | lat_prior | tokens x' lat'
// fdbk_prior | z_l | z_x | q|k|v | att] (its GEMMs and kernels write planes 2-7 in place, one
// launch after the tick loop writes the LayerNorm planes 0-1 from the port grids), which the
// backward reads in place of recomputing its ticks' forward stages; the backward's kernels and
// GEMMs write planes 8-13, the gradients that meet the weights [d_o | d_q|k|v | d_z_x | d_z_l |
// d_lat_prior | d_fdbk_prior], directly. Nothing is copied between planes and tick buffers. A tick's
// cells lie 2S - 1 cells apart in a plane (one stride per strided-batched GEMM), and a layer's
// cells are consecutive, so each weight gradient is one GEMM per layer over all of its cells at
// the end.
__host__ __device__ constexpr int plane_units(int p) {  // units of B x D per cell
  return (p == 3 || p == 7 || p == 8) ? 3 : (p == 6 || p == 9) ? 9 : 1;
}
constexpr int kSavedUnits = 36;  // sum of plane_units over the planes
enum { PL_LN_LEFT, PL_LN_DIAG, PL_LAT, PL_TOK, PL_ZL, PL_ZX, PL_QKV, PL_ATT, PL_DO, PL_DQKV, PL_DZX,
       PL_DZL, PL_DLP, PL_DFP };

__host__ __device__ inline int64_t plane_offset(int p, int64_t cells, int64_t BD) {
  int64_t u = 0;
  for (int q = 0; q < p; ++q) u += plane_units(q);
  return u * cells * BD;
}

constexpr size_t kBlkBlasWs = 32u << 20;

struct BlockWs {
  unsigned* sync;  // persistent forward: [0] barrier counter, [1] error word, [2] abort flag
  bf16* lnr;       // LayerNorm ring of the tick path: [3][left | diag][L][B][D]
  bf16 *ln, *lat, *tok, *z, *zx, *qkv, *att, *o;
  bf16* glpf;  // [L, D, D] folded lateral-gate weights G_L P_fb
  void* blas;
  void* blas_side;
};

size_t block_ws_layout(int64_t nmax, int64_t L, int64_t B, int64_t D, BlockWs* w, void* base) {
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t rowb = (size_t)nmax * B * D * sizeof(bf16);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += al(bytes);
    return o;
  };
  const size_t o_sync = take(256);  // first: flb_block_grid_status reads it at offset 0
  const size_t o_lnr = take((size_t)3 * 2 * L * B * D * sizeof(bf16));
  const size_t o_ln = take(2 * rowb), o_lat = take(rowb), o_tok = take(3 * rowb), o_z = take(rowb), o_zx = take(rowb),
               o_qkv = take(9 * rowb), o_att = take(3 * rowb), o_o = take(3 * rowb),
               o_blas = take(kBlkBlasWs), o_blas_side = take(kBlkBlasWs),
               o_glpf = take((size_t)L * D * D * sizeof(bf16));
  if (w && base) {
    uint8_t* p = reinterpret_cast<uint8_t*>(base);
    w->sync = (unsigned*)(p + o_sync);
    w->lnr = (bf16*)(p + o_lnr);
    w->ln = (bf16*)(p + o_ln);
    w->lat = (bf16*)(p + o_lat);
    w->tok = (bf16*)(p + o_tok);
    w->z = (bf16*)(p + o_z);
    w->zx = (bf16*)(p + o_zx);
    w->qkv = (bf16*)(p + o_qkv);
    w->att = (bf16*)(p + o_att);
    w->o = (bf16*)(p + o_o);
    w->blas = p + o_blas;
    w->blas_side = p + o_blas_side;
    w->glpf = (bf16*)(p + o_glpf);
  }
  return off;
}

int64_t max_cells_per_tick(int64_t L, int64_t S) {
  const int64_t a = (L + 1) / 2;
  return a < S ? a : S;
}

#include "flb_persist.cuh"

// Shapes the persistent forward takes: batch 16, D a multiple of 128 up to 1024 (128-feature
// tiles, K in 64-element atoms), the activation tile (48 rows x D bf16) plus a ring of at least
// two weight atoms within the shared-memory budget.
bool persist_fits(int64_t L, int64_t S, int64_t B, int64_t D, int64_t H) {
  (void)L;
  (void)S;
  return B == kPsB && D % 128 == 0 && D >= 128 && D <= 1024 && D % H == 0 && D / H <= 128;
}

// 2-D map over rows x K (bf16, K contiguous), boxes of box_rows rows x 64 K, 128-byte swizzle.
int make_rows_map(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int box_rows) {
  const uint64_t dims[2] = {(uint64_t)K, (uint64_t)rows};
  const uint64_t strides[1] = {(uint64_t)K * 2};
  const uint32_t box[2] = {64, (uint32_t)box_rows};
  return make_tmap(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_persist(const flb_block_weights* W, const bf16* glpf, const bf16* xb, bf16* g,
                   int64_t port_stride, const BlockWs& w, int L, int S, int D, int H, float eps,
                   cudaStream_t s, int drop_cta, int drop_bar, uint32_t spin_limit) {
  PsMaps maps;
  const void* bases[6] = {W->w_prior_lat, W->w_prior_fdbk, glpf, W->w_gate_x, W->w_qkv, W->w_o};
  for (int i = 0; i < 6; ++i) {
    const int64_t rows = (int64_t)(i == PS_QKV ? 3 : 1) * L * D;
    int st = make_rows_map(&maps.m[i], bases[i], rows, D, 128);
    if (st != FLB_OK) return st;
  }
  // activation buffers read by TMA: x', lat', fdbk_prior [nmax * 16, D]; attention [nmax * 48, D]
  const int64_t nmax = max_cells_per_tick(L, S);
  bf16* xr = w.o;
  bf16* latr = w.o + nmax * kPsB * D;
  const void* abases[4] = {xr, latr, w.tok, w.att};
  for (int i = 0; i < 4; ++i) {
    const int box = i == 3 ? 3 * kPsB : kPsB;
    int st = make_rows_map(&maps.m[PS_A_XR + i], abases[i], nmax * box, D, box);
    if (st != FLB_OK) return st;
  }
  const int act_bytes = 3 * kPsB * D * 2;
  int stages = (kPsSmemCap - 2048 - act_bytes) / kPsAtom;
  if (stages > kPsMaxStages) stages = kPsMaxStages;
  if (stages < 2) return fail(FLB_ERR_UNSUPPORTED, "block_grid persistent: shared memory too small");
  const int smem = 1024 + stages * kPsAtom + act_bytes;
  PsArgs a{};
  a.ln_lat_w = W->ln_lat_w;
  a.ln_lat_b = W->ln_lat_b;
  a.ln_fdbk_w = W->ln_fdbk_w;
  a.ln_fdbk_b = W->ln_fdbk_b;
  a.b_gate_l = W->b_gate_l;
  a.b_gate_x = W->b_gate_x;
  a.v_a = W->v_a;
  a.x = xb;
  a.g = g;
  a.port_stride = port_stride;
  a.lat = w.lat;
  a.zl = w.z;
  a.fdbk = w.tok;
  a.xr = xr;
  a.latr = latr;
  a.qkv = w.qkv;
  a.att = w.att;
  a.ctr = w.sync;
  a.err = reinterpret_cast<int*>(w.sync + 1);
  a.abort_flag = reinterpret_cast<int*>(w.sync + 2);
  a.L = L;
  a.S = S;
  a.D = D;
  a.H = H;
  a.F = D / 128;
  a.KA = D / 64;
  a.stages = stages;
  a.ticks = L + 2 * S - 2;
  a.act_off = (uint32_t)(stages * kPsAtom);
  a.eps = eps;
  a.spin_limit = spin_limit;
  a.drop_cta = drop_cta;
  a.drop_bar = drop_bar;
  int st = ensure_dyn_smem((const void*)flb_persist_fwd_kernel, smem, "block_grid persistent smem attribute");
  if (st != FLB_OK) return st;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, flb_persist_fwd_kernel,
                                                                kPsThreads, smem);
  if (e != cudaSuccess) return check_cuda(e, "block_grid persistent occupancy");
  if (per_sm < 1) return fail(FLB_ERR_LAUNCH, "block_grid persistent: kernel does not fit on an SM");
  e = cudaMemsetAsync(w.sync, 0, 256, s);
  if (e != cudaSuccess) return check_cuda(e, "block_grid persistent memset");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_sms());
  cfg.blockDim = dim3(kPsThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: they wait on each other
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, flb_persist_fwd_kernel, maps, a);
  count_launches(1);
  return check_cuda(e, "block_grid persistent launch");
}

}  // namespace

size_t block_grid_workspace_bytes(int64_t L, int64_t S, int64_t B, int64_t D) {
  return block_ws_layout(max_cells_per_tick(L, S), L, B, D, nullptr, nullptr);
}

namespace {

// A per-device side stream and fork/join events: GEMMs that are off a tick's critical chain
// (the lateral prior of the forward, the weight-gradient GEMMs of the backward) run on it while
// the chain continues on the caller's stream. Created on the first call on a device and kept
// until exit.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork[5] = {}, join = nullptr, fwd_fork = nullptr, fwd_join = nullptr,
              fwd_join2 = nullptr;
};

int side_stream(SideStream** out) {
  static std::mutex mu;
  static SideStream per_dev[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(FLB_ERR_UNSUPPORTED, "block_grid: device index >= 64");
  std::lock_guard<std::mutex> lock(mu);
  SideStream& ss = per_dev[dev];
  if (ss.s == nullptr) {
    cudaError_t e = cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking);
    for (int i = 0; e == cudaSuccess && i < 5; ++i)
      e = cudaEventCreateWithFlags(&ss.fork[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ss.fwd_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ss.fwd_join, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ss.fwd_join2, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      ss.s = nullptr;
      return check_cuda(e, "block_grid side stream");
    }
  }
  *out = &ss;
  return FLB_OK;
}

// Forward buffers of one tick (bf16): LayerNorm outputs [2][n][B][D], lat_prior [n][B][D],
// tokens [n][B][3][D] (x', lat', fdbk_prior), gate pre-activations [n][B][D] (the forward reuses
// one buffer for both), q|k|v [n][3B][3D], attention output [n][3B][D].
// Cell i of the tick at base + i * units * cs: cs = B x D in the work buffers, or (2S - 1) x B x D
// when the pointers are the tick's first cell in the kept planes (the training forward writes
// its intermediates there in place). ln is always a work buffer.
struct TickBufs {
  bf16 *ln, *lat, *tok, *zl, *zx, *qkv, *att;
  int64_t cs;
};

// stages 1-6 of a tick (everything up to the attention output)
// the side stream and its cuBLAS handle for GEMMs off the critical chain of a tick
struct Side {
  SideStream* ss;
  cublasHandle_t h;
};

// w_glpf: the per-layer products G_L P_fb [L, D, D] (inference), or null. With them the lateral
// gate's pre-activation comes straight from the LayerNorm output, z_l = LN(diag) (G_L P_fb)^T,
// and both priors run on the side stream next to it.
int tick_forward(cublasHandle_t hb, const Side& side, const flb_block_weights* W, const bf16* xb,
                 const bf16* g, int64_t port_stride, const TickBufs& b, int T, int l0, int n,
                 int L, int S, int B, int D, int H, float eps, cudaStream_t s,
                 const bf16* w_glpf = nullptr, const bf16* lnr = nullptr) {
  const long long DD = (long long)D * D, BD = (long long)B * D;
  int st;
  cudaError_t e = cudaSuccess;
  // LayerNorm outputs of the tick's cells: from the ring the previous ticks' output kernels
  // filled (lnr: [T % 3][left | diag][layer][B][D], cells two layers apart), or computed here
  const bf16 *ln_left = b.ln, *ln_diag = b.ln + n * BD;
  long long ln_stride = BD;
  if (lnr) {
    const long long LBD = (long long)L * BD;
    ln_left = lnr + (long long)(T % 3) * 2 * LBD + (long long)l0 * BD;
    ln_diag = ln_left + LBD;
    ln_stride = 2 * BD;
  } else {
    e = launch_pdl(blk_ln_kernel, dim3((2 * n * B + 7) / 8), dim3(256), 0, s, g + port_stride,
                   g + 2 * port_stride, W->ln_lat_w, W->ln_lat_b, W->ln_fdbk_w, W->ln_fdbk_b, b.ln,
                   T, l0, n, L, S, B, D, eps);
    if (e != cudaSuccess) return check_cuda(e, "block_grid LayerNorm launch");
  }
  e = cudaEventRecord(side.ss->fwd_fork, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(side.ss->s, side.ss->fwd_fork, 0);
  if (e != cudaSuccess) return check_cuda(e, "block_grid tick fork");
  const bf16* Wpl = reinterpret_cast<const bf16*>(W->w_prior_lat) + (int64_t)l0 * DD;
  const bf16* Wpf = reinterpret_cast<const bf16*>(W->w_prior_fdbk) + (int64_t)l0 * DD;
  const bf16* Wgl = reinterpret_cast<const bf16*>(W->w_gate_l) + (int64_t)l0 * DD;
  const bf16* Wgx = reinterpret_cast<const bf16*>(W->w_gate_x) + (int64_t)l0 * DD;
  const bf16* Wqkv = reinterpret_cast<const bf16*>(W->w_qkv) + (int64_t)l0 * 3 * DD;
  // priors: lat_prior -> b.lat (side stream: first needed by the lateral gate kernel);
  // fdbk_prior -> token slot 2 (row pitch 3D)
  const int64_t cs = b.cs;
  if ((st = gemm_rm(side.h, false, true, B, D, D, ln_left, D, ln_stride, Wpl, D, 2 * DD, b.lat, D,
                    cs, n, 0.f, CUDA_R_16BF)) != FLB_OK)
    return st;
  e = cudaEventRecord(side.ss->fwd_join, side.ss->s);
  if (e != cudaSuccess) return check_cuda(e, "block_grid tick join");
  if (w_glpf) {
    // fdbk_prior on the side stream (first needed by the q|k|v GEMM); z_l from the folded weights
    if ((st = gemm_rm(side.h, false, true, B, D, D, ln_diag, D, ln_stride, Wpf, D, 2 * DD,
                      b.tok + 2 * D, 3 * D, 3 * cs, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    e = cudaEventRecord(side.ss->fwd_join2, side.ss->s);
    if (e != cudaSuccess) return check_cuda(e, "block_grid tick join");
    if ((st = gemm_rm(hb, false, true, B, D, D, ln_diag, D, ln_stride, w_glpf + (int64_t)l0 * DD, D,
                      2 * DD, b.zl, D, cs, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
  } else {
    if ((st = gemm_rm(hb, false, true, B, D, D, ln_diag, D, ln_stride, Wpf, D, 2 * DD, b.tok + 2 * D,
                      3 * D, 3 * cs, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    // lateral gate
    if ((st = gemm_rm(hb, false, true, B, D, D, b.tok + 2 * D, 3 * D, 3 * cs, Wgl, D, 2 * DD, b.zl,
                      D, cs, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
  }
  e = cudaStreamWaitEvent(s, side.ss->fwd_join, 0);
  if (e != cudaSuccess) return check_cuda(e, "block_grid tick join");
  const dim3 ew_grid((unsigned)((D / 2 + 127) / 128), (unsigned)(n * B));
  e = launch_pdl(blk_gate_kernel, ew_grid, dim3(128), 0, s, b.zl, W->b_gate_l, b.lat, g, xb, 0,
                 b.tok + D, cs, T, l0, S, B, D);
  if (e != cudaSuccess) return check_cuda(e, "block_grid gate launch");
  // sensory gate
  if ((st = gemm_rm(hb, false, true, B, D, D, b.tok + D, 3 * D, 3 * cs, Wgx, D, 2 * DD, b.zx, D, cs,
                    n, 0.f, CUDA_R_16BF)) != FLB_OK)
    return st;
  e = launch_pdl(blk_gate_kernel, ew_grid, dim3(128), 0, s, b.zx, W->b_gate_x,
                 static_cast<const bf16*>(nullptr), g, xb, 1, b.tok, cs, T, l0, S, B, D);
  if (e != cudaSuccess) return check_cuda(e, "block_grid gate launch");
  if (w_glpf) {
    e = cudaStreamWaitEvent(s, side.ss->fwd_join2, 0);
    if (e != cudaSuccess) return check_cuda(e, "block_grid tick join");
  }
  // q | k | v of the 3 tokens: [n, 3B, D] x [3D, D]^T
  if ((st = gemm_rm(hb, false, true, 3 * B, 3 * D, D, b.tok, D, 3 * cs, Wqkv, D, 6 * DD, b.qkv,
                    3 * D, 9 * cs, n, 0.f, CUDA_R_16BF)) != FLB_OK)
    return st;
  e = launch_pdl(blk_attn3_kernel, dim3((n * B * H + 7) / 8), dim3(256), 0, s, b.qkv, W->v_a,
                 b.att, cs, l0, n, B, D, H);
  return check_cuda(e, "block_grid attention launch");
}

}  // namespace

int block_grid_fwd_ex(const flb_block_weights* W, const void* x, void* grids, int64_t L,
                      int64_t S, int64_t B, int64_t D, int64_t H, float eps, void* ws,
                      size_t ws_bytes, cudaStream_t s, int path, int drop_cta, int drop_bar,
                      uint32_t spin_limit, void* saved) {
  // the persistent forward only on request: at the end-to-end shape (12 layers x 1024
  // positions, d_model 768, batch 16) it measured 111 ms per forward against 80 ms tick by tick
  const bool persist = persist_fits(L, S, B, D, H) && path == FLB_BLOCK_PATH_PERSISTENT;
  if (path == FLB_BLOCK_PATH_PERSISTENT && !persist)
    return fail(FLB_ERR_UNSUPPORTED, "block_grid persistent forward: needs batch 16 and D a multiple of 128 up to 1024");
  if (persist && saved)
    return fail(FLB_ERR_UNSUPPORTED, "block_grid: the persistent forward keeps no intermediates");
  BlockWs w;
  block_ws_layout(max_cells_per_tick(L, S), L, B, D, &w, ws);
  cublasHandle_t hb;
  int st = blas(s, w.blas, kBlkBlasWs, &hb);
  if (st != FLB_OK) return st;
  Side side{};
  if ((st = side_stream(&side.ss)) != FLB_OK) return st;
  if ((st = blas(side.ss->s, w.blas_side, kBlkBlasWs, &side.h, 1)) != FLB_OK) return st;
  const bf16* xb = reinterpret_cast<const bf16*>(x);
  bf16* g = reinterpret_cast<bf16*>(grids);
  const int64_t port_stride = (L * S + L) * B * D;  // the engine's grids keep L dock rows
  const long long DD = D * D, BD = B * D;
  const int Li = (int)L, Si = (int)S, Bi = (int)B, Di = (int)D, Hi = (int)H;
  const int ticks = (int)(L + 2 * S - 2);
  const TickBufs work{w.ln, w.lat, w.tok, w.z, w.zx, w.qkv, w.att, BD};
  bf16* planes = reinterpret_cast<bf16*>(saved);
  // inference: fold the lateral gate onto the feedback prior once per call, G_L P_fb per layer
  if ((st = gemm_rm(hb, false, false, Di, Di, Di, W->w_gate_l, Di, DD, W->w_prior_fdbk, Di, DD,
                    w.glpf, Di, DD, Li, 0.f, CUDA_R_16BF)) != FLB_OK)
    return st;
  if (persist)
    return launch_persist(W, w.glpf, xb, g, port_stride, w, Li, Si, Di, Hi, eps, s, drop_cta,
                          drop_bar, spin_limit ? spin_limit : kPsSpinLimit);
  // the LayerNorm ring starts as the normalised zero rows (the LayerNorm biases)
  cudaError_t ie = launch_pdl(blk_ln_init_kernel, dim3((unsigned)((D / 2 + 127) / 128), (unsigned)(6 * L * B)),
                              dim3(128), 0, s, w.lnr, W->ln_lat_b, W->ln_fdbk_b, Li, Bi, Di);
  if (ie != cudaSuccess) return check_cuda(ie, "block_grid LayerNorm init launch");
  int launches = 1;
  for (int T = 0; T < ticks; ++T) {
    const Tick tk = tick_of(T, Li, Si);
    const int n = tk.n, l0 = tk.l0;
    if (n == 0) continue;
    // training: the tick's intermediates go straight to their planes (cell i of the tick
    // 2S - 1 cells after cell i - 1), where the backward reads them
    TickBufs tb = work;
    if (planes) {
      const int64_t c0 = (int64_t)l0 * S + (T - l0) / 2;  // flat index of the tick's first cell
      auto at = [&](int p) { return planes + plane_offset(p, L * S, BD) + c0 * plane_units(p) * BD; };
      tb = TickBufs{w.ln, at(PL_LAT), at(PL_TOK), at(PL_ZL), at(PL_ZX), at(PL_QKV), at(PL_ATT),
                    (2 * S - 1) * BD};
    }
    if ((st = tick_forward(hb, side, W, xb, g, port_stride, tb, T, l0, n, Li, Si, Bi, Di, Hi, eps,
                           s, w.glpf, w.lnr)) != FLB_OK)
      return st;
    const bf16* Wo = reinterpret_cast<const bf16*>(W->w_o) + (int64_t)l0 * DD;
    if ((st = gemm_rm(hb, false, true, 3 * Bi, Di, Di, tb.att, Di, 3 * tb.cs, Wo, Di, 2 * DD, w.o,
                      Di, 3 * BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    // residuals, aux and the next ticks' LayerNorms: a warp per (cell, batch row)
    const int out_threads = std::max(32, (Di / 8 + 31) / 32 * 32);
    cudaError_t e = launch_pdl(blk_out_ln_kernel, dim3((unsigned)(n * Bi)), dim3(out_threads), 0,
                               s, w.o, tb.lat, tb.tok, tb.cs, xb, g, port_stride, w.lnr, W->ln_lat_w,
                               W->ln_lat_b, W->ln_fdbk_w, W->ln_fdbk_b, eps, T, l0, n, Li, Si, Bi, Di);
    if (e != cudaSuccess) return check_cuda(e, "block_grid output launch");
    launches += 4;  // own kernels: two gates, attention, output (the GEMMs are cuBLAS's)
  }
  if (planes) {
    // the LayerNorm planes of every cell, from the port grids the ticks wrote
    const int64_t rows = 2 * L * S * B;
    cudaError_t e = launch_pdl(blk_ln_planes_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0,
                               s, g + port_stride, g + 2 * port_stride, W->ln_lat_w, W->ln_lat_b,
                               W->ln_fdbk_w, W->ln_fdbk_b, planes + plane_offset(PL_LN_LEFT, L * S, BD),
                               Li, Si, Bi, Di, eps);
    if (e != cudaSuccess) return check_cuda(e, "block_grid LayerNorm planes launch");
    ++launches;
  }
  count_launches(launches);
  return check_cuda(cudaGetLastError(), "flb block grid launch");
}

int block_grid_fwd(const flb_block_weights* W, const void* x, void* grids, int64_t L, int64_t S,
                   int64_t B, int64_t D, int64_t H, float eps, void* ws, size_t ws_bytes,
                   cudaStream_t s) {
  return block_grid_fwd_ex(W, x, grids, L, S, B, D, H, eps, ws, ws_bytes, s, FLB_BLOCK_PATH_AUTO,
                           -1, -1, 0, nullptr);
}

int block_grid_status(const void* ws, cudaStream_t s) {
  int h[3] = {0, 0, 0};
  cudaError_t e = cudaMemcpyAsync(h, ws, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return check_cuda(e, "block_grid status");
  if (h[1] != 0)
    return fail(FLB_ERR_TIMEOUT, "block_grid persistent forward: a bounded device wait gave up (code " +
                                     std::to_string(h[1]) + ")");
  return FLB_OK;
}

// =============================================================================================
// Backward of the FLB block grid (training). Ticks in reverse; per tick the forward stages are
// recomputed from the saved port grids, then (for all of the tick's cells at once):
//   residual/aux -> d_o, d_top, d_lat_prior, d_fdbk_prior          [own kernel]
//   d_att = d_o W_o, dW_o += d_o^T att                              [GEMMs]
//   3-token attention backward -> d_q | d_k | d_v, dv_a             [own kernel]
//   dT = d_qkv W_qkv, dW_qkv += d_qkv^T T                           [GEMMs]
//   sensory gate backward (routes d_top), lateral gate backward      [own kernels + GEMMs]
//   prior GEMMs, then the LayerNorm backward (routes d_left, d_diag) [GEMMs + own kernel]
// Each port output has exactly one consumer (top -> the cell above, left -> the next column,
// bottom-left -> the cell below in the next column) and consumers run at later ticks, so the
// routed gradients are plain additions into fp32 gradient grids, complete when the producing
// cell's tick comes. Weight gradients accumulate into per-layer fp32 stacks (the cells of a
// tick are distinct layers). Math: the chain rule of models/FLB_Model.py:32-96 and of the
// attention (kernels/additive_attention.py:91-130) on 3 tokens.
// =============================================================================================

namespace {

__device__ __forceinline__ float sigm(float z) { return 1.f / (1.f + __expf(-z)); }

// external bf16 port grads (or zero) -> fp32 gradient grids of ports 0-2, [L*S][B][D] each
__global__ void blk_dg_init_kernel(const bf16* __restrict__ g0, const bf16* __restrict__ g1,
                                   const bf16* __restrict__ g2, float* __restrict__ dG,
                                   int64_t per_port) {
  pdl_wait();
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < 3 * per_port;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int p = (int)(e / per_port);
    const int64_t r = e - p * per_port;
    const bf16* src = p == 0 ? g0 : (p == 1 ? g1 : g2);
    dG[e] = src ? __bfloat162float(src[r]) : 0.f;
  }
}

// residuals and aux: grid (pairs, n*B rows)
__global__ void blk_bwd_out_kernel(const float* __restrict__ dG, int64_t per_port,
                                   const bf16* __restrict__ ext3, const bf16* __restrict__ grids,
                                   int64_t port_stride, const bf16* __restrict__ lat,
                                   const bf16* __restrict__ tok, bf16* __restrict__ d_o, int64_t cs,
                                   float* __restrict__ d_top, float* __restrict__ d_lp,
                                   float* __restrict__ d_fp, int T, int l0, int S, int B, int D) {
  pdl_wait();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= D / 2) return;
  const int rb = blockIdx.y;
  const int i = rb / B, b = rb - i * B;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const int64_t off = (cell_row(l, t, S) * B + b) * D;
  const float2 dhx = reinterpret_cast<const float2*>(dG + off)[j];
  const float2 dhl = reinterpret_cast<const float2*>(dG + per_port + off)[j];
  const float2 dhf = reinterpret_cast<const float2*>(dG + 2 * per_port + off)[j];
  float2 da = make_float2(0.f, 0.f);
  if (ext3) da = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(ext3 + off)[j]);
  auto ld2 = [&](const bf16* p) {
    return __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(p)[j]);
  };
  const float2 hl = ld2(grids + port_stride + off), hf = ld2(grids + 2 * port_stride + off);
  const int64_t cr = (int64_t)i * cs + (int64_t)b * D;  // row of a one-unit cell array
  const float2 lp = ld2(lat + cr), fp = ld2(tok + 3 * cr + 2 * D);
  reinterpret_cast<__nv_bfloat162*>(d_o + 3 * cr)[j] = __floats2bfloat162_rn(dhx.x, dhx.y);
  reinterpret_cast<__nv_bfloat162*>(d_o + 3 * cr + D)[j] = __floats2bfloat162_rn(dhl.x, dhl.y);
  reinterpret_cast<__nv_bfloat162*>(d_o + 3 * cr + 2 * D)[j] = __floats2bfloat162_rn(dhf.x, dhf.y);
  reinterpret_cast<float2*>(d_top + (int64_t)rb * D)[j] = dhx;
  reinterpret_cast<float2*>(d_lp + (int64_t)rb * D)[j] =
      make_float2(dhl.x + 2.f * (lp.x - hl.x) * da.x, dhl.y + 2.f * (lp.y - hl.y) * da.y);
  reinterpret_cast<float2*>(d_fp + (int64_t)rb * D)[j] =
      make_float2(dhf.x + 2.f * (fp.x - hf.x) * da.x, dhf.y + 2.f * (fp.y - hf.y) * da.y);
}

// 3-token attention backward, one warp per (cell, batch row, head)
__global__ void blk_attn3_bwd_kernel(const bf16* __restrict__ qkv, const float* __restrict__ v_a,
                                     const bf16* __restrict__ d_att, bf16* __restrict__ d_qkv,
                                     int64_t cs, float* __restrict__ d_va, int l0, int n, int B,
                                     int D, int H) {
  pdl_wait();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.x * warps + (threadIdx.x >> 5);
  if (task >= n * B * H) return;
  const int h = task % H;
  const int64_t rb = task / H;
  const int i = (int)(rb / B);
  const int dh = D / H;
  const int64_t wrow = ((int64_t)(l0 + 2 * i) * H + h) * dh;
  const float* w = v_a + wrow;
  const int64_t cr = (int64_t)i * cs + (rb - (int64_t)i * B) * D;  // one-unit row of (cell, b)
  const bf16* base = qkv + 9 * cr + h * dh;
  const bf16* dob = d_att + rb * 3 * D + h * dh;
  float q[4][3], k[4][3], v[4][3], dout[4][3], wd[4];
  float s[3][3], dp[3][3];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int c = 0; c < 3; ++c) s[a][c] = dp[a][c] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int d = lane + 32 * kk;
    const bool ok = d < dh;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      q[kk][r] = ok ? __bfloat162float(base[r * 3 * D + d]) : 0.f;
      k[kk][r] = ok ? __bfloat162float(base[r * 3 * D + D + d]) : 0.f;
      v[kk][r] = ok ? __bfloat162float(base[r * 3 * D + 2 * D + d]) : 0.f;
      dout[kk][r] = ok ? __bfloat162float(dob[r * D + d]) : 0.f;
    }
    wd[kk] = ok ? w[d] : 0.f;
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        s[a][c] = fmaf(wd[kk], ok ? tanh_approx(q[kk][a] + k[kk][c]) : 0.f, s[a][c]);
        dp[a][c] = fmaf(dout[kk][a], v[kk][c], dp[a][c]);
      }
  }
  const float scale = rsqrtf((float)dh);
  float p[3][3], ds[3][3];
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      s[a][c] = warp_sum(s[a][c]) * scale;
      dp[a][c] = warp_sum(dp[a][c]);
      m = fmaxf(m, s[a][c]);
    }
    float l = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      p[a][c] = __expf(s[a][c] - m);
      l += p[a][c];
    }
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      p[a][c] /= l;
      dot += p[a][c] * dp[a][c];
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) ds[a][c] = p[a][c] * (dp[a][c] - dot) * scale;
  }
  bf16* dbase = d_qkv + 9 * cr + h * dh;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const int d = lane + 32 * kk;
    if (d >= dh) break;
    float dq[3] = {0.f, 0.f, 0.f}, dk[3] = {0.f, 0.f, 0.f}, dw = 0.f;
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const float tt = tanh_approx(q[kk][a] + k[kk][c]);
        const float g = ds[a][c] * wd[kk] * (1.f - tt * tt);
        dq[a] += g;
        dk[c] += g;
        dw = fmaf(ds[a][c], tt, dw);
      }
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const float dv = p[0][r] * dout[kk][0] + p[1][r] * dout[kk][1] + p[2][r] * dout[kk][2];
      dbase[r * 3 * D + d] = __float2bfloat16_rn(dq[r]);
      dbase[r * 3 * D + D + d] = __float2bfloat16_rn(dk[r]);
      dbase[r * 3 * D + 2 * D + d] = __float2bfloat16_rn(dv);
    }
    atomicAdd(d_va + wrow + d, dw);
  }
}

// sensory gate backward: grid (pairs, cells), loop over the batch rows. Finishes d_top and routes
// it (to the port-0 gradient of the cell above, or to dx for layer 0).
__global__ void blk_gx_bwd_kernel(const float* __restrict__ dT, const bf16* __restrict__ zx,
                                  const float* __restrict__ b_gx, const bf16* __restrict__ grids,
                                  const bf16* __restrict__ x, const float* __restrict__ d_top,
                                  float* __restrict__ dG0, float* __restrict__ dx,
                                  bf16* __restrict__ d_zx, float* __restrict__ d_lr,
                                  const float* __restrict__ d_fp, bf16* __restrict__ d_fp_h,
                                  int64_t cs, bf16* __restrict__ dcat, float* __restrict__ db_gx,
                                  int T, int l0, int S, int B, int D) {
  pdl_wait();
  // block: 32 feature pairs (x) by up to 16 batch rows (y); the bias gradient is summed over
  // the rows in a fixed order (deterministic)
  __shared__ float2 part[16][32];
  const int j = blockIdx.x * 32 + threadIdx.x;
  const bool live = j < D / 2;
  const int i = blockIdx.y;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  float2 acc = make_float2(0.f, 0.f);
  if (live) {
    const float2 bias = reinterpret_cast<const float2*>(b_gx + (int64_t)l * D)[j];
    for (int b = threadIdx.y; b < B; b += blockDim.y) {
      const int64_t rb = (int64_t)i * B + b;
      const int64_t cr = (int64_t)i * cs + (int64_t)b * D;
      const float2 dxr = reinterpret_cast<const float2*>(dT + (rb * 3) * D)[j];
      const float2 z = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(zx + cr)[j]);
      const float2 top = __bfloat1622float2(
          reinterpret_cast<const __nv_bfloat162*>(top_row(grids, x, l, t, b, S, B, D))[j]);
      const float s0 = sigm(z.x + bias.x), s1 = sigm(z.y + bias.y);
      const float2 dt0 = reinterpret_cast<const float2*>(d_top + rb * D)[j];
      const float2 dtop = make_float2(dt0.x + dxr.x * s0, dt0.y + dxr.y * s1);
      if (l > 0) {
        float2* dst = reinterpret_cast<float2*>(dG0 + (cell_row(l - 1, t, S) * B + b) * D) + j;
        const float2 o = *dst;
        *dst = make_float2(o.x + dtop.x, o.y + dtop.y);
      } else {
        reinterpret_cast<float2*>(dx + ((int64_t)b * S + t) * D)[j] = dtop;
      }
      const float dz0 = dxr.x * top.x * s0 * (1.f - s0), dz1 = dxr.y * top.y * s1 * (1.f - s1);
      reinterpret_cast<__nv_bfloat162*>(d_zx + cr)[j] = __floats2bfloat162_rn(dz0, dz1);
      acc.x += dz0;
      acc.y += dz1;
      reinterpret_cast<float2*>(d_lr + rb * D)[j] =
          reinterpret_cast<const float2*>(dT + (rb * 3 + 1) * D)[j];
      // d_fdbk_prior so far (residual + aux, then the q|k|v token's share), in bf16: the
      // operand of the G_L GEMM that adds d_zL G_L in place (no separate cast); with dcat also
      // the first half of the feedback LayerNorm's input-gradient operand
      const float2 dtf = reinterpret_cast<const float2*>(dT + (rb * 3 + 2) * D)[j];
      const float2 o = reinterpret_cast<const float2*>(d_fp + rb * D)[j];
      const __nv_bfloat162 fp2 = __floats2bfloat162_rn(o.x + dtf.x, o.y + dtf.y);
      reinterpret_cast<__nv_bfloat162*>(d_fp_h + cr)[j] = fp2;
      if (dcat) reinterpret_cast<__nv_bfloat162*>(dcat + rb * 2 * D)[j] = fp2;
    }
  }
  part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (live && threadIdx.y == 0) {
    float2 sum = part[0][threadIdx.x];
    for (int y = 1; y < (int)blockDim.y; ++y) {
      sum.x += part[y][threadIdx.x].x;
      sum.y += part[y][threadIdx.x].y;
    }
    float2* db = reinterpret_cast<float2*>(db_gx + (int64_t)l * D) + j;
    const float2 o = *db;
    *db = make_float2(o.x + sum.x, o.y + sum.y);
  }
}

// lateral gate backward: grid (pairs, cells), loop over the batch rows; finishes d_lat_prior
__global__ void blk_gl_bwd_kernel(const float* __restrict__ d_lr, const bf16* __restrict__ zl,
                                  const float* __restrict__ b_gl, const bf16* __restrict__ lat,
                                  float* __restrict__ d_lp, bf16* __restrict__ d_lp_h,
                                  bf16* __restrict__ d_zl, int64_t cs, bf16* __restrict__ dcat,
                                  float* __restrict__ db_gl, int l0, int B, int D) {
  pdl_wait();
  __shared__ float2 part[16][32];  // as blk_gx_bwd_kernel: 32 pairs by up to 16 rows
  const int j = blockIdx.x * 32 + threadIdx.x;
  const bool live = j < D / 2;
  const int i = blockIdx.y;
  const int l = l0 + 2 * i;
  float2 acc = make_float2(0.f, 0.f);
  if (live) {
    const float2 bias = reinterpret_cast<const float2*>(b_gl + (int64_t)l * D)[j];
    for (int b = threadIdx.y; b < B; b += blockDim.y) {
      const int64_t rb = (int64_t)i * B + b;
      const int64_t cr = (int64_t)i * cs + (int64_t)b * D;
      const float2 dl = reinterpret_cast<const float2*>(d_lr + rb * D)[j];
      const float2 z = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(zl + cr)[j]);
      const float2 lp = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(lat + cr)[j]);
      const float s0 = sigm(z.x + bias.x), s1 = sigm(z.y + bias.y);
      const float2 o = reinterpret_cast<const float2*>(d_lp + rb * D)[j];
      const float2 dlp = make_float2(o.x + dl.x * s0, o.y + dl.y * s1);
      reinterpret_cast<__nv_bfloat162*>(d_lp_h + cr)[j] = __floats2bfloat162_rn(dlp.x, dlp.y);
      const float dz0 = dl.x * lp.x * s0 * (1.f - s0), dz1 = dl.y * lp.y * s1 * (1.f - s1);
      const __nv_bfloat162 dz2 = __floats2bfloat162_rn(dz0, dz1);
      reinterpret_cast<__nv_bfloat162*>(d_zl + cr)[j] = dz2;
      if (dcat) reinterpret_cast<__nv_bfloat162*>(dcat + rb * 2 * D + D)[j] = dz2;
      acc.x += dz0;
      acc.y += dz1;
    }
  }
  part[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (live && threadIdx.y == 0) {
    float2 sum = part[0][threadIdx.x];
    for (int y = 1; y < (int)blockDim.y; ++y) {
      sum.x += part[y][threadIdx.x].x;
      sum.y += part[y][threadIdx.x].y;
    }
    float2* db = reinterpret_cast<float2*>(db_gl + (int64_t)l * D) + j;
    const float2 o = *db;
    *db = make_float2(o.x + sum.x, o.y + sum.y);
  }
}

// LayerNorm backward: block per (32 feature pairs, which, cell), threads (pair, batch row).
// Phase 1, a warp per batch row over the whole row: the row's mean, 1/std and the two
// reductions of the input gradient (c1 = mean of g*gamma, c2 = mean of g*gamma*xhat); every
// block of a cell recomputes them for its rows (~77 KB of L2 reads at d_model 768, batch 16),
// which spreads the kernel over (D/64) x 2 x cells blocks instead of one per cell. Phase 2, a
// thread per (feature pair, row), coalesced, no atomics: the input gradient routed to the
// producer's port gradient (left -> port 1 of (l, t-1), bottom-left -> port 2 of (l+1, t-1)),
// and dgamma / dbeta of the cell's layer summed over the rows in a fixed order.
__global__ void blk_ln_bwd_kernel(const bf16* __restrict__ grids, int64_t port_stride,
                                  const float* __restrict__ dA, const float* __restrict__ lw0,
                                  const float* __restrict__ lw1, float* __restrict__ dG,
                                  int64_t per_port, float* __restrict__ dw0,
                                  float* __restrict__ db0, float* __restrict__ dw1,
                                  float* __restrict__ db1, int T, int l0, int n, int L, int S,
                                  int B, int D, float eps) {
  pdl_wait();
  extern __shared__ float stat[];  // [B][4]: mean, rstd, c1, c2
  __shared__ float2 part_g[16][32], part_b[16][32];
  const int which = blockIdx.y / n, i = blockIdx.y % n;
  const int l = l0 + 2 * i, t = (T - l) / 2;
  const int warps = blockDim.y, warp = threadIdx.y, lane = threadIdx.x;
  const float* gamma = (which ? lw1 : lw0) + (int64_t)l * D;
  const bool has_src = t > 0 && (which == 0 || l + 1 < L);
  const int64_t src_cell = which == 0 ? cell_row(l, t - 1, S) : cell_row(l + 1, t - 1, S);
  const bf16* src = grids + (which ? 2 : 1) * port_stride + src_cell * B * D;
  float* dst = dG + (which ? 2 : 1) * per_port + src_cell * B * D;
  const float* da = dA + (int64_t)(which * n + i) * B * D;
  const int nch = D / 8;
  for (int b = warp; b < B; b += warps) {
    float xv[kMaxChunks][8];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = lane + 32 * k;
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (has_src && c < nch) raw = reinterpret_cast<const uint4*>(src + (int64_t)b * D)[c];
      const uint32_t* r = reinterpret_cast<const uint32_t*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[e]));
        xv[k][2 * e] = f.x;
        xv[k][2 * e + 1] = f.y;
        s += f.x + f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    }
    s = warp_sum(s);
    ss = warp_sum(ss);
    const float mean = s / D;
    const float rstd = rsqrtf(fmaxf(ss / D - mean * mean, 0.f) + eps);
    float c1 = 0.f, c2 = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = lane + 32 * k;
      if (c >= nch) break;
      const float4* g4 = reinterpret_cast<const float4*>(da + (int64_t)b * D + 8 * c);
      const float4* w4 = reinterpret_cast<const float4*>(gamma + 8 * c);
      const float4 ga = g4[0], gb = g4[1], wa = w4[0], wb = w4[1];
      const float g[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
      const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float dxh = g[e] * w[e];
        c1 += dxh;
        c2 += dxh * (xv[k][e] - mean) * rstd;
      }
    }
    c1 = warp_sum(c1) / D;
    c2 = warp_sum(c2) / D;
    if (lane == 0) {
      stat[4 * b] = mean;
      stat[4 * b + 1] = rstd;
      stat[4 * b + 2] = c1;
      stat[4 * b + 3] = c2;
    }
  }
  __syncthreads();
  float* dw = (which ? dw1 : dw0) + (int64_t)l * D;
  float* db = (which ? db1 : db0) + (int64_t)l * D;
  const int jp = blockIdx.x * 32 + lane;
  float2 dgam = make_float2(0.f, 0.f), dbet = make_float2(0.f, 0.f);
  if (jp < D / 2) {
    const float2 gm = reinterpret_cast<const float2*>(gamma)[jp];
    for (int b = warp; b < B; b += warps) {
      const float mean = stat[4 * b], rstd = stat[4 * b + 1], c1 = stat[4 * b + 2],
                  c2 = stat[4 * b + 3];
      const float2 xx = has_src ? __bfloat1622float2(
                                      reinterpret_cast<const __nv_bfloat162*>(src + (int64_t)b * D)[jp])
                                : make_float2(0.f, 0.f);
      const float2 g = reinterpret_cast<const float2*>(da + (int64_t)b * D)[jp];
      const float xh0 = (xx.x - mean) * rstd, xh1 = (xx.y - mean) * rstd;
      dgam.x += g.x * xh0;
      dgam.y += g.y * xh1;
      dbet.x += g.x;
      dbet.y += g.y;
      if (has_src) {
        float2* o = reinterpret_cast<float2*>(dst + (int64_t)b * D) + jp;
        const float2 v = *o;
        *o = make_float2(v.x + rstd * (g.x * gm.x - c1 - xh0 * c2),
                         v.y + rstd * (g.y * gm.y - c1 - xh1 * c2));
      }
    }
  }
  part_g[warp][lane] = dgam;
  part_b[warp][lane] = dbet;
  __syncthreads();
  if (jp < D / 2 && warp == 0) {
    for (int y = 1; y < warps; ++y) {
      dgam.x += part_g[y][lane].x;
      dgam.y += part_g[y][lane].y;
      dbet.x += part_b[y][lane].x;
      dbet.y += part_b[y][lane].y;
    }
    float2* pw = reinterpret_cast<float2*>(dw) + jp;
    float2* pb = reinterpret_cast<float2*>(db) + jp;
    const float2 ow = *pw, ob = *pb;
    *pw = make_float2(ow.x + dgam.x, ow.y + dgam.y);
    *pb = make_float2(ob.x + dbet.x, ob.y + dbet.y);
  }
}

struct BlockBwdWs {
  TickBufs f;
  bf16 *d_o, *d_att, *d_qkv, *d_zx, *d_zl, *d_lp_h, *d_fp_h;
  // with the intermediates kept: [d_fdbk_prior partial | d_z_l] rows of a tick (pitch 2D), and
  // per layer [P_fb ; G_L P_fb] ([2D, D]), the operands of the feedback LayerNorm's input gradient
  bf16 *dcat, *wcat;
  float *dT, *d_top, *d_lp, *d_fp, *d_lr, *dA, *dG, *dx;
  void* blas;
  void* blas_side;
};

size_t block_bwd_ws_layout(int64_t L, int64_t S, int64_t B, int64_t D, BlockBwdWs* w, void* base) {
  const int64_t nmax = max_cells_per_tick(L, S);
  auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
  const size_t rowh = (size_t)nmax * B * D * sizeof(bf16), rowf = (size_t)nmax * B * D * 4;
  size_t off = 0;
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  auto take = [&](size_t bytes) -> uint8_t* {
    uint8_t* r = p ? p + off : nullptr;
    off += al(bytes);
    return r;
  };
  BlockBwdWs t;
  t.f.ln = (bf16*)take(2 * rowh);
  t.f.lat = (bf16*)take(rowh);
  t.f.tok = (bf16*)take(3 * rowh);
  t.f.zl = (bf16*)take(rowh);
  t.f.zx = (bf16*)take(rowh);
  t.f.qkv = (bf16*)take(9 * rowh);
  t.f.att = (bf16*)take(3 * rowh);
  t.f.cs = B * D;
  t.d_o = (bf16*)take(3 * rowh);
  t.d_att = (bf16*)take(3 * rowh);
  t.d_qkv = (bf16*)take(9 * rowh);
  t.d_zx = (bf16*)take(rowh);
  t.d_zl = (bf16*)take(rowh);
  t.d_lp_h = (bf16*)take(rowh);
  t.d_fp_h = (bf16*)take(rowh);
  t.dcat = (bf16*)take(2 * rowh);
  t.wcat = (bf16*)take((size_t)L * 2 * D * D * sizeof(bf16));
  t.dT = (float*)take(3 * rowf);
  t.d_top = (float*)take(rowf);
  t.d_lp = (float*)take(rowf);
  t.d_fp = (float*)take(rowf);
  t.d_lr = (float*)take(rowf);
  t.dA = (float*)take(2 * rowf);
  t.dG = (float*)take((size_t)3 * L * S * B * D * 4);
  t.dx = nullptr;
  t.blas = take(kBlkBlasWs);
  t.blas_side = take(kBlkBlasWs);
  if (w) *w = t;
  return off;
}

}  // namespace

size_t block_grid_saved_bytes(int64_t L, int64_t S, int64_t B, int64_t D) {
  return (size_t)L * S * kSavedUnits * B * D * sizeof(bf16);
}

size_t block_grid_bwd_workspace_bytes(int64_t L, int64_t S, int64_t B, int64_t D) {
  return block_bwd_ws_layout(L, S, B, D, nullptr, nullptr);
}

int block_grid_bwd(const flb_block_weights* W, const void* x, const void* grids,
                   const void* const* dgrids, float* dx, const flb_block_grads* G, int64_t L,
                   int64_t S, int64_t B, int64_t D, int64_t H, float eps, void* ws,
                   size_t ws_bytes, cudaStream_t s, void* saved) {
  bf16* planes = reinterpret_cast<bf16*>(saved);  // null: recompute
  BlockBwdWs w;
  block_bwd_ws_layout(L, S, B, D, &w, ws);
  SideStream* side;
  int st = side_stream(&side);
  if (st != FLB_OK) return st;
  cublasHandle_t hb, hs;
  if ((st = blas(s, w.blas, kBlkBlasWs, &hb)) != FLB_OK) return st;
  if ((st = blas(side->s, w.blas_side, kBlkBlasWs, &hs, 1)) != FLB_OK) return st;
  // fork: the side stream waits for event k of the tick; join: the caller's stream waits for the
  // side stream before the next tick reuses the tick buffers the side GEMMs read
  auto fork = [&](int k) -> int {
    cudaError_t e = cudaEventRecord(side->fork[k], s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side->s, side->fork[k], 0);
    return check_cuda(e, "block_grid_bwd fork");
  };
  auto join = [&]() -> int {
    cudaError_t e = cudaEventRecord(side->join, side->s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, side->join, 0);
    return check_cuda(e, "block_grid_bwd join");
  };
  const bf16* xb = reinterpret_cast<const bf16*>(x);
  const bf16* g = reinterpret_cast<const bf16*>(grids);
  const int64_t port_stride = (L * S + L) * B * D;
  const int64_t per_port = L * S * B * D;
  const long long DD = D * D, BD = B * D;
  const int Li = (int)L, Si = (int)S, Bi = (int)B, Di = (int)D, Hi = (int)H;
  const int ticks = (int)(L + 2 * S - 2);
  const int ew = 4 * num_sms();
  cudaError_t ce = launch_pdl(blk_dg_init_kernel, dim3(ew), dim3(256), 0, s,
                              (const bf16*)dgrids[0], (const bf16*)dgrids[1],
                              (const bf16*)dgrids[2], w.dG, per_port);
  if (ce != cudaSuccess) return check_cuda(ce, "block_grid_bwd launch");
  ce = cudaMemsetAsync(dx, 0, (size_t)B * S * D * 4, s);
  if (ce != cudaSuccess) return check_cuda(ce, "block_grid_bwd dx reset");
  const bf16* ext3 = (const bf16*)dgrids[3];
  int launches = 1;
  if (saved) {
    // per layer [P_fb ; G_L P_fb] ([2D, D] bf16): P_fb copied in, the product below it
    ce = cudaMemcpy2DAsync(w.wcat, 2 * DD * sizeof(bf16), W->w_prior_fdbk, DD * sizeof(bf16),
                           DD * sizeof(bf16), (size_t)L, cudaMemcpyDeviceToDevice, s);
    if (ce != cudaSuccess) return check_cuda(ce, "block_grid_bwd weight copy");
    if ((st = gemm_rm(hb, false, false, Di, Di, Di, W->w_gate_l, Di, DD, W->w_prior_fdbk, Di, DD,
                      w.wcat + DD, Di, 2 * DD, Li, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
  }
  for (int T = ticks - 1; T >= 0; --T) {
    const Tick tk = tick_of(T, Li, Si);
    const int n = tk.n, l0 = tk.l0;
    if (n == 0) continue;
    // The tick's forward intermediates and its gradient operands, cell i of the tick at
    // base + i * units * cs: with the forward's intermediates kept, the planes themselves (a
    // tick's cells lie 2S - 1 cells apart there; nothing is copied in or out), else the work
    // buffers the recomputed forward fills (cs = B x D)
    int64_t cs = BD;
    const bf16 *f_lat = w.f.lat, *f_tok = w.f.tok, *f_zl = w.f.zl, *f_zx = w.f.zx,
               *f_qkv = w.f.qkv;
    bf16 *d_o = w.d_o, *d_qkv = w.d_qkv, *d_zx = w.d_zx, *d_zl = w.d_zl, *d_lp_h = w.d_lp_h,
         *d_fp_h = w.d_fp_h;
    if (saved) {
      cs = (2 * S - 1) * BD;
      const int64_t c0 = (int64_t)l0 * S + (T - l0) / 2;  // flat index of the tick's first cell
      auto at = [&](int p) { return planes + plane_offset(p, L * S, BD) + c0 * plane_units(p) * BD; };
      f_lat = at(PL_LAT);
      f_tok = at(PL_TOK);
      f_zl = at(PL_ZL);
      f_zx = at(PL_ZX);
      f_qkv = at(PL_QKV);
      d_o = at(PL_DO);
      d_qkv = at(PL_DQKV);
      d_zx = at(PL_DZX);
      d_zl = at(PL_DZL);
      d_lp_h = at(PL_DLP);
      d_fp_h = at(PL_DFP);
    } else if ((st = tick_forward(hb, Side{side, hs}, W, xb, g, port_stride, w.f, T, l0, n, Li, Si,
                                  Bi, Di, Hi, eps, s)) != FLB_OK) {
      return st;
    }
    const dim3 ew_grid((unsigned)((D / 2 + 127) / 128), (unsigned)(n * Bi));
    // gate backward blocks: 32 feature pairs by up to 16 batch rows, one grid row per cell
    const dim3 pair_grid((unsigned)((D / 2 + 31) / 32), (unsigned)n);
    const dim3 pair_block(32, (unsigned)std::min<int64_t>(B, 16));
    if ((ce = launch_pdl(blk_bwd_out_kernel, ew_grid, dim3(128), 0, s, w.dG, per_port, ext3, g,
                         port_stride, f_lat, f_tok, d_o, cs, w.d_top, w.d_lp, w.d_fp, T, l0,
                         Si, Bi, Di)) != cudaSuccess)
      return check_cuda(ce, "block_grid_bwd launch");
    const bf16* Wo = reinterpret_cast<const bf16*>(W->w_o) + (int64_t)l0 * DD;
    const bf16* Wqkv = reinterpret_cast<const bf16*>(W->w_qkv) + (int64_t)l0 * 3 * DD;
    const bf16* Wgx = reinterpret_cast<const bf16*>(W->w_gate_x) + (int64_t)l0 * DD;
    const bf16* Wgl = reinterpret_cast<const bf16*>(W->w_gate_l) + (int64_t)l0 * DD;
    const bf16* Wpl = reinterpret_cast<const bf16*>(W->w_prior_lat) + (int64_t)l0 * DD;
    const bf16* Wpf = reinterpret_cast<const bf16*>(W->w_prior_fdbk) + (int64_t)l0 * DD;
    // output projection
    if ((st = gemm_rm(hb, false, false, 3 * Bi, Di, Di, d_o, Di, 3 * cs, Wo, Di, 2 * DD, w.d_att,
                      Di, 3 * BD, n, 0.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    if (!saved && (st = fork(0)) != FLB_OK) return st;
    if (!saved && (st = gemm_rm(hs, true, false, Di, Di, 3 * Bi, w.d_o, Di, 3 * BD, w.f.att, Di, 3 * BD,
                      G->w_o + (int64_t)l0 * DD, Di, 2 * DD, n, 1.f)) != FLB_OK)
      return st;
    if ((ce = launch_pdl(blk_attn3_bwd_kernel, dim3((n * Bi * Hi + 7) / 8), dim3(256), 0, s,
                         f_qkv, W->v_a, w.d_att, d_qkv, cs, G->v_a, l0, n, Bi, Di, Hi)) !=
        cudaSuccess)
      return check_cuda(ce, "block_grid_bwd launch");
    // q | k | v projections
    if ((st = gemm_rm(hb, false, false, 3 * Bi, Di, 3 * Di, d_qkv, 3 * Di, 9 * cs, Wqkv, Di,
                      6 * DD, w.dT, Di, 3 * BD, n, 0.f)) != FLB_OK)
      return st;
    if (!saved && (st = fork(1)) != FLB_OK) return st;
    if (!saved && (st = gemm_rm(hs, true, false, 3 * Di, Di, 3 * Bi, w.d_qkv, 3 * Di, 9 * BD, w.f.tok, Di,
                      3 * BD, G->w_qkv + (int64_t)l0 * 3 * DD, Di, 6 * DD, n, 1.f)) != FLB_OK)
      return st;
    // sensory gate
    if ((ce = launch_pdl(blk_gx_bwd_kernel, pair_grid, pair_block, 0, s, w.dT, f_zx, W->b_gate_x,
                         g, xb, w.d_top, w.dG, dx, d_zx, w.d_lr, w.d_fp, d_fp_h, cs,
                         saved ? w.dcat : nullptr, G->b_gate_x, T, l0, Si, Bi, Di)) != cudaSuccess)
      return check_cuda(ce, "block_grid_bwd launch");
    if ((st = gemm_rm(hb, false, false, Bi, Di, Di, d_zx, Di, cs, Wgx, Di, 2 * DD, w.d_lr, Di, BD,
                      n, 1.f)) != FLB_OK)
      return st;
    if (!saved && (st = fork(2)) != FLB_OK) return st;
    if (!saved && (st = gemm_rm(hs, true, false, Di, Di, Bi, w.d_zx, Di, BD, w.f.tok + D, 3 * Di, 3 * BD,
                      G->w_gate_x + (int64_t)l0 * DD, Di, 2 * DD, n, 1.f)) != FLB_OK)
      return st;
    // lateral gate
    if ((ce = launch_pdl(blk_gl_bwd_kernel, pair_grid, pair_block, 0, s, w.d_lr, f_zl,
                         W->b_gate_l, f_lat, w.d_lp, d_lp_h, d_zl, cs, saved ? w.dcat : nullptr,
                         G->b_gate_l, l0, Bi, Di)) != cudaSuccess)
      return check_cuda(ce, "block_grid_bwd launch");
    // d_fdbk_prior = bf16(d_zL G_L + its bf16 partial from the sensory-gate backward); with the
    // intermediates kept it is formed after the tick loop for all cells at once (the tick's
    // chain needs only its product with P_fb, below)
    if (!saved && (st = gemm_rm(hb, false, false, Bi, Di, Di, d_zl, Di, cs, Wgl, Di, 2 * DD, d_fp_h,
                                Di, cs, n, 1.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    if (!saved && (st = fork(3)) != FLB_OK) return st;
    if (!saved && (st = gemm_rm(hs, true, false, Di, Di, Bi, w.d_zl, Di, BD, w.f.tok + 2 * D, 3 * Di, 3 * BD,
                      G->w_gate_l + (int64_t)l0 * DD, Di, 2 * DD, n, 1.f)) != FLB_OK)
      return st;
    // priors (with the intermediates kept, the lateral prior's input gradient runs on the side
    // stream beside the z_l / cast / feedback-prior chain; joined before the LayerNorm backward)
    if (saved) {
      if ((st = fork(4)) != FLB_OK) return st;
      if ((st = gemm_rm(hs, false, false, Bi, Di, Di, d_lp_h, Di, cs, Wpl, Di, 2 * DD, w.dA, Di,
                        BD, n, 0.f)) != FLB_OK)
        return st;
    } else if ((st = gemm_rm(hb, false, false, Bi, Di, Di, w.d_lp_h, Di, BD, Wpl, Di, 2 * DD, w.dA,
                             Di, BD, n, 0.f)) != FLB_OK) {
      return st;
    }
    if (saved) {
      // d_LN_diag = d_fdbk_prior P_fb = [partial | d_zL] [P_fb ; G_L P_fb]: one K = 2D GEMM
      if ((st = gemm_rm(hb, false, false, Bi, Di, 2 * Di, w.dcat, 2 * Di, 2 * BD,
                        w.wcat + (int64_t)l0 * 2 * DD, Di, 4 * DD, w.dA + n * BD, Di, BD, n,
                        0.f)) != FLB_OK)
        return st;
    } else if ((st = gemm_rm(hb, false, false, Bi, Di, Di, d_fp_h, Di, cs, Wpf, Di, 2 * DD,
                             w.dA + n * BD, Di, BD, n, 0.f)) != FLB_OK) {
      return st;
    }
    if (!saved && (st = fork(4)) != FLB_OK) return st;
    if (!saved && (st = gemm_rm(hs, true, false, Di, Di, Bi, w.d_lp_h, Di, BD, w.f.ln, Di, BD,
                      G->w_prior_lat + (int64_t)l0 * DD, Di, 2 * DD, n, 1.f)) != FLB_OK)
      return st;
    if (!saved && (st = gemm_rm(hs, true, false, Di, Di, Bi, w.d_fp_h, Di, BD, w.f.ln + n * BD, Di, BD,
                      G->w_prior_fdbk + (int64_t)l0 * DD, Di, 2 * DD, n, 1.f)) != FLB_OK)
      return st;
    if (saved && (st = join()) != FLB_OK) return st;
    if ((ce = launch_pdl(blk_ln_bwd_kernel, dim3((unsigned)((D / 2 + 31) / 32), (unsigned)(2 * n)),
                         pair_block, 4 * B * sizeof(float), s, g,
                         port_stride, w.dA, W->ln_lat_w, W->ln_fdbk_w, w.dG, per_port,
                         G->ln_lat_w, G->ln_lat_b, G->ln_fdbk_w, G->ln_fdbk_b, T, l0, n, Li, Si,
                         Bi, Di, eps)) != cudaSuccess)
      return check_cuda(ce, "block_grid_bwd launch");
    if (!saved && (st = join()) != FLB_OK) return st;
    launches += saved ? 5 : 9;  // own kernels: 5 backward (+ 4 of the recomputed forward)
  }
  if (saved) {
    // Weight gradients: per layer, one GEMM over all of its cells (K = S x rows), from the
    // gradient planes the ticks filled and the activations the forward kept. Each layer's cells
    // are consecutive in every plane: batch = layers, stride = one layer's cells.
    const int64_t LS = L * S;
    auto pl = [&](int p) { return planes + plane_offset(p, LS, BD); };
    const long long c1 = (long long)S * BD, c3 = 3 * c1, c9 = 9 * c1;  // a layer's cells, per plane
    const int K1 = (int)(S * B), K3 = 3 * K1;
    // d_fdbk_prior of every cell = bf16(its partial + d_zL G_L), per layer over all its rows
    if ((st = gemm_rm(hb, false, false, K1, Di, Di, pl(PL_DZL), Di, c1, W->w_gate_l, Di, DD,
                      pl(PL_DFP), Di, c1, Li, 1.f, CUDA_R_16BF)) != FLB_OK)
      return st;
    if ((st = gemm_rm(hb, true, false, Di, Di, K3, pl(PL_DO), Di, c3, pl(PL_ATT), Di, c3, G->w_o, Di,
                      DD, Li, 1.f)) != FLB_OK)
      return st;
    if ((st = gemm_rm(hb, true, false, 3 * Di, Di, K3, pl(PL_DQKV), 3 * Di, c9, pl(PL_TOK), Di, c3,
                      G->w_qkv, Di, 3 * DD, Li, 1.f)) != FLB_OK)
      return st;
    // token slots 1 (lat') and 2 (fdbk_prior): rows of pitch 3D inside the token plane
    if ((st = gemm_rm(hb, true, false, Di, Di, K1, pl(PL_DZX), Di, c1, pl(PL_TOK) + D, 3 * Di, c3,
                      G->w_gate_x, Di, DD, Li, 1.f)) != FLB_OK)
      return st;
    if ((st = gemm_rm(hb, true, false, Di, Di, K1, pl(PL_DZL), Di, c1, pl(PL_TOK) + 2 * D, 3 * Di, c3,
                      G->w_gate_l, Di, DD, Li, 1.f)) != FLB_OK)
      return st;
    if ((st = gemm_rm(hb, true, false, Di, Di, K1, pl(PL_DLP), Di, c1, pl(PL_LN_LEFT), Di, c1,
                      G->w_prior_lat, Di, DD, Li, 1.f)) != FLB_OK)
      return st;
    if ((st = gemm_rm(hb, true, false, Di, Di, K1, pl(PL_DFP), Di, c1, pl(PL_LN_DIAG), Di, c1,
                      G->w_prior_fdbk, Di, DD, Li, 1.f)) != FLB_OK)
      return st;
  }
  count_launches(launches);
  return check_cuda(cudaGetLastError(), "flb block grid backward launch");
}

}  // namespace flb
