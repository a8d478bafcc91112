// Persistent forward of the FLB block grid (inference, bf16, batch 16): ONE cooperative launch
// evaluates every tick of the (layers x positions) grid, one CTA per SM.
//
// A tick's cells (l = l0, l0+2, ..., t = (T - l) / 2) go through five stages separated by grid
// barriers (a counter in global memory, release add / acquire poll, bounded):
//   1. lat_prior = LN(left) P_lat^T, fdbk_prior = LN(diag) P_fb^T, z_l = LN(diag) (G_L P_fb)^T
//   2. z_x = lat' G_X^T                     with lat' = lat_prior * sigmoid(z_l + b_L)
//   3. q | k | v of the tokens [x', lat', fdbk_prior], x' = top * sigmoid(z_x + b_X)
//   4. additive attention over the 3 tokens, one warp per (cell, batch row, head)
//   5. o = W_o att; h_x = o0 + top, h_lat = o1 + lat_prior, h_fdbk = o2 + fdbk_prior,
//      aux = (lat_prior - h_lat)^2 + (fdbk_prior - h_fdbk)^2 into the four port grids
// (models/FLB_Model.py:37-62, 75-96). Each projection is split into tiles of 128 output
// features x the whole K of one cell: swap-AB tcgen05 MMAs (M = 128 features, N = 16 or 48
// rows, K = 16 per instruction) accumulate in TMEM. The activation rows sit in shared memory in
// the 128-byte-swizzled K-major layout the MMA reads. Stages 1 and 2 compute them while writing
// them there (the LayerNorm; lat'), every load of a thread issued before the first is used;
// stages 3 and 5 load them by TMA from buffers the previous stage's epilogues wrote (x' is
// computed in stage 2's epilogue, lat' written once per cell by stage 2's first feature tile).
// Epilogue inputs that do not depend on the MMA are loaded while it runs.
//
// Tiles are dealt round-robin over the CTAs in one sequence that runs across ticks, so that the
// weight bytes of a tick (about 57 MB at 12 layers, d_model 768) spread over every SM. Warp
// roles: 8 compute warps (activations, epilogues, attention, barriers), one producer warp that
// streams this CTA's weight slices by TMA (16 KB atoms of 128 rows x 64 K, no multicast)
// through a ring of shared-memory stages, and one MMA warp. Weights do not depend on any
// stage, so the producer runs ahead across stage and tick boundaries and the next tile's
// weights are in flight while the grid waits at a barrier.
//
// Values are rounded to bf16 where the tick-by-tick path stores them, so both paths compute the
// same quantities. Data written by other CTAs of this launch is read with ld.global.cg (L2).
// Every wait is bounded; a wait that gives up records a code in the error word, raises the
// abort flag so that the other CTAs leave their barriers, drains this CTA's copies and MMAs in
// flight, frees TMEM and returns.
// Included by flb_block.cu inside its namespace, after the tick helpers it uses.
#pragma once

constexpr int kPsCompute = 8;                      // compute warps
constexpr int kPsThreads = (kPsCompute + 2) * 32;  // + producer warp + MMA warp
constexpr int kPsAtom = 128 * 128;                 // weight atom: 128 rows x 64 K bf16 = 16 KB
constexpr int kPsMaxStages = 16;
constexpr int kPsSmemCap = 227 * 1024;
constexpr int kPsB = 16;                           // batch rows (the MMA's N = 16 / 48)
constexpr uint32_t kPsWaitLimit = 1u << 22;        // mbarrier polls
constexpr uint32_t kPsSpinLimit = 1u << 25;        // grid-barrier polls (with backoff)
// A tile's K steps rotate over kPsAcc TMEM accumulators (64 columns apart) so that consecutive
// MMAs do not wait on each other's accumulator; the epilogue adds them in a fixed order.
constexpr int kPsAcc = 4;
constexpr int kPsTmemCols = 64 * kPsAcc;

enum { PS_PLAT = 0, PS_PFB = 1, PS_GLPF = 2, PS_GX = 3, PS_QKV = 4, PS_WO = 5 };

// Activation maps (TMA sources of stages 3 and 5), after the six weight maps.
enum { PS_A_XR = 6, PS_A_LATR = 7, PS_A_FDBK = 8, PS_A_ATT = 9 };

struct PsMaps {
  CUtensorMap m[10];  // weight stacks [L * n_out, D] in PS_* order; activation buffers
};

struct PsArgs {
  const float *ln_lat_w, *ln_lat_b, *ln_fdbk_w, *ln_fdbk_b, *b_gate_l, *b_gate_x, *v_a;
  const bf16* x;  // [B, S, D]
  bf16* g;        // port grids
  int64_t port_stride;
  bf16 *lat, *zl, *fdbk, *xr, *latr, *qkv, *att;  // per-cell buffers of the current tick
  unsigned* ctr;                           // grid barrier counter (zeroed before the launch)
  int* err;                                // error word (first code wins)
  int* abort_flag;
  int L, S, D, H, F, KA, stages, ticks;
  uint32_t act_off;  // byte offset of the activation tile (after the ring)
  float eps;
  uint32_t spin_limit;
  int drop_cta, drop_bar;  // failure-detection test: this CTA skips this barrier's arrival
};

struct PsTile {
  int stage, cell, mat, ft, rows;
};

// Tick-local tile j of n cells: stage 1 [0, 3nF) (cell, matrix PLAT|PFB|GLPF, feature tile),
// stage 2 [3nF, 4nF), stage 3 [4nF, 7nF) (q|k|v: 3F feature tiles), stage 5 [7nF, 8nF).
__device__ __forceinline__ PsTile ps_tile(int j, int n, int F) {
  const int nF = n * F;
  PsTile t;
  if (j < 3 * nF) {
    t.stage = 1;
    t.cell = j / (3 * F);
    const int r = j - t.cell * 3 * F;
    t.mat = r / F;
    t.ft = r - t.mat * F;
    t.rows = kPsB;
  } else if (j < 4 * nF) {
    const int r = j - 3 * nF;
    t.stage = 2;
    t.cell = r / F;
    t.mat = PS_GX;
    t.ft = r - t.cell * F;
    t.rows = kPsB;
  } else if (j < 7 * nF) {
    const int r = j - 4 * nF;
    t.stage = 3;
    t.cell = r / (3 * F);
    t.mat = PS_QKV;
    t.ft = r - t.cell * 3 * F;
    t.rows = 3 * kPsB;
  } else {
    const int r = j - 7 * nF;
    t.stage = 5;
    t.cell = r / F;
    t.mat = PS_WO;
    t.ft = r - t.cell * F;
    t.rows = 3 * kPsB;
  }
  return t;
}

// First tick-local tile >= lo dealt to CTA c: the tiles of the whole launch are numbered in one
// sequence (base = tiles of the earlier ticks) and tile k goes to CTA k mod G.
__device__ __forceinline__ int ps_first(int lo, int c, int G, int base_mod) {
  int off = (c - (base_mod + lo) % G) % G;
  if (off < 0) off += G;
  return lo + off;
}

__device__ __forceinline__ void ps_bar_compute() {
  asm volatile("bar.sync 1, %0;" ::"n"(kPsCompute * 32) : "memory");
}
__device__ __forceinline__ unsigned ps_ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ps_fail(const PsArgs& p, volatile int* stop, int code) {
  atomicCAS(p.err, 0, code);
  atomicExch(p.abort_flag, 1);
  *stop = 1;
}
// Bounded mbarrier wait that also gives up when this CTA is stopping.
__device__ __forceinline__ bool ps_wait(uint64_t* bar, uint32_t phase, volatile int* stop) {
  for (uint32_t i = 0; i < kPsWaitLimit; ++i) {
    if (sm100::mbar_try_wait(bar, phase)) return true;
    if (*stop) return false;
  }
  return false;
}

__device__ __forceinline__ uint4 ldcg16(const bf16* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[e]));
    f[2 * e] = v.x;
    f[2 * e + 1] = v.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
    o[e] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
// 16-byte chunk c (elements 8c .. 8c+7 of K) of activation row `row` in a tile of R rows:
// K atoms of 64 elements, each R rows x 128 bytes, 128-byte swizzle.
__device__ __forceinline__ uint4* ps_act_chunk(uint8_t* act, int R, int row, int c) {
  return reinterpret_cast<uint4*>(act + (c >> 3) * (R * 128) + sm100::sw128_offset(row, c & 7));
}
__device__ __forceinline__ void load_f8(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Stage 1 activation: LayerNorm of the left (P_lat) or bottom-left (P_fb, G_L P_fb) neighbour
// rows of the cell, warp per row with statistics as blk_ln_kernel (zero boundary rows normalise
// to the bias). A warp's rows are loaded before any is reduced.
__device__ __forceinline__ void ps_act_ln(const PsArgs& p, int mat, int l, int t, uint8_t* act,
                                          int warp, int lane) {
  constexpr int RPW = kPsB / kPsCompute;  // rows per warp
  const int D = p.D, nch = D / 8, S = p.S;
  const bool left = mat == PS_PLAT;
  const float* lw = (left ? p.ln_lat_w : p.ln_fdbk_w) + (int64_t)l * D;
  const float* lb = (left ? p.ln_lat_b : p.ln_fdbk_b) + (int64_t)l * D;
  uint4 raw[RPW][kMaxChunks];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int b = warp + kPsCompute * r;
    const bf16* src = nullptr;
    if (t > 0) {
      if (left) src = p.g + p.port_stride + (cell_row(l, t - 1, S) * kPsB + b) * D;
      else if (l + 1 < p.L) src = p.g + 2 * p.port_stride + (cell_row(l + 1, t - 1, S) * kPsB + b) * D;
    }
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = lane + 32 * k;
      raw[r][k] = (src && c < nch) ? ldcg16(src + 8 * c) : make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int b = warp + kPsCompute * r;
    float v[kMaxChunks][8];
    float s = 0.f, ss = 0.f;
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      unpack8(raw[r][k], v[k]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s += v[k][2 * e] + v[k][2 * e + 1];
        ss += v[k][2 * e] * v[k][2 * e] + v[k][2 * e + 1] * v[k][2 * e + 1];
      }
    }
    s = warp_sum(s);
    ss = warp_sum(ss);
    const float mean = s / D;
    const float rstd = rsqrtf(fmaxf(ss / D - mean * mean, 0.f) + p.eps);
#pragma unroll
    for (int k = 0; k < kMaxChunks; ++k) {
      const int c = lane + 32 * k;
      if (c >= nch) break;
      float w8[8], b8[8], o[8];
      load_f8(lw + 8 * c, w8);
      load_f8(lb + 8 * c, b8);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[k][e] - mean) * rstd * w8[e] + b8[e];
      *ps_act_chunk(act, kPsB, b, c) = pack8(o);
    }
  }
}

// Stage 2 activation: lat' = lat_prior * sigmoid(z_l + b_L) (as blk_gate_kernel, mode 0), also
// stored to the lat' buffer when `store` (one CTA per cell), for stage 3's TMA. D <= 1024: a
// thread's (at most 8) chunks are loaded before any is used.
__device__ __forceinline__ void ps_act_latr(const PsArgs& p, int cell, int l, uint8_t* act, int tid,
                                            bool store) {
  constexpr int U = 8;
  const int D = p.D, nch = D / 8, total = kPsB * nch;
  uint4 m[U], z[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int q = tid + kPsCompute * 32 * u;
    if (q < total) {
      const int b = q / nch, c = q - b * nch;
      const int64_t o = ((int64_t)cell * kPsB + b) * D + 8 * c;
      m[u] = ldcg16(p.lat + o);
      z[u] = ldcg16(p.zl + o);
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int q = tid + kPsCompute * 32 * u;
    if (q < total) {
      const int b = q / nch, c = q - b * nch;
      float mf[8], zf[8], bi[8], r[8];
      unpack8(m[u], mf);
      unpack8(z[u], zf);
      load_f8(p.b_gate_l + (int64_t)l * D + 8 * c, bi);
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = mf[e] * (1.f / (1.f + __expf(-(zf[e] + bi[e]))));
      const uint4 val = pack8(r);
      *ps_act_chunk(act, kPsB, b, c) = val;
      if (store) *reinterpret_cast<uint4*>(p.latr + ((int64_t)cell * kPsB + b) * D + 8 * c) = val;
    }
  }
}

// Stages 3 and 5: the activation rows by TMA (one thread). Stage 3 rows are token-major
// (x' rows 0-15, lat' 16-31, fdbk_prior 32-47); stage 5 rows are the attention output's
// (3b + token).
__device__ __forceinline__ void ps_act_tma(const PsMaps& maps, const PsTile& tl, int KA,
                                           uint8_t* act, uint64_t* bar) {
  using namespace sm100;
  fence_async_global();  // the buffers were written by generic stores before the grid barrier
  if (tl.stage == 3) {
    mbar_arrive_expect_tx(bar, (uint32_t)(3 * KA * kPsB * 128));
    for (int r = 0; r < 3; ++r) {
      const CUtensorMap* m = &maps.m[r == 0 ? PS_A_XR : r == 1 ? PS_A_LATR : PS_A_FDBK];
      for (int a = 0; a < KA; ++a)
        tma_load_2d(act + a * (3 * kPsB * 128) + r * (kPsB * 128), m, bar, a * 64, tl.cell * kPsB);
    }
  } else {
    mbar_arrive_expect_tx(bar, (uint32_t)(KA * 3 * kPsB * 128));
    for (int a = 0; a < KA; ++a)
      tma_load_2d(act + a * (3 * kPsB * 128), &maps.m[PS_A_ATT], bar, a * 64, tl.cell * 3 * kPsB);
  }
}

// Epilogue inputs that do not depend on the MMA, loaded before its completion is awaited. Warp
// w's thread holds feature f = ft*128 + 32(w%4) + lane and accumulator columns 8h .. 8h+7 (16-row
// tiles) or 24h .. 24h+23 (48-row tiles), h = w / 4. Stage 2: the top rows b = 8h + c; stage 5:
// top, lat_prior and fdbk_prior of rows b = 8h + bb, as pre[3bb + 0|1|2].
struct PsPre {
  float v[24];
};

__device__ __forceinline__ const bf16* ps_top(const PsArgs& p, int l, int t, int b) {
  return l > 0 ? p.g + (cell_row(l - 1, t, p.S) * kPsB + b) * p.D : p.x + ((int64_t)b * p.S + t) * p.D;
}

__device__ __forceinline__ void ps_prefetch(const PsArgs& p, const PsTile& tl, int l, int t, int tid,
                                            PsPre& pre) {
  const int warp = tid >> 5, lane = tid & 31;
  const int half = warp >> 2;
  const int f = tl.ft * 128 + 32 * (warp & 3) + lane;
  if (tl.stage == 2) {
#pragma unroll
    for (int c = 0; c < 8; ++c) pre.v[c] = ld_bf16_cg(ps_top(p, l, t, 8 * half + c) + f);
  } else if (tl.stage == 5) {
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) {
      const int b = 8 * half + bb;
      const int64_t rb = (int64_t)tl.cell * kPsB + b;
      pre.v[3 * bb] = ld_bf16_cg(ps_top(p, l, t, b) + f);
      pre.v[3 * bb + 1] = ld_bf16_cg(p.lat + rb * p.D + f);
      pre.v[3 * bb + 2] = ld_bf16_cg(p.fdbk + rb * p.D + f);
    }
  }
}

__device__ __forceinline__ float round_bf16f(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// 8 accumulator columns at taddr summed over the kPsAcc accumulators (in index order).
__device__ __forceinline__ void ps_tmem_sum8(uint32_t taddr, float* out) {
  using namespace sm100;
  uint32_t r[kPsAcc][8];
#pragma unroll
  for (int k = 0; k < kPsAcc; ++k) tmem_ld8(taddr + 64 * k, r[k]);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float v = __uint_as_float(r[0][c]);
#pragma unroll
    for (int k = 1; k < kPsAcc; ++k) v += __uint_as_float(r[k][c]);
    out[c] = v;
  }
}

// Epilogue of a tile: TMEM lane quarter w % 4, column half w / 4 (see PsPre).
__device__ __forceinline__ void ps_epilogue(const PsArgs& p, const PsTile& tl, int l, int t,
                                            uint32_t tmem, int tid, const PsPre& pre) {
  using namespace sm100;
  const int warp = tid >> 5, lane = tid & 31;
  const int q4 = warp & 3, half = warp >> 2;
  const int64_t D = p.D;
  const uint32_t taddr = tmem + ((uint32_t)(32 * q4) << 16);
  const int f = tl.ft * 128 + 32 * q4 + lane;
  if (tl.rows == kPsB) {
    float r[8];
    ps_tmem_sum8(taddr + 8 * half, r);
    if (tl.stage == 2) {
      // x' = top * sigmoid(z_x + b_X) (z_x rounded to bf16 as the tick path stores it)
      const float bx = __ldg(p.b_gate_x + (int64_t)l * D + f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int b = 8 * half + c;
        const float z = round_bf16f(r[c]);
        p.xr[((int64_t)tl.cell * kPsB + b) * D + f] =
            __float2bfloat16_rn(pre.v[c] * (1.f / (1.f + __expf(-(z + bx)))));
      }
      return;
    }
    bf16* out = tl.mat == PS_PLAT ? p.lat : tl.mat == PS_PFB ? p.fdbk : p.zl;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int b = 8 * half + c;
      out[((int64_t)tl.cell * kPsB + b) * D + f] = __float2bfloat16_rn(r[c]);
    }
    return;
  }
  float acc[24];
  ps_tmem_sum8(taddr + 24 * half, acc);
  ps_tmem_sum8(taddr + 24 * half + 8, acc + 8);
  ps_tmem_sum8(taddr + 24 * half + 16, acc + 16);
  if (tl.stage == 3) {
    // column j = 16 token + b -> q|k|v row 3b + token
    bf16* dst = p.qkv + (int64_t)tl.cell * 3 * kPsB * 3 * D + f;
#pragma unroll
    for (int c = 0; c < 24; ++c) {
      const int j = 24 * half + c, tok = j >> 4, b = j & 15;
      dst[(int64_t)(3 * b + tok) * 3 * D] = __float2bfloat16_rn(acc[c]);
    }
    return;
  }
  // o = W_o att, columns (b, token); residuals and aux into the port grids (as blk_out_kernel)
#pragma unroll
  for (int bb = 0; bb < 8; ++bb) {
    const int b = 8 * half + bb;
    const float top = pre.v[3 * bb], lp = pre.v[3 * bb + 1], fp = pre.v[3 * bb + 2];
    const bf16 hx = __float2bfloat16_rn(round_bf16f(acc[3 * bb]) + top);
    const bf16 hl = __float2bfloat16_rn(round_bf16f(acc[3 * bb + 1]) + lp);
    const bf16 hf = __float2bfloat16_rn(round_bf16f(acc[3 * bb + 2]) + fp);
    const float dl = lp - __bfloat162float(hl), df = fp - __bfloat162float(hf);
    const int64_t off = (cell_row(l, t, p.S) * kPsB + b) * D + f;
    p.g[off] = hx;
    p.g[p.port_stride + off] = hl;
    p.g[2 * p.port_stride + off] = hf;
    p.g[3 * p.port_stride + off] = __float2bfloat16_rn(dl * dl + df * df);
  }
}
// Grid barrier of the compute warps. Returns false when this CTA stops (a barrier that gave up
// here or elsewhere).
__device__ __forceinline__ bool ps_grid_sync(const PsArgs& p, unsigned& target, int& bar_index,
                                             volatile int* stop) {
  sm100::fence_async_global();  // this thread's stores may be read by TMA after the barrier
  ps_bar_compute();
  target += gridDim.x;
  if (threadIdx.x == 0 && !*stop) {
    __threadfence();
    if (!((int)blockIdx.x == p.drop_cta && bar_index == p.drop_bar)) atomicAdd(p.ctr, 1u);
    for (uint32_t it = 0;; ++it) {
      if (ps_ld_acquire(p.ctr) >= target) break;
      if (*(volatile int*)p.abort_flag) {
        *stop = 1;
        break;
      }
      if (it > p.spin_limit) {
        ps_fail(p, stop, 31);
        break;
      }
      if (it > 32) __nanosleep(40);
    }
    __threadfence();
  }
  ++bar_index;
  ps_bar_compute();
  return !*stop;
}

__global__ void __launch_bounds__(kPsThreads, 1)
flb_persist_fwd_kernel(const __grid_constant__ PsMaps maps, const PsArgs p) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* act = sm + p.act_off;
  __shared__ __align__(8) uint64_t full[kPsMaxStages], freed[kPsMaxStages];
  __shared__ __align__(8) uint64_t act_full, acc_full, drain;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int stop;
  __shared__ uint32_t consumed, issued;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, c = blockIdx.x;
  const int STG = p.stages;
  if (tid == 0) {
    for (int s = 0; s < STG; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&freed[s], 1);
    }
    mbar_init(&act_full, 1);
    mbar_init(&acc_full, 1);
    mbar_init(&drain, 1);
    fence_mbar_init();
    stop = 0;
    consumed = issued = 0;
  }
  if (warp == kPsCompute + 1) {
    tmem_alloc(&tmem_slot, kPsTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  const uint32_t tmem = tmem_slot;

  if (warp == kPsCompute) {
    // ---- producer: this CTA's weight atoms, in tile order, through the ring ----------------
    if (lane == 0) {
      for (int i = 0; i < 10; ++i) tma_prefetch_desc(&maps.m[i]);
      const uint64_t keep = l2_evict_last_policy();  // the weights are re-read every other tick
      uint32_t aseq = 0;
      int base_mod = 0;
      for (int T = 0; T < p.ticks && !stop; ++T) {
        const Tick tk = tick_of(T, p.L, p.S);
        if (tk.n == 0) continue;
        const int nt = 8 * tk.n * p.F;
        for (int j = ps_first(0, c, G, base_mod); j < nt && !stop; j += G) {
          const PsTile tl = ps_tile(j, tk.n, p.F);
          const int l = tk.l0 + 2 * tl.cell;
          const int row = l * (tl.mat == PS_QKV ? 3 * p.D : p.D) + tl.ft * 128;
          for (int a = 0; a < p.KA; ++a) {
            const int s = aseq % STG;
            if (aseq >= (uint32_t)STG && !ps_wait(&freed[s], ((aseq / STG) - 1) & 1u, &stop)) {
              if (!stop) ps_fail(p, &stop, 34);
              break;
            }
            mbar_arrive_expect_tx(&full[s], kPsAtom);
            tma_load_2d_hint(sm + s * kPsAtom, &maps.m[tl.mat], &full[s], a * 64, row, keep);
            ++aseq;
          }
        }
        base_mod = (base_mod + nt) % G;
      }
      issued = aseq;
    }
  } else if (warp == kPsCompute + 1) {
    // ---- MMA issuer ---------------------------------------------------------------------------
    if (lane == 0) {
      uint32_t aseq = 0, tseq = 0;
      int base_mod = 0;
      const uint32_t wa = smem_u32(sm), xa = smem_u32(act);
      for (int T = 0; T < p.ticks && !stop; ++T) {
        const Tick tk = tick_of(T, p.L, p.S);
        if (tk.n == 0) continue;
        const int nt = 8 * tk.n * p.F;
        for (int j = ps_first(0, c, G, base_mod); j < nt && !stop; j += G) {
          const PsTile tl = ps_tile(j, tk.n, p.F);
          if (!ps_wait(&act_full, tseq & 1u, &stop)) {
            if (!stop) ps_fail(p, &stop, 32);
            break;
          }
          tc_fence_after();
          const uint32_t idesc = make_idesc_f16(128, tl.rows, 1, 0, 0);
          const uint32_t act_atom = (uint32_t)tl.rows * 128u;
          bool ok = true;
          for (int a = 0; a < p.KA; ++a) {
            const int s = aseq % STG;
            if (!ps_wait(&full[s], (aseq / STG) & 1u, &stop)) {
              if (!stop) ps_fail(p, &stop, 33);
              ok = false;
              break;
            }
            // the mbarrier wait orders the TMA's shared-memory writes before these reads (both
            // async proxy); no tcgen05 fence here, it would wait for the previous atom's MMAs
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16(tmem + 64 * (kk % kPsAcc),
                       make_smem_desc(wa + s * kPsAtom + kk * 32, 16, 1024, kSwizzle128B),
                       make_smem_desc(xa + a * act_atom + kk * 32, 16, 1024, kSwizzle128B),
                       idesc, (a * 4 + kk >= kPsAcc) ? 1u : 0u);
            umma_commit(&freed[s]);
            ++aseq;
          }
          if (!ok) break;
          umma_commit(&acc_full);
          ++tseq;
        }
        base_mod = (base_mod + nt) % G;
      }
      consumed = aseq;
      // nothing of this thread's may still run on the tensor cores at exit
      umma_commit(&drain);
      if (!mbar_wait(&drain, 0, kPsWaitLimit)) ps_fail(p, &stop, 36);
    }
  } else {
    // ---- compute warps -------------------------------------------------------------------------
    uint32_t tseq = 0;
    unsigned target = 0;
    int bar_index = 0, base_mod = 0;
    for (int T = 0; T < p.ticks; ++T) {
      const Tick tk = tick_of(T, p.L, p.S);
      if (tk.n == 0) continue;
      const int nF = tk.n * p.F;
      for (int st = 0; st < 5; ++st) {
        if (st == 3) {
          // stage 4: the 3-token attention, one warp per (cell, batch row, head)
          const int tasks = tk.n * kPsB * p.H;
          for (int task = c * kPsCompute + warp; task < tasks; task += G * kPsCompute)
            attn3_task(p.qkv, p.v_a, p.att, (int64_t)kPsB * p.D, tk.l0, kPsB, p.D, p.H, task, lane);
        } else {
          // tile ranges of stages 1, 2, 3, (4), 5
          const int lo = st == 0 ? 0 : st == 1 ? 3 * nF : st == 2 ? 4 * nF : 7 * nF;
          const int hi = st == 0 ? 3 * nF : st == 1 ? 4 * nF : st == 2 ? 7 * nF : 8 * nF;
          for (int j = ps_first(lo, c, G, base_mod); j < hi; j += G) {
            const PsTile tl = ps_tile(j, tk.n, p.F);
            const int l = tk.l0 + 2 * tl.cell, t = (T - l) / 2;
            if (tl.stage <= 2) {
              if (tl.stage == 1) ps_act_ln(p, tl.mat, l, t, act, warp, lane);
              else ps_act_latr(p, tl.cell, l, act, tid, tl.ft == 0);
              fence_async_shared();
              ps_bar_compute();
              if (tid == 0) mbar_arrive(&act_full);
            } else if (tid == 0) {
              ps_act_tma(maps, tl, p.KA, act, &act_full);
            }
            PsPre pre;
            ps_prefetch(p, tl, l, t, tid, pre);
            if (tid == 0 && !ps_wait(&acc_full, tseq & 1u, &stop) && !stop) ps_fail(p, &stop, 35);
            ps_bar_compute();
            if (stop) goto done;
            tc_fence_after();
            ps_epilogue(p, tl, l, t, tmem, tid, pre);
            tc_fence_before();
            ++tseq;
          }
        }
        if (!ps_grid_sync(p, target, bar_index, &stop)) goto done;
      }
      base_mod = (base_mod + 8 * nF) % G;
    }
  done:;
  }
  __syncthreads();
  // copies this CTA issued that no MMA consumed (a stop in mid-run) must land before exit
  if (warp == kPsCompute && lane == 0) {
    for (uint32_t a = consumed; a < issued; ++a)
      if (!mbar_wait(&full[a % STG], (a / STG) & 1u, kPsWaitLimit)) {
        ps_fail(p, &stop, 36);
        break;
      }
  }
  __syncthreads();
  if (warp == kPsCompute + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPsTmemCols);
  }
}
