// Blackwell (sm_100a) additive-attention forward for bf16/fp16 inputs, head dim 64 or 128.
//
// Per CTA: 128 query rows of one (batch, head). D / 32 threads share a row, each holding 32 of
// its head dims: 8 warps (D = 64, two CTAs per SM) or 16 warps (D = 128, one CTA per SM), so
// 16 warps per SM hide the MUFU and shared-memory latencies at 128 registers per thread.
//   * K and V tiles of 64 keys stream into shared memory with TMA (3-D tensor maps over
//     [BH, N, D], no multicast), 3 stages, completion on mbarriers.
//   * Scores are an FMA/MUFU elementwise reduction, not a GEMM: each thread keeps its part of
//     the q row in fp32 registers and, for every key, accumulates w'[d] * tanh.approx(q[d] +
//     k[d]) with fp32 FADD / MUFU / FFMA (w' = w * log2(e) / sqrt(D), so scores are in log2
//     units); a shuffle butterfly over the row's lanes completes the sum. K is read from shared
//     memory with broadcast 16-byte loads. On B200 the packed tanh.approx.{f16x2,bf16x2} forms
//     deliver the same elements per second as the f32 form, so fp32 costs nothing and keeps
//     full accumulation precision.
//   * Softmax: every lane of a row holds the row's full scores, so no further reduction. The
//     row keeps a reference max m fixed from its first keys; P = exp2(s - m). Only if a later
//     group's max exceeds m by more than 8 (P would exceed 256) is the row rescaled: its P
//     pieces of the tile at once, the accumulator rows in TMEM at the end of the tile (rare: the
//     scores of this operator are bounded by sum|w|/sqrt(D)).
//   * P (bf16/fp16, the dtype of V) is written by the threads into a K-major 128-byte-swizzled
//     shared tile; one elected thread issues tcgen05.mma (M=128, N=D, K=16 steps) with V as an
//     MN-major operand, accumulating O in TMEM. MMA completion (tcgen05.commit -> mbarrier)
//     gates the reuse of the P and V buffers, so the tensor core runs one tile behind the
//     score computation.
//   * Epilogue: tcgen05.ld of the rows, scale by 1/l, store; lse = (m + log2 l) * ln 2.
// Every mbarrier wait is bounded; a wait that gives up records an error code in the error
// word (workspace) and the kernel still releases its TMEM and exits.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace flb {

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr float kRescaleThreshold = 8.f;  // log2 units

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 64;
  static constexpr int TPR = D / 32;               // threads per query row, 32 dims each
  static constexpr int THREADS = BM * TPR;         // 256 (D = 64) or 512 (D = 128)
  static constexpr int MIN_BLOCKS = (D == 64) ? 2 : 1;
  static constexpr int STAGES = 3;
  static constexpr int KTILE = BN * D * 2;   // bytes, bf16/fp16
  static constexpr int VTILE = BN * D * 2;
  static constexpr int PTILE = BM * BN * 2;  // 16 KB
  static constexpr int OFF_V = 0;                          // 1024-aligned (swizzled)
  static constexpr int OFF_P = OFF_V + STAGES * VTILE;     // 1024-aligned (swizzled)
  static constexpr int OFF_K = OFF_P + 2 * PTILE;
  static constexpr int OFF_W = OFF_K + STAGES * KTILE;
  static constexpr int SMEM = OFF_W + D * 4 + 1024;        // + slack for 1024-alignment
  static constexpr int TMEM_COLS = D;                      // 64 or 128 (power of two >= 32)
};

template <typename T> struct Unpack;
template <> struct Unpack<__nv_bfloat16> {
  static __device__ __forceinline__ void run(uint32_t v, float& a, float& b) {
    a = __uint_as_float(v << 16);
    b = __uint_as_float(v & 0xFFFF0000u);
  }
  static __device__ __forceinline__ uint32_t pack(float a, float b, float& ra, float& rb) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    ra = __low2float(h);
    rb = __high2float(h);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr int is_bf16 = 1;
};
template <> struct Unpack<__half> {
  static __device__ __forceinline__ void run(uint32_t v, float& a, float& b) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    float2 f = __half22float2(h);
    a = f.x;
    b = f.y;
  }
  static __device__ __forceinline__ uint32_t pack(float a, float b, float& ra, float& rb) {
    __half2 h = __floats2half2_rn(a, b);
    float2 f = __half22float2(h);
    ra = f.x;
    rb = f.y;
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static constexpr int is_bf16 = 0;
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed half-precision helpers of the backward's tanh grid. On B200 tanh.approx.f16x2 and the
// f16x2 add/mul/fma deliver as many elements per second as their f32 forms with half the
// instructions, and that stage is issue-bound.
__device__ __forceinline__ __half2 tanh_h2(__half2 x) {
  uint32_t r, v = *reinterpret_cast<uint32_t*>(&x);
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(r) : "r"(v));
  return *reinterpret_cast<__half2*>(&r);
}
__device__ __forceinline__ void red_shared_f32(float* p, float v) {
  asm volatile("red.shared.add.f32 [%0], %1;" ::"r"(sm100::smem_u32(p)), "f"(v) : "memory");
}
template <typename T> __device__ __forceinline__ __half2 to_h2(uint32_t packed);
template <> __device__ __forceinline__ __half2 to_h2<__half>(uint32_t packed) {
  return *reinterpret_cast<__half2*>(&packed);
}
template <> __device__ __forceinline__ __half2 to_h2<__nv_bfloat16>(uint32_t packed) {
  return __floats2half2_rn(__uint_as_float(packed << 16), __uint_as_float(packed & 0xFFFF0000u));
}

template <int D, typename T>
__global__ void __launch_bounds__(FwdCfg<D>::THREADS, FwdCfg<D>::MIN_BLOCKS)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                   const T* __restrict__ q, T* __restrict__ out, float* __restrict__ lse,
                   float* __restrict__ scores, const float* __restrict__ w,
                   const int32_t* __restrict__ w_index, int N, int causal, int nbh,
                   int scores_vec, float* __restrict__ part_o, float* __restrict__ part_ml,
                   int* __restrict__ err) {
  using namespace sm100;
  using C = FwdCfg<D>;
  using U = Unpack<T>;
  constexpr int TPR = C::TPR;     // threads per query row
  constexpr int DH = D / TPR;     // head dims per thread (32)
  constexpr int KPT = 8 / TPR;    // keys of each 8-key group this thread scores into P
  constexpr int RPW = 32 / TPR;   // rows per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t mma_bar[2];
  __shared__ uint32_t tmem_slot;
  __shared__ float sAlpha[C::BM];  // per-row accumulator rescale of the current tile
  __shared__ float sL[C::BM];      // per-row softmax denominators for the epilogue

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // TPR consecutive lanes of a warp share a query row, each owning DH of its head dims. Warp w
  // serves TMEM lane quarter w % 4 (the only lanes its tcgen05.ld/st may touch): rows
  // 32 (w % 4) + RPW (w / 4) + lane / TPR of the 128-row tile.
  const int quarter = warp & 3, wsub = warp >> 2;
  const int dh = lane % TPR;
  const int mrow = 32 * quarter + RPW * wsub + lane / TPR;
  // 1-D grid over (work item, head), heaviest items of every head first (causal work grows with
  // the block index): the longest CTAs start in the first wave, not in the tail. A work item is
  // a query block, or, when part_o is given (causal, few CTAs per SM), half of the key tiles of
  // a query block qb >= 1: items u = 0, 1 are the two halves of block nqb - 1, u = 2, 3 those
  // of block nqb - 2, ..., and the last item is block 0 whole. Each half writes fp32 partials
  // (unnormalised O, reference max and row sum) that a combine kernel merges.
  const int nqb = (N + C::BM - 1) / C::BM;
  const bool split = part_o != nullptr;
  const int lin = blockIdx.x;
  const int bh = lin % nbh;
  const int u = lin / nbh;
  int qb, half = -1;
  if (split) {
    qb = u < 2 * (nqb - 1) ? nqb - 1 - (u >> 1) : 0;
    if (qb > 0) half = u & 1;
  } else {
    qb = causal ? (nqb - 1 - u) : u;
  }
  const int m0 = qb * C::BM;
  const int row = m0 + mrow;
  const bool row_ok = row < N;
  const int kend = causal ? min(N, m0 + C::BM) : N;
  const int ntiles_all = (kend + C::BN - 1) / C::BN;
  // a half's key tiles: [0, mid) or [mid, ntiles_all). For qb >= 1 the first key of the second
  // half, 64 mid <= 64 (qb + 1) <= 128 qb, is at or before every row of the block, so each half's
  // first key group holds a valid key of every row (its reference max is finite)
  const int mid = (ntiles_all + 1) / 2;
  const int tile0 = half == 1 ? mid : 0;
  const int ntiles = half < 0 ? ntiles_all : (half == 0 ? mid : ntiles_all - mid);
  const int warp_last_row = m0 + 32 * quarter + RPW * wsub + RPW - 1;

  float* sW = reinterpret_cast<float*>(sm + C::OFF_W);
  if (tid < D) sW[tid] = w[(int64_t)w_index[bh] * D + tid] * (kLog2e * rsqrtf((float)D));
  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) mbar_init(&full_bar[s], 1);
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  // this thread's half of the q row -> fp32 registers
  float qr[DH];
  {
    const uint4* src = reinterpret_cast<const uint4*>(
        q + ((int64_t)bh * N + (row_ok ? row : 0)) * D + dh * DH);
#pragma unroll
    for (int c = 0; c < DH / 8; ++c) {
      uint4 v = row_ok ? src[c] : make_uint4(0, 0, 0, 0);
      U::run(v.x, qr[8 * c + 0], qr[8 * c + 1]);
      U::run(v.y, qr[8 * c + 2], qr[8 * c + 3]);
      U::run(v.z, qr[8 * c + 4], qr[8 * c + 5]);
      U::run(v.w, qr[8 * c + 6], qr[8 * c + 7]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tmem_quarter = tmem + ((uint32_t)(quarter * 32) << 16);

  auto issue_tile = [&](int t) {
    const int s = t % C::STAGES;
    mbar_arrive_expect_tx(&full_bar[s], C::KTILE + C::VTILE);
    tma_load_3d(sm + C::OFF_K + s * C::KTILE, &tmK, &full_bar[s], 0, (tile0 + t) * C::BN, bh);
#pragma unroll
    for (int vb = 0; vb < D / 64; ++vb)
      tma_load_3d(sm + C::OFF_V + s * C::VTILE + vb * (C::BN * 128), &tmV, &full_bar[s], vb * 64,
                  (tile0 + t) * C::BN, bh);
  };
  if (tid == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int t = 0; t < min(ntiles, C::STAGES - 1); ++t) issue_tile(t);
  }

  // m_ref, l and the P values are per row; both threads of a row compute the same full scores
  // (a + b == b + a exactly), so they take identical softmax decisions. Each thread adds only
  // its own four keys of every group to l and writes only their 8 bytes of the P chunk.
  float m_ref = 0.f, l = 0.f, alpha_tile = 1.f;
  const uint32_t idesc = make_idesc_f16(128, D, U::is_bf16, 0, 1);

  for (int t = 0; t < ntiles; ++t) {
    const int s = t % C::STAGES;
    const int j0 = (tile0 + t) * C::BN;
    if (!mbar_wait(&full_bar[s], (uint32_t)(t / C::STAGES) & 1u, kWaitLimit)) atomicExch(err, 1);
    const uint8_t* sK = sm + C::OFF_K + s * C::KTILE;
    const int b = t & 1;
    // P buffer b was last read by MMA t-2
    if (t >= 2 && !mbar_wait(&mma_bar[b], (uint32_t)((t - 2) >> 1) & 1u, kWaitLimit))
      atomicExch(err, 3);
    uint8_t* sP = sm + C::OFF_P + b * C::PTILE;

    // Streaming over groups of 8 keys: scores (log2 units) -> P chunk of 16 bytes.
#pragma unroll 1
    for (int g = 0; g < C::BN / 8; ++g) {
      const int jg = j0 + g * 8;
      float s8[8];
      if (causal && jg > warp_last_row) {  // warp-uniform: all 8 keys masked for every row
#pragma unroll
        for (int e = 0; e < 8; ++e) s8[e] = -INFINITY;
      } else {
        float acc[8][2];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e][0] = acc[e][1] = 0.f;
        const uint8_t* kg = sK + (g * 8) * D * 2 + dh * DH * 2;
        const float4* wh = reinterpret_cast<const float4*>(sW + dh * DH);
#pragma unroll
        for (int c = 0; c < DH / 8; ++c) {
          const float4 w0 = wh[2 * c];
          const float4 w1 = wh[2 * c + 1];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint4 kk = reinterpret_cast<const uint4*>(kg + e * D * 2)[c];
            float k0, k1, k2, k3, k4, k5, k6, k7;
            U::run(kk.x, k0, k1);
            U::run(kk.y, k2, k3);
            U::run(kk.z, k4, k5);
            U::run(kk.w, k6, k7);
            acc[e][0] = fmaf(w0.x, tanh_approx(qr[8 * c + 0] + k0), acc[e][0]);
            acc[e][1] = fmaf(w0.y, tanh_approx(qr[8 * c + 1] + k1), acc[e][1]);
            acc[e][0] = fmaf(w0.z, tanh_approx(qr[8 * c + 2] + k2), acc[e][0]);
            acc[e][1] = fmaf(w0.w, tanh_approx(qr[8 * c + 3] + k3), acc[e][1]);
            acc[e][0] = fmaf(w1.x, tanh_approx(qr[8 * c + 4] + k4), acc[e][0]);
            acc[e][1] = fmaf(w1.y, tanh_approx(qr[8 * c + 5] + k5), acc[e][1]);
            acc[e][0] = fmaf(w1.z, tanh_approx(qr[8 * c + 6] + k6), acc[e][0]);
            acc[e][1] = fmaf(w1.w, tanh_approx(qr[8 * c + 7] + k7), acc[e][1]);
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // butterfly over the TPR lanes of the row: every lane ends with the same sum
          float full = acc[e][0] + acc[e][1];
#pragma unroll
          for (int o = 1; o < TPR; o <<= 1) full += __shfl_xor_sync(0xffffffffu, full, o);
          const int key = jg + e;
          const bool ok = key < N && (!causal || key <= row);
          s8[e] = ok ? full : -INFINITY;
        }
      }
      // this thread's keys of the group: KPT dh .. KPT dh + KPT - 1
      float sk[KPT];
#pragma unroll
      for (int e = 0; e < KPT; ++e) {
        sk[e] = s8[e];
#pragma unroll
        for (int o = 1; o < TPR; ++o)
          if (dh == o) sk[e] = s8[KPT * o + e];
      }
      if (scores != nullptr && row_ok) {
        const int k0 = jg + KPT * dh;
        float* dst = scores + ((int64_t)bh * N + row) * attn_scores_ld(N) + k0;
        if (scores_vec && k0 + KPT - 1 < N && (!causal || k0 + KPT - 1 <= row)) {
          if constexpr (KPT == 4)
            *reinterpret_cast<float4*>(dst) =
                make_float4(sk[0] * kLn2, sk[1] * kLn2, sk[2] * kLn2, sk[3] * kLn2);
          else
            *reinterpret_cast<float2*>(dst) = make_float2(sk[0] * kLn2, sk[1] * kLn2);
        } else {
#pragma unroll
          for (int e = 0; e < KPT; ++e)
            if (k0 + e < N && (!causal || k0 + e <= row)) dst[e] = sk[e] * kLn2;
        }
      }
      float gm = s8[0];
#pragma unroll
      for (int e = 1; e < 8; ++e) gm = fmaxf(gm, s8[e]);

      // reference max: fixed by the first group of the row; raised (rarely) when a group's max
      // exceeds it by more than the threshold. The accumulator rows in TMEM are rescaled once,
      // at the end of the tile (alpha_tile), before the tile's MMA.
      if (t == 0 && g == 0) {
        m_ref = row_ok ? gm : 0.f;
      } else if (row_ok && gm > m_ref + kRescaleThreshold) {
        const float alpha = ex2_approx(m_ref - gm);
        l *= alpha;
        alpha_tile *= alpha;
        m_ref = gm;
        // this thread's pieces of chunks 0..g-1 of the tile's P row used the old reference
        for (int c = 0; c < g; ++c) {
          uint32_t* pc = reinterpret_cast<uint32_t*>(sP + sw128_offset(mrow, c) + 2 * KPT * dh);
#pragma unroll
          for (int e = 0; e < KPT / 2; ++e) {
            float lo, hi, r0, r1;
            U::run(pc[e], lo, hi);
            pc[e] = U::pack(lo * alpha, hi * alpha, r0, r1);
          }
        }
      }
      uint32_t pk[KPT / 2];
#pragma unroll
      for (int e = 0; e < KPT / 2; ++e) {
        const float p0 = row_ok ? ex2_approx(sk[2 * e] - m_ref) : 0.f;
        const float p1 = row_ok ? ex2_approx(sk[2 * e + 1] - m_ref) : 0.f;
        float r0, r1;
        pk[e] = U::pack(p0, p1, r0, r1);
        l += r0 + r1;
      }
      uint8_t* pdst = sP + sw128_offset(mrow, g) + 2 * KPT * dh;
      if constexpr (KPT == 4)
        *reinterpret_cast<uint2*>(pdst) = make_uint2(pk[0], pk[1]);
      else
        *reinterpret_cast<uint32_t*>(pdst) = pk[0];
    }
    if (dh == 0) sAlpha[mrow] = alpha_tile;
    fence_async_shared();
    tc_fence_before();
    if (__syncthreads_or(alpha_tile != 1.f) && t > 0) {
      // rare: some row raised its reference max in this tile. The accumulator holds tiles < t:
      // wait for the last issued MMA (tile t-1), then warps 0-3 scale their lane quarters.
      if (warp < 4) {
        if (!mbar_wait(&mma_bar[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1u, kWaitLimit))
          atomicExch(err, 2);
        tc_fence_after();
        const float a = sAlpha[32 * warp + lane];
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
          uint32_t r[32];
          tmem_ld32(tmem_quarter + cb * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * a);
          tmem_st32(tmem_quarter + cb * 32, r);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncthreads();
    }
    alpha_tile = 1.f;

    // ---- one thread: O += P @ V on the tensor core, then refill the freed stage ----------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t pa = smem_u32(sP);
      const uint32_t vbase = smem_u32(sm + C::OFF_V + s * C::VTILE);
#pragma unroll
      for (int kk = 0; kk < C::BN / 16; ++kk) {
        const uint64_t adesc = make_smem_desc(pa + kk * 32, 16, 1024, kSwizzle128B);
        const uint64_t bdesc = make_smem_desc(vbase + kk * 2048, C::BN * 128, 1024, kSwizzle128B);
        umma_f16(tmem, adesc, bdesc, idesc, (t > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&mma_bar[b]);
      const int tn = t + C::STAGES - 1;
      if (tn < ntiles) {
        // stage tn % STAGES was last read by tile t-1 (K by all threads before this tile's
        // barrier, V by MMA t-1)
        if (t >= 1 && !mbar_wait(&mma_bar[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1u, kWaitLimit))
          atomicExch(err, 4);
        fence_async_shared();
        issue_tile(tn);
      }
    }
    __syncwarp();
  }

  // ---- epilogue --------------------------------------------------------------------------
  {
    const int tl = ntiles - 1;
    if (!mbar_wait(&mma_bar[tl & 1], (uint32_t)(tl >> 1) & 1u, kWaitLimit)) atomicExch(err, 5);
  }
  float l_row = l;
#pragma unroll
  for (int o = 1; o < TPR; o <<= 1) l_row += __shfl_xor_sync(0xffffffffu, l_row, o);
  // a half of a split block: its partial state goes to the workspace for the combine kernel
  const int64_t item = ((int64_t)bh * nqb + qb) * 2 + (half < 0 ? 0 : half);
  if (dh == 0) {
    sL[mrow] = l_row;
    if (half >= 0)
      reinterpret_cast<float2*>(part_ml)[item * C::BM + mrow] = make_float2(m_ref, l_row);
    else if (row_ok)
      lse[(int64_t)bh * N + row] = (m_ref + __log2f(l_row)) * kLn2;
  }
  __syncthreads();
  tc_fence_after();
  if (half >= 0) {
    // unnormalised fp32 rows of O (relative to the row's reference max), straight from TMEM
    float* prow = part_o + (item * C::BM + 32 * quarter + lane) * D + wsub * DH;
#pragma unroll
    for (int cb = 0; cb < DH / 32; ++cb) {
      uint32_t r[32];
      tmem_ld32(tmem_quarter + wsub * DH + cb * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < 8; ++g)
        reinterpret_cast<float4*>(prow + cb * 32)[g] =
            make_float4(__uint_as_float(r[4 * g]), __uint_as_float(r[4 * g + 1]),
                        __uint_as_float(r[4 * g + 2]), __uint_as_float(r[4 * g + 3]));
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
    return;
  }
  // warp w stores columns [DH (w / 4), DH (w / 4 + 1)) of the 32 rows of its lane quarter
  const int orow_m = 32 * quarter + lane;
  const bool orow_ok = m0 + orow_m < N;
  const float lsum = sL[orow_m];
  const float inv_l = (orow_ok && lsum > 0.f) ? 1.f / lsum : 0.f;
  T* orow = out + ((int64_t)bh * N + (orow_ok ? m0 + orow_m : 0)) * D + wsub * DH;
#pragma unroll
  for (int cb = 0; cb < DH / 32; ++cb) {
    uint32_t r[32];
    tmem_ld32(tmem_quarter + wsub * DH + cb * 32, r);
    tmem_wait_ld();
    if (orow_ok) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float r0, r1;
          pk[e] = U::pack(__uint_as_float(r[8 * g + 2 * e]) * inv_l,
                          __uint_as_float(r[8 * g + 2 * e + 1]) * inv_l, r0, r1);
        }
        reinterpret_cast<uint4*>(orow + cb * 32)[g] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

// Merges the two halves of every split query block (blocks 1 .. nqb - 1 of each head): one warp
// per query row, lanes over head dims. With the halves' reference maxima m0, m1 (log2 units),
// row sums l0, l1 and unnormalised rows O0, O1: M = max(m0, m1), a_i = 2^(m_i - M),
// out = (a0 O0 + a1 O1) / (a0 l0 + a1 l1), lse = (M + log2(a0 l0 + a1 l1)) ln 2.
template <int D, typename T>
__global__ void attn_fwd_combine_kernel(const float* __restrict__ part_o,
                                        const float* __restrict__ part_ml, T* __restrict__ out,
                                        float* __restrict__ lse, int N, int nbh) {
  constexpr int BM = FwdCfg<D>::BM;
  const int nqb = (N + BM - 1) / BM;
  const int64_t per_bh = (int64_t)(nqb - 1) * BM;
  const int64_t rid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (rid >= per_bh * nbh) return;
  const int bh = (int)(rid / per_bh);
  const int qb = 1 + (int)((rid % per_bh) / BM), mrow = (int)(rid % BM);
  const int row = qb * BM + mrow;
  if (row >= N) return;
  const int64_t i0 = (((int64_t)bh * nqb + qb) * 2) * BM + mrow, i1 = i0 + BM;
  const float2 ml0 = reinterpret_cast<const float2*>(part_ml)[i0];
  const float2 ml1 = reinterpret_cast<const float2*>(part_ml)[i1];
  const float M = fmaxf(ml0.x, ml1.x);
  const float a0 = ex2_approx(ml0.x - M), a1 = ex2_approx(ml1.x - M);
  const float lsum = ml0.y * a0 + ml1.y * a1;
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  const float2* o0 = reinterpret_cast<const float2*>(part_o + i0 * D);
  const float2* o1 = reinterpret_cast<const float2*>(part_o + i1 * D);
  uint32_t* dst = reinterpret_cast<uint32_t*>(out + ((int64_t)bh * N + row) * D);
#pragma unroll
  for (int c = lane; c < D / 2; c += 32) {
    const float2 x0 = o0[c], x1 = o1[c];
    float r0, r1;
    dst[c] = Unpack<T>::pack((x0.x * a0 + x1.x * a1) * inv, (x0.y * a0 + x1.y * a1) * inv, r0, r1);
  }
  if (lane == 0) lse[(int64_t)bh * N + row] = (M + __log2f(lsum)) * kLn2;
}

// Whether a causal forward splits its query blocks 1 .. nqb - 1 into key-range halves: when the
// grid would hold fewer than four CTAs per SM, the longest causal blocks (their key range grows
// with the block index) would otherwise leave the last wave's SMs idle.
bool fwd_split(int64_t BH, int64_t N, int flags) {
  if (!(flags & FLB_ATTN_CAUSAL) || N < 256) return false;
  const int64_t nqb = (N + 127) / 128;
  return BH * nqb < 4 * (int64_t)num_sms();
}
// Workspace of a split forward: 256 B error word, then the partial O rows [BH, nqb, 2, 128, D]
// and the (max, sum) pairs [BH, nqb, 2, 128] (fp32).
size_t fwd_part_o_bytes(int64_t BH, int64_t N, int64_t D) {
  return (size_t)BH * ((N + 127) / 128) * 2 * 128 * D * sizeof(float);
}
size_t fwd_part_ml_bytes(int64_t BH, int64_t N) {
  return (size_t)BH * ((N + 127) / 128) * 2 * 128 * 2 * sizeof(float);
}

template <int D, typename T>
int launch_fwd_tc(const void* q, const void* k, const void* v, const float* w, const int32_t* wi,
                  void* out, float* lse, float* scores, int64_t BH, int N, int causal, int* err,
                  float* part_o, float* part_ml, cudaStream_t s) {
  using C = FwdCfg<D>;
  const CUtensorMapDataType dt =
      Unpack<T>::is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tmK, tmV;
  const uint64_t dims[3] = {(uint64_t)D, (uint64_t)N, (uint64_t)BH};
  const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)N * D * 2};
  const uint32_t boxK[3] = {(uint32_t)D, (uint32_t)C::BN, 1};
  const uint32_t boxV[3] = {64, (uint32_t)C::BN, 1};
  int st = make_tmap(&tmK, k, dt, 3, dims, strides, boxK, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st != FLB_OK) return st;
  st = make_tmap(&tmV, v, dt, 3, dims, strides, boxV, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != FLB_OK) return st;
  st = ensure_dyn_smem((const void*)attn_fwd_tc_kernel<D, T>, C::SMEM, "attn_fwd_tc smem attribute");
  if (st != FLB_OK) return st;
  const int64_t nqb = (N + C::BM - 1) / C::BM;
  const unsigned grid = (unsigned)((part_o ? 2 * nqb - 1 : nqb) * BH);
  // vector score stores (8 / TPR floats) need an aligned base (rows are padded to 16 bytes)
  const int kpt = 8 / C::TPR;
  const int scores_vec = (reinterpret_cast<uintptr_t>(scores) & (uintptr_t)(4 * kpt - 1)) == 0;
  attn_fwd_tc_kernel<D, T><<<grid, C::THREADS, C::SMEM, s>>>(
      tmK, tmV, (const T*)q, (T*)out, lse, scores, w, wi, N, causal, (int)BH, scores_vec, part_o,
      part_ml, err);
  count_launches(1);
  if (part_o) {
    const int64_t rows = BH * (nqb - 1) * C::BM;
    attn_fwd_combine_kernel<D, T><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(part_o, part_ml,
                                                                             (T*)out, lse, N, (int)BH);
    count_launches(1);
  }
  return check_cuda(cudaGetLastError(), "attn_fwd_tc launch");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int attn_fwd_fast_supported(int64_t BH, int64_t N, int64_t D, int dtype, int flags) {
  if (flags & (FLB_ATTN_EXACT_TANH | FLB_ATTN_FORCE_GENERIC)) return 0;
  if (!(dtype == FLB_BF16 || dtype == FLB_F16)) return 0;
  if (!(D == 64 || D == 128)) return 0;
  if (N < 1 || BH < 1 || BH > 65535) return 0;
  return 1;
}

size_t attn_fwd_fast_workspace(int64_t BH, int64_t N, int64_t D, int, int flags) {
  if (!fwd_split(BH, N, flags)) return 256;
  return 256 + fwd_part_o_bytes(BH, N, D) + fwd_part_ml_bytes(BH, N);
}

int attn_fwd_fast(const void* q, const void* k, const void* v, const float* w, const int32_t* wi,
                  void* out, float* lse, float* scores, int64_t BH, int N, int D, int dtype,
                  int flags, void* ws, size_t ws_bytes, cudaStream_t s) {
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(FLB_ERR_ALIGN, "attn_fwd: q/k/v/out must be 16-byte aligned for the tcgen05 path");
  int* err = reinterpret_cast<int*>(ws);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e != cudaSuccess) return check_cuda(e, "attn_fwd error-word reset");
  const int causal = (flags & FLB_ATTN_CAUSAL) ? 1 : 0;
  float* po = nullptr;
  float* pml = nullptr;
  if (fwd_split(BH, N, flags)) {
    if (ws_bytes < attn_fwd_fast_workspace(BH, N, D, dtype, flags))
      return fail(FLB_ERR_WORKSPACE, "attn_fwd: workspace smaller than flb_attn_fwd_workspace_bytes()");
    po = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + 256);
    pml = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(po) + fwd_part_o_bytes(BH, N, D));
  }
  if (dtype == FLB_BF16) {
    return D == 64 ? launch_fwd_tc<64, __nv_bfloat16>(q, k, v, w, wi, out, lse, scores, BH, N, causal, err, po, pml, s)
                   : launch_fwd_tc<128, __nv_bfloat16>(q, k, v, w, wi, out, lse, scores, BH, N, causal, err, po, pml, s);
  }
  return D == 64 ? launch_fwd_tc<64, __half>(q, k, v, w, wi, out, lse, scores, BH, N, causal, err, po, pml, s)
                 : launch_fwd_tc<128, __half>(q, k, v, w, wi, out, lse, scores, BH, N, causal, err, po, pml, s);
}

// =============================================================================================
// Backward (bf16/fp16, D = 64), consuming the scores saved by the forward.
//
// One CTA per (128-key block, batch*head), 32 warps (1024 threads, at most 64 registers each, one
// CTA per SM), looping over 128-query tiles (causal: only tiles at or below the key block). Per
// query tile:
//   1. dP = dO . V^T on the tensor core (A = dO tile, K-major; B = the CTA's V block, K-major;
//      M = N = 128, K = 64) into TMEM columns [0, 128).
//   2. Phase A (TMEM lane = query row; the 8 warps of a lane quarter take 16 keys each): P =
//      exp(s - lse) from the saved scores, dS = P * (dP - Delta); P goes to shared memory as the
//      MN-major A operand of step 3, dS (fp16, scaled per tile by a power of two) to a shared tile.
//   3. dV += P^T . dO on the tensor core: P is read MN-major (M = keys), and the same swizzled dO
//      tile serves as an MN-major B operand (N = d); accumulator in TMEM columns [128, 192).
//   4. Phase B, the tanh grid (the MUFU-bound part): warp w owns keys 16 (w % 8) .. +15 for query
//      rows 32 (w / 8) .. +31, lane l head dims 2l, 2l+1, in packed f16x2. For every row:
//      t = tanh(q + k), s = 1 - t^2; dK accumulates dS s per key (f16 over the tile's rows, then
//      fp32 in TMEM columns [256, 512)), dw accumulates dS t, dQ's per-row sum over the warp's
//      keys goes into a shared fp32 tile with shared-memory reductions, flushed to a global fp32
//      accumulator once per tile (one vector red.add per four elements per CTA and tile).
// 32 warps (8 per scheduler) are what keep both the MUFU and the FMA pipe busy through each
// row's dependency chains; keeping the dK partials in TMEM instead of registers is what lets
// that many warps fit the register file, and 16 keys per warp halve the per-row loads and
// reductions per key against 8.
// A prep kernel computes Delta = rowsum(dO * O) and clears the dQ accumulator; a finish kernel
// scales dQ by w' and casts it. dQ[i,d] = w'[d] sum_j dS (1 - t^2), dK[j,d] = w'[d] sum_i dS
// (1 - t^2), dw[d] = sum dS t / sqrt(D), w' = w / sqrt(D) (kernels/additive_attention.py:91-130).
// =============================================================================================

namespace {

// dst[0..3] += {a, b, c, d} as one vector reduction (dst 16-byte aligned)
__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

struct BwdCfg {
  static constexpr int D = 64, BM = 128, BN = 128;
  static constexpr int NT = 1024;                          // 32 warps, <= 64 registers each
  static constexpr int TILE = BM * D * 2;                  // 16 KB (a q or dO tile, bf16/fp16)
  static constexpr int SC_BOX = BM * 32 * 4;               // 16 KB: scores of 128 rows x 32 keys
  static constexpr int OFF_V = 0;                          // V block [128 keys x 64] swizzled
  static constexpr int OFF_DO = OFF_V + BN * D * 2;        // 2 stages, swizzled
  static constexpr int OFF_Q = OFF_DO + 2 * TILE;          // 2 stages, plain rows
  // P tile (2 x 16 KB MN-major atoms). Between the dV MMA of a tile and the P writes of the
  // next one it holds score boxes 0-1 (keys 0-63) of the next tile; OFF_SC holds boxes 2-3.
  static constexpr int OFF_P = OFF_Q + 2 * TILE;
  static constexpr int OFF_SC = OFF_P + BM * BN * 2;
  static constexpr int DS_LD = BN + 8;                     // row pitch (halves) of the dS tile
  // dS and dQ tiles carry one extra row: a zero dS row and a dummy dQ row that an odd last
  // row of phase B's two-row step points at, so that step needs no branch
  static constexpr int OFF_DS = OFF_SC + 2 * SC_BOX;             // fp16 [129 x DS_LD]
  static constexpr int OFF_DQ = OFF_DS + (BM + 1) * DS_LD * 2;   // fp32 [129 x 64]
  static constexpr int SMEM = OFF_DQ + (BM + 1) * D * 4 + 1024;
  // TMEM columns: dP [0,128), dV [128,192), and from 256 the fp32 dK partials of phase B: warp
  // (16-key group kg, 32-row quarter rq) owns 32 columns at 256 + 32 (kg / 4 + 2 rq) of lane
  // quarter kg % 4 (column 2 j + c: key j of the group, head dim 2 lane + c)
  static constexpr int TMEM_COLS = 512;
  static constexpr int DK_COL0 = 256;
  static_assert(OFF_P % 1024 == 0 && OFF_SC % 1024 == 0, "swizzled boxes need 1 KB alignment");
};

template <typename T>
__global__ void bwd_prep_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                float* __restrict__ delta, float* __restrict__ dq_acc,
                                int64_t rows) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (r >= rows) return;
  using U = Unpack<T>;
  const uint32_t* op = reinterpret_cast<const uint32_t*>(o + r * 64);
  const uint32_t* dp = reinterpret_cast<const uint32_t*>(dout + r * 64);
  float a0, a1, b0, b1;
  U::run(op[lane], a0, a1);
  U::run(dp[lane], b0, b1);
  float s = warp_sum(a0 * b0 + a1 * b1);
  if (lane == 0) delta[r] = s;
  reinterpret_cast<float2*>(dq_acc + r * 64)[lane] = make_float2(0.f, 0.f);
}

template <typename T>
__global__ void bwd_finish_kernel(const float* __restrict__ dq_acc, const float* __restrict__ w,
                                  const int32_t* __restrict__ w_index, T* __restrict__ dq,
                                  int N, int64_t rows) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one float2 each
  if (idx >= rows * 32) return;
  const int64_t r = idx / 32;
  const int d = (int)(idx % 32) * 2;
  const int64_t bh = r / N;
  const float* wr = w + (int64_t)w_index[bh] * 64;
  const float2 a = reinterpret_cast<const float2*>(dq_acc)[idx];
  float r0, r1;
  reinterpret_cast<uint32_t*>(dq)[idx] =
      Unpack<T>::pack(a.x * wr[d] * 0.125f, a.y * wr[d + 1] * 0.125f, r0, r1);
}

template <typename T>
__global__ void __launch_bounds__(BwdCfg::NT, 1)
attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmSC,
                   const T* __restrict__ k, const float* __restrict__ w,
                   const int32_t* __restrict__ w_index, const float* __restrict__ lse,
                   const float* __restrict__ delta, float* __restrict__ dq_acc,
                   T* __restrict__ dk, T* __restrict__ dv, float* __restrict__ dw, int N,
                   int causal, int nbh, int* __restrict__ err) {
  using namespace sm100;
  using C = BwdCfg;
  using U = Unpack<T>;
  constexpr int D = C::D;
  constexpr int NT = C::NT;  // 32 warps
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full_bar[2];
  __shared__ __align__(8) uint64_t dp_bar, dv_bar, sc_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ unsigned s_amax;  // max |dS| of the current tile (float bits; non-negative floats order as ints)
  __shared__ float s_dw[D];    // the CTA's dw partial, one global atomic per head dim at the end

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 1-D grid over (key block, head); key blocks ascend = most query tiles first, so every head's
  // heaviest CTAs start in the first wave
  const int kb = blockIdx.x / nbh;
  const int bh = blockIdx.x % nbh;
  const int kb0 = kb * C::BN;
  const int nqt = (N + C::BM - 1) / C::BM;
  const int t_first = causal ? kb : 0;
  const int ntiles = nqt - t_first;
  const float inv_sqrt_d = 0.125f;
  const float* wrow = w + (int64_t)w_index[bh] * D;
  const T* kbh = k + (int64_t)bh * N * D;

  if (tid == 0) {
    mbar_init(&full_bar[0], 1);
    mbar_init(&full_bar[1], 1);
    mbar_init(&dp_bar, 1);
    mbar_init(&dv_bar, 1);
    mbar_init(&sc_bar, 1);
    fence_mbar_init();
    s_amax = 0u;
  }
  if (tid < D) s_dw[tid] = 0.f;
  if (warp == 0) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  float* sDQ = reinterpret_cast<float*>(sm + C::OFF_DQ);
  for (int i = tid; i < (C::BM + 1) * D; i += NT) sDQ[i] = 0.f;
  if (tid < C::DS_LD)
    reinterpret_cast<__half*>(sm + C::OFF_DS)[C::BM * C::DS_LD + tid] = __float2half(0.f);
  // phase B ownership: warp w holds keys 16 (w % 8) .. +15 of the block for query rows
  // 32 (w / 8) .. +31 of every tile; lane l holds head dims 2l, 2l+1
  const int kg = warp & 7, rq = warp >> 3;
  __half2 kr[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int key = kb0 + kg * 16 + j;
    kr[j] = key < N ? to_h2<T>(reinterpret_cast<const uint32_t*>(kbh + (int64_t)key * D)[lane])
                    : __floats2half2_rn(0.f, 0.f);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // this warp's dK accumulator columns (its lane quarter = its key group's, lane = head dim pair)
  const uint32_t dk_taddr =
      tmem + ((uint32_t)(32 * (warp & 3)) << 16) + C::DK_COL0 + 32 * ((kg >> 2) + 2 * rq);
  {
    uint32_t z[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) z[i] = 0u;
    tmem_st16(dk_taddr, z);
    tmem_st16(dk_taddr + 16, z);
    tmem_wait_st();
  }

  auto issue_tile = [&](int t) {  // t: 0-based tile counter
    const int st = t & 1;
    const int q0 = (t_first + t) * C::BM;
    mbar_arrive_expect_tx(&full_bar[st], 2 * C::TILE);
    tma_load_3d(sm + C::OFF_DO + st * C::TILE, &tmDO, &full_bar[st], 0, q0, bh);
    tma_load_3d(sm + C::OFF_Q + st * C::TILE, &tmQ, &full_bar[st], 0, q0, bh);
  };
  const uint32_t idesc_dp = make_idesc_f16(128, 128, U::is_bf16, 0, 0);
  const uint32_t idesc_dv = make_idesc_f16(128, 64, U::is_bf16, 1, 1);
  auto issue_dp = [&](int t) {  // requires Q/dO tile t resident
    const uint32_t a = smem_u32(sm + C::OFF_DO + (t & 1) * C::TILE);
    const uint32_t b = smem_u32(sm + C::OFF_V);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      umma_f16(tmem, make_smem_desc(a + kk * 32, 16, 1024, kSwizzle128B),
               make_smem_desc(b + kk * 32, 16, 1024, kSwizzle128B), idesc_dp, kk > 0 ? 1u : 0u);
    umma_commit(&dp_bar);
  };
  // saved scores of query tile t: four swizzled boxes of 32 keys x 128 rows (OOB rows and keys
  // read as zero and are masked in phase A); boxes 0-1 land in the P buffer, 2-3 in OFF_SC
  auto issue_scores = [&](int t) {
    const int q0 = (t_first + t) * C::BM;
    mbar_arrive_expect_tx(&sc_bar, 4 * C::SC_BOX);
#pragma unroll
    for (int g = 0; g < 4; ++g)
      tma_load_3d(sm + (g < 2 ? C::OFF_P : C::OFF_SC - 2 * C::SC_BOX) + g * C::SC_BOX, &tmSC,
                  &sc_bar, kb0 + 32 * g, q0, bh);
  };

  if (tid == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmSC);
    // V block and the first query tile share stage 0's barrier: one arrive.expect_tx per phase
    mbar_arrive_expect_tx(&full_bar[0], C::BN * D * 2 + 2 * C::TILE);
    tma_load_3d(sm + C::OFF_V, &tmV, &full_bar[0], 0, kb0, bh);
    tma_load_3d(sm + C::OFF_DO, &tmDO, &full_bar[0], 0, t_first * C::BM, bh);
    tma_load_3d(sm + C::OFF_Q, &tmQ, &full_bar[0], 0, t_first * C::BM, bh);
    issue_scores(0);
    if (ntiles > 1) issue_tile(1);
    if (!mbar_wait(&full_bar[0], 0, kWaitLimit)) atomicExch(err, 11);
    tc_fence_after();
    issue_dp(0);
  }
  __syncwarp();

  // phase A ownership: TMEM lane quarter (warp & 3) = query rows, 16-key group (warp >> 2) of 8;
  // the group's scores are half of one 32-key box (four of its 16-byte chunks)
  const int arow = 32 * (warp & 3) + lane;
  const int agrp = warp >> 2;
  const int abox = agrp >> 1;
  const uint8_t* sc_row = sm + (abox < 2 ? C::OFF_P : C::OFF_SC - 2 * C::SC_BOX) +
                          abox * C::SC_BOX + arow * 128;
  const int sc_chunk0 = 4 * (agrp & 1);

  // per-row phase A inputs (lse, Delta), loaded one tile ahead
  float lse2 = 0.f, dlt = 0.f;
  auto load_row_stats = [&](int t) {
    const int i = (t_first + t) * C::BM + arow;
    lse2 = i < N ? lse[(int64_t)bh * N + i] * kLog2e : 0.f;
    dlt = i < N ? delta[(int64_t)bh * N + i] : 0.f;
  };
  load_row_stats(0);

  float dwa0 = 0.f, dwa1 = 0.f;
  __half* sDS = reinterpret_cast<__half*>(sm + C::OFF_DS);  // dS tile, scaled, fp16

  for (int t = 0; t < ntiles; ++t) {
    const int q0 = (t_first + t) * C::BM;
    const int st = t & 1;
    // every thread observes the TMA barrier of this tile (phase B reads the Q tile)
    if (!mbar_wait(&full_bar[st], (uint32_t)(t >> 1) & 1u, kWaitLimit)) atomicExch(err, 10);
    if (!mbar_wait(&dp_bar, (uint32_t)t & 1u, kWaitLimit)) atomicExch(err, 12);
    if (t >= 1 && !mbar_wait(&dv_bar, (uint32_t)(t - 1) & 1u, kWaitLimit)) atomicExch(err, 13);
    if (!mbar_wait(&sc_bar, (uint32_t)t & 1u, kWaitLimit)) atomicExch(err, 17);
    tc_fence_after();
    // ---- phase A: P and dS for (row arow, keys 16*agrp .. +15) ------------------------------
    // P = exp(s - lse) is formed from the saved scores before the barrier and kept packed in
    // the dtype of V (8 registers for 16 keys), the operand precision of the dV MMA
    uint32_t pk[8];
    {
      const int i = q0 + arow;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float4 v4 =
            *reinterpret_cast<const float4*>(sc_row + (((sc_chunk0 + c) ^ (arow & 7)) << 4));
        const float s4[4] = {v4.x, v4.y, v4.z, v4.w};
        float p4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = kb0 + 16 * agrp + 4 * c + e;
          const bool ok = i < N && key < N && (!causal || key <= i);
          p4[e] = ok ? ex2_approx(s4[e] * kLog2e - lse2) : 0.f;
        }
        float r0, r1;
        pk[2 * c] = U::pack(p4[0], p4[1], r0, r1);
        pk[2 * c + 1] = U::pack(p4[2], p4[3], r0, r1);
      }
    }
    if constexpr (U::is_bf16) {
      // phase B adds q + k in f16x2: convert this tile's Q rows in place, once
      uint32_t* q32 = reinterpret_cast<uint32_t*>(sm + C::OFF_Q + st * C::TILE);
#pragma unroll
      for (int i = tid; i < C::BM * D / 2; i += NT) {
        const __half2 h = to_h2<T>(q32[i]);
        q32[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      fence_async_shared();  // the stage is refilled by TMA later
    }
    // boxes 0-1 share the P buffer: every thread's scores are read before P is written
    __syncthreads();
    float ds[16];
    {
      // P as the MN-major A operand of the dV MMA: keys 0-63 in the first 16 KB atom, 64-127 in
      // the second; 8 keys per 16-byte chunk of a query row
      uint8_t* sP = sm + C::OFF_P + (agrp >> 2) * (C::BM * 128);
      float amax = 0.f;
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        *reinterpret_cast<uint4*>(sP + sw128_offset(arow, 2 * (agrp & 3) + g)) =
            make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
        uint32_t r[8];
        tmem_ld8(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 16 * agrp + 8 * g, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float p0, p1;
          U::run(pk[4 * g + e], p0, p1);
          ds[8 * g + 2 * e] = p0 * (__uint_as_float(r[2 * e]) - dlt);
          ds[8 * g + 2 * e + 1] = p1 * (__uint_as_float(r[2 * e + 1]) - dlt);
          amax = fmaxf(amax, fmaxf(fabsf(ds[8 * g + 2 * e]), fabsf(ds[8 * g + 2 * e + 1])));
        }
      }
      amax = warp_max(amax);
      if (lane == 0) atomicMax(&s_amax, __float_as_uint(amax));
    }
    __syncthreads();
    // a power-of-two scale per tile keeps the half-precision sums of phase B inside fp16's
    // normal range: max |dS| * scale lies in [256, 512)
    const float amax_tile = __uint_as_float(s_amax);
    const int ex = amax_tile > 0.f ? ilogbf(amax_tile) : 0;
    const float ds_scale = ldexpf(1.f, 8 - ex), ds_unscale = ldexpf(1.f, ex - 8);
    {
      __half* dsrow = sDS + arow * C::DS_LD + 16 * agrp;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __half2 h = __floats2half2_rn(ds[8 * c + 2 * e] * ds_scale,
                                        ds[8 * c + 2 * e + 1] * ds_scale);
          v[e] = *reinterpret_cast<uint32_t*>(&h);
        }
        reinterpret_cast<uint4*>(dsrow)[c] = make_uint4(v[0], v[1], v[2], v[3]);
      }
    }
    fence_async_shared();
    tc_fence_before();
    __syncthreads();

    // ---- one thread: dV += P^T dO, dP for the next tile, the next tile's scores -------------
    if (tid == 0) {
      tc_fence_after();
      const uint32_t pa = smem_u32(sm + C::OFF_P);
      const uint32_t ob = smem_u32(sm + C::OFF_DO + st * C::TILE);
#pragma unroll
      for (int kk = 0; kk < C::BM / 16; ++kk)
        umma_f16(tmem + 128, make_smem_desc(pa + kk * 2048, C::BM * 128, 1024, kSwizzle128B),
                 make_smem_desc(ob + kk * 2048, C::BM * 128, 1024, kSwizzle128B), idesc_dv,
                 (t > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&dv_bar);
      if (t + 1 < ntiles) {
        if (!mbar_wait(&full_bar[(t + 1) & 1], (uint32_t)((t + 1) >> 1) & 1u, kWaitLimit))
          atomicExch(err, 14);
        tc_fence_after();
        issue_dp(t + 1);
        // the P buffer is free once the dV MMA of this tile has read it
        if (!mbar_wait(&dv_bar, (uint32_t)t & 1u, kWaitLimit)) atomicExch(err, 18);
        fence_async_shared();
        issue_scores(t + 1);
      }
    }
    __syncwarp();
    // next tile's lse and Delta: global loads in flight during the tanh grid below
    if (t + 1 < ntiles) load_row_stats(t + 1);

    // ---- phase B: the tanh grid, packed f16x2 (lane = head dims 2l, 2l+1) ----------------------
    // 32 warps (8 per scheduler) keep the MUFU and FMA pipes fed across each row's dependency
    // chains. The Q tile holds f16x2 pairs here (converted in place in phase A).
    {
      const __half2* sQh = reinterpret_cast<const __half2*>(sm + C::OFF_Q + st * C::TILE);
      const int key_lo = kb0 + kg * 16;
      const int rmax = min(C::BM, N - q0);
      // causal: rows r < key_lo - q0 mask every key of this warp
      const int r_begin = causal ? max(32 * rq, key_lo - q0) : 32 * rq;
      const int r_end = min(32 * rq + 32, rmax);
      const __half2 hz = __floats2half2_rn(0.f, 0.f);
      const __half2 one2 = __floats2half2_rn(1.f, 1.f);
      constexpr int DS_ROW = C::DS_LD / 8;  // uint4 per dS row
      if (r_begin < r_end) {
        // dK of the warp's keys over its rows of this tile, in f16 (|sum| <= 32 * 512), moved to
        // the fp32 accumulators in TMEM at the end of the tile
        __half2 dk2[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) dk2[j] = hz;
        // rows are addressed through running pointers (row strides: Q 32 half2, dS DS_LD halves,
        // dQ partials D floats)
        const __half2* qp = sQh + r_begin * (D / 2) + lane;
        const uint4* dsp = reinterpret_cast<const uint4*>(sDS + kg * 16) + r_begin * DS_ROW;
        float* dqp = sDQ + r_begin * D + lane;
#pragma unroll 1
        for (int r = r_begin; r < r_end; ++r) {
          // one query row against the warp's 16 keys, five f16x2 FMA-pipe ops per key: x = q + k,
          // s = 1 - t^2 and three fused accumulations: dS s into dK (per key) and dQ (over the
          // keys), dS t into dw
          const __half2 q2 = *qp;
          const uint4 dv0 = dsp[0], dv1 = dsp[1];
          const uint32_t dsu[8] = {dv0.x, dv0.y, dv0.z, dv0.w, dv1.x, dv1.y, dv1.z, dv1.w};
          __half2 dqa = hz, dqb = hz, dwa = hz, dwb = hz;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const __half2 tt = tanh_h2(__hadd2(q2, kr[j]));
            const __half2 dpair = *reinterpret_cast<const __half2*>(&dsu[j >> 1]);
            const __half2 d2 = (j & 1) ? __high2half2(dpair) : __low2half2(dpair);
            const __half2 s2 = __hfma2(__hneg2(tt), tt, one2);
            dk2[j] = __hfma2(d2, s2, dk2[j]);
            if (j & 1) {
              dqb = __hfma2(d2, s2, dqb);
              dwb = __hfma2(d2, tt, dwb);
            } else {
              dqa = __hfma2(d2, s2, dqa);
              dwa = __hfma2(d2, tt, dwa);
            }
          }
          // dQ partials (scaled; the flush unscales): layout [row][c * 32 + lane] for head dim
          // 2 * lane + c (conflict-free); |sum| <= 16 * 512
          const float2 dqf = __half22float2(__hadd2(dqa, dqb));
          red_shared_f32(dqp, dqf.x);
          red_shared_f32(dqp + 32, dqf.y);
          const float2 dwf = __half22float2(__hadd2(dwa, dwb));
          dwa0 = fmaf(dwf.x, ds_unscale, dwa0);
          dwa1 = fmaf(dwf.y, ds_unscale, dwa1);
          qp += D / 2;
          dsp += DS_ROW;
          dqp += D;
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t a[16];
          tmem_ld16(dk_taddr + 16 * hh, a);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2 f = __half22float2(dk2[8 * hh + j]);
            a[2 * j] = __float_as_uint(fmaf(f.x, ds_unscale, __uint_as_float(a[2 * j])));
            a[2 * j + 1] = __float_as_uint(fmaf(f.y, ds_unscale, __uint_as_float(a[2 * j + 1])));
          }
          tmem_st16(dk_taddr + 16 * hh, a);
        }
        tmem_wait_st();
      }
    }
    __syncthreads();
    // ---- flush dQ partials of this tile; refill the stage this tile used ----------------------
    {
      const int rows = min(C::BM, N - q0);
      float* dst = dq_acc + ((int64_t)bh * N + q0) * D;
      // four consecutive head dims per thread, one vector reduction each: dims d, d+2 sit at
      // [d/2, d/2+1] of the even half of the row's partials, d+1, d+3 in the odd half
      for (int e = 4 * tid; e < rows * D; e += 4 * NT) {
        const int rr = e / D, d = e % D;
        float2* ev = reinterpret_cast<float2*>(&sDQ[rr * D + (d >> 1)]);
        float2* od = reinterpret_cast<float2*>(&sDQ[rr * D + 32 + (d >> 1)]);
        const float2 a = *ev, b = *od;
        red_add_v4(dst + e, a.x * ds_unscale, b.x * ds_unscale, a.y * ds_unscale, b.y * ds_unscale);
        *ev = make_float2(0.f, 0.f);
        *od = make_float2(0.f, 0.f);
      }
      if (tid == 0) s_amax = 0u;
    }
    if (tid == 0 && t + 2 < ntiles) {
      // stage st: Q read by phase B (done: barrier above), dO read by dV MMA t
      if (!mbar_wait(&dv_bar, (uint32_t)t & 1u, kWaitLimit)) atomicExch(err, 15);
      fence_async_shared();
      issue_tile(t + 2);
    }
    tc_fence_before();  // the dK accumulators in TMEM are read by other warps in the epilogue
    __syncthreads();
  }

  // ---- epilogue: dV from TMEM (warps 0-7: lane quarter x column half), dK and dw from registers
  if (!mbar_wait(&dv_bar, (uint32_t)(ntiles - 1) & 1u, kWaitLimit)) atomicExch(err, 16);
  tc_fence_after();
  if (warp < 8) {
    const int key = kb0 + 32 * (warp & 3) + lane;
    const int cb = warp >> 2;  // columns 32*cb .. +31 of dV
    uint32_t r[32];
    tmem_ld32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 128 + 32 * cb, r);
    tmem_wait_ld();
    if (key < N) {
      T* dst = dv + ((int64_t)bh * N + key) * D + 32 * cb;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float r0, r1;
          pk[e] = U::pack(__uint_as_float(r[8 * g + 2 * e]), __uint_as_float(r[8 * g + 2 * e + 1]),
                          r0, r1);
        }
        reinterpret_cast<uint4*>(dst)[g] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  }
  // dK: the first row quarter's warp adds the other three quarters' accumulators (same lane
  // quarter, 64, 128 and 192 columns further) and stores the key group's rows
  red_shared_f32(&s_dw[2 * lane], dwa0);
  red_shared_f32(&s_dw[2 * lane + 1], dwa1);
  if (rq == 0) {
    const float w0 = wrow[2 * lane] * inv_sqrt_d, w1 = wrow[2 * lane + 1] * inv_sqrt_d;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint32_t a[16];
      tmem_ld16(dk_taddr + 16 * hh, a);
      tmem_wait_ld();
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = __uint_as_float(a[i]);
#pragma unroll
      for (int p = 1; p < 4; ++p) {
        tmem_ld16(dk_taddr + 64 * p + 16 * hh, a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] += __uint_as_float(a[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int key = kb0 + kg * 16 + 8 * hh + j;
        if (key < N) {
          float r0, r1;
          reinterpret_cast<uint32_t*>(dk + ((int64_t)bh * N + key) * D)[lane] =
              U::pack(acc[2 * j] * w0, acc[2 * j + 1] * w1, r0, r1);
        }
      }
    }
  }
  __syncthreads();
  if (tid < D) atomicAdd(dw + (int64_t)w_index[bh] * D + tid, s_dw[tid] * inv_sqrt_d);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C::TMEM_COLS);
}

template <typename T>
int launch_bwd_tc(const void* q, const void* k, const void* v, const float* w, const int32_t* wi,
                  const void* o, const float* lse, const float* scores, const void* dout, void* dq,
                  void* dk, void* dv, float* dw, int64_t BH, int N, int causal, void* ws,
                  cudaStream_t s) {
  using C = BwdCfg;
  const CUtensorMapDataType dt =
      Unpack<T>::is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t dims[3] = {64, (uint64_t)N, (uint64_t)BH};
  const uint64_t strides[2] = {128, (uint64_t)N * 128};
  const uint32_t box[3] = {64, 128, 1};
  CUtensorMap tmQ, tmDO, tmV, tmSC;
  int st = make_tmap(&tmQ, q, dt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st == FLB_OK) st = make_tmap(&tmDO, dout, dt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st == FLB_OK) st = make_tmap(&tmV, v, dt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st != FLB_OK) return st;
  {
    // saved scores [BH, N, ld] fp32, boxes of 32 keys (128 bytes, swizzled) x 128 rows
    const uint64_t ld = (uint64_t)attn_scores_ld(N);
    const uint64_t sdims[3] = {(uint64_t)N, (uint64_t)N, (uint64_t)BH};
    const uint64_t sstrides[2] = {ld * 4, (uint64_t)N * ld * 4};
    const uint32_t sbox[3] = {32, 128, 1};
    st = make_tmap(&tmSC, scores, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, sdims, sstrides, sbox,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != FLB_OK) return st;
  }
  uint8_t* wsb = reinterpret_cast<uint8_t*>(ws);
  int* err = reinterpret_cast<int*>(wsb);
  float* delta = reinterpret_cast<float*>(wsb + 256);
  float* dq_acc = delta + ((BH * N + 63) / 64) * 64;
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e != cudaSuccess) return check_cuda(e, "attn_bwd error-word reset");
  const int64_t rows = BH * N;
  bwd_prep_kernel<T><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>((const T*)o, (const T*)dout, delta,
                                                                dq_acc, rows);
  st = ensure_dyn_smem((const void*)attn_bwd_tc_kernel<T>, C::SMEM, "attn_bwd_tc smem attribute");
  if (st != FLB_OK) return st;
  const unsigned grid = (unsigned)(((N + C::BN - 1) / C::BN) * BH);
  attn_bwd_tc_kernel<T><<<grid, C::NT, C::SMEM, s>>>(tmQ, tmDO, tmV, tmSC, (const T*)k, w, wi, lse,
                                                   delta, dq_acc, (T*)dk, (T*)dv, dw, N, causal,
                                                   (int)BH, err);
  bwd_finish_kernel<T><<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(dq_acc, w, wi, (T*)dq, N,
                                                                           rows);
  count_launches(3);
  return check_cuda(cudaGetLastError(), "attn_bwd_tc launch");
}

}  // namespace

int attn_bwd_fast_supported(int64_t BH, int64_t N, int64_t D, int dtype, int flags) {
  if (flags & (FLB_ATTN_EXACT_TANH | FLB_ATTN_FORCE_GENERIC)) return 0;
  if (!(dtype == FLB_BF16 || dtype == FLB_F16)) return 0;
  if (D != 64) return 0;
  if (N < 1 || BH < 1 || BH > 65535) return 0;
  return 1;
}

size_t attn_bwd_fast_workspace(int64_t BH, int64_t N, int64_t D, int, int) {
  const size_t rows = (size_t)(BH * N);
  return 256 + ((rows + 63) / 64) * 64 * sizeof(float) + rows * (size_t)D * sizeof(float);
}

int attn_bwd_fast(const void* q, const void* k, const void* v, const float* w, const int32_t* wi,
                  const void* o, const float* lse, const float* scores, const void* dout, void* dq,
                  void* dk, void* dv, float* dw, int64_t BH, int N, int D, int dtype, int flags,
                  void* ws, size_t ws_bytes, cudaStream_t s) {
  if (D != 64 || scores == nullptr) return fail(FLB_ERR_UNSUPPORTED, "attn_bwd_fast: needs D=64 and saved scores");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(dout) || !aligned16(o) ||
      !aligned16(dq) || !aligned16(dk) || !aligned16(dv))
    return fail(FLB_ERR_ALIGN, "attn_bwd: tensors must be 16-byte aligned for the tcgen05 path");
  if (ws_bytes < attn_bwd_fast_workspace(BH, N, D, dtype, flags))
    return fail(FLB_ERR_WORKSPACE, "attn_bwd: workspace too small");
  const int causal = (flags & FLB_ATTN_CAUSAL) ? 1 : 0;
  if (dtype == FLB_BF16)
    return launch_bwd_tc<__nv_bfloat16>(q, k, v, w, wi, o, lse, scores, dout, dq, dk, dv, dw, BH, N,
                                        causal, ws, s);
  return launch_bwd_tc<__half>(q, k, v, w, wi, o, lse, scores, dout, dq, dk, dv, dw, BH, N, causal,
                               ws, s);
}

}  // namespace flb
