// Generic additive-attention kernels (CUDA cores, fp32 accumulation), one warp per row.
//
// Forward restates the math of kernels/additive_attention.py:10-86 (scores, /sqrt(D),
// softmax, P@V) without materialising the [N,N,D] tanh grid: lane l owns head dims
// d = l, l+32, ..., keys are processed 32 at a time, per-lane partial scores are combined by a
// transposing warp reduction so that lane jj ends with the score of key j0+jj, and an online
// softmax carries the row max. The +1e-6 of the Triton kernel's denominator (:78) is not
// applied: the eager ground truth (kernels/kernel_tests.py:8-29) and the backward (:107) have
// none, and with the max subtracted the denominator is >= 1, so the difference is < 1e-6
// relative.
//
// Backward restates compiled_backward_math (kernels/additive_attention.py:91-130) with the
// standard identity rowsum(P * dP) = rowsum(dO * O):
//   dS = P * (dP - Delta),  dQ[i,d] = w'[d] sum_j dS (1 - t^2),  dK[j,d] = w'[d] sum_i dS (1 - t^2),
//   dV = P^T dO,  dw[d] = sum_{i,j} dS t / sqrt(D),   with w' = w / sqrt(D), t = tanh(q+k).
// Two passes (query-owned for dQ/dw, key-owned for dK/dV) avoid atomics on dQ/dK.
#include "common.cuh"
#include <math.h>

namespace flb {

namespace {

constexpr int kWarpsPerBlock = 8;

template <typename T, int DPL, bool EXACT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
attn_fwd_generic_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                        const float* __restrict__ w, const int32_t* __restrict__ w_index,
                        T* __restrict__ out, float* __restrict__ lse, float* __restrict__ scores,
                        int64_t BH, int N, int D, float inv_scale, int causal) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= BH * (int64_t)N) return;
  const int64_t bh = row / N;
  const int i = (int)(row - bh * N);
  const int64_t base = bh * (int64_t)N * D;
  const float* wrow = w + (int64_t)w_index[bh] * D;

  float qv[DPL], wv[DPL], acc[DPL];
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    const int d = lane + 32 * c;
    const bool ok = d < D;
    qv[c] = ok ? ld(q + base + (int64_t)i * D + d) : 0.f;
    wv[c] = ok ? wrow[d] * inv_scale : 0.f;
    acc[c] = 0.f;
  }
  const int jmax = causal ? (i + 1) : N;
  float m = -INFINITY, l = 0.f;

  for (int j0 = 0; j0 < jmax; j0 += 32) {
    float part[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      float s = 0.f;
      if (j0 + jj < jmax) {
        const T* kr = k + base + (int64_t)(j0 + jj) * D;
#pragma unroll
        for (int c = 0; c < DPL; ++c) {
          const int d = lane + 32 * c;
          const float kd = (d < D) ? ld(kr + d) : 0.f;
          s = fmaf(wv[c], tanh_f<EXACT>(qv[c] + kd), s);
        }
      }
      part[jj] = s;
    }
    float s = transpose_reduce32(part);
    const bool valid = (j0 + lane) < jmax;
    if (scores != nullptr && valid) scores[row * attn_scores_ld(N) + j0 + lane] = s;
    s = valid ? s : -INFINITY;
    const float m_new = fmaxf(m, warp_max(s));
    const float alpha = exp_f<EXACT>(m - m_new);
    const float p = valid ? exp_f<EXACT>(s - m_new) : 0.f;
    l = l * alpha + warp_sum(p);
#pragma unroll
    for (int c = 0; c < DPL; ++c) acc[c] *= alpha;
    const int nk = min(32, jmax - j0);
    for (int jj = 0; jj < nk; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const T* vr = v + base + (int64_t)(j0 + jj) * D;
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        const int d = lane + 32 * c;
        if (d < D) acc[c] = fmaf(pj, ld(vr + d), acc[c]);
      }
    }
    m = m_new;
  }
  const float inv_l = 1.f / l;
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    const int d = lane + 32 * c;
    if (d < D) st(out + base + (int64_t)i * D + d, acc[c] * inv_l);
  }
  if (lane == 0) lse[row] = m + log_f<EXACT>(l);
}

// Query-owned backward pass: dQ, dw, and Delta_i = sum_d dO * O (written for the key pass).
template <typename T, int DPL, bool EXACT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
attn_bwd_dq_generic_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                           const float* __restrict__ w, const int32_t* __restrict__ w_index,
                           const T* __restrict__ o, const float* __restrict__ lse,
                           const T* __restrict__ dout, T* __restrict__ dq, float* __restrict__ dw,
                           float* __restrict__ delta, int64_t BH, int N, int D, float inv_scale,
                           int causal) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= BH * (int64_t)N) return;
  const int64_t bh = row / N;
  const int i = (int)(row - bh * N);
  const int64_t base = bh * (int64_t)N * D;
  const int64_t wrow_off = (int64_t)w_index[bh] * D;

  float qv[DPL], wv[DPL], dov[DPL], dqa[DPL], dwa[DPL];
  float dlt = 0.f;
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    const int d = lane + 32 * c;
    const bool ok = d < D;
    qv[c] = ok ? ld(q + base + (int64_t)i * D + d) : 0.f;
    wv[c] = ok ? w[wrow_off + d] * inv_scale : 0.f;
    dov[c] = ok ? ld(dout + base + (int64_t)i * D + d) : 0.f;
    const float ov = ok ? ld(o + base + (int64_t)i * D + d) : 0.f;
    dlt = fmaf(dov[c], ov, dlt);
    dqa[c] = 0.f;
    dwa[c] = 0.f;
  }
  dlt = warp_sum(dlt);
  if (lane == 0) delta[row] = dlt;
  const float lse_i = lse[row];
  const int jmax = causal ? (i + 1) : N;

  for (int j0 = 0; j0 < jmax; j0 += 32) {
    float ps[32], pdp[32];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      float s = 0.f, dp = 0.f;
      if (j0 + jj < jmax) {
        const T* kr = k + base + (int64_t)(j0 + jj) * D;
        const T* vr = v + base + (int64_t)(j0 + jj) * D;
#pragma unroll
        for (int c = 0; c < DPL; ++c) {
          const int d = lane + 32 * c;
          const bool ok = d < D;
          const float kd = ok ? ld(kr + d) : 0.f;
          const float vd = ok ? ld(vr + d) : 0.f;
          s = fmaf(wv[c], tanh_f<EXACT>(qv[c] + kd), s);
          dp = fmaf(dov[c], vd, dp);
        }
      }
      ps[jj] = s;
      pdp[jj] = dp;
    }
    const float s = transpose_reduce32(ps);
    const float dp = transpose_reduce32(pdp);
    const bool valid = (j0 + lane) < jmax;
    const float p = valid ? exp_f<EXACT>(s - lse_i) : 0.f;
    const float ds = p * (dp - dlt);
    const int nk = min(32, jmax - j0);
    for (int jj = 0; jj < nk; ++jj) {
      const float dsj = __shfl_sync(0xffffffffu, ds, jj);
      const T* kr = k + base + (int64_t)(j0 + jj) * D;
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        const int d = lane + 32 * c;
        if (d < D) {
          const float t = tanh_f<EXACT>(qv[c] + ld(kr + d));
          dqa[c] = fmaf(dsj, fmaf(-t, t, 1.f), dqa[c]);
          dwa[c] = fmaf(dsj, t, dwa[c]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    const int d = lane + 32 * c;
    if (d < D) {
      st(dq + base + (int64_t)i * D + d, dqa[c] * wv[c]);
      atomicAdd(dw + wrow_off + d, dwa[c] * inv_scale);
    }
  }
}

// Key-owned backward pass: dK and dV for key row j.
template <typename T, int DPL, bool EXACT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
attn_bwd_dkdv_generic_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                             const float* __restrict__ w, const int32_t* __restrict__ w_index,
                             const float* __restrict__ lse, const T* __restrict__ dout,
                             const float* __restrict__ delta, T* __restrict__ dk, T* __restrict__ dv,
                             int64_t BH, int N, int D, float inv_scale, int causal) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  if (row >= BH * (int64_t)N) return;
  const int64_t bh = row / N;
  const int j = (int)(row - bh * N);
  const int64_t base = bh * (int64_t)N * D;
  const int64_t wrow_off = (int64_t)w_index[bh] * D;

  float kv[DPL], vv[DPL], wv[DPL], dka[DPL], dva[DPL];
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    const int d = lane + 32 * c;
    const bool ok = d < D;
    kv[c] = ok ? ld(k + base + (int64_t)j * D + d) : 0.f;
    vv[c] = ok ? ld(v + base + (int64_t)j * D + d) : 0.f;
    wv[c] = ok ? w[wrow_off + d] * inv_scale : 0.f;
    dka[c] = 0.f;
    dva[c] = 0.f;
  }
  const int i_begin = causal ? j : 0;
  const int64_t rbase = bh * (int64_t)N;

  for (int i0 = i_begin; i0 < N; i0 += 32) {
    float ps[32], pdp[32];
#pragma unroll
    for (int ii = 0; ii < 32; ++ii) {
      float s = 0.f, dp = 0.f;
      if (i0 + ii < N) {
        const T* qr = q + base + (int64_t)(i0 + ii) * D;
        const T* dor = dout + base + (int64_t)(i0 + ii) * D;
#pragma unroll
        for (int c = 0; c < DPL; ++c) {
          const int d = lane + 32 * c;
          const bool ok = d < D;
          const float qd = ok ? ld(qr + d) : 0.f;
          const float dod = ok ? ld(dor + d) : 0.f;
          s = fmaf(wv[c], tanh_f<EXACT>(qd + kv[c]), s);
          dp = fmaf(dod, vv[c], dp);
        }
      }
      ps[ii] = s;
      pdp[ii] = dp;
    }
    const float s = transpose_reduce32(ps);
    const float dp = transpose_reduce32(pdp);
    const bool valid = (i0 + lane) < N;
    float p = 0.f, ds = 0.f;
    if (valid) {
      p = exp_f<EXACT>(s - lse[rbase + i0 + lane]);
      ds = p * (dp - delta[rbase + i0 + lane]);
    }
    const int nq = min(32, N - i0);
    for (int ii = 0; ii < nq; ++ii) {
      const float pi = __shfl_sync(0xffffffffu, p, ii);
      const float dsi = __shfl_sync(0xffffffffu, ds, ii);
      const T* qr = q + base + (int64_t)(i0 + ii) * D;
      const T* dor = dout + base + (int64_t)(i0 + ii) * D;
#pragma unroll
      for (int c = 0; c < DPL; ++c) {
        const int d = lane + 32 * c;
        if (d < D) {
          const float t = tanh_f<EXACT>(ld(qr + d) + kv[c]);
          dka[c] = fmaf(dsi, fmaf(-t, t, 1.f), dka[c]);
          dva[c] = fmaf(pi, ld(dor + d), dva[c]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < DPL; ++c) {
    const int d = lane + 32 * c;
    if (d < D) {
      st(dk + base + (int64_t)j * D + d, dka[c] * wv[c]);
      st(dv + base + (int64_t)j * D + d, dva[c]);
    }
  }
}

template <typename T, int DPL, bool EXACT>
cudaError_t launch_fwd(const void* q, const void* k, const void* v, const float* w,
                       const int32_t* wi, void* out, float* lse, float* scores, int64_t BH, int N,
                       int D, int causal, cudaStream_t s) {
  const int64_t rows = BH * N;
  const unsigned grid = (unsigned)((rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
  attn_fwd_generic_kernel<T, DPL, EXACT><<<grid, kWarpsPerBlock * 32, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, w, wi, (T*)out, lse, scores, BH, N, D,
      1.f / sqrtf((float)D), causal);
  return cudaGetLastError();
}

template <typename T, int DPL, bool EXACT>
cudaError_t launch_bwd(const void* q, const void* k, const void* v, const float* w,
                       const int32_t* wi, const void* o, const float* lse, const void* dout,
                       void* dq, void* dk, void* dv, float* dw, float* delta, int64_t BH, int N,
                       int D, int causal, cudaStream_t s) {
  const int64_t rows = BH * N;
  const unsigned grid = (unsigned)((rows + kWarpsPerBlock - 1) / kWarpsPerBlock);
  const float inv_scale = 1.f / sqrtf((float)D);
  attn_bwd_dq_generic_kernel<T, DPL, EXACT><<<grid, kWarpsPerBlock * 32, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, w, wi, (const T*)o, lse, (const T*)dout, (T*)dq, dw,
      delta, BH, N, D, inv_scale, causal);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_bwd_dkdv_generic_kernel<T, DPL, EXACT><<<grid, kWarpsPerBlock * 32, 0, s>>>(
      (const T*)q, (const T*)k, (const T*)v, w, wi, lse, (const T*)dout, delta, (T*)dk, (T*)dv, BH,
      N, D, inv_scale, causal);
  return cudaGetLastError();
}

template <typename T, bool EXACT>
cudaError_t dispatch_fwd_dpl(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, void* out, float* lse, float* sc, int64_t BH, int N,
                             int D, int causal, cudaStream_t s) {
  if (D <= 32) return launch_fwd<T, 1, EXACT>(q, k, v, w, wi, out, lse, sc, BH, N, D, causal, s);
  if (D <= 64) return launch_fwd<T, 2, EXACT>(q, k, v, w, wi, out, lse, sc, BH, N, D, causal, s);
  if (D <= 128) return launch_fwd<T, 4, EXACT>(q, k, v, w, wi, out, lse, sc, BH, N, D, causal, s);
  return launch_fwd<T, 8, EXACT>(q, k, v, w, wi, out, lse, sc, BH, N, D, causal, s);
}

template <typename T, bool EXACT>
cudaError_t dispatch_bwd_dpl(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, const void* o, const float* lse,
                             const void* dout, void* dq, void* dk, void* dv, float* dw,
                             float* delta, int64_t BH, int N, int D, int causal, cudaStream_t s) {
#define FLB_BWD(DPL_) \
  return launch_bwd<T, DPL_, EXACT>(q, k, v, w, wi, o, lse, dout, dq, dk, dv, dw, delta, BH, N, D, causal, s)
  if (D <= 32) FLB_BWD(1);
  if (D <= 64) FLB_BWD(2);
  if (D <= 128) FLB_BWD(4);
  FLB_BWD(8);
#undef FLB_BWD
}

}  // namespace

cudaError_t attn_fwd_generic(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, void* out, float* lse, float* sc, int64_t BH,
                             int N, int D, int dtype, bool exact, bool causal, cudaStream_t s) {
  const int c = causal ? 1 : 0;
  switch (dtype) {
    case FLB_F32:
      return exact ? dispatch_fwd_dpl<float, true>(q, k, v, w, wi, out, lse, sc, BH, N, D, c, s)
                   : dispatch_fwd_dpl<float, false>(q, k, v, w, wi, out, lse, sc, BH, N, D, c, s);
    case FLB_F16:
      return exact ? dispatch_fwd_dpl<__half, true>(q, k, v, w, wi, out, lse, sc, BH, N, D, c, s)
                   : dispatch_fwd_dpl<__half, false>(q, k, v, w, wi, out, lse, sc, BH, N, D, c, s);
    default:
      return exact ? dispatch_fwd_dpl<__nv_bfloat16, true>(q, k, v, w, wi, out, lse, sc, BH, N, D, c, s)
                   : dispatch_fwd_dpl<__nv_bfloat16, false>(q, k, v, w, wi, out, lse, sc, BH, N, D, c, s);
  }
}

cudaError_t attn_bwd_generic(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, const void* o, const float* lse, const void* dout,
                             void* dq, void* dk, void* dv, float* dw, float* delta, int64_t BH,
                             int N, int D, int dtype, bool exact, bool causal, cudaStream_t s) {
  const int c = causal ? 1 : 0;
#define FLB_BWD_T(T_)                                                                           \
  return exact ? dispatch_bwd_dpl<T_, true>(q, k, v, w, wi, o, lse, dout, dq, dk, dv, dw, delta, \
                                            BH, N, D, c, s)                                     \
               : dispatch_bwd_dpl<T_, false>(q, k, v, w, wi, o, lse, dout, dq, dk, dv, dw,      \
                                             delta, BH, N, D, c, s)
  switch (dtype) {
    case FLB_F32: FLB_BWD_T(float);
    case FLB_F16: FLB_BWD_T(__half);
    default: FLB_BWD_T(__nv_bfloat16);
  }
#undef FLB_BWD_T
}

}  // namespace flb
