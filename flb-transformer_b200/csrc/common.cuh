// Shared helpers for the FLB B200 kernels: status plumbing, dtype access, warp reductions.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>
#include "../../include/flb_b200.h"

namespace flb {

// ---- host-side status --------------------------------------------------------------------
void set_error(const std::string& msg);
void count_launches(int n);
int fail(int status, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Raises a kernel's dynamic shared-memory limit to `bytes` on the CURRENT device. The attribute
// belongs to the device's context, so it is set once per (device, kernel) and remembered under a
// lock (host threads may launch on different devices at once).
int ensure_dyn_smem(const void* kernel, int bytes, const char* what);

inline int dtype_size(int dtype) {
  switch (dtype) {
    case FLB_F32: return 4;
    case FLB_F16: return 2;
    case FLB_BF16: return 2;
    default: return 0;
  }
}

// Row pitch (floats) of the saved attention scores [BH, N, ld]: rows padded to 16 bytes, the
// stride alignment TMA needs.
__host__ __device__ inline int64_t attn_scores_ld(int64_t N) { return (N + 3) & ~(int64_t)3; }

// SM count of the current device (a cheap attribute query, so no cache that could go stale when a
// process drives several devices)
inline int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// ---- device-side dtype access ------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float v) { *p = __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float ld(const T* p) { return Elem<T>::load(p); }
template <typename T> __device__ __forceinline__ void st(T* p, float v) { Elem<T>::store(p, v); }

__device__ __forceinline__ void atomic_add_elem(float* p, float v) { atomicAdd(p, v); }
__device__ __forceinline__ void atomic_add_elem(__half* p, float v) { atomicAdd(p, __float2half_rn(v)); }
__device__ __forceinline__ void atomic_add_elem(__nv_bfloat16* p, float v) { atomicAdd(p, __float2bfloat16_rn(v)); }

// ---- math ---------------------------------------------------------------------------------
// tanh.approx.f32: MUFU hardware tanh (PTX ISA, sm_75+), max relative error about 2^-11.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <bool EXACT> __device__ __forceinline__ float tanh_f(float x) {
  if constexpr (EXACT) return tanhf(x); else return tanh_approx(x);
}
template <bool EXACT> __device__ __forceinline__ float exp_f(float x) {
  if constexpr (EXACT) return expf(x); else return __expf(x);
}
template <bool EXACT> __device__ __forceinline__ float log_f(float x) {
  if constexpr (EXACT) return logf(x); else return __logf(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Transposing reduction: on entry lane l holds a[0..31] (one partial per key); on exit lane l
// returns sum over lanes of a[l]. 31 shuffles per lane instead of 32 x 5.
__device__ __forceinline__ float transpose_reduce32(float (&a)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int half = 16; half >= 1; half >>= 1) {
    const bool upper = (lane & half) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      // keep the half of the entries selected by this lane's bit, send the other half
      float send = upper ? a[i] : a[i + half];
      float keep = upper ? a[i + half] : a[i];
      float recv = __shfl_xor_sync(0xffffffffu, send, half);
      a[i] = keep + recv;
    }
  }
  return a[0];
}

}  // namespace flb
