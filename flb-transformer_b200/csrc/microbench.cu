// Throughput probes for the roofline denominators of the attention score stage:
// MUFU tanh (f32, f16x2, bf16x2), MUFU ex2, FFMA and HFMA2 issue, measured on this device at
// the clocks it runs at. Each thread runs 8 independent dependency chains so the pipe, not the
// latency, is the limit; every SM gets 8 warps per scheduler.
#include "common.cuh"

namespace flb {

namespace {

constexpr int kChains = 8;
constexpr int kIters = 4096;

template <int KIND>
__global__ void __launch_bounds__(1024) probe_kernel(uint32_t* sink, uint32_t seed) {
  uint32_t r[kChains];
#pragma unroll
  for (int c = 0; c < kChains; ++c) {
    // small distinct values so tanh/ex2 stay in the normal range
    const float f = 0.01f * (float)((threadIdx.x + c + seed) & 63) - 0.3f;
    if (KIND == 1 || KIND == 5) {
      __half2 h = __floats2half2_rn(f, -f);
      r[c] = *reinterpret_cast<uint32_t*>(&h);
    } else if (KIND == 2) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f, -f);
      r[c] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      r[c] = __float_as_uint(f);
    }
  }
  const uint32_t hmul = 0x3BFF3BFFu, hadd = 0x14001400u;  // ~0.9995, ~0.001 in each f16 half
  uint32_t acc1[kChains] = {}, acc2[kChains] = {}, acc3[kChains] = {};
  float f1[kChains] = {}, f2[kChains] = {}, f3[kChains] = {};
  for (int it = 0; it < kIters; ++it) {
#pragma unroll
    for (int c = 0; c < kChains; ++c) {
      if constexpr (KIND == 0) {
        float f = __uint_as_float(r[c]);
        asm volatile("tanh.approx.f32 %0, %0;" : "+f"(f));
        r[c] = __float_as_uint(f);
      } else if constexpr (KIND == 1) {
        asm volatile("tanh.approx.f16x2 %0, %0;" : "+r"(r[c]));
      } else if constexpr (KIND == 2) {
        asm volatile("tanh.approx.bf16x2 %0, %0;" : "+r"(r[c]));
      } else if constexpr (KIND == 3) {
        float f = __uint_as_float(r[c]);
        asm volatile("ex2.approx.ftz.f32 %0, %0;" : "+f"(f));
        r[c] = __float_as_uint(f);
      } else if constexpr (KIND == 4) {
        float f = __uint_as_float(r[c]);
        asm volatile("fma.rn.f32 %0, %0, %1, %2;" : "+f"(f) : "f"(0.9995f), "f"(0.001f));
        r[c] = __float_as_uint(f);
      } else if constexpr (KIND == 5) {
        asm volatile("fma.rn.f16x2 %0, %0, %1, %2;" : "+r"(r[c]) : "r"(hmul), "r"(hadd));
      } else if constexpr (KIND == 6) {
        // the attention backward's tanh-grid step on a packed pair: t = tanh(q + k),
        // u = ds t, g = ds - u t, three accumulations (g twice, u once)
        uint32_t x, t, u, g;
        asm volatile("add.rn.f16x2 %0, %1, %2;" : "=r"(x) : "r"(r[c]), "r"(hadd));
        asm volatile("tanh.approx.f16x2 %0, %1;" : "=r"(t) : "r"(x));
        asm volatile("mul.rn.f16x2 %0, %1, %2;" : "=r"(u) : "r"(hmul), "r"(t));
        asm volatile("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(g) : "r"(u ^ 0x80008000u), "r"(t), "r"(hmul));
        asm volatile("add.rn.f16x2 %0, %0, %1;" : "+r"(acc1[c]) : "r"(g));
        asm volatile("add.rn.f16x2 %0, %0, %1;" : "+r"(acc2[c]) : "r"(g));
        asm volatile("add.rn.f16x2 %0, %0, %1;" : "+r"(acc3[c]) : "r"(u));
        r[c] ^= (t & 0x00010001u);
      } else if constexpr (KIND == 7) {
        // the same step in fp32 on one element
        float q = __uint_as_float(r[c]), t, u, g;
        asm volatile("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(q + 0.001f));
        u = 0.9995f * t;
        g = fmaf(-u, t, 0.9995f);
        f1[c] += g;
        f2[c] += g;
        f3[c] += u;
        r[c] = __float_as_uint(q) ^ (__float_as_uint(t) & 1u);
      } else {
        // the forward's score step: s += w * tanh(q + k) in fp32
        float q = __uint_as_float(r[c]);
        float t;
        asm volatile("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(q + 0.001f));
        f1[c] = fmaf(0.9995f, t, f1[c]);
        r[c] = __float_as_uint(q) ^ (__float_as_uint(t) & 1u);
      }
    }
  }
  uint32_t acc = 0;
#pragma unroll
  for (int c = 0; c < kChains; ++c)
    acc ^= r[c] ^ acc1[c] ^ acc2[c] ^ acc3[c] ^ __float_as_uint(f1[c] + f2[c] + f3[c]);
  sink[blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

template <int KIND>
int run_probe(void* scratch, double* ops_per_s) {
  const int sms = num_sms();
  const int threads = 1024;
  const int blocks = sms;  // one 1024-thread block per SM = 8 warps per scheduler
  cudaEvent_t a, b;
  if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess)
    return fail(FLB_ERR_CUDA, "microbench: event create failed");
  probe_kernel<KIND><<<blocks, threads>>>((uint32_t*)scratch, 1u);  // warm-up
  cudaEventRecord(a);
  const int reps = 5;
  for (int i = 0; i < reps; ++i) probe_kernel<KIND><<<blocks, threads>>>((uint32_t*)scratch, 2u + i);
  cudaEventRecord(b);
  cudaError_t e = cudaEventSynchronize(b);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (e != cudaSuccess) return check_cuda(e, "microbench");
  const double elems_per_instr = (KIND == 1 || KIND == 2 || KIND == 5 || KIND == 6) ? 2.0 : 1.0;
  const double ops = (double)reps * blocks * threads * kIters * kChains * elems_per_instr;
  *ops_per_s = ops / (ms * 1e-3);
  return FLB_OK;
}

}  // namespace

int microbench(int kind, void* scratch, double* ops_per_s) {
  switch (kind) {
    case 0: return run_probe<0>(scratch, ops_per_s);
    case 1: return run_probe<1>(scratch, ops_per_s);
    case 2: return run_probe<2>(scratch, ops_per_s);
    case 3: return run_probe<3>(scratch, ops_per_s);
    case 4: return run_probe<4>(scratch, ops_per_s);
    case 5: return run_probe<5>(scratch, ops_per_s);
    case 6: return run_probe<6>(scratch, ops_per_s);
    case 7: return run_probe<7>(scratch, ops_per_s);
    case 8: return run_probe<8>(scratch, ops_per_s);
    default: return fail(FLB_ERR_UNSUPPORTED, "microbench: unknown kind");
  }
}

}  // namespace flb
