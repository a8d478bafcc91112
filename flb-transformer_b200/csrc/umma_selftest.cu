// Known-answer check of the tensor-core operand layouts the fast kernels depend on:
// D[128 x N] = A[128 x 64] * B, bf16 in, f32 out, one CTA.
//   A is written by threads into a K-major 128B-swizzled tile (as the attention kernel writes P).
//   variant 0: B given as [N rows x 64 K] (K contiguous), TMA-loaded K-major (wavefront cell).
//   variant 1: B given as [64 K rows x N cols] (N contiguous), TMA-loaded MN-major (P @ V).
// N is 64 or 128 (variant 1 with N = 128 uses two 64-column TMA boxes, exercising LBO).
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace flb {

namespace {

constexpr int kM = 128;
constexpr int kK = 64;

template <int N, int VARIANT>
__global__ void __launch_bounds__(128)
umma_selftest_kernel(const __nv_bfloat16* __restrict__ A, const __grid_constant__ CUtensorMap tmB,
                     float* __restrict__ Dout, int* __restrict__ err) {
  using namespace sm100;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-align the dynamic smem base (swizzle atoms are address-based)
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;                    // 128 x 128 B = 16 KB
  uint8_t* sB = smem + kM * 128;         // N x 128 B (variant 0) or 64 x 128 B x (N/64) (variant 1)
  __shared__ __align__(8) uint64_t bar_tma, bar_mma;
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  if (tid == 0) {
    mbar_init(&bar_tma, 1);
    mbar_init(&bar_mma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 128);
    tmem_relinquish();
  }
  // A: row tid, 8 chunks of 16 bytes, swizzled
  {
    const uint4* src = reinterpret_cast<const uint4*>(A + (size_t)tid * kK);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 val = src[c];
      *reinterpret_cast<uint4*>(sA + sw128_offset(tid, c)) = val;
    }
  }
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (tid == 0) {
    constexpr uint32_t bytesB = N * kK * 2;
    mbar_arrive_expect_tx(&bar_tma, bytesB);
    if (VARIANT == 0) {
      tma_load_2d(sB, &tmB, &bar_tma, 0, 0);              // box {64 K, N rows}
    } else {
#pragma unroll
      for (int nb = 0; nb < N / 64; ++nb)
        tma_load_2d(sB + nb * (kK * 128), &tmB, &bar_tma, nb * 64, 0);  // box {64 N, 64 K}
    }
    if (!mbar_wait(&bar_tma, 0, 1u << 24)) atomicExch(err, 1);
    tc_fence_after();
    const uint32_t idesc = make_idesc_f16(kM, N, 1, 0, VARIANT == 1 ? 1 : 0);
    const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
#pragma unroll
    for (int ks = 0; ks < kK / 16; ++ks) {
      const uint64_t adesc = make_smem_desc(a_base + ks * 32, 16, 1024, kSwizzle128B);
      uint64_t bdesc;
      if (VARIANT == 0)
        bdesc = make_smem_desc(b_base + ks * 32, 16, 1024, kSwizzle128B);
      else  // MN-major: 16 K rows per step = 2048 bytes; next 64-column atom at kK*128 bytes
        bdesc = make_smem_desc(b_base + ks * 2048, kK * 128, 1024, kSwizzle128B);
      umma_f16(tmem, adesc, bdesc, idesc, ks > 0 ? 1u : 0u);
    }
    umma_commit(&bar_mma);
  }
  __syncwarp();
  if (!mbar_wait(&bar_mma, 0, 1u << 24)) atomicExch(err, 2);
  tc_fence_after();
  // read back: warp w owns rows 32w..32w+31
#pragma unroll
  for (int cb = 0; cb < N / 32; ++cb) {
    uint32_t r[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cb * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) Dout[(size_t)tid * N + cb * 32 + j] = __uint_as_float(r[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace

int umma_selftest(int variant, int n, const void* A, const void* B, float* D, int* err,
                  cudaStream_t s) {
  if (!(n == 64 || n == 128) || !(variant == 0 || variant == 1))
    return fail(FLB_ERR_SHAPE, "umma_selftest: variant 0/1, n 64/128");
  CUtensorMap tm;
  int st;
  if (variant == 0) {
    uint64_t dims[2] = {(uint64_t)kK, (uint64_t)n};
    uint64_t strides[1] = {(uint64_t)kK * 2};
    uint32_t box[2] = {64, (uint32_t)n};
    st = make_tmap(&tm, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    uint64_t dims[2] = {(uint64_t)n, (uint64_t)kK};
    uint64_t strides[1] = {(uint64_t)n * 2};
    uint32_t box[2] = {64, (uint32_t)kK};
    st = make_tmap(&tm, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (st != FLB_OK) return st;
  const size_t smem = 1024 + kM * 128 + (size_t)n * kK * 2;
  cudaError_t e;
#define FLB_LAUNCH(N_, V_)                                                                      \
  do {                                                                                         \
    e = cudaFuncSetAttribute(umma_selftest_kernel<N_, V_>,                                      \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);           \
    if (e == cudaSuccess)                                                                      \
      umma_selftest_kernel<N_, V_><<<1, 128, smem, s>>>((const __nv_bfloat16*)A, tm, D, err);   \
  } while (0)
  if (variant == 0 && n == 64) FLB_LAUNCH(64, 0);
  else if (variant == 0) FLB_LAUNCH(128, 0);
  else if (n == 64) FLB_LAUNCH(64, 1);
  else FLB_LAUNCH(128, 1);
#undef FLB_LAUNCH
  if (e != cudaSuccess) return check_cuda(e, "umma_selftest attribute");
  return check_cuda(cudaGetLastError(), "umma_selftest launch");
}

}  // namespace flb
