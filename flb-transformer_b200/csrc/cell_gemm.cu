// Small-M GEMMs of the FLB block cells on tcgen05: per tick, for each cell i of the tick,
//   Y_i[m][j] = sum_k X_i[m][k] W_i[j][k]      (m < M rows, j < N outputs, k < K)
// with M = batch or 3 x batch rows (16 .. 64), N = d_model or 3 d_model, K = d_model, and each
// cell's weights W_i an [N, K] slice of a per-layer stack (the tick's layers are two apart).
// These replace one cuBLAS strided-batched call per projection of a tick (the prior, gate, q|k|v
// and output projections of models/FLB_Model.py:32-96 evaluated for the tick's cells).
//
// Swap-AB: the tensor core computes Y_i^T[128 x M] = W_i[128 rows of N x K] . X_i^T, so the
// weight slice is the M=128 operand and the few rows of X are the N operand; one CTA per
// (128 outputs, cell), 128 threads, the accumulator in TMEM (one lane per output).
// K is streamed in 64-element atoms (128-byte rows, 128-byte swizzle) through a ring of stages
// by TMA: weights first — they do not depend on the previous kernel, so with programmatic
// dependent launch they stream while that kernel drains — then, after griddepcontrol.wait, the
// rows of X. One thread issues loads and MMAs; a stage is refilled once the MMAs that read it
// have completed. The epilogue stores Y (bf16) from TMEM with each warp writing 32 consecutive
// outputs of a row.
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

namespace flb {

namespace {

constexpr uint32_t kCellGemmWaitLimit = 1u << 22;
constexpr int kCellGemmMaxStages = 12;
constexpr int kCellGemmSmemBudget = 200 * 1024;

struct CellGemmParams {
  __nv_bfloat16* y;   // cell i, row m, output j at y + i * stride_y + m * ldy + j
  int64_t ldy, stride_y;
  int M, N, K, stages;
  int w_row0, w_cell_rows;  // cell i's weight rows start at row w_row0 + i * w_cell_rows
  int* err;
};

__device__ __forceinline__ void pdl_wait_only() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__global__ void __launch_bounds__(128, 1)
cell_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                 CellGemmParams p) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[kCellGemmMaxStages], empty[kCellGemmMaxStages], done;
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * 128, cell = blockIdx.y;
  const int KA = p.K / 64, S = p.stages;
  const uint32_t a_bytes = 128u * 128u, b_bytes = (uint32_t)p.M * 128u;
  const uint32_t st_bytes = a_bytes + b_bytes;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (tid == 0) {
    const int wrow = p.w_row0 + cell * p.w_cell_rows + n0;
    auto stage_a = [&](int s) { return sm + s * st_bytes; };
    auto stage_b = [&](int s) { return sm + s * st_bytes + a_bytes; };
    const int first = std::min(S, KA);
    for (int a = 0; a < first; ++a) {
      mbar_arrive_expect_tx(&full[a], st_bytes);
      tma_load_2d(stage_a(a), &tmW, &full[a], a * 64, wrow);
    }
    pdl_wait_only();  // X is the previous kernel's output
    for (int a = 0; a < first; ++a) tma_load_3d(stage_b(a), &tmX, &full[a], a * 64, 0, cell);
    const uint32_t idesc = make_idesc_f16(128, p.M, 1, 0, 0);
    for (int a = 0; a < KA; ++a) {
      const int s = a % S;
      if (!mbar_wait(&full[s], (uint32_t)(a / S) & 1u, kCellGemmWaitLimit) && p.err)
        atomicExch(p.err, 1);
      tc_fence_after();
      const uint32_t sa = smem_u32(stage_a(s)), sb = smem_u32(stage_b(s));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f16(tmem, make_smem_desc(sa + kk * 32, 16, 1024, kSwizzle128B),
                 make_smem_desc(sb + kk * 32, 16, 1024, kSwizzle128B), idesc,
                 (a > 0 || kk > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
      // refill the stage of the previous atom: its MMAs have had one atom's time to finish
      const int prev = a - 1;
      if (prev >= 0 && prev + S < KA) {
        const int ps = prev % S;
        if (!mbar_wait(&empty[ps], (uint32_t)(prev / S) & 1u, kCellGemmWaitLimit) && p.err)
          atomicExch(p.err, 2);
        mbar_arrive_expect_tx(&full[ps], st_bytes);
        tma_load_2d(stage_a(ps), &tmW, &full[ps], (prev + S) * 64, wrow);
        tma_load_3d(stage_b(ps), &tmX, &full[ps], (prev + S) * 64, 0, cell);
      }
    }
    umma_commit(&done);
  }
  __syncwarp();
  if (!mbar_wait(&done, 0u, kCellGemmWaitLimit) && p.err) atomicExch(p.err, 3);
  tc_fence_after();
  pdl_trigger();
  __nv_bfloat16* y = p.y + (int64_t)cell * p.stride_y + n0 + warp * 32 + lane;
  for (int cb = 0; cb < p.M; cb += 32) {
    uint32_t acc[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + cb, acc);
    tmem_wait_ld();
    const int nb = min(32, p.M - cb);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= nb) break;
      y[(int64_t)(cb + j) * p.ldy] = __float2bfloat16_rn(__uint_as_float(acc[j]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

}  // namespace

// Shapes the kernel takes: M rows a multiple of 16 up to 64, N a multiple of 128, K a multiple
// of 64, 16-byte aligned operand bases and row / cell pitches.
bool cell_gemm_supported(int M, int N, int K, const void* W, const void* X, int64_t ldx,
                         int64_t stride_x, const void* Y, int64_t ldy, int64_t stride_y) {
  const uintptr_t al = (uintptr_t)W | (uintptr_t)X;
  return M >= 16 && M <= 64 && M % 16 == 0 && N % 128 == 0 && K % 64 == 0 && K >= 64 &&
         (al & 15u) == 0 && (ldx * 2) % 16 == 0 && (stride_x * 2) % 16 == 0 &&
         ((uintptr_t)Y & 1u) == 0 && ldy >= N && stride_y >= 0;
}

// Y_i = X_i W_i^T for the n cells of a tick (see the file comment). W: a stack [w_rows_total, K]
// (bf16, row-major); cell i uses rows w_row0 + i * w_cell_rows .. + N. X: cell i's rows at
// X + i * stride_x, pitch ldx (elements). Launched with programmatic dependent launch.
int cell_gemm(const void* W, int64_t w_rows_total, int w_row0, int w_cell_rows, const void* X,
              int64_t ldx, int64_t stride_x, int n_cells, int M, int N, int K, void* Y,
              int64_t ldy, int64_t stride_y, int* err, cudaStream_t s) {
  if (n_cells <= 0) return FLB_OK;
  if (!cell_gemm_supported(M, N, K, W, X, ldx, stride_x, Y, ldy, stride_y))
    return fail(FLB_ERR_UNSUPPORTED, "cell_gemm: unsupported shape or alignment");
  CUtensorMap mW, mX;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)w_rows_total};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, 128};
    int st = make_tmap(&mW, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != FLB_OK) return st;
  }
  {
    const uint64_t dims[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)n_cells};
    const uint64_t strides[2] = {(uint64_t)ldx * 2, (uint64_t)(stride_x > 0 ? stride_x : ldx * M) * 2};
    const uint32_t box[3] = {64, (uint32_t)M, 1};
    int st = make_tmap(&mX, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (st != FLB_OK) return st;
  }
  const int st_bytes = 128 * 128 + M * 128;
  const int stages = std::max(1, std::min({K / 64, kCellGemmMaxStages, kCellGemmSmemBudget / st_bytes}));
  const int smem = stages * st_bytes + 1024;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(cell_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kCellGemmSmemBudget + 1024);
    if (e != cudaSuccess) return check_cuda(e, "cell_gemm smem attribute");
    attr = true;
  }
  CellGemmParams p{};
  p.y = reinterpret_cast<__nv_bfloat16*>(Y);
  p.ldy = ldy;
  p.stride_y = stride_y;
  p.M = M;
  p.N = N;
  p.K = K;
  p.stages = stages;
  p.w_row0 = w_row0;
  p.w_cell_rows = w_cell_rows;
  p.err = err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(N / 128), (unsigned)n_cells);
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = la;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, cell_gemm_kernel, mW, mX, p);
  count_launches(1);
  return check_cuda(e, "cell_gemm launch");
}

}  // namespace flb
