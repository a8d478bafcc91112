// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver
// entry point, so the library does not link libcuda directly).
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "common.cuh"

namespace flb {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tiled tensor map over a row-major array. dims[0] is the contiguous (innermost) extent;
// strides_bytes[i] is the byte stride of dimension i+1. The box inner extent times the element
// size must be a multiple of 16 bytes and, with 128B swizzle, at most 128 bytes.
inline int make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int rank,
                     const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                     CUtensorMapSwizzle swz) {
  auto enc = tmap_encoder();
  if (!enc) return fail(FLB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(FLB_ERR_ALIGN, "TMA base address must be 16-byte aligned");
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0) return fail(FLB_ERR_ALIGN, "TMA stride must be a multiple of 16 bytes");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(m, dt, (cuuint32_t)rank, const_cast<void*>(base), (const cuuint64_t*)dims,
                   (const cuuint64_t*)strides_bytes, (const cuuint32_t*)box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FLB_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return FLB_OK;
}

}  // namespace flb
