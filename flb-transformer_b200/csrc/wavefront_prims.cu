// Wavefront engine data-movement kernels for the generic-layer path.
//
// gather      : restates fetch_mapped_context_kernel (wavefront/wavefront_kernel.py:27-82):
//               routing >= 0 reads the source cell of the dependency's port grid, -2 reads the
//               x row spatial_map[cell], -1 and padding cells write zeros.
// index_copy  : dst[dst_rows[k]] (=|+=) src[src_rows[k]] over a [rows, batch, dim] view; covers the
//               per-port index_put_ of execute_forward (csrc/wavefront_backend.cpp:40-43), the
//               per-cell parameter-gradient index_put_ (:97-106) or its per-layer sum
//               (wavefront/wavefront_engine.py:132-139 done on the fly), and the index_add_
//               routing of dependency gradients (csrc/wavefront_backend.cpp:109-130).
// Both are HBM/L2-bound element copies; the dim axis is the fastest index so warps touch
// contiguous runs.
#include "common.cuh"

namespace flb {

namespace {

template <typename T>
__global__ void gather_kernel(const T* __restrict__ x, int64_t xs0, int64_t xs1, int64_t xs2,
                              const T* __restrict__ grids, int64_t gs0, int64_t gs1, int64_t gs2,
                              int64_t gs3, const int32_t* __restrict__ routing,
                              const int32_t* __restrict__ port_map,
                              const int32_t* __restrict__ spatial_map,
                              const int32_t* __restrict__ active, int64_t n_active,
                              int64_t n_cells, T* __restrict__ out, int64_t os0, int64_t os1,
                              int64_t os2, int64_t os3, int64_t n_deps, int64_t batch,
                              int64_t dim) {
  const int64_t total = n_deps * n_active * batch * dim;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = idx;
    const int64_t d = r % dim; r /= dim;
    const int64_t b = r % batch; r /= batch;
    const int64_t s = r % n_active;
    const int64_t i = r / n_active;
    const int64_t cell = active[s];
    const int32_t t = (cell >= 0 && cell < n_cells) ? routing[cell * n_deps + i] : -1;
    T val;
    if (t >= 0) {
      val = grids[(int64_t)port_map[i] * gs0 + (int64_t)t * gs1 + b * gs2 + d * gs3];
    } else if (t == -2) {
      val = x[b * xs0 + (int64_t)spatial_map[cell] * xs1 + d * xs2];
    } else {
      val = T(0.f);
    }
    out[i * os0 + s * os1 + b * os2 + d * os3] = val;
  }
}

template <typename TS, typename TD>
__global__ void index_copy_kernel(const TS* __restrict__ src, int64_t ss0, int64_t ss1,
                                  int64_t ss2, const int64_t* __restrict__ src_rows,
                                  TD* __restrict__ dst, int64_t ds0, int64_t ds1, int64_t ds2,
                                  const int64_t* __restrict__ dst_rows, int64_t n_rows,
                                  int64_t batch, int64_t dim, int accumulate) {
  const int64_t total = n_rows * batch * dim;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = idx;
    const int64_t e = r % dim; r /= dim;
    const int64_t b = r % batch;
    const int64_t k = r / batch;
    const float val = ld(src + src_rows[k] * ss0 + b * ss1 + e * ss2);
    TD* p = dst + dst_rows[k] * ds0 + b * ds1 + e * ds2;
    if (accumulate) atomic_add_elem(p, val); else st(p, val);
  }
}

inline unsigned grid_for(int64_t total, int threads) {
  const int64_t want = (total + threads - 1) / threads;
  const int64_t cap = (int64_t)num_sms() * 16;
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace

int wf_gather(const void* x, const int64_t xs[3], const void* grids, const int64_t gs[4],
              const int32_t* routing, const int32_t* port_map, const int32_t* spatial_map,
              const int32_t* active, int64_t n_active, int64_t n_cells, void* out,
              const int64_t os[4], int64_t n_deps, int64_t batch, int64_t dim, int dtype,
              cudaStream_t s) {
  const int64_t total = n_deps * n_active * batch * dim;
  if (total == 0) return FLB_OK;
  const unsigned g = grid_for(total, 256);
#define FLB_G(T_)                                                                          \
  gather_kernel<T_><<<g, 256, 0, s>>>((const T_*)x, xs[0], xs[1], xs[2], (const T_*)grids,  \
                                      gs[0], gs[1], gs[2], gs[3], routing, port_map,        \
                                      spatial_map, active, n_active, n_cells, (T_*)out,     \
                                      os[0], os[1], os[2], os[3], n_deps, batch, dim)
  switch (dtype) {
    case FLB_F32: FLB_G(float); break;
    case FLB_F16: FLB_G(__half); break;
    case FLB_BF16: FLB_G(__nv_bfloat16); break;
    default: return fail(FLB_ERR_DTYPE, "wf_gather: unsupported dtype");
  }
#undef FLB_G
  count_launches(1);
  return check_cuda(cudaGetLastError(), "wf_gather launch");
}

int wf_index_copy(const void* src, int src_dtype, const int64_t ss[3], const int64_t* src_rows,
                  void* dst, int dst_dtype, const int64_t ds[3], const int64_t* dst_rows,
                  int64_t n_rows, int64_t batch, int64_t dim, int accumulate, cudaStream_t s) {
  const int64_t total = n_rows * batch * dim;
  if (total == 0) return FLB_OK;
  const unsigned g = grid_for(total, 256);
#define FLB_IC(TS_, TD_)                                                                        \
  index_copy_kernel<TS_, TD_><<<g, 256, 0, s>>>((const TS_*)src, ss[0], ss[1], ss[2], src_rows,  \
                                                (TD_*)dst, ds[0], ds[1], ds[2], dst_rows, n_rows, \
                                                batch, dim, accumulate)
#define FLB_ICD(TS_)                                                          \
  switch (dst_dtype) {                                                        \
    case FLB_F32: FLB_IC(TS_, float); break;                                  \
    case FLB_F16: FLB_IC(TS_, __half); break;                                 \
    case FLB_BF16: FLB_IC(TS_, __nv_bfloat16); break;                         \
    default: return fail(FLB_ERR_DTYPE, "wf_index_copy: unsupported dst dtype"); \
  }
  switch (src_dtype) {
    case FLB_F32: FLB_ICD(float); break;
    case FLB_F16: FLB_ICD(__half); break;
    case FLB_BF16: FLB_ICD(__nv_bfloat16); break;
    default: return fail(FLB_ERR_DTYPE, "wf_index_copy: unsupported src dtype");
  }
#undef FLB_ICD
#undef FLB_IC
  count_launches(1);
  return check_cuda(cudaGetLastError(), "wf_index_copy launch");
}

}  // namespace flb
