// extern "C" boundary of libflb_b200.so: argument validation, dispatch to the kernels, status
// codes and the thread-local error message.
#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include "common.cuh"

namespace flb {

static thread_local std::string g_last_error;
static std::atomic<uint64_t> g_launches{0};

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

void set_error(const std::string& msg) { g_last_error = msg; }
int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}
int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FLB_OK;
  g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return FLB_ERR_CUDA;
}

int ensure_dyn_smem(const void* kernel, int bytes, const char* what) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;  // (device, kernel) -> bytes set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, what);
  std::lock_guard<std::mutex> lock(mu);
  auto it = done.find({dev, kernel});
  if (it != done.end() && it->second >= bytes) return FLB_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return check_cuda(e, what);
  done[{dev, kernel}] = bytes;
  return FLB_OK;
}

// kernels (defined in the other translation units)
cudaError_t attn_fwd_generic(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, void* out, float* lse, float* scores, int64_t BH,
                             int N, int D, int dtype, bool exact, bool causal, cudaStream_t s);
cudaError_t attn_bwd_generic(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, const void* o, const float* lse, const void* dout,
                             void* dq, void* dk, void* dv, float* dw, float* delta, int64_t BH,
                             int N, int D, int dtype, bool exact, bool causal, cudaStream_t s);
int attn_fwd_fast_supported(int64_t BH, int64_t N, int64_t D, int dtype, int flags);
size_t attn_fwd_fast_workspace(int64_t BH, int64_t N, int64_t D, int dtype, int flags);
int attn_fwd_fast(const void* q, const void* k, const void* v, const float* w, const int32_t* wi,
                  void* out, float* lse, float* scores, int64_t BH, int N, int D, int dtype,
                  int flags, void* ws, size_t ws_bytes, cudaStream_t s);
int attn_bwd_fast_supported(int64_t BH, int64_t N, int64_t D, int dtype, int flags);
size_t attn_bwd_fast_workspace(int64_t BH, int64_t N, int64_t D, int dtype, int flags);
int attn_bwd_fast(const void* q, const void* k, const void* v, const float* w, const int32_t* wi,
                  const void* o, const float* lse, const float* scores, const void* dout, void* dq,
                  void* dk, void* dv,
                  float* dw, int64_t BH, int N, int D, int dtype, int flags, void* ws,
                  size_t ws_bytes, cudaStream_t s);
int wf_gather(const void* x, const int64_t xs[3], const void* grids, const int64_t gs[4],
              const int32_t* routing, const int32_t* port_map, const int32_t* spatial_map,
              const int32_t* active, int64_t n_active, int64_t n_cells, void* out,
              const int64_t os[4], int64_t n_deps, int64_t batch, int64_t dim, int dtype,
              cudaStream_t s);
int wf_index_copy(const void* src, int src_dtype, const int64_t ss[3], const int64_t* src_rows,
                  void* dst, int dst_dtype, const int64_t ds[3], const int64_t* dst_rows,
                  int64_t n_rows, int64_t batch, int64_t dim, int accumulate, cudaStream_t s);
size_t block_grid_workspace_bytes(int64_t L, int64_t S, int64_t B, int64_t D);
int block_grid_fwd(const flb_block_weights* W, const void* x, void* grids, int64_t L, int64_t S,
                   int64_t B, int64_t D, int64_t H, float eps, void* ws, size_t ws_bytes,
                   cudaStream_t s);
int block_grid_fwd_ex(const flb_block_weights* W, const void* x, void* grids, int64_t L,
                      int64_t S, int64_t B, int64_t D, int64_t H, float eps, void* ws,
                      size_t ws_bytes, cudaStream_t s, int path, int drop_cta, int drop_bar,
                      uint32_t spin_limit, void* saved);
size_t block_grid_saved_bytes(int64_t L, int64_t S, int64_t B, int64_t D);
int block_grid_status(const void* ws, cudaStream_t s);
size_t block_grid_bwd_workspace_bytes(int64_t L, int64_t S, int64_t B, int64_t D);
int block_grid_bwd(const flb_block_weights* W, const void* x, const void* grids,
                   const void* const* dgrids, float* dx, const flb_block_grads* G, int64_t L,
                   int64_t S, int64_t B, int64_t D, int64_t H, float eps, void* ws,
                   size_t ws_bytes, cudaStream_t s, void* saved);
size_t grid_workspace_bytes(int64_t R, int64_t C, int64_t B, int64_t H, int64_t G, int has_U);
int grid_fwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
             const float* bias, const void* top, void* h_out, int64_t R, int64_t C, int64_t B,
             int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout, cudaStream_t s);
int grid_bwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
             const void* top, const void* h_out, const void* dh, float* dW_l, float* dW_t,
             float* dU, float* dbias, void* dx, void* dtop, int64_t R, int64_t C, int64_t B,
             int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout, cudaStream_t s);
int grid_fwd_impl(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const float* bias, const void* top, void* h_out, int64_t R, int64_t C,
                  int64_t B, int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout,
                  cudaStream_t s, int64_t drop_cell, uint32_t spin_limit,
                  const flb_grid_band* band, void* saved_top);
size_t grid_band_block_bytes(int64_t C, int64_t B, int64_t H);
int grid_band_fwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const float* bias, const void* top, void* h_out, void* saved_top, int64_t R,
                  int64_t C, int64_t B, int64_t H, int64_t G, const flb_grid_band* band, void* ws,
                  size_t ws_bytes, int check_timeout, cudaStream_t s);
int grid_band_bwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const void* top, const void* h_out, const void* dh, float* dW_l, float* dW_t,
                  float* dU, float* dbias, void* dx, void* dtop, int64_t R, int64_t C, int64_t B,
                  int64_t H, int64_t G, const flb_grid_band* band, void* ws, size_t ws_bytes,
                  int check_timeout, cudaStream_t s);
int ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
int ipc_open(const void* handle, void** dev_ptr);
int ipc_close(void* dev_ptr);
int ipc_free(void* dev_ptr);
int grid_fwd_static(const void* W_l, const void* W_t, const float* bias, const void* top,
                    void* h_out, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                    int check_timeout, cudaStream_t s);
int microbench(int kind, void* scratch, double* ops_per_s);
int umma_selftest(int variant, int n, const void* A, const void* B, float* D, int* err,
                  cudaStream_t s);

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int check_attn_common(const void* q, const void* k, const void* v, const float* w,
                             const int32_t* wi, int64_t BH, int64_t N, int64_t D, int dtype) {
  if (dtype_size(dtype) == 0) return fail(FLB_ERR_DTYPE, "attention: dtype must be f32, f16 or bf16");
  if (BH < 0 || N < 0 || D <= 0) return fail(FLB_ERR_SHAPE, "attention: BH, N >= 0 and D > 0 required");
  if (D > 256) return fail(FLB_ERR_UNSUPPORTED, "attention: head dim D > 256 is not supported");
  if (N > (int64_t)INT32_MAX / 2) return fail(FLB_ERR_SHAPE, "attention: N too large");
  if (BH * N > 0 && (!q || !k || !v || !w || !wi))
    return fail(FLB_ERR_SHAPE, "attention: null input pointer");
  const size_t es = (size_t)dtype_size(dtype);
  if (!aligned(q, es) || !aligned(k, es) || !aligned(v, es) || !aligned(w, 4) || !aligned(wi, 4))
    return fail(FLB_ERR_ALIGN, "attention: pointers must be aligned to their element size");
  return FLB_OK;
}

static int check_block_args(const flb_block_weights* weights, const void* x, const void* grids,
                            int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads) {
  if (!weights || !x || !grids) return fail(FLB_ERR_SHAPE, "block_grid: null pointer");
  const flb_block_weights& w = *weights;
  if (!w.ln_lat_w || !w.ln_lat_b || !w.ln_fdbk_w || !w.ln_fdbk_b || !w.w_prior_lat ||
      !w.w_prior_fdbk || !w.w_gate_l || !w.b_gate_l || !w.w_gate_x || !w.b_gate_x || !w.w_qkv ||
      !w.w_o || !w.v_a)
    return fail(FLB_ERR_SHAPE, "block_grid: null weight pointer");
  if (L < 1 || S < 1 || batch < 1 || D < 16 || heads < 1)
    return fail(FLB_ERR_SHAPE, "block_grid: sizes must be positive (D >= 16)");
  if (D % 16 != 0 || D % heads != 0)
    return fail(FLB_ERR_SHAPE, "block_grid: D must be a multiple of 16 and of heads");
  if (D > 1024 || D / heads > 128)
    return fail(FLB_ERR_UNSUPPORTED, "block_grid: D <= 1024 and D / heads <= 128 required");
  if ((L * S + L) * batch * D * 4 > ((int64_t)1 << 40) || 3 * batch * D > (1 << 30) ||
      L + 2 * S > (1 << 30))
    return fail(FLB_ERR_SHAPE, "block_grid: grid too large");
  const int64_t nmax = (L + 1) / 2 < S ? (L + 1) / 2 : S;
  if (nmax * batch > 65535)
    return fail(FLB_ERR_UNSUPPORTED, "block_grid: cells per tick x batch must be <= 65535");
  if (((uintptr_t)x | (uintptr_t)grids | (uintptr_t)w.w_prior_lat | (uintptr_t)w.w_prior_fdbk |
       (uintptr_t)w.w_gate_l | (uintptr_t)w.w_gate_x | (uintptr_t)w.w_qkv | (uintptr_t)w.w_o) & 15u)
    return fail(FLB_ERR_ALIGN, "block_grid: bf16 tensors must be 16-byte aligned");
  return FLB_OK;
}

}  // namespace flb

using namespace flb;

extern "C" {

const char* flb_last_error(void) { return g_last_error.c_str(); }
const char* flb_version(void) { return "flb_b200 0.1 (sm_100a)"; }
uint64_t flb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int64_t flb_attn_scores_ld(int64_t N) { return N < 0 ? 0 : attn_scores_ld(N); }

size_t flb_attn_fwd_workspace_bytes(int64_t BH, int64_t N, int64_t D, int dtype, int flags) {
  if (attn_fwd_fast_supported(BH, N, D, dtype, flags))
    return attn_fwd_fast_workspace(BH, N, D, dtype, flags);
  return 0;
}

int flb_attn_fwd(const void* q, const void* k, const void* v, const float* w,
                 const int32_t* w_index, void* out, float* lse, float* scores, int64_t BH,
                 int64_t N, int64_t D, int dtype, int flags, void* workspace,
                 size_t workspace_bytes, void* stream) {
  int st = check_attn_common(q, k, v, w, w_index, BH, N, D, dtype);
  if (st != FLB_OK) return st;
  if (BH * N == 0) return FLB_OK;
  if (!out || !lse) return fail(FLB_ERR_SHAPE, "attn_fwd: null output pointer");
  cudaStream_t s = as_stream(stream);
  if (attn_fwd_fast_supported(BH, N, D, dtype, flags)) {
    const size_t need = attn_fwd_fast_workspace(BH, N, D, dtype, flags);
    if (workspace_bytes < need || (need > 0 && !workspace))
      return fail(FLB_ERR_WORKSPACE, "attn_fwd: workspace smaller than flb_attn_fwd_workspace_bytes()");
    return attn_fwd_fast(q, k, v, w, w_index, out, lse, scores, BH, (int)N, (int)D, dtype,
                         flags, workspace, workspace_bytes, s);
  }
  cudaError_t e = attn_fwd_generic(q, k, v, w, w_index, out, lse, scores, BH, (int)N, (int)D, dtype,
                                   (flags & FLB_ATTN_EXACT_TANH) != 0, (flags & FLB_ATTN_CAUSAL) != 0, s);
  if (e == cudaSuccess) count_launches(1);
  return check_cuda(e, "attn_fwd (generic) launch");
}

size_t flb_attn_bwd_workspace_bytes(int64_t BH, int64_t N, int64_t D, int dtype, int flags) {
  const size_t generic = (size_t)(BH * N) * sizeof(float);
  if (attn_bwd_fast_supported(BH, N, D, dtype, flags)) {
    const size_t fast = attn_bwd_fast_workspace(BH, N, D, dtype, flags);
    return fast > generic ? fast : generic;
  }
  return generic;
}

int flb_attn_bwd(const void* q, const void* k, const void* v, const float* w,
                 const int32_t* w_index, const void* out, const float* lse,
                 const float* scores, const void* dout, void* dq, void* dk, void* dv, float* dw,
                 int64_t BH, int64_t N, int64_t D,
                 int64_t n_w_rows, int dtype, int flags, void* workspace, size_t workspace_bytes,
                 void* stream) {
  int st = check_attn_common(q, k, v, w, w_index, BH, N, D, dtype);
  if (st != FLB_OK) return st;
  if (BH * N == 0) return FLB_OK;
  if (!out || !lse || !dout || !dq || !dk || !dv || !dw)
    return fail(FLB_ERR_SHAPE, "attn_bwd: null pointer");
  if (n_w_rows <= 0) return fail(FLB_ERR_SHAPE, "attn_bwd: n_w_rows must be positive");
  const size_t need = flb_attn_bwd_workspace_bytes(BH, N, D, dtype, flags);
  if (workspace_bytes < need || !workspace)
    return fail(FLB_ERR_WORKSPACE, "attn_bwd: workspace smaller than flb_attn_bwd_workspace_bytes()");
  cudaStream_t s = as_stream(stream);
  if (scores != nullptr && attn_bwd_fast_supported(BH, N, D, dtype, flags))
    return attn_bwd_fast(q, k, v, w, w_index, out, lse, scores, dout, dq, dk, dv, dw, BH,
                         (int)N, (int)D, dtype, flags, workspace, workspace_bytes, s);
  cudaError_t e = attn_bwd_generic(q, k, v, w, w_index, out, lse, dout, dq, dk, dv, dw,
                                   (float*)workspace, BH, (int)N, (int)D, dtype,
                                   (flags & FLB_ATTN_EXACT_TANH) != 0, (flags & FLB_ATTN_CAUSAL) != 0, s);
  if (e == cudaSuccess) count_launches(2);
  return check_cuda(e, "attn_bwd (generic) launch");
}

int flb_wf_gather(const void* x, const int64_t x_strides[3], const void* grids,
                  const int64_t grid_strides[4], const int32_t* routing, const int32_t* port_map,
                  const int32_t* spatial_map, const int32_t* active_cells, int64_t n_active,
                  int64_t n_cells, void* gathered, const int64_t gathered_strides[4],
                  int64_t n_deps, int64_t batch, int64_t dim, int dtype, void* stream) {
  if (n_active < 0 || n_cells < 0 || n_deps < 0 || batch < 0 || dim < 0)
    return fail(FLB_ERR_SHAPE, "wf_gather: negative size");
  if (n_deps * n_active * batch * dim > 0 &&
      (!x || !grids || !routing || !port_map || !spatial_map || !active_cells || !gathered))
    return fail(FLB_ERR_SHAPE, "wf_gather: null pointer");
  return wf_gather(x, x_strides, grids, grid_strides, routing, port_map, spatial_map,
                   active_cells, n_active, n_cells, gathered, gathered_strides, n_deps, batch,
                   dim, dtype, as_stream(stream));
}

int flb_wf_index_copy(const void* src, int src_dtype, const int64_t src_strides[3],
                      const int64_t* src_rows, void* dst, int dst_dtype,
                      const int64_t dst_strides[3], const int64_t* dst_rows, int64_t n_rows,
                      int64_t batch, int64_t dim, int accumulate, void* stream) {
  if (n_rows < 0 || batch < 0 || dim < 0) return fail(FLB_ERR_SHAPE, "wf_index_copy: negative size");
  if (n_rows * batch * dim > 0 && (!src || !src_rows || !dst || !dst_rows))
    return fail(FLB_ERR_SHAPE, "wf_index_copy: null pointer");
  return wf_index_copy(src, src_dtype, src_strides, src_rows, dst, dst_dtype, dst_strides,
                       dst_rows, n_rows, batch, dim, accumulate, as_stream(stream));
}

size_t flb_block_grid_workspace_bytes(int64_t L, int64_t S, int64_t batch, int64_t D) {
  if (L < 1 || S < 1 || batch < 1 || D < 1) return 0;
  return block_grid_workspace_bytes(L, S, batch, D);
}

int flb_block_grid_fwd(const flb_block_weights* weights, const void* x, void* grids, int64_t L,
                       int64_t S, int64_t batch, int64_t D, int64_t heads, float ln_eps,
                       void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_block_args(weights, x, grids, L, S, batch, D, heads);
  if (st != FLB_OK) return st;
  const size_t need = block_grid_workspace_bytes(L, S, batch, D);
  if (!workspace || workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "block_grid_fwd: workspace smaller than flb_block_grid_workspace_bytes()");
  return block_grid_fwd(weights, x, grids, L, S, batch, D, heads, ln_eps, workspace,
                        workspace_bytes, as_stream(stream));
}

int flb_block_grid_fwd_ex(const flb_block_weights* weights, const void* x, void* grids,
                          int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads,
                          float ln_eps, void* workspace, size_t workspace_bytes, int path,
                          void* stream) {
  int st = check_block_args(weights, x, grids, L, S, batch, D, heads);
  if (st != FLB_OK) return st;
  if (path < FLB_BLOCK_PATH_AUTO || path > FLB_BLOCK_PATH_PERSISTENT)
    return fail(FLB_ERR_SHAPE, "block_grid_fwd_ex: unknown path");
  const size_t need = block_grid_workspace_bytes(L, S, batch, D);
  if (!workspace || workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "block_grid_fwd_ex: workspace smaller than flb_block_grid_workspace_bytes()");
  return block_grid_fwd_ex(weights, x, grids, L, S, batch, D, heads, ln_eps, workspace,
                           workspace_bytes, as_stream(stream), path, -1, -1, 0, nullptr);
}

int flb_block_grid_status(const void* workspace, void* stream) {
  if (!workspace) return fail(FLB_ERR_WORKSPACE, "block_grid_status: null workspace");
  return block_grid_status(workspace, as_stream(stream));
}

int flb_block_grid_fwd_drop_barrier_test(const flb_block_weights* weights, const void* x,
                                         void* grids, int64_t L, int64_t S, int64_t batch,
                                         int64_t D, int64_t heads, float ln_eps, void* workspace,
                                         size_t workspace_bytes, int64_t drop_cta,
                                         int64_t drop_barrier, uint32_t spin_limit, void* stream) {
  int st = check_block_args(weights, x, grids, L, S, batch, D, heads);
  if (st != FLB_OK) return st;
  const size_t need = block_grid_workspace_bytes(L, S, batch, D);
  if (!workspace || workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "block_grid drop test: workspace smaller than flb_block_grid_workspace_bytes()");
  if (drop_cta < 0 || drop_cta >= num_sms() || drop_barrier < 0 || spin_limit < 1)
    return fail(FLB_ERR_SHAPE, "block_grid drop test: drop_cta must name a CTA of the launch, drop_barrier >= 0, spin_limit >= 1");
  st = block_grid_fwd_ex(weights, x, grids, L, S, batch, D, heads, ln_eps, workspace,
                         workspace_bytes, as_stream(stream), FLB_BLOCK_PATH_PERSISTENT,
                         (int)drop_cta, (int)drop_barrier, spin_limit, nullptr);
  if (st != FLB_OK) return st;
  return block_grid_status(workspace, as_stream(stream));
}

size_t flb_block_grid_bwd_workspace_bytes(int64_t L, int64_t S, int64_t batch, int64_t D) {
  if (L < 1 || S < 1 || batch < 1 || D < 1) return 0;
  return block_grid_bwd_workspace_bytes(L, S, batch, D);
}

int flb_block_grid_bwd(const flb_block_weights* weights, const void* x, const void* grids,
                       const void* dgrid0, const void* dgrid1, const void* dgrid2,
                       const void* dgrid3, float* dx, const flb_block_grads* grads, int64_t L,
                       int64_t S, int64_t batch, int64_t D, int64_t heads, float ln_eps,
                       void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_block_args(weights, x, grids, L, S, batch, D, heads);
  if (st != FLB_OK) return st;
  if (!dx || !grads) return fail(FLB_ERR_SHAPE, "block_grid_bwd: null dx or grads");
  const flb_block_grads& g = *grads;
  if (!g.ln_lat_w || !g.ln_lat_b || !g.ln_fdbk_w || !g.ln_fdbk_b || !g.w_prior_lat ||
      !g.w_prior_fdbk || !g.w_gate_l || !g.b_gate_l || !g.w_gate_x || !g.b_gate_x || !g.w_qkv ||
      !g.w_o || !g.v_a)
    return fail(FLB_ERR_SHAPE, "block_grid_bwd: null gradient pointer");
  if (((uintptr_t)dgrid0 | (uintptr_t)dgrid1 | (uintptr_t)dgrid2 | (uintptr_t)dgrid3 |
       (uintptr_t)dx) & 15u)
    return fail(FLB_ERR_ALIGN, "block_grid_bwd: gradient grids and dx must be 16-byte aligned");
  const size_t need = block_grid_bwd_workspace_bytes(L, S, batch, D);
  if (!workspace || workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "block_grid_bwd: workspace smaller than flb_block_grid_bwd_workspace_bytes()");
  const void* dg[4] = {dgrid0, dgrid1, dgrid2, dgrid3};
  return block_grid_bwd(weights, x, grids, dg, dx, grads, L, S, batch, D, heads, ln_eps,
                        workspace, workspace_bytes, as_stream(stream), nullptr);
}

size_t flb_block_grid_saved_bytes(int64_t L, int64_t S, int64_t batch, int64_t D) {
  if (L < 1 || S < 1 || batch < 1 || D < 1) return 0;
  return block_grid_saved_bytes(L, S, batch, D);
}

int flb_block_grid_fwd_save(const flb_block_weights* weights, const void* x, void* grids, int64_t L,
                            int64_t S, int64_t batch, int64_t D, int64_t heads, float ln_eps,
                            void* workspace, size_t workspace_bytes, void* saved,
                            size_t saved_bytes, void* stream) {
  int st = check_block_args(weights, x, grids, L, S, batch, D, heads);
  if (st != FLB_OK) return st;
  const size_t need = block_grid_workspace_bytes(L, S, batch, D);
  if (!workspace || workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "block_grid_fwd_save: workspace smaller than flb_block_grid_workspace_bytes()");
  if (!saved || saved_bytes < block_grid_saved_bytes(L, S, batch, D))
    return fail(FLB_ERR_WORKSPACE, "block_grid_fwd_save: saved buffer smaller than flb_block_grid_saved_bytes()");
  if ((uintptr_t)saved & 15u) return fail(FLB_ERR_ALIGN, "block_grid_fwd_save: saved must be 16-byte aligned");
  return block_grid_fwd_ex(weights, x, grids, L, S, batch, D, heads, ln_eps, workspace,
                           workspace_bytes, as_stream(stream), FLB_BLOCK_PATH_TICKS, -1, -1, 0, saved);
}

int flb_block_grid_bwd_saved(const flb_block_weights* weights, const void* x, const void* grids,
                             const void* dgrid0, const void* dgrid1, const void* dgrid2,
                             const void* dgrid3, float* dx, const flb_block_grads* grads,
                             int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads,
                             float ln_eps, void* workspace, size_t workspace_bytes,
                             void* saved, size_t saved_bytes, void* stream) {
  if (!saved || saved_bytes < block_grid_saved_bytes(L, S, batch, D))
    return fail(FLB_ERR_WORKSPACE, "block_grid_bwd_saved: saved buffer smaller than flb_block_grid_saved_bytes()");
  if ((uintptr_t)saved & 15u) return fail(FLB_ERR_ALIGN, "block_grid_bwd_saved: saved must be 16-byte aligned");
  int st = check_block_args(weights, x, grids, L, S, batch, D, heads);
  if (st != FLB_OK) return st;
  if (!dx || !grads) return fail(FLB_ERR_SHAPE, "block_grid_bwd_saved: null dx or grads");
  const flb_block_grads& g = *grads;
  if (!g.ln_lat_w || !g.ln_lat_b || !g.ln_fdbk_w || !g.ln_fdbk_b || !g.w_prior_lat ||
      !g.w_prior_fdbk || !g.w_gate_l || !g.b_gate_l || !g.w_gate_x || !g.b_gate_x || !g.w_qkv ||
      !g.w_o || !g.v_a)
    return fail(FLB_ERR_SHAPE, "block_grid_bwd_saved: null gradient pointer");
  if (((uintptr_t)dgrid0 | (uintptr_t)dgrid1 | (uintptr_t)dgrid2 | (uintptr_t)dgrid3 |
       (uintptr_t)dx) & 15u)
    return fail(FLB_ERR_ALIGN, "block_grid_bwd_saved: gradient grids and dx must be 16-byte aligned");
  const size_t need = block_grid_bwd_workspace_bytes(L, S, batch, D);
  if (!workspace || workspace_bytes < need)
    return fail(FLB_ERR_WORKSPACE, "block_grid_bwd_saved: workspace smaller than flb_block_grid_bwd_workspace_bytes()");
  const void* dg[4] = {dgrid0, dgrid1, dgrid2, dgrid3};
  return block_grid_bwd(weights, x, grids, dg, dx, grads, L, S, batch, D, heads, ln_eps,
                        workspace, workspace_bytes, as_stream(stream), saved);
}

size_t flb_grid_workspace_bytes(int64_t R, int64_t C, int64_t B, int64_t H, int64_t G, int has_U) {
  return grid_workspace_bytes(R, C, B, H, G, has_U);
}

int flb_grid_fwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                 const float* bias, const void* top, void* h_out, int64_t R, int64_t C,
                 int64_t B, int64_t H, int64_t G, void* workspace, size_t workspace_bytes,
                 int check_timeout, void* stream) {
  return grid_fwd(x, x_layout, W_l, W_t, U, bias, top, h_out, R, C, B, H, G, workspace,
                  workspace_bytes, check_timeout, as_stream(stream));
}

int flb_grid_bwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                 const void* top, const void* h_out, const void* dh, float* dW_l, float* dW_t,
                 float* dU, float* dbias, void* dx, void* dtop, int64_t R, int64_t C, int64_t B,
                 int64_t H, int64_t G, void* workspace, size_t workspace_bytes, int check_timeout,
                 void* stream) {
  return grid_bwd(x, x_layout, W_l, W_t, U, top, h_out, dh, dW_l, dW_t, dU, dbias, dx, dtop, R,
                  C, B, H, G, workspace, workspace_bytes, check_timeout, as_stream(stream));
}

int flb_grid_fwd_drop_flag_test(const void* x, int x_layout, const void* W_l, const void* W_t,
                                const void* U, const float* bias, const void* top, void* h_out,
                                int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                                void* workspace, size_t workspace_bytes, int64_t drop_row,
                                int64_t drop_col, uint32_t spin_limit, void* stream) {
  if (drop_row < 0 || drop_row >= R || drop_col < 0 || drop_col >= C)
    return fail(FLB_ERR_SHAPE, "grid drop-flag test: cell outside the grid");
  return grid_fwd_impl(x, x_layout, W_l, W_t, U, bias, top, h_out, R, C, B, H, G, workspace,
                       workspace_bytes, 1, as_stream(stream), drop_row * C + drop_col,
                       spin_limit, nullptr, nullptr);
}

size_t flb_grid_band_block_bytes(int64_t C, int64_t B, int64_t H) {
  if (C < 1 || B < 1 || H < 1) return 0;
  return grid_band_block_bytes(C, B, H);
}

int flb_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) { return ipc_alloc(bytes, dev_ptr, handle); }
int flb_ipc_open(const void* handle, void** dev_ptr) { return ipc_open(handle, dev_ptr); }
int flb_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return fail(FLB_ERR_SHAPE, "ipc_close: null pointer");
  return ipc_close(dev_ptr);
}
int flb_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return fail(FLB_ERR_SHAPE, "ipc_free: null pointer");
  return ipc_free(dev_ptr);
}

int flb_grid_band_fwd(const void* x, int x_layout, const void* W_l, const void* W_t,
                      const void* U, const float* bias, const void* top, void* h_out,
                      void* saved_top, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                      const flb_grid_band* band, void* workspace, size_t workspace_bytes,
                      int check_timeout, void* stream) {
  return grid_band_fwd(x, x_layout, W_l, W_t, U, bias, top, h_out, saved_top, R, C, B, H, G, band,
                       workspace, workspace_bytes, check_timeout, as_stream(stream));
}

int flb_grid_band_bwd(const void* x, int x_layout, const void* W_l, const void* W_t,
                      const void* U, const void* top, const void* h_out, const void* dh,
                      float* dW_l, float* dW_t, float* dU, float* dbias, void* dx, void* dtop,
                      int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                      const flb_grid_band* band, void* workspace, size_t workspace_bytes,
                      int check_timeout, void* stream) {
  return grid_band_bwd(x, x_layout, W_l, W_t, U, top, h_out, dh, dW_l, dW_t, dU, dbias, dx, dtop,
                       R, C, B, H, G, band, workspace, workspace_bytes, check_timeout,
                       as_stream(stream));
}

int flb_grid_fwd_static(const void* W_l, const void* W_t, const float* bias, const void* top,
                        void* h_out, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                        int check_timeout, void* stream) {
  return grid_fwd_static(W_l, W_t, bias, top, h_out, R, C, B, H, G, check_timeout,
                         as_stream(stream));
}

int flb_microbench(int kind, void* scratch, double* ops_per_s) {
  if (!scratch || !ops_per_s) return fail(FLB_ERR_SHAPE, "microbench: null pointer");
  return microbench(kind, scratch, ops_per_s);
}

int flb_selftest_umma(int variant, int n, const void* A, const void* B, float* D, int* err,
                      void* stream) {
  if (!A || !B || !D || !err) return fail(FLB_ERR_SHAPE, "selftest_umma: null pointer");
  return umma_selftest(variant, n, A, B, D, err, as_stream(stream));
}

}  // extern "C"
