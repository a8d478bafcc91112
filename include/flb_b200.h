/*
 * flb_b200.h — C ABI of the B200 (sm_100a) implementation of FLB-Transformer's two hot paths:
 *   (1) fused additive attention  s[i,j] = sum_d w[d] * tanh(q[i,d] + k[j,d]) / sqrt(D),
 *       row softmax, out = P @ V, forward and backward;
 *   (2) the anti-diagonal wavefront engine (dependency gather, port scatter, gradient routing)
 *       and the persistent tanh grid-cell kernels.
 *
 * Conventions shared by every entry point:
 *   - all pointers are DEVICE pointers unless stated otherwise; the library never allocates,
 *     never frees and never synchronises the stream (except where an error word is read back,
 *     which is stated per function);
 *   - every call is enqueued on `stream` (a cudaStream_t passed as void*; NULL = legacy stream);
 *   - the return value is an flb_status; FLB_OK == 0.  flb_last_error() returns a thread-local
 *     message for the last non-zero status raised on the calling thread;
 *   - dtypes are flb_dtype codes; q/k/v/out and grid tensors share one dtype per call.
 */
#ifndef FLB_B200_H
#define FLB_B200_H

#include <stdint.h>
#include <stddef.h>

/* Only the C API is exported from libflb_b200.so (built with -fvisibility=hidden). */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  FLB_OK = 0,
  FLB_ERR_SHAPE = 1,        /* bad or inconsistent sizes / strides                     */
  FLB_ERR_DTYPE = 2,        /* unsupported dtype code                                  */
  FLB_ERR_ALIGN = 3,        /* pointer or stride not aligned as the kernel requires    */
  FLB_ERR_TIMEOUT = 4,      /* a bounded device-side wait gave up (error word set)     */
  FLB_ERR_LAUNCH = 5,       /* kernel launch failed                                    */
  FLB_ERR_UNSUPPORTED = 6,  /* valid request this build does not implement             */
  FLB_ERR_CUDA = 7,         /* a CUDA runtime / driver / cuBLAS call failed            */
  FLB_ERR_WORKSPACE = 8     /* workspace missing or smaller than the size query says   */
} flb_status;

typedef enum { FLB_F32 = 0, FLB_F16 = 1, FLB_BF16 = 2 } flb_dtype;

/* attention flags */
#define FLB_ATTN_CAUSAL      1  /* mask j > i (extension; the reference has no mask)          */
#define FLB_ATTN_EXACT_TANH  2  /* tanhf/expf instead of tanh.approx / ex2.approx             */
#define FLB_ATTN_FORCE_GENERIC 4 /* use the CUDA-core kernels even where a tcgen05 kernel fits */

const char* flb_last_error(void);
const char* flb_version(void);
/* Number of kernels this library has launched in this process (all threads, all devices). */
uint64_t flb_launch_count(void);

/* ------------------------------------------------------------------------------------------
 * Fused additive attention.
 * Layout: q, k, v, out are contiguous [BH, N, D] (BH = prod(batch dims) * H) in `dtype`.
 * w is a float32 table [n_w_rows, D]; head bh uses row w_index[bh] (int32, device), which is
 * how a v_a broadcast to [..., H, 1, D] is expressed without materialising it.
 * lse (float32 [BH, N]) receives the natural-log row log-sum-exp of the scaled scores.
 * ------------------------------------------------------------------------------------------ */

/* Replaces FusedAdditiveAttentionFunc.forward + fused_additive_attention_kernel
 * (kernels/additive_attention.py:137-181 and :10-86). Scale 1/sqrt(D) as at :66,:145.
 * scores: optional float32 [BH, N, flb_attn_scores_ld(N)] output of the scaled scores s[i,j]
 * (row pitch padded to 16 bytes; padding and, when causal, entries with j > i are left
 * unwritten). When the backward is going to run, saving them lets it skip the score
 * recomputation (one full tanh pass); NULL = do not save.
 * Workspace: flb_attn_fwd_workspace_bytes(); may be NULL when that returns 0. */
int flb_attn_fwd(const void* q, const void* k, const void* v,
                 const float* w, const int32_t* w_index,
                 void* out, float* lse, float* scores,
                 int64_t BH, int64_t N, int64_t D, int dtype, int flags,
                 void* workspace, size_t workspace_bytes, void* stream);

size_t flb_attn_fwd_workspace_bytes(int64_t BH, int64_t N, int64_t D, int dtype, int flags);

/* Row pitch, in floats, of the saved scores: N rounded up to a multiple of 4 (16-byte rows, as
 * the backward's TMA loads need). No reference counterpart (the reference saves no scores). */
int64_t flb_attn_scores_ld(int64_t N);

/* Replaces FusedAdditiveAttentionFunc.backward -> compiled_backward_math
 * (kernels/additive_attention.py:188-198 and :91-130).
 * Inputs q,k,v,out,lse,dout as produced by flb_attn_fwd; outputs dq,dk,dv in `dtype`
 * ([BH,N,D], overwritten) and dw, a float32 [n_w_rows, D] table that is ACCUMULATED into
 * (caller zeroes it), matching the reduction of grad_va over broadcast dims (:126-128).
 * scores: the [BH, N, flb_attn_scores_ld(N)] scores saved by flb_attn_fwd, or NULL to
 * recompute them.
 * Workspace: flb_attn_bwd_workspace_bytes(). */
int flb_attn_bwd(const void* q, const void* k, const void* v,
                 const float* w, const int32_t* w_index,
                 const void* out, const float* lse, const float* scores, const void* dout,
                 void* dq, void* dk, void* dv, float* dw,
                 int64_t BH, int64_t N, int64_t D, int64_t n_w_rows, int dtype, int flags,
                 void* workspace, size_t workspace_bytes, void* stream);

size_t flb_attn_bwd_workspace_bytes(int64_t BH, int64_t N, int64_t D, int dtype, int flags);

/* ------------------------------------------------------------------------------------------
 * Wavefront engine primitives (generic-layer path).
 * Strides are in ELEMENTS.
 * ------------------------------------------------------------------------------------------ */

/* Replaces fetch_mapped_context_kernel / run_fetch_kernel (wavefront/wavefront_kernel.py:27-82,
 * :84-106) and its Python twin fetch_mapped_context (:6-25).
 * For every slot s < n_active and dependency i < n_deps, with cell = active_cells[s] and
 * t = routing[cell*n_deps + i] (cells >= n_cells are padding and read as t = -1):
 *   t >= 0  -> gathered[i, s, b, :] = grids[port_map[i], t, b, :]
 *   t == -2 -> gathered[i, s, b, :] = x[b, spatial_map[cell], :]
 *   t == -1 -> gathered[i, s, b, :] = 0
 * grids strides (port, cell, batch, dim); x strides (batch, seq, dim);
 * gathered strides (dep, slot, batch, dim). */
int flb_wf_gather(const void* x, const int64_t x_strides[3],
                  const void* grids, const int64_t grid_strides[4],
                  const int32_t* routing, const int32_t* port_map, const int32_t* spatial_map,
                  const int32_t* active_cells, int64_t n_active, int64_t n_cells,
                  void* gathered, const int64_t gathered_strides[4],
                  int64_t n_deps, int64_t batch, int64_t dim, int dtype, void* stream);

/* Indexed row copy / accumulate, the data movement of the C++ orchestrator's per-tick
 * scatters. Replaces, with one primitive:
 *   - the per-port index_put_ of cell outputs into the stacked grids
 *     (csrc/wavefront_backend.cpp:40-43),
 *   - the per-cell index_put_ of parameter gradients (csrc/wavefront_backend.cpp:97-106) and,
 *     with accumulate != 0 and per-layer destination rows, the later per-layer sum
 *     (wavefront/wavefront_engine.py:132-139) done on the fly,
 *   - the index_add_ routing of dependency gradients into the gradient grids and into grad_x
 *     (csrc/wavefront_backend.cpp:109-130).
 * For k < n_rows, b < batch, e < dim:
 *   dst[dst_rows[k]*ds[0] + b*ds[1] + e*ds[2]]  (=, or += when accumulate)
 *       src[src_rows[k]*ss[0] + b*ss[1] + e*ss[2]]
 * Row index arrays are int64 (device). src and dst dtypes may differ (e.g. bf16 gradients into
 * float32 accumulators). Accumulation uses atomics; with accumulate == 0 and repeated dst rows
 * the surviving write is unspecified, as for index_put_. */
int flb_wf_index_copy(const void* src, int src_dtype, const int64_t src_strides[3],
                      const int64_t* src_rows,
                      void* dst, int dst_dtype, const int64_t dst_strides[3],
                      const int64_t* dst_rows,
                      int64_t n_rows, int64_t batch, int64_t dim, int accumulate, void* stream);

/* ------------------------------------------------------------------------------------------
 * Persistent tanh grid cell (the wavefront grid layer), bf16 storage / fp32 accumulation:
 *   h[r][c] = tanh(W_l[g] h[r][c-1] + W_t[g] h[r-1][c] + add[r][c] + bias[g]),  g = r if
 *   per_row_weights else 0; h[r][-1] = 0; h[-1][c] = top[c] (or 0 when top == NULL);
 *   add = x[r][c] @ U^T (hoisted GEMM) when U != NULL, else 0.
 * This is the cell of the wavefront engine with dependencies ((-1,0),port 0) and
 * ((0,-1),port 1) (wavefront/wavefront_api.py:12-14), evaluated by one persistent kernel with
 * per-cell dependency flags instead of one host tick per anti-diagonal
 * (csrc/wavefront_backend.cpp:16-44).
 * Shapes: R rows, C cols, B batch, H hidden (H in {128,256}; B a multiple of 16, <= 64).
 * x: [B, R, C, H] bf16 (row-major, x_layout 0) or [R, C, B, H] (x_layout 1).
 * W_l, W_t: [G, H, H] bf16 (nn.Linear layout [out, in]); U: [H, H] bf16 or NULL; bias: [G, H] f32.
 * top: [C, B, H] bf16 or NULL. h_out: [R, C, B, H] bf16 (engine grid order: cell-major).
 * Workspace: flb_grid_workspace_bytes() (the backward takes its own, of the same size).
 * A device error word is read back (one 4-byte D2H copy, stream-synchronising) only when
 * check_timeout != 0.
 * ------------------------------------------------------------------------------------------ */
size_t flb_grid_workspace_bytes(int64_t R, int64_t C, int64_t B, int64_t H, int64_t G, int has_U);

int flb_grid_fwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                 const float* bias, const void* top, void* h_out,
                 int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                 void* workspace, size_t workspace_bytes, int check_timeout, void* stream);

/* Backward of flb_grid_fwd. dh: [R, C, B, H] bf16 upstream gradient of h_out.
 * Outputs (float32, OVERWRITTEN): dW_l, dW_t [G,H,H]; dU [H,H] (when U was given);
 * dbias [G,H]; bf16 outputs: dx (same layout as x, when U was given, else NULL) and
 * dtop [C,B,H] (when top was given, else NULL). */
int flb_grid_bwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                 const void* top, const void* h_out, const void* dh,
                 float* dW_l, float* dW_t, float* dU, float* dbias, void* dx, void* dtop,
                 int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                 void* workspace, size_t workspace_bytes, int check_timeout, void* stream);

/* ------------------------------------------------------------------------------------------
 * Row bands: one grid layer split by rows across the GPUs of a node, one process per GPU.
 * No counterpart in the reference, which runs on one device (training/trainer.py:31); this is
 * the row-band partitioning of the grid layer (one exchange step per column).
 * The band of rows row0 .. row0 + R - 1 (of rows_total) runs its persistent sweep while the
 * neighbouring bands run theirs on other GPUs; the rows at the band edges exchange [C, B, H]
 * bf16 halos through NVLink peer memory, column by column, inside the sweep kernels:
 *   forward:  the last row of the band above stores h[row0 - 1][c] into this rank's receive
 *             block and releases a per-column flag; this band's row 0 waits for the flag,
 *             loads the halo from local memory by TMA, keeps a copy in saved_top, and
 *             acknowledges, so that the next call may overwrite it;
 *   backward: mirrored, with dz of the first row of the band below, consumed by this band's
 *             last row through W_t[row0 + R] (all ranks hold all weights).
 * Each rank allocates its receive block with flb_ipc_alloc(flb_grid_band_block_bytes(C,B,H)),
 * shares the handle with its neighbours, and maps theirs with flb_ipc_open. Flags carry an
 * epoch: every rank passes the same epoch to its k-th band forward (1, 2, 3, ...) and, counted
 * separately, to its k-th band backward. Ranks must issue their band calls in the same order;
 * a rank that never arrives makes its neighbours' bounded waits give up (FLB_ERR_TIMEOUT when
 * check_timeout != 0). Weight gradients of a band are partial sums over its rows: all-reduce
 * them across the ranks (their rows outside the band are zero with per-row weights).
 * ------------------------------------------------------------------------------------------ */
typedef struct flb_grid_band {
  int64_t row0;             /* global index of this band's first row */
  int64_t rows_total;       /* rows of the whole grid */
  void* own_block;          /* this rank's receive block (flb_ipc_alloc) */
  void* up_block;           /* the band above's block mapped here (flb_ipc_open); NULL iff row0 == 0 */
  void* down_block;         /* the band below's block; NULL iff row0 + R == rows_total */
  int epoch;                /* >= 1, see above */
} flb_grid_band;

#define FLB_IPC_HANDLE_BYTES 80
size_t flb_grid_band_block_bytes(int64_t C, int64_t B, int64_t H);
/* Device allocation on the current GPU, zero-filled, exportable to other processes: writes the
 * pointer and a FLB_IPC_HANDLE_BYTES-byte handle (CUDA's IPC handle and the GPU's UUID). */
int flb_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
/* Maps another process's flb_ipc_alloc allocation (by its handle) into this process. Fails with
 * FLB_ERR_UNSUPPORTED when it lives on the current GPU: band kernels wait on each other and
 * must run on different GPUs. */
int flb_ipc_open(const void* handle, void** dev_ptr);
int flb_ipc_close(void* dev_ptr);
int flb_ipc_free(void* dev_ptr);

/* Forward of one band. Arguments as for flb_grid_fwd with R = the band's rows, x and h_out the
 * band's rows, and G in {1, rows_total} (per-row weights indexed by global row). top: the grid's
 * top row, only for the first band (else NULL). saved_top: [C, B, H] bf16, required below the
 * first band: receives h[row0 - 1][.] for the backward. Workspace: flb_grid_workspace_bytes(R,
 * C, B, H, G, has_U). */
int flb_grid_band_fwd(const void* x, int x_layout, const void* W_l, const void* W_t,
                      const void* U, const float* bias, const void* top, void* h_out,
                      void* saved_top, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                      const flb_grid_band* band, void* workspace, size_t workspace_bytes,
                      int check_timeout, void* stream);
/* Backward of one band. As flb_grid_bwd; top: the first band's top (or NULL), below it the
 * saved_top of the forward; dtop only for the first band. dW_l, dW_t, dU, dbias: this band's
 * partial sums (all-reduce across the ranks). */
int flb_grid_band_bwd(const void* x, int x_layout, const void* W_l, const void* W_t,
                      const void* U, const void* top, const void* h_out, const void* dh,
                      float* dW_l, float* dW_t, float* dU, float* dbias, void* dx, void* dtop,
                      int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                      const flb_grid_band* band, void* workspace, size_t workspace_bytes,
                      int check_timeout, void* stream);

/* Allocation-free form of flb_grid_fwd for callers that cannot allocate device memory when they
 * run the layer (a serving process with its memory carved into a fixed pool up front, code running
 * inside another runtime's allocator). No counterpart in the reference. It takes no workspace:
 * its scratch (error word and per-cell dependency flags) is a static device array of the library,
 * 512 KB + 256 B on every device that loads it, held until process exit, which limits it to
 * R * C <= 65536 cells (larger grids are rejected with FLB_ERR_SHAPE). It evaluates the engine
 * form of the cell (no x U^T term: x enters through `top`, or not at all). The first call on a
 * device looks the array's address up and caches it, so make that call before any stream
 * capture. All calls share the array and each clears what it uses; calls whose kernels could
 * overlap on the GPU race on it and must be ordered. Arguments as for flb_grid_fwd. */
int flb_grid_fwd_static(const void* W_l, const void* W_t, const float* bias, const void* top,
                        void* h_out, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                        int check_timeout, void* stream);

/* ------------------------------------------------------------------------------------------
 * FLB block cells (inference forward).
 * Replaces the per-tick evaluation of FLB_Block cells by the engine (batched_forward under
 * torch.vmap, wavefront/wavefront_engine.py:185-198, models/FLB_Model.py:32-96) for the FLB
 * grid: L layers x S positions, dependencies top -> port 0, left -> port 1, bottom-left ->
 * port 2, four ports, 8-head additive attention over the three tokens.
 * Weights are per-layer stacks (nn.Linear layout [out, in], bf16) and float32 vectors; w_qkv is
 * [L, 3D, D] = W_q, W_k, W_v of each layer stacked by rows.
 * ------------------------------------------------------------------------------------------ */
typedef struct flb_block_weights {
  const float* ln_lat_w;   /* [L, D] norm_lat weight, bias */
  const float* ln_lat_b;
  const float* ln_fdbk_w;  /* [L, D] norm_fdbk weight, bias */
  const float* ln_fdbk_b;
  const void* w_prior_lat;   /* bf16 [L, D, D] proj_lateral */
  const void* w_prior_fdbk;  /* bf16 [L, D, D] proj_feedback */
  const void* w_gate_l;      /* bf16 [L, D, D] flb_attention.linear_gate_L; bias f32 [L, D] */
  const float* b_gate_l;
  const void* w_gate_x;      /* bf16 [L, D, D] flb_attention.linear_gate_X; bias f32 [L, D] */
  const float* b_gate_x;
  const void* w_qkv;         /* bf16 [L, 3D, D] W_q | W_k | W_v */
  const void* w_o;           /* bf16 [L, D, D] W_o */
  const float* v_a;          /* [L, H, D/H] */
} flb_block_weights;

size_t flb_block_grid_workspace_bytes(int64_t L, int64_t S, int64_t batch, int64_t D);

/* Whole-grid forward of FLB block cells on `stream` (no host synchronisation).
 * x: bf16 [batch, S, D] (row 0's top input). grids: bf16 [4, L*S + L, batch, D], the engine's
 * port grids (cell l*S + t; the last L rows are its boundary dock and are not touched); every
 * cell of ports 0-3 is written: h_x, h_lat, h_fdbk and the auxiliary loss term. D must be a
 * multiple of 16 and of `heads`, D <= 1024 and D / heads <= 128; ln_eps is the LayerNorms'
 * epsilon. Runs tick by tick (own kernels and cuBLAS projections); flb_block_grid_fwd_ex also
 * offers the persistent path. */
int flb_block_grid_fwd(const flb_block_weights* weights, const void* x, void* grids,
                       int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads,
                       float ln_eps, void* workspace, size_t workspace_bytes, void* stream);

#define FLB_BLOCK_PATH_AUTO       0  /* the faster path measured on B200: tick by tick */
#define FLB_BLOCK_PATH_TICKS      1  /* tick by tick */
#define FLB_BLOCK_PATH_PERSISTENT 2  /* persistent; FLB_ERR_UNSUPPORTED for other shapes */

/* flb_block_grid_fwd with the evaluation path chosen (no reference counterpart: the reference
 * has one path, the engine's tick loop). The persistent path (batch 16, D a multiple of 128 up
 * to 1024) evaluates the whole grid in ONE cooperative kernel, one CTA per SM: every projection
 * on tcgen05 tensor cores with weights streamed by TMA, the elementwise steps fused into its
 * activation loads and epilogues, grid barriers between a tick's five stages. It is
 * deterministic (bit-identical across runs). */
int flb_block_grid_fwd_ex(const flb_block_weights* weights, const void* x, void* grids,
                          int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads,
                          float ln_eps, void* workspace, size_t workspace_bytes, int path,
                          void* stream);

/* Error word of the last persistent forward run with `workspace` (no reference counterpart):
 * synchronises `stream`, returns FLB_ERR_TIMEOUT if a bounded wait in the kernel gave up (the
 * grids are then incomplete), else FLB_OK. */
int flb_block_grid_status(const void* workspace, void* stream);

/* Failure-detection check of the persistent forward's grid barriers (no reference
 * counterpart). Runs the persistent forward with CTA drop_cta never arriving at its
 * drop_barrier-th grid barrier and the barrier-poll bound lowered to spin_limit: the other CTAs
 * give up, record the error word and raise the abort flag, every CTA drains its copies and MMAs
 * and returns, and the call returns FLB_ERR_TIMEOUT (read back synchronously) with the context
 * still usable. No GPU fault or trap is involved. */
int flb_block_grid_fwd_drop_barrier_test(const flb_block_weights* weights, const void* x,
                                         void* grids, int64_t L, int64_t S, int64_t batch,
                                         int64_t D, int64_t heads, float ln_eps, void* workspace,
                                         size_t workspace_bytes, int64_t drop_cta,
                                         int64_t drop_barrier, uint32_t spin_limit, void* stream);

/* Training forward that keeps the intermediates of every cell (no reference counterpart: the
 * reference's autograd keeps the vmapped cells' tensors): flb_block_grid_fwd (tick by tick,
 * cuBLAS projections) that also writes, per cell, its LayerNorm outputs, lat_prior, the three
 * tokens, z_l, z_x, q|k|v and the attention output into `saved` (flb_block_grid_saved_bytes()
 * bytes, 16-byte aligned: L * S * 36 * batch * D bf16), which flb_block_grid_bwd_saved reads
 * back instead of recomputing each tick's forward stages; that backward also keeps the
 * gradients that meet the weights there and forms every weight gradient after its tick loop,
 * one GEMM per weight over all layers. */
size_t flb_block_grid_saved_bytes(int64_t L, int64_t S, int64_t batch, int64_t D);
int flb_block_grid_fwd_save(const flb_block_weights* weights, const void* x, void* grids, int64_t L,
                            int64_t S, int64_t batch, int64_t D, int64_t heads, float ln_eps,
                            void* workspace, size_t workspace_bytes, void* saved,
                            size_t saved_bytes, void* stream);

/* Gradient accumulators of flb_block_grid_bwd: float32 stacks shaped like the matching fields
 * of flb_block_weights (w_qkv: [L, 3D, D], v_a: [L, H, D/H]). Gradients are ADDED into them. */
typedef struct flb_block_grads {
  float* ln_lat_w;
  float* ln_lat_b;
  float* ln_fdbk_w;
  float* ln_fdbk_b;
  float* w_prior_lat;
  float* w_prior_fdbk;
  float* w_gate_l;
  float* b_gate_l;
  float* w_gate_x;
  float* b_gate_x;
  float* w_qkv;
  float* w_o;
  float* v_a;
} flb_block_grads;

size_t flb_block_grid_bwd_workspace_bytes(int64_t L, int64_t S, int64_t batch, int64_t D);

/* Backward of flb_block_grid_fwd (training). Replaces the engine's per-tick backward for FLB
 * blocks (execute_backward with the vmapped vjp of the cell, csrc/wavefront_backend.cpp:48-132,
 * wavefront/wavefront_engine.py:200-236). Arguments as for flb_block_grid_fwd, with `grids`
 * the port grids that forward wrote; dgrid0..dgrid3: bf16 [L*S, batch, D] upstream gradients
 * of the four port grids (NULL = zero). dx: float32 [batch, S, D] gradient of x (overwritten).
 * grads: weight-gradient accumulators (added into). Every tick recomputes its forward stages
 * from the saved grids; nothing but the grids is kept from the forward. */
int flb_block_grid_bwd(const flb_block_weights* weights, const void* x, const void* grids,
                       const void* dgrid0, const void* dgrid1, const void* dgrid2,
                       const void* dgrid3, float* dx, const flb_block_grads* grads,
                       int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads,
                       float ln_eps, void* workspace, size_t workspace_bytes, void* stream);

/* flb_block_grid_bwd with the intermediates flb_block_grid_fwd_save kept (same `grids`, weights
 * and x as that forward): each tick reads its cells' intermediates in `saved` in place instead of
 * recomputing the forward stages, and writes the gradients that meet the weights into `saved`
 * (its other planes), from which every weight gradient is formed after the tick loop; `saved`
 * is therefore written. */
int flb_block_grid_bwd_saved(const flb_block_weights* weights, const void* x, const void* grids,
                             const void* dgrid0, const void* dgrid1, const void* dgrid2,
                             const void* dgrid3, float* dx, const flb_block_grads* grads,
                             int64_t L, int64_t S, int64_t batch, int64_t D, int64_t heads,
                             float ln_eps, void* workspace, size_t workspace_bytes,
                             void* saved, size_t saved_bytes, void* stream);

/* Failure-detection check of the grid kernels' bounded dependency waits (no reference
 * counterpart). Runs flb_grid_fwd with the flag of cell (drop_row, drop_col) never released and
 * the flag-wait bound lowered to spin_limit polls: the cells waiting on it give up, record the
 * error word and finish their row, so the call returns FLB_ERR_TIMEOUT (read back
 * synchronously) and the context stays usable. No GPU fault or trap is involved. */
int flb_grid_fwd_drop_flag_test(const void* x, int x_layout, const void* W_l, const void* W_t,
                                const void* U, const float* bias, const void* top, void* h_out,
                                int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                                void* workspace, size_t workspace_bytes, int64_t drop_row,
                                int64_t drop_col, uint32_t spin_limit, void* stream);

/* ------------------------------------------------------------------------------------------
 * Measurement helpers (used by bench.py for the roofline denominators).
 * ------------------------------------------------------------------------------------------ */

/* Times a saturating loop of one instruction class on every SM and returns the measured
 * throughput in operations (elements) per second through *ops_per_s (host pointer).
 * kind: 0 = tanh.approx.f32, 1 = tanh.approx.f16x2 (2 elements/instr), 2 = tanh.approx.bf16x2,
 *       3 = ex2.approx.f32, 4 = FFMA f32, 5 = HFMA2 f16x2 (2 elements/instr),
 *       6 = the attention backward's per-element tanh-grid step in f16x2 (tanh elements),
 *       7 = the same step in f32, 8 = the forward's score step (FADD, tanh, FFMA) in f32.
 * Synchronises the device. scratch: device buffer of >= 4 * 148 * 1024 bytes. */
int flb_microbench(int kind, void* scratch, double* ops_per_s);

/* Known-answer check of the tcgen05 operand layouts (no reference counterpart; a build check).
 * D[128 x n] (f32, row-major) = A[128 x 64] (bf16, row-major) * op(B), where
 * variant 0: B is [n x 64] row-major (D = A B^T, K-major operand, wavefront-cell form);
 * variant 1: B is [64 x n] row-major (D = A B,   MN-major operand, P@V form). n in {64, 128}.
 * *err (device int, caller-zeroed) becomes non-zero if a bounded wait gave up. */
int flb_selftest_umma(int variant, int n, const void* A, const void* B, float* D, int* err,
                      void* stream);

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* FLB_B200_H */
