// Persistent tanh grid cell: the wavefront grid layer as one kernel per direction.
//
//   h[r][c] = tanh(W_l[g] h[r][c-1] + W_t[g] h[r-1][c] + add[r][c] + bias[g]),   g = r or 0
//
// with h[r][-1] = 0, h[-1][c] = top[c] (or 0), add = x[r][c] U^T (one hoisted cuBLAS GEMM).
// This is the cell of the wavefront engine with dependencies ((-1,0), port 0) and
// ((0,-1), port 1) (wavefront/wavefront_api.py:12-14). The reference evaluates it with one host
// tick per anti-diagonal (csrc/wavefront_backend.cpp:16-44: gather launch, vmapped cell, scatter);
// here a single launch advances the whole grid:
//   * one CTA per (grid row, 128 output features); rows are co-resident (grid <= the device's
//     resident-CTA capacity) and a CTA walks its row left to right;
//   * per-cell dependency flags in global memory say when both 128-feature halves of a cell are
//     stored; one thread polls the left and top neighbours' flags together (ld.acquire.gpu, with
//     an iteration bound: on expiry an error word is set and the kernel carries on, so it never
//     hangs) and starts each neighbour's load the moment its flags are set. A cell's two halves'
//     flags are adjacent words read by one 64-bit acquire load: acquires complete one after
//     another, so a poll costs two L2 round trips instead of four (W4 sweep 5% faster);
//   * the neighbours' h ([batch x hidden] bf16 each) arrive by TMA straight from the output grid;
//     coordinates outside the grid (c-1 < 0, r-1 < 0) are zero-filled by the TMA unit, which is
//     exactly the zero boundary;
//   * the cell GEMM, z^T[128 x B] = [W_l | W_t][128 x 2H] . [h_left ; h_top][2H x B], runs on
//     tcgen05 with the CTA's weight slice resident in shared memory and the accumulator in TMEM,
//     the W_l half as soon as h_left has landed;
//   * the epilogue adds bias and the hoisted x U^T (prefetched one cell ahead), applies tanh and
//     stores h (bf16) into the output grid; after a CTA barrier one thread releases the cell's
//     flag (st.release, which is cumulative over the stores the barrier ordered before it).
// The backward is the mirrored reverse sweep producing dz = dh_total * (1 - h^2) with
// dh_total = dh_ext + W_l^T dz[r][c+1] + W_t^T dz[r+1][c]; weight gradients are then plain
// cuBLAS GEMMs over dz and the saved h (and x), and db is reduced inside the sweep.
#include <cublas_v2.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"
#include "blas.cuh"

namespace flb {

namespace {

constexpr uint32_t kWaitLimit = 1u << 22;      // mbarrier polls
constexpr uint32_t kFlagSpinLimit = 1u << 26;  // flag polls (~ seconds with the backoff)

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Both feature halves' flags of a cell (adjacent words, 8-byte aligned) in one acquire load.
__device__ __forceinline__ unsigned long long ld_acquire_b64(const int* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
template <int NH>
__device__ __forceinline__ bool halves_set(const int* f) {
  if constexpr (NH == 2) return ld_acquire_b64(f) == 0x0000000100000001ull;
  else return ld_acquire(f) == 1;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// System scope: flags written by another GPU over NVLink, or written into another GPU's memory.
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool wait_flag_sys(const int* p, int want, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (ld_acquire_sys(p) == want) return true;
    if (i > 64) __nanosleep(128);
  }
  return false;
}
// Shared -> global tile store (no multicast) and its bulk-group completion.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
      "r"(sm100::smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(sm100::smem_u32(dst)),
      "l"(tmap), "r"(sm100::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

constexpr int kGridThreads = 256;  // 8 warps: thread 0 polls, thread 32 issues MMAs, all run the epilogue

template <int H>
struct GridCfg {
  static constexpr int KATOMS = 2 * H / 64;          // 64-element K atoms of [left | top]
  static constexpr int W_ATOM = 128 * 128;            // bytes: 128 rows x 128 B
  static constexpr int OFF_W = 0;
  static constexpr int OFF_IN = KATOMS * W_ATOM;      // B operand atoms follow
  // epilogue operands of a cell, staged by TMA: [B][128] fp32 (add) or 2 x [B][128] bf16 (h, dh)
  __host__ __device__ static int off_ep(int B) { return OFF_IN + KATOMS * B * 128; }
  // one epilogue stage: [B][128] fp32, or [B][128] bf16 h and dh
  __host__ __device__ static int ep_bytes(int B) { return B * 128 * 4; }
  __host__ __device__ static int smem(int B, int stages) {
    return off_ep(B) + stages * ep_bytes(B) + 1024;
  }
  static constexpr int kMaxDynSmem = 226 * 1024;  // under the 227 KB per-block limit with static
  // two stages (the next cell's operands prefetched during this cell) when they fit
  static int ep_stages(int B) { return smem(B, 2) <= kMaxDynSmem ? 2 : 1; }
};

struct GridParams {
  const float* add;      // hoisted x U^T (fp32, [R, C, B, H]) or null
  int ep_stages;         // epilogue operand stages in shared memory (1 or 2)
  const float* bias;     // [G, H] (forward) ; unused in backward
  __nv_bfloat16* out;    // forward: h grid [R, C, B, H]; backward: dz grid [R, C, B, H]
  __nv_bfloat16* out2;   // backward: dz in x layout [B, R, C, H] or null
  const __nv_bfloat16* h;    // backward: forward output h [R, C, B, H]
  const __nv_bfloat16* dh;   // backward: upstream gradient [R, C, B, H]
  float* dbias;          // backward: [G, H] accumulated
  int* flags;            // [R, C, 2]
  int R, C, B, G, has_top, reverse;
  int* err;
  int64_t drop_cell;     // failure-detection check: this cell's flag is never released (-1: none)
  uint32_t spin_limit;   // flag polls before a wait gives up
  // Row bands: this launch is rows row0 .. row0 + R - 1 of a taller grid (weights are indexed by
  // global row), and its edge rows exchange [C, B, H] halos with the neighbouring bands on other
  // GPUs. The in-edge row (forward: row 0, backward: row R - 1) reads its other-row input from the
  // local receive buffer (tmTop) once the neighbour's per-column flags say it landed, then
  // acknowledges; the out-edge row (forward: row R - 1, backward: row 0) also stores its output
  // into the neighbour's receive buffer, after that neighbour acknowledged the previous epoch.
  int row0;
  const int* halo_in_flags;  // local [C][2], set to epoch by the neighbour (null: no in-halo)
  int* halo_in_ack;          // neighbour's [C][2], set to epoch here once a column is loaded
  __nv_bfloat16* halo_out;   // neighbour's receive buffer [C, B, H] (null: no out-halo)
  int* halo_out_flags;       // neighbour's [C][2]
  const int* halo_out_ack;   // local [C][2], the neighbour's acknowledgements
  int epoch;                 // this call's halo epoch (>= 1; the previous call's is epoch - 1)
  int save_top;              // forward: keep the received halo rows through tmSave
};

// One kernel body for both directions. Forward (reverse = 0): rows ascend, cells walk right,
// inputs are h[r][c-1] (left) and h[r-1][c] (top). Backward (reverse = 1): rows descend, cells
// walk left, inputs are dz[r][c+1] and dz[r+1][c], weights are the transposed W_l^T, W_t^T.
template <int H>
__global__ void __launch_bounds__(kGridThreads, 1)
grid_sweep_kernel(const __grid_constant__ CUtensorMap tmWa, const __grid_constant__ CUtensorMap tmWb,
                  const __grid_constant__ CUtensorMap tmIn, const __grid_constant__ CUtensorMap tmTop,
                  const __grid_constant__ CUtensorMap tmE1, const __grid_constant__ CUtensorMap tmE2,
                  const __grid_constant__ CUtensorMap tmSave, GridParams p) {
  using namespace sm100;
  using Cfg = GridCfg<H>;
  constexpr int NH = H / 128;  // feature halves (CTAs per row)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t bar_w, bar_l, bar_t, bar_mma, bar_ep[2];
  __shared__ uint32_t tmem_slot;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int half = blockIdx.x % NH;
  const int worker = blockIdx.x / NH;
  const int nworkers = gridDim.x / NH;
  const int B = p.B;
  const int R = p.R, C = p.C;

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_l, 1);  // same-row input landed
    mbar_init(&bar_t, 1);  // other-row input landed
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_ep[0], 1);
    mbar_init(&bar_ep[1], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmWa);
    tma_prefetch_desc(&tmWb);
    tma_prefetch_desc(&tmIn);
    if (p.has_top) tma_prefetch_desc(&tmTop);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t idesc = make_idesc_f16(128, B, 1, 0, 0);
  const int wq = warp & 3;  // TMEM lane quarter: features 32 wq .. +31 of the half
  const int f = half * 128 + wq * 32 + lane;  // this thread's output feature
  uint32_t n_wload = 0, n_cell = 0;
  uint32_t ep_issued = 0, ep_used = 0;  // epilogue operand tiles issued / consumed (stage = k % S)
  const int S = p.ep_stages;
  float db_acc = 0.f;
  int db_group = -1;

  for (int ri = worker; ri < R; ri += nworkers) {
    const int r = p.reverse ? (R - 1 - ri) : ri;
    const int g = (p.G > 1) ? p.row0 + r : 0;
    // The other-row edge uses the weights of the row that consumes it: forward, cell (r, c)
    // reads h[r-1][c] through its own W_t[r]; backward, dz[r+1][c] flows back through W_t[r+1].
    const int g_other = (p.G > 1 && p.reverse) ? min(p.row0 + r + 1, p.G - 1) : g;
    const bool in_edge = p.reverse ? (r == R - 1) : (r == 0);
    const bool halo_in = in_edge && p.halo_in_flags != nullptr;
    const bool halo_out = (p.reverse ? (r == 0) : (r == R - 1)) && p.halo_out != nullptr;
    if (ri == worker || p.G > 1) {
      if (tid == 0) {
        mbar_arrive_expect_tx(&bar_w, Cfg::KATOMS * Cfg::W_ATOM);
#pragma unroll
        for (int a = 0; a < H / 64; ++a) {
          tma_load_2d(sm + Cfg::OFF_W + a * Cfg::W_ATOM, &tmWa, &bar_w, a * 64, g * H + half * 128);
          tma_load_2d(sm + Cfg::OFF_W + (H / 64 + a) * Cfg::W_ATOM, &tmWb, &bar_w, a * 64,
                      g_other * H + half * 128);
        }
      }
      if (!mbar_wait(&bar_w, n_wload & 1u, kWaitLimit)) atomicExch(p.err, 1);
      ++n_wload;
    }
    // this thread's bias for the row (loaded once per row, off the cells' chain)
    const float bias_f = p.reverse ? 0.f : p.bias[(int64_t)g * H + f];
    if (p.reverse && db_group != g) {  // flush the bias-gradient partial of the previous group
      if (db_group >= 0) atomicAdd(p.dbias + (int64_t)db_group * H + f, db_acc);
      db_acc = 0.f;
      db_group = g;
    }
    for (int ci = 0; ci < C; ++ci) {
      const int c = p.reverse ? (C - 1 - ci) : ci;
      const int c_nb = p.reverse ? c + 1 : c - 1;   // same-row neighbour
      const int r_nb = p.reverse ? r + 1 : r - 1;   // other-row neighbour
      const bool stage_add = !p.reverse && p.add != nullptr;
      if (tid == 0 && (p.reverse || stage_add)) {
        // Epilogue operands do not depend on the recurrence: fetch them before waiting on it,
        // with two stages one cell ahead (a row's first cell fetches its own too).
        auto issue_ep = [&](int cj) {
          const int cc = p.reverse ? (C - 1 - cj) : cj;
          const int st = (int)(ep_issued % (uint32_t)S);
          uint8_t* sE = sm + Cfg::off_ep(B) + st * Cfg::ep_bytes(B);
          if (p.reverse) {
            mbar_arrive_expect_tx(&bar_ep[st], 2 * B * 128 * 2);
            tma_load_4d(sE, &tmE1, &bar_ep[st], half * 128, 0, cc, r);                 // h
            tma_load_4d(sE + B * 128 * 2, &tmE2, &bar_ep[st], half * 128, 0, cc, r);   // dh
          } else {
            mbar_arrive_expect_tx(&bar_ep[st], B * 128 * 4);
            tma_load_4d(sE, &tmE1, &bar_ep[st], half * 128, 0, cc, r);  // add rows (r, c, b)
          }
          ++ep_issued;
        };
        if (S == 1 || ci == 0) issue_ep(ci);
        if (S == 2 && ci + 1 < C) issue_ep(ci + 1);
      }
      if (tid == 0) {
        uint8_t* sIn = sm + Cfg::OFF_IN;
        constexpr int kAtoms = H / 64;
        const uint32_t part = (uint32_t)kAtoms * B * 128;  // bytes of one input tile
        // Each input is loaded as soon as its producer's flags (both feature halves) are set;
        // out-of-grid neighbours are zero-filled by TMA (the zero boundary) without a wait.
        auto issue_left = [&]() {
          fence_async_global();  // order the acquired generic stores before the TMA reads
          mbar_arrive_expect_tx(&bar_l, part);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a)
            tma_load_4d(sIn + a * B * 128, &tmIn, &bar_l, a * 64, 0, c_nb, r);
        };
        auto issue_top = [&]() {
          fence_async_global();
          mbar_arrive_expect_tx(&bar_t, part);
#pragma unroll
          for (int a = 0; a < kAtoms; ++a) {
            if (in_edge && p.has_top)
              tma_load_3d(sIn + (kAtoms + a) * B * 128, &tmTop, &bar_t, a * 64, 0, c);
            else
              tma_load_4d(sIn + (kAtoms + a) * B * 128, &tmIn, &bar_t, a * 64, 0, c, r_nb);
          }
        };
        const bool left_dep = c_nb >= 0 && c_nb < C;
        const bool top_dep = r_nb >= 0 && r_nb < R;
        const int* lflag = p.flags + ((int64_t)r * C + (left_dep ? c_nb : 0)) * 2;
        const int* tflag = p.flags + ((int64_t)(top_dep ? r_nb : 0) * C + c) * 2;
        // the other-row input of a band's edge row is the halo of the neighbouring band
        const int* hflag = halo_in ? p.halo_in_flags + c * 2 : nullptr;
        bool lready = !left_dep, tready = !top_dep && !halo_in;
        if (lready) issue_left();
        if (tready) issue_top();
        for (uint32_t i = 0; !(lready && tready) && i < p.spin_limit; ++i) {
          if (!lready && halves_set<NH>(lflag)) {
            lready = true;
            issue_left();
          }
          // a band's halo flags are polled at system scope, which costs far more per load:
          // only once the same-row input is in
          if (!tready && !(halo_in && !lready)) {
            bool set = true;
            if (halo_in) {
              for (int hh = 0; hh < NH; ++hh) set &= ld_acquire_sys(hflag + hh) == p.epoch;
            } else {
              set = halves_set<NH>(tflag);
            }
            if (set) {
              tready = true;
              issue_top();
            }
          }
          if (i > 64) __nanosleep(64);
        }
        if (!(lready && tready)) {  // gave up: record it, keep the barrier phases in step
          // 2: a same-grid flag never came (an edge row polls its halo only once the same-row
          // input is in, so a same-row timeout must not be reported as a halo timeout); 6: halo
          atomicExch(p.err, (!lready || !halo_in) ? 2 : 6);
          if (!lready) issue_left();
          if (!tready) issue_top();
        }
        if (halo_in) {
          if (!mbar_wait(&bar_t, n_cell & 1u, kWaitLimit)) atomicExch(p.err, 3);
          if (p.save_top) {  // this CTA's feature half of the received rows, back out of shared memory
#pragma unroll
            for (int a = half * 2; a < half * 2 + 2; ++a)
              tma_store_3d(&tmSave, sIn + (kAtoms + a) * B * 128, a * 64, 0, c);
            bulk_commit();
          }
          st_release_sys(p.halo_in_ack + c * 2 + half, p.epoch);
        }
        if (halo_out) {  // the neighbour has loaded the previous epoch's column c: it may be rewritten
          bool ok_ack = true;
          for (int hh = 0; hh < NH; ++hh)
            ok_ack &= wait_flag_sys(p.halo_out_ack + c * 2 + hh, p.epoch - 1, p.spin_limit);
          if (!ok_ack) atomicExch(p.err, 6);
        }
        // the next cell's loads overwrite these rows: the store must have read them by then
        if (halo_in && p.save_top) bulk_wait_read_all();
      } else if (tid == 32) {
        // The MMAs are issued by their own thread (warp 1) so that the same-row half of K runs
        // as soon as its tile has landed, while thread 0 still polls for the other-row input
        // (an M = 128 K-step takes ~120 cycles to issue whatever N is: the same-row half is
        // ~0.6 us at H = 256).
        const uint32_t wa = smem_u32(sm + Cfg::OFF_W), ia = smem_u32(sm + Cfg::OFF_IN);
        auto mma_range = [&](int k0, int k1) {
#pragma unroll
          for (int kk = k0; kk < k1; ++kk) {
            const uint64_t adesc = make_smem_desc(wa + (kk >> 2) * Cfg::W_ATOM + (kk & 3) * 32, 16, 1024, kSwizzle128B);
            const uint64_t bdesc = make_smem_desc(ia + (kk >> 2) * B * 128 + (kk & 3) * 32, 16, 1024, kSwizzle128B);
            umma_f16(tmem, adesc, bdesc, idesc, kk > 0 ? 1u : 0u);
          }
        };
        if (!mbar_wait(&bar_l, n_cell & 1u, kWaitLimit)) atomicExch(p.err, 3);
        tc_fence_after();
        mma_range(0, H / 16);
        if (!mbar_wait(&bar_t, n_cell & 1u, kWaitLimit)) atomicExch(p.err, 3);
        tc_fence_after();
        mma_range(H / 16, 2 * H / 16);
        umma_commit(&bar_mma);
      }
      // a halo wait lasts as long as the other GPU takes to get there (its launch may start late):
      // hold the CTA here, behind thread 0's bounded spins, rather than in the MMA barrier's
      // shorter bounded wait
      if (halo_in || halo_out) __syncthreads();
      __syncwarp();
      if (!mbar_wait(&bar_mma, n_cell & 1u, kWaitLimit)) atomicExch(p.err, 4);
      tc_fence_after();
      ++n_cell;

      // ---- epilogue: this thread owns feature f for every batch element --------------------
      const int64_t cell = (int64_t)r * C + c;
      const uint8_t* sE = sm + Cfg::off_ep(B) + (int)(ep_used % (uint32_t)S) * Cfg::ep_bytes(B);
      const int fl = wq * 32 + lane;  // feature within this CTA's half
      const int cg = warp >> 2;       // column group: batch rows 16 cg .. +15 of each 32
      if (p.reverse || stage_add) {
        if (!mbar_wait(&bar_ep[ep_used % (uint32_t)S], (ep_used / (uint32_t)S) & 1u, kWaitLimit))
          atomicExch(p.err, 5);
        ++ep_used;
      }
      // Eight warps: two per TMEM lane quarter, each with 16 of every 32 batch columns, so that
      // each scheduler has two warps to overlap the per-column chains (shared-memory operand,
      // tanh, convert). All 16 columns' arithmetic first, then the stores.
      for (int cb = 0; cb < B; cb += 32) {
        const int c0 = cb + 16 * cg;           // first batch row of this warp
        const int nb = max(0, min(16, B - c0));
        uint32_t acc[16];
        tmem_ld16(tmem + ((uint32_t)(wq * 32) << 16) + c0, acc);
        tmem_wait_ld();
        __nv_bfloat16 ov[16];
        if (!p.reverse) {
          const float* sEf = reinterpret_cast<const float*>(sE);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float a = (stage_add && j < nb) ? sEf[(c0 + j) * 128 + fl] : 0.f;
            ov[j] = __float2bfloat16_rn(tanh_approx(__uint_as_float(acc[j]) + bias_f + a));
          }
        } else {
          const __nv_bfloat16* sH = reinterpret_cast<const __nv_bfloat16*>(sE);
          const __nv_bfloat16* sD = reinterpret_cast<const __nv_bfloat16*>(sE + B * 128 * 2);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float dz = 0.f;
            if (j < nb) {
              const float hv = __bfloat162float(sH[(c0 + j) * 128 + fl]);
              const float dhv = __bfloat162float(sD[(c0 + j) * 128 + fl]);
              dz = (__uint_as_float(acc[j]) + dhv) * (1.f - hv * hv);
            }
            ov[j] = __float2bfloat16_rn(dz);
            db_acc += dz;  // zero past nb: the sum over the batch is unchanged
          }
        }
        // Out through shared memory: the warp's 16 x 32 tile (batch rows x features) is written
        // into this cell's operand stage, whose contents every warp has read by the barrier, and
        // leaves as 16-byte row chunks (2 stores per thread instead of 16 two-byte ones).
        __syncthreads();
        __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(const_cast<uint8_t*>(sE)) + warp * 512;
#pragma unroll
        for (int j = 0; j < 16; ++j) stg[j * 32 + lane] = ov[j];
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int row = (lane >> 2) + 8 * i, ch = lane & 3;
          if (row < nb) {
            const uint4 v = *reinterpret_cast<const uint4*>(stg + row * 32 + ch * 8);
            const int b = c0 + row;
            const int fo = half * 128 + wq * 32 + ch * 8;
            *reinterpret_cast<uint4*>(p.out + (cell * B + b) * H + fo) = v;
            if (halo_out) *reinterpret_cast<uint4*>(p.halo_out + ((int64_t)c * B + b) * H + fo) = v;
            if (p.reverse && p.out2)
              *reinterpret_cast<uint4*>(p.out2 + (((int64_t)b * R + r) * C + c) * H + fo) = v;
          }
        }
        fence_async_shared();  // a later TMA load overwrites this stage
        __syncwarp();
      }
      tc_fence_before();
      __syncthreads();
      // The barrier orders every thread's stores of this cell before thread 0's release, and a
      // release is cumulative: consumers that acquire the flag see all of them.
      if (tid == 0 && cell != p.drop_cell) {
        st_release(p.flags + cell * 2 + half, 1);
        if (halo_out) {  // the halo stores reach the other GPU before its flag
          __threadfence_system();
          st_release_sys(p.halo_out_flags + c * 2 + half, p.epoch);
        }
      }
    }
  }
  if (p.reverse && db_group >= 0) atomicAdd(p.dbias + (int64_t)db_group * H + f, db_acc);
  if (tid == 0 && p.save_top && p.halo_in_flags != nullptr) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

__global__ void transpose_weights_kernel(const __nv_bfloat16* __restrict__ W,
                                         __nv_bfloat16* __restrict__ WT, int G, int H) {
  // WT[g][i][o] = W[g][o][i]
  __shared__ __nv_bfloat16 tile[32][33];
  const int g = blockIdx.z;
  const int o0 = blockIdx.y * 32, i0 = blockIdx.x * 32;
  const __nv_bfloat16* src = W + (int64_t)g * H * H;
  __nv_bfloat16* dst = WT + (int64_t)g * H * H;
  for (int y = threadIdx.y; y < 32; y += blockDim.y)
    tile[y][threadIdx.x] = src[(int64_t)(o0 + y) * H + i0 + threadIdx.x];
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y)
    dst[(int64_t)(i0 + y) * H + o0 + threadIdx.x] = tile[threadIdx.x][y];
}

__global__ void sum_rows_kernel(const float* __restrict__ src, float* __restrict__ dst, int R,
                                int64_t n, int first) {
  // dst[e] = sum_{r >= first} src[r][e]
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  float s = 0.f;
  for (int r = first; r < R; ++r) s += src[(int64_t)r * n + e];
  dst[e] = s;
}

// ---- workspace layout ------------------------------------------------------------------------------
constexpr size_t kBlasWs = 32u << 20;
struct GridWs {
  int* err;       // 256 B
  int* flags;     // R*C*2 ints
  float* add;     // hoisted U x, [R*C*B, H] fp32 (only with U)
  __nv_bfloat16* dz;    // [R, C, B, H]
  __nv_bfloat16* dzx;   // [B, R, C, H] (only with U and x_layout 0)
  __nv_bfloat16* wt;    // transposed W_l, W_t: 2 x [G, H, H]
  float* wtmp;    // [R, H, H] per-row weight-gradient partials
  void* blas;     // cuBLAS workspace
  size_t total;
};

size_t al(size_t x) { return (x + 255) & ~(size_t)255; }

GridWs carve(void* base, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G, int has_U) {
  GridWs w{};
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  size_t o = 0;
  auto take = [&](size_t n) { uint8_t* q = p ? p + o : nullptr; o += al(n); return q; };
  const size_t cells = (size_t)(R * C);
  w.err = (int*)take(256);
  w.flags = (int*)take(cells * 2 * sizeof(int));
  w.add = has_U ? (float*)take(cells * B * H * sizeof(float)) : nullptr;
  w.dz = (__nv_bfloat16*)take(cells * B * H * 2);
  w.dzx = has_U ? (__nv_bfloat16*)take(cells * B * H * 2) : nullptr;
  w.wt = (__nv_bfloat16*)take((size_t)2 * G * H * H * 2);
  w.wtmp = (float*)take((size_t)R * H * H * sizeof(float));
  w.blas = take(kBlasWs);
  w.total = o;
  return w;
}

int make_w_map(CUtensorMap* m, const void* W, int64_t G, int64_t H) {
  const uint64_t dims[2] = {(uint64_t)H, (uint64_t)(G * H)};
  const uint64_t strides[1] = {(uint64_t)H * 2};
  const uint32_t box[2] = {64, 128};
  return make_tmap(m, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}
int make_grid_map(CUtensorMap* m, const void* X, int64_t R, int64_t C, int64_t B, int64_t H) {
  const uint64_t dims[4] = {(uint64_t)H, (uint64_t)B, (uint64_t)C, (uint64_t)R};
  const uint64_t strides[3] = {(uint64_t)H * 2, (uint64_t)(B * H * 2), (uint64_t)(C * B * H * 2)};
  const uint32_t box[4] = {64, (uint32_t)B, 1, 1};
  return make_tmap(m, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}
int make_top_map(CUtensorMap* m, const void* T, int64_t C, int64_t B, int64_t H) {
  const uint64_t dims[3] = {(uint64_t)H, (uint64_t)B, (uint64_t)C};
  const uint64_t strides[2] = {(uint64_t)H * 2, (uint64_t)(B * H * 2)};
  const uint32_t box[3] = {64, (uint32_t)B, 1};
  return make_tmap(m, T, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// Epilogue staging maps: a cell's [B x 128] slice of a [R, C, B, H] grid (bf16 or fp32).
int make_ep_map(CUtensorMap* m, const void* X, CUtensorMapDataType dt, int esz, int64_t R,
                int64_t C, int64_t B, int64_t H) {
  const uint64_t dims[4] = {(uint64_t)H, (uint64_t)B, (uint64_t)C, (uint64_t)R};
  const uint64_t strides[3] = {(uint64_t)H * esz, (uint64_t)(B * H * esz), (uint64_t)(C * B * H * esz)};
  const uint32_t box[4] = {128, (uint32_t)B, 1, 1};
  return make_tmap(m, X, dt, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int H>
int launch_sweep(const CUtensorMap& wa, const CUtensorMap& wb, const CUtensorMap& in,
                 const CUtensorMap& top, const CUtensorMap& e1, const CUtensorMap& e2,
                 const CUtensorMap& save, const GridParams& p, cudaStream_t s, int* grid_ctas) {
  const int smem = GridCfg<H>::smem(p.B, p.ep_stages);
  int st = ensure_dyn_smem((const void*)grid_sweep_kernel<H>, GridCfg<H>::kMaxDynSmem,
                           "grid_sweep smem attribute");
  if (st != FLB_OK) return st;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grid_sweep_kernel<H>, kGridThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return fail(FLB_ERR_LAUNCH, "grid_sweep: kernel does not fit on an SM");
  constexpr int NH = H / 128;
  // every CTA must be resident at once (they wait on one another): cap the workers
  const int capacity = per_sm * num_sms();
  int workers = std::min<int>(p.R, capacity / NH);
  if (workers < 1) return fail(FLB_ERR_LAUNCH, "grid_sweep: not enough resident CTAs");
  *grid_ctas = workers * NH;
  grid_sweep_kernel<H><<<workers * NH, kGridThreads, smem, s>>>(wa, wb, in, top, e1, e2, save, p);
  count_launches(1);
  return check_cuda(cudaGetLastError(), "grid_sweep launch");
}

int check_grid_args(int64_t R, int64_t C, int64_t B, int64_t H, int64_t G) {
  if (R < 1 || C < 1) return fail(FLB_ERR_SHAPE, "grid: R and C must be >= 1");
  if (!(H == 128 || H == 256)) return fail(FLB_ERR_UNSUPPORTED, "grid: hidden must be 128 or 256");
  if (B < 16 || B > 64 || B % 16 != 0) return fail(FLB_ERR_UNSUPPORTED, "grid: batch must be 16, 32, 48 or 64");
  if (!(G == 1 || G == R)) return fail(FLB_ERR_SHAPE, "grid: G must be 1 (shared) or R (per row)");
  if (R * C > (int64_t)1 << 26) return fail(FLB_ERR_SHAPE, "grid: too many cells");
  return FLB_OK;
}

int read_err(const int* err, cudaStream_t s, const char* what) {
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return check_cuda(e, what);
  if (h != 0) return fail(FLB_ERR_TIMEOUT, std::string(what) + ": a bounded device wait gave up (code " + std::to_string(h) + ")");
  return FLB_OK;
}

// A rank's receive block for row bands (in its own memory, mapped into its neighbours):
// [fwd halo C*B*H bf16][bwd halo C*B*H bf16][fwd flags C*2][bwd flags C*2][fwd acks C*2]
// [bwd acks C*2] (int32), each part 256-byte aligned. The forward halo is written by the band
// above (its last row), the backward halo by the band below (its first row's dz); acks are
// written by the band that consumed this rank's outgoing halo.
struct BandBlock {
  __nv_bfloat16 *fwd_halo, *bwd_halo;
  int *fwd_flags, *bwd_flags, *fwd_acks, *bwd_acks;
  size_t total;
};
BandBlock band_block(void* base, int64_t C, int64_t B, int64_t H) {
  BandBlock k{};
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  size_t o = 0;
  auto take = [&](size_t n) { uint8_t* q = p ? p + o : nullptr; o += al(n); return q; };
  k.fwd_halo = (__nv_bfloat16*)take((size_t)(C * B * H) * 2);
  k.bwd_halo = (__nv_bfloat16*)take((size_t)(C * B * H) * 2);
  k.fwd_flags = (int*)take((size_t)C * 2 * sizeof(int));
  k.bwd_flags = (int*)take((size_t)C * 2 * sizeof(int));
  k.fwd_acks = (int*)take((size_t)C * 2 * sizeof(int));
  k.bwd_acks = (int*)take((size_t)C * 2 * sizeof(int));
  k.total = o;
  return k;
}

int check_band(const flb_grid_band* band, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G) {
  if (!band) return check_grid_args(R, C, B, H, G);
  int st = check_grid_args(R, C, B, H, 1);
  if (st != FLB_OK) return st;
  const int64_t T = band->rows_total;
  if (band->row0 < 0 || R < 1 || band->row0 + R > T || T > (int64_t)1 << 20)
    return fail(FLB_ERR_SHAPE, "grid band: rows row0 .. row0 + R - 1 must lie in 0 .. rows_total - 1");
  if (!(G == 1 || G == T)) return fail(FLB_ERR_SHAPE, "grid band: G must be 1 or rows_total");
  if (!band->own_block) return fail(FLB_ERR_SHAPE, "grid band: null own_block");
  if ((band->up_block == nullptr) != (band->row0 == 0))
    return fail(FLB_ERR_SHAPE, "grid band: up_block must be given exactly when row0 > 0");
  if ((band->down_block == nullptr) != (band->row0 + R == T))
    return fail(FLB_ERR_SHAPE, "grid band: down_block must be given exactly when rows follow this band");
  if (band->epoch < 1) return fail(FLB_ERR_SHAPE, "grid band: epoch must be >= 1");
  return FLB_OK;
}

}  // namespace

size_t grid_band_block_bytes(int64_t C, int64_t B, int64_t H) {
  return band_block(nullptr, C, B, H).total;
}

size_t grid_workspace_bytes(int64_t R, int64_t C, int64_t B, int64_t H, int64_t G, int has_U) {
  return carve(nullptr, R, C, B, H, G, has_U).total;
}

int grid_fwd_impl(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const float* bias, const void* top, void* h_out, int64_t R, int64_t C,
                  int64_t B, int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout,
                  cudaStream_t s, int64_t drop_cell, uint32_t spin_limit,
                  const flb_grid_band* band, void* saved_top) {
  int st = check_band(band, R, C, B, H, G);
  if (st != FLB_OK) return st;
  if (!W_l || !W_t || !bias || !h_out || (U && !x)) return fail(FLB_ERR_SHAPE, "grid_fwd: null pointer");
  const bool from_up = band && band->up_block;
  if (from_up && (top || !saved_top))
    return fail(FLB_ERR_SHAPE, "grid band fwd: below the first band, top must be NULL and saved_top given");
  BandBlock own{}, up{}, down{};
  if (band) {
    own = band_block(band->own_block, C, B, H);
    if (band->up_block) up = band_block(band->up_block, C, B, H);
    if (band->down_block) down = band_block(band->down_block, C, B, H);
  }
  GridWs w = carve(ws, R, C, B, H, G, U != nullptr);
  if (!ws || ws_bytes < w.total) return fail(FLB_ERR_WORKSPACE, "grid_fwd: workspace smaller than flb_grid_workspace_bytes()");
  cudaError_t e = cudaMemsetAsync(w.err, 0, 256, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(w.flags, 0, (size_t)R * C * 2 * sizeof(int), s);
  if (e != cudaSuccess) return check_cuda(e, "grid_fwd memset");
  if (U) {  // add = x U^T, always in the grid's [R, C, B, H] order (a cell's rows contiguous)
    cublasHandle_t h;
    if ((st = blas(s, w.blas, kBlasWs, &h)) != FLB_OK) return st;
    if (x_layout == 1)
      st = gemm_rm(h, false, true, (int)(R * C * B), (int)H, (int)H, x, (int)H, 0, U, (int)H, 0,
                   w.add, (int)H, 0, 1, 0.f);
    else  // x [B, R, C, H]: one batch per b, its R*C rows written with a pitch of B rows
      st = gemm_rm(h, false, true, (int)(R * C), (int)H, (int)H, x, (int)H, (long long)(R * C * H),
                   U, (int)H, 0, w.add, (int)(B * H), (long long)H, (int)B, 0.f);
    if (st != FLB_OK) return st;
  }
  CUtensorMap mWl, mWt, mIn, mTop;
  if ((st = make_w_map(&mWl, W_l, G, H)) != FLB_OK) return st;
  if ((st = make_w_map(&mWt, W_t, G, H)) != FLB_OK) return st;
  if ((st = make_grid_map(&mIn, h_out, R, C, B, H)) != FLB_OK) return st;
  const void* top_src = from_up ? (const void*)own.fwd_halo : top;
  if (top_src) {
    if ((st = make_top_map(&mTop, top_src, C, B, H)) != FLB_OK) return st;
  } else {
    mTop = mIn;
  }
  CUtensorMap mSave = mIn;
  if (from_up && (st = make_top_map(&mSave, saved_top, C, B, H)) != FLB_OK) return st;
  CUtensorMap mAdd = mIn;
  if (U && (st = make_ep_map(&mAdd, w.add, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, R, C, B, H)) != FLB_OK)
    return st;
  GridParams p{};
  p.add = U ? w.add : nullptr;
  p.ep_stages = H == 256 ? GridCfg<256>::ep_stages((int)B) : GridCfg<128>::ep_stages((int)B);
  p.bias = bias;
  p.out = (__nv_bfloat16*)h_out;
  p.flags = w.flags;
  p.R = (int)R; p.C = (int)C; p.B = (int)B; p.G = (int)G;
  p.has_top = top_src != nullptr;
  p.reverse = 0;
  p.err = w.err;
  p.drop_cell = drop_cell;
  p.spin_limit = spin_limit;
  if (band) {
    p.row0 = (int)band->row0;
    p.epoch = band->epoch;
    if (from_up) {
      p.halo_in_flags = own.fwd_flags;
      p.halo_in_ack = up.fwd_acks;
      p.save_top = 1;
    }
    if (band->down_block) {
      p.halo_out = down.fwd_halo;
      p.halo_out_flags = down.fwd_flags;
      p.halo_out_ack = own.fwd_acks;
    }
  }
  int ctas = 0;
  st = H == 256 ? launch_sweep<256>(mWl, mWt, mIn, mTop, mAdd, mAdd, mSave, p, s, &ctas)
                : launch_sweep<128>(mWl, mWt, mIn, mTop, mAdd, mAdd, mSave, p, s, &ctas);
  if (st != FLB_OK) return st;
  return check_timeout ? read_err(w.err, s, "grid_fwd") : FLB_OK;
}

int grid_fwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
             const float* bias, const void* top, void* h_out, int64_t R, int64_t C, int64_t B,
             int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout, cudaStream_t s) {
  return grid_fwd_impl(x, x_layout, W_l, W_t, U, bias, top, h_out, R, C, B, H, G, ws, ws_bytes,
                       check_timeout, s, -1, kFlagSpinLimit, nullptr, nullptr);
}

int grid_band_fwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const float* bias, const void* top, void* h_out, void* saved_top, int64_t R,
                  int64_t C, int64_t B, int64_t H, int64_t G, const flb_grid_band* band, void* ws,
                  size_t ws_bytes, int check_timeout, cudaStream_t s) {
  if (!band) return fail(FLB_ERR_SHAPE, "grid_band_fwd: null band");
  return grid_fwd_impl(x, x_layout, W_l, W_t, U, bias, top, h_out, R, C, B, H, G, ws, ws_bytes,
                       check_timeout, s, -1, kFlagSpinLimit, band, saved_top);
}

int grid_bwd_impl(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const void* top, const void* h_out, const void* dh, float* dW_l, float* dW_t,
                  float* dU, float* dbias, void* dx, void* dtop, int64_t R, int64_t C, int64_t B,
                  int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout,
                  cudaStream_t s, const flb_grid_band* band) {
  int st = check_band(band, R, C, B, H, G);
  if (st != FLB_OK) return st;
  if (!W_l || !W_t || !h_out || !dh || !dW_l || !dW_t || !dbias || (U && (!x || !dU)))
    return fail(FLB_ERR_SHAPE, "grid_bwd: null pointer");
  if (band && band->up_block && dtop)
    return fail(FLB_ERR_SHAPE, "grid band bwd: dtop exists only for the first band");
  BandBlock own{}, up{}, down{};
  if (band) {
    own = band_block(band->own_block, C, B, H);
    if (band->up_block) up = band_block(band->up_block, C, B, H);
    if (band->down_block) down = band_block(band->down_block, C, B, H);
  }
  const int64_t row0 = band ? band->row0 : 0;
  GridWs w = carve(ws, R, C, B, H, G, U != nullptr);
  if (!ws || ws_bytes < w.total) return fail(FLB_ERR_WORKSPACE, "grid_bwd: workspace smaller than flb_grid_workspace_bytes()");
  cudaError_t e = cudaMemsetAsync(w.err, 0, 256, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(w.flags, 0, (size_t)R * C * 2 * sizeof(int), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dbias, 0, (size_t)G * H * sizeof(float), s);
  if (e == cudaSuccess && G > 1 && G != R) {  // per-row weights of a band: other bands' rows are 0
    e = cudaMemsetAsync(dW_l, 0, (size_t)G * H * H * sizeof(float), s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dW_t, 0, (size_t)G * H * H * sizeof(float), s);
  }
  if (e != cudaSuccess) return check_cuda(e, "grid_bwd memset");
  // transposed weights: A operand rows are input features
  __nv_bfloat16* WlT = w.wt;
  __nv_bfloat16* WtT = w.wt + G * H * H;
  dim3 tg((unsigned)(H / 32), (unsigned)(H / 32), (unsigned)G), tb(32, 8);
  transpose_weights_kernel<<<tg, tb, 0, s>>>((const __nv_bfloat16*)W_l, WlT, (int)G, (int)H);
  transpose_weights_kernel<<<tg, tb, 0, s>>>((const __nv_bfloat16*)W_t, WtT, (int)G, (int)H);
  count_launches(2);
  CUtensorMap mWl, mWt, mIn, mBelow;
  if ((st = make_w_map(&mWl, WlT, G, H)) != FLB_OK) return st;
  if ((st = make_w_map(&mWt, WtT, G, H)) != FLB_OK) return st;
  if ((st = make_grid_map(&mIn, w.dz, R, C, B, H)) != FLB_OK) return st;
  const bool from_down = band && band->down_block;
  mBelow = mIn;
  if (from_down && (st = make_top_map(&mBelow, own.bwd_halo, C, B, H)) != FLB_OK) return st;
  GridParams p{};
  p.out = w.dz;
  p.out2 = (U && x_layout == 0) ? w.dzx : nullptr;
  p.h = (const __nv_bfloat16*)h_out;
  p.dh = (const __nv_bfloat16*)dh;
  p.dbias = dbias;
  p.flags = w.flags;
  p.R = (int)R; p.C = (int)C; p.B = (int)B; p.G = (int)G;
  p.has_top = from_down ? 1 : 0;  // the last row's row below: the halo from the next band
  p.reverse = 1;
  p.ep_stages = H == 256 ? GridCfg<256>::ep_stages((int)B) : GridCfg<128>::ep_stages((int)B);
  p.err = w.err;
  p.drop_cell = -1;
  p.spin_limit = kFlagSpinLimit;
  if (band) {
    p.row0 = (int)row0;
    p.epoch = band->epoch;
    if (from_down) {
      p.halo_in_flags = own.bwd_flags;
      p.halo_in_ack = down.bwd_acks;
    }
    if (band->up_block) {
      p.halo_out = up.bwd_halo;
      p.halo_out_flags = up.bwd_flags;
      p.halo_out_ack = own.bwd_acks;
    }
  }
  int ctas = 0;
  CUtensorMap mH, mDH;
  if ((st = make_ep_map(&mH, h_out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, C, B, H)) != FLB_OK) return st;
  if ((st = make_ep_map(&mDH, dh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, R, C, B, H)) != FLB_OK) return st;
  st = H == 256 ? launch_sweep<256>(mWl, mWt, mIn, mBelow, mH, mDH, mIn, p, s, &ctas)
                : launch_sweep<128>(mWl, mWt, mIn, mBelow, mH, mDH, mIn, p, s, &ctas);
  if (st != FLB_OK) return st;

  cublasHandle_t hb;
  if ((st = blas(s, w.blas, kBlasWs, &hb)) != FLB_OK) return st;
  const int Hi = (int)H;
  const long long cellHB = (long long)B * H;         // elements per cell
  const long long rowHB = (long long)C * cellHB;     // elements per grid row
  const __nv_bfloat16* hh = (const __nv_bfloat16*)h_out;
  float* tmp = w.wtmp;
  // dW_l[r] = sum_{c>=1, b} dz[r][c][b][:]^T h[r][c-1][b][:]  (per row, K = (C-1) B)
  if (C > 1) {
    float* dst = (G > 1) ? dW_l + row0 * H * H : tmp;
    st = gemm_rm(hb, true, false, Hi, Hi, (int)((C - 1) * B), w.dz + cellHB, Hi, rowHB, hh, Hi,
                 rowHB, dst, Hi, (long long)H * H, (int)R, 0.f);
    if (st != FLB_OK) return st;
    if (G == 1) {
      sum_rows_kernel<<<(unsigned)((H * H + 255) / 256), 256, 0, s>>>(tmp, dW_l, (int)R, H * H, 0);
      count_launches(1);
    }
  } else {
    e = cudaMemsetAsync(dW_l, 0, (size_t)G * H * H * sizeof(float), s);
    if (e != cudaSuccess) return check_cuda(e, "grid_bwd memset dW_l");
  }
  // dW_t[r] = sum_{c, b} dz[r][c]^T h[r-1][c]  (r >= 1), and dz[0]^T top for r = 0 (for a band
  // below the first, top is the band above's last row as received in the forward)
  {
    float* dst = (G > 1) ? dW_t + row0 * H * H : tmp;
    if (R > 1) {
      st = gemm_rm(hb, true, false, Hi, Hi, (int)(C * B), w.dz + rowHB, Hi, rowHB, hh, Hi, rowHB,
                   dst + (long long)H * H, Hi, (long long)H * H, (int)(R - 1), 0.f);
      if (st != FLB_OK) return st;
    }
    if (top) {
      st = gemm_rm(hb, true, false, Hi, Hi, (int)(C * B), w.dz, Hi, 0, top, Hi, 0, dst, Hi, 0, 1, 0.f);
    } else {
      e = cudaMemsetAsync(dst, 0, (size_t)H * H * sizeof(float), s);
      st = check_cuda(e, "grid_bwd memset dW_t row 0");
    }
    if (st != FLB_OK) return st;
    if (G == 1) {
      sum_rows_kernel<<<(unsigned)((H * H + 255) / 256), 256, 0, s>>>(tmp, dW_t, (int)R, H * H, 0);
      count_launches(1);
    }
  }
  if (U) {
    const __nv_bfloat16* dzx = (x_layout == 0) ? w.dzx : w.dz;
    const int M = (int)(R * C * B);
    // dU = dz^T x ; dx = dz U
    st = gemm_rm(hb, true, false, Hi, Hi, M, dzx, Hi, 0, x, Hi, 0, dU, Hi, 0, 1, 0.f);
    if (st != FLB_OK) return st;
    if (dx) {
      st = gemm_rm(hb, false, false, M, Hi, Hi, dzx, Hi, 0, U, Hi, 0, (float*)dx, Hi, 0, 1, 0.f,
                   CUDA_R_16BF);
      if (st != FLB_OK) return st;
    }
  }
  if (top && dtop) {  // dtop[c] = dz[0][c] W_t[0]
    st = gemm_rm(hb, false, false, (int)(C * B), Hi, Hi, w.dz, Hi, 0, W_t, Hi, 0, (float*)dtop, Hi,
                 0, 1, 0.f, CUDA_R_16BF);
    if (st != FLB_OK) return st;
  }
  return check_timeout ? read_err(w.err, s, "grid_bwd") : FLB_OK;
}

int grid_bwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
             const void* top, const void* h_out, const void* dh, float* dW_l, float* dW_t,
             float* dU, float* dbias, void* dx, void* dtop, int64_t R, int64_t C, int64_t B,
             int64_t H, int64_t G, void* ws, size_t ws_bytes, int check_timeout, cudaStream_t s) {
  return grid_bwd_impl(x, x_layout, W_l, W_t, U, top, h_out, dh, dW_l, dW_t, dU, dbias, dx, dtop,
                       R, C, B, H, G, ws, ws_bytes, check_timeout, s, nullptr);
}

int grid_band_bwd(const void* x, int x_layout, const void* W_l, const void* W_t, const void* U,
                  const void* top, const void* h_out, const void* dh, float* dW_l, float* dW_t,
                  float* dU, float* dbias, void* dx, void* dtop, int64_t R, int64_t C, int64_t B,
                  int64_t H, int64_t G, const flb_grid_band* band, void* ws, size_t ws_bytes,
                  int check_timeout, cudaStream_t s) {
  if (!band) return fail(FLB_ERR_SHAPE, "grid_band_bwd: null band");
  return grid_bwd_impl(x, x_layout, W_l, W_t, U, top, h_out, dh, dW_l, dW_t, dU, dbias, dx, dtop,
                       R, C, B, H, G, ws, ws_bytes, check_timeout, s, band);
}

// ---- device memory shared with the other ranks of a node (CUDA IPC) ----------------------------
// The exported handle is CUDA's 64-byte IPC handle followed by the owning GPU's 16-byte UUID.
constexpr size_t kIpcCudaBytes = sizeof(cudaIpcMemHandle_t);
static_assert(kIpcCudaBytes + 16 == FLB_IPC_HANDLE_BYTES, "handle layout");

int current_uuid(unsigned char out[16]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  cudaDeviceProp prop{};
  if (e == cudaSuccess) e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) return check_cuda(e, "ipc: device properties");
  memcpy(out, prop.uuid.bytes, 16);
  return FLB_OK;
}

int ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  if (!dev_ptr || !handle || bytes == 0) return fail(FLB_ERR_SHAPE, "ipc_alloc: null pointer or zero size");
  unsigned char* out = static_cast<unsigned char*>(handle);
  int st = current_uuid(out + kIpcCudaBytes);
  if (st != FLB_OK) return st;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return check_cuda(e, "ipc_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);  // flags and epochs start at 0
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(out), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return check_cuda(e, "ipc_alloc: export");
  }
  *dev_ptr = p;
  return FLB_OK;
}

int ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return fail(FLB_ERR_SHAPE, "ipc_open: null pointer");
  const unsigned char* in = static_cast<const unsigned char*>(handle);
  // kernels on the two sides wait on each other: they must run on different GPUs
  unsigned char mine[16];
  int st = current_uuid(mine);
  if (st != FLB_OK) return st;
  if (memcmp(mine, in + kIpcCudaBytes, 16) == 0)
    return fail(FLB_ERR_UNSUPPORTED, "ipc_open: the allocation lives on this GPU; row bands need one GPU per rank");
  cudaIpcMemHandle_t h;
  memcpy(&h, in, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return check_cuda(e, "ipc_open: cudaIpcOpenMemHandle");
  *dev_ptr = p;
  return FLB_OK;
}

int ipc_close(void* dev_ptr) {
  return check_cuda(cudaIpcCloseMemHandle(dev_ptr), "ipc_close");
}

int ipc_free(void* dev_ptr) { return check_cuda(cudaFree(dev_ptr), "ipc_free"); }

// =============================================================================================
// Allocation-free grid forward.
//
// Some callers cannot allocate device memory at the moment they run this layer: a serving process
// that carved all of its device memory into a fixed pool up front, code running inside another
// runtime's allocator, or a call site that must not touch the CUDA allocator at all. For them
// flb_grid_fwd_static takes no workspace: its scratch (the error word and the per-cell dependency
// flags) lives in the file-scope array below, sized for at most kStaticMaxCells grid cells. The
// array belongs to the library's module on every device that loads it (512 KB + 256 B) and stays
// there until the process exits. Calls share it: each call clears the part it uses before its
// kernel runs, and two calls whose kernels overlap on the GPU (different streams, no ordering
// between them) would race on the flags, so such calls must be ordered. On the first call on a
// device the host looks the array's device address up (cudaGetSymbolAddress, with that device
// current) and caches it; make that first call before any stream capture.
// =============================================================================================
constexpr int64_t kStaticMaxCells = 65536;
constexpr int kStaticErrInts = 64;  // 256 bytes, the error word and padding
static __device__ __align__(256) int g_grid_static_scratch[kStaticErrInts + kStaticMaxCells * 2];

int grid_fwd_static(const void* W_l, const void* W_t, const float* bias, const void* top,
                    void* h_out, int64_t R, int64_t C, int64_t B, int64_t H, int64_t G,
                    int check_timeout, cudaStream_t s) {
  int st = check_grid_args(R, C, B, H, G);
  if (st != FLB_OK) return st;
  if (!W_l || !W_t || !bias || !h_out) return fail(FLB_ERR_SHAPE, "grid_fwd_static: null pointer");
  if (R * C > kStaticMaxCells)
    return fail(FLB_ERR_SHAPE, "grid_fwd_static: " + std::to_string(R * C) +
                                   " cells exceed the static scratch limit of " +
                                   std::to_string(kStaticMaxCells) +
                                   " cells; use flb_grid_fwd with a workspace");
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static int* dev_ptr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "grid_fwd_static: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FLB_ERR_UNSUPPORTED, "grid_fwd_static: device index too large");
  int* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_grid_static_scratch);
      if (e != cudaSuccess) return check_cuda(e, "grid_fwd_static: cudaGetSymbolAddress");
      dev_ptr[dev] = static_cast<int*>(p);
    }
    base = dev_ptr[dev];
  }
  int* err = base;
  int* flags = base + kStaticErrInts;
  // the previous call left its flags and error word behind: clear what this call reads
  e = cudaMemsetAsync(err, 0, kStaticErrInts * sizeof(int), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(flags, 0, (size_t)R * C * 2 * sizeof(int), s);
  if (e != cudaSuccess) return check_cuda(e, "grid_fwd_static: clear scratch");
  CUtensorMap mWl, mWt, mIn, mTop;
  if ((st = make_w_map(&mWl, W_l, G, H)) != FLB_OK) return st;
  if ((st = make_w_map(&mWt, W_t, G, H)) != FLB_OK) return st;
  if ((st = make_grid_map(&mIn, h_out, R, C, B, H)) != FLB_OK) return st;
  if (top) {
    if ((st = make_top_map(&mTop, top, C, B, H)) != FLB_OK) return st;
  } else {
    mTop = mIn;
  }
  GridParams p{};
  p.add = nullptr;
  p.ep_stages = 1;
  p.bias = bias;
  p.out = (__nv_bfloat16*)h_out;
  p.flags = flags;
  p.R = (int)R; p.C = (int)C; p.B = (int)B; p.G = (int)G;
  p.has_top = top != nullptr;
  p.reverse = 0;
  p.err = err;
  p.drop_cell = -1;
  p.spin_limit = kFlagSpinLimit;
  int ctas = 0;
  st = H == 256 ? launch_sweep<256>(mWl, mWt, mIn, mTop, mIn, mIn, mIn, p, s, &ctas)
                : launch_sweep<128>(mWl, mWt, mIn, mTop, mIn, mIn, mIn, p, s, &ctas);
  if (st != FLB_OK) return st;
  return check_timeout ? read_err(err, s, "grid_fwd_static") : FLB_OK;
}

}  // namespace flb
