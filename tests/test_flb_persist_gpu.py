"""The persistent native forward of the FLB block grid (one cooperative launch evaluates every
tick: tcgen05 projections, grid barriers between a tick's stages) on a B200:
  * against the reference FLB_Transformer in float32 at batch 16, d_model 128 (golden made by
    running the reference, weights regenerated from a seed): logits and aux within the bf16
    tolerance 2e-2 of the largest magnitude;
  * against the tick-by-tick native path (own kernels + cuBLAS) on the same weights, every port
    grid, at several (layers, positions, d_model, heads), including the end-to-end configuration's
    cell (d_model 768, 12 heads) and more cells per tick than SMs can take in one round;
  * bit-for-bit repeatable (the tiles' K order is fixed, no atomics on data);
  * its error word clear after a run, and its grid barriers' failure detection: a CTA that never
    arrives makes the others give up (FLB_ERR_TIMEOUT), and the next run is correct.
"""
from __future__ import annotations

import ctypes
import os
import sys

import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))

from flb_weights import set_hashed_weights  # noqa: E402

pytestmark = pytest.mark.gpu

PATH_AUTO, PATH_TICKS, PATH_PERSISTENT = 0, 1, 2
TIMEOUT = 4


def _model(V, D, L, S, B, H, seed, cuda):
    from flb_model import FLBTransformer
    m = FLBTransformer(V, hidden_dim=D, num_layers=L, seq_len=S, batch_size=B, num_heads=H)
    set_hashed_weights(m, seed)
    return m.to(cuda).eval()


class _Run:
    """flb_block_grid_fwd_ex on one model's engine, through the C ABI."""

    def __init__(self, m, tok):
        import flb_native as nat
        from wavefront.flb_cells import BlockWeightStacks
        self.nat = nat
        cfg = m.engine.config
        self.L, self.S = cfg.grid_shape
        self.B, self.D = cfg.batch_size, cfg.dim
        self.w = BlockWeightStacks(list(m.layers))
        with torch.no_grad():
            self.x = m.embedding(tok).to(torch.bfloat16).contiguous()
        self.ws_bytes = nat.lib.flb_block_grid_workspace_bytes(self.L, self.S, self.B, self.D)
        self.ws = nat.workspace(self.ws_bytes, self.x.device)

    def grids(self):
        return torch.zeros(4, self.L * self.S + self.L, self.B, self.D, dtype=torch.bfloat16,
                           device=self.x.device)

    def __call__(self, path, grids=None):
        g = self.grids() if grids is None else grids
        nat = self.nat
        st = nat.lib.flb_block_grid_fwd_ex(
            ctypes.cast(ctypes.pointer(self.w.struct), ctypes.c_void_p), self.x.data_ptr(),
            g.data_ptr(), self.L, self.S, self.B, self.D, self.w.heads, self.w.eps,
            nat.ptr(self.ws), self.ws_bytes, path, nat.stream_of(g))
        nat.check(st, "flb_block_grid_fwd_ex")
        return g

    def status(self):
        return self.nat.lib.flb_block_grid_status(self.nat.ptr(self.ws),
                                                  self.nat.stream_of(self.x))

    def cells(self, g):
        return g[:, : self.L * self.S]


def _max_rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()


def test_persistent_against_reference_golden(cuda):
    """Logits, aux loss and next contexts of the model whose engine runs the persistent forward,
    against the reference model in float32 (golden flb_model_b16.pt)."""
    g = torch.load(os.path.join(os.path.dirname(__file__), "golden", "flb_model_b16.pt"))
    c = g["config"]
    m = _model(c["vocab"], c["hidden"], c["layers"], c["seq_len"], c["batch"], 8,
               c["weight_seed"], cuda)
    tok = g["tokens"].to(cuda)
    m.engine.native_flb_path = PATH_PERSISTENT
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        logits, aux, (lat, fdbk) = m(tok)
        m.engine.native_cells = False
        lg, ag, _ = m(tok)
    ref = g["logits"].to(cuda)
    e_nat, e_gen = _max_rel(logits, ref), _max_rel(lg, ref)
    assert e_nat < 2e-2, (e_nat, e_gen)
    assert abs(aux.item() - g["aux_loss"].item()) <= 2e-2 * abs(g["aux_loss"].item()) + 1e-6
    assert _max_rel(lat, g["next_lat"].to(cuda)) < 2e-2
    assert _max_rel(fdbk, g["next_fdbk"].to(cuda)) < 2e-2


@pytest.mark.parametrize("L,S,D,H", [(3, 4, 128, 8), (5, 7, 256, 4), (6, 5, 768, 12),
                                     (24, 13, 768, 12)])
def test_persistent_matches_tick_path(cuda, L, S, D, H):
    """Every port grid of the persistent forward against the tick-by-tick native path (both
    bf16 with fp32 accumulation; the tiles' K order differs from cuBLAS's): 2e-2 of each grid's
    largest magnitude. (24, 13, 768, 12) has up to 12 cells per tick: 216 stage-1 tiles, more
    than one per SM."""
    torch.manual_seed(0)
    m = _model(50, D, L, S, 16, H, 11 + L, cuda)
    tok = torch.randint(0, 50, (16, S), device=cuda)
    run = _Run(m, tok)
    gp = run(PATH_PERSISTENT)
    assert run.status() == 0
    gt = run(PATH_TICKS)
    torch.cuda.synchronize()
    for p in range(4):
        a, b = run.cells(gp)[p], run.cells(gt)[p]
        assert torch.isfinite(a.float()).all(), p
        # port 3, aux = (lat_prior - bf16(o1 + lat_prior))^2 + ...: o is rounded against
        # lat_prior's bf16 ulp, so a last-bit change of o moves aux by more than 2e-2 of its max
        assert _max_rel(a, b) < (4e-2 if p == 3 else 2e-2), (p, _max_rel(a, b))
    # the dock rows past the cells are not touched
    assert not run.grids()[:, L * S:].any() and not gp[:, L * S:].any()


def test_persistent_repeatable_and_default_path(cuda):
    """Two persistent runs give identical grids; the default path is the tick-by-tick one."""
    m = _model(50, 256, 4, 6, 16, 8, 3, cuda)
    tok = torch.randint(0, 50, (16, 6), device=cuda, generator=torch.Generator(cuda).manual_seed(1))
    run = _Run(m, tok)
    a = run(PATH_PERSISTENT)
    b = run(PATH_PERSISTENT)
    c = run(PATH_AUTO)
    d = run(PATH_TICKS)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(c, d)


def test_persistent_through_engine_graph(cuda):
    """engine.native_flb_path = 2 routes the model's forward to the persistent kernel, and its
    CUDA-graph capture (one cooperative launch) replays to the same logits as eager."""
    from wavefront.wavefront_graph import GraphedWavefrontEngine
    m = _model(50, 256, 4, 6, 16, 8, 7, cuda)
    tok = torch.randint(0, 50, (16, 6), device=cuda, generator=torch.Generator(cuda).manual_seed(3))
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        lt, _, _ = m(tok)
        m.engine.native_flb_path = PATH_PERSISTENT
        lp, _, _ = m(tok)
        x = m.embedding(tok)
        graphed = GraphedWavefrontEngine(m.engine, x, backward=False)
        lg, _, _ = m(tok, engine=graphed)
    assert _max_rel(lp, lt) < 2e-2
    assert torch.equal(lg, lp)


def test_persistent_rejects_other_shapes(cuda):
    """Batch 3 or d_model 64 is not a persistent shape: path 2 returns FLB_ERR_UNSUPPORTED."""
    m = _model(50, 64, 3, 4, 3, 8, 3, cuda)
    tok = torch.randint(0, 50, (3, 4), device=cuda)
    run = _Run(m, tok)
    with pytest.raises(RuntimeError, match="UNSUPPORTED"):
        run(PATH_PERSISTENT)
    run(PATH_AUTO)  # the tick-by-tick path takes it


@pytest.mark.parametrize("drop_cta,drop_barrier", [(5, 0), (0, 7)])
def test_persistent_barrier_timeout_detected(cuda, drop_cta, drop_barrier):
    """One CTA never arrives at one grid barrier: the others' bounded polls give up, the error
    word is set and every CTA returns (FLB_ERR_TIMEOUT, read back synchronously); the context
    stays usable and the next run matches a clean one."""
    m = _model(50, 256, 4, 6, 16, 8, 3, cuda)
    tok = torch.randint(0, 50, (16, 6), device=cuda, generator=torch.Generator(cuda).manual_seed(2))
    run = _Run(m, tok)
    clean = run(PATH_PERSISTENT)
    g = run.grids()
    nat = run.nat
    st = nat.lib.flb_block_grid_fwd_drop_barrier_test(
        ctypes.cast(ctypes.pointer(run.w.struct), ctypes.c_void_p), run.x.data_ptr(),
        g.data_ptr(), run.L, run.S, run.B, run.D, run.w.heads, run.w.eps, nat.ptr(run.ws),
        run.ws_bytes, drop_cta, drop_barrier, 1 << 12, nat.stream_of(g))
    assert st == TIMEOUT
    assert run.status() == TIMEOUT
    again = run(PATH_PERSISTENT)
    assert run.status() == 0
    torch.cuda.synchronize()
    assert torch.equal(again, clean)
