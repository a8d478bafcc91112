"""GPU parity of the wavefront engine: the CUDA gather against the reference's gather goldens,
and the engine (C++ tick loop + CUDA scatters) against the reference engine's outputs and
gradients on the configurations of the reference's own tests."""
import copy
import math

import pytest
import torch
import torch.nn as nn

from oracle import wavefront as ow

pytestmark = pytest.mark.gpu


def test_gather_matches_reference_goldens(cuda, wf_golden):
    from wavefront import WavefrontConfig, WavefrontEngine, run_fetch_kernel
    for c in wf_golden["gather_cases"]:
        cfg = WavefrontConfig(grid_shape=c["grid"], batch_size=c["batch"], dim=c["dim"])
        eng = WavefrontEngine(cfg, nn.ModuleList([nn.Identity() for _ in range(cfg.grid_shape[0])]))
        eng = eng.to(cuda)
        x = c["x"].to(cuda)
        eng._init_buffers(x)
        n = math.prod(cfg.grid_shape)
        active = torch.arange(n, dtype=torch.int32, device=cuda)
        out = torch.full((2, n, cfg.batch_size, cfg.dim), 7.0, device=cuda)
        run_fetch_kernel(x, c["stacked_grids"].to(cuda), eng.routing_map, eng.port_map,
                         eng.spatial_map_buffer, cfg, active, out)
        assert torch.equal(out.cpu(), c["expected"]), c["grid"]


def test_gather_padding_slots_and_dtypes(cuda):
    """Padding cells (index num_cells) write zeros; bf16/fp16 gathers copy bits exactly."""
    from wavefront import WavefrontConfig, WavefrontEngine, run_fetch_kernel
    cfg = WavefrontConfig(grid_shape=(3, 5), batch_size=3, dim=40)
    eng = WavefrontEngine(cfg, nn.ModuleList([nn.Identity() for _ in range(3)])).to(cuda)
    for dt in (torch.float32, torch.bfloat16, torch.float16):
        x = torch.randn(3, 5, 40, device=cuda).to(dt)
        eng._init_buffers(x)
        grids = torch.randn(2, 15 + 3, 3, 40, device=cuda).to(dt)
        active = torch.tensor([4, 15, 7, 15], dtype=torch.int32, device=cuda)
        out = torch.full((2, 4, 3, 40), 3.0, device=cuda).to(dt)
        run_fetch_kernel(x, grids, eng.routing_map, eng.port_map, eng.spatial_map_buffer, cfg,
                         active, out)
        exp = ow.gather(x.cpu(), grids.cpu(), [4, 15, 7, 15], eng.routing_map.tolist(), [0, 1],
                        (3, 5), 2)
        assert torch.equal(out.cpu(), exp)


def _layers_from_golden(case, c, cuda):
    from test_oracle import DummyLayer, TanhCellRef
    mods = []
    for sd in c["params"]:
        m = DummyLayer(c["dim"]) if case == "engine_dummy_2x3" else TanhCellRef(c["dim"])
        m.load_state_dict(sd)
        mods.append(m)
    return nn.ModuleList(mods).to(cuda)


@pytest.mark.parametrize("case", ["engine_dummy_2x3", "engine_tanh_3x5"])
def test_engine_matches_reference_engine(cuda, wf_golden, case):
    """Outputs, x.grad and every parameter gradient against the reference engine (fp32,
    atol 1e-5 as in wavefront/wavefront_test.py:229-230)."""
    from wavefront import WavefrontConfig, WavefrontEngine
    c = wf_golden[case]
    cfg = WavefrontConfig(grid_shape=c["grid"], batch_size=c["batch"], dim=c["dim"])
    layers = _layers_from_golden(case, c, cuda)
    eng = WavefrontEngine(cfg, layers).to(cuda)
    x = c["x"].to(cuda).requires_grad_(True)
    grids = eng(x)
    for p in range(2):
        assert torch.allclose(grids[p].cpu(), c["grids"][p], atol=1e-5)
    loss = grids[0][-1].sum() + 0.5 * grids[1].square().sum()
    loss.backward()
    assert torch.allclose(x.grad.cpu(), c["x_grad"], atol=1e-5)
    for l, m in enumerate(layers):
        for n, p in m.named_parameters():
            assert torch.allclose(p.grad.cpu(), c["param_grads"][l][n], atol=1e-4), (l, n)
    # a second call on the same engine reuses the buffers and gives the same answer
    x2 = c["x"].to(cuda).requires_grad_(True)
    g2 = eng(x2)
    assert torch.allclose(g2[0].cpu(), c["grids"][0], atol=1e-5)


def test_engine_flb_dependencies_against_pure_loop(cuda):
    """Three dependencies with a feedback offset (1,-1) and four ports, as FLB_Transformer
    configures the engine (models/FLB_Model.py:111-121)."""
    from wavefront import WavefrontConfig, WavefrontEngine
    torch.manual_seed(3)
    deps = [((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)]
    cfg = WavefrontConfig(grid_shape=(3, 5), batch_size=2, dim=8, dependencies=deps, num_ports=4)

    class Cell(nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = nn.Linear(24, 32)

        def forward(self, a, b, c):
            o = torch.tanh(self.lin(torch.cat([a, b, c], -1)))
            return o[..., :8], o[..., 8:16], o[..., 16:24], o[..., 24:]

    base = nn.ModuleList([Cell() for _ in range(3)])
    x = torch.randn(2, 5, 8)
    lp = copy.deepcopy(base)
    xp = x.clone().requires_grad_(True)
    grids = ow.pure_loop((3, 5), deps, 4, lp, xp)
    pure = [torch.stack([torch.stack(r) for r in grids[p]]).reshape(-1, 2, 8) for p in range(4)]
    (pure[0].sum() + pure[3].square().sum()).backward()

    le = copy.deepcopy(base).to(cuda)
    eng = WavefrontEngine(cfg, le).to(cuda)
    xe = x.to(cuda).requires_grad_(True)
    out = eng(xe)
    for p in range(4):
        assert torch.allclose(out[p].cpu(), pure[p].detach(), atol=1e-5)
    (out[0].sum() + out[3].square().sum()).backward()
    assert torch.allclose(xe.grad.cpu(), xp.grad, atol=1e-5)
    for a, b in zip(le.parameters(), lp.parameters()):
        assert torch.allclose(a.grad.cpu(), b.grad, atol=1e-5)


class _FlbLikeCell(nn.Module):
    """Three inputs (feedforward, lateral, feedback), four outputs, as the FLB block's ports."""

    def __init__(self, dim):
        super().__init__()
        self.lin = nn.Linear(3 * dim, 4 * dim)
        self.dim = dim

    def forward(self, a, b, c):
        o = torch.tanh(self.lin(torch.cat([a, b, c], -1)))
        d = self.dim
        return o[..., :d], o[..., d:2 * d], o[..., 2 * d:3 * d], o[..., 3 * d:]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_graphed_engine_matches_eager(cuda, dtype):
    """CUDA-graph replay of the per-tick loops (GraphedWavefrontEngine) against the eager
    engine: outputs, x.grad and parameter grads over three calls with new inputs, with an
    in-place parameter update between calls (the graph re-reads the live parameters)."""
    from wavefront import WavefrontConfig, WavefrontEngine, GraphedWavefrontEngine
    torch.manual_seed(11)
    deps = [((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)]
    cfg = WavefrontConfig(grid_shape=(4, 6), batch_size=3, dim=16, dependencies=deps,
                          num_ports=4)
    base = nn.ModuleList([_FlbLikeCell(16) for _ in range(4)])
    la, lb = copy.deepcopy(base).to(cuda), copy.deepcopy(base).to(cuda)
    eng_a = WavefrontEngine(cfg, la).to(cuda)
    eng_b = WavefrontEngine(cfg, lb).to(cuda)
    x0 = torch.randn(3, 6, 16, device=cuda).to(dtype)
    graphed = GraphedWavefrontEngine(eng_b, x0)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for it in range(3):
        x = torch.randn(3, 6, 16, device=cuda).to(dtype)
        xa = x.clone().requires_grad_(True)
        xb = x.clone().requires_grad_(True)
        oa = eng_a(xa)
        ob = graphed(xb)
        for p in range(4):
            assert torch.allclose(oa[p].float(), ob[p].float(), atol=tol), (it, p)
        (oa[0].float().sum() + oa[3].float().square().sum()).backward()
        (ob[0].float().sum() + ob[3].float().square().sum()).backward()
        assert torch.allclose(xa.grad.float(), xb.grad.float(), atol=tol), it
        for pa, pb in zip(la.parameters(), lb.parameters()):
            scale = max(1.0, pa.grad.abs().max().item())
            assert torch.allclose(pa.grad, pb.grad, atol=tol * scale), it
        with torch.no_grad():
            for pa, pb in zip(la.parameters(), lb.parameters()):
                pa.mul_(0.9)
                pb.mul_(0.9)


def test_graphed_engine_rejects_other_shapes_and_fast_path(cuda):
    from wavefront import WavefrontConfig, WavefrontEngine, GraphedWavefrontEngine
    from wavefront.grid_layer import TanhGridCell
    cfg = WavefrontConfig(grid_shape=(2, 3), batch_size=2, dim=8,
                          dependencies=[((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)], num_ports=4)
    eng = WavefrontEngine(cfg, nn.ModuleList([_FlbLikeCell(8) for _ in range(2)])).to(cuda)
    g = GraphedWavefrontEngine(eng, torch.randn(2, 3, 8, device=cuda))
    with pytest.raises(ValueError):
        g(torch.randn(2, 4, 8, device=cuda))
    fast_cfg = WavefrontConfig(grid_shape=(2, 3), batch_size=16, dim=128)
    fast = WavefrontEngine(fast_cfg, nn.ModuleList([TanhGridCell(128) for _ in range(2)])).to(cuda)
    with pytest.raises(ValueError):
        GraphedWavefrontEngine(fast, torch.randn(16, 3, 128, device=cuda).bfloat16())


def test_index_copy_modes(cuda):
    import flb_native as nat
    src = torch.randn(6, 3, 5, device=cuda)
    dst = torch.zeros(4, 3, 5, device=cuda, dtype=torch.bfloat16)
    sr = torch.tensor([0, 2, 5], device=cuda)
    dr = torch.tensor([3, 1, 3], device=cuda)
    nat.check(nat.lib.flb_wf_index_copy(src.data_ptr(), 0, nat.strides(*src.stride()), sr.data_ptr(),
                                        dst.data_ptr(), 2, nat.strides(*dst.stride()), dr.data_ptr(),
                                        3, 3, 5, 1, nat.stream_of(src)), "index_copy")
    exp = torch.zeros(4, 3, 5)
    exp.index_add_(0, dr.cpu(), src.cpu()[sr.cpu()])
    assert torch.allclose(dst.float().cpu(), exp.bfloat16().float(), atol=2e-2)
