"""GPU parity of the persistent tanh grid kernels (flb_grid_fwd / flb_grid_bwd) against the
oracle's pure anti-diagonal loop, and of the engine fast path against the per-tick engine.

Tolerances: bf16 storage with fp32 accumulation. h (values in [-1, 1]): max-abs 2e-2 plus half
a bf16 ulp of the value. Every gradient travels back through the recurrence, whose dz is stored
in bf16 at each cell (as the reference engine's bf16 gradient grids are), and the weight and bias
gradients are sums over R*C*B products; gradients are therefore compared relative to the
tensor's largest magnitude: max|a - ref| <= 2e-2 * max(1, max|ref|)."""
import math

import pytest
import torch

from oracle import wavefront as ow

pytestmark = pytest.mark.gpu


def excess_half(a, ref):
    a, ref = a.double().cpu(), ref.double().cpu()
    return ((a - ref).abs() - (2e-2 + 2.0 ** -8 * ref.abs())).max().item()


def rel_err(a, ref):
    a, ref = a.double().cpu(), ref.double().cpu()
    return ((a - ref).abs().max() / max(1.0, ref.abs().max().item())).item()


def oracle_grads(x, Wl, Wt, U, b, top, dh, dtype=torch.float64):
    ts = [None if t is None else t.to(dtype).clone().requires_grad_(True)
          for t in (x, Wl, Wt, U, b, top)]
    h = ow.tanh_grid_forward(*ts)
    h.backward(dh.to(dtype))
    return h.detach(), [None if t is None else t.grad for t in ts]


def bf(t):
    return None if t is None else t.bfloat16()


@pytest.mark.parametrize("R,C,B,H,G,with_U,with_top", [
    (3, 4, 16, 128, 1, True, False),
    (5, 7, 32, 256, 1, True, False),
    (4, 5, 16, 256, 4, False, True),      # per-row weights, x at row 0 only (engine semantics)
    (6, 3, 48, 128, 6, True, True),
    (1, 9, 64, 128, 1, True, False),
    (9, 1, 16, 256, 1, True, True),
])
def test_grid_layer_matches_oracle(cuda, R, C, B, H, G, with_U, with_top):
    from wavefront.grid_layer import wavefront_grid_layer
    x, Wl, Wt, U, b, top, dh = ow.tanh_grid_make_inputs(B, R, C, H, G=G, seed=R * 7 + C,
                                                        with_U=with_U, with_top=with_top)
    b = torch.randn(G, H) * 0.1
    x, Wl, Wt, U, top, dh = (bf(t) for t in (x, Wl, Wt, U, top, dh))
    href, gref = oracle_grads(x, Wl, Wt, U, b, top, dh)
    dev = [None if t is None else t.to(cuda).requires_grad_(True) for t in (x, Wl, Wt, U, b, top)]
    h = wavefront_grid_layer(dev[0] if with_U else torch.zeros(B, R, C, H, device=cuda, dtype=torch.bfloat16),
                             dev[1], dev[2], dev[3], dev[4], dev[5])
    assert h.shape == (R, C, B, H)
    assert excess_half(h, href) <= 0
    h.backward(dh.to(cuda))
    names = ["x", "W_l", "W_t", "U", "b", "top"]
    for name, t, r in zip(names, dev, gref):
        if t is None or r is None or (name == "x" and not with_U):
            continue
        assert t.grad is not None, name
        assert rel_err(t.grad, r) < 2e-2, (name, rel_err(t.grad, r))


def test_w4_full_size(cuda):
    """The benchmark configuration: 64x64 grid, batch 32, hidden 256, forward + backward,
    against the oracle loop evaluated in float32 on the same bf16 inputs."""
    from wavefront.grid_layer import wavefront_grid_layer, grid_inputs
    x, Wl, Wt, U, b, dh = grid_inputs(32, 64, 64, 256, "cpu", seed=3)
    href, gref = oracle_grads(x, Wl.unsqueeze(0), Wt.unsqueeze(0), U, b.float().unsqueeze(0), None,
                              dh, dtype=torch.float32)
    dev = [t.to(cuda).requires_grad_(True) for t in (x, Wl, Wt, U, b)]
    h = wavefront_grid_layer(*dev)
    assert excess_half(h, href) <= 0
    h.backward(dh.to(cuda))
    assert rel_err(dev[0].grad, gref[0]) < 2e-2
    for t, r in zip(dev[1:], [gref[1][0], gref[2][0], gref[3], gref[4][0]]):
        assert rel_err(t.grad, r) < 2e-2


def test_grid_repeatable_and_second_call(cuda):
    from wavefront.grid_layer import wavefront_grid_layer, grid_inputs
    x, Wl, Wt, U, b, _ = grid_inputs(16, 8, 8, 128, cuda, seed=1)
    h1 = wavefront_grid_layer(x, Wl, Wt, U, b)
    h2 = wavefront_grid_layer(x, Wl, Wt, U, b)
    assert torch.equal(h1, h2)  # a fixed-order recurrence: bitwise repeatable


def test_engine_fast_path_matches_per_tick_engine(cuda):
    """An engine of TanhGridCell layers in bf16 runs the persistent kernels; the same engine with
    a cell subclass (not recognised, so the per-tick path runs) must agree."""
    import copy
    import torch.nn as nn
    from wavefront import WavefrontConfig, WavefrontEngine
    from wavefront.grid_layer import TanhGridCell

    class PlainCell(TanhGridCell):
        pass

    torch.manual_seed(2)
    R, C, B, H = 4, 6, 16, 128
    cfg = WavefrontConfig(grid_shape=(R, C), batch_size=B, dim=H)
    fast_layers = nn.ModuleList([TanhGridCell(H) for _ in range(R)])
    for l in fast_layers:
        l.b.data.normal_(0, 0.1)
    slow_layers = nn.ModuleList([PlainCell(H) for _ in range(R)])
    slow_layers.load_state_dict(fast_layers.state_dict())
    fast_layers, slow_layers = fast_layers.to(cuda), slow_layers.to(cuda)
    x = torch.randn(B, C, H, device=cuda).bfloat16()
    outs = []
    for layers in (fast_layers, slow_layers):
        eng = WavefrontEngine(cfg, layers).to(cuda)
        xx = x.clone().requires_grad_(True)
        g = eng(xx)
        (g[0].float().square().sum() + g[1][-1].float().sum()).backward()
        outs.append((g[0].detach(), xx.grad, [p.grad.clone() for p in layers.parameters()]))
    (h_f, gx_f, gp_f), (h_s, gx_s, gp_s) = outs
    assert excess_half(h_f, h_s.float()) <= 0
    assert rel_err(gx_f, gx_s.float()) < 2e-2
    for a, r in zip(gp_f, gp_s):
        assert rel_err(a, r) < 2e-2


def test_bounded_wait_reports_timeout(cuda):
    """Failure detection without a GPU fault: a dependency flag that nothing releases makes the
    waiting cells give up after a short bound; the call reports FLB_ERR_TIMEOUT and the context
    stays usable for the next call."""
    import flb_native as nat
    from wavefront.grid_layer import wavefront_grid_layer, grid_inputs
    R, C, B, H = 3, 3, 16, 128
    x, Wl, Wt, U, b, _ = grid_inputs(B, R, C, H, cuda, seed=4)
    h = torch.empty(R, C, B, H, device=cuda, dtype=torch.bfloat16)
    bias = b.float().unsqueeze(0).contiguous()
    ws_bytes = nat.lib.flb_grid_workspace_bytes(R, C, B, H, 1, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda)
    st = nat.lib.flb_grid_fwd_drop_flag_test(x.data_ptr(), 0, Wl.data_ptr(), Wt.data_ptr(),
                                             U.data_ptr(), bias.data_ptr(), None, h.data_ptr(),
                                             R, C, B, H, 1, ws.data_ptr(), ws_bytes, 1, 1, 20000,
                                             nat.stream_of(h))
    assert st == 4  # FLB_ERR_TIMEOUT
    msg = nat.lib.flb_last_error().decode()
    assert "gave up" in msg
    # cells (1, 2) and (2, 1) wait on the withheld flag of (1, 1) through the same grid's flags:
    # code 2 (a halo timeout would be code 6)
    assert "(code 2)" in msg
    h2 = wavefront_grid_layer(x, Wl, Wt, U, b)  # the device is still healthy
    torch.cuda.synchronize()
    assert torch.isfinite(h2.float()).all()
