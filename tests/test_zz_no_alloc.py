"""The allocation-free grid forward (flb_grid_fwd_static), for callers that cannot allocate device
memory when they run the layer: it keeps its scratch in a static device array of the library
instead of taking a workspace. Checked through the C ABI against the workspace entry point
(flb_grid_fwd) on two calls in a row, since every call reuses the array the previous call left
behind. Outputs must agree within the grid tests' tolerance for h (2e-2 plus half a bf16 ulp);
the two entry points run the same kernel, so they are expected to agree exactly."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(R, C, B, H, G, seed, with_top, device):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(H)
    Wl = (torch.randn(G, H, H, generator=g) * s).bfloat16().to(device)
    Wt = (torch.randn(G, H, H, generator=g) * s).bfloat16().to(device)
    b = (torch.randn(G, H, generator=g) * 0.1).float().to(device)
    top = torch.randn(C, B, H, generator=g).bfloat16().to(device) if with_top else None
    return Wl, Wt, b, top


def _with_workspace(nat, Wl, Wt, b, top, R, C, B, H, G):
    h = torch.empty(R, C, B, H, dtype=torch.bfloat16, device=Wl.device)
    n = nat.lib.flb_grid_workspace_bytes(R, C, B, H, G, 0)
    ws = torch.empty(n, dtype=torch.uint8, device=Wl.device)
    nat.check(nat.lib.flb_grid_fwd(None, 1, Wl.data_ptr(), Wt.data_ptr(), None, b.data_ptr(),
                                   nat.ptr(top), h.data_ptr(), R, C, B, H, G, ws.data_ptr(), n, 1,
                                   nat.stream_of(h)), "flb_grid_fwd")
    return h


def _static(nat, Wl, Wt, b, top, R, C, B, H, G):
    h = torch.full((R, C, B, H), float("nan"), dtype=torch.bfloat16, device=Wl.device)
    nat.check(nat.lib.flb_grid_fwd_static(Wl.data_ptr(), Wt.data_ptr(), b.data_ptr(),
                                          nat.ptr(top), h.data_ptr(), R, C, B, H, G, 1,
                                          nat.stream_of(h)), "flb_grid_fwd_static")
    return h


def _excess(a, ref):
    a, ref = a.double().cpu(), ref.double().cpu()
    return ((a - ref).abs() - (2e-2 + 2.0 ** -8 * ref.abs())).max().item()


@pytest.mark.parametrize("R,C,B,H,G,with_top", [(6, 9, 32, 256, 6, True), (4, 5, 16, 128, 1, False)])
def test_static_scratch_matches_workspace_entry_point(cuda, R, C, B, H, G, with_top):
    import flb_native as nat
    ref = None
    for call in range(2):  # the second call finds the first call's flags and error word
        Wl, Wt, b, top = _inputs(R, C, B, H, G, seed=10 + call, with_top=with_top, device=cuda)
        ref = _with_workspace(nat, Wl, Wt, b, top, R, C, B, H, G)
        got = _static(nat, Wl, Wt, b, top, R, C, B, H, G)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert _excess(got, ref) <= 0


def test_static_scratch_rejects_grids_beyond_its_limit(cuda):
    import flb_native as nat
    R, C, B, H, G = 300, 300, 16, 128, 1  # 90000 cells > 65536
    Wl, Wt, b, _ = _inputs(2, 2, B, H, G, seed=1, with_top=False, device=cuda)
    st = nat.lib.flb_grid_fwd_static(Wl.data_ptr(), Wt.data_ptr(), b.data_ptr(), None,
                                     Wl.data_ptr(), R, C, B, H, G, 0, nat.stream_of(Wl))
    assert st == 1  # FLB_ERR_SHAPE, rejected before any launch
    assert "static scratch limit" in nat.lib.flb_last_error().decode()
