"""One process driving two GPUs: kernel attributes (the dynamic shared-memory limit the tcgen05
kernels need) and the static scratch address are per device, so a call on device 1 after calls
on device 0 must set up device 1 for itself. Checked through the public attention op and the
C ABI's allocation-free grid forward: the same inputs give the same results on both devices
(the kernels are deterministic for these launches: the forward has no atomics). Skipped with
fewer than two GPUs."""
import math

import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu


def _two_devices():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    return torch.device("cuda:0"), torch.device("cuda:1")


def test_attention_forward_on_two_devices():
    from kernels.additive_attention import attention_forward
    d0, d1 = _two_devices()
    q, k, v, w = oa.make_inputs(2, 2, 300, 64, seed=3, dtype=torch.bfloat16)
    outs = []
    for dev in (d0, d1, d0):
        with torch.cuda.device(dev):
            o, lse, _, _, _ = attention_forward(*(t.to(dev) for t in (q, k, v, w)), True)
            torch.cuda.synchronize(dev)
            outs.append((o.cpu(), lse.cpu()))
    ref = oa.attention_forward(q, k, v, w, causal=True)[0]
    for o, lse in outs:
        assert torch.equal(o, outs[0][0]) and torch.equal(lse, outs[0][1])
        assert ((o.double() - ref).abs() - (2e-2 + 2.0 ** -8 * ref.abs())).max().item() <= 0


def test_static_grid_forward_on_two_devices():
    import flb_native as nat
    d0, d1 = _two_devices()
    R, C, B, H, G = 4, 5, 16, 128, 1
    g = torch.Generator().manual_seed(5)
    s = 1.0 / math.sqrt(H)
    Wl = (torch.randn(G, H, H, generator=g) * s).bfloat16()
    Wt = (torch.randn(G, H, H, generator=g) * s).bfloat16()
    b = (torch.randn(G, H, generator=g) * 0.1).float()
    top = torch.randn(C, B, H, generator=g).bfloat16()
    outs = []
    for dev in (d0, d1):
        with torch.cuda.device(dev):
            t = [x.to(dev) for x in (Wl, Wt, b, top)]
            h = torch.empty(R, C, B, H, dtype=torch.bfloat16, device=dev)
            nat.check(nat.lib.flb_grid_fwd_static(t[0].data_ptr(), t[1].data_ptr(),
                                                  t[2].data_ptr(), t[3].data_ptr(), h.data_ptr(),
                                                  R, C, B, H, G, 1, nat.stream_of(h)),
                      "flb_grid_fwd_static")
            torch.cuda.synchronize(dev)
            outs.append(h.cpu())
    assert torch.isfinite(outs[0].float()).all()
    assert torch.equal(outs[0], outs[1])
