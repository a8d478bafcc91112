"""Known-answer checks of the tcgen05 / TMA operand layouts and the throughput probes."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant,n", [(0, 64), (0, 128), (1, 64), (1, 128)])
def test_umma_layouts(cuda, variant, n):
    import flb_native as nat
    g = torch.Generator().manual_seed(variant * 10 + n)
    A = torch.randn(128, 64, generator=g).bfloat16()
    B = torch.randn(n, 64, generator=g).bfloat16() if variant == 0 else \
        torch.randn(64, n, generator=g).bfloat16()
    ref = A.float() @ (B.float().T if variant == 0 else B.float())
    Ad, Bd = A.to(cuda).contiguous(), B.to(cuda).contiguous()
    D = torch.full((128, n), float("nan"), device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    nat.check(nat.lib.flb_selftest_umma(variant, n, Ad.data_ptr(), Bd.data_ptr(), D.data_ptr(),
                                        err.data_ptr(), nat.stream_of(D)), "selftest")
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.allclose(D.cpu(), ref, atol=1e-3, rtol=1e-3)


def test_microbench_rates_plausible(cuda):
    import flb_native as nat
    rates = {k: nat.microbench(k, cuda) for k in range(6)}
    # every probe reports a positive, finite rate below 1e15 elements/s
    for k, r in rates.items():
        assert 1e10 < r < 1e15, (k, r)
