"""The tcgen05 projection GEMM of the FLB block cells (flb_cell_gemm) against torch on the same bf16
inputs (fp32 accumulation both ways): the tick shapes of the FLB model at d_model 768 (priors and
gates M = batch rows, N = K = 768; q|k|v M = 3 x batch, N = 2304; output projection M = 3 x batch,
N = 768), cells two layers apart in a weight stack, and input / output rows with a pitch wider
than the row (the token tensor's slots)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,n_cells,ldx_mul,ldy_mul", [
    (16, 768, 768, 6, 1, 1),     # priors / gates, batch 16
    (16, 768, 768, 5, 3, 3),     # token-slot rows in and out (pitch 3 D)
    (48, 2304, 768, 6, 1, 1),    # q | k | v of the three tokens
    (48, 768, 768, 3, 1, 1),     # output projection
    (32, 256, 128, 1, 1, 2),     # small K: fewer atoms than stages
    (64, 384, 1024, 2, 1, 1),
])
def test_cell_gemm_matches_torch(cuda, M, N, K, n_cells, ldx_mul, ldy_mul):
    import flb_native as nat
    g = torch.Generator().manual_seed(M + N + K)
    L = 2 * n_cells + 1
    l0 = 1
    W = (torch.randn(L, N, K, generator=g) / K ** 0.5).to(cuda, torch.bfloat16)
    ldx, ldy = K * ldx_mul, N * ldy_mul
    X = torch.randn(n_cells, M, ldx, generator=g).to(cuda, torch.bfloat16)
    Y = torch.full((n_cells, M, ldy), 7.0, device=cuda, dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(2):  # two calls in a row: barriers and TMEM start clean every launch
        st = nat.lib.flb_cell_gemm(W.data_ptr(), L * N, l0 * N, 2 * N, X.data_ptr(), ldx, M * ldx,
                                   n_cells, M, N, K, Y.data_ptr(), ldy, M * ldy, err.data_ptr(),
                                   nat.stream_of(Y))
        assert st == 0, nat.lib.flb_last_error()
        torch.cuda.synchronize()
        assert err.item() == 0
        for i in range(n_cells):
            ref = X[i, :, :K].float() @ W[l0 + 2 * i].float().T
            got = Y[i, :, :N].float()
            assert (got - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-2
        if ldy > N:  # columns beyond N untouched
            assert (Y[:, :, N:].float() == 7.0).all()


def test_cell_gemm_rejects_unsupported(cuda):
    import flb_native as nat
    W = torch.zeros(128, 64, device=cuda, dtype=torch.bfloat16)
    X = torch.zeros(8, 64, device=cuda, dtype=torch.bfloat16)
    Y = torch.zeros(8, 128, device=cuda, dtype=torch.bfloat16)
    st = nat.lib.flb_cell_gemm(W.data_ptr(), 128, 0, 0, X.data_ptr(), 64, 0, 1, 8, 128, 64,
                               Y.data_ptr(), 128, 0, None, nat.stream_of(Y))
    assert st == 6  # FLB_ERR_UNSUPPORTED: M = 8
