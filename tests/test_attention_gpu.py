"""GPU parity of the additive-attention kernels against the reference goldens and the oracle.

Tolerances (max-abs, on outputs and gradients):
  fp32 with tanh.approx / ex2.approx : 2e-3
  fp32 exact mode (tanhf / expf)     : 1e-5
  bf16 / fp16 inputs                 : 2e-2, plus the rounding of a bf16 output itself
                                       (half a bf16 ulp of the value, 2^-8 |ref|; one ulp,
                                       2^-7 |ref|, when two bf16 results are compared)
The oracle evaluates the reference math in float64 on the same input values."""
import math

import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

TOL_APPROX, TOL_EXACT, TOL_HALF = 2e-3, 1e-5, 2e-2


def run(q, k, v, w, dout=None, causal=False, exact=False):
    from kernels import fused_additive_attention
    ts = [t.clone().requires_grad_(dout is not None) for t in (q, k, v, w)]
    out = fused_additive_attention(*ts, causal=causal, exact=exact)
    if dout is None:
        return out.detach(), None
    out.backward(dout)
    return out.detach(), [t.grad for t in ts]


def maxdiff(a, b):
    return (a.double().cpu() - b.double().cpu()).abs().max().item()


def excess_half(a, ref, ulps=0.5):
    """max over elements of |a - ref| - (2e-2 + ulps * 2^-7 * |ref|); <= 0 passes."""
    a, ref = a.double().cpu(), ref.double().cpu()
    return ((a - ref).abs() - (TOL_HALF + ulps * 2.0 ** -7 * ref.abs())).max().item()


@pytest.mark.parametrize("exact", [False, True])
def test_kat_reference_config(cuda, attn_golden, exact):
    g = attn_golden["kat_b2h8n3d32"]
    dev = [g[n].to(cuda) for n in ("q", "k", "v", "v_a", "dout")]
    out, grads = run(*dev[:4], dout=dev[4], exact=exact)
    tol = TOL_EXACT if exact else TOL_APPROX
    assert maxdiff(out, g["out"]) < tol
    for name, gr in zip(("dq", "dk", "dv", "dv_a"), grads):
        assert gr.shape == g[name].shape
        assert maxdiff(gr, g[name]) < tol, name


def test_vmap_reference_config(cuda, attn_golden):
    from kernels import fused_additive_attention
    g = attn_golden["vmap_l4"]
    out = torch.vmap(fused_additive_attention)(*(g[n].to(cuda) for n in ("q", "k", "v", "v_a")))
    assert maxdiff(out, g["out"]) < TOL_APPROX


@pytest.mark.parametrize("exact", [False, True])
def test_n96_golden(cuda, attn_golden, exact):
    g = attn_golden["b2h2n96d64"]
    dev = [g[n].to(cuda) for n in ("q", "k", "v", "v_a", "dout")]
    out, grads = run(*dev[:4], dout=dev[4], exact=exact)
    tol = TOL_EXACT if exact else TOL_APPROX
    assert maxdiff(out, g["out"]) < tol
    for name, gr in zip(("dq", "dk", "dv", "dv_a"), grads):
        assert maxdiff(gr, g[name]) < tol, name


def test_a1_config_forward(cuda):
    """B2 H4 N256 D64 fp32 non-causal (the CPU-runnable benchmark configuration)."""
    q, k, v, w = oa.make_inputs(2, 4, 256, 64, seed=0)
    ref, _ = oa.attention_forward(q, k, v, w, row_chunk=64)
    out, _ = run(*(t.to(cuda) for t in (q, k, v, w)))
    assert maxdiff(out, ref) < TOL_APPROX


@pytest.mark.parametrize("N,D", [(1, 32), (3, 32), (33, 16), (100, 48), (130, 64), (257, 96),
                                 (64, 128), (40, 256), (65, 8)])
@pytest.mark.parametrize("causal", [False, True])
def test_ragged_shapes_fp32(cuda, N, D, causal):
    q, k, v, w, g = oa.make_inputs(2, 3, N, D, seed=N + D, with_grad_out=True)
    ref = oa.attention_forward(q, k, v, w, causal=causal)[0]
    rg = oa.attention_backward(q, k, v, w, g, causal=causal)
    out, grads = run(*(t.to(cuda) for t in (q, k, v, w)), dout=g.to(cuda), causal=causal)
    assert maxdiff(out, ref) < TOL_APPROX
    for a, b in zip(grads, rg):
        assert maxdiff(a, b) < TOL_APPROX


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N,D,causal", [(200, 64, True), (256, 64, False), (130, 128, True),
                                        (77, 32, False)])
def test_half_precision(cuda, dtype, N, D, causal):
    q, k, v, w, g = oa.make_inputs(2, 2, N, D, seed=5, with_grad_out=True, dtype=dtype)
    ref = oa.attention_forward(q, k, v, w, causal=causal)[0]
    rg = oa.attention_backward(q, k, v, w, g, causal=causal)
    out, grads = run(*(t.to(cuda) for t in (q, k, v, w)), dout=g.to(cuda), causal=causal)
    assert out.dtype == dtype
    assert excess_half(out, ref) <= 0
    for a, b in zip(grads, rg):
        assert excess_half(a, b) <= 0


def test_a2_config_sampled_heads(cuda):
    """B8 H16 N2048 D64 bf16 causal, forward + backward on the GPU; parity checked on sampled
    (batch, head) slices against the oracle (the full tensor grid does not fit the oracle)."""
    B, H, N, D = 8, 16, 2048, 64
    q, k, v, w, g = oa.make_inputs(B, H, N, D, seed=0, with_grad_out=True, dtype=torch.bfloat16)
    out, grads = run(*(t.to(cuda) for t in (q, k, v, w)), dout=g.to(cuda), causal=True)
    assert torch.isfinite(out.float()).all()
    for b, h in ((0, 0), (7, 15)):
        sl = lambda t: t[b:b + 1, h:h + 1]
        ref = oa.attention_forward(sl(q), sl(k), sl(v), w[h:h + 1], causal=True, row_chunk=256)[0]
        assert excess_half(sl(out), ref) <= 0
    b, h = 3, 9
    sl = lambda t: t[b:b + 1, h:h + 1]
    rq, rk, rv, _ = oa.attention_backward(sl(q), sl(k), sl(v), w[h:h + 1], sl(g), causal=True,
                                          dtype=torch.float32)
    for a, r in zip(grads[:3], (rq, rk, rv)):
        assert excess_half(sl(a), r) <= 0
    assert torch.isfinite(grads[3]).all()


def test_v_a_broadcast_shapes(cuda):
    """v_a of shape [B, H, 1, D] (per-batch) and [1, H, 1, D] broadcast like the reference."""
    q, k, v, _, g = oa.make_inputs(3, 2, 20, 16, seed=9, with_grad_out=True)
    for wshape in ((3, 2, 1, 16), (1, 2, 1, 16), (2, 1, 16)):
        w = torch.randn(*wshape) * 0.25
        ref = oa.attention_forward(q, k, v, w)[0]
        rg = oa.attention_backward(q, k, v, w, g)
        out, grads = run(*(t.to(cuda) for t in (q, k, v, w)), dout=g.to(cuda))
        assert maxdiff(out, ref) < TOL_APPROX
        assert grads[3].shape == w.shape
        for a, b in zip(grads, rg):
            assert maxdiff(a, b) < TOL_APPROX


def test_large_weights_stable(cuda):
    """Scores far from zero (w 40x the benchmark scale, |s| up to ~30): the softmax must not
    overflow. fp32 runs in exact mode (tol 1e-4); bf16 tolerance scales with |w| (5e-2)."""
    q, k, v, w = oa.make_inputs(1, 2, 300, 64, seed=2, w_std=40.0 / 8)
    for dtype, tol, exact in ((torch.float32, 1e-4, True), (torch.bfloat16, 5e-2, False)):
        qq, kk, vv, ww = (t.to(dtype) for t in (q, k, v, w))
        ref = oa.attention_forward(qq, kk, vv, ww, causal=True)[0]
        out, _ = run(*(t.to(cuda) for t in (qq, kk, vv, ww)), causal=True, exact=exact)
        assert torch.isfinite(out.float()).all()
        assert maxdiff(out, ref) < tol


def test_empty_batch(cuda):
    from kernels import fused_additive_attention
    q = torch.zeros(0, 2, 5, 8, device=cuda)
    w = torch.zeros(2, 1, 8, device=cuda)
    assert fused_additive_attention(q, q, q, w).shape == q.shape


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N,D,causal", [(n, d, c) for (n, d) in [(1, 64), (63, 64), (65, 64),
                                                                  (129, 64), (1000, 64),
                                                                  (127, 128), (300, 128),
                                                                  (2049, 64)]
                                        for c in (False, True)])
def test_tensor_core_path_matches_generic(cuda, dtype, N, D, causal):
    """The tcgen05 forward (bf16/fp16, D in {64,128}) against the CUDA-core kernel on the same
    inputs, and both against the oracle on one head."""
    from kernels.additive_attention import attention_forward
    q, k, v, w = (t.to(cuda) for t in oa.make_inputs(2, 3, N, D, seed=N, dtype=dtype))
    fast, lse_f, _, _, _ = attention_forward(q, k, v, w, causal)
    gen, lse_g, _, _, _ = attention_forward(q, k, v, w, causal, force_generic=True)
    assert excess_half(fast, gen, ulps=1.0) <= 0
    assert maxdiff(lse_f, lse_g) < 1e-2
    ref = oa.attention_forward(q[:1, :1].cpu(), k[:1, :1].cpu(), v[:1, :1].cpu(), w[:1].cpu(),
                               causal=causal, row_chunk=256)
    assert excess_half(fast[:1, :1], ref[0]) <= 0
    assert maxdiff(lse_f[0], ref[1][0, 0]) < 1e-2


def test_saved_scores_match_oracle(cuda):
    from kernels.additive_attention import attention_forward
    N, D = 150, 64
    q, k, v, w = oa.make_inputs(1, 2, N, D, seed=8, dtype=torch.bfloat16)
    for causal in (False, True):
        for force_generic in (False, True):
            _, _, _, _, sc = attention_forward(*(t.to(cuda) for t in (q, k, v, w)), causal,
                                               force_generic=force_generic, save_scores=True)
            qq, kk, ww = q.double(), k.double(), w.double()
            ref = (torch.tanh(qq.unsqueeze(-2) + kk.unsqueeze(-3)) * ww.unsqueeze(-2)).sum(-1) / 8.0
            assert sc.shape[-1] == (N + 3) // 4 * 4  # rows padded to 16 bytes
            got = sc[..., :N].reshape(1, 2, N, N).double().cpu()
            if causal:
                mask = torch.ones(N, N, dtype=torch.bool).tril()
                got, ref = got[..., mask], ref[..., mask]
            assert (got - ref).abs().max().item() < 2e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N,causal", [(1, False), (100, True), (128, False), (129, True),
                                      (300, False), (300, True), (1000, True)])
def test_tensor_core_backward_matches_generic(cuda, dtype, N, causal):
    """The tcgen05 backward (D = 64, saved scores) against the CUDA-core backward and the
    oracle."""
    from kernels.additive_attention import attention_forward, attention_backward
    D = 64
    q, k, v, w, g = (t.to(cuda) for t in oa.make_inputs(2, 3, N, D, seed=N + 1, dtype=dtype,
                                                           with_grad_out=True))
    out, lse, table, idx, sc = attention_forward(q, k, v, w, causal, save_scores=True)
    fast = attention_backward(q, k, v, w, out, lse, g, table, idx, causal, scores=sc)
    gen = attention_backward(q, k, v, w, out, lse, g, table, idx, causal, force_generic=True)
    for a, b in zip(fast, gen):
        assert torch.isfinite(a.float()).all()
        assert excess_half(a, b, ulps=1.0) <= 0
    rg = oa.attention_backward(q[:1, :2].cpu(), k[:1, :2].cpu(), v[:1, :2].cpu(), w[:2].cpu(),
                               g[:1, :2].cpu(), causal=causal, dtype=torch.float64)
    for a, r in zip(fast[:3], rg[:3]):
        assert excess_half(a[:1, :2], r) <= 0
