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


A2_SLICES = ((0, 0), (3, 9), (7, 15))


@pytest.fixture(scope="module")
def a2_run(cuda):
    """B8 H16 N2048 D64 bf16 causal: one forward + backward of the whole configuration on the
    GPU (the launch the benchmark times), kept for the parity checks below."""
    B, H, N, D = 8, 16, 2048, 64
    q, k, v, w, g = oa.make_inputs(B, H, N, D, seed=0, with_grad_out=True, dtype=torch.bfloat16)
    out, grads = run(*(t.to(cuda) for t in (q, k, v, w)), dout=g.to(cuda), causal=True)
    return (q, k, v, w, g), out.cpu(), [t.cpu() for t in grads]


def test_a2_config_sampled_heads(a2_run):
    """Forward output and every input gradient of the full A2 launch, checked on three sampled
    (batch, head) slices (first, middle, last) against the oracle (the full tensors do not fit
    the oracle's memory; the slices are whole: every query row and key of the unit)."""
    (q, k, v, w, g), out, grads = a2_run
    assert torch.isfinite(out.float()).all()
    for b, h in A2_SLICES:
        sl = lambda t: t[b:b + 1, h:h + 1]
        ref = oa.attention_forward(sl(q), sl(k), sl(v), w[h:h + 1], causal=True, row_chunk=256)[0]
        assert excess_half(sl(out), ref) <= 0, (b, h)
        rq, rk, rv, _ = oa.attention_backward(sl(q), sl(k), sl(v), w[h:h + 1], sl(g),
                                              causal=True, dtype=torch.float32, row_chunk=64)
        for name, a, r in zip(("dq", "dk", "dv"), grads[:3], (rq, rk, rv)):
            assert excess_half(sl(a), r) <= 0, (name, b, h)


def test_a2_dv_a_all_units(a2_run):
    """dv_a is the one reduction across (batch, head) units: each head's row of the gradient
    sums the contributions of all 8 batch elements (atomics from every key block of every unit
    in the kernel). Checked against the oracle's grad_va evaluated on the host in float32 for
    all 128 units. Each head's row sums ~17 M products dS * tanh with heavy cancellation (every
    softmax row's dS sums to zero) to values of magnitude ~8, where a bf16 ulp alone is 0.06, so
    the error is bounded relative to the tensor's largest magnitude, as for the grid layer's
    weight gradients: max|a - ref| <= 2e-2 * max(1, max|ref|)."""
    (q, k, v, w, g), _, grads = a2_run
    B, H = q.shape[:2]
    ref = torch.zeros(H, 1, q.shape[-1], dtype=torch.float64)
    for b in range(B):
        for h in range(H):
            sl = lambda t: t[b:b + 1, h:h + 1]
            ref[h] += oa.attention_backward(sl(q), sl(k), sl(v), w[h:h + 1], sl(g), causal=True,
                                            dtype=torch.float32, row_chunk=64)[3][0].double()
    dva = grads[3]
    assert dva.shape == w.shape and dva.dtype == w.dtype
    scale = max(1.0, ref.abs().max().item())
    assert maxdiff(dva, ref) <= 2e-2 * scale


A3_RESCALE_HEAD = 5
A3_SLICES = ((0, 0), (3, 7), (1, A3_RESCALE_HEAD))
A3_ROWS = ((0, 128), (4032, 4160), (8064, 8192))


@pytest.fixture(scope="module")
def a3_run(cuda):
    """B4 H8 N8192 D128 bf16 causal forward of the whole configuration on the GPU. Head 5 is set
    up so that the kernel's row-rescale path runs on every row i >= 8: its score vector is
    w ~ N(0, 1) and its keys 0-7 are -8 sign(w), so the first key group of every row scores about
    -sum|w|/sqrt(D) (~ -9, ~ -13 in log2 units) and later keys exceed that first-group maximum by
    more than the kernel's threshold (8 log2 units)."""
    from kernels.additive_attention import attention_forward
    B, H, N, D = 4, 8, 8192, 128
    q, k, v, w = oa.make_inputs(B, H, N, D, seed=7, dtype=torch.bfloat16)
    w, k = w.clone(), k.clone()
    gw = torch.Generator().manual_seed(70)
    w[A3_RESCALE_HEAD] = torch.randn(1, D, generator=gw).bfloat16()
    k[:, A3_RESCALE_HEAD, :8, :] = (-8.0 * torch.sign(w[A3_RESCALE_HEAD].float())).bfloat16()
    out, lse, _, _, _ = attention_forward(*(t.to(cuda) for t in (q, k, v, w)), True)
    return (q, k, v, w), out.cpu(), lse.view(B, H, N).cpu()


def _check_a3_rows(q, k, v, out, lse, cases):
    """out/lse [b, h, N, ...] of the cases (b, h, score vector [1, 1, D], rescale head?) against
    the oracle on the first, a middle and the last 128 query rows; returns how many sampled rows
    of rescale heads take the rescale path (from the oracle's scores)."""
    rescaled_rows = 0
    for b, h, wv, rescale in cases:
        sl = lambda t: t[b:b + 1, h:h + 1]
        tol = 5e-2 if rescale else TOL_HALF
        for r0, r1 in A3_ROWS:
            ref_o, ref_l = oa.attention_forward(sl(q), sl(k), sl(v), wv, causal=True,
                                                row_range=(r0, r1), row_chunk=32)
            got = out[b, h, r0:r1].double()
            excess = ((got - ref_o[0, 0]).abs() - (tol + 2.0 ** -8 * ref_o[0, 0].abs())).max()
            assert excess.item() <= 0, (b, h, r0)
            assert maxdiff(lse[b, h, r0:r1], ref_l[0, 0]) < 1e-2, (b, h, r0)
            if rescale:
                s2 = oa.attention_scores(sl(q), sl(k), wv, causal=True,
                                         row_range=(r0, r1), dtype=torch.float32)[0, 0]
                s2 = s2 * 1.4426950408889634  # log2 units, as the kernel compares
                first = s2[:, :8].max(dim=-1).values
                rescaled_rows += int((s2.max(dim=-1).values > first + 8.0).sum())
    return rescaled_rows


def test_a3_config_sampled_rows(a3_run):
    """Long-context configuration B4 H8 N8192 D128 bf16 causal, forward, the whole launch on the
    GPU (32 units: one CTA per query block); output and lse checked against the oracle on
    sampled rows of three (batch, head) slices (each softmax row is independent, so sampled rows
    are exact checks), one of them the head set up to take the rescale path (confirmed on the
    oracle's scores). Bound: 2e-2 plus half a bf16 ulp; for the rescale head 5e-2 (score errors
    grow with sum|w|, as in test_large_weights_stable). lse: 1e-2 absolute."""
    (q, k, v, w), out, lse = a3_run
    assert torch.isfinite(out.float()).all()
    cases = [(b, h, w[h:h + 1], h == A3_RESCALE_HEAD) for b, h in A3_SLICES]
    assert _check_a3_rows(q, k, v, out, lse, cases) >= 3 * 128 - 8


def test_a3_shard_of_four_units_splits_blocks(cuda, a3_run):
    """The long-context configuration's share of one GPU out of eight: 4 (batch, head) units.
    With that few CTAs the causal forward splits each query block but the first into two
    key-range halves merged by a combine kernel. Checked against the oracle on sampled rows
    (the rescale head among them) and against the unsplit 32-unit launch on the same units
    (one bf16 ulp plus 2e-2; lse 1e-2)."""
    from kernels.additive_attention import attention_forward
    import flb_native as nat
    (q, k, v, w), out_all, lse_all = a3_run
    units = [(1, 2), (1, 3), (1, 4), (1, A3_RESCALE_HEAD)]
    qs, ks, vs = (torch.stack([t[b, h] for b, h in units]).unsqueeze(1) for t in (q, k, v))
    ws = torch.stack([w[h] for _, h in units]).unsqueeze(1)          # [4, 1, 1, D]
    ws_bytes = nat.lib.flb_attn_fwd_workspace_bytes(4, 8192, 128, nat.BF16, nat.ATTN_CAUSAL)
    assert ws_bytes > 256  # the split path is the one taken at this size
    out, lse, _, _, _ = attention_forward(*(t.to(cuda) for t in (qs, ks, vs, ws)), True)
    out, lse = out.cpu(), lse.view(4, 1, -1).cpu()
    for i, (b, h) in enumerate(units):
        assert excess_half(out[i, 0], out_all[b, h], ulps=1.0) <= 0, (b, h)
        assert maxdiff(lse[i, 0], lse_all[b, h]) < 1e-2
    cases = [(i, 0, ws[i], h == A3_RESCALE_HEAD) for i, (_, h) in enumerate(units)
             if i in (0, 3)]
    assert _check_a3_rows(qs, ks, vs, out, lse, cases) >= 128 * 3 - 8


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
