"""CPU oracle for the fused additive attention (TEST INFRASTRUCTURE ONLY).

Restates the reference's eager ground truth so the CUDA kernels can be checked against it.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may use it;
the product path never does.

  forward  : kernels/kernel_tests.py:8-29 (pure_torch_additive_attention): tanh of the
             broadcast sum, times v_a, summed over d, divided by sqrt(D), softmax, matmul.
  backward : kernels/additive_attention.py:91-130 (compiled_backward_math), written out
             explicitly (dV = P^T dO, dP = dO V^T, dS = P (dP - rowsum(P dP)) / sqrt(D),
             dQ = sum_j dS w (1-t^2), dK = sum_i dS w (1-t^2), dw = sum dS t reduced over the
             broadcast dims of v_a).
  causal   : an extension the reference does not have: scores with j > i are set to -inf
             before the softmax.

Everything is evaluated in float64 (or the dtype passed) from the given inputs; bf16/f16
inputs are first converted, so the oracle is the reference math on the same input values.
Large configurations are evaluated by query-row chunks (the forward is row-independent) and,
for the backward, on whole (batch, head) slices.
"""
from __future__ import annotations

import math

import torch


def _align_va(v_a: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """v_a [..., H, 1, D] aligned to q's rank (kernels/additive_attention.py:153-155)."""
    while v_a.ndim < q.ndim:
        v_a = v_a.unsqueeze(-4)
    return v_a


def attention_forward(q, k, v, v_a, causal=False, dtype=torch.float64, row_chunk=None,
                      row_range=None):
    """Oracle forward. Returns (out, lse) in `dtype`; lse is the natural-log row logsumexp of
    the scaled scores, shape q.shape[:-1]. With row_range=(r0, r1) only query rows r0..r1-1 are
    evaluated (each softmax row is independent of the others) and the results hold those rows."""
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    w = _align_va(v_a.to(dtype), q)  # [..., H, 1, D]
    D, N = q.shape[-1], q.shape[-2]
    scale = math.sqrt(D)
    r0, r1 = row_range if row_range is not None else (0, N)
    chunk = row_chunk or max(1, r1 - r0)
    outs, lses = [], []
    for i0 in range(r0, r1, chunk):
        qi = q[..., i0:min(r1, i0 + chunk), :]
        inter = torch.tanh(qi.unsqueeze(-2) + k.unsqueeze(-3))          # [..., n, N, D]
        scores = (inter * w.unsqueeze(-2)).sum(dim=-1) / scale         # [..., n, N]
        if causal:
            rows = torch.arange(i0, i0 + qi.shape[-2]).unsqueeze(-1)
            cols = torch.arange(N).unsqueeze(0)
            scores = scores.masked_fill(cols > rows, float("-inf"))
        lses.append(torch.logsumexp(scores, dim=-1))
        attn = torch.softmax(scores, dim=-1)
        outs.append(torch.matmul(attn, v))
    return torch.cat(outs, dim=-2), torch.cat(lses, dim=-1)


def attention_scores(q, k, v_a, causal=False, dtype=torch.float64, row_range=None):
    """The scaled scores s[..., i, j] = sum_d v_a[d] tanh(q[i, d] + k[j, d]) / sqrt(D) of query
    rows row_range (default all), masked to -inf above the diagonal when causal
    (kernels/kernel_tests.py:19-23)."""
    q, k = q.to(dtype), k.to(dtype)
    w = _align_va(v_a.to(dtype), q)
    D, N = q.shape[-1], q.shape[-2]
    r0, r1 = row_range if row_range is not None else (0, N)
    qi = q[..., r0:r1, :]
    s = (torch.tanh(qi.unsqueeze(-2) + k.unsqueeze(-3)) * w.unsqueeze(-2)).sum(dim=-1) / math.sqrt(D)
    if causal:
        rows = torch.arange(r0, r1).unsqueeze(-1)
        s = s.masked_fill(torch.arange(N).unsqueeze(0) > rows, float("-inf"))
    return s


def attention_backward(q, k, v, v_a, grad_out, causal=False, dtype=torch.float64, row_chunk=None):
    """Oracle backward (explicit restatement of compiled_backward_math).
    Returns (dq, dk, dv, dv_a) in `dtype`, dv_a shaped like v_a.

    With row_chunk, query rows are processed in chunks of that many rows: a softmax row needs
    only its own scores, so each chunk forms P, dP and dS for its rows over all keys, writes its
    rows of dq, and adds its contributions to dk, dv and dv_a (the sums over query rows). When
    causal, a chunk ending at row i1 reads only keys < i1 (the rest are masked to zero weight).
    The result is the same math as the unchunked form, in bounded memory."""
    q, k, v, g = q.to(dtype), k.to(dtype), v.to(dtype), grad_out.to(dtype)
    va = v_a.to(dtype)
    w = _align_va(va, q)
    D, N = q.shape[-1], q.shape[-2]
    scale = math.sqrt(D)
    wv = w.unsqueeze(-2)                                                # [..., 1, 1, D]
    chunk = row_chunk or N
    grad_q = torch.zeros_like(q)
    grad_k = torch.zeros_like(k)
    grad_v = torch.zeros_like(v)
    grad_w_full = None
    for i0 in range(0, N, chunk):
        i1 = min(N, i0 + chunk)
        kend = i1 if causal else N
        qi, gi = q[..., i0:i1, :], g[..., i0:i1, :]
        kk, vv = k[..., :kend, :], v[..., :kend, :]
        inter = torch.tanh(qi.unsqueeze(-2) + kk.unsqueeze(-3))        # [..., n, kend, D]
        scores = (inter * wv).sum(dim=-1) / scale
        if causal:
            rows = torch.arange(i0, i1).unsqueeze(-1)
            cols = torch.arange(kend).unsqueeze(0)
            scores = scores.masked_fill(cols > rows, float("-inf"))
        attn = torch.softmax(scores, dim=-1)
        grad_v[..., :kend, :] += torch.matmul(attn.transpose(-1, -2), gi)
        grad_attn = torch.matmul(gi, vv.transpose(-1, -2))
        grad_scores = attn * (grad_attn - (attn * grad_attn).sum(dim=-1, keepdim=True)) / scale
        pre = grad_scores.unsqueeze(-1) * wv * (1.0 - inter ** 2)
        grad_q[..., i0:i1, :] = pre.sum(dim=-2)
        grad_k[..., :kend, :] += pre.sum(dim=-3)
        part = (grad_scores.unsqueeze(-1) * inter).sum(dim=(-2, -3))   # [..., H, D]
        grad_w_full = part if grad_w_full is None else grad_w_full + part
    if grad_w_full is None:  # N == 0
        grad_w_full = torch.zeros(q.shape[:-2] + (D,), dtype=dtype)
    grad_w_full = grad_w_full.unsqueeze(-2)                              # [..., H, 1, D]
    # reduce over the dims the aligned v_a was broadcast along, then drop the aligning dims
    grad_va = grad_w_full
    for d in range(w.ndim):
        if w.shape[d] == 1 and grad_va.shape[d] != 1:
            grad_va = grad_va.sum(dim=d, keepdim=True)
    return grad_q, grad_k, grad_v, grad_va.reshape(va.shape)


def make_inputs(B, H, N, D, dtype=torch.float32, seed=0, device="cpu", w_std=None,
                with_grad_out=False):
    """Seeded synthetic inputs with the distributions of the benchmark configurations:
    Q, K, V ~ N(0, 1); w ~ N(0, 1/D) shaped [H, 1, D]; optional dO ~ N(0, 1)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, H, N, D, generator=gen)
    k = torch.randn(B, H, N, D, generator=gen)
    v = torch.randn(B, H, N, D, generator=gen)
    std = (1.0 / math.sqrt(D)) if w_std is None else w_std
    w = torch.randn(H, 1, D, generator=gen) * std
    out = [q.to(dtype).to(device), k.to(dtype).to(device), v.to(dtype).to(device),
           w.to(dtype).to(device)]
    if with_grad_out:
        out.append(torch.randn(B, H, N, D, generator=gen).to(dtype).to(device))
    return out
