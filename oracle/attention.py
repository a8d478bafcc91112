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


def attention_forward(q, k, v, v_a, causal=False, dtype=torch.float64, row_chunk=None):
    """Oracle forward. Returns (out, lse) in `dtype`; lse is the natural-log row logsumexp of
    the scaled scores, shape q.shape[:-1]."""
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    w = _align_va(v_a.to(dtype), q)  # [..., H, 1, D]
    D, N = q.shape[-1], q.shape[-2]
    scale = math.sqrt(D)
    chunk = row_chunk or N
    outs, lses = [], []
    for i0 in range(0, N, chunk):
        qi = q[..., i0:i0 + chunk, :]
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


def attention_backward(q, k, v, v_a, grad_out, causal=False, dtype=torch.float64):
    """Oracle backward (explicit restatement of compiled_backward_math).
    Returns (dq, dk, dv, dv_a) in `dtype`, dv_a shaped like v_a."""
    q, k, v, g = q.to(dtype), k.to(dtype), v.to(dtype), grad_out.to(dtype)
    va = v_a.to(dtype)
    w = _align_va(va, q)
    D, N = q.shape[-1], q.shape[-2]
    scale = math.sqrt(D)
    inter = torch.tanh(q.unsqueeze(-2) + k.unsqueeze(-3))               # [..., N, N, D]
    wv = w.unsqueeze(-2)                                                # [..., 1, 1, D]
    scores = (inter * wv).sum(dim=-1) / scale
    if causal:
        mask = torch.ones(N, N, dtype=torch.bool).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    attn = torch.softmax(scores, dim=-1)
    grad_v = torch.matmul(attn.transpose(-1, -2), g)
    grad_attn = torch.matmul(g, v.transpose(-1, -2))
    grad_scores = attn * (grad_attn - (attn * grad_attn).sum(dim=-1, keepdim=True)) / scale
    pre = grad_scores.unsqueeze(-1) * wv * (1.0 - inter ** 2)
    grad_q = pre.sum(dim=-2)
    grad_k = pre.sum(dim=-3)
    grad_w_full = (grad_scores.unsqueeze(-1) * inter).sum(dim=(-2, -3), keepdim=False)  # [..., H, D]
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
