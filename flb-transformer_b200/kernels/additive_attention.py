"""Fused additive attention on B200 (sm_100a).

Drop-in for the reference operator (kernels/additive_attention.py of FLB-Transformer):

    fused_additive_attention(q, k, v, v_a) -> out

    s[..., h, i, j] = sum_d v_a[..., h, 0, d] * tanh(q[..., h, i, d] + k[..., h, j, d]) / sqrt(D)
    out = softmax_j(s) @ v

q, k, v: [..., H, N, D] (any leading batch dims), v_a broadcastable to [..., H, 1, D]; the
output has q's shape and dtype. Autograd returns gradients for all four inputs, and
torch.vmap is supported (the wavefront engine vmaps it over cells). Two keyword extensions
the reference does not have: causal=True masks keys j > i, exact=True evaluates tanh/exp with
tanhf/expf instead of the hardware approximations.

The compute runs in libflb_b200.so (flb_attn_fwd / flb_attn_bwd); there is no CPU path and no
fallback: non-CUDA tensors raise.
"""
from __future__ import annotations

import math

import torch

import flb_native as nat

__all__ = ["FusedAdditiveAttentionFunc", "fused_additive_attention"]


def _w_table(v_a: torch.Tensor, q: torch.Tensor):
    """Compact float32 table of v_a rows and the per-(batch, head) row index.

    Mirrors the alignment of the reference forward (kernels/additive_attention.py:153-159):
    v_a is unsqueezed at -4 until it has q's rank and broadcast to batch_shape + (H, 1, D).
    Instead of materialising the broadcast, each flattened (batch, head) gets the index of
    the v_a row it reads; gradients are reduced into the same table.
    """
    D, H = q.shape[-1], q.shape[-3]
    batch_shape = q.shape[:-3]
    if v_a.shape[-1] != D:
        raise ValueError(f"v_a last dim {v_a.shape[-1]} != head dim {D}")
    table = v_a.detach().reshape(-1, D).to(torch.float32).contiguous()
    idx = torch.arange(table.shape[0], dtype=torch.int32, device=q.device).reshape(v_a.shape[:-1])
    while idx.ndim < q.ndim - 1:
        idx = idx.unsqueeze(-3)
    idx = torch.broadcast_to(idx, batch_shape + (H, 1)).reshape(-1).contiguous()
    return table, idx


def _flags(causal: bool, exact: bool, force_generic: bool = False) -> int:
    return ((nat.ATTN_CAUSAL if causal else 0) | (nat.ATTN_EXACT_TANH if exact else 0)
            | (nat.ATTN_FORCE_GENERIC if force_generic else 0))


def attention_forward(q, k, v, v_a, causal=False, exact=False, force_generic=False,
                      save_scores=False):
    """Run flb_attn_fwd. Returns (out [..,H,N,D], lse float32 [BH, N], w_table, w_index,
    scores float32 [BH, N, flb_attn_scores_ld(N)] or None; columns >= N are padding)."""
    nat.require_cuda(q, k, v, v_a)
    if not (q.shape == k.shape == v.shape):
        raise ValueError(f"q, k, v shapes differ: {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k and v must share a dtype")
    shape = q.shape
    D, N, H = shape[-1], shape[-2], shape[-3]
    BH = math.prod(shape[:-3]) * H
    qf = q.reshape(BH, N, D).contiguous()
    kf = k.reshape(BH, N, D).contiguous()
    vf = v.reshape(BH, N, D).contiguous()
    table, idx = _w_table(v_a, q)
    out = torch.empty_like(qf)
    lse = torch.empty((BH, N), dtype=torch.float32, device=q.device)
    scores = (torch.empty((BH, N, int(nat.lib.flb_attn_scores_ld(N))), dtype=torch.float32,
                          device=q.device)
              if save_scores else None)
    dt = nat.dtype_code(q.dtype)
    flags = _flags(causal, exact, force_generic)
    ws_bytes = nat.lib.flb_attn_fwd_workspace_bytes(BH, N, D, dt, flags)
    ws = nat.workspace(ws_bytes, q.device)
    nat.check(nat.lib.flb_attn_fwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), table.data_ptr(),
                                   idx.data_ptr(), out.data_ptr(), lse.data_ptr(),
                                   nat.ptr(scores), BH, N, D, dt, flags, nat.ptr(ws), ws_bytes,
                                   nat.stream_of(q)),
              "flb_attn_fwd")
    return out.view(shape), lse, table, idx, scores


def attention_backward(q, k, v, v_a, out, lse, grad_out, table, idx, causal=False, exact=False,
                       force_generic=False, scores=None):
    """Run flb_attn_bwd. Returns (dq, dk, dv, dv_a) shaped like the inputs."""
    shape = q.shape
    D, N, H = shape[-1], shape[-2], shape[-3]
    BH = math.prod(shape[:-3]) * H
    qf = q.reshape(BH, N, D).contiguous()
    kf = k.reshape(BH, N, D).contiguous()
    vf = v.reshape(BH, N, D).contiguous()
    of = out.reshape(BH, N, D).contiguous()
    go = grad_out.reshape(BH, N, D).contiguous()
    if go.dtype != q.dtype:
        go = go.to(q.dtype)
    dq = torch.empty_like(qf)
    dk = torch.empty_like(kf)
    dv = torch.empty_like(vf)
    dw = torch.zeros_like(table)
    dt = nat.dtype_code(q.dtype)
    flags = _flags(causal, exact, force_generic)
    ws_bytes = nat.lib.flb_attn_bwd_workspace_bytes(BH, N, D, dt, flags)
    ws = nat.workspace(ws_bytes, q.device)
    nat.check(nat.lib.flb_attn_bwd(qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), table.data_ptr(),
                                   idx.data_ptr(), of.data_ptr(), lse.data_ptr(),
                                   nat.ptr(scores), go.data_ptr(),
                                   dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dw.data_ptr(),
                                   BH, N, D, table.shape[0], dt, flags, nat.ptr(ws), ws_bytes,
                                   nat.stream_of(q)),
              "flb_attn_bwd")
    return (dq.view(shape), dk.view(shape), dv.view(shape),
            dw.view(v_a.shape).to(v_a.dtype))


# Saved scores cost 4 bytes per (query, key) pair; above this many bytes the backward
# recomputes them instead.
SAVE_SCORES_LIMIT_BYTES = 16 << 30


def _save_scores_ok(q) -> bool:
    D, N, H = q.shape[-1], q.shape[-2], q.shape[-3]
    BH = math.prod(q.shape[:-3]) * H
    return (q.dtype in (torch.bfloat16, torch.float16) and D in (64, 128)
            and BH * N * N * 4 <= SAVE_SCORES_LIMIT_BYTES)


def _unwrap_functorch(t):
    """The plain tensor inside torch.func's wrappers (first-order gradients only)."""
    from torch._C._functorch import is_functorch_wrapped_tensor, get_unwrapped
    while isinstance(t, torch.Tensor) and is_functorch_wrapped_tensor(t):
        t = get_unwrapped(t)
    return t


class FusedAdditiveAttentionFunc(torch.autograd.Function):
    """Same structure as the reference Function (kernels/additive_attention.py:135-203):
    forward / setup_context / backward / vmap, and `apply(q, k, v, v_a)` returns one tensor.
    The forward additionally keeps the row log-sum-exp for the backward (the reference saves
    only q, k, v, v_a and recomputes everything, :184-198); it travels from forward to
    setup_context on the output tensor and is detached from it there."""

    @staticmethod
    def forward(q, k, v, v_a, causal=False, exact=False):
        # grad mode is off inside Function.forward; the inputs' flags say whether a backward
        # can follow
        need_grad = any(t.requires_grad for t in (q, k, v, v_a))
        out, lse, table, idx, scores = attention_forward(
            q, k, v, v_a, causal, exact, save_scores=need_grad and _save_scores_ok(q))
        out._flb_aux = (lse, table, idx, scores)
        return out

    @staticmethod
    def setup_context(ctx, inputs, output):
        q, k, v, v_a = inputs[:4]
        causal = inputs[4] if len(inputs) > 4 else False
        exact = inputs[5] if len(inputs) > 5 else False
        ctx.causal, ctx.exact = bool(causal), bool(exact)
        # Under torch.func transforms (the wavefront engine's vjp of a cell that calls this op)
        # `output` is a functorch wrapper, not the tensor forward returned, and the auxiliary
        # tensors are not reachable; the backward then recomputes lse with one more forward.
        aux = output.__dict__.pop("_flb_aux", None)
        if aux is None:
            ctx.recompute = True
            ctx.save_for_backward(q, k, v, v_a, output)
            return
        lse, table, idx, scores = aux
        ctx.recompute = False
        ctx.has_scores = scores is not None
        extra = (scores,) if scores is not None else ()
        ctx.save_for_backward(q, k, v, v_a, output, lse, table, idx, *extra)

    @staticmethod
    @torch.compiler.disable
    def backward(ctx, grad_out):
        saved = ctx.saved_tensors
        if ctx.recompute:
            # functorch hands the saved inputs back wrapped; the kernels need their storage
            q, k, v, v_a, _ = (_unwrap_functorch(t) for t in saved)
            grad_out = _unwrap_functorch(grad_out)
            out, lse, table, idx, _ = attention_forward(q, k, v, v_a, ctx.causal, ctx.exact)
            scores = None
        else:
            q, k, v, v_a, out, lse, table, idx = saved[:8]
            scores = saved[8] if ctx.has_scores else None
        dq, dk, dv, dva = attention_backward(q, k, v, v_a, out, lse, grad_out, table, idx,
                                             ctx.causal, ctx.exact, scores=scores)
        return dq, dk, dv, dva, None, None

    @staticmethod
    def vmap(info, in_dims, q, k, v, v_a, causal=False, exact=False):
        # Physical tensors: move every vmapped dim to the front (the reference assumes it is
        # already there, :200-203), expand unbatched q/k/v, and align a vmapped v_a with q's
        # leading dim so it broadcasts over the remaining batch dims.
        size = info.batch_size
        qd, kd, vd, ad = in_dims[:4]

        def front(t, d):
            if d is None:
                return t.unsqueeze(0).expand(size, *t.shape)
            return t.movedim(d, 0)

        q, k, v = front(q, qd), front(k, kd), front(v, vd)
        if ad is not None:
            v_a = v_a.movedim(ad, 0)
            while v_a.ndim < q.ndim:
                v_a = v_a.unsqueeze(1)
        out = FusedAdditiveAttentionFunc.apply(q, k, v, v_a, causal, exact)
        return out, 0


def fused_additive_attention(q, k, v, v_a, causal: bool = False, exact: bool = False):
    """Public entry point, same signature as the reference (kernels/additive_attention.py:205)
    plus the causal/exact keywords."""
    return FusedAdditiveAttentionFunc.apply(q, k, v, v_a, causal, exact)
