"""Native forward of FLB block cells on the wavefront grid (inference).

When an engine's layers are FLB blocks (the reference's FLB_Block / FLB_Attention_Layer, or
flb_model's FLBBlock / FLBAttentionLayer: same math and parameter names) on the FLB grid
configuration (dependencies top -> port 0, left -> port 1, bottom-left -> port 2, four ports)
and no gradient is needed, the engine evaluates the whole grid with flb_block_grid_fwd: per
tick a handful of launches over all of the tick's cells (strided GEMMs on the stacked weights
read in place, LayerNorm, gate, three-token attention and residual kernels) instead of the
per-tick gather, weight index_select, vmapped cell and scatters. bf16 compute only (the
reference model runs under bf16 autocast). Training (a backward) keeps the generic path.
"""
from __future__ import annotations

import ctypes

import torch

import flb_native as nat

_FLB_DEPS = [((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)]
_BLOCK_TYPES = ("FLB_Block", "FLBBlock")
_ATTN_TYPES = ("FLB_Attention_Layer", "FLBAttentionLayer")


def _is_flb_block(m) -> bool:
    a = getattr(m, "flb_attention", None)
    if type(m).__name__ not in _BLOCK_TYPES or type(a).__name__ not in _ATTN_TYPES:
        return False
    try:
        return (m.proj_lateral.bias is None and m.proj_feedback.bias is None
                and m.norm_lat.weight is not None and m.norm_fdbk.weight is not None
                and a.linear_gate_L.bias is not None and a.linear_gate_X.bias is not None
                and all(getattr(a, n).bias is None for n in ("W_q", "W_k", "W_v", "W_o")))
    except AttributeError:
        return False


def native_flb_applies(engine, x: torch.Tensor) -> bool:
    """Whether engine(x) can run as flb_block_grid_fwd (forward only)."""
    if not getattr(engine, "native_cells", True):
        return False
    cfg = engine.config
    layers = list(engine.layers)
    deps = [(tuple(o), p) for o, p in cfg.dependencies]
    if deps != _FLB_DEPS or cfg.num_ports != 4 or len(cfg.grid_shape) != 2:
        return False
    if not layers or len(layers) != cfg.grid_shape[0] or not all(_is_flb_block(l) for l in layers):
        return False
    compute = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype
    D = cfg.dim
    H = layers[0].flb_attention.num_heads
    eps = layers[0].norm_lat.eps
    same = all(l.flb_attention.num_heads == H and l.norm_lat.eps == eps and l.norm_fdbk.eps == eps
               for l in layers)
    return (same and compute == torch.bfloat16 and D % 16 == 0 and D % H == 0 and D <= 1024
            and D // H <= 128
            and tuple(x.shape) == (cfg.batch_size, cfg.grid_shape[1], D))


def no_grad_needed(engine, x) -> bool:
    if not torch.is_grad_enabled():
        return True
    return not (x.requires_grad or any(p.requires_grad for p in engine.layers.parameters()))


class BlockWeightStacks:
    """The layers' weights as per-layer stacks in the layout flb_block_grid_fwd reads (bf16
    matrices, float32 vectors), built from the live parameters."""

    def __init__(self, layers):
        with torch.no_grad():
            def st(get, dtype):
                return torch.stack([get(l) for l in layers]).to(dtype).contiguous()
            bf, f32 = torch.bfloat16, torch.float32
            a = [l.flb_attention for l in layers]
            H, dh = a[0].num_heads, a[0].head_dim
            self.t = {
                "ln_lat_w": st(lambda l: l.norm_lat.weight, f32),
                "ln_lat_b": st(lambda l: l.norm_lat.bias, f32),
                "ln_fdbk_w": st(lambda l: l.norm_fdbk.weight, f32),
                "ln_fdbk_b": st(lambda l: l.norm_fdbk.bias, f32),
                "w_prior_lat": st(lambda l: l.proj_lateral.weight, bf),
                "w_prior_fdbk": st(lambda l: l.proj_feedback.weight, bf),
                "w_gate_l": st(lambda l: l.flb_attention.linear_gate_L.weight, bf),
                "b_gate_l": st(lambda l: l.flb_attention.linear_gate_L.bias, f32),
                "w_gate_x": st(lambda l: l.flb_attention.linear_gate_X.weight, bf),
                "b_gate_x": st(lambda l: l.flb_attention.linear_gate_X.bias, f32),
                "w_qkv": st(lambda l: torch.cat([l.flb_attention.W_q.weight,
                                                 l.flb_attention.W_k.weight,
                                                 l.flb_attention.W_v.weight], 0), bf),
                "w_o": st(lambda l: l.flb_attention.W_o.weight, bf),
                "v_a": st(lambda l: l.flb_attention.v_a.reshape(H, dh), f32),
            }
        self.struct = nat.BlockWeights(**{k: v.data_ptr() for k, v in self.t.items()})
        self.heads = H
        self.eps = float(layers[0].norm_lat.eps)


def native_flb_forward(engine, static_x: torch.Tensor, grids: torch.Tensor, weights=None) -> None:
    """Evaluate every cell of the engine's grid into `grids` ([ports, cells + L, batch, dim],
    bf16) from static_x ([batch, seq, dim], bf16), with the layers' current weights."""
    cfg = engine.config
    L, S = cfg.grid_shape
    B, D = cfg.batch_size, cfg.dim
    w = weights or BlockWeightStacks(list(engine.layers))
    ws_bytes = nat.lib.flb_block_grid_workspace_bytes(L, S, B, D)
    ws = nat.workspace(ws_bytes, grids.device)
    nat.check(nat.lib.flb_block_grid_fwd(
        ctypes.cast(ctypes.pointer(w.struct), ctypes.c_void_p), static_x.data_ptr(), grids.data_ptr(), L, S, B, D, w.heads,
        w.eps, nat.ptr(ws), ws_bytes, nat.stream_of(grids)), "flb_block_grid_fwd")
