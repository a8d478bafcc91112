"""Native forward and backward of FLB block cells on the wavefront grid.

When an engine's layers are FLB blocks (the reference's FLB_Block / FLB_Attention_Layer, or
flb_model's FLBBlock / FLBAttentionLayer: same math and parameter names) on the FLB grid
configuration (dependencies top -> port 0, left -> port 1, bottom-left -> port 2, four ports),
the engine evaluates the whole grid with flb_block_grid_fwd: per tick a handful of launches
over all of the tick's cells (strided GEMMs on the stacked weights read in place, LayerNorm,
gate, three-token attention and residual kernels) instead of the per-tick gather, weight
index_select, vmapped cell and scatters. With gradients required it runs behind
FLBGridFunction, whose backward is flb_block_grid_bwd (ticks in reverse, per-tick recompute,
per-layer fp32 weight-gradient stacks). bf16 compute only (the reference model runs under bf16
autocast). Setting engine.native_flb_path = 2 (FLB_BLOCK_PATH_PERSISTENT) runs the inference
forward as one persistent tcgen05 kernel instead (batch 16, d_model a multiple of 128). A
training forward keeps every cell's intermediates (flb_block_grid_fwd_save) so that the backward
restores them instead of recomputing its ticks' forward stages, and keeps the gradients that
meet the weights beside them to form every weight gradient in a few large GEMMs at its end;
engine.native_flb_save = False trades that memory (L * S * 36 * batch * d_model bf16) for the
recompute and per-tick weight-gradient GEMMs.
"""
from __future__ import annotations

import ctypes
import math

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


def saved_buffer(engine, device) -> torch.Tensor | None:
    """The engine's buffer for a training forward's per-cell intermediates
    (flb_block_grid_saved_bytes), or None when engine.native_flb_save is False (the backward
    then recomputes each tick's forward stages). One buffer per engine, like its static grids:
    a forward overwrites what the previous one kept."""
    if not getattr(engine, "native_flb_save", True):
        return None
    cfg = engine.config
    L, S = cfg.grid_shape
    nbytes = nat.lib.flb_block_grid_saved_bytes(L, S, cfg.batch_size, cfg.dim)
    ws = engine.graph_workspace
    buf = ws.get("flb_saved")
    if buf is None or buf.numel() != nbytes or buf.device != torch.device(device):
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        ws["flb_saved"] = buf
    return buf


def native_flb_forward(engine, static_x: torch.Tensor, grids: torch.Tensor, weights=None,
                       saved: torch.Tensor | None = None) -> None:
    """Evaluate every cell of the engine's grid into `grids` ([ports, cells + L, batch, dim],
    bf16) from static_x ([batch, seq, dim], bf16), with the layers' current weights. With
    `saved` (saved_buffer) the cells' intermediates are kept for native_flb_backward."""
    cfg = engine.config
    L, S = cfg.grid_shape
    B, D = cfg.batch_size, cfg.dim
    w = weights or BlockWeightStacks(list(engine.layers))
    ws_bytes = nat.lib.flb_block_grid_workspace_bytes(L, S, B, D)
    ws = nat.workspace(ws_bytes, grids.device)
    wptr = ctypes.cast(ctypes.pointer(w.struct), ctypes.c_void_p)
    if saved is not None:
        nat.check(nat.lib.flb_block_grid_fwd_save(
            wptr, static_x.data_ptr(), grids.data_ptr(), L, S, B, D, w.heads, w.eps, nat.ptr(ws),
            ws_bytes, saved.data_ptr(), saved.numel(), nat.stream_of(grids)),
            "flb_block_grid_fwd_save")
        return
    # engine.native_flb_path: FLB_BLOCK_PATH_* (0 = the default, 2 = the persistent kernel)
    path = int(getattr(engine, "native_flb_path", 0))
    nat.check(nat.lib.flb_block_grid_fwd_ex(
        wptr, static_x.data_ptr(), grids.data_ptr(), L, S, B, D, w.heads,
        w.eps, nat.ptr(ws), ws_bytes, path, nat.stream_of(grids)), "flb_block_grid_fwd_ex")


# parameter name inside a block -> (gradient stack, slice of its per-layer entry)
def _grad_slot(name: str, D: int):
    table = {
        "norm_lat.weight": ("ln_lat_w", None), "norm_lat.bias": ("ln_lat_b", None),
        "norm_fdbk.weight": ("ln_fdbk_w", None), "norm_fdbk.bias": ("ln_fdbk_b", None),
        "proj_lateral.weight": ("w_prior_lat", None),
        "proj_feedback.weight": ("w_prior_fdbk", None),
        "flb_attention.linear_gate_L.weight": ("w_gate_l", None),
        "flb_attention.linear_gate_L.bias": ("b_gate_l", None),
        "flb_attention.linear_gate_X.weight": ("w_gate_x", None),
        "flb_attention.linear_gate_X.bias": ("b_gate_x", None),
        "flb_attention.W_q.weight": ("w_qkv", slice(0, D)),
        "flb_attention.W_k.weight": ("w_qkv", slice(D, 2 * D)),
        "flb_attention.W_v.weight": ("w_qkv", slice(2 * D, 3 * D)),
        "flb_attention.W_o.weight": ("w_o", None),
        "flb_attention.v_a": ("v_a", None),
    }
    return table[name]


class FLBGridFunction(torch.autograd.Function):
    """The FLB grid, forward and backward in the native kernels. apply(engine, x, *params) with
    params = every block's parameters in (layer, named_parameters) order; returns the four port
    grids (views of the engine's static grids, as the per-tick engine returns)."""

    @staticmethod
    def forward(ctx, engine, x, *params):
        engine._init_buffers(x)
        ws = engine.graph_workspace
        ws["static_x"].copy_(x)
        w = BlockWeightStacks(list(engine.layers))
        saved = saved_buffer(engine, x.device)
        native_flb_forward(engine, ws["static_x"], ws["static_stacked_grids"], weights=w,
                           saved=saved)
        ctx.engine, ctx.weights, ctx.saved = engine, w, saved
        ctx.x_meta = (x.shape, x.dtype)
        n = math.prod(engine.config.grid_shape)
        return tuple(ws["static_stacked_grids"][p][:n] for p in range(engine.config.num_ports))

    @staticmethod
    def backward(ctx, *grad_grids):
        gstacks, dx = native_flb_backward(ctx.engine, ctx.weights, grad_grids, saved=ctx.saved)
        shape, dtype = ctx.x_meta
        return (None, dx.to(dtype).reshape(shape), *flb_param_grads(ctx.engine, gstacks))


def native_flb_backward(engine, w, grad_grids, saved: torch.Tensor | None = None):
    """flb_block_grid_bwd over the engine's saved grids (flb_block_grid_bwd_saved with the
    forward's intermediates when `saved` holds them): (fp32 gradient stacks keyed like the
    weight stacks, dx float32 [batch, seq, dim])."""
    cfg = engine.config
    L, S = cfg.grid_shape
    B, D = cfg.batch_size, cfg.dim
    ws = engine.graph_workspace
    dev = ws["static_x"].device
    gstacks = {k: torch.zeros(v.shape, dtype=torch.float32, device=dev) for k, v in w.t.items()}
    gstruct = nat.BlockGrads(**{k: v.data_ptr() for k, v in gstacks.items()})
    dg = [g.to(torch.bfloat16).contiguous() if g is not None else None for g in grad_grids]
    dx = torch.empty((B, S, D), dtype=torch.float32, device=dev)
    ws_bytes = nat.lib.flb_block_grid_bwd_workspace_bytes(L, S, B, D)
    wsb = nat.workspace(ws_bytes, dev)
    args = (ctypes.cast(ctypes.pointer(w.struct), ctypes.c_void_p), ws["static_x"].data_ptr(),
            ws["static_stacked_grids"].data_ptr(), *[nat.ptr(g) for g in dg], dx.data_ptr(),
            ctypes.cast(ctypes.pointer(gstruct), ctypes.c_void_p), L, S, B, D, w.heads, w.eps,
            nat.ptr(wsb), ws_bytes)
    if saved is not None:
        nat.check(nat.lib.flb_block_grid_bwd_saved(*args, saved.data_ptr(), saved.numel(),
                                                   nat.stream_of(dx)), "flb_block_grid_bwd_saved")
    else:
        nat.check(nat.lib.flb_block_grid_bwd(*args, nat.stream_of(dx)), "flb_block_grid_bwd")
    return gstacks, dx


def flb_param_grads(engine, gstacks):
    """Per-parameter gradients (each parameter's shape and dtype, in (layer, named_parameters)
    order) from the fp32 gradient stacks."""
    D = engine.config.dim
    grads = []
    for li, layer in enumerate(engine.layers):
        for name, p in layer.named_parameters():
            key, sl = _grad_slot(name, D)
            gl = gstacks[key][li]
            if sl is not None:
                gl = gl[sl]
            grads.append(gl.reshape(p.shape).to(p.dtype, copy=True))
    return grads


def native_flb_train_forward(engine, x):
    params = [p for layer in engine.layers for _, p in layer.named_parameters()]
    return FLBGridFunction.apply(engine, x, *params)
