"""Greedy decoding for FLBTransformer (the reference has no decode API).

The model's grid has a fixed width seq_len and its carried contexts reach no cell (the
engine's routing never reads the boundary dock), so a step re-runs the whole grid over the
last seq_len tokens (a sliding window) and appends the argmax of the last position's logits.
With `graphed=True` the engine's forward tick loop is captured once as a CUDA graph and every
step is one graph replay.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def greedy_decode(model, prompt: torch.Tensor, steps: int, graphed: bool = True, engine=None):
    """prompt [batch, seq_len] int64 token ids -> [batch, steps] generated ids. `engine` may
    pass in a GraphedWavefrontEngine captured earlier (for repeated decodes)."""
    from wavefront.wavefront_graph import GraphedWavefrontEngine
    if prompt.dim() != 2 or prompt.shape[1] != model.config.grid_shape[1]:
        raise ValueError(f"prompt must be [batch, {model.config.grid_shape[1]}]")
    window = prompt.clone()
    if engine is None and graphed and steps > 0:
        x = model.emb_dropout(model.embedding(window))
        engine = GraphedWavefrontEngine(model.engine, x, backward=False)
    out = torch.empty(prompt.shape[0], steps, dtype=prompt.dtype, device=prompt.device)
    for s in range(steps):
        logits, _, _ = model(window, engine=engine)
        nxt = logits[:, -1].argmax(-1)
        out[:, s] = nxt
        window = torch.cat([window[:, 1:], nxt[:, None]], dim=1)
    return out
