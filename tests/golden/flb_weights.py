"""Deterministic FLB model weights for goldens that must not store them.

set_hashed_weights(model, seed) fills every parameter of an FLB model (this package's FLBTransformer
or the reference's FLB_Transformer: same parameter names) from numpy's RandomState(seed), whose
stream is fixed across numpy versions, walking the parameters in sorted-name order. Values are
rounded to bf16-representable floats so that a bf16 copy of the model holds exactly the weights
the float32 golden ran with. Scales: LayerNorm weight 1 + 0.1 u and bias 0.1 u, v_a 0.5 n (so the
attention weights matter), embedding n, other weights and biases u / sqrt(fan_in), with u
uniform in [-1, 1) and n standard normal.
"""
from __future__ import annotations

import numpy as np
import torch


def set_hashed_weights(model: torch.nn.Module, seed: int) -> None:
    rs = np.random.RandomState(seed)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name in sorted(params):
            p = params[name]
            shape = tuple(p.shape)
            if "norm" in name:
                u = rs.uniform(-1.0, 1.0, shape)
                v = 1.0 + 0.1 * u if name.endswith("weight") else 0.1 * u
            elif name.endswith("v_a"):
                v = 0.5 * rs.standard_normal(shape)
            elif name.startswith("embedding"):
                v = rs.standard_normal(shape)
            else:
                fan_in = shape[-1] if name.endswith("weight") else model_dim(params)
                v = rs.uniform(-1.0, 1.0, shape) / np.sqrt(fan_in)
            t = torch.from_numpy(np.asarray(v, dtype=np.float32))
            p.copy_(t.to(torch.bfloat16).to(torch.float32))


def model_dim(params) -> int:
    return int(params["embedding.weight"].shape[1])
