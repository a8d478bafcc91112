"""Data-parallel use of the wavefront grid layer and engine across the GPUs of one node.

The batch rows of a grid are independent (every cell's GEMMs are row-wise in the batch), so a
job shards the batch over ranks with no collective on the data path: each rank runs the whole
grid on its rows. The layer's weights are replicated parameters; their gradients are sums over
the batch, so the one exchange step is an all-reduce of the weight gradients after the backward
(3 H^2 + H floats for the tanh cell, ~787 KB at H = 256), issued as one flattened buffer.

Plain torch.distributed code: NCCL on GPUs, gloo for the CPU tests of the host-side logic.
"""
from __future__ import annotations

import torch

from kernels.sharding import shard_range


def shard_batch(t: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """This rank's contiguous slice of `t` along its batch dimension `dim` (a view)."""
    start, stop = shard_range(t.shape[dim], rank, world)
    return t.narrow(dim, start, stop - start)


def all_reduce_grads(params, group=None) -> None:
    """Sum the .grad of every parameter in `params` over the ranks of `group`, in place, as one
    flattened all_reduce (parameters without a gradient contribute zeros)."""
    import torch.distributed as dist
    params = [p for p in params]
    if not params or not (dist.is_available() and dist.is_initialized()):
        return
    if dist.get_world_size(group) == 1:
        return
    for p in params:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
    flat = torch.cat([p.grad.reshape(-1).float() for p in params])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    off = 0
    for p in params:
        n = p.grad.numel()
        p.grad.copy_(flat[off:off + n].view_as(p.grad))
        off += n
