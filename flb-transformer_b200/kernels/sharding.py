"""Data-parallel use of the additive attention across the GPUs of one node.

The operator's (batch, head) units are independent, so a job shards them over ranks with no
collective on the data path: each rank runs fused_additive_attention on its own units. The one
exchange step is in the backward: v_a is a parameter every rank holds, so its gradient (a sum over
all units) is all-reduced. With NCCL over NVLink that is one small all_reduce per step
(H * D floats per v_a).

Helpers here are plain torch.distributed code (NCCL on GPUs; gloo works for CPU tests of the
host-side logic).
"""
from __future__ import annotations

import torch


def shard_range(n_units: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of `n_units` owned by `rank` of `world`; shards differ in size by
    at most one unit and together cover every unit exactly once."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch_heads(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of a [B, H, N, D] tensor along the flattened (batch, head) units, as a
    [units, 1, N, D] view-compatible tensor (units = the rank's share of B * H)."""
    B, H = t.shape[0], t.shape[1]
    start, stop = shard_range(B * H, rank, world)
    return t.reshape(B * H, 1, *t.shape[2:])[start:stop]


def head_index_of_units(B: int, H: int, rank: int, world: int) -> torch.Tensor:
    """Head index of each unit this rank owns (to pick the v_a row a unit uses)."""
    start, stop = shard_range(B * H, rank, world)
    return torch.arange(start, stop) % H


def all_reduce_v_a_grad(v_a: torch.Tensor, group=None) -> None:
    """Sum v_a.grad over the ranks of `group` in place (the backward's exchange step)."""
    import torch.distributed as dist
    if v_a.grad is None:
        v_a.grad = torch.zeros_like(v_a)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(v_a.grad, op=dist.ReduceOp.SUM, group=group)
