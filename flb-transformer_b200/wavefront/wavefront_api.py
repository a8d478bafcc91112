"""Wavefront configuration and anti-diagonal schedule.

Same public surface as the reference (wavefront/wavefront_api.py:5-68): `WavefrontConfig`
and `generate_wavefront_schedule(config) -> list[list[coord]]`, with identical results,
including the order of cells inside a tick (post-order of a depth-first walk started from
every coordinate in row-major order). The walk here uses an explicit stack, so dependency
chains longer than Python's recursion limit are fine.
"""
from __future__ import annotations

import dataclasses
import itertools
from typing import List, Tuple


@dataclasses.dataclass
class WavefrontConfig:
    grid_shape: Tuple[int, ...]
    batch_size: int
    dim: int = 256
    # (spatial_offset, port_index) per dependency, in the cell's input order
    dependencies: List[Tuple[Tuple[int, ...], int]] = dataclasses.field(
        default_factory=lambda: [((-1, 0), 0), ((0, -1), 1)]
    )
    num_ports: int = 2
    requires_grad: bool = True


def _in_grid(coord, shape) -> bool:
    return all(0 <= c < s for c, s in zip(coord, shape))


def compute_ticks(config: WavefrontConfig) -> dict:
    """tick(c) = 1 + max(tick(d) for in-grid dependencies d), -1 + 1 = 0 for none.
    Returns {coord: tick} in the reference's insertion order (wavefront_api.py:25-58)."""
    shape = tuple(config.grid_shape)
    offsets = [tuple(off) for off, _ in config.dependencies]
    tick_map: dict = {}
    for start in itertools.product(*[range(s) for s in shape]):
        if start in tick_map:
            continue
        # frame: [coord, next dependency index, running max]
        stack = [[start, 0, -1]]
        on_stack = {start}
        while stack:
            frame = stack[-1]
            coord, di, best = frame
            if di < len(offsets):
                frame[1] = di + 1
                dep = tuple(c + d for c, d in zip(coord, offsets[di]))
                if not _in_grid(dep, shape):
                    continue
                if dep in tick_map:
                    frame[2] = max(best, tick_map[dep])
                    continue
                if dep in on_stack:
                    raise ValueError(f"cyclic wavefront dependencies through {dep}")
                stack.append([dep, 0, -1])
                on_stack.add(dep)
                continue
            tick_map[coord] = best + 1
            stack.pop()
            on_stack.discard(coord)
            if stack:
                stack[-1][2] = max(stack[-1][2], best + 1)
    return tick_map


def generate_wavefront_schedule(config: WavefrontConfig) -> List[List[Tuple[int, ...]]]:
    """Cells grouped by tick, ticks ascending (wavefront_api.py:20-68)."""
    tick_map = compute_ticks(config)
    schedule: dict = {}
    for coord, tick in tick_map.items():
        schedule.setdefault(tick, []).append(coord)
    return [schedule[t] for t in sorted(schedule)]
