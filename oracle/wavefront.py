"""CPU oracle for the wavefront engine (TEST INFRASTRUCTURE ONLY).

Restates, on the host, the reference algorithms the CUDA path must reproduce. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may use it.

  schedule      : wavefront/wavefront_api.py:20-68 (tick = 1 + max tick of in-grid deps).
  routing_map   : wavefront/wavefront_engine.py:416-438 (source cell, -2 = x, -1 = zero).
  compile       : wavefront/wavefront_engine.py:380-414 (per-tick cells padded with num_cells).
  fetch         : wavefront/wavefront_kernel.py:6-25 (fetch_mapped_context).
  pure_loop     : the anti-diagonal loop of wavefront/wavefront_test.py:94-111 and :206-215,
                  which the reference's own test uses as ground truth for the engine.
  tanh_grid     : the cell h[i,j] = tanh(W_l h[i,j-1] + W_t h[i-1,j] + U x[i,j] + b) with a
                  zero boundary, evaluated by the same pure loop (used for the grid-layer
                  benchmark configuration, which the reference engine cannot express because
                  it delivers x to row 0 only).
"""
from __future__ import annotations

import itertools
import math
import sys

import torch


def schedule(grid_shape, dependencies):
    sys.setrecursionlimit(max(10000, sys.getrecursionlimit()))
    tick_map = {}

    def get_tick(coord):
        if coord in tick_map:
            return tick_map[coord]
        best = -1
        for off, _ in dependencies:
            dep = tuple(c + d for c, d in zip(coord, off))
            if all(0 <= dep[i] < grid_shape[i] for i in range(len(coord))):
                best = max(best, get_tick(dep))
        tick_map[coord] = best + 1
        return best + 1

    for coord in itertools.product(*[range(s) for s in grid_shape]):
        get_tick(coord)
    groups = {}
    for coord, t in tick_map.items():
        groups.setdefault(t, []).append(coord)
    return [groups[t] for t in sorted(groups)]


def flat(coord, grid_shape):
    idx, stride = 0, 1
    for d in reversed(range(len(grid_shape))):
        idx += coord[d] * stride
        stride *= grid_shape[d]
    return idx


def routing_map(grid_shape, dependencies):
    n = math.prod(grid_shape)
    out = [-1] * (n * len(dependencies))
    for coord in itertools.product(*[range(s) for s in grid_shape]):
        cur = flat(coord, grid_shape)
        for di, (off, _) in enumerate(dependencies):
            tgt = tuple(c + d for c, d in zip(coord, off))
            if all(0 <= tgt[i] < grid_shape[i] for i in range(len(coord))):
                out[cur * len(dependencies) + di] = flat(tgt, grid_shape)
            elif tgt[0] == -1 and all(0 <= tgt[i] < grid_shape[i] for i in range(1, len(coord))):
                out[cur * len(dependencies) + di] = -2
    return out


def compile_schedule(grid_shape, dependencies):
    sched = schedule(grid_shape, dependencies)
    n = math.prod(grid_shape)
    m = max(len(g) for g in sched)
    cells, layers = [], []
    for g in sched:
        c = [flat(x, grid_shape) for x in g] + [n] * (m - len(g))
        l = [x[0] for x in g] + [-1] * (m - len(g))
        cells.append(c)
        layers.append(l)
    return cells, layers, m


def gather(x, grids, active_cells, routing, port_map, grid_shape, n_deps):
    """Vectorised restatement of fetch_mapped_context over a tick's active cells.
    x [batch, seq, dim]; grids [ports, cells(+pad), batch, dim] -> [deps, slots, batch, dim]."""
    n = math.prod(grid_shape)
    seq = n // grid_shape[0]
    out = torch.zeros((n_deps, len(active_cells)) + tuple(grids.shape[2:]), dtype=grids.dtype)
    for s, cell in enumerate(active_cells):
        if cell >= n:
            continue
        for i in range(n_deps):
            t = routing[cell * n_deps + i]
            if t >= 0:
                out[i, s] = grids[port_map[i], t]
            elif t == -2:
                out[i, s] = x[:, cell % seq, :]
    return out


def _fetch(grid_shape, x, out_grids, coord, dep):
    (l, t), ((dl, dt), port) = coord, dep
    tl, tt = l + dl, t + dt
    if 0 <= tl < grid_shape[0] and 0 <= tt < grid_shape[1]:
        return out_grids[port][tl][tt]
    if tl == -1 and 0 <= tt < grid_shape[1]:
        return x[:, tt, :]
    return torch.zeros_like(x[:, 0, :])


def pure_loop(grid_shape, dependencies, num_ports, layers, x):
    """Anti-diagonal loop of the reference test (2-D grids). Each layers[l] is called with the
    fetched [batch, dim] dependency tensors and returns num_ports tensors. Returns the port
    grids as lists [port][l][t] (autograd-connected)."""
    sched = schedule(grid_shape, dependencies)
    grids = [[[None] * grid_shape[1] for _ in range(grid_shape[0])] for _ in range(num_ports)]
    for group in sched:
        for (l, t) in group:
            fetched = [_fetch(grid_shape, x, grids, (l, t), d) for d in dependencies]
            outs = layers[l](*fetched)
            for p in range(num_ports):
                grids[p][l][t] = outs[p]
    return grids


def tanh_grid_forward(x, W_l, W_t, U, b, top=None):
    """Pure-loop forward of the tanh grid cell, float64 by default on the inputs' dtype.
    x [B, R, C, H] (U may be None: no x term), W_l/W_t [G, H, H] (G = 1 shared or R per row),
    b [G, H], top [C, B, H] or None. Returns h [R, C, B, H]."""
    B, R, C, H = x.shape
    G = W_l.shape[0]
    zero = torch.zeros(B, H, dtype=x.dtype)
    rows = []
    for i in range(R):
        g = i if G > 1 else 0
        row = []
        for j in range(C):
            left = row[j - 1] if j > 0 else zero
            up = rows[i - 1][j] if i > 0 else (top[j] if top is not None else zero)
            z = left @ W_l[g].T + up @ W_t[g].T + b[g]
            if U is not None:
                z = z + x[:, i, j, :] @ U.T
            row.append(torch.tanh(z))
        rows.append(row)
    return torch.stack([torch.stack(r) for r in rows])


def tanh_grid_backward(x, W_l, W_t, U, b, h, dh, top=None):
    """Reverse sweep of tanh_grid_forward (the chain rule of the same loop, cells visited in
    reverse row-major order), without an autograd graph. h [R, C, B, H] is the forward output,
    dh its upstream gradient. Returns (dx, dW_l, dW_t, dU, db, dtop); dU is None when U is,
    dtop when top is."""
    B, R, C, H = x.shape
    G = W_l.shape[0]
    zero = torch.zeros(B, H, dtype=h.dtype)
    dW_l, dW_t = torch.zeros_like(W_l), torch.zeros_like(W_t)
    db = torch.zeros_like(b)
    dU = torch.zeros_like(U) if U is not None else None
    dx = torch.zeros_like(x)
    dtop = torch.zeros(C, B, H, dtype=h.dtype) if top is not None else None
    dz = [[None] * C for _ in range(R)]
    for i in reversed(range(R)):
        g = i if G > 1 else 0
        g_down = (i + 1 if G > 1 else 0) if i + 1 < R else g
        for j in reversed(range(C)):
            gh = dh[i, j].clone()
            if j + 1 < C:
                gh = gh + dz[i][j + 1] @ W_l[g]
            if i + 1 < R:
                gh = gh + dz[i + 1][j] @ W_t[g_down]
            d = gh * (1 - h[i, j] * h[i, j])
            dz[i][j] = d
            left = h[i, j - 1] if j > 0 else zero
            up = h[i - 1, j] if i > 0 else (top[j] if top is not None else zero)
            dW_l[g] += d.T @ left
            dW_t[g] += d.T @ up
            db[g] += d.sum(0)
            if U is not None:
                dU += d.T @ x[:, i, j, :]
                dx[:, i, j, :] = d @ U
            if i == 0 and top is not None:
                dtop[j] = d @ W_t[g]
        if i + 2 < R:
            dz[i + 2] = None  # rows below i + 1 are no longer needed
    return dx, dW_l, dW_t, dU, db, dtop


def tanh_grid_make_inputs(B, R, C, H, G=1, seed=0, with_U=True, with_top=False):
    """Seeded inputs with the benchmark distributions: x ~ N(0,1) [B,R,C,H];
    W_l, W_t, U ~ N(0, 1/H); b = 0; upstream grad dh ~ N(0,1) [R,C,B,H]."""
    gen = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(H)
    x = torch.randn(B, R, C, H, generator=gen)
    W_l = torch.randn(G, H, H, generator=gen) * s
    W_t = torch.randn(G, H, H, generator=gen) * s
    U = torch.randn(H, H, generator=gen) * s if with_U else None
    b = torch.zeros(G, H)
    top = torch.randn(C, B, H, generator=gen) if with_top else None
    dh = torch.randn(R, C, B, H, generator=gen)
    return x, W_l, W_t, U, b, top, dh
