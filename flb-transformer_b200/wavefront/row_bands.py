"""Row bands: one tanh grid layer split by grid rows across the GPUs of a node.

Each rank of a process group (one process per GPU) evaluates a contiguous band of grid rows with
the persistent sweep kernels (`flb_grid_band_fwd` / `flb_grid_band_bwd`). The bands run at the
same time as one pipelined wavefront: the rows at a band's edges exchange [C, B, H] halos with
the neighbouring bands inside the kernels, column by column, through NVLink peer memory. Each
rank owns a receive block in its own memory (CUDA IPC allocation); its neighbours map it and
store into it:

* forward: the band above stores h of its last row, column c, into this rank's block and
  releases a per-column flag; this band's first row waits on the flag, loads the halo from local
  memory, keeps a copy for the backward and acknowledges, so the next call may overwrite it;
* backward: the band below stores dz of its first row; this band's last row consumes it through
  W_t of the next row, as the unsplit sweep does.

The reference evaluates the grid on one device (training/trainer.py:31); this is the row-band
partitioning of the grid layer. Weight gradients of a band are partial sums over its rows:
all-reduce them across the ranks afterwards (`wavefront.sharding.all_reduce_grads`).

Calls are collective in the SPMD sense: every rank calls `layer` (and its backward) the same
number of times in the same order, since the halo flags carry a per-call epoch.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

import flb_native as nat

__all__ = ["band_rows", "exchange_handles", "GridRowBands"]


def band_rows(rows_total: int, world: int, rank: int) -> tuple[int, int]:
    """(row0, rows) of `rank`'s band: rows split as evenly as possible, the first
    rows_total % world ranks taking one more row. Every band needs at least one row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"band_rows: rank {rank} outside a world of {world}")
    if rows_total < world:
        raise ValueError(f"band_rows: {rows_total} rows cannot give each of {world} ranks a band")
    base, extra = divmod(rows_total, world)
    rows = base + (1 if rank < extra else 0)
    row0 = rank * base + min(rank, extra)
    return row0, rows


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' receive-block handles, in rank order (an all-gather over the group)."""
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class _BandFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W_l, W_t, U, b, top, bands, x_layout):
        R, C, B, H = bands.rows, bands.C, bands.B, bands.H
        G = W_l.shape[0]
        dev = W_l.device
        bf = lambda t: None if t is None else t.to(torch.bfloat16).contiguous()
        xb, Wl, Wt, Ub, tb = bf(x), bf(W_l), bf(W_t), bf(U), bf(top)
        bias = b.to(torch.float32).contiguous()
        h = torch.empty((R, C, B, H), dtype=torch.bfloat16, device=dev)
        saved = (torch.empty((C, B, H), dtype=torch.bfloat16, device=dev)
                 if bands.up is not None else None)
        band = bands._band(bands.next_fwd_epoch())
        ws_bytes = nat.lib.flb_grid_workspace_bytes(R, C, B, H, G, int(Ub is not None))
        ws = nat.workspace(ws_bytes, dev)
        nat.check(nat.lib.flb_grid_band_fwd(
            nat.ptr(xb), x_layout, Wl.data_ptr(), Wt.data_ptr(), nat.ptr(Ub), bias.data_ptr(),
            nat.ptr(tb), h.data_ptr(), nat.ptr(saved), R, C, B, H, G, ctypes.byref(band),
            ws.data_ptr(), ws_bytes, int(bands.check_timeout), nat.stream_of(h)),
            "flb_grid_band_fwd")
        ctx.save_for_backward(xb, Wl, Wt, Ub, tb if saved is None else saved, h)
        ctx.bands, ctx.x_layout, ctx.has_top = bands, x_layout, top is not None
        ctx.dtypes = (None if x is None else x.dtype, W_l.dtype, W_t.dtype,
                      None if U is None else U.dtype, b.dtype, None if top is None else top.dtype)
        return h

    @staticmethod
    def backward(ctx, dh):
        xb, Wl, Wt, Ub, tb, h = ctx.saved_tensors
        bands = ctx.bands
        R, C, B, H = bands.rows, bands.C, bands.B, bands.H
        G = Wl.shape[0]
        dev = h.device
        dhb = dh.to(torch.bfloat16).contiguous()
        f32 = dict(dtype=torch.float32, device=dev)
        dWl, dWt = torch.empty((G, H, H), **f32), torch.empty((G, H, H), **f32)
        db = torch.empty((G, H), **f32)
        dU = torch.empty((H, H), **f32) if Ub is not None else None
        dx = torch.empty_like(xb) if Ub is not None else None
        dtop = torch.empty_like(tb) if ctx.has_top else None
        band = bands._band(bands.next_bwd_epoch())
        ws_bytes = nat.lib.flb_grid_workspace_bytes(R, C, B, H, G, int(Ub is not None))
        ws = nat.workspace(ws_bytes, dev)
        nat.check(nat.lib.flb_grid_band_bwd(
            nat.ptr(xb), ctx.x_layout, Wl.data_ptr(), Wt.data_ptr(), nat.ptr(Ub), nat.ptr(tb),
            h.data_ptr(), dhb.data_ptr(), dWl.data_ptr(), dWt.data_ptr(), nat.ptr(dU),
            db.data_ptr(), nat.ptr(dx), nat.ptr(dtop), R, C, B, H, G, ctypes.byref(band),
            ws.data_ptr(), ws_bytes, int(bands.check_timeout), nat.stream_of(h)),
            "flb_grid_band_bwd")
        tx, tWl, tWt, tU, tb_, ttop = ctx.dtypes
        return (None if dx is None else dx.to(tx), dWl.to(tWl), dWt.to(tWt),
                None if dU is None else dU.to(tU), db.to(tb_),
                None if dtop is None else dtop.to(ttop), None, None)


class GridRowBands:
    """This rank's band of a rows_total x cols grid layer (batch `batch`, hidden `hidden`) and its
    halo links to the neighbouring bands. Collective: every rank of `group` constructs it with the
    same sizes, each on its own GPU (the current CUDA device).

    `layer(x, W_l, W_t, U, b, top=None, x_layout=0)` returns this band's h [rows, C, B, H]:
    x is the band's rows of the grid input ([B, rows, C, H] for x_layout 0, [rows, C, B, H] for
    1; U may be None), W_l/W_t [H, H] shared or [rows_total, H, H] per row (all ranks hold all
    weights), b [H] or [rows_total, H]; top [C, B, H] is the grid's top row, given on the first
    band only. Differentiable; weight gradients are this band's partial sums.
    """

    def __init__(self, rows_total: int, cols: int, batch: int, hidden: int, group=None,
                 check_timeout: bool = False):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.rows_total, self.C, self.B, self.H = rows_total, cols, batch, hidden
        self.row0, self.rows = band_rows(rows_total, self.world, self.rank)
        self.check_timeout = check_timeout
        self.fwd_epoch = 0
        self.bwd_epoch = 0
        self.up = self.down = None
        self.own = None
        nbytes = nat.lib.flb_grid_band_block_bytes(cols, batch, hidden)
        if nbytes == 0:
            raise ValueError("GridRowBands: bad grid sizes")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(nat.IPC_HANDLE_BYTES)
        nat.check(nat.lib.flb_ipc_alloc(nbytes, ctypes.byref(own), handle), "flb_ipc_alloc")
        self.own = own
        handles = exchange_handles(handle.raw, group)
        try:
            if self.rank > 0:
                self.up = self._open(handles[self.rank - 1])
            if self.rank + 1 < self.world:
                self.down = self._open(handles[self.rank + 1])
        except Exception:
            self.close(barrier=False)
            raise
        dist.barrier(group=group)

    @staticmethod
    def _open(handle: bytes) -> ctypes.c_void_p:
        p = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(handle, nat.IPC_HANDLE_BYTES)
        nat.check(nat.lib.flb_ipc_open(buf, ctypes.byref(p)), "flb_ipc_open")
        return p

    def next_fwd_epoch(self) -> int:
        self.fwd_epoch += 1
        return self.fwd_epoch

    def next_bwd_epoch(self) -> int:
        self.bwd_epoch += 1
        return self.bwd_epoch

    def _band(self, epoch: int) -> nat.GridBand:
        return nat.GridBand(self.row0, self.rows_total, self.own.value,
                            None if self.up is None else self.up.value,
                            None if self.down is None else self.down.value, epoch)

    def layer(self, x, W_l, W_t, U, b, top=None, x_layout: int = 0):
        nat.require_cuda(x, W_l, W_t, U, b, top)
        if top is not None and self.rank > 0:
            raise ValueError("GridRowBands.layer: top belongs to the first band")
        if W_l.dim() == 2:
            W_l, W_t = W_l.unsqueeze(0), W_t.unsqueeze(0)
        if b.dim() == 1:
            b = b.unsqueeze(0)
        if W_l.shape[0] not in (1, self.rows_total):
            raise ValueError("GridRowBands.layer: per-row weights must cover all rows_total rows")
        want = ((self.B, self.rows, self.C, self.H) if x_layout == 0
                else (self.rows, self.C, self.B, self.H))
        if x is not None and tuple(x.shape) != want:
            raise ValueError(f"GridRowBands.layer: x of this band must be {want}, got {tuple(x.shape)}")
        return _BandFunction.apply(x, W_l, W_t, U, b, top, self, x_layout)

    def close(self, barrier: bool = True) -> None:
        """Unmap the neighbours' blocks and free this rank's. Collective: this rank's kernels
        must be done before the mappings go, and the neighbours' before the block goes."""
        if barrier:
            torch.cuda.synchronize()
        for name in ("up", "down"):
            p = getattr(self, name)
            if p is not None:
                nat.lib.flb_ipc_close(p)
                setattr(self, name, None)
        if barrier:
            dist.barrier(group=self.group)
        if self.own is not None:
            nat.lib.flb_ipc_free(self.own)
            self.own = None
