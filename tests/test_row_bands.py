"""Host-side logic of the row-band split of the grid layer (wavefront/row_bands.py), on CPU:
the band partition, the handle exchange as world_size-2 gloo ranks, and the decomposition the
band kernels implement, restated with the oracle: each band sweeps its rows with the band above's
last row as its top row, the backward hands each band's top-row gradient to the band above, and
the all-reduced partial weight gradients equal the unsplit grid's (checked against the oracle on
the whole grid)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def test_band_rows_partition():
    from wavefront.row_bands import band_rows
    for rows in (1, 2, 5, 8, 63, 64):
        for world in range(1, 9):
            if world > rows:
                with pytest.raises(ValueError):
                    band_rows(rows, world, 0)
                continue
            seen, sizes = [], []
            for r in range(world):
                row0, n = band_rows(rows, world, r)
                assert n >= 1
                seen.extend(range(row0, row0 + n))
                sizes.append(n)
            assert seen == list(range(rows))
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        band_rows(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _band_worker(rank, world, port, res_path, G_per_row):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "flb-transformer_b200"))
    sys.path.insert(0, repo)
    import torch.distributed as dist
    from oracle import wavefront as ow
    from wavefront.row_bands import band_rows, exchange_handles
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        handles = exchange_handles(bytes([rank]) * 80)
        ok_handles = handles == [bytes([r]) * 80 for r in range(world)]

        B, R, C, H = 2, 5, 4, 8
        G = R if G_per_row else 1
        g = torch.Generator().manual_seed(11)
        x = torch.randn(B, R, C, H, generator=g, dtype=torch.float64)
        W_l = torch.randn(G, H, H, generator=g, dtype=torch.float64) / H ** 0.5
        W_t = torch.randn(G, H, H, generator=g, dtype=torch.float64) / H ** 0.5
        U = torch.randn(H, H, generator=g, dtype=torch.float64) / H ** 0.5
        b = torch.randn(G, H, generator=g, dtype=torch.float64) * 0.1
        top = torch.randn(C, B, H, generator=g, dtype=torch.float64)
        dh = torch.randn(R, C, B, H, generator=g, dtype=torch.float64)

        row0, n = band_rows(R, world, rank)
        rows = slice(row0, row0 + n)
        wsl = (lambda t: t[rows]) if G > 1 else (lambda t: t)
        # forward: the band above's last row is this band's top row
        if rank == 0:
            halo = top
        else:
            halo = torch.empty(C, B, H, dtype=torch.float64)
            dist.recv(halo, src=rank - 1)
        h = ow.tanh_grid_forward(x[:, rows], wsl(W_l), wsl(W_t), U, wsl(b), top=halo)
        if rank + 1 < world:
            dist.send(h[-1].contiguous(), dst=rank + 1)
        # backward: the band below's top-row gradient joins this band's last-row gradient
        dh_band = dh[rows].clone()
        if rank + 1 < world:
            d_below = torch.empty(C, B, H, dtype=torch.float64)
            dist.recv(d_below, src=rank + 1)
            dh_band[-1] += d_below
        dx, dWl, dWt, dU, db, dtop = ow.tanh_grid_backward(x[:, rows], wsl(W_l), wsl(W_t), U,
                                                           wsl(b), h, dh_band, top=halo)
        if rank > 0:
            dist.send(dtop.contiguous(), dst=rank - 1)
        # partial weight gradients, all-reduced
        full = lambda t, like: t if G == 1 else torch.zeros_like(like).index_copy_(
            0, torch.arange(row0, row0 + n), t)
        grads = [full(dWl, W_l), full(dWt, W_t), dU, full(db, b)]
        for t in grads:
            dist.all_reduce(t)
        parts = [None] * world
        dist.all_gather_object(parts, (rank, h, dx, dtop if rank == 0 else None))
        if rank == 0:
            ref_h = ow.tanh_grid_forward(x, W_l, W_t, U, b, top=top)
            r_dx, r_dWl, r_dWt, r_dU, r_db, r_dtop = ow.tanh_grid_backward(x, W_l, W_t, U, b,
                                                                           ref_h, dh, top=top)
            parts.sort(key=lambda p: p[0])
            got_h = torch.cat([p[1] for p in parts], 0)
            got_dx = torch.cat([p[2] for p in parts], 1)
            close = lambda a, c: torch.allclose(a, c, atol=1e-10, rtol=1e-10)
            res = {"handles": ok_handles, "h": close(got_h, ref_h), "dx": close(got_dx, r_dx),
                   "dWl": close(grads[0], r_dWl), "dWt": close(grads[1], r_dWt),
                   "dU": close(grads[2], r_dU), "db": close(grads[3], r_db),
                   "dtop": close(parts[0][3], r_dtop)}
            torch.save(res, res_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("per_row", [False, True])
def test_two_rank_band_decomposition(tmp_path, per_row):
    port = _free_port()
    res = str(tmp_path / "res.pt")
    mp.start_processes(_band_worker, args=(2, port, res, per_row), nprocs=2,
                       start_method="spawn", join=True)
    r = torch.load(res)
    assert all(r.values()), r
