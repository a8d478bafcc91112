"""Row bands of the grid layer across GPUs (wavefront/row_bands.py, flb_grid_band_fwd/bwd).

Two or four ranks, one GPU each (skipped with fewer GPUs): each rank sweeps its band while the halos
cross NVLink inside the kernels, and the result is compared with the unsplit grid layer run on
the rank's own GPU: h bit for bit without the x term (the same cell arithmetic); with it, h and
dx within bf16 rounding (the hoisted x U^T GEMM runs over fewer rows); the all-reduced weight
gradients within fp32 summation-order tolerance. Two calls in a row exercise the per-call epochs
and acknowledgements. A separate check runs two ranks on ONE GPU without launching any kernel:
mapping a block that lives on the same GPU is refused."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, backend):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "flb-transformer_b200"))
    sys.path.insert(0, repo)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60))
    return dist


CASES = {
    # B, R, C, H, per-row weights, with U (x term), with top
    "w4_band": (32, 8, 12, 256, False, True, True),
    "per_row_uneven": (16, 7, 9, 128, True, False, False),
}


def _band_worker(rank, world, port, res_path, case):
    dist = _setup(rank, world, port, "nccl")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        from wavefront.grid_layer import wavefront_grid_layer
        from wavefront.row_bands import GridRowBands
        B, R, C, H, per_row, with_U, with_top = CASES[case]
        G = R if per_row else 1
        g = torch.Generator().manual_seed(3)
        bf = dict(dtype=torch.bfloat16)
        x = torch.randn(B, R, C, H, generator=g).to(dev, **bf)
        W_l = (torch.randn(G, H, H, generator=g) / H ** 0.5).to(dev, **bf)
        W_t = (torch.randn(G, H, H, generator=g) / H ** 0.5).to(dev, **bf)
        U = (torch.randn(H, H, generator=g) / H ** 0.5).to(dev, **bf) if with_U else None
        b = (torch.randn(G, H, generator=g) * 0.1).to(dev)
        top = torch.randn(C, B, H, generator=g).to(dev, **bf) if with_top else None
        dh = torch.randn(R, C, B, H, generator=g).to(dev, **bf)

        def leaves():
            return [None if t is None else t.clone().requires_grad_(True)
                    for t in (x, W_l, W_t, U, b, top)]

        # the unsplit layer on this rank's GPU
        fx, fWl, fWt, fU, fb, ftop = leaves()
        ref = wavefront_grid_layer(fx, fWl, fWt, fU, fb, top=ftop)
        ref.backward(dh)

        bands = GridRowBands(R, C, B, H, check_timeout=True)
        rows = slice(bands.row0, bands.row0 + bands.rows)
        res = {}
        for call in range(2):
            lx, lWl, lWt, lU, lb, ltop = leaves()
            xb = lx[:, rows].detach().clone().requires_grad_(True)
            h = bands.layer(xb, lWl, lWt, lU, lb, top=ltop if rank == 0 else None)
            h.backward(dh[rows])
            grads = [t.grad for t in (lWl, lWt, lb) + ((lU,) if with_U else ())]
            for t in grads:
                dist.all_reduce(t)
            refs = [fWl.grad, fWt.grad, fb.grad] + ([fU.grad] if with_U else [])
            if with_U:  # the hoisted x U^T GEMM runs over fewer rows: cuBLAS may sum differently
                res[f"h{call}"] = (h.float() - ref[rows].float()).abs().max().item() <= 8e-3
            else:
                res[f"h{call}"] = torch.equal(h, ref[rows])
            if with_U:
                res[f"dx{call}"] = torch.allclose(xb.grad.float(), fx.grad[:, rows].float(),
                                                  atol=2e-2, rtol=2e-2)
            for i, (a, r_) in enumerate(zip(grads, refs)):
                # bf16 weights get bf16 gradients: each rank's partial is rounded before the sum
                tol = 8e-3 if a.dtype == torch.bfloat16 else 1e-4
                err = (a.float() - r_.float()).abs().max().item()
                res[f"w{i}_{call}"] = err <= tol * max(1.0, r_.abs().max().item())
                res[f"w{i}_{call}_err"] = err
            if rank == 0 and with_top:
                res[f"dtop{call}"] = torch.allclose(ltop.grad.float(), ftop.grad.float(),
                                                    atol=2e-2, rtol=2e-2)
        bands.close()
        out = [None] * world
        dist.all_gather_object(out, res)
        if rank == 0:
            torch.save(out, res_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("case", sorted(CASES))
def test_row_bands_match_unsplit_grid(tmp_path, case, world):
    """2 ranks: a first and a last band. 4 ranks: two middle bands as well (a halo in from
    above and out to below in the same sweep), and with 7 rows a band of a single row, whose
    one row is both edges."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"row bands over {world} ranks need {world} GPUs")
    res = str(tmp_path / "res.pt")
    mp.start_processes(_band_worker, args=(world, _free_port(), res, case), nprocs=world,
                       start_method="spawn", join=True)
    out = torch.load(res)
    for rank, r in enumerate(out):
        flags = {k: v for k, v in r.items() if not k.endswith("_err")}
        assert flags and all(flags.values()), (rank, r)


def _same_gpu_worker(rank, world, port, res_path):
    dist = _setup(rank, world, port, "gloo")
    try:
        import ctypes
        torch.cuda.set_device(0)
        import flb_native as nat
        from wavefront.row_bands import exchange_handles
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(nat.IPC_HANDLE_BYTES)
        nat.check(nat.lib.flb_ipc_alloc(4096, ctypes.byref(own), handle), "flb_ipc_alloc")
        handles = exchange_handles(handle.raw)
        peer = ctypes.c_void_p()
        st = nat.lib.flb_ipc_open(ctypes.create_string_buffer(handles[1 - rank], nat.IPC_HANDLE_BYTES),
                                  ctypes.byref(peer))
        dist.barrier()
        nat.lib.flb_ipc_free(own)
        out = [None] * world
        dist.all_gather_object(out, st)
        if rank == 0:
            torch.save(out, res_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_band_peer_on_same_gpu_is_refused(tmp_path):
    res = str(tmp_path / "res.pt")
    mp.start_processes(_same_gpu_worker, args=(2, _free_port(), res), nprocs=2,
                       start_method="spawn", join=True)
    out = torch.load(res)
    assert out == [6, 6]  # FLB_ERR_UNSUPPORTED on both ranks
