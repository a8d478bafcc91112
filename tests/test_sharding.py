"""Host-side logic of the multi-GPU path, run as world_size-2 gloo ranks on CPU: the (batch, head)
shards cover every unit once, and the v_a-gradient all-reduce of sharded work equals the gradient
of the unsharded problem (checked with the oracle, since the kernels need a GPU)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def test_shard_range_covers_units_once():
    from kernels.sharding import shard_range
    for n in (1, 7, 32, 128, 1000):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                a, b = shard_range(n, r, world)
                assert 0 <= a <= b <= n
                seen.extend(range(a, b))
            assert seen == list(range(n))
            sizes = [shard_range(n, r, world)[1] - shard_range(n, r, world)[0] for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, res_path):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "flb-transformer_b200"))
    sys.path.insert(0, repo)
    import torch.distributed as dist
    from kernels.sharding import shard_batch_heads, head_index_of_units, all_reduce_v_a_grad
    from oracle import attention as oa
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, w, g = oa.make_inputs(2, 3, 9, 8, seed=5, with_grad_out=True, dtype=torch.float64)
        qs, ks, vs, gs = (shard_batch_heads(t, rank, world) for t in (q, k, v, g))
        heads = head_index_of_units(2, 3, rank, world)
        wv = w.clone().requires_grad_(True)
        # each unit uses its head's row of v_a: gather rows, oracle forward, backward
        wu = wv[heads]                                  # [units, 1, D]
        out, _ = oa.attention_forward(qs, ks, vs, wu.unsqueeze(1))
        out.backward(gs)
        all_reduce_v_a_grad(wv)
        out_list = [None] * world
        dist.all_gather_object(out_list, (rank, out.detach()))
        if rank == 0:
            full_out, _ = oa.attention_forward(q, k, v, w)
            ref_dw = oa.attention_backward(q, k, v, w, g)[3]
            got_out = torch.cat([o for _, o in sorted(out_list, key=lambda x: x[0])], 0)
            ok_out = torch.allclose(got_out, full_out.reshape(6, 1, 9, 8), atol=1e-12)
            ok_dw = torch.allclose(wv.grad, ref_dw, atol=1e-12)
            torch.save({"ok_out": ok_out, "ok_dw": ok_dw}, res_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_attention_gradient(tmp_path):
    port = _free_port()
    res = str(tmp_path / "res.pt")
    mp.start_processes(_worker, args=(2, port, res), nprocs=2, start_method="spawn", join=True)
    r = torch.load(res)
    assert r["ok_out"] and r["ok_dw"]


def _grid_worker(rank, world, port, res_path):
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "flb-transformer_b200"))
    sys.path.insert(0, repo)
    import torch.distributed as dist
    from wavefront.sharding import shard_batch, all_reduce_grads
    from oracle import wavefront as ow
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, W_l, W_t, U, b, _, dh = ow.tanh_grid_make_inputs(5, 3, 4, 8, G=1, seed=9)
        params = [t.double().clone().requires_grad_(True) for t in (W_l, W_t, U, b)]
        xs = shard_batch(x.double(), rank, world, dim=0)       # x [B, R, C, H]
        dhs = shard_batch(dh.double(), rank, world, dim=2)     # dh [R, C, B, H]
        h = ow.tanh_grid_forward(xs, *params)
        h.backward(dhs)
        all_reduce_grads(params)
        if rank == 0:
            full = [t.double().clone().requires_grad_(True) for t in (W_l, W_t, U, b)]
            hf = ow.tanh_grid_forward(x.double(), *full)
            hf.backward(dh.double())
            ok = all(torch.allclose(p.grad, f.grad, atol=1e-12) for p, f in zip(params, full))
            torch.save({"ok": ok}, res_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_batch_sharded_grid_weight_gradients(tmp_path):
    """Batch-sharded grid layer: the all-reduced weight gradients equal the unsharded ones
    (odd batch 5 over 2 ranks: shards of 3 and 2 rows)."""
    port = _free_port()
    res = str(tmp_path / "res.pt")
    mp.start_processes(_grid_worker, args=(2, port, res), nprocs=2, start_method="spawn",
                       join=True)
    assert torch.load(res)["ok"]
