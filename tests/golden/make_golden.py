"""Generate the golden fixtures in tests/golden/ by running the REFERENCE implementation.

Run in a container where the reference is checked out at $FLB_REFERENCE_DIR (default
/root/reference; read-only) and its
C++ orchestrator has been compiled by oracle/build_ref.py:

    python oracle/build_ref.py && python tests/golden/make_golden.py

Everything here runs on CPU:
  * attention: the reference's eager ground truth pure_torch_additive_attention
    (kernels/kernel_tests.py:8-29), gradients by autograd through it, and the reference
    backward compiled_backward_math (kernels/additive_attention.py:91-130) for cross-check;
  * wavefront: the reference schedule / routing / compile functions, its Python gather twin
    fetch_mapped_context, and the reference WavefrontEngine itself (its C++ tick loop from
    oracle/_ref, with the Triton gather replaced by a loop over fetch_mapped_context and
    torch.compile forced to eager), on the configurations of the reference's own tests
    (wavefront/wavefront_test.py) and on a per-row tanh grid cell;
  * the FLB model: the reference FLB_Transformer end to end (logits, aux loss, contexts,
    parameter gradients of cross-entropy + aux) on a small configuration.
The fixtures are small (under 2 MB in total) and are committed; this script is how they were made.
"""
from __future__ import annotations

import copy
import math
import os
import sys

import torch

REF = os.environ.get("FLB_REFERENCE_DIR", "/root/reference")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle", "_ref"))
sys.path.insert(0, REF)

import torch.nn as nn  # noqa: E402

torch.compiler.set_stance("force_eager")


def attention_goldens():
    from kernels.kernel_tests import pure_torch_additive_attention
    from kernels.additive_attention import compiled_backward_math

    out = {}
    # the reference test configuration (kernels/kernel_tests.py:55-64)
    torch.manual_seed(42)
    B, H, S, D = 2, 8, 3, 32
    q = torch.randn(B, H, S, D)
    k = torch.randn(B, H, S, D)
    v = torch.randn(B, H, S, D)
    va = torch.randn(H, 1, D)
    qq, kk, vv, aa = [t.clone().requires_grad_(True) for t in (q, k, v, va)]
    o = pure_torch_additive_attention(qq, kk, vv, aa)
    g = torch.randn_like(o)
    o.backward(g)
    cb = compiled_backward_math(q, k, v, va, g, math.sqrt(D))
    out["kat_b2h8n3d32"] = dict(q=q, k=k, v=v, v_a=va, dout=g, out=o.detach(),
                                dq=qq.grad, dk=kk.grad, dv=vv.grad, dv_a=aa.grad,
                                cb_dq=cb[0], cb_dk=cb[1], cb_dv=cb[2], cb_dv_a=cb[3])
    # vmap over a Layers dim (kernels/kernel_tests.py:89-106)
    L = 4
    ql, kl, vl = (torch.randn(L, B, H, S, D) for _ in range(3))
    al = torch.randn(L, H, 1, D)
    ol = torch.vmap(pure_torch_additive_attention)(ql, kl, vl, al)
    out["vmap_l4"] = dict(q=ql, k=kl, v=vl, v_a=al, out=ol)
    # a longer sequence with the benchmark distributions
    gen = torch.Generator().manual_seed(7)
    B, H, N, D = 2, 2, 96, 64
    q, k, v = (torch.randn(B, H, N, D, generator=gen) for _ in range(3))
    va = torch.randn(H, 1, D, generator=gen) / math.sqrt(D)
    g = torch.randn(B, H, N, D, generator=gen)
    qq, kk, vv, aa = [t.clone().requires_grad_(True) for t in (q, k, v, va)]
    o = pure_torch_additive_attention(qq, kk, vv, aa)
    o.backward(g)
    out["b2h2n96d64"] = dict(q=q, k=k, v=v, v_a=va, dout=g, out=o.detach(), dq=qq.grad,
                             dk=kk.grad, dv=vv.grad, dv_a=aa.grad)
    return out


def wavefront_goldens():
    import wavefront.wavefront_engine as we
    from wavefront.wavefront_api import WavefrontConfig, generate_wavefront_schedule
    from wavefront.wavefront_kernel import fetch_mapped_context
    from wavefront.wavefront_test import DummyLayer, _test_fetch

    def cpu_fetch(x, stacked_grids, routing_map, port_map, spatial_map, config, active, gathered):
        n = math.prod(config.grid_shape)
        grids = [stacked_grids[p][:n] for p in range(config.num_ports)]
        gathered.zero_()
        for s, cell in enumerate(active.tolist()):
            if cell >= n:
                continue
            ing = fetch_mapped_context(x, grids, cell, routing_map, config)
            for d, t in enumerate(ing):
                gathered[d, s] = t
        return gathered

    we.run_fetch_kernel = cpu_fetch
    out = {}

    # schedules (wavefront_test.py:50-72)
    c2 = WavefrontConfig(grid_shape=(4, 4), batch_size=1)
    c3 = WavefrontConfig(grid_shape=(3, 8, 8), batch_size=1,
                         dependencies=[((-1, 0, 0), 0), ((0, -1, 0), 1), ((0, 0, -1), 1)])
    cf = WavefrontConfig(grid_shape=(4, 6), batch_size=1,
                         dependencies=[((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)], num_ports=4)
    out["schedule_4x4"] = generate_wavefront_schedule(c2)
    out["schedule_3x8x8"] = generate_wavefront_schedule(c3)
    out["schedule_flb_4x6"] = generate_wavefront_schedule(cf)

    # routing map / compiled schedule of the mapped-fetcher test (wavefront_test.py:147-184)
    cfg = WavefrontConfig(grid_shape=(3, 4), batch_size=2, dim=8)
    layers = nn.ModuleList([DummyLayer(cfg.dim, 2, 2) for _ in range(3)])
    eng = we.WavefrontEngine(cfg, layers)
    out["routing_3x4"] = eng.routing_map.clone()
    out["compiled_3x4"] = (eng.compiled_cells, eng.compiled_layers, eng.max_cells_per_tick)
    engf = we.WavefrontEngine(cf, nn.ModuleList([nn.Identity() for _ in range(4)]))
    out["routing_flb_4x6"] = engf.routing_map.clone()
    out["compiled_flb_4x6"] = (engf.compiled_cells, engf.compiled_layers, engf.max_cells_per_tick)

    # gather cases of test_triton_kernel_isolated (wavefront_test.py:244-249), via the Python twin
    gcases = []
    gen = torch.Generator().manual_seed(11)
    for tc in [{"batch": 1, "dim": 8, "grid": (3, 4)}, {"batch": 4, "dim": 32, "grid": (2, 2)},
               {"batch": 3, "dim": 12, "grid": (2, 3)}, {"batch": 2, "dim": 256, "grid": (4, 4)}]:
        c = WavefrontConfig(grid_shape=tc["grid"], batch_size=tc["batch"], dim=tc["dim"])
        e = we.WavefrontEngine(c, nn.ModuleList([DummyLayer(c.dim, 2, 2) for _ in range(c.grid_shape[0])]))
        n = math.prod(c.grid_shape)
        x = torch.randn(c.batch_size, c.grid_shape[1], c.dim, generator=gen)
        sg = torch.randn(2, n + 1, c.batch_size, c.dim, generator=gen)
        grids = [sg[p][:n] for p in range(2)]
        res = torch.zeros(2, n, c.batch_size, c.dim)
        for cell in range(n):
            ing = fetch_mapped_context(x, grids, cell, e.routing_map, c)
            for d in range(2):
                res[d, cell] = ing[d]
        gcases.append(dict(grid=tc["grid"], batch=tc["batch"], dim=tc["dim"], x=x,
                           stacked_grids=sg, routing=e.routing_map.clone(), expected=res))
    out["gather_cases"] = gcases

    # engine vs pure loop (wavefront_test.py:186-232), on CPU with the reference engine
    def engine_case(grid, batch, dim, layer_fn, seed, loss_cell=-1):
        torch.manual_seed(seed)
        c = WavefrontConfig(grid_shape=grid, batch_size=batch, dim=dim)
        x = torch.randn(batch, grid[1], dim)
        base = nn.ModuleList([layer_fn(dim) for _ in range(grid[0])])
        xe = x.clone().requires_grad_(True)
        le = copy.deepcopy(base)
        e = we.WavefrontEngine(c, le)
        grids = e(xe)
        loss = grids[0][loss_cell].sum() + 0.5 * grids[1].square().sum()
        loss.backward()
        xp = x.clone().requires_grad_(True)
        lp = copy.deepcopy(base)
        pg = [[[None] * grid[1] for _ in range(grid[0])] for _ in range(2)]
        for group in generate_wavefront_schedule(c):
            for (l, t) in group:
                f = [_test_fetch(c.grid_shape, xp, pg, (l, t), d) for d in c.dependencies]
                o = lp[l](*f)
                for p in range(2):
                    pg[p][l][t] = o[p]
        pure0 = torch.stack([torch.stack(r) for r in pg[0]]).reshape(-1, batch, dim)
        pure1 = torch.stack([torch.stack(r) for r in pg[1]]).reshape(-1, batch, dim)
        lp_loss = pure0[loss_cell].sum() + 0.5 * pure1.square().sum()
        lp_loss.backward()
        return dict(grid=grid, batch=batch, dim=dim, x=x,
                    params=[{k: v.detach().clone() for k, v in m.state_dict().items()} for m in base],
                    grids=[g.detach().clone() for g in grids], x_grad=xe.grad.clone(),
                    param_grads=[{k: p.grad.clone() for k, p in m.named_parameters()} for m in le],
                    pure_grids=[pure0.detach(), pure1.detach()], pure_x_grad=xp.grad.clone(),
                    pure_param_grads=[{k: p.grad.clone() for k, p in m.named_parameters()} for m in lp])

    out["engine_dummy_2x3"] = engine_case((2, 3), 2, 4, lambda d: DummyLayer(d, 2, 2), 42)

    class TanhCell(nn.Module):
        """h = tanh(W_l left + W_t top + b), emitted on both ports."""
        def __init__(self, dim):
            super().__init__()
            s = 1.0 / math.sqrt(dim)
            self.W_l = nn.Parameter(torch.randn(dim, dim) * s)
            self.W_t = nn.Parameter(torch.randn(dim, dim) * s)
            self.b = nn.Parameter(torch.randn(dim) * 0.1)

        def forward(self, top, left):
            h = torch.tanh(left @ self.W_l.T + top @ self.W_t.T + self.b)
            return h, h

    out["engine_tanh_3x5"] = engine_case((3, 5), 16, 64, TanhCell, 5)
    return out


def _reference_flb_on_cpu():
    """models.FLB_Model with its attention op replaced by the reference's eager ground truth
    (the Triton kernel has no CPU path) and the engine's gather by fetch_mapped_context."""
    import wavefront.wavefront_engine as we
    import models.FLB_Model as fm
    from kernels.kernel_tests import pure_torch_additive_attention
    from wavefront.wavefront_kernel import fetch_mapped_context

    def cpu_fetch(x, stacked_grids, routing_map, port_map, spatial_map, config, active, gathered):
        n = math.prod(config.grid_shape)
        grids = [stacked_grids[p][:n] for p in range(config.num_ports)]
        gathered.zero_()
        for s, cell in enumerate(active.tolist()):
            if cell >= n:
                continue
            for d, t in enumerate(fetch_mapped_context(x, grids, cell, routing_map, config)):
                gathered[d, s] = t
        return gathered

    we.run_fetch_kernel = cpu_fetch
    fm.fused_additive_attention = pure_torch_additive_attention
    return fm


def flb_model_goldens():
    """The reference FLB_Transformer (models/FLB_Model.py) end to end on CPU, eval mode, on a
    small configuration, the engine as in wavefront_goldens()."""
    fm = _reference_flb_on_cpu()
    torch.manual_seed(21)
    V, D, L, S, B = 40, 32, 3, 5, 2
    model = fm.FLB_Transformer(V, hidden_dim=D, num_layers=L, seq_len=S, batch_size=B)
    with torch.no_grad():  # larger v_a than the 0.02 init so the attention weights matter
        for layer in model.layers:
            layer.flb_attention.v_a.normal_(0.0, 0.5)
    model.eval()
    tokens = torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(3))
    targets = torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(4))
    logits, aux, (lat, fdbk) = model(tokens)
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, V), targets.reshape(-1)) + aux
    loss.backward()
    return dict(config=dict(vocab=V, hidden=D, layers=L, seq_len=S, batch=B),
                state_dict={k: v.detach().clone() for k, v in model.state_dict().items()},
                tokens=tokens, targets=targets, logits=logits.detach(), aux_loss=aux.detach(),
                next_lat=lat.detach().clone(), next_fdbk=fdbk.detach().clone(),
                loss=loss.detach(),
                grads={k: p.grad.clone() for k, p in model.named_parameters()
                       if p.grad is not None})


def flb_model_b16_goldens():
    """The reference FLB_Transformer forward (eval, float32, CPU) at batch 16 and d_model 128 (its
    8 heads of 16): the shape class of the persistent native forward. The weights are not stored:
    flb_weights.set_hashed_weights(model, 5) regenerates them (bf16-representable values)."""
    from flb_weights import set_hashed_weights
    fm = _reference_flb_on_cpu()
    V, D, L, S, B = 40, 128, 3, 4, 16
    model = fm.FLB_Transformer(V, hidden_dim=D, num_layers=L, seq_len=S, batch_size=B)
    set_hashed_weights(model, 5)
    model.eval()
    tokens = torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(6))
    with torch.no_grad():
        logits, aux, (lat, fdbk) = model(tokens)
    return dict(config=dict(vocab=V, hidden=D, layers=L, seq_len=S, batch=B, weight_seed=5),
                tokens=tokens, logits=logits.clone(), aux_loss=aux.clone(),
                next_lat=lat.clone(), next_fdbk=fdbk.clone())


GOLDENS = {"attention.pt": attention_goldens, "wavefront.pt": wavefront_goldens,
           "flb_model.pt": flb_model_goldens, "flb_model_b16.pt": flb_model_b16_goldens}


def main(names):
    """python make_golden.py [file ...]: regenerate the named fixtures (default: all)."""
    for f in names or list(GOLDENS):
        torch.save(GOLDENS[f](), os.path.join(HERE, f))
        print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")


if __name__ == "__main__":
    main(sys.argv[1:])
