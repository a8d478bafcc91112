"""CUDA-graph replay of the WavefrontEngine's per-tick path.

The generic-layer engine runs one host tick per anti-diagonal: a gather, the user's cell under
torch.vmap (forward) or torch.func.vjp (backward), and a scatter, driven by the C++ loop of
`wavefront_backend`. Per tick the GPU work is small and the host work (vmap dispatch, launch
overhead) dominates. Every tick reads and writes the engine's static buffers only (the
reference engine keeps them for the same purpose, wavefront/wavefront_engine.py:275-378), so
the whole forward loop and the whole backward loop can each be captured once as a CUDA graph
and replayed per call: one graph launch instead of thousands of kernel launches and Python
calls.

    g = GraphedWavefrontEngine(engine, x_example)      # or engine.graphed(x_example)
    grids = g(x)                                        # same outputs as engine(x)
    loss(grids).backward()                              # x.grad and every parameter's .grad

Contract (what capture freezes):
  * x has the example's shape and dtype; call under the same autocast state as the capture;
  * the layers' parameter tensors stay the same objects (in-place optimizer updates are seen:
    the graph re-stacks them from their addresses at every replay);
  * the returned grids are views of the engine's static output buffers, as in the eager engine
    (and the reference's): the next call overwrites them;
  * the cell must be capturable (no host synchronisation, no data-dependent shapes).
Tanh grid cells that take the persistent-kernel fast path need no graph; the runner refuses
them (call the engine directly). FLB block cells (bf16) capture the native whole-grid forward
and backward (wavefront.flb_cells) instead of the tick loops.
"""
from __future__ import annotations

import math

import torch

import flb_native as nat
import wavefront_backend
from .wavefront_engine import refresh_stacked_params, layer_grad_accumulators
from .wavefront_kernel import run_fetch_kernel


class _GraphedEngineFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, runner, x, n_states, *rest):
        states, params = rest[:n_states], rest[n_states:]
        ctx.runner = runner
        ctx.has_states = [s is not None for s in states]
        ctx.n_params = len(params)
        eng = runner.engine
        ws = eng.graph_workspace
        nc, dock = runner.num_cells, runner.num_layers
        ws["static_x"].copy_(x)
        grids = ws["static_stacked_grids"]
        grids[:, nc:nc + dock].zero_()
        for p, s in enumerate(states):
            if s is not None:
                grids[p][nc:nc + dock].copy_(s)
        runner.g_fwd.replay()
        return tuple(grids[p][:nc] for p in range(eng.config.num_ports))

    @staticmethod
    def backward(ctx, *grad_grids):
        runner = ctx.runner
        eng = runner.engine
        ws = eng.graph_workspace
        nc, dock = runner.num_cells, runner.num_layers
        for i, g in enumerate(grad_grids):
            if g is not None:
                ws["static_grad_outputs"][i][:nc].copy_(g)
            else:
                ws["static_grad_outputs"][i][:nc].zero_()
        if runner.g_bwd is None:
            raise RuntimeError("GraphedWavefrontEngine was captured with backward=False")
        runner.g_bwd.replay()
        if runner.native_flb:
            from .flb_cells import flb_param_grads
            grad_params = flb_param_grads(eng, runner.flb_grads)
            return (None, runner.flb_dx.to(ws["static_x"].dtype).clone(), None,
                    *([None] * len(ctx.has_states)), *grad_params)
        grad_x = ws["static_grad_x"].clone()
        grad_states = [ws["static_current_grad_grids"][p][nc:nc + dock].clone() if has else None
                       for p, has in enumerate(ctx.has_states)]
        # copies: autograd may keep a returned gradient as param.grad itself, and the
        # accumulators are overwritten by the next replay
        grad_params = [runner.accs[name][li].to(p.dtype, copy=True)
                       for li, name, p in runner.param_slots]
        return (None, grad_x, None, *grad_states, *grad_params)


class GraphedWavefrontEngine:
    """Forward and backward tick loops of `engine` captured as two CUDA graphs (see module
    docstring). `x` is an example input: its shape and dtype are frozen; its values are only
    used for the warm-up runs. backward=False captures the forward only (inference)."""

    def __init__(self, engine, x: torch.Tensor, warmup: int = 2, backward: bool = True):
        nat.require_cuda(x)
        from .grid_layer import fast_path_applies
        if fast_path_applies(engine, x):
            raise ValueError("GraphedWavefrontEngine: these layers take the persistent grid "
                             "kernels already; call the engine directly")
        self.engine = engine
        self.with_backward = backward
        cfg = engine.config
        self.num_cells = math.prod(cfg.grid_shape)
        self.num_layers = cfg.grid_shape[0]
        self.x_shape, self.x_dtype = tuple(x.shape), x.dtype
        engine._init_buffers(x)
        from .flb_cells import native_flb_applies
        # FLB block cells: the graphs capture the native whole-grid forward and backward
        self.native_flb = native_flb_applies(engine, x)
        ws = engine.graph_workspace
        self.accs = layer_grad_accumulators(ws, engine.stacked_params, self.num_layers, x.device)
        # (layer index, stacked-parameter name, parameter) in the order grads are returned
        self.param_slots = [(li, name, p) for li, layer in enumerate(engine.layers)
                            for name, p in layer.named_parameters()]
        missing = [n for _, n, _ in self.param_slots if n not in self.accs]
        if missing:
            raise ValueError(f"GraphedWavefrontEngine: layers differ in parameters ({missing})")

        with torch.no_grad():
            ws["static_x"].copy_(x)
            ws["static_stacked_grids"][:, self.num_cells:self.num_cells + self.num_layers].zero_()
            for g in ws["static_grad_outputs"]:
                g.zero_()
        # warm-up outside capture (lazy initialisation in vmap / cuBLAS / the library), then
        # one capture per direction in a shared memory pool
        side = torch.cuda.Stream(x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._forward_loop()
                if backward:
                    self._backward_loop()
        torch.cuda.current_stream(x.device).wait_stream(side)
        pool = torch.cuda.graph_pool_handle()
        self.g_fwd = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.g_fwd, pool=pool):
            self._forward_loop()
        self.g_bwd = None
        if backward:
            self.g_bwd = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.g_bwd, pool=pool):
                self._backward_loop()

    # the captured bodies: static buffers in, static buffers out
    def _forward_loop(self):
        eng, cfg = self.engine, self.engine.config
        ws = eng.graph_workspace
        if self.native_flb:
            from .flb_cells import native_flb_forward, BlockWeightStacks, saved_buffer
            self.flb_weights = BlockWeightStacks(list(eng.layers))
            # a graph for training keeps the cells' intermediates for the backward graph
            self.flb_saved = saved_buffer(eng, ws["static_x"].device) if self.with_backward else None
            native_flb_forward(eng, ws["static_x"], ws["static_stacked_grids"],
                               weights=self.flb_weights, saved=self.flb_saved)
            return
        refresh_stacked_params(eng.layers, eng.stacked_params)
        with torch.no_grad():
            wavefront_backend.execute_forward(
                eng.active_cells_buffer.shape[0], cfg.num_ports, run_fetch_kernel,
                eng.batched_forward, eng.active_cells_buffer, ws["static_x"],
                ws["static_stacked_grids"], eng.routing_map, eng.port_map,
                eng.spatial_map_buffer, eng.gathered_out_buffer, eng.bwd_cache,
                eng.stacked_params, cfg)

    def _backward_loop(self):
        eng, cfg = self.engine, self.engine.config
        ws = eng.graph_workspace
        if self.native_flb:
            from .flb_cells import native_flb_backward
            n = self.num_cells
            self.flb_grads, self.flb_dx = native_flb_backward(
                eng, self.flb_weights, [g[:n] for g in ws["static_grad_outputs"]],
                saved=self.flb_saved)
            return
        wavefront_backend.execute_backward(
            eng.active_cells_buffer.shape[0], cfg.num_ports, len(cfg.dependencies),
            self.num_cells, eng.compiled_backward, eng.active_cells_buffer,
            eng.gathered_out_buffer, ws["static_grad_x"], ws["static_current_grad_grids"],
            ws["static_grad_outputs"], self.accs, eng.bwd_cache, eng.stacked_params,
            cfg.dependencies)

    def __call__(self, x: torch.Tensor, initial_states: dict | None = None):
        nat.require_cuda(x)
        if tuple(x.shape) != self.x_shape or x.dtype != self.x_dtype:
            raise ValueError(f"GraphedWavefrontEngine: captured for x {self.x_shape} "
                             f"{self.x_dtype}, got {tuple(x.shape)} {x.dtype}")
        ports = self.engine.config.num_ports
        states = [(initial_states or {}).get(p) for p in range(ports)]
        params = [p for _, _, p in self.param_slots]
        return _GraphedEngineFunction.apply(self, x, ports, *states, *params)
