"""Wavefront engine: grid-structured layers evaluated along anti-diagonals.

Same API as the reference (wavefront/wavefront_engine.py): `WavefrontEngine(config, layers)`
is an nn.Module whose forward(x, initial_states=None) returns `num_ports` grids of shape
[num_cells, batch, dim] (cells in row-major order), differentiable w.r.t. x and every layer
parameter; `WavefrontEngineFunction` is its autograd.Function.

What runs where:
  * the per-tick loop is the native C++ module `wavefront_backend` (execute_forward /
    execute_backward, the reference's signatures); its gathers and scatters are CUDA kernels
    of libflb_b200.so;
  * the cell itself is the user's layer, called batched over a tick's cells through
    torch.vmap / torch.func.vjp exactly as in the reference (:185-236) - that is what a
    generic nn.Module layer needs;
  * parameter gradients are accumulated per layer on the fly (float32 [num_layers, *shape]),
    instead of the reference's per-cell copies ([num_cells + 1, *shape], :99-104), which
    need ~1 GB per 256x256 matrix at a 64x64 grid.

For the tanh grid cell (wavefront.grid_layer.TanhGridCell) the engine bypasses the tick loop
and runs the persistent single-kernel wavefront (flb_grid_fwd / flb_grid_bwd).
"""
from __future__ import annotations

import math
import itertools

import torch
import torch.nn as nn
from torch.func import stack_module_state
from torch.amp import custom_fwd, custom_bwd

from .wavefront_api import WavefrontConfig, generate_wavefront_schedule
from .wavefront_kernel import run_fetch_kernel
import flb_native as nat
import wavefront_backend


def refresh_stacked_params(layers, stacked_params) -> None:
    """Copy the layers' live parameters into the engine's stacked [num_layers, ...] copies."""
    with torch.no_grad():
        live, _ = stack_module_state(list(layers))
        if live:
            torch._foreach_copy_(list(stacked_params.values()), list(live.values()))


def layer_grad_accumulators(ws, stacked_params, num_layers, device) -> dict:
    """float32 [num_layers, *param] gradient accumulators, created once per workspace."""
    if "layer_grad_accumulators" not in ws:
        ws["layer_grad_accumulators"] = {
            k: torch.zeros((num_layers,) + v.shape[1:], dtype=torch.float32, device=device)
            for k, v in stacked_params.items()
        }
    return ws["layer_grad_accumulators"]


class WavefrontEngineFunction(torch.autograd.Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, compiled_backward, x, layers, config, routing_map, port_map,
                active_cells_buffer, active_layers_buffer, gathered_out_buffer, stacked_params,
                bwd_cache, graph_workspace, spatial_map_buffer, batched_forward, *initial_states):
        ctx.compiled_backward = compiled_backward
        ctx.has_initial_states = [s is not None for s in initial_states]
        ctx.active_cells_buffer = active_cells_buffer
        ctx.gathered_out_buffer = gathered_out_buffer
        ctx.layers = layers
        ctx.config = config
        ctx.stacked_params = stacked_params
        ctx.bwd_cache = bwd_cache
        ctx.graph_workspace = graph_workspace

        num_cells = math.prod(config.grid_shape)
        num_ticks = active_cells_buffer.shape[0]
        static_x = graph_workspace["static_x"]
        static_stacked_grids = graph_workspace["static_stacked_grids"]

        refresh_stacked_params(layers, stacked_params)
        static_x.copy_(x)

        with torch.no_grad():
            wavefront_backend.execute_forward(
                num_ticks, config.num_ports, run_fetch_kernel, batched_forward,
                active_cells_buffer, static_x, static_stacked_grids, routing_map, port_map,
                spatial_map_buffer, gathered_out_buffer, bwd_cache, stacked_params, config)

        ctx.save_for_backward(static_x, static_stacked_grids)
        return tuple(static_stacked_grids[p][:num_cells] for p in range(config.num_ports))

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, *grad_output_grids):
        x, _ = ctx.saved_tensors
        layers, config = ctx.layers, ctx.config
        num_cells = math.prod(config.grid_shape)
        num_deps = len(config.dependencies)
        num_ticks = ctx.active_cells_buffer.shape[0]
        num_layers = config.grid_shape[0]
        ws = ctx.graph_workspace

        accs = layer_grad_accumulators(ws, ctx.stacked_params, num_layers, x.device)
        for i, g in enumerate(grad_output_grids):
            if g is not None:
                ws["static_grad_outputs"][i][:num_cells].copy_(g)
            else:
                ws["static_grad_outputs"][i][:num_cells].zero_()

        wavefront_backend.execute_backward(
            num_ticks, config.num_ports, num_deps, num_cells, ctx.compiled_backward,
            ctx.active_cells_buffer, ctx.gathered_out_buffer, ws["static_grad_x"],
            ws["static_current_grad_grids"], ws["static_grad_outputs"], accs, ctx.bwd_cache,
            ctx.stacked_params, config.dependencies)

        with torch.no_grad():
            for i, layer in enumerate(layers):
                for name, param in layer.named_parameters():
                    g = accs[name][i].to(param.dtype)
                    if param.grad is None:
                        param.grad = g.clone()
                    else:
                        param.grad.add_(g)

        grad_initial_states = []
        for p, has in enumerate(ctx.has_initial_states):
            grad_initial_states.append(
                ws["static_current_grad_grids"][p][num_cells:num_cells + num_layers].clone()
                if has else None)
        return tuple([None, ws["static_grad_x"].clone()] + [None] * 12 + grad_initial_states)


class WavefrontEngine(nn.Module):
    def __init__(self, config: WavefrontConfig, layers: nn.ModuleList):
        super().__init__()
        self.config = config
        self.layers = layers
        self.schedule = generate_wavefront_schedule(config)
        r_map = self._build_routing_map()
        self.register_buffer("routing_map", r_map)
        self.routing_map_list = r_map.tolist()
        self.register_buffer("port_map", torch.tensor([d[1] for d in config.dependencies],
                                                      dtype=torch.int32))
        self.compiled_cells, self.compiled_layers, self.max_cells_per_tick = self._compile_schedule()
        self.active_cells_buffer = None
        self.active_layers_buffer = None
        self.gathered_out_buffer = None

        def pure_layer_forward(params, *inputs):
            with torch.amp.autocast("cuda", dtype=inputs[0].dtype):
                reshaped = tuple(inp.unsqueeze(1) for inp in inputs)
                outs = torch.func.functional_call(self.layers[0], params, reshaped)
                return tuple(o.squeeze(1).to(inputs[0].dtype) for o in outs)

        self.batched_forward = torch.vmap(pure_layer_forward, randomness="different")

        def core_backward(cell_params, tracked, grads):
            return torch.func.vjp(self.batched_forward, cell_params, *tracked)[1](grads)

        def static_backward_step(cell_params, tracked, grads):
            # zero tensors stand in for missing / storage-less gradients (reference :200-233)
            ref = tracked[0]
            def safe(t):
                if t is None or t.numel() == 0:
                    return torch.zeros(ref.shape, dtype=ref.dtype, device=ref.device)
                return t
            return core_backward(cell_params, tuple(safe(t) for t in tracked),
                                 tuple(safe(g) for g in grads))

        self.compiled_backward = static_backward_step

    def forward(self, x: torch.Tensor, initial_states: dict = None):
        nat.require_cuda(x)
        from .grid_layer import engine_fast_path
        fast = engine_fast_path(self, x, initial_states)
        if fast is not None:
            return fast
        from .flb_cells import (native_flb_applies, no_grad_needed, native_flb_forward,
                                native_flb_train_forward)
        if native_flb_applies(self, x) and not no_grad_needed(self, x):
            # FLB block cells, training: flb_block_grid_fwd / flb_block_grid_bwd
            return native_flb_train_forward(self, x)
        if native_flb_applies(self, x):
            # FLB block cells, inference: the whole grid in flb_block_grid_fwd (no tick loop
            # through Python; initial states reach no cell, as in the per-tick path)
            self._init_buffers(x)
            ws = self.graph_workspace
            ws["static_x"].copy_(x)
            native_flb_forward(self, ws["static_x"], ws["static_stacked_grids"])
            n = math.prod(self.config.grid_shape)
            return tuple(ws["static_stacked_grids"][p][:n] for p in range(self.config.num_ports))
        if initial_states is None:
            initial_states = {}
        self._init_buffers(x)
        num_cells = math.prod(self.config.grid_shape)
        dock = self.config.grid_shape[0]
        grids = self.graph_workspace["static_stacked_grids"]
        grids[:, num_cells:num_cells + dock].zero_()
        states = []
        for p in range(self.config.num_ports):
            if p in initial_states:
                grids[p][num_cells:num_cells + dock].copy_(initial_states[p])
                states.append(initial_states[p])
            else:
                states.append(None)
        return WavefrontEngineFunction.apply(
            self.compiled_backward, x, self.layers, self.config, self.routing_map,
            self.port_map, self.active_cells_buffer, self.active_layers_buffer,
            self.gathered_out_buffer, self.stacked_params, self.bwd_cache, self.graph_workspace,
            self.spatial_map_buffer, self.batched_forward, *states)

    def graphed(self, x: torch.Tensor, warmup: int = 2, backward: bool = True):
        """This engine's per-tick forward (and backward) captured as CUDA graphs for inputs
        shaped like `x` (wavefront.wavefront_graph.GraphedWavefrontEngine)."""
        from .wavefront_graph import GraphedWavefrontEngine
        return GraphedWavefrontEngine(self, x, warmup=warmup, backward=backward)

    # ---- host-side set-up (reference :275-438) ------------------------------------------------
    def _init_buffers(self, x):
        compute_dtype = (torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda")
                         else x.dtype)
        if (self.active_cells_buffer is not None and self.active_cells_buffer.device == x.device
                and self.gathered_out_buffer.dtype == compute_dtype):
            return
        dev = x.device
        if self.port_map.device != dev:
            self.routing_map = self.routing_map.to(dev)
            self.port_map = self.port_map.to(dev)
        cfg = self.config
        num_ticks = len(self.compiled_cells)
        num_deps = len(cfg.dependencies)
        num_cells = math.prod(cfg.grid_shape)
        seq_len = cfg.grid_shape[1]
        layers_n = cfg.grid_shape[0]
        self.spatial_map_buffer = torch.tensor([i % seq_len for i in range(num_cells)] + [0],
                                               dtype=torch.int32, device=dev)
        self.active_cells_buffer = torch.tensor(self.compiled_cells, dtype=torch.int32, device=dev)
        self.active_layers_buffer = torch.tensor(self.compiled_layers, dtype=torch.int32, device=dev)
        self.gathered_out_buffer = torch.zeros(
            (num_ticks, num_deps, self.max_cells_per_tick, x.shape[0], cfg.dim),
            device=dev, dtype=compute_dtype)
        if not hasattr(self, "stacked_params"):
            params, _ = stack_module_state(list(self.layers))
            self.stacked_params = {k: v.detach().clone() for k, v in params.items()}
        else:
            self.stacked_params = {k: v.to(dev) for k, v in self.stacked_params.items()}

        # per-tick index lists, built on the host once (int64 for the native loop)
        routing = self.routing_map_list
        self.bwd_cache = {}
        for t, (cells, lays) in enumerate(zip(self.compiled_cells, self.compiled_layers)):
            valid_idx = [s for s, l in enumerate(lays) if l >= 0]
            valid_cells = [cells[s] for s in valid_idx]
            deps = []
            for i in range(num_deps):
                tg = [routing[c * num_deps + i] for c in valid_cells]
                x_idx = [k for k, v in enumerate(tg) if v == -2]
                grid_idx = [k for k, v in enumerate(tg) if v >= 0]
                deps.append({
                    "x_idx": torch.tensor(x_idx, dtype=torch.int64, device=dev),
                    "x_targets": torch.tensor([valid_cells[k] % (num_cells // layers_n)
                                               for k in x_idx], dtype=torch.int64, device=dev),
                    "grid_idx": torch.tensor(grid_idx, dtype=torch.int64, device=dev),
                    "grid_targets": torch.tensor([tg[k] for k in grid_idx], dtype=torch.int64,
                                                 device=dev),
                })
            self.bwd_cache[t] = {
                "safe_layer_indices": torch.tensor([max(l, 0) for l in lays], dtype=torch.int64,
                                                   device=dev),
                "valid_cells": torch.tensor(valid_cells, dtype=torch.int64, device=dev),
                "valid_idx": torch.tensor(valid_idx, dtype=torch.int64, device=dev),
                "valid_layers": torch.tensor([lays[s] for s in valid_idx], dtype=torch.int64,
                                             device=dev),
                "deps": deps,
            }

        batch, dim = cfg.batch_size, cfg.dim
        dock = cfg.grid_shape[0]
        if (not hasattr(self, "graph_workspace")
                or self.graph_workspace["static_x"].dtype != compute_dtype
                or self.graph_workspace["static_x"].device != dev):
            self.graph_workspace = {
                "static_x": torch.zeros((batch, seq_len, dim), device=dev, dtype=compute_dtype),
                "static_stacked_grids": torch.zeros((cfg.num_ports, num_cells + dock, batch, dim),
                                                    device=dev, dtype=compute_dtype),
                "static_grad_x": torch.zeros((batch, seq_len, dim), device=dev, dtype=compute_dtype),
                "static_grad_outputs": [torch.zeros((num_cells + dock, batch, dim), device=dev,
                                                    dtype=compute_dtype) for _ in range(cfg.num_ports)],
                "static_current_grad_grids": [torch.zeros((num_cells + dock, batch, dim), device=dev,
                                                          dtype=compute_dtype)
                                              for _ in range(cfg.num_ports)],
            }

    def _compile_schedule(self):
        shape = self.config.grid_shape
        num_cells = math.prod(shape)
        max_cells = max(len(g) for g in self.schedule)
        cells_out, layers_out = [], []
        for group in self.schedule:
            cells = [self._flat(c) for c in group]
            lays = [c[0] for c in group]
            cells += [num_cells] * (max_cells - len(cells))
            lays += [-1] * (max_cells - len(lays))
            cells_out.append(cells)
            layers_out.append(lays)
        return cells_out, layers_out, max_cells

    def _flat(self, coord) -> int:
        idx, stride = 0, 1
        for d in reversed(range(len(self.config.grid_shape))):
            idx += coord[d] * stride
            stride *= self.config.grid_shape[d]
        return idx

    def _build_routing_map(self) -> torch.Tensor:
        """int32 [cells * deps]: source flat cell (>= 0), -2 = x input (the offset leaves the
        grid only through row -1), -1 = zero (reference :416-438)."""
        shape = self.config.grid_shape
        deps = self.config.dependencies
        out = torch.full((math.prod(shape) * len(deps),), -1, dtype=torch.int32)
        for coord in itertools.product(*[range(s) for s in shape]):
            cur = self._flat(coord)
            for di, (off, _) in enumerate(deps):
                tgt = tuple(c + d for c, d in zip(coord, off))
                pos = cur * len(deps) + di
                if all(0 <= tgt[i] < shape[i] for i in range(len(coord))):
                    out[pos] = self._flat(tgt)
                elif tgt[0] == -1 and all(0 <= tgt[i] < shape[i] for i in range(1, len(coord))):
                    out[pos] = -2
        return out
