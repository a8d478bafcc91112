"""Dependency gather of the wavefront engine.

`fetch_mapped_context` is the per-cell Python twin used for host-side checks (same contract as
wavefront/wavefront_kernel.py:6-25 of the reference). `run_fetch_kernel` has the reference
launcher's signature (:84-106) but runs the library's CUDA gather (flb_wf_gather), which
restates fetch_mapped_context_kernel (:27-82). The C++ tick loop recognises it by the
`__flb_native__` attribute and calls flb_wf_gather directly, without a Python round trip.
"""
from __future__ import annotations

import math

import torch

import flb_native as nat


def fetch_mapped_context(x, output_grids, cell_idx, routing_map, config):
    num_deps = len(config.dependencies)
    ingredients = []
    base = cell_idx * num_deps
    for i in range(num_deps):
        target = int(routing_map[base + i])
        _, port = config.dependencies[i]
        if target == -1:
            ingredients.append(torch.zeros_like(output_grids[0][0]))
        elif target == -2:
            spatial_size = output_grids[0].shape[0] // config.grid_shape[0]
            x_flat = x.view(config.batch_size, spatial_size, config.dim)
            ingredients.append(x_flat[:, cell_idx % spatial_size, :])
        else:
            ingredients.append(output_grids[port][target])
    return ingredients


def run_fetch_kernel(x, stacked_grids, routing_map, port_map, spatial_map, config,
                     active_cells_tensor, gathered_out):
    """gathered_out[dep, slot, b, :] for every active slot; see flb_wf_gather."""
    nat.require_cuda(x, stacked_grids, gathered_out)
    if not (x.dtype == stacked_grids.dtype == gathered_out.dtype):
        raise TypeError("x, stacked_grids and gathered_out must share a dtype")
    num_deps = len(config.dependencies)
    num_cells = math.prod(config.grid_shape)
    routing = routing_map.to(torch.int32).contiguous()
    ports = port_map.to(torch.int32).contiguous()
    spatial = spatial_map.to(torch.int32).contiguous()
    active = active_cells_tensor.to(torch.int32).contiguous()
    nat.check(nat.lib.flb_wf_gather(
        x.data_ptr(), nat.strides(*x.stride()), stacked_grids.data_ptr(),
        nat.strides(*stacked_grids.stride()), routing.data_ptr(), ports.data_ptr(),
        spatial.data_ptr(), active.data_ptr(), active.numel(), num_cells,
        gathered_out.data_ptr(), nat.strides(*gathered_out.stride()), num_deps, x.shape[0],
        config.dim, nat.dtype_code(x.dtype), nat.stream_of(x)), "flb_wf_gather")
    return gathered_out


run_fetch_kernel.__flb_native__ = True
