// wavefront_backend: the C++ tick-loop orchestrator of the wavefront engine, with the exact
// signatures of the reference module (csrc/wavefront_backend.cpp:7-15, :48-56, bound at
// :134-137) so wavefront/wavefront_engine.py and any caller of the reference module use it
// unchanged.
//
// Differences from the reference, none visible at the Python boundary:
//   - the dependency gather runs the library's CUDA gather (flb_wf_gather) directly from C++
//     when the engine passes the native launcher (it carries `__flb_native__`); any other
//     `run_fetch_kernel` callable is honoured as a Python callback;
//   - every index_put_ / index_add_ of the tick loop is one flb_wf_index_copy launch on the
//     current CUDA stream (no ATen indexing kernels);
//   - parameter gradients go straight into per-layer accumulators when the accumulator's
//     leading dimension is not num_cells + 1 and the tick cache carries "valid_layers"
//     (the reference keeps one copy per cell: [num_cells + 1, *param.shape]);
//   - the GIL is held only around the Python callbacks' own calls.
// There is no CPU path: every tensor must be a CUDA tensor.
#include <torch/extension.h>
#include <pybind11/pybind11.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/cuda/CUDAGuard.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "flb_b200.h"

namespace py = pybind11;

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return FLB_F32;
    case at::kHalf: return FLB_F16;
    case at::kBFloat16: return FLB_BF16;
    default: throw std::invalid_argument("wavefront_backend: unsupported dtype " +
                                         std::string(c10::toString(t.scalar_type())));
  }
}

void check(int st, const char* what) {
  if (st != FLB_OK) throw std::runtime_error(std::string(what) + ": " + flb_last_error());
}

void require_cuda(const at::Tensor& t, const char* name) {
  if (!t.is_cuda())
    throw std::invalid_argument(std::string("wavefront_backend: ") + name +
                                " must be a CUDA tensor (this backend has no CPU path)");
}

void* cur_stream(const at::Tensor& t) {
  return reinterpret_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

at::Tensor as_i64(const at::Tensor& t) {
  return t.scalar_type() == at::kLong ? t.contiguous() : t.to(at::kLong).contiguous();
}

// View of a tensor as [rows, batch, dim] strides (elements).
struct RBD {
  int64_t s[3];
};
RBD rbd(const at::Tensor& t) {
  if (t.dim() == 3) return {{t.stride(0), t.stride(1), t.stride(2)}};
  if (t.dim() == 2) return {{t.stride(0), 0, t.stride(1)}};
  throw std::invalid_argument("wavefront_backend: expected a 2-D or 3-D tensor");
}

// dst[dst_rows] (=|+=) src[src_rows] on [rows, batch, dim] views
void index_copy(const at::Tensor& src, const at::Tensor& src_rows, const at::Tensor& dst,
                const at::Tensor& dst_rows, bool accumulate) {
  const int64_t n = src_rows.numel();
  if (n == 0) return;
  if (dst_rows.numel() != n) throw std::invalid_argument("wavefront_backend: row index length mismatch");
  RBD ss = rbd(src), ds = rbd(dst);
  const int64_t batch = src.dim() == 3 ? src.size(1) : 1;
  const int64_t dim = src.size(src.dim() - 1);
  check(flb_wf_index_copy(src.data_ptr(), dtype_code(src), ss.s, src_rows.data_ptr<int64_t>(),
                          dst.data_ptr(), dtype_code(dst), ds.s, dst_rows.data_ptr<int64_t>(), n,
                          batch, dim, accumulate ? 1 : 0, cur_stream(dst)),
        "flb_wf_index_copy");
}

int64_t cfg_int(const py::object& config, const char* name) {
  return py::cast<int64_t>(config.attr(name));
}

}  // namespace

// FORWARD: restates execute_forward (csrc/wavefront_backend.cpp:7-45).
void execute_forward(int num_ticks, int num_ports, py::function run_fetch_kernel,
                     py::function batched_forward, torch::Tensor active_cells_buffer,
                     torch::Tensor static_x, torch::Tensor static_stacked_grids,
                     torch::Tensor routing_map, torch::Tensor port_map,
                     torch::Tensor spatial_map_buffer, torch::Tensor gathered_out_buffer,
                     py::dict bwd_cache, py::dict stacked_params, py::object config) {
  require_cuda(static_stacked_grids, "static_stacked_grids");
  require_cuda(gathered_out_buffer, "gathered_out_buffer");
  c10::cuda::CUDAGuard guard(static_stacked_grids.device());
  const bool native = py::hasattr(run_fetch_kernel, "__flb_native__");
  const int64_t num_deps = py::len(config.attr("dependencies"));
  py::tuple grid_shape = config.attr("grid_shape");
  int64_t num_cells = 1;
  for (auto g : grid_shape) num_cells *= py::cast<int64_t>(g);
  const int dt = dtype_code(static_stacked_grids);
  if (native) {
    require_cuda(static_x, "static_x");
    if (static_x.scalar_type() != static_stacked_grids.scalar_type() ||
        gathered_out_buffer.scalar_type() != static_stacked_grids.scalar_type())
      throw std::invalid_argument("wavefront_backend: x, grids and gathered buffers must share a dtype");
  }
  // per-port grid views [cells, batch, dim]
  std::vector<at::Tensor> port_grids;
  for (int p = 0; p < num_ports; ++p) port_grids.push_back(static_stacked_grids[p]);

  for (int i = 0; i < num_ticks; ++i) {
    at::Tensor cell_indices = active_cells_buffer[i];
    at::Tensor gathered_out = gathered_out_buffer[i];  // [deps, max_cells, batch, dim]

    if (native) {
      const int64_t xs[3] = {static_x.stride(0), static_x.stride(1), static_x.stride(2)};
      const int64_t gs[4] = {static_stacked_grids.stride(0), static_stacked_grids.stride(1),
                             static_stacked_grids.stride(2), static_stacked_grids.stride(3)};
      const int64_t os[4] = {gathered_out.stride(0), gathered_out.stride(1),
                             gathered_out.stride(2), gathered_out.stride(3)};
      check(flb_wf_gather(static_x.data_ptr(), xs, static_stacked_grids.data_ptr(), gs,
                          routing_map.data_ptr<int32_t>(), port_map.data_ptr<int32_t>(),
                          spatial_map_buffer.data_ptr<int32_t>(), cell_indices.data_ptr<int32_t>(),
                          cell_indices.numel(), num_cells, gathered_out.data_ptr(), os, num_deps,
                          static_x.size(0), static_x.size(2), dt, cur_stream(gathered_out)),
            "flb_wf_gather");
    } else {
      run_fetch_kernel(static_x, static_stacked_grids, routing_map, port_map, spatial_map_buffer,
                       config, cell_indices, gathered_out);
    }

    py::dict tick_cache = bwd_cache[py::cast(i)].cast<py::dict>();
    at::Tensor safe_layer_indices = tick_cache["safe_layer_indices"].cast<at::Tensor>();
    at::Tensor valid_cells = as_i64(tick_cache["valid_cells"].cast<at::Tensor>());
    at::Tensor valid_idx = as_i64(tick_cache["valid_idx"].cast<at::Tensor>());

    py::dict tick_cell_params;
    for (auto item : stacked_params) {
      at::Tensor param = item.second.cast<at::Tensor>();
      tick_cell_params[item.first] = param.index_select(0, safe_layer_indices.to(at::kLong));
    }
    std::vector<at::Tensor> ingredients = torch::unbind(gathered_out, 0);
    py::tuple py_ingredients = py::cast(ingredients);
    py::tuple out_tuple = batched_forward(tick_cell_params, *py_ingredients);

    for (int p = 0; p < num_ports; ++p) {
      at::Tensor port_output = out_tuple[p].cast<at::Tensor>();
      require_cuda(port_output, "cell output");
      index_copy(port_output, valid_idx, port_grids[p], valid_cells, /*accumulate=*/false);
    }
  }
}

// BACKWARD: restates execute_backward (csrc/wavefront_backend.cpp:48-132).
void execute_backward(int num_ticks, int num_ports, int num_deps, int num_cells,
                      py::function batched_backward_step, torch::Tensor active_cells_buffer,
                      torch::Tensor gathered_out_buffer, torch::Tensor static_grad_x,
                      std::vector<torch::Tensor> static_current_grad_grids,
                      std::vector<torch::Tensor> static_grad_outputs,
                      py::dict static_cell_grad_accumulators, py::dict bwd_cache,
                      py::dict stacked_params, py::list dependencies) {
  require_cuda(gathered_out_buffer, "gathered_out_buffer");
  require_cuda(static_grad_x, "static_grad_x");
  c10::cuda::CUDAGuard guard(gathered_out_buffer.device());

  // 1. clean the slate (csrc/wavefront_backend.cpp:57-62)
  static_grad_x.zero_();
  for (auto& g : static_current_grad_grids) g.zero_();
  for (auto item : static_cell_grad_accumulators) item.second.cast<at::Tensor>().zero_();

  // 2. starting errors (:64-67)
  for (int i = 0; i < num_ports; ++i)
    static_current_grad_grids[i].slice(0, 0, num_cells).copy_(static_grad_outputs[i].slice(0, 0, num_cells));

  // grad_x viewed as [seq, batch, dim] so index rows are sequence positions (index_add_ on dim 1)
  at::Tensor gx_view = static_grad_x.transpose(0, 1);

  for (int t = num_ticks - 1; t >= 0; --t) {
    at::Tensor cell_indices = active_cells_buffer[t];
    at::Tensor gathered_tensors = gathered_out_buffer[t];

    py::dict tick_cache = bwd_cache[py::cast(t)].cast<py::dict>();
    at::Tensor safe_layer_indices = tick_cache["safe_layer_indices"].cast<at::Tensor>();
    at::Tensor valid_idx = as_i64(tick_cache["valid_idx"].cast<at::Tensor>());
    at::Tensor valid_cells = as_i64(tick_cache["valid_cells"].cast<at::Tensor>());
    const bool has_layers = tick_cache.contains("valid_layers");

    py::dict cell_params;
    for (auto item : stacked_params)
      cell_params[item.first] = item.second.cast<at::Tensor>().index_select(0, safe_layer_indices.to(at::kLong));

    std::vector<at::Tensor> tracked = torch::unbind(gathered_tensors, 0);
    py::tuple py_tracked = py::cast(tracked);

    at::Tensor cell_rows = as_i64(cell_indices);
    std::vector<at::Tensor> batched_grads;
    for (int p = 0; p < num_ports; ++p)
      batched_grads.push_back(static_current_grad_grids[p].index_select(0, cell_rows));
    py::tuple py_batched_grads = py::cast(batched_grads);

    py::tuple grad_returns = batched_backward_step(cell_params, py_tracked, py_batched_grads);

    // 5. parameter gradients (:96-106)
    py::dict grad_params = grad_returns[0].cast<py::dict>();
    for (auto item : grad_params) {
      if (item.second.is_none()) continue;
      at::Tensor g = item.second.cast<at::Tensor>();
      at::Tensor acc = static_cell_grad_accumulators[item.first].cast<at::Tensor>();
      if (!acc.is_contiguous()) throw std::invalid_argument("wavefront_backend: accumulators must be contiguous");
      at::Tensor g2 = g.reshape({g.size(0), -1});
      at::Tensor acc2 = acc.view({acc.size(0), -1});
      const bool per_cell = acc.size(0) == (int64_t)num_cells + 1 || !has_layers;
      if (per_cell) {
        index_copy(g2, valid_idx, acc2, valid_cells, /*accumulate=*/false);
      } else {
        at::Tensor valid_layers = as_i64(tick_cache["valid_layers"].cast<at::Tensor>());
        index_copy(g2, valid_idx, acc2, valid_layers, /*accumulate=*/true);
      }
    }

    // 6. dependency gradients (:108-130)
    py::list deps_cache = tick_cache["deps"].cast<py::list>();
    for (int i = 0; i < num_deps; ++i) {
      py::tuple dep_tuple = dependencies[i].cast<py::tuple>();
      const int source_port = dep_tuple[1].cast<int>();
      py::dict dep_cache = deps_cache[i].cast<py::dict>();
      at::Tensor dep_grads = grad_returns[i + 1].cast<at::Tensor>();  // [max_cells, batch, dim]

      at::Tensor x_targets = dep_cache["x_targets"].cast<at::Tensor>();
      if (x_targets.numel() > 0) {
        at::Tensor x_idx = as_i64(dep_cache["x_idx"].cast<at::Tensor>());
        at::Tensor src_rows = valid_idx.index_select(0, x_idx);
        index_copy(dep_grads, src_rows, gx_view, as_i64(x_targets), /*accumulate=*/true);
      }
      at::Tensor grid_targets = dep_cache["grid_targets"].cast<at::Tensor>();
      if (grid_targets.numel() > 0) {
        at::Tensor grid_idx = as_i64(dep_cache["grid_idx"].cast<at::Tensor>());
        at::Tensor src_rows = valid_idx.index_select(0, grid_idx);
        index_copy(dep_grads, src_rows, static_current_grad_grids[source_port],
                   as_i64(grid_targets), /*accumulate=*/true);
      }
    }
  }
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "FLB wavefront tick-loop orchestrator (B200 build; CUDA tensors only)";
  m.def("execute_forward", &execute_forward, "C++ Forward Pass Loop");
  m.def("execute_backward", &execute_backward, "C++ Backward Pass Loop");
}
