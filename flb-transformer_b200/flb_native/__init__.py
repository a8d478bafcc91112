"""ctypes binding of libflb_b200.so, the C ABI declared in include/flb_b200.h.

Every compute entry point of this package goes through here. There is no fallback: if the
library is missing, importing this module raises, and every call that reports a non-zero
status raises RuntimeError with the library's message.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(_HERE)
LIB_PATH = os.path.join(_ROOT, "libflb_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build the CUDA library first "
        f"(python {os.path.join(_ROOT, 'build.py')})")

lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)

F32, F16, BF16 = 0, 1, 2
ATTN_CAUSAL, ATTN_EXACT_TANH, ATTN_FORCE_GENERIC = 1, 2, 4

STATUS_NAMES = {0: "OK", 1: "SHAPE", 2: "DTYPE", 3: "ALIGN", 4: "TIMEOUT", 5: "LAUNCH",
                6: "UNSUPPORTED", 7: "CUDA", 8: "WORKSPACE"}

_vp, _i64, _i32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_i64p = ctypes.POINTER(ctypes.c_int64)
_dblp = ctypes.POINTER(ctypes.c_double)

# name -> (restype, argtypes); keep in the order of include/flb_b200.h
PROTOTYPES = {
    "flb_last_error": (ctypes.c_char_p, []),
    "flb_version": (ctypes.c_char_p, []),
    "flb_launch_count": (ctypes.c_uint64, []),
    "flb_attn_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32,
                            _i32, _vp, _sz, _vp]),
    "flb_attn_fwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32, _i32]),
    "flb_attn_scores_ld": (_i64, [_i64]),
    "flb_attn_bwd":(_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                            _i64, _i64, _i64, _i64, _i32, _i32, _vp, _sz, _vp]),
    "flb_attn_bwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i32, _i32]),
    "flb_wf_gather": (_i32, [_vp, _i64p, _vp, _i64p, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _i64p,
                             _i64, _i64, _i64, _i32, _vp]),
    "flb_wf_index_copy": (_i32, [_vp, _i32, _i64p, _vp, _vp, _i32, _i64p, _vp, _i64, _i64, _i64,
                                 _i32, _vp]),
    "flb_block_grid_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "flb_block_grid_fwd": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
                                  _vp, _sz, _vp]),
    "flb_block_grid_fwd_ex": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
                                     _vp, _sz, _i32, _vp]),
    "flb_block_grid_status": (_i32, [_vp, _vp]),
    "flb_block_grid_fwd_drop_barrier_test": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                                    ctypes.c_float, _vp, _sz, _i64, _i64,
                                                    ctypes.c_uint32, _vp]),
    "flb_block_grid_saved_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "flb_block_grid_fwd_save": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                       ctypes.c_float, _vp, _sz, _vp, _sz, _vp]),
    "flb_block_grid_bwd_saved": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                        _i64, _i64, _i64, ctypes.c_float, _vp, _sz, _vp, _sz,
                                        _vp]),
    "flb_block_grid_bwd_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64]),
    "flb_block_grid_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                  _i64, _i64, ctypes.c_float, _vp, _sz, _vp]),
    "flb_grid_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64, _i32]),
    "flb_grid_fwd": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                            _vp, _sz, _i32, _vp]),
    "flb_grid_bwd": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                            _i64, _i64, _i64, _i64, _i64, _vp, _sz, _i32, _vp]),
    "flb_grid_fwd_drop_flag_test": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64,
                                           _i64, _i64, _i64, _vp, _sz, _i64, _i64, ctypes.c_uint32,
                                           _vp]),
    "flb_grid_fwd_static": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                   _vp]),
    "flb_grid_band_block_bytes": (_sz, [_i64, _i64, _i64]),
    "flb_ipc_alloc": (_i32, [_sz, ctypes.POINTER(ctypes.c_void_p), _vp]),
    "flb_ipc_open": (_i32, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "flb_ipc_close": (_i32, [_vp]),
    "flb_ipc_free": (_i32, [_vp]),
    "flb_grid_band_fwd": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                 _i64, _i64, _vp, _vp, _sz, _i32, _vp]),
    "flb_grid_band_bwd": (_i32, [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _sz, _i32,
                                 _vp]),
    "flb_microbench": (_i32, [_i32, _vp, _dblp]),
    "flb_selftest_umma": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp, _vp]),
}


class BlockWeights(ctypes.Structure):
    """flb_block_weights of include/flb_b200.h (device pointers, same field order)."""
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "ln_lat_w", "ln_lat_b", "ln_fdbk_w", "ln_fdbk_b", "w_prior_lat", "w_prior_fdbk",
        "w_gate_l", "b_gate_l", "w_gate_x", "b_gate_x", "w_qkv", "w_o", "v_a")]


IPC_HANDLE_BYTES = 80  # FLB_IPC_HANDLE_BYTES


class GridBand(ctypes.Structure):
    """flb_grid_band of include/flb_b200.h."""
    _fields_ = [("row0", ctypes.c_int64), ("rows_total", ctypes.c_int64),
                ("own_block", ctypes.c_void_p), ("up_block", ctypes.c_void_p),
                ("down_block", ctypes.c_void_p), ("epoch", ctypes.c_int)]


class BlockGrads(ctypes.Structure):
    """flb_block_grads of include/flb_b200.h (float32 device pointers, same field order)."""
    _fields_ = [(n, ctypes.c_void_p) for n, _ in BlockWeights._fields_]


for _name, (_res, _args) in PROTOTYPES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def launch_count() -> int:
    """Kernels launched by libflb_b200.so in this process so far."""
    return int(lib.flb_launch_count())


def version() -> str:
    return lib.flb_version().decode()


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib.flb_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed with FLB_ERR_{STATUS_NAMES.get(status, status)}: {msg}")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.float16:
        return F16
    if dt == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {dt}; expected float32, float16 or bfloat16")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def strides(*vals: int) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*vals)


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "flb-transformer_b200 runs on CUDA tensors only (sm_100a kernels; no CPU path); "
                f"got a tensor on {t.device}")


def workspace(nbytes: int, device: torch.device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def microbench(kind: int, device: torch.device | str = "cuda") -> float:
    """Measured throughput (elements/s) of one instruction class; see flb_microbench."""
    scratch = torch.empty(4 * 1024 * torch.cuda.get_device_properties(device).multi_processor_count,
                          dtype=torch.uint8, device=device)
    out = ctypes.c_double(0.0)
    check(lib.flb_microbench(kind, scratch.data_ptr(), ctypes.byref(out)), "flb_microbench")
    return out.value
