"""ctypes binding of libdcr_b200.so (the C ABI declared in include/dcr_b200.h).

The library is loaded from ``dcr_b200/lib/libdcr_b200.so`` (built in-tree by
``dcr_b200.build``). There is no fallback: if the library is missing, or CUDA is not
available, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

from dcr_b200.build import LIB_PATH

DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}

# dcr_status codes (include/dcr_b200.h)
DCR_OK = 0
DCR_ERR_NULL = 1
DCR_ERR_SHAPE = 2
DCR_ERR_K_RANGE = 3
DCR_ERR_DTYPE = 4
DCR_ERR_ALIGN = 5
DCR_ERR_WORKSPACE = 6
DCR_ERR_CUDA = 7
DCR_ERR_DEVICE_TIMEOUT = 8
DCR_ERR_NOALLOC_LIMIT = 9
DCR_ERR_DEVICE_INDEX = 16
DCR_ERR_DEVICE_SHARD = 32
IPC_HANDLE_BYTES = 64
PROJ_RANK = 16

# Every exported symbol with its (restype, argtypes); tests check this list against the
# header and the library's dynamic symbol table.
_vp, _i32, _i64, _f32, _f64, _sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64,
                                     ctypes.c_float, ctypes.c_double, ctypes.c_size_t)
SIGNATURES = {
    "dcr_version": (_i32, []),
    "dcr_status_string": (ctypes.c_char_p, [_i32]),
    "dcr_adaptive_k_window": (_i32, [_i32, _i32, _f64]),
    "dcr_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "dcr_unit_query": (_i32, [_vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp]),
    "dcr_score": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _f32, _i32, _i32, _i32, _i32, _i32,
                         _vp, _i64, _vp]),
    "dcr_select": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp]),
    "dcr_select_workspace_bytes": (_sz, [_i32, _i32]),
    "dcr_select_ws": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _sz, _vp]),
    "dcr_attend": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _vp, _i32, _i32, _i32,
                          _i32, _i32, _i32, _vp, _vp, _sz, _vp]),
    "dcr_select_indices": (_i32, [_vp, _vp, _i32, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
                                  _i32, _f32, _vp, _vp, _sz, _vp]),
    "dcr_decode": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _i32,
                          _i32, _i32, _f32, _vp, _vp, _sz, _vp]),
    "dcr_decode_noalloc": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _i32,
                                  _i32, _i32, _i32, _i32, _f32, _vp, _vp]),
    "dcr_decode_timed": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
                                _i32, _i32, _i32, _f32, _vp, _vp, _sz, _vp,
                                ctypes.POINTER(_vp)]),
    "dcr_decode_prefix": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
                                 _i32, _i32, _i32, _f32, _vp, _vp, _sz, _vp, _i32]),
    "dcr_project_keys": (_i32, [_vp, _i32, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _vp,
                                _i64, _i64, _vp]),
    "dcr_cache_append": (_i32, [_vp, _vp, _i32, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _vp,
                                _i64, _i64, _i32, _i32, _vp, _i32, _vp, _i64, _i64, _vp]),
    "dcr_score_projected": (_i32, [_vp, _i32, _i64, _i64, _vp, _f32, _vp, _i32, _vp, _i32,
                                   _i32, _i32, _i32, _i32, _vp, _i64, _vp]),
    "dcr_select_indices_projected": (_i32, [_vp, _vp, _i32, _i64, _i64, _vp, _i32, _vp, _i32,
                                            _i32, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _sz,
                                            _vp]),
    "dcr_decode_projected": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                                    _f32, _vp, _vp, _sz, _vp]),
    "dcr_decode_prologue": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp,
                                   _vp, _vp, _i64, _i64, _i32, _i32, _vp, _i32, _vp, _i64, _i64,
                                   _vp, _f32, _vp]),
    "dcr_decode_prologue_strided": (_i32, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _i32, _i32, _i32,
                                           _i32, _i32, _vp, _vp, _vp, _i64, _i64, _i32, _i32,
                                           _vp, _i32, _vp, _i64, _i64, _vp, _f32, _vp]),
    "dcr_runner_create": (_i32, [_vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _i32, _i32, _i32, _i32, _i32, _i32, _f32, _vp]),
    "dcr_runner_step": (_i32, [_vp, _vp, _vp]),
    "dcr_runner_query_buffer": (_vp, [_vp]),
    "dcr_runner_output_buffer": (_vp, [_vp]),
    "dcr_runner_destroy": (_i32, [_vp]),
    "dcr_add_rmsnorm": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _vp]),
    "dcr_silu_mul": (_i32, [_vp, _vp, _i32, _i64, _vp, _vp]),
    "dcr_silu_mul_packed": (_i32, [_vp, _i32, _i32, _i32, _vp, _vp]),
    "dcr_shard_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "dcr_shard_score": (_i32, [_vp, _vp, _i32, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32,
                               _f32, _vp, _vp, _sz, _vp]),
    "dcr_shard_refine": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _sz, _vp]),
    "dcr_shard_attend": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
                                _i32, _i32, _i32, _vp, _i32, _i32, _vp, _vp, _sz, _vp]),
    "dcr_shard_combine": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "dcr_shard_selection": (_i32, [_vp, _sz, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp,
                                   _vp]),
    "dcr_xchg_bytes": (_sz, [_i32, _i32, _i32]),
    "dcr_xchg_create": (_i32, [_i32, _i32, _i32, ctypes.POINTER(_vp), _vp]),
    "dcr_xchg_open": (_i32, [_vp, _i32, _i32, _vp, ctypes.POINTER(_vp)]),
    "dcr_xchg_close": (_i32, [ctypes.POINTER(_vp), _i32, _i32]),
    "dcr_xchg_destroy": (_i32, [_vp]),
    "dcr_xchg_reset": (_i32, [_vp, _i32, _i32, _i32, _vp]),
    "dcr_shard_decode_peer": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32, _i32,
                                     _i32, _i32, _i32, _i32, _f32, ctypes.POINTER(_vp), _i32,
                                     _i32, _i32, _vp, _vp, _sz, _vp]),
    "dcr_shard_decode_peer_timed": (_i32, [_vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _i32,
                                           _i32, _i32, _i32, _i32, _i32, _f32,
                                           ctypes.POINTER(_vp), _i32, _i32, _i32, _vp, _vp, _sz,
                                           _vp, ctypes.POINTER(_vp)]),
    "dcr_read_device_status": (_i32, [ctypes.POINTER(_i32), _i32]),
    "dcr_binary_version": (_i32, [ctypes.POINTER(_i32)]),
}

_lib = None


class DCRError(RuntimeError):
    """A libdcr_b200 entry point returned a non-zero dcr_status."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: dcr_status {status} ({status_string(status)})")


def load() -> ctypes.CDLL:
    """Load libdcr_b200.so once; raise loudly if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libdcr_b200.so not found at {LIB_PATH}; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'` (or python -m "
                "dcr_b200.build). There is no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().dcr_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != DCR_OK:
        raise DCRError(status, where)


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("libdcr_b200 requires CUDA tensors (no CPU fallback).")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def read_device_status(clear: bool = True) -> int:
    """Synchronise and return the sticky device status bits (DCR_ERR_DEVICE_*)."""
    v = ctypes.c_int(0)
    check(load().dcr_read_device_status(ctypes.byref(v), 1 if clear else 0),
          "dcr_read_device_status")
    return v.value
