"""ctypes binding of libmoe_b200.so (the C ABI declared in include/moe_b200.h).

The library is loaded from this package directory.  There is no fallback: if the
shared library is missing or a call fails, a RuntimeError is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_NAME = "libmoe_b200.so"
LIB_PATH = os.environ.get("MOE_B200_LIB") or os.path.join(
    os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

MOE_F32, MOE_F16, MOE_BF16 = 0, 1, 2
_DTYPE_CODE = {torch.float32: MOE_F32, torch.float16: MOE_F16, torch.bfloat16: MOE_BF16}

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_ptr = ctypes.c_void_p
_c_size = ctypes.c_size_t

# name -> (restype, argtypes); must match include/moe_b200.h.
SIGNATURES = {
    "moe_version": (ctypes.c_char_p, []),
    "moe_last_error_string": (ctypes.c_char_p, []),
    "moe_read_device_error": (_c_int, [ctypes.POINTER(_c_int)]),
    "moe_peek_device_error": (_c_int, [_c_ptr, _c_ptr]),
    "moe_selftest_bounded_wait": (_c_int, [ctypes.c_uint64, _c_ptr, _c_ptr]),
    "moe_write_probe": (_c_int, [_c_ptr, ctypes.c_size_t, _c_ptr]),
    "moe_ipc_malloc": (_c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _c_ptr]),
    "moe_ipc_open": (_c_int, [_c_ptr, ctypes.POINTER(ctypes.c_void_p)]),
    "moe_ipc_close": (_c_int, [_c_ptr]),
    "moe_ipc_free": (_c_int, [_c_ptr]),
    "moe_ep_slot_map": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
                                 _c_i64, _c_ptr, _c_ptr, _c_ptr]),
    "moe_ep_dispatch": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64,
                                 _c_ptr, _c_ptr]),
    "moe_ep_combine": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_ptr, _c_ptr, _c_int, _c_i64, _c_i32,
                                _c_i64, _c_ptr, _c_ptr, _c_ptr]),
    "moe_ep_combine_bwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_int, _c_ptr, _c_ptr, _c_ptr, _c_int,
                                    _c_i64, _c_i32, _c_i64, _c_ptr, _c_ptr, _c_ptr]),
    "moe_add_rows": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_int, _c_ptr]),
    "moe_ep_barrier": (_c_int, [_c_ptr, _c_i32, _c_i32, _c_ptr, ctypes.c_uint64, _c_ptr, _c_ptr]),
    "moe_ep_put_counts": (_c_int, [_c_ptr, _c_i32, _c_ptr, _c_i32, _c_i32, _c_ptr]),
    "moe_topk_softmax_fwd": (_c_int, [_c_ptr, _c_int, _c_i64, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_ptr]),
    "moe_topk_softmax_bwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_int, _c_i64, _c_i32, _c_i32, _c_ptr, _c_ptr]),
    "moe_permute_workspace_bytes": (_c_size, [_c_i64, _c_i32, _c_i32]),
    "moe_permute": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_i64, _c_i32, _c_i64, _c_i32, _c_i64,
                             _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr]),
    "moe_permute_capacity": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_i64, _c_i32, _c_i64, _c_i32,
                                      _c_i32, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_size,
                                      _c_ptr]),
    "moe_permute_index": (_c_int, [_c_ptr, _c_i64, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                   _c_size, _c_ptr]),
    "moe_gmm_fwd_gather": (_c_int, [_c_ptr, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i64,
                                    _c_i64, _c_i64, _c_i32, _c_int, _c_int, _c_ptr]),
    "moe_gmm_gate_up_fwd_gather": (_c_int, [_c_ptr, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                            _c_ptr, _c_ptr, _c_i32, _c_i64, _c_i64, _c_i64, _c_i32,
                                            _c_int, _c_int, _c_ptr]),
    "moe_gmm_wgrad_gather": (_c_int, [_c_ptr, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i64,
                                      _c_i64, _c_i64, _c_i32, _c_int, _c_int, _c_ptr]),
    "moe_permute_noalloc": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_i64, _c_i32, _c_i64, _c_i32,
                                     _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr]),
    "moe_permute_noalloc_max_slots": (_c_size, [_c_i32]),
    "moe_swiglu_fwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_int, _c_ptr]),
    "moe_swiglu_bwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_int, _c_ptr]),
    "moe_scatter_rows": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_i64, _c_i32, _c_i64, _c_ptr, _c_ptr]),
    "moe_unpermute_fwd": (_c_int, [_c_ptr, _c_int, _c_ptr, _c_ptr, _c_int, _c_i64, _c_i32, _c_i64,
                                   _c_ptr, _c_ptr]),
    "moe_unpermute_bwd": (_c_int, [_c_ptr, _c_ptr, _c_int, _c_ptr, _c_ptr, _c_int, _c_i64, _c_i32,
                                   _c_i64, _c_ptr, _c_ptr, _c_ptr]),
    "moe_gmm_fwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i64, _c_i64, _c_i64, _c_i32,
                             _c_int, _c_int, _c_ptr]),
    "moe_gmm_gate_up_fwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i32,
                                     _c_i64, _c_i64, _c_i64, _c_i32, _c_int, _c_int, _c_ptr]),
    "moe_gmm_dgrad_swiglu_bwd": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
                                          _c_i32, _c_i64, _c_i64, _c_i64, _c_i32, _c_int, _c_int,
                                          _c_ptr]),
    "moe_gmm_dgrad": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i64, _c_i64, _c_i64, _c_i32,
                               _c_int, _c_int, _c_ptr]),
    "moe_gmm_dgrad_dual": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i64,
                                    _c_i64, _c_i64, _c_i64, _c_i32, _c_int, _c_int, _c_ptr]),
    "moe_gmm_wgrad": (_c_int, [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i64, _c_i64, _c_i64, _c_i32,
                               _c_int, _c_int, _c_ptr]),
}

_lib = None
_lock = threading.Lock()

# Instrumentation used by bench.py: number of library kernels launched so far, and an
# optional list that collects (name, start_event, end_event, flops) around every grouped
# GEMM call (CUDA events on the launching stream).
launch_count = 0
gemm_timing: list | None = None


def count_launches(n: int) -> None:
    global launch_count
    launch_count += n


def load() -> ctypes.CDLL:
    """Loads the shared library once; raises RuntimeError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_NAME} is not built ({LIB_PATH} missing); run "
                    "`python -m moe_ops_b200.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().moe_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {status}): {msg}")


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "moe_ops_b200 runs on CUDA tensors only (sm_100a kernels); got a tensor on "
                f"{t.device}")


def read_device_error() -> int:
    """Reads and clears the library's device-side error word (synchronises)."""
    code = _c_int(0)
    check(load().moe_read_device_error(ctypes.byref(code)), "moe_read_device_error")
    return code.value
