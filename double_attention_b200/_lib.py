"""ctypes binding of the C ABI in ``include/da_b200.h``.

The shared library ``libda_b200.so`` is built in-tree by
``double_attention_b200.build``.  There is no fallback: when the library is
missing or fails to load, :func:`lib` raises, so no caller can silently run
another implementation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libda_b200.so"

DA_OK = 0
DA_ERR_NULL = 1
DA_ERR_SHAPE = 2
DA_ERR_DTYPE = 3
DA_ERR_ALIGN = 4
DA_ERR_UNSUPPORTED = 5
DA_ERR_DEVICE_TIMEOUT = 6
DA_ERR_CUDA = 7
DA_ERR_WORKSPACE = 8

DA_F16 = 0
DA_BF16 = 1
DA_F32 = 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> argument types; every entry point returns int.
SIGNATURES: dict[str, list] = {
    "da_dict_norm_fwd": [_p, _i64, _i64, _f32, _i32, _p, _p, _p, _p, _p],
    "da_dict_norm_pair_fwd": [_p, _p, _i32, _i64, _i64, _f32, _i32, _p, _p, _p, _p, _p, _p, _p, _p],
    "da_temperatures": [_p, _i32, _f32, _f32, _p, _i32, _i32, _f32, _f32, _p, _p, _p],
    "da_gemm_segments": [_p, _i64, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _p, _p, _p, _p, _p],
    "da_dict_norm_bwd": [_p, _p, _p, _p, _i64, _i64, _f32, _p, _i32, _p],
    "da_dict_norm_bwd_typed": [_p, _i32, _p, _p, _p, _i64, _i64, _f32, _p, _i32, _i32, _p],
    "da_temperatures_bwd": [_p, _i32, _f32, _f32, _p, _p, _p, _p, _i32, _i32, _f32, _f32, _p, _p, _p, _p],
    "da_col_norm_max": [_p, _i64, _i64, _i32, _p, _p],
    "da_set_debug_trace": [_p],
    "da_route_fwd_static": [_p, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _f32, _i32, _i32,
                            _p, _p, _p, _p, _p, _p],
    "da_gemm": [_p, _i64, _i32, _p, _i64, _i32, _p, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _p, _p],
    "da_attn_fwd": [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _i32, _i32, _i32, _i32, _i32, _i32,
                    _p, _i32, _i32, _p, _p, _p, _f32, _p, _p, _p, _p],
    "da_attn_fwd_workspace_size": [_i32, _i32, _i32, _i32],  # returns int64 (set below)
    "da_attn_fwd_ws": [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _i32, _i32, _i32, _i32, _i32, _i32,
                       _p, _i32, _i32, _p, _p, _p, _f32, _p, _p, _p, _i64, _p, _p],
    "da_attn_bwd_delta": [_p, _p, _i64, _i32, _i32, _p, _p],
    "da_gemm_ex": [_p, _i64, _p, _i64, _i32, _i64, _p, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i32, _p, _i32,
                   _p, _i64, _p, _p],
    "da_gemm_splitk_workspace_elems": [_i64, _i64, _i64, _i32],  # returns int64 (set below)
    "da_col_sum_workspace_elems": [_i64, _i64],  # returns int64 (set below)
    "da_col_sum": [_p, _i64, _i64, _i64, _i32, _p, _p, _i64, _p],
    "da_gemm_splitk": [_p, _i64, _i32, _p, _i64, _i32, _p, _i64, _i64, _i64, _i64, _i32, _i32, _p, _i64, _p, _p],
    "da_gemm_splitk_store": [_p, _i64, _i32, _p, _i64, _i32, _p, _i64, _i32, _i64, _i64, _i64, _i32, _i32, _p, _i64,
                             _p, _p],
    "da_gemm_splitk_grouped": [_p, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _p, _i64, _p,
                               _p],
    "da_route_bwd": [_p, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i32, _p, _p, _p, _f32, _i32, _i32, _p, _p, _p,
                     _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p],
    "da_route_bwd_workspace_size": [_i64, _i32, _i64, _i64],  # returns int64 (set below)
    "da_route_bwd_fused": [_p, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i32, _p, _p, _p, _f32, _i32, _i32, _p,
                           _p, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _p],
    "da_attn_bwd_workspace_size": [_i32, _i32, _i32],  # returns int64 (set below)
    "da_attn_bwd_split_workspace_size": [_i32, _i32, _i32, _i32, _i32, _i32],  # returns int64 (set below)
    "da_attn_bwd_mixed": [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32,
                          _i32, _i32, _p, _i32, _i32, _p, _p, _p, _p, _i32, _p, _p, _p, _p, _p, _p, _i64, _p, _p],
    "da_attn_bwd_mixed_ow": [_p, _i64, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32,
                          _i32, _i32, _p, _i32, _i32, _p, _p, _p, _p, _i32, _p, _p, _p, _p, _p, _p, _i64, _p, _p],
    "da_selftest_mma": [_i32, _i32, _i32, _i32, _p, _p, _p, _p, _p],
    "da_selftest_wait_timeout": [_i64, _i32, _p, _p, _p],
    "da_route_var_weights": [_p, _i64, _i32, _p, _i64, _i32, _i32, _i32, _f32, _f32, _p, _f32, _p, _p, _p],
    "da_route_var_output": [_p, _i64, _i32, _i32, _i32, _f32, _p, _p, _p],
    "da_route_var_output_bwd": [_p, _p, _p, _i64, _i32, _i32, _i32, _f32, _p, _p, _p],
    "da_route_var_weights_bwd": [_p, _p, _i64, _i32, _p, _p, _i32, _f32, _f32, _p, _i32, _p, _p, _p, _p, _i64, _p],
    "da_route_var_input_bwd": [_p, _p, _i64, _p, _i64, _i32, _i32, _i32, _f32, _p, _i64, _p],
    "da_route_fwd": [_p, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i32, _p, _p, _p, _p, _f32, _i32, _i32,
                     _p, _p, _p, _p, _p, _i32, _p, _p],
    "da_add_layernorm_fwd": [_p, _p, _i32, _p, _p, _i64, _i64, _f32, _p, _p, _i32, _p, _p, _p],
    "da_add_layernorm_bwd": [_p, _i32, _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _i32, _p, _i32, _p, _p, _p],
    "da_layernorm_bwd_blocks": [_i64],
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class DAError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, name: str, status: int, detail: str) -> None:
        super().__init__(f"{name} failed with status {status}: {detail}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m double_attention_b200.build` "
                    "(the B200 kernels have no fallback implementation)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int
            handle.da_status_string.argtypes = [ctypes.c_int]
            handle.da_status_string.restype = ctypes.c_char_p
            handle.da_version.argtypes = []
            handle.da_version.restype = ctypes.c_char_p
            handle.da_last_cuda_error.argtypes = []
            handle.da_last_cuda_error.restype = ctypes.c_int
            handle.da_route_bwd_workspace_size.argtypes = [_i64, _i32, _i64, _i64]
            handle.da_route_bwd_workspace_size.restype = ctypes.c_int64
            handle.da_attn_bwd_workspace_size.restype = ctypes.c_int64
            handle.da_attn_bwd_split_workspace_size.restype = ctypes.c_int64
            handle.da_attn_fwd_workspace_size.restype = ctypes.c_int64
            handle.da_gemm_splitk_workspace_elems.restype = ctypes.c_int64
            handle.da_col_sum_workspace_elems.restype = ctypes.c_int64
            handle.da_kernel_launches.argtypes = []
            handle.da_kernel_launches.restype = ctypes.c_uint64
            _lib = handle
    return _lib


def check(name: str, status: int) -> None:
    """Map a status code to an exception (NotImplementedError for variants)."""
    if status == DA_OK:
        return
    handle = lib()
    detail = handle.da_status_string(status).decode()
    if status == DA_ERR_CUDA:
        detail += f" (cuda error {handle.da_last_cuda_error()})"
    if status == DA_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{name}: {detail}")
    if status in (DA_ERR_SHAPE, DA_ERR_DTYPE, DA_ERR_ALIGN, DA_ERR_NULL):
        raise ValueError(f"{name}: {detail}")
    raise DAError(name, status, detail)


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))


def kernel_launches() -> int:
    """Kernels launched by the library so far in this process."""
    return int(lib().da_kernel_launches())


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device | None = None) -> int:
    """Raw handle of the current CUDA stream of `device` (the current device if None)."""
    idx = device.index if device is not None else None
    if idx is None:
        idx = torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(idx)


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return DA_F16
    if dtype == torch.bfloat16:
        return DA_BF16
    if dtype == torch.float32:
        return DA_F32
    raise ValueError(f"unsupported dtype {dtype}")
