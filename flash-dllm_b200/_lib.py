"""ctypes binding of ``libflashdllm_b200.so`` (declared in ``include/flashdllm_b200.h``).

The library is the only compute path: importing this module raises if the
shared object is missing or fails to load -- there is no CPU or PyTorch
fallback.  ``call(name, *args)`` invokes an entry point and raises
:class:`FdllmError` on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libflashdllm_b200.so")

_p = C.c_void_p
_i32 = C.c_int32
_i64 = C.c_int64
_f32 = C.c_float
_f64 = C.c_double
_sz = C.c_size_t
_int = C.c_int

# name -> (restype, argtypes); mirrors include/flashdllm_b200.h
SIGNATURES = {
    "fdllm_version": (C.c_char_p, []),
    "fdllm_error_string": (C.c_char_p, [_int]),
    "fdllm_status_read": (_int, [_p, _p]),
    "fdllm_rmsnorm": (_int, [_p, _p, _p, _i32, _i32, _f32, _p]),
    "fdllm_add_rmsnorm": (_int, [_p, _p, _p, _p, _p, _i32, _i32, _f32, _p]),
    "fdllm_swiglu": (_int, [_p, _p, _p, _i64, _i32, _i64, _p]),
    "fdllm_qkv_set_plan": (_int, [_i32, _i32, _i32, _i32, _i32]),
    "fdllm_gemm_set_plan": (_int, [_i32, _i32, _i32, _i32, _i32]),
    "fdllm_gemm_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32]),
    "fdllm_gemm_bf16": (_int, [_p, _p, _p, _p, _i32, _i32, _i32, _i64, _i64, _p, _sz, _p]),
    "fdllm_gemm_swiglu": (_int, [_p, _p, _p, _i32, _i32, _i32, _i64, _p, _sz, _p]),
    "fdllm_qkv_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "fdllm_qkv_rope_cache": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i64, _p, _sz, _p]),
    "fdllm_qkv_rope_cache_noalloc": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i64, _p]),
    "fdllm_verify_qkv": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i32, _i32, _i32, _i64, _p, _sz, _p]),
    "fdllm_attn_plan_capacity": (_int, [_i32, _i32]),
    "fdllm_attn_plan_bytes": (_sz, [_i32, _i32]),
    "fdllm_plan_cache_attention": (_int, [_p, _i32, _p, _i32, _i32, _i32, _i32, _i32, _p, _sz, _p]),
    "fdllm_attn_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "fdllm_attn_cache": (_int, [_p, _p, _p, _p, _p, _i32, _p, _f32, _i32, _i32, _i32, _i64, _f32, _i32, _p, _i32,
                                _p, _sz, _p]),
    "fdllm_verify_attn": (_int, [_p, _p, _p, _p, _p, _p, _p, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _i64,
                                 _f32, _i32, _p, _sz, _p]),
    "fdllm_row_stats": (_int, [_p, _i64, _i32, _i32, _p, _p, _p, _p, _p]),
    "fdllm_window_accept": (_int, [_p, _p, _p, _p, _p, _i32, _i64, _i64, _f64, _i32, _i64, _p, _p, _p, _p, _p, _p,
                                   _p]),
    "fdllm_verify_accept": (_int, [_p, _p, _p, _p, _p, _i32, _i64, _f64, _i64, _p, _p, _p, _p]),
    "fdllm_cache_build": (_int, [_p, _i32, _i32, _i64, _i64, _p, _p, _p, _p, _p, _p, _p]),
    "fdllm_verify_build": (_int, [_p, _i32, _i32, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p]),
    "fdllm_refresh_sort": (_int, [_p, _i32, _i64, _p, _p, _i64, _p]),
}


class FdllmError(RuntimeError):
    def __init__(self, name: str, code: int, info=None):
        msg = _LIB.fdllm_error_string(code).decode()
        super().__init__(f"{name} failed: {msg} (status {code}{'' if info is None else f', info {info}'})")
        self.code = code
        self.info = info


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m flash_dllm_b200.build` "
            "(there is no fallback path)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = _load()


def lib():
    return _LIB


def call(name: str, *args) -> None:
    rc = getattr(_LIB, name)(*args)
    if rc != 0:
        raise FdllmError(name, rc)


def ptr(t) -> int:
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_ERROR_HOOKS = []


def on_device_error(fn) -> None:
    """Register ``fn()`` to run when :func:`check_device_status` finds an
    error (before it raises): the workspace owner re-zeroes its buffers."""
    _ERROR_HOOKS.append(fn)


def check_device_status(stream=None) -> None:
    """Synchronise and raise if any kernel recorded a device-side error.

    A kernel that stopped on an error can leave split-K counters or CTA-pair
    handoff flags set in its workspace; the registered hooks zero the
    workspaces in place (same addresses, so captured CUDA graphs stay valid)
    before the error is raised, so a caller that catches it can go on."""
    out = (C.c_int32 * 4)()
    s = stream if stream is not None else stream_handle()
    call("fdllm_status_read", C.cast(out, C.c_void_p), s)
    if out[0] != 0:
        for fn in _ERROR_HOOKS:
            fn()
        torch.cuda.synchronize()
        raise FdllmError(f"device kernel {out[2]}", out[0], out[1])
