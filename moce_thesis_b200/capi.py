"""ctypes binding of the C ABI in ``include/moce_b200.h``.

This is the binding a non-torch caller (or a test that wants to exercise the
exact C entry points) uses: every function takes raw device pointers, sizes
and a stream handle.  ``lib()`` loads ``moce_thesis_b200/lib/libmoce_b200.so``
and raises if it is missing -- there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libmoce_b200.so")

MOCE_OK, MOCE_ERR_INVALID, MOCE_ERR_UNSUPPORTED, MOCE_ERR_CUDA, MOCE_ERR_WORKSPACE = range(5)
MOCE_F32, MOCE_BF16, MOCE_F16 = 0, 1, 2

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/moce_b200.h
SIGNATURES = {
    "moce_last_error": (ctypes.c_char_p, []),
    "moce_version": (ctypes.c_char_p, []),
    "moce_route_build": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p]),
    "moce_pool": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p]),
    "moce_schedule_steps": (_i32, [_i64]),
    "moce_schedule_build": (_i32, [_p, _i64, _i64, _i64, _i32, _p, _p, _p]),
    "moce_pool_residual": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _p]),
    "moce_mix_scheduled": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _i64, _i64, _p, _p, _p, _p, _f32, _f32,
                                  _p, _p, _p]),
    "moce_tc_stage_bytes": (_sz, [_i64, _i64, _i64]),
    "moce_tc_supported": (_i32, [_i32, _i64, _i64, _i64]),
    "moce_pool_stage": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _p, _p]),
    "moce_mix_tc": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _f32, _f32, _p, _p, _p]),
    "moce_mix_tc_t": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p]),
    "moce_temperature": (_i32, [_p, _i64, _i64, _p, _i64, _i64, _p, _p, _f32, _f32, _p, _p]),
    "moce_temperature_mlp": (_i32, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _f32, _f32, _p, _p, _p]),
    "moce_forward_tc_mlp": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _p, _p, _p, _p,
                                   _f32, _f32, _p, _p, _p, _p, _p, _p]),
    "moce_tc_fault": (_i32, [_p, _i32]),
    "moce_tc_wait_limit_ns": (_i64, [_i64]),
    "moce_tc_fault_info": (_i32, [_p, _i32, _i32]),
    "moce_forward_tc": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p, _f32, _f32, _p, _p, _p,
                                _p, _p]),
    "moce_forward_tc_ep": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _i64, _i64, _p, _p, _f32, _f32, _p, _p, _i32,
                                  _p, _p, _p, _p, _p]),
    "moce_px_supported": (_i32, [_i32, _i64, _i64, _i64]),
    "moce_mix_px": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _f32, _f32, _p, _p, _p]),
    "moce_mix_px_t": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p]),
    "moce_gx_supported": (_i32, [_i32, _i64, _i64, _i64]),
    "moce_mix_gx": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _f32, _f32, _p, _p, _p]),
    "moce_mix_gx_t": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p]),
    "moce_gate_temperature": (_i32, [_p, _i32, _p, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _f32, _f32,
                                     _p, _p, _p]),
    "moce_mix": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p, _p]),
    "moce_forward_dynamic_temp": (_i32, [_p, _i32, _p, _i32, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "moce_gate_route_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "moce_gate_route": (_i32, [_p, _i32, _p, _p, _i32, _p, _p, _p, _p, _f32, _f32, _f32, _p, _i64, _i64, _i64,
                               _i64, _i64, _p, _sz, _p]),
    "moce_noalloc_scratch_bytes": (_sz, []),
    "moce_gate_route_noalloc": (_i32, [_p, _i32, _p, _p, _i32, _p, _p, _p, _p, _f32, _f32, _f32, _p, _i64, _i64,
                                       _i64, _i64, _i64, _p]),
    "moce_backward_workspace_bytes": (_sz, [_i64, _i64, _i64, _i64, _i64]),
    "moce_backward": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p,
                             _f32, _f32, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "moce_aux_workspace_bytes": (_sz, [_i64, _i64]),
    "moce_aux_loss": (_i32, [_p, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _p, _p, _sz, _p]),
    "moce_aux_loss_backward": (_i32, [_p, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _p, _p, _p, _sz, _p]),
    "moce_bn_act": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i32, _p, _p]),
    "moce_backward_t": (_i32, [_p, _p, _i32, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _p, _p, _p,
                               _p, _p, _sz, _p]),
}

_lib = None


def lib():
    """Load the native library (once) and declare its signatures."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python -m moce_thesis_b200.build`")
        handle = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str = "moce") -> None:
    if rc != MOCE_OK:
        msg = lib().moce_last_error().decode(errors="replace")
        raise RuntimeError(f"{what}: status {rc}: {msg}")


def call(name: str, *args):
    """Call a status-returning entry point and raise on failure."""
    rc = getattr(lib(), name)(*args)
    check(rc, name)
    return rc


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def dtype_code(t) -> int:
    import torch
    return {torch.float32: MOCE_F32, torch.bfloat16: MOCE_BF16, torch.float16: MOCE_F16}[t.dtype]


def stream_handle(device=None) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream
