"""Loader of libferryb.so (the C ABI declared in include/ferryb.h).

The library is built in-tree (ferry_b200/libferryb.so, see build.py).  There
is no fallback: if it is missing or a call fails, a RuntimeError is raised,
as the reference's TORCH_CHECKs raise RuntimeError into Python
(ferry/csrc/expert_ops.cpp:20-34).
"""
import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / 'libferryb.so'

_i64, _i32, _vp, _u64 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64
_dbl, _f32 = ctypes.c_double, ctypes.c_float

# name -> (restype, argtypes); every symbol declared in include/ferryb.h.
SIGNATURES = {
    'ferryb_last_error': (ctypes.c_char_p, []),
    'ferryb_version': (_i32, []),
    'ferryb_device_sm_count': (_i32, [_i32]),
    'ferryb_execute_experts_workspace': (_i64, [_i64, _i64, _i64, _i64]),
    'ferryb_execute_experts': (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp,
                                      _i64, _i64, _vp, _vp, _i64, _vp]),
}

_lib = None


class FerrybError(RuntimeError):
    pass


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FerrybError(f'{LIB_PATH} is missing: build it with `python -m ferry_b200.build`')
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def call(name, *args):
    status = getattr(lib(), name)(*args)
    if status != 0:
        msg = lib().ferryb_last_error().decode(errors='replace')
        raise FerrybError(f'{name} failed (status {status}): {msg}')
    return status


def ptr(t):
    """Device/host address of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise FerrybError('expected CUDA tensors (this path has no CPU fallback)')


def host_i64(values):
    arr = (ctypes.c_int64 * max(1, len(values)))(*[int(v) for v in values])
    return arr
