"""ctypes binding of the in-tree C-ABI library ``_lib/libsm100_marlin.so``.

The library is the only compute path: if it is missing or cannot be loaded
every operator raises (there is no CPU or PyTorch fallback).
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsm100_marlin.so")

_lock = threading.Lock()
_lib = None

_c_int = ctypes.c_int
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_size = ctypes.c_size_t

# name -> (restype, argtypes); every name is declared in include/sm100_marlin.h
SIGNATURES = {
    "sm100_marlin_mul_2_4": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _c_int,
                                      _c_int, _vp, _c_int, _c_int, _c_int, _c_int]),
    "sm100_marlin_mul_2_4_meta3": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp,
                                            _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _c_int]),
    "sm100_marlin_mul_2_4_ex": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp,
                                         _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _c_int,
                                         _c_int, _vp, _size]),
    "sm100_marlin_mul_2_4_epilogue": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp,
                                               _c_int, _c_int, _vp, _c_int, _c_int, _c_int, _c_int,
                                               _c_int, _vp, _c_int]),
    "sm100_marlin_mul_2_4_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                              _vp, _c_int, _c_int, _vp, _c_int, _c_int, _c_int,
                                              _c_int]),
    "sm100_marlin_mul_2_4_meta_diag": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                                _vp, _c_int, _c_int, _vp, _c_int]),
    "sm100_marlin_scratch_bytes": (_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "sm100_marlin_meta3_pack": (_c_int, [_vp, _vp, _i64, _vp, _vp]),
    "sm100_marlin_meta3_unpack": (_c_int, [_vp, _vp, _i64, _vp]),
    "sm100_marlin_meta3_decode_words": (_c_int, [_vp, _vp, _vp, _i64, _vp]),
    "sm100_marlin_device_status": (_c_int, [_c_int, ctypes.POINTER(_c_int)]),
    "sm100_marlin_error_string": (ctypes.c_char_p, [_c_int]),
    "sm100_marlin_last_cuda_error": (ctypes.c_char_p, []),
    "sm100_marlin_set_trace_buffer": (_c_int, [_vp]),
    "sm100_marlin_set_overlap": (_c_int, [_c_int]),
    "sm100_marlin_set_decode_kernel": (_c_int, [_c_int]),
    "sm100_marlin_pack_2_4": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _vp, _vp, _vp, _c_int,
                                       _vp]),
    "sm100_marlin_mul_2_4_gather": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _vp,
                                             _c_int, _c_int, _vp, _c_int, _vp, _vp, _vp, _vp, _vp,
                                             _vp, _c_int, _c_int, _c_int]),
    "sm100_marlin_gather_wait": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _vp]),
    "sm100_marlin_ipc_alloc": (_c_int, [_size, _c_int, ctypes.POINTER(_vp)]),
    "sm100_marlin_ipc_free": (_c_int, [_vp, _c_int]),
    "sm100_marlin_ipc_get_handle": (_c_int, [_vp, _c_int, _vp]),
    "sm100_marlin_ipc_open": (_c_int, [_vp, _c_int, ctypes.POINTER(_vp)]),
    "sm100_marlin_ipc_close": (_c_int, [_vp, _c_int]),
}

OK = 0
ERR_PROB_SHAPE = 1
ERR_KERN_SHAPE = 2
ERR_CUDA = 3
ERR_ALIGNMENT = 4
ERR_ARGUMENT = 5
ERR_SCRATCH = 6

DECODE_AUTO = 0
DECODE_STREAM_K = 1
DECODE_TMEM = 2


_fast = None
_fast_tried = False


def fast():
    """The CPython binding of the GEMM entry points (``_fastcall``, built by
    ``build.build_fastcall``), or None when it has not been built: callers
    then use the ctypes table, which reaches the same C ABI."""
    global _fast, _fast_tried
    if not _fast_tried:
        _fast_tried = True
        load()  # the binding links the library: make sure it is present first
        try:
            from . import _fastcall
            _fast = _fastcall
        except ImportError:
            _fast = None
    return _fast


def load(path: str = LIB_PATH):
    """Load (once) and return the library; raise if it is not built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"sm_100a library not built ({path} missing); run `python -m csed499ii_b200.build`"
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def describe(code: int) -> str:
    lib = load()
    msg = lib.sm100_marlin_error_string(code).decode()
    if code == ERR_CUDA:
        msg += ": " + lib.sm100_marlin_last_cuda_error().decode()
    return msg


def device_status(dev: int) -> int:
    """Read and clear the device status word (bounded-wait timeouts)."""
    lib = load()
    out = ctypes.c_int(0)
    rc = lib.sm100_marlin_device_status(dev, ctypes.byref(out))
    if rc != OK:
        raise RuntimeError(f"sm100_marlin_device_status failed: {describe(rc)}")
    return out.value
