"""ctypes binding of libsa_b200.so (the C ABI in include/streaming_attention.h).

The library is loaded from this package directory.  There is no fallback: if
the library is missing or fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
# SA_DEVICE_CHECKS=1 loads the build with device-side index checks instead
CHECKS = os.environ.get("SA_DEVICE_CHECKS", "0") == "1"
LIB_PATH = os.path.join(_PKG, "libsa_b200_checks.so" if CHECKS else "libsa_b200.so")

SA_OK = 0
SA_ERR_INVALID_ARG = -1
SA_ERR_UNSUPPORTED = -2
SA_ERR_CUDA = -3
SA_ERR_TIMEOUT = -4
SA_ERR_WORKSPACE = -5
SA_ERR_DEVICE_CHECK = -6

COMPRESSORS = {"none": 0, "sorted_pair": 1, "random": 2}
# storage dtype of the segment-mean reps (SA_REP_*)
REP_DTYPES = {"float32": 0, "float16": 1, "bfloat16": 2}
MAX_DEGREE = 3

_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t

# name -> argtypes; every function returns int status
SIGNATURES = {
    "sa_version": [],
    "sa_workspace_status": [_vp, _vp],
    "sa_device_checks_enabled": [],
    "sa_set_moment_fork": [_i32],
    "sa_moment_fork_enabled": [],
    "sa_set_wait_limit_ns": [ctypes.c_uint64],
    "sa_set_stage_events": [ctypes.POINTER(_vp), _i32],
    "sa_feature_count": [_i32, _i32, ctypes.POINTER(_i64)],
    "sa_block_counts": [_i64, _i32, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    "sa_compress_blocks": [_vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "sa_low_moments_workspace_size": [_i64, _i64, _i32, _i32, _i32, _i32, ctypes.POINTER(_sz)],
    "sa_low_moments": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _sz, _vp],
    "sa_residual_combine_workspace_size": [_i64, _i64, _i32, _i32, _i32, _i32, ctypes.POINTER(_sz)],
    "sa_residual_combine": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _f32,
                            _f32, _vp, _vp, _sz, _vp],
    "sa_fast_attention_workspace_size": [_i64, _i64, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_sz)],
    "sa_fast_attention": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _vp, _vp, _f32, _vp,
                          _vp, _vp, _sz, _vp],
    "sa_fast_attention_static_scratch": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _vp,
                                         _vp, _f32, _vp, _vp, _vp],
    "sa_shard_state_floats": [_i64, _i32, _i32, _i32, ctypes.POINTER(_i64)],
    "sa_shard_workspace_size": [_i64, _i64, _i32, _i32, _i32, _i32, _i64, ctypes.POINTER(_sz)],
    "sa_shard_begin": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _vp, _vp, _i64, _i64,
                       _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    "sa_shard_end": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _f32, _vp, _i32, _i64, _vp, _vp,
                     _vp, _i64, _vp, _vp, _sz, _vp],
    "sa_stream_update": [_vp, _vp, _i32, _i32, _i32, _f32, _vp, _vp, _vp],
    "sa_stream_compress": [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "sa_stream_query_workspace_size": [_i32, _i32, _i32, ctypes.POINTER(_sz)],
    "sa_segment_mean_reps": [_vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp],
    "sa_article_segment_mean_workspace_size": [_i64, _i64, _i32, _i32, _i32, _i32, _i32, ctypes.POINTER(_sz)],
    "sa_flash_causal_attention_workspace_size": [_i64, _i64, _i32, _i32, ctypes.POINTER(_sz)],
    "sa_flash_causal_attention": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _f32, _vp, _vp, _sz, _vp],
    "sa_article_segment_mean": [_vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _f32,
                                _vp, _vp, _sz, _vp],
    "sa_stream_query": [_vp, _i32, _i32, _i32, _f32, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _f32, _vp, _vp,
                        _vp, _sz, _vp],
}

_lock = threading.Lock()
_lib = None


class SAError(RuntimeError):
    """A CUDA-side failure reported by libsa_b200.so."""


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m streaming_attention_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_int
            lib.sa_last_error.argtypes = []
            lib.sa_last_error.restype = ctypes.c_char_p
            _lib = lib
    return _lib


def last_error() -> str:
    return load().sa_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Map a status code to the exception the reference raises for it."""
    if rc == SA_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == SA_ERR_INVALID_ARG or rc == SA_ERR_WORKSPACE:
        raise ValueError(msg)
    if rc == SA_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise SAError(f"{msg} (status {rc})")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
