"""The C ABI library loads and exports every entry point the header declares.

Runs on CPU: only host-side functions (counts, workspace sizing) and argument
checks that return before any CUDA call are exercised here.
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from streaming_attention_b200 import _lib

HEADER = os.path.join(ROOT, "include", "streaming_attention.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(sa_\w+)\s*\(", text, flags=re.M)))


def test_library_builds_and_exports_every_declared_symbol():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 9
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in the header but not exported"
    # every declared function has a ctypes signature in the binding
    for s in syms:
        assert s in _lib.SIGNATURES or s == "sa_last_error", s


def test_status_codes_match_header():
    text = open(HEADER).read()
    for name in ("SA_OK", "SA_ERR_INVALID_ARG", "SA_ERR_UNSUPPORTED", "SA_ERR_CUDA", "SA_ERR_TIMEOUT",
                 "SA_ERR_WORKSPACE", "SA_COMPRESSOR_NONE", "SA_COMPRESSOR_SORTED_PAIR", "SA_COMPRESSOR_RANDOM"):
        m = re.search(rf"#define {name} \(?(-?\d+)\)?", text)
        assert m, name
        val = int(m.group(1))
        if name.startswith("SA_COMPRESSOR_"):
            key = name[len("SA_COMPRESSOR_"):].lower()
            assert _lib.COMPRESSORS[key] == val
        else:
            assert getattr(_lib, name) == val


@pytest.mark.parametrize("d,t,expect", [(64, 2, 2145), (32, 2, 561), (16, 3, 969), (12, 2, 91), (5, 0, 1),
                                        (7, 1, 8), (64, 3, 47905)])
def test_feature_count(d, t, expect):
    lib = _lib.load()
    out = ctypes.c_int64(0)
    assert lib.sa_feature_count(d, t, ctypes.byref(out)) == 0
    assert out.value == expect


def test_feature_count_rejects_degree_above_three():
    lib = _lib.load()
    out = ctypes.c_int64(0)
    assert lib.sa_feature_count(8, 4, ctypes.byref(out)) == _lib.SA_ERR_UNSUPPORTED
    assert "degree" in _lib.last_error()
    assert lib.sa_feature_count(8, -1, ctypes.byref(out)) == _lib.SA_ERR_INVALID_ARG


@pytest.mark.parametrize("n,bs,comp,nc,m", [(1024, 128, 1, 7, 64), (129, 128, 1, 1, 64), (128, 128, 1, 0, 64),
                                            (200, 33, 2, 6, 17), (50, 2, 1, 24, 1), (4096, 256, 0, 15, 256),
                                            (0, 16, 1, 0, 8), (1, 16, 1, 0, 8)])
def test_block_counts(n, bs, comp, nc, m):
    lib = _lib.load()
    a, b = ctypes.c_int64(-1), ctypes.c_int64(-1)
    assert lib.sa_block_counts(n, bs, comp, ctypes.byref(a), ctypes.byref(b)) == 0
    assert (a.value, b.value) == (nc, m)


def test_workspace_size_and_argument_errors_without_gpu():
    lib = _lib.load()
    sz = ctypes.c_size_t(0)
    assert lib.sa_fast_attention_workspace_size(256, 8192, 64, 64, 2, 128, 1, ctypes.byref(sz)) == 0
    R = 63 * 64
    # tensor-core layout: G partial slices of the low sums and the fp32 moment state of G
    # feature groups, hi/lo copies of k, v (transposed) and of the reps, rep weights and
    # indices, and the gathered rep values before their transposing split
    fixed = 4 * 256 * 8192 * 64 * 4 + 4 * 256 * R * 64 * 4 + 256 * R * 4 + 256 * R * 4 + 256 * R * 64 * 4
    per_group = 256 * 8192 * 65 * 4 + 256 * 5 * 128 * 64 * 4   # five state tiles of 128 features per group
    groups = (sz.value - fixed) // per_group
    assert groups == 4   # 2376 padded features (d = 64, degree 2) in 19 tiles
    assert fixed + groups * per_group <= sz.value < fixed + groups * per_group + 4096
    # argument errors return before any CUDA call
    assert lib.sa_fast_attention(None, None, None, 1, 16, 8, 8, 2, 0, 1.0, 1, None, None, None, 1e-12, None, None,
                                 None, 0, None) == _lib.SA_ERR_INVALID_ARG
    assert "block_size" in _lib.last_error()
    assert lib.sa_fast_attention(None, None, None, 1, 16, 8, 8, 5, 4, 1.0, 1, None, None, None, 1e-12, None, None,
                                 None, 0, None) == _lib.SA_ERR_UNSUPPORTED
    assert lib.sa_fast_attention(None, None, None, 0, 16, 8, 8, 2, 4, 1.0, 7, None, None, None, 1e-12, None, None,
                                 None, 0, None) == _lib.SA_ERR_INVALID_ARG
    assert "compressor" in _lib.last_error()
    assert lib.sa_fast_attention(None, None, None, 1, 16, 8, 8, 2, 4, 1.0, 1, None, None, None, 1e-12, None, None,
                                 None, 0, None) == _lib.SA_ERR_INVALID_ARG
    assert "null" in _lib.last_error()
    # empty problem is a no-op
    assert lib.sa_fast_attention(None, None, None, 0, 16, 8, 8, 2, 4, 1.0, 1, None, None, None, 1e-12, None, None,
                                 None, 0, None) == 0
    with pytest.raises(ValueError):
        _lib.check(_lib.SA_ERR_INVALID_ARG, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.SA_ERR_UNSUPPORTED, "x")
    with pytest.raises(_lib.SAError):
        _lib.check(_lib.SA_ERR_TIMEOUT, "x")


def test_moment_fork_switch_is_per_thread():
    import threading
    lib = _lib.load()
    assert lib.sa_moment_fork_enabled() == 1
    assert lib.sa_set_moment_fork(0) == _lib.SA_OK
    try:
        assert lib.sa_moment_fork_enabled() == 0
        seen = []
        t = threading.Thread(target=lambda: seen.append(lib.sa_moment_fork_enabled()))
        t.start()
        t.join()
        assert seen == [1]   # another host thread keeps the default
    finally:
        lib.sa_set_moment_fork(1)
    assert lib.sa_moment_fork_enabled() == 1
