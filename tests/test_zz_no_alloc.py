"""The allocation-free entry point gives the same result as the workspace one.

sa_fast_attention_static_scratch serves callers that cannot allocate device
memory themselves (their HBM belongs to another allocator, or their serving
loop forbids cudaMalloc after start-up, or they are plain C callers without a
device allocator): it runs the same forward as sa_fast_attention but takes its
scratch from an array built into the library.  Here it is called through the
C ABI twice in a row, on two different problems, and each result is compared
with sa_fast_attention given a normal workspace.  The file is named so that
pytest collects it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from streaming_attention_b200 import _lib, draws, workloads

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the fp32 tolerance used by every parity test


def _problem(cfg, seed, dev, **over):
    c = workloads.config(cfg, **over)
    q, k, v = workloads.make_inputs(c, seed=seed, device=dev)
    bh = c["B"] * c["H"]
    n, d, dv = c["N"], c["d"], c["dv"]
    t = draws.draw_tables(seed=seed, batch=c["B"], heads=c["H"], n=n, d=d, block_size=c["block_size"],
                          compressor=c["compressor"], device=dev)
    return c, (q.reshape(bh, n, d).contiguous(), k.reshape(bh, n, d).contiguous(),
               v.reshape(bh, n, dv).contiguous()), t


def _args(c, qkv, t):
    q, k, v = qkv
    bh, n, d = q.shape
    scale = workloads.attention_scale(c)
    comp = _lib.COMPRESSORS[c["compressor"]]
    ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
    return (q.data_ptr(), k.data_ptr(), v.data_ptr(), bh, n, d, v.shape[-1], c["degree"], c["block_size"], scale,
            comp, ptr(t.dirs), ptr(t.coins), ptr(t.perms), 1e-12)


def _with_workspace(lib, c, qkv, t, stream):
    bh, n, _ = qkv[0].shape
    out = torch.empty(bh, n, qkv[2].shape[-1], device=qkv[0].device)
    idx = torch.empty(bh, max(1, t.completed_blocks * t.reps_per_block), device=qkv[0].device, dtype=torch.int32)
    size = ctypes.c_size_t(0)
    _lib.check(lib.sa_fast_attention_workspace_size(bh, n, qkv[0].shape[-1], qkv[2].shape[-1], c["degree"],
                                                    c["block_size"], _lib.COMPRESSORS[c["compressor"]],
                                                    ctypes.byref(size)), "workspace size")
    ws = torch.empty(size.value, device=qkv[0].device, dtype=torch.uint8)
    _lib.check(lib.sa_fast_attention(*_args(c, qkv, t), out.data_ptr(), idx.data_ptr(), ws.data_ptr(), ws.numel(),
                                     stream), "sa_fast_attention")
    return out, idx


def _static(lib, c, qkv, t, stream, with_idx=True):
    bh, n, _ = qkv[0].shape
    out = torch.empty(bh, n, qkv[2].shape[-1], device=qkv[0].device)
    idx = (torch.empty(bh, max(1, t.completed_blocks * t.reps_per_block), device=qkv[0].device, dtype=torch.int32)
           if with_idx else None)
    _lib.check(lib.sa_fast_attention_static_scratch(*_args(c, qkv, t), out.data_ptr(),
                                                    None if idx is None else idx.data_ptr(), stream),
               "sa_fast_attention_static_scratch")
    return out, idx


def test_static_scratch_entry_point_matches_workspace_entry_point():
    assert torch.cuda.is_available(), "GPU test"
    dev = torch.device("cuda:0")
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    # two calls in a row on different problems: the second one sees the first one's leftovers
    problems = [_problem(3, 11, dev, B=1, H=3, N=2000, block_size=128),
                _problem(1, 12, dev, B=2, H=1, N=700, d=32, dv=32, block_size=64)]
    for c, qkv, t in problems:
        ref, ref_idx = _with_workspace(lib, c, qkv, t, stream)
        got, got_idx = _static(lib, c, qkv, t, stream)
        torch.cuda.synchronize(dev)
        err = O.relative_l2(got.cpu().numpy(), ref.cpu().numpy())
        assert err < TOL, err
        assert torch.equal(got_idx, ref_idx)


def test_static_scratch_rejects_problems_above_its_size():
    assert torch.cuda.is_available(), "GPU test"
    lib = _lib.load()
    # config 3 in full needs ~0.8 GB of scratch: far above the built-in array
    rc = lib.sa_fast_attention_static_scratch(None, None, None, 256, 8192, 64, 64, 2, 128, 0.125, 1, None, None, None,
                                              1e-12, None, None, None)
    assert rc == _lib.SA_ERR_INVALID_ARG
    assert "static scratch" in _lib.last_error()


def test_static_scratch_call_allocates_no_device_memory():
    """The device's free memory is the same before and after a call (the
    outputs are made before the first reading); rep_idx=None makes the call
    keep the selected indices in the built-in array as well."""
    assert torch.cuda.is_available(), "GPU test"
    dev = torch.device("cuda:0")
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    c, qkv, t = _problem(3, 13, dev, B=1, H=2, N=1500, block_size=128)
    ref, _ = _with_workspace(lib, c, qkv, t, stream)
    _static(lib, c, qkv, t, stream, with_idx=False)      # loads the device code on this device
    torch.cuda.synchronize(dev)
    bh, n, _ = qkv[0].shape
    out = torch.full((bh, n, qkv[2].shape[-1]), float("nan"), device=dev)
    torch.cuda.synchronize(dev)
    free0 = torch.cuda.mem_get_info(dev)[0]
    _lib.check(lib.sa_fast_attention_static_scratch(*_args(c, qkv, t), out.data_ptr(), None, stream),
               "sa_fast_attention_static_scratch")
    torch.cuda.synchronize(dev)
    free1 = torch.cuda.mem_get_info(dev)[0]
    assert free1 == free0, (free0, free1)
    err = O.relative_l2(out.cpu().numpy(), ref.cpu().numpy())
    assert err < TOL, err
