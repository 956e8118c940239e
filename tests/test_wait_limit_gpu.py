"""Failure detection on the GPU without a fault: the bounded device-side waits.

Every wait of the tensor-core kernels (an mbarrier that a TMA copy, an MMA
commit or another warp completes) gives up after the process-wide wait limit
(sa_set_wait_limit_ns, 2 s by default).  The CTA that gives up drains the copies
and products it issued, frees its TMEM, writes the wait's code into the status
word at the start of the workspace and returns; sa_workspace_status then
reports SA_ERR_TIMEOUT.  Here the limit is set to 1 ns, so that waits run out
on an ordinary small problem; the status must say so, and the next call with
the default limit on the same context must give the normal result.
"""

import ctypes

import pytest
import torch

from oracle import oracle as O
from streaming_attention_b200 import _lib, draws, workloads

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _forward(lib, c, q, k, v, t, ws, out, stream):
    bh, n, d = q.shape
    rc = lib.sa_fast_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), bh, n, d, v.shape[-1], c["degree"],
                               c["block_size"], workloads.attention_scale(c), _lib.COMPRESSORS[c["compressor"]],
                               t.dirs.data_ptr(), t.coins.data_ptr(), None, 1e-12, out.data_ptr(), None,
                               ws.data_ptr(), ws.numel(), stream)
    _lib.check(rc, "sa_fast_attention")


def test_wait_limit_runs_out_and_the_next_call_is_correct():
    assert torch.cuda.is_available(), "GPU test"
    dev = torch.device("cuda:0")
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    c = workloads.config(3, B=1, H=4, N=2048)
    q, k, v = workloads.make_inputs(c, seed=5, device=dev)
    bh, n, d, dv = 4, c["N"], c["d"], c["dv"]
    q, k, v = q.reshape(bh, n, d).contiguous(), k.reshape(bh, n, d).contiguous(), v.reshape(bh, n, dv).contiguous()
    t = draws.draw_tables(seed=0, batch=1, heads=4, n=n, d=d, block_size=c["block_size"],
                          compressor=c["compressor"], device=dev)
    size = ctypes.c_size_t(0)
    _lib.check(lib.sa_fast_attention_workspace_size(bh, n, d, dv, c["degree"], c["block_size"],
                                                    _lib.COMPRESSORS[c["compressor"]], ctypes.byref(size)), "size")
    ws = torch.empty(size.value, device=dev, dtype=torch.uint8)
    ref = torch.empty(bh, n, dv, device=dev)
    _forward(lib, c, q, k, v, t, ws, ref, stream)
    assert lib.sa_workspace_status(ws.data_ptr(), stream) == _lib.SA_OK

    out = torch.zeros(bh, n, dv, device=dev)
    try:
        _lib.check(lib.sa_set_wait_limit_ns(1), "sa_set_wait_limit_ns")
        _forward(lib, c, q, k, v, t, ws, out, stream)
        rc = lib.sa_workspace_status(ws.data_ptr(), stream)
    finally:
        lib.sa_set_wait_limit_ns(0)
    assert rc == _lib.SA_ERR_TIMEOUT, rc
    assert "wait" in _lib.last_error()
    # the context is still usable: a normal call on the same workspace gives the normal result
    torch.cuda.synchronize(dev)
    _forward(lib, c, q, k, v, t, ws, out, stream)
    assert lib.sa_workspace_status(ws.data_ptr(), stream) == _lib.SA_OK
    err = O.relative_l2(out.cpu().numpy(), ref.cpu().numpy())
    assert err < TOL, err
