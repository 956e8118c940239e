"""GPU parity of the segment-mean variant (triton_article_causal_attention,
triton_article_attention.py:448-578) through sa_article_segment_mean.

Bars: the reps equal the reference's build_segment_mean_coreset within the
rounding bound of a float32 sum of compress_stride terms (torch's mean sums in
its own order), plus one unit of the storage dtype for 16-bit inputs; outputs within 1e-5 relative L2 of the float64 oracle fed the
reference's reps; compress_stride 1 within 1e-5 of the reference's exact
attention and bit-identical to the fast path with compressor none (the same
kernels; the exp cap at 80 is not reached).
"""

import os

import numpy as np
import pytest
import torch

import streaming_attention_b200 as sa
from conftest import load_golden, segment_golden_names
from oracle import oracle as O
from test_oracle_golden import _rep_tolerance

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _inputs(g, dev):
    dt = getattr(torch, g["meta"]["dtype"])
    return tuple(torch.from_numpy(g[x]).to(dev).to(dt) for x in "qkv")


@pytest.mark.parametrize("name", segment_golden_names())
def test_segment_reps_match_reference_fixture(name, dev):
    g = load_golden(name)
    m = g["meta"]
    q, k, v = _inputs(g, dev)
    rk, rv, mm = sa.build_segment_mean_coreset(k.reshape(-1, m["n"], m["d"]), v.reshape(-1, m["n"], m["dv"]),
                                               block_size=m["bs"], compress_stride=m["stride"])
    assert mm == int(g["reps_per_block"])
    assert rk.dtype == k.dtype and rv.dtype == v.dtype
    rk, rv = rk.float().cpu().numpy(), rv.float().cpu().numpy()
    assert rk.shape == g["rep_k"].shape and rv.shape == g["rep_v"].shape
    for got, want in ((rk, g["rep_k"]), (rv, g["rep_v"])):
        np.testing.assert_allclose(got, want, rtol=0, atol=_rep_tolerance(want, m["dtype"], m["stride"]))


@pytest.mark.parametrize("name", segment_golden_names())
@pytest.mark.parametrize("degree", [0, 1, 2])
def test_segment_attention_matches_oracle_on_reference_reps(name, degree, dev):
    g = load_golden(name)
    m = g["meta"]
    q, k, v = _inputs(g, dev)
    out, st = sa.triton_article_causal_attention(q, k, v, degree=degree, block_size=m["bs"],
                                                 compress_stride=m["stride"], return_stats=True)
    assert out.dtype == torch.float32 and out.shape == v.shape
    n = m["n"]
    qs, ks, vs = (g[x].reshape(-1, n, g[x].shape[-1]) for x in "qkv")
    got = out.reshape(-1, n, m["dv"]).cpu().numpy()
    for h in range(qs.shape[0]):
        ref = O.segment_mean_attention(qs[h], ks[h], vs[h], degree=degree, block_size=m["bs"],
                                       compress_stride=m["stride"], rep_k=g["rep_k"][h], rep_v=g["rep_v"][h])
        assert O.relative_l2(got[h], ref) < TOL, (h, O.relative_l2(got[h], ref))
    if m["stride"] == 1:
        assert O.relative_l2(got, g["exact"].reshape(got.shape)) < TOL
    R = g["rep_k"].shape[-2]
    elem = q.element_size()
    assert st.coreset_items_per_sequence == R
    assert st.coreset_bytes_per_sequence == R * (m["d"] + m["dv"]) * elem
    assert st.kv_bytes_per_sequence == n * (m["d"] + m["dv"]) * elem
    assert st.score_matrix_bytes_per_sequence == n * n * elem
    assert st.output_bytes_per_sequence == n * m["dv"] * 4
    assert (st.degree, st.block_size, st.compress_stride) == (degree, m["bs"], m["stride"])


@pytest.mark.parametrize("d,dv,bs,stride,simt", [
    (64, 64, 128, 2, False),    # tensor-core residual and moments
    (32, 128, 64, 4, False),    # dv 128: tensor-core residual, CUDA-core moments
    (96, 40, 32, 2, False),     # d > 64: CUDA-core residual
    (16, 8, 6, 3, False),       # block_size % 4 != 0: CUDA-core path
    (64, 64, 128, 2, True),     # the CUDA-core path on request
    (48, 200, 32, 8, False),    # dv > 128: value column slices
])
def test_segment_shapes_against_oracle(d, dv, bs, stride, simt, dev, monkeypatch):
    if simt:
        monkeypatch.setenv("SA_FORCE_SIMT", "1")
    n, heads = 700, 3
    gen = torch.Generator().manual_seed(d * 1000 + dv)
    q = torch.randn(1, heads, n, d, generator=gen) * 0.4
    k = torch.randn(1, heads, n, d, generator=gen) * 0.4
    v = torch.randn(1, heads, n, dv, generator=gen)
    out = sa.triton_article_causal_attention(q.to(dev), k.to(dev), v.to(dev), degree=2, block_size=bs,
                                             compress_stride=stride)
    got = out[0].cpu().numpy()
    for h in range(heads):
        ref = O.segment_mean_attention(q[0, h].numpy(), k[0, h].numpy(), v[0, h].numpy(), degree=2, block_size=bs,
                                       compress_stride=stride)
        assert O.relative_l2(got[h], ref) < TOL


def test_segment_stride1_equals_fast_path_without_compression(dev):
    """Same kernels, same reps (every earlier key, weight 1): bit-identical."""
    gen = torch.Generator().manual_seed(5)
    q, k = (torch.randn(2, 4, 2048, 64, generator=gen).mul(0.3).to(dev) for _ in range(2))
    v = torch.randn(2, 4, 2048, 64, generator=gen).to(dev)
    a = sa.triton_article_causal_attention(q, k, v, degree=2, block_size=128, compress_stride=1)
    b = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=128, compressor="none")
    assert torch.equal(a, b)


def test_segment_exp_cap_against_oracle(dev):
    """Scores well above 80: the cap keeps every weight finite, as in the reference."""
    gen = torch.Generator().manual_seed(11)
    n, d = 300, 32
    q = torch.randn(n, d, generator=gen)
    q = q / q.norm(dim=1, keepdim=True) * 12.0
    k = q * 0.9 + 0.1 * torch.randn(n, d, generator=gen)   # self scores near 130
    v = torch.randn(n, 16, generator=gen)
    out = sa.triton_article_causal_attention(q.to(dev), k.to(dev), v.to(dev), degree=2, block_size=32,
                                             compress_stride=2, scale=1.0)
    ref = O.segment_mean_attention(q.numpy(), k.numpy(), v.numpy(), degree=2, block_size=32, compress_stride=2,
                                   scale=1.0)
    assert np.isfinite(ref).all() and torch.isfinite(out).all()
    assert float((q @ k.T).max()) > 100.0
    assert O.relative_l2(out.cpu().numpy(), ref) < TOL


def test_segment_errors_dtypes_and_edges(dev):
    x = torch.zeros(8, 4, device=dev)
    with pytest.raises(NotImplementedError, match="degree 0, 1, or 2"):
        sa.triton_article_causal_attention(x, x, x, degree=3)
    with pytest.raises(ValueError, match="must be positive"):
        sa.triton_article_causal_attention(x, x, x, block_size=0)
    with pytest.raises(ValueError, match="divisible by compress_stride"):
        sa.triton_article_causal_attention(x, x, x, block_size=6, compress_stride=4)
    with pytest.raises(ValueError, match="require CUDA tensors"):
        sa.triton_article_causal_attention(x.cpu(), x.cpu(), x.cpu())
    with pytest.raises(ValueError, match="q and k must match"):
        sa.triton_article_causal_attention(x, x[:, :3], x)
    with pytest.raises(ValueError, match=r"v must be \[N,Dv\]"):
        sa.triton_article_causal_attention(x, x, x[:7])
    big = torch.zeros(4, 130, device=dev)
    with pytest.raises(ValueError, match="D <= 128"):
        sa.triton_article_causal_attention(big, big, x[:4])
    with pytest.raises(ValueError, match="Dv <= 256"):
        sa.triton_article_causal_attention(x, x, torch.zeros(8, 257, device=dev))
    # half inputs, half output; n < block_size has no reps
    h = torch.randn(2, 3, 40, 16, device=dev).half()
    out, st = sa.triton_article_causal_attention(h, h, h, block_size=64, output_dtype=torch.float16,
                                                 return_stats=True)
    assert out.dtype == torch.float16 and st.coreset_items_per_sequence == 0
    ref = O.segment_mean_attention(h[1, 2].float().cpu().numpy(), h[1, 2].float().cpu().numpy(),
                                   h[1, 2].float().cpu().numpy(), block_size=64, compress_stride=2)
    assert O.relative_l2(out[1, 2].float().cpu().numpy(), ref) < 2e-3
    # empty batch
    e = torch.zeros(0, 2, 16, 8, device=dev)
    assert sa.triton_article_causal_attention(e, e, e).shape == (0, 2, 16, 8)
    # the rep builder's own checks
    with pytest.raises(ValueError, match="must be"):
        sa.build_segment_mean_coreset(x, x, block_size=4, compress_stride=2)
    with pytest.raises(ValueError, match="divisible"):
        sa.build_segment_mean_coreset(x[None], x[None], block_size=6, compress_stride=4)
