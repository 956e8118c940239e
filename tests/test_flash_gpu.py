"""GPU parity of the exact causal attention (triton_flash_causal_attention,
triton_article_attention.py:580-637) through sa_flash_causal_attention.

Bars: within 1e-5 relative L2 of the float64 masked-softmax oracle on every
shape either kernel takes (tensor cores: d <= 64, dv <= 128; CUDA cores
otherwise), through many moves of the running maximum, and at the config 2
shape against the fast path with compressor none (the exact decomposition)
and against torch's own fp32 attention.
"""

import numpy as np
import pytest
import torch

import streaming_attention_b200 as sa
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _check(q, k, v, out, scale=None):
    qs, ks, vs = (x.reshape(-1, x.shape[-2], x.shape[-1]).double().cpu().numpy() for x in (q, k, v))
    got = out.reshape(qs.shape[0], qs.shape[1], -1).double().cpu().numpy()
    for h in range(qs.shape[0]):
        ref = O.classical(qs[h], ks[h], vs[h], scale=scale)
        err = O.relative_l2(got[h], ref)
        assert err < TOL, (h, err)


@pytest.mark.parametrize("n", [1, 2, 63, 64, 65, 127, 128, 129, 700])
@pytest.mark.parametrize("d,dv", [(64, 64), (32, 32), (16, 128), (64, 96), (96, 40), (128, 256), (48, 200)])
def test_flash_matches_oracle(n, d, dv, dev):
    gen = torch.Generator().manual_seed(n * 7 + d + dv)
    q = torch.randn(2, 2, n, d, generator=gen)
    k = torch.randn(2, 2, n, d, generator=gen)
    v = torch.randn(2, 2, n, dv, generator=gen)
    out = sa.triton_flash_causal_attention(q.to(dev), k.to(dev), v.to(dev))
    assert out.shape == (2, 2, n, dv) and out.dtype == torch.float32
    _check(q, k, v, out)


@pytest.mark.parametrize("simt", [False, True])
def test_flash_running_maximum_moves(simt, dev, monkeypatch):
    """Keys grow along the sequence, so the row maximum climbs by about six
    units per 64-key tile to about 105: the lazily moved maximum rescales O
    over and over, and exp of the raw scores would lose the small ones.  The
    bar allows for the scores' own fp32 rounding: 4 ulps of the largest score."""
    if simt:
        monkeypatch.setenv("SA_FORCE_SIMT", "1")
    n, d = 1200, 64
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(3, n, d, generator=gen)
    q = q / q.norm(dim=-1, keepdim=True)
    dirn = torch.randn(d, generator=gen)
    dirn = dirn / dirn.norm()
    q = 0.7 * q + 0.7 * dirn
    grow = torch.linspace(0.0, 150.0, n)[None, :, None]
    k = torch.randn(3, n, d, generator=gen) * 0.5 + grow * dirn
    v = torch.randn(3, n, 64, generator=gen)
    out = sa.triton_flash_causal_attention(q[None].to(dev), k[None].to(dev), v[None].to(dev), scale=1.0)[0]
    assert torch.isfinite(out).all()
    top = float((q @ k.transpose(-1, -2)).tril().abs().max())
    assert top > 90.0
    tol = max(TOL, 4 * 2.0 ** -24 * top)
    qs, ks, vs = (x.double().numpy() for x in (q, k, v))
    got = out.double().cpu().numpy()
    for h in range(3):
        assert O.relative_l2(got[h], O.classical(qs[h], ks[h], vs[h], scale=1.0)) < tol


def test_flash_config2_against_fast_path_and_torch(dev):
    """Config 2's shape (B=4, H=8, N=4096, d=dv=64, scale 1/8): the exact
    decomposition of the fast path (compressor none) and torch's fp32 attention."""
    gen = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(4, 8, 4096, 64, generator=gen).to(dev) for _ in range(3))
    out = sa.triton_flash_causal_attention(q, k, v)
    fast = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=256, compressor="none")
    assert sa.safe_relative_l2(out, fast) < TOL
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert sa.safe_relative_l2(out, ref) < TOL


def test_flash_simt_and_tensor_cores_agree(dev, monkeypatch):
    gen = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, 4, 1000, 64, generator=gen).to(dev) for _ in range(3))
    a = sa.triton_flash_causal_attention(q, k, v)
    monkeypatch.setenv("SA_FORCE_SIMT", "1")
    b = sa.triton_flash_causal_attention(q, k, v)
    assert sa.safe_relative_l2(a, b) < TOL


def test_flash_errors_and_dtypes(dev):
    x = torch.zeros(8, 4, device=dev)
    with pytest.raises(ValueError, match="require CUDA tensors"):
        sa.triton_flash_causal_attention(x.cpu(), x.cpu(), x.cpu())
    with pytest.raises(ValueError, match="D <= 128"):
        big = torch.zeros(4, 130, device=dev)
        sa.triton_flash_causal_attention(big, big, x[:4])
    with pytest.raises(ValueError, match="Dv <= 256"):
        sa.triton_flash_causal_attention(x, x, torch.zeros(8, 300, device=dev))
    with pytest.raises(ValueError, match="q and k must match"):
        sa.triton_flash_causal_attention(x, x[:, :2], x)
    h = torch.randn(300, 32, device=dev).half()
    out = sa.triton_flash_causal_attention(h, h, h, output_dtype=torch.float16)
    assert out.dtype == torch.float16 and out.shape == (300, 32)
    ref = O.classical(h.double().cpu().numpy(), h.double().cpu().numpy(), h.double().cpu().numpy())
    assert O.relative_l2(out.double().cpu().numpy(), ref) < 2e-3
    e = torch.zeros(2, 0, 5, 8, device=dev)
    assert sa.triton_flash_causal_attention(e, e, e).shape == (2, 0, 5, 8)
