"""GPU parity of the streaming class (ArticleStreamingAttention,
streaming_taylor_coreset_attention.py:523-616) through the sa_stream_* C ABI.

Bars: per-token outputs within 1e-5 relative L2 of the reference fixtures;
coreset sizes per token, the final merge-and-reduce items (keys, values,
weights) and the number of compressions equal to the reference's.
"""

import numpy as np
import pytest
import torch

import streaming_attention_b200 as sa
from conftest import load_golden, stream_golden_names
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _run(att, q, k, v):
    outs, items, dens = [], [], []
    for i in range(q.shape[0]):
        att.update(k[i], v[i])
        o, st = att.query(q[i], return_stats=True)
        outs.append(o.cpu().numpy())
        items.append(st.coreset_items)
        dens.append(st.denominator)
    return np.stack(outs), np.asarray(items), np.asarray(dens)


@pytest.mark.parametrize("name", stream_golden_names())
def test_streaming_matches_reference_fixture(name, dev):
    g = load_golden(name)
    m = g["meta"]
    att = sa.ArticleStreamingAttention(m["d"], m["dv"], degree=m["degree"], block_size=m["bs"], scale=None,
                                       compressor=m["compressor"], device=dev, seed=m["seed"])
    q, k, v = (torch.from_numpy(g[x]) for x in "qkv")
    out, items, dens = _run(att, q, k, v)
    assert O.relative_l2(out, g["out"]) < TOL
    np.testing.assert_array_equal(items, g["items"])
    np.testing.assert_allclose(dens, g["den"], rtol=TOL)
    fk, fv, fw = (x.cpu().numpy() for x in att.items())
    np.testing.assert_array_equal(fk, g["final_keys"])
    np.testing.assert_array_equal(fv, g["final_values"])
    np.testing.assert_array_equal(fw, g["final_weights"])
    assert att.num_compressions == int(g["compressions"])
    assert att.length == m["n"]
    st = att.state_size_bytes()
    assert st == int(g["state_bytes"][-1])


@pytest.mark.parametrize("comp", ["sorted_pair", "random"])
def test_streaming_at_transformer_width_against_the_oracle(comp, dev):
    """d = dv = 64, degree 2 (2145 features), blocks of 32: several merge levels."""
    n, d, dv, bs = 300, 64, 64, 32
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(n, d, generator=gen)
    k = torch.randn(n, d, generator=gen)
    v = torch.randn(n, dv, generator=gen)
    q, k = q / q.norm(dim=1, keepdim=True) * 4.0, k / k.norm(dim=1, keepdim=True) * 4.0
    att = sa.ArticleStreamingAttention(d, dv, degree=2, block_size=bs, compressor=comp, device=dev, seed=9)
    out, items, _ = _run(att, q, k, v)
    ref, _, _, ref_items, final, comps = O.stream_attention(q.numpy(), k.numpy(), v.numpy(), degree=2,
                                                            block_size=bs, compressor=comp, seed=9)
    assert O.relative_l2(out, ref) < TOL
    np.testing.assert_array_equal(items, ref_items)
    np.testing.assert_array_equal(att.items()[2].cpu().numpy(), final.weights)
    assert att.num_compressions == comps


def test_streaming_errors_and_dtypes(dev):
    att = sa.ArticleStreamingAttention(4, 3, block_size=4, device=dev, dtype=torch.float16)
    with pytest.raises(ValueError, match=r"key must have shape \[4\]"):
        att.update(torch.zeros(5), torch.zeros(3))
    with pytest.raises(ValueError, match=r"value must have shape \[3\]"):
        att.update(torch.zeros(4), torch.zeros(2))
    att.update(torch.ones(4), torch.ones(3))
    with pytest.raises(ValueError, match=r"query must have shape \[4\]"):
        att.query(torch.zeros(3))
    out = att.query(torch.ones(4))
    assert out.dtype == torch.float16 and out.device.type == "cuda"
    # a single key: softmax over one item is its value
    torch.testing.assert_close(out.float().cpu(), torch.ones(3), rtol=1e-3, atol=1e-3)
    bad = sa.ArticleStreamingAttention(2, 1, block_size=2, compressor="bogus", device=dev)
    bad.update(torch.zeros(2), torch.zeros(1))
    with pytest.raises(ValueError, match="compressor must be one of"):
        bad.update(torch.zeros(2), torch.zeros(1))
