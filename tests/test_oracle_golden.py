"""Pin the CPU oracle against fixtures produced by the reference itself.

The oracle (oracle/oracle.py) is the checker for every GPU parity test, so it
is checked first: coreset selections must be bit-exact, outputs within 1e-5
relative L2 of the float32 reference (the oracle runs in float64).
"""

import json

import numpy as np
import pytest

from conftest import golden_names, load_golden, stream_golden_names
from oracle import oracle as O


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_fixture(name):
    g = load_golden(name)
    m = g["meta"]
    B, H = g["q"].shape[:2]
    for b in range(B):
        for h in range(H):
            hs = m["attn_seed"] + b * H + h
            out, ln, ld, tn, td, reps, stats = O.fast_attention_single(
                g["q"][b, h], g["k"][b, h], g["v"][b, h], degree=m["degree"], block_size=m["bs"],
                scale=m["scale"], compressor=m["compressor"], seed=hs, device_type="cpu")
            # coreset selection: bit-exact global indices and weights
            np.testing.assert_array_equal(reps.idx.astype(np.int32), g["rep_idx"][b, h])
            np.testing.assert_array_equal(reps.weight.astype(np.float32), g["rep_w"][b, h])
            # low term and output within float32-reference tolerance
            assert O.relative_l2(ln, g["low_num"][b, h]) < 1e-5
            assert O.relative_l2(ld, g["low_den"][b, h]) < 1e-5
            assert O.relative_l2(out, g["out"][b, h]) < 1e-5, name
            if m["compressor"] == "none":
                assert O.relative_l2(out, g["exact"][b, h]) < 1e-5
            if m["degree"] <= 2 and stats is not None and m["stats"]:
                # the fixture's stats are the CPU (stream-mode) ones
                for key, val in m["stats"].items():
                    assert stats[key] == val, (key, stats[key], val)


def test_exp_taylor_known_values():
    z = np.load(__import__("conftest").GOLDEN + "/misc.npz")
    x = z["taylor_x"]
    for t in range(5):
        np.testing.assert_allclose(O.exp_taylor(x.astype(np.float32), t), z[f"taylor_{t}"], rtol=1e-6, atol=1e-6)
    # test_streaming_attention.py:27-31 known answers
    y = O.exp_taylor(np.array([0.0, 1.0, -1.0]), 3)
    np.testing.assert_allclose(y, [1.0, 1 + 1 + 0.5 + 1 / 6, 1 - 1 + 0.5 - 1 / 6])


def test_feature_map_order_and_counts():
    z = np.load(__import__("conftest").GOLDEN + "/misc.npz")
    counts = json.loads(bytes(z["feat_counts"]).decode())
    for key, val in counts.items():
        d, t = map(int, key.split("_"))
        assert O.num_features(d, t) == val
    np.testing.assert_allclose(O.key_features(z["fm_key"], 3), z["fm_kf"], rtol=1e-6)
    np.testing.assert_allclose(O.query_features(z["fm_qry"], 3), z["fm_qf"], rtol=1e-6)
    np.testing.assert_allclose(O.key_features(z["x2"], 2), z["f2k"], rtol=1e-6)
    np.testing.assert_allclose(O.query_features(z["x2"], 2), z["f2q"], rtol=1e-6)
    # <phi_k(k), phi_q(q)> = P_t(k.q)
    rng = np.random.default_rng(0)
    for d, t in [(5, 3), (7, 2), (3, 1), (4, 0)]:
        kk, qq = rng.standard_normal(d), rng.standard_normal(d)
        lhs = O.key_features(kk, t) @ O.query_features(qq, t)
        assert abs(lhs - O.exp_taylor(np.array(kk @ qq), t)) < 1e-12


def test_low_terms_match_direct_polynomial_sum():
    rng = np.random.default_rng(1)
    n, d, dv = 70, 5, 3
    q, k, v = rng.standard_normal((n, d)), rng.standard_normal((n, d)), rng.standard_normal((n, dv))
    for t in range(4):
        ln, ld = O.low_terms(q, k, v, degree=t, scale=0.3, chunk=16)
        p = np.tril(O.exp_taylor((q @ k.T) * 0.3, t))
        np.testing.assert_allclose(ld, p.sum(-1), rtol=1e-11)
        np.testing.assert_allclose(ln, p @ v, rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("name", ["cfg1_full", "cfg3_small", "cfg2_small", "random_ragged", "degree3_random",
                                  "sorted_pair_odd_bs"])
def test_row_oracle_matches_full_oracle(name):
    g = load_golden(name)
    m = g["meta"]
    n = g["q"].shape[2]
    rows = np.unique(np.r_[0, n - 1, np.arange(0, n, max(1, n // 37))])
    q, k, v = g["q"][0, 0], g["k"][0, 0], g["v"][0, 0]
    full = O.fast_attention_single(q, k, v, degree=m["degree"], block_size=m["bs"], scale=m["scale"],
                                   compressor=m["compressor"], seed=m["attn_seed"])[0]
    part = O.fast_attention_rows(q, k, v, rows, degree=m["degree"], block_size=m["bs"], scale=m["scale"],
                                 compressor=m["compressor"], seed=m["attn_seed"])
    np.testing.assert_allclose(part, full[rows], rtol=1e-9, atol=1e-11)


def test_low_terms_before_block_plus_block_exp_is_the_output():
    g = load_golden("cfg3_small")
    q, k, v = (g[x][0, 0] for x in "qkv")
    s = 1 / 8.0
    ln, ld = O.low_terms_before_block(q, k, v, degree=2, scale=s, bs=128)
    full_ln, full_ld = O.low_terms(q, k, v, degree=2, scale=s)
    # the difference is the current block's polynomial part
    x = (q.astype(np.float64) @ k.T.astype(np.float64)) * s
    n = q.shape[0]
    blk = np.arange(n) // 128
    cur = (blk[:, None] == blk[None, :]) & (np.arange(n)[None, :] <= np.arange(n)[:, None])
    p = np.where(cur, O.exp_taylor(x, 2), 0)
    np.testing.assert_allclose(ln + p @ v, full_ln, rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(ld + p.sum(-1), full_ld, rtol=1e-12)


@pytest.mark.parametrize("name", stream_golden_names())
def test_streaming_oracle_matches_reference_fixture(name):
    """ArticleStreamingAttention restated: per-token outputs, coreset sizes, the
    final merge-and-reduce items (bit-exact) and the number of compressions."""
    g = load_golden(name)
    m = g["meta"]
    out, ld, td, items, final, comps = O.stream_attention(
        g["q"], g["k"], g["v"], degree=m["degree"], block_size=m["bs"], compressor=m["compressor"], seed=m["seed"])
    assert O.relative_l2(out, g["out"]) < 1e-5
    np.testing.assert_array_equal(items, g["items"])
    np.testing.assert_array_equal(final.keys, g["final_keys"])
    np.testing.assert_array_equal(final.values, g["final_values"])
    np.testing.assert_array_equal(final.weights, g["final_weights"])
    assert comps == int(g["compressions"])
    np.testing.assert_allclose(ld + td, g["den"], rtol=1e-5)


def test_streaming_oracle_rejects_small_blocks():
    with pytest.raises(ValueError, match="block_size must be at least 2"):
        O.stream_attention(np.zeros((3, 2)), np.zeros((3, 2)), np.zeros((3, 1)), block_size=1)
