"""Host-side logic on CPU: draw tables, stats formulas, argument checks."""

import numpy as np
import pytest
import torch

import streaming_attention_b200 as sa
from conftest import golden_names, load_golden
from oracle import oracle as O
from streaming_attention_b200 import draws, fast


@pytest.mark.parametrize("comp,bs", [("sorted_pair", 16), ("sorted_pair", 33), ("sorted_pair", 2),
                                     ("random", 16), ("random", 1)])
def test_draw_tables_replay_the_reference_stream(comp, bs):
    B, H, n, d, seed = 2, 3, 150, 6, 5
    t = draws.draw_tables(seed=seed, batch=B, heads=H, n=n, d=d, block_size=bs, compressor=comp,
                          device=torch.device("cpu"), cache=False)
    nc = (n - 1) // bs
    assert t.completed_blocks == nc
    for b in range(B):
        for h in range(H):
            ref = O.block_draws(seed + b * H + h, n, d, bs, comp)
            assert len(ref) == nc
            for c, dr in enumerate(ref):
                if dr.perm is not None:
                    np.testing.assert_array_equal(t.perms[b * H + h, c].numpy(), dr.perm)
                else:
                    np.testing.assert_array_equal(t.dirs[b * H + h, c].numpy(), dr.direction)
                    np.testing.assert_array_equal(t.coins[b * H + h, c].numpy(), dr.u)


def test_draw_tables_head_range_is_a_slice_of_the_full_grid():
    kw = dict(seed=3, batch=2, heads=4, n=100, d=5, block_size=10, compressor="sorted_pair",
              device=torch.device("cpu"), cache=False)
    full = draws.draw_tables(**kw)
    part = draws.draw_tables(head_range=(3, 6), **kw)
    assert torch.equal(full.dirs[3:6], part.dirs)
    assert torch.equal(full.coins[3:6], part.coins)


@pytest.mark.parametrize("name", [n for n in golden_names() if load_golden(n)["meta"]["degree"] <= 2])
def test_stats_formula_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    if not m["stats"]:
        pytest.skip("no stats recorded")
    n, d = g["q"].shape[2:]
    dv = g["v"].shape[-1]
    # the fixture ran the reference on CPU with low_mode="stream"
    st = fast._stats(n, d, dv, m["degree"], m["bs"], m["compressor"], "stream", 2048, 4)
    for key, val in m["stats"].items():
        assert getattr(st, key) == val, key


def test_stats_auto_low_mode_resolves_by_input_device():
    """low_mode="auto" means "stream" for host inputs and "prefix" for CUDA inputs
    (fast_article_attention.py:616); the fixture ran the reference on CPU."""
    g = load_golden("reftest_shapes_sorted_pair")
    m = g["meta"]
    n, d = g["q"].shape[2:]
    dv = g["v"].shape[-1]
    host = fast._stats(n, d, dv, m["degree"], m["bs"], m["compressor"], "auto", 2048, 4, "cpu")
    for key, val in m["stats"].items():
        assert getattr(host, key) == val, key
    dev = fast._stats(n, d, dv, m["degree"], m["bs"], m["compressor"], "auto", 2048, 4, "cuda")
    F = sa.num_taylor_features(d, m["degree"])
    assert dev.scratch_low_prefix_bytes == n * F * (1 + dv) * 4
    assert host.scratch_low_prefix_bytes == F * (1 + dv) * 4


def test_num_taylor_features():
    assert sa.num_taylor_features(64, 2) == 2145
    assert sa.num_taylor_features(16, 3) == 969
    with pytest.raises(NotImplementedError):
        sa.num_taylor_features(8, 4)
    with pytest.raises(ValueError):
        sa.num_taylor_features(8, -1)


def test_argument_errors_match_reference_messages():
    q = torch.zeros(8, 4)
    f = sa.fast_article_causal_attention
    with pytest.raises(ValueError, match=r"q,k,v must have shapes"):
        f(q, q[0], q)
    with pytest.raises(ValueError, match="same shape"):
        f(q, torch.zeros(8, 5), q)
    with pytest.raises(ValueError, match="same sequence length"):
        f(q, q, torch.zeros(7, 4))
    with pytest.raises(ValueError, match="query_chunk_size must be positive"):
        f(q, q, q, query_chunk_size=0)
    with pytest.raises(ValueError, match="block_size must be positive"):
        f(q, q, q, block_size=0)
    with pytest.raises(ValueError, match="mode must be one of"):
        f(q, q, q, low_mode="fast")
    with pytest.raises(NotImplementedError):
        f(q, q, q, degree=4)
    with pytest.raises(ValueError, match="compressor must be one of"):
        f(q, q, q, compressor="bogus", block_size=2)
    with pytest.raises(ValueError, match=r"q/k/v must be \[N,D\] or \[B,H,N,D\]"):
        f(q[None], q[None], q[None])
    with pytest.raises(ValueError, match="identical shape"):
        f(q[None, None], q[None, None, :4], q[None, None])
    with pytest.raises(ValueError, match=r"v must have shape \[B,H,N,Dv\]"):
        f(q[None, None], q[None, None], q[None, None, :7])
    # CPU tensors: no CPU fallback
    with pytest.raises(ValueError, match="CUDA"):
        f(q, q, q)


def test_streaming_class_checks_arguments_like_the_reference():
    """ArticleStreamingAttention's constructor errors (streaming_taylor_coreset_attention.py:
    :137-161 feature map, :359-360 coreset), raised before any device work."""
    from streaming_attention_b200 import ArticleStreamingAttention
    with pytest.raises(ValueError, match="dim must be positive"):
        ArticleStreamingAttention(0, 4)
    with pytest.raises(ValueError, match="degree must be non-negative"):
        ArticleStreamingAttention(4, 4, degree=-1)
    with pytest.raises(ValueError, match="exceeding max_monomials=10"):
        ArticleStreamingAttention(8, 4, degree=2, max_monomials=10)
    with pytest.raises(ValueError, match="block_size must be at least 2"):
        ArticleStreamingAttention(4, 4, block_size=1)
    with pytest.raises(ValueError, match="Unsupported dtype"):
        ArticleStreamingAttention(4, 4, dtype="int8")
    with pytest.raises(NotImplementedError):
        ArticleStreamingAttention(4, 4, degree=4)


def test_bench_csv_columns_and_inputs_match_the_reference_benchmark():
    """benchmark_attention.py's CSV header (:205-229) and make_data (:70-101)."""
    from streaming_attention_b200 import bench_csv
    header = ("n,d,dv,degree,block_size,compressor,data,radius,scale,device,dtype,rel_l2,max_abs,mean_abs,"
              "classical_median_ms,classical_best_ms,article_median_ms,article_best_ms,article_final_state_bytes,"
              "article_max_state_bytes,article_max_coreset_items,classical_kv_bytes,classical_naive_scores_bytes")
    assert ",".join(bench_csv.COLUMNS) == header
    # the config 1 fixture was drawn by the reference's make-data with the same generator calls
    g = load_golden("cfg1_full")
    q, k, v = bench_csv.make_data(1024, 32, 32, radius=1.0, data="unit_ball", seed=0)
    np.testing.assert_array_equal(q.numpy(), g["q"].reshape(1024, 32))
    np.testing.assert_array_equal(v.numpy(), g["v"].reshape(1024, 32))


def test_host_chunk_plan_tapers_and_covers_every_sequence():
    from streaming_attention_b200.fast import _chunk_plan
    assert _chunk_plan(256, 61) == [61, 61, 61, 37, 18, 9, 7, 2]
    assert _chunk_plan(6, 2) == [2, 2, 1, 1]
    assert _chunk_plan(1, 61) == [1]
    for bh in range(1, 200, 7):
        for base in (1, 3, 16, 61):
            plan = _chunk_plan(bh, base)
            assert sum(plan) == bh and max(plan) <= base and min(plan) >= 1
