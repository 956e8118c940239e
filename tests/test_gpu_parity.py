"""GPU parity: the CUDA path (through the C ABI) against the reference fixtures
and the CPU oracle.

Bars: coreset selections bit-exact; outputs within 1e-5 relative L2 (the
fp32 tolerance); compressor none within 1e-5 of exact softmax attention.
"""

import ctypes

import numpy as np
import pytest
import torch

import streaming_attention_b200 as sa
from conftest import golden_names, load_golden
from oracle import oracle as O
from streaming_attention_b200 import _lib, fast, workloads

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def _run_golden(g, dev):
    m = g["meta"]
    q, k, v = (torch.from_numpy(g[x]).to(dev) for x in "qkv")
    out = sa.fast_article_causal_attention(q, k, v, degree=m["degree"], block_size=m["bs"], scale=m["scale"],
                                           compressor=m["compressor"], seed=m["attn_seed"])
    return out.cpu().numpy()


@pytest.mark.parametrize("name", golden_names())
def test_output_matches_reference_fixture(name, dev):
    g = load_golden(name)
    out = _run_golden(g, dev)
    assert out.shape == g["out"].shape
    err = O.relative_l2(out, g["out"])
    assert err < TOL, f"{name}: rel L2 {err:.3e}"
    if g["meta"]["compressor"] == "none":
        assert O.relative_l2(out, g["exact"]) < TOL


@pytest.mark.parametrize("name", [n for n in golden_names() if load_golden(n)["meta"]["compressor"] != "none"])
def test_coreset_selection_is_bit_exact(name, dev):
    g = load_golden(name)
    m = g["meta"]
    B, H = g["q"].shape[:2]
    for b in range(B):
        for h in range(H):
            k = torch.from_numpy(g["k"][b, h]).to(dev)
            v = torch.from_numpy(g["v"][b, h]).to(dev)
            r = sa.build_completed_block_reps(k, v, block_size=m["bs"], compressor=m["compressor"],
                                              seed=m["attn_seed"] + b * H + h)
            np.testing.assert_array_equal(r.indices.cpu().numpy(), g["rep_idx"][b, h])
            np.testing.assert_array_equal(r.weights.cpu().numpy(), g["rep_w"][b, h])
            idx = r.indices.long()
            assert torch.equal(r.keys, k[idx]) and torch.equal(r.values, v[idx])


def test_batched_selection_matches_per_head(dev):
    g = load_golden("random_ragged")
    m = g["meta"]
    q, k, v = (torch.from_numpy(g[x]).to(dev) for x in "qkv")
    B, H, n, d = q.shape
    _, rep_idx = fast._run(q.reshape(B * H, n, d), k.reshape(B * H, n, d), v.reshape(B * H, n, -1), batch=B,
                           heads=H, degree=2, block_size=m["bs"], scale=m["scale"], compressor=m["compressor"],
                           seed=m["attn_seed"], eps=1e-12, want_rep_idx=True)
    np.testing.assert_array_equal(rep_idx.cpu().numpy(), g["rep_idx"].reshape(B * H, -1))


CASES = [
    # (label, config id, overrides)
    ("cfg3_heads", 3, dict(B=1, H=3, N=2048)),
    ("cfg2_heads", 2, dict(B=1, H=2, N=2048)),
    ("cfg4_heads", 4, dict(B=1, H=2, N=2048)),
    ("cfg5_heads", 5, dict(B=1, H=2, N=3072)),
    ("cfg1", 1, dict()),
    ("odd_dims", 3, dict(B=2, H=1, N=777, d=24, dv=40, block_size=96)),
    ("tiny_dims", 1, dict(N=333, d=3, dv=1, block_size=7)),
    ("d128", 3, dict(B=1, H=1, N=600, d=128, dv=128, block_size=64, radius=6.0)),
]


@pytest.mark.parametrize("label,cfg,over", CASES, ids=[c[0] for c in CASES])
def test_matches_oracle_on_config_shaped_inputs(label, cfg, over, dev):
    c = workloads.config(cfg, **over)
    q, k, v = workloads.make_inputs(c, seed=1)
    out = sa.fast_article_causal_attention(q.to(dev), k.to(dev), v.to(dev), degree=c["degree"],
                                           block_size=c["block_size"], scale=c["scale"],
                                           compressor=c["compressor"], seed=7).cpu().numpy()
    ref, _ = O.fast_attention(q.numpy(), k.numpy(), v.numpy(), degree=c["degree"], block_size=c["block_size"],
                              scale=c["scale"], compressor=c["compressor"], seed=7)
    err = O.relative_l2(out, ref)
    assert err < TOL, f"{label}: rel L2 {err:.3e}"


def test_deterministic(dev):
    c = workloads.config(3, B=1, H=4, N=1024)
    q, k, v = workloads.make_inputs(c, seed=2, device=dev)
    kw = dict(degree=2, block_size=128, compressor="sorted_pair", seed=3)
    a = sa.fast_article_causal_attention(q, k, v, **kw)
    b = sa.fast_article_causal_attention(q, k, v, **kw)
    assert torch.equal(a, b)


def test_host_tensors_stream_through_the_gpu(dev, monkeypatch):
    """CPU inputs (as the reference takes them) run on the GPU in chunks and come
    back on the host; every sequence is computed exactly as in one device call
    (the device call forks its moment scan onto a second stream, the chunks run
    theirs in order: the same arithmetic either way)."""
    c = workloads.config(3, B=2, H=3, N=700)
    q, k, v = workloads.make_inputs(c, seed=5)
    kw = dict(degree=2, block_size=128, compressor="sorted_pair", seed=7)
    ref = sa.fast_article_causal_attention(q.to(dev), k.to(dev), v.to(dev), **kw).cpu()
    # small chunks: 6 sequences in chunks of 2, 2, 1, 1 over the four device slots
    monkeypatch.setattr(fast, "_HOST_CHUNK_BYTES", 700 * (2 * 64 + 64) * 4 * 2)
    out = sa.fast_article_causal_attention(q.pin_memory(), k.pin_memory(), v.pin_memory(), **kw)
    assert out.device.type == "cpu"
    assert torch.equal(out, ref)
    assert _lib.load().sa_moment_fork_enabled() == 1   # the host path gives the thread's setting back
    out2 = sa.fast_article_causal_attention(q, k, v, **kw)   # pageable inputs
    assert torch.equal(out2, ref)
    one = sa.fast_article_causal_attention(q[1, 2], k[1, 2], v[1, 2], seed=12)
    assert torch.equal(one, sa.fast_article_causal_attention(q[1, 2].to(dev), k[1, 2].to(dev), v[1, 2].to(dev),
                                                             seed=12).cpu())


def test_stats_and_two_dim_entry(dev):
    g = load_golden("reftest_shapes_sorted_pair")
    q, k, v = (torch.from_numpy(g[x][0, 0]).to(dev) for x in "qkv")
    out, st = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=32, scale=1.0,
                                               compressor="sorted_pair", low_mode="stream", return_stats=True)
    assert out.shape == (96, 5)
    for key, val in g["meta"]["stats"].items():
        assert getattr(st, key) == val
    assert O.relative_l2(out.cpu().numpy(), g["out"][0, 0]) < TOL


def test_host_inputs_report_the_reference_cpu_stats(dev):
    """Host tensors with low_mode="auto": the stats the reference reports for
    CPU inputs (the streaming low path), the output computed on the GPU."""
    g = load_golden("reftest_shapes_sorted_pair")
    q, k, v = (torch.from_numpy(g[x][0, 0]) for x in "qkv")
    out, st = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=32, scale=1.0,
                                               compressor="sorted_pair", return_stats=True)
    assert out.device.type == "cpu"
    for key, val in g["meta"]["stats"].items():
        assert getattr(st, key) == val, key
    assert O.relative_l2(out.numpy(), g["out"][0, 0]) < TOL


def test_float64_inputs_are_computed_and_returned(dev):
    """float64 inputs: computed in float32 by the kernels, returned as float64."""
    g = load_golden("cfg1_full")
    q, k, v = (torch.from_numpy(g[x]).to(dev).double() for x in "qkv")
    out = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=128, scale=1.0)
    assert out.dtype == torch.float64
    assert O.relative_l2(out.cpu().numpy(), g["out"]) < TOL
    att = sa.ArticleStreamingAttention(32, 32, block_size=16, dtype="float64", device=dev)
    att.update(k[0, 0, 0], v[0, 0, 0])
    y = att.query(q[0, 0, 0])
    assert y.dtype == torch.float64
    assert att.state_size_bytes() == (att.features * 33 + 64) * 8


def test_half_precision_inputs_and_strided_views(dev):
    g = load_golden("cfg1_full")
    q, k, v = (torch.from_numpy(g[x]).to(dev) for x in "qkv")
    # a non-contiguous view of the same data
    qt = q.transpose(2, 3).contiguous().transpose(2, 3)
    out = sa.fast_article_causal_attention(qt, k, v, degree=2, block_size=128, scale=1.0)
    assert O.relative_l2(out.cpu().numpy(), g["out"]) < TOL
    out16 = sa.fast_article_causal_attention(q.half(), k.half(), v.half(), degree=2, block_size=128, scale=1.0)
    assert out16.dtype == torch.float16
    assert O.relative_l2(out16.float().cpu().numpy(), g["out"]) < 2e-3


def test_low_moment_entry_point_through_the_c_abi(dev):
    """sa_low_moments alone against the oracle's low sums over earlier blocks."""
    c = workloads.config(3, B=1, H=2, N=700, block_size=96)
    q, k, v = workloads.make_inputs(c, seed=4)
    bh, n, d, dv = 2, c["N"], c["d"], c["dv"]
    s = workloads.attention_scale(c)
    qd, kd, vd = (x.reshape(bh, n, -1).contiguous().to(dev) for x in (q, k, v))
    low = torch.empty(bh, n, dv + 1, device=dev)
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.sa_low_moments_workspace_size(bh, n, d, dv, 2, 96, ctypes.byref(nbytes)), "ws")
    ws = torch.empty(max(nbytes.value, 256), device=dev, dtype=torch.uint8)
    _lib.call("sa_low_moments", qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), bh, n, d, dv, 2, 96, s,
              low.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert int(ws[:4].view(torch.int32).item()) == 0
    low = low.cpu().numpy()
    for h in range(bh):
        ln, ld = O.low_terms_before_block(q.reshape(bh, n, d)[h].numpy(), k.reshape(bh, n, d)[h].numpy(),
                                          v.reshape(bh, n, dv)[h].numpy(), degree=2, scale=s, bs=96)
        assert O.relative_l2(low[h, :, :dv], ln) < TOL
        assert O.relative_l2(low[h, :, dv], ld) < TOL


def test_c_abi_reports_errors_as_status(dev):
    lib = _lib.load()
    x = torch.zeros(1, 8, 4, device=dev)
    rc = lib.sa_fast_attention(x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 8, 4, 4, 2, 4, 1.0, 1, None, None, None,
                               1e-12, x.data_ptr(), None, x.data_ptr(), 4, None)
    assert rc == _lib.SA_ERR_WORKSPACE
    assert "workspace" in _lib.last_error()


def test_full_size_config2_matches_exact_attention(dev):
    """Config 2 at its full size: the decomposition with compressor none is
    exact attention (classical softmax computed by torch in fp32)."""
    c = workloads.config(2)
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda")
    torch.backends.cuda.matmul.allow_tf32 = False
    out = sa.fast_article_causal_attention(q, k, v, degree=2, block_size=256, compressor="none")
    errs = []
    for b in range(c["B"]):
        exact = sa.classical_causal_attention(q[b].double(), k[b].double(), v[b].double())
        errs.append((torch.linalg.vector_norm(out[b].double() - exact) / torch.linalg.vector_norm(exact)).item())
    assert max(errs) < TOL, errs


@pytest.mark.parametrize("cfg", [3, 4, 5])
def test_full_length_sequences_on_sampled_rows(cfg, dev):
    """Full sequence length of configs 3-5 (fewer heads), checked on sampled
    query rows against the row oracle, plus bit-exact selections."""
    c = workloads.config(cfg, B=1, H=1)
    q, k, v = workloads.make_inputs(c, seed=5, device=dev, generator_device="cuda")
    out = sa.fast_article_causal_attention(q, k, v, degree=c["degree"], block_size=c["block_size"],
                                           scale=c["scale"], compressor=c["compressor"], seed=9)
    n = c["N"]
    rows = np.unique(np.r_[0, 1, c["block_size"], n // 2 + 3, n - c["block_size"] - 1, n - 1,
                           np.random.default_rng(0).integers(0, n, 24)])
    qc, kc, vc = (x[0, 0].cpu().numpy() for x in (q, k, v))
    reps = O.build_reps(kc, c["block_size"], c["compressor"], 9)
    ref = O.fast_attention_rows(qc, kc, vc, rows, degree=c["degree"], block_size=c["block_size"],
                                scale=c["scale"], compressor=c["compressor"], seed=9, reps=reps)
    err = O.relative_l2(out[0, 0].cpu().numpy()[rows], ref)
    assert err < TOL, err
    r = sa.build_completed_block_reps(k[0, 0], v[0, 0], block_size=c["block_size"],
                                      compressor=c["compressor"], seed=9)
    mism = np.flatnonzero(r.indices.cpu().numpy() != reps.idx.astype(np.int32))
    assert mism.size == 0, f"{mism.size} selection mismatches"
