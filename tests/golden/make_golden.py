"""Generate the golden fixtures under tests/golden/ by running the reference.

This script imports the reference Python modules (fast_article_attention.py and
streaming_taylor_coreset_attention.py from the PositiveLoss/streaming-attention
checkout) and records, for a set of small seeded cases, the inputs and the
reference's outputs:

* the attention output of ``fast_article_causal_attention``
  (fast_article_attention.py:635-719),
* the coreset selection of every completed block, recovered as global token
  indices by matching the representative key rows returned by
  ``_build_completed_block_reps`` (fast_article_attention.py:365-434) against
  the block's own key rows (keys are continuous random draws, so an exact row
  match is unambiguous),
* the representative weights, and the ``FastArticleStats`` fields;
* for the segment-mean variant (triton_article_attention.py), the reps of
  ``build_segment_mean_coreset`` and, at compress_stride 1, the exact
  attention it reduces to (``segment_*.npz``);
* the selections of every completed block of full-length config-shaped
  sequences (``selections_full.npz``: block-local indices and a digest of the
  keys, which selection_inputs.py regenerates at test time).

Degree 3 is outside the reference fast path (``num_taylor_features`` raises at
fast_article_attention.py:141-142).  For degree 3 the fixture is composed from
reference pieces: the low term from ``TaylorMomentSketch``
(streaming_taylor_coreset_attention.py:229-296, one update+query per token) and
the residual from ``_block_coreset_residual_tail`` (degree-agnostic,
fast_article_attention.py:467-514).

Run it where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path to reference checkout>

The fixtures are written next to this script as ``<case>.npz``.  Nothing at
test time reads the reference; the tests only read the ``.npz`` files.
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(path: str):
    sys.path.insert(0, path)
    fa = importlib.import_module("fast_article_attention")
    st = importlib.import_module("streaming_taylor_coreset_attention")
    return fa, st


def _make_inputs(fa, B, H, n, d, dv, data, radius, seed):
    """Seeded inputs.  2-D (B*H == 1) cases use the fast-path generator
    (fast_article_attention.py:727-758); 4-D cases draw [B,H,N,*] in the same
    q,k,v,rq,rk order (the batched generator of the reference CLI)."""
    if B * H == 1:
        q, k, v = fa._make_data(n, d, dv, radius=radius, data=data,
                                device=torch.device("cpu"), dtype=torch.float32, seed=seed)
        return q[None, None], k[None, None], v[None, None]
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    q = torch.randn(B, H, n, d, generator=g)
    k = torch.randn(B, H, n, d, generator=g)
    v = torch.randn(B, H, n, dv, generator=g)
    if data == "unit_ball":
        qn = torch.clamp(torch.linalg.vector_norm(q, dim=-1, keepdim=True), min=1e-12)
        kn = torch.clamp(torch.linalg.vector_norm(k, dim=-1, keepdim=True), min=1e-12)
        rq = torch.rand(B, H, n, 1, generator=g).pow(1.0 / d) * radius
        rk = torch.rand(B, H, n, 1, generator=g).pow(1.0 / d) * radius
        q = q / qn * rq
        k = k / kn * rk
    elif data == "unit_sphere":
        q = q / torch.clamp(torch.linalg.vector_norm(q, dim=-1, keepdim=True), min=1e-12) * radius
        k = k / torch.clamp(torch.linalg.vector_norm(k, dim=-1, keepdim=True), min=1e-12) * radius
    elif data == "scaled_normal":
        q = q * radius
        k = k * radius
    elif data != "normal":
        raise ValueError(data)
    return q, k, v


def _selected_indices(fa, k, v, bs, compressor, seed):
    """Global token indices and weights of the reference's reps for one head."""
    n = k.shape[0]
    reps = fa._build_completed_block_reps(k, v, block_size=bs, compressor=compressor, seed=seed)
    if compressor == "none":
        return np.arange(n, dtype=np.int32), np.ones(n, dtype=np.float32)
    idx = []
    af = reps.active_from.numpy()
    for r in range(reps.keys.shape[0]):
        end = int(af[r])
        start = end - bs
        blk = k[start:end]
        hit = torch.nonzero((blk == reps.keys[r][None, :]).all(dim=1)).flatten()
        assert hit.numel() >= 1, "representative key not found in its block"
        # duplicates are impossible for continuous draws; take the first match
        idx.append(start + int(hit[0]))
        assert torch.equal(v[start + int(hit[0])], reps.values[r])
    return np.asarray(idx, dtype=np.int32), reps.weights.numpy().astype(np.float32)


def _degree3_reference(fa, st, q, k, v, *, bs, scale, compressor, seed, eps=1e-12):
    """Degree-3 output composed from reference pieces (see module docstring)."""
    n, d = q.shape
    dv = v.shape[1]
    s = float(1.0 / math.sqrt(d) if scale is None else scale)
    sketch = st.TaylorMomentSketch(d, dv, 3, scale=s, device="cpu")
    low_num = torch.empty(n, dv)
    low_den = torch.empty(n)
    for i in range(n):
        sketch.update(k[i], v[i])
        num, den = sketch.query(q[i])
        low_num[i] = num
        low_den[i] = den
    if compressor == "none":
        tail_num, tail_den, _ = fa._full_residual_tail(q, k, v, degree=3, scale=s, query_chunk_size=2048)
    else:
        tail_num, tail_den, _, _ = fa._block_coreset_residual_tail(
            q, k, v, degree=3, block_size=bs, scale=s, compressor=compressor,
            seed=seed, query_chunk_size=2048)
    out = (low_num + tail_num) / torch.clamp((low_den + tail_den)[:, None], min=eps)
    return out, low_num, low_den


CASES = [
    # name, B, H, n, d, dv, degree, bs, scale, compressor, data, radius, seed, attn_seed
    # the reference's own unit tests (test_fast_article_attention.py:10-55)
    dict(name="reftest_exact_none", B=1, H=1, n=64, d=8, dv=7, degree=2, bs=16, scale=1.0,
         compressor="none", data="reftest0", radius=0.1, seed=0, attn_seed=0),
    dict(name="reftest_shapes_sorted_pair", B=1, H=1, n=96, d=12, dv=5, degree=2, bs=32, scale=1.0,
         compressor="sorted_pair", data="reftest1", radius=0.1, seed=1, attn_seed=0),
    # config 1 exactly
    dict(name="cfg1_full", B=1, H=1, n=1024, d=32, dv=32, degree=2, bs=128, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=0, attn_seed=0),
    # config-3-shaped heads at reduced N
    dict(name="cfg3_small", B=1, H=1, n=1024, d=64, dv=64, degree=2, bs=128, scale=None,
         compressor="sorted_pair", data="unit_sphere", radius=4.0, seed=0, attn_seed=0),
    # config-2-shaped (compressor none) at reduced N
    dict(name="cfg2_small", B=1, H=1, n=512, d=64, dv=64, degree=2, bs=256, scale=None,
         compressor="none", data="normal", radius=1.0, seed=0, attn_seed=0),
    # config-5-shaped heads (normal data, bs 256) at reduced N
    dict(name="cfg5_small", B=1, H=1, n=768, d=64, dv=64, degree=2, bs=256, scale=None,
         compressor="sorted_pair", data="normal", radius=1.0, seed=3, attn_seed=0),
    # random compressor, ragged last block, multi-head seeds
    dict(name="random_ragged", B=2, H=2, n=300, d=16, dv=12, degree=2, bs=64, scale=1.0,
         compressor="random", data="unit_ball", radius=1.0, seed=5, attn_seed=7),
    # sorted_pair with odd block size (odd tail, weight 1) and ragged last block
    dict(name="sorted_pair_odd_bs", B=1, H=3, n=200, d=16, dv=8, degree=2, bs=33, scale=0.5,
         compressor="sorted_pair", data="normal", radius=1.0, seed=2, attn_seed=11),
    # block size 2 -> the n<=2 random fallback of the sorted_pair compressor
    dict(name="sorted_pair_bs2", B=1, H=1, n=50, d=8, dv=8, degree=2, bs=2, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=4, attn_seed=0),
    # block size 1 (every completed block keeps its single key at weight 1)
    dict(name="sorted_pair_bs1", B=1, H=1, n=20, d=4, dv=3, degree=2, bs=1, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=4, attn_seed=3),
    # n < bs, n == bs, n == bs + 1, n == 1
    dict(name="edge_n_lt_bs", B=1, H=1, n=40, d=8, dv=8, degree=2, bs=64, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=6, attn_seed=0),
    dict(name="edge_n_eq_bs", B=1, H=1, n=64, d=8, dv=8, degree=2, bs=64, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=6, attn_seed=0),
    dict(name="edge_n_bs_plus1", B=1, H=1, n=65, d=8, dv=8, degree=2, bs=64, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=6, attn_seed=0),
    dict(name="edge_n1", B=1, H=1, n=1, d=8, dv=8, degree=2, bs=64, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=6, attn_seed=0),
    # degrees 0 and 1
    dict(name="degree0", B=1, H=1, n=160, d=16, dv=16, degree=0, bs=32, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=8, attn_seed=0),
    dict(name="degree1", B=1, H=1, n=160, d=16, dv=16, degree=1, bs=32, scale=1.0,
         compressor="random", data="unit_ball", radius=1.0, seed=8, attn_seed=0),
    # degree 3 (extension; composed reference, see _degree3_reference)
    dict(name="degree3_random", B=1, H=2, n=384, d=16, dv=32, degree=3, bs=64, scale=1.0,
         compressor="random", data="unit_ball", radius=1.0, seed=9, attn_seed=0),
    dict(name="degree3_sorted_pair", B=1, H=1, n=200, d=6, dv=5, degree=3, bs=32, scale=1.0,
         compressor="sorted_pair", data="unit_ball", radius=1.0, seed=10, attn_seed=0),
    dict(name="degree3_none", B=1, H=1, n=96, d=6, dv=5, degree=3, bs=16, scale=1.0,
         compressor="none", data="unit_ball", radius=1.0, seed=10, attn_seed=0),
]


def _case_inputs(fa, c):
    if c["data"] == "reftest0":
        # test_fast_article_attention.py:11-15
        torch.manual_seed(0)
        q = torch.randn(c["n"], c["d"]) * 0.1
        k = torch.randn(c["n"], c["d"]) * 0.1
        v = torch.randn(c["n"], c["dv"])
        return q[None, None], k[None, None], v[None, None]
    if c["data"] == "reftest1":
        # test_fast_article_attention.py:33-37
        torch.manual_seed(1)
        q = torch.randn(c["n"], c["d"]) * 0.1
        k = torch.randn(c["n"], c["d"]) * 0.1
        v = torch.randn(c["n"], c["dv"])
        return q[None, None], k[None, None], v[None, None]
    return _make_inputs(fa, c["B"], c["H"], c["n"], c["d"], c["dv"], c["data"], c["radius"], c["seed"])


def make_case(fa, st, c):
    q, k, v = _case_inputs(fa, c)
    B, H, n, d = q.shape
    dv = v.shape[-1]
    out = torch.empty(B, H, n, dv)
    low_num = np.zeros((B, H, n, dv), np.float32)
    low_den = np.zeros((B, H, n), np.float32)
    idx_all, w_all = [], []
    stats = {}
    for b in range(B):
        for h in range(H):
            hs = c["attn_seed"] + b * H + h
            if c["degree"] <= 2:
                o, sts = fa.fast_article_causal_attention(
                    q[b, h], k[b, h], v[b, h], degree=c["degree"], block_size=c["bs"],
                    scale=c["scale"], compressor=c["compressor"], seed=hs,
                    low_mode="stream", return_stats=True)
                out[b, h] = o
                s = fa._attention_scale(c["scale"], d)
                ln, ld, _ = fa.low_degree_taylor_causal_sums(q[b, h], k[b, h], v[b, h], degree=c["degree"],
                                                             scale=s, mode="stream")
                low_num[b, h] = ln.numpy()
                low_den[b, h] = ld.numpy()
                stats = {f: int(getattr(sts, f)) for f in sts.__dataclass_fields__}
            else:
                o, ln, ld = _degree3_reference(fa, st, q[b, h], k[b, h], v[b, h], bs=c["bs"],
                                               scale=c["scale"], compressor=c["compressor"], seed=hs)
                out[b, h] = o
                low_num[b, h] = ln.numpy()
                low_den[b, h] = ld.numpy()
            idx, w = _selected_indices(fa, k[b, h], v[b, h], c["bs"], c["compressor"], hs)
            idx_all.append(idx)
            w_all.append(w)
    # the 4-D entry point must agree with the per-head loop (fast_article_attention.py:683-704)
    if c["degree"] <= 2 and B * H > 1:
        o4 = fa.fast_article_causal_attention(q, k, v, degree=c["degree"], block_size=c["bs"],
                                              scale=c["scale"], compressor=c["compressor"],
                                              seed=c["attn_seed"], low_mode="stream")
        assert torch.equal(o4, out)
    s = fa._attention_scale(c["scale"], d)
    exact = torch.stack([torch.stack([fa.classical_causal_attention(q[b, h], k[b, h], v[b, h], scale=s)
                                      for h in range(H)]) for b in range(B)])
    meta = dict(c)
    meta["stats"] = stats
    arrays = dict(
        q=q.numpy(), k=k.numpy(), v=v.numpy(), out=out.numpy(), exact=exact.numpy(),
        low_num=low_num, low_den=low_den,
        rep_idx=np.stack(idx_all).reshape(B, H, -1) if idx_all and idx_all[0].size else np.zeros((B, H, 0), np.int32),
        rep_w=np.stack(w_all).reshape(B, H, -1) if w_all and w_all[0].size else np.zeros((B, H, 0), np.float32),
        meta=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8),
    )
    np.savez_compressed(os.path.join(HERE, c["name"] + ".npz"), **arrays)
    return arrays


def make_misc(fa, st):
    """Known answers that are not attention outputs."""
    x = torch.tensor([0.0, 1.0, -1.0, 0.5, -2.0, 3.0])
    taylor = {str(t): fa.exp_taylor(x, t).numpy() for t in range(5)}
    feats = {}
    for d, t in [(1, 0), (3, 1), (4, 2), (5, 3), (12, 2), (64, 2), (16, 3), (32, 2)]:
        fm = st.SymmetricTaylorFeatureMap(d, t, device="cpu")
        feats[f"{d}_{t}"] = fm.total_features
    # feature order and key coefficients for a small degree-3 map
    fm = st.SymmetricTaylorFeatureMap(4, 3, device="cpu")
    g = torch.Generator().manual_seed(123)
    key = torch.randn(4, generator=g)
    qry = torch.randn(4, generator=g)
    kf = torch.cat(fm.key_features_by_degree(key)).numpy()
    qf = torch.cat(fm.query_features_by_degree(qry)).numpy()
    # degree-2 fast features (fast_article_attention.py:151-181)
    x2 = torch.randn(3, 5, generator=g)
    f2k = fa._taylor_features_degree012(x2, 2, key_side=True).numpy()
    f2q = fa._taylor_features_degree012(x2, 2, key_side=False).numpy()
    np.savez_compressed(
        os.path.join(HERE, "misc.npz"),
        taylor_x=x.numpy(), **{f"taylor_{t}": v for t, v in taylor.items()},
        feat_counts=np.frombuffer(json.dumps(feats).encode(), dtype=np.uint8),
        fm_key=key.numpy(), fm_qry=qry.numpy(), fm_kf=kf, fm_qf=qf,
        x2=x2.numpy(), f2k=f2k, f2q=f2q,
    )


def make_streaming(fa, st):
    """ArticleStreamingAttention (merge-and-reduce) per-token outputs
    (streaming_taylor_coreset_attention.py:523-616)."""
    out = {}
    for name, comp, n, d, dv, bs, t in [("stream_sorted_pair", "sorted_pair", 100, 4, 3, 8, 2),
                                        ("stream_random", "random", 90, 5, 4, 6, 2),
                                        ("stream_deg3", "sorted_pair", 70, 3, 2, 4, 3),
                                        ("stream_odd_block", "sorted_pair", 75, 6, 5, 5, 2),
                                        ("stream_none", "none", 40, 4, 3, 8, 1)]:
        g = torch.Generator().manual_seed(42)
        q = torch.randn(n, d, generator=g) * 0.5
        k = torch.randn(n, d, generator=g) * 0.5
        v = torch.randn(n, dv, generator=g)
        att = st.ArticleStreamingAttention(d, dv, degree=t, block_size=bs, scale=None,
                                           compressor=comp, device="cpu", seed=17)
        outs, items, sbytes, dens = [], [], [], []
        for i in range(n):
            att.update(k[i], v[i])
            o, s = att.query(q[i], return_stats=True)
            outs.append(o.numpy())
            items.append(s.coreset_items)
            sbytes.append(s.state_bytes)
            dens.append(s.denominator)
        final = att.coreset.items()   # pending buffer, then levels 0, 1, ...
        out[name] = dict(q=q.numpy(), k=k.numpy(), v=v.numpy(), out=np.stack(outs),
                         items=np.asarray(items), state_bytes=np.asarray(sbytes),
                         den=np.asarray(dens, np.float64), final_keys=final.keys.numpy(),
                         final_values=final.values.numpy(), final_weights=final.weights.numpy(),
                         compressions=np.asarray(att.coreset.num_compressions),
                         meta=np.frombuffer(json.dumps(dict(compressor=comp, n=n, d=d, dv=dv, bs=bs,
                                                            degree=t, seed=17)).encode(), dtype=np.uint8))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out[name])


SEGMENT_CASES = [
    # name, (B, H) or None for 2-D, n, d, dv, block_size, compress_stride, key/value dtype
    ("segment_stride2", (1, 2), 300, 16, 8, 32, 2, "float32"),
    ("segment_stride4_ragged", None, 257, 24, 12, 16, 4, "float32"),
    ("segment_stride1_exact", (2, 1), 200, 8, 5, 32, 1, "float32"),
    ("segment_stride3", None, 200, 12, 6, 48, 3, "float32"),
    ("segment_one_rep_per_block", None, 129, 8, 4, 16, 16, "float32"),
    ("segment_no_completed_block", None, 64, 8, 4, 64, 8, "float32"),
    ("segment_float16", (1, 2), 160, 16, 8, 32, 2, "float16"),
    ("segment_bfloat16", None, 140, 16, 16, 16, 4, "bfloat16"),
]


def make_segment(path: str):
    """The segment-mean variant (triton_article_attention.py): the reps of
    ``build_segment_mean_coreset`` (:190-245, plain torch, run here on the CPU)
    and, for compress_stride 1, the exact attention of
    ``torch_classical_causal_attention`` (:123-143), which the variant matches
    up to roundoff (its docstring, :472-474).  The Triton kernel itself needs
    a GPU and Triton; its arithmetic is restated in the oracle."""
    sys.path.insert(0, path)
    tr = importlib.import_module("triton_article_attention")
    for name, bhs, n, d, dv, bs, stride, dt in SEGMENT_CASES:
        g = torch.Generator().manual_seed(1234 + n)
        shape = (bhs[0], bhs[1]) if bhs else ()
        q = torch.randn(*shape, n, d, generator=g) * 0.6
        k = torch.randn(*shape, n, d, generator=g) * 0.6
        v = torch.randn(*shape, n, dv, generator=g)
        dtype = getattr(torch, dt)
        q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
        k3, v3 = (k.reshape(-1, n, d), v.reshape(-1, n, dv))
        rk, rv, m = tr.build_segment_mean_coreset(k3, v3, block_size=bs, compress_stride=stride)
        rec = dict(q=q.float().numpy(), k=k.float().numpy(), v=v.float().numpy(), rep_k=rk.float().numpy(),
                   rep_v=rv.float().numpy(), reps_per_block=np.asarray(m))
        if stride == 1:
            rec["exact"] = tr.torch_classical_causal_attention(q.double(), k.double(), v.double()).numpy()
        rec["meta"] = np.frombuffer(json.dumps(dict(n=n, d=d, dv=dv, bs=bs, stride=stride, dtype=dt,
                                                    batched=bhs is not None)).encode(), dtype=np.uint8)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)


def make_selections(fa) -> None:
    """selections_full.npz: the reference's coreset selection of every completed
    block of full-length config-shaped sequences (all heads of configs 3 and 4,
    two heads of config 5), as block-local indices (uint8: block_size <= 256),
    with a SHA-256 of each sequence's keys (regenerated at test time by
    selection_inputs.keys_for)."""
    sys.path.insert(0, HERE)
    import selection_inputs as si

    rec = {}
    meta = {}
    for cfg_id, c in si.CONFIGS.items():
        N, bs = c["N"], c["bs"]
        nc = (N - 1) // bs
        m = (bs + 1) // 2
        local = np.zeros((len(c["heads"]), nc * m), np.uint8)
        digest = np.zeros((len(c["heads"]), 32), np.uint8)
        for row, head in enumerate(c["heads"]):
            k = si.keys_for(cfg_id, head)
            digest[row] = si.keys_digest(k)
            kt = torch.from_numpy(k)
            idx, _ = _selected_indices(fa, kt, torch.zeros(N, 1), bs, c["compressor"], seed=head)
            starts = (np.arange(nc * m) // m) * bs
            loc = idx.astype(np.int64) - starts
            assert loc.min() >= 0 and loc.max() < bs
            local[row] = loc.astype(np.uint8)
        rec[f"cfg{cfg_id}_local"] = local
        rec[f"cfg{cfg_id}_digest"] = digest
        rec[f"cfg{cfg_id}_heads"] = np.asarray(c["heads"], np.int32)
        meta[str(cfg_id)] = {k_: v_ for k_, v_ in c.items() if k_ != "heads"}
        print(f"config {cfg_id}: {len(c['heads'])} sequences, {nc} blocks each", flush=True)
    rec["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "selections_full.npz"), **rec)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--only", default=None)
    ap.add_argument("--streaming-only", action="store_true")
    ap.add_argument("--segment-only", action="store_true")
    ap.add_argument("--selections-only", action="store_true",
                    help="only selections_full.npz (full-size selection pins)")
    args = ap.parse_args()
    torch.set_num_threads(1)
    if args.selections_only:
        fa, _ = _load_reference(args.reference)
        make_selections(fa)
        print("wrote selections_full")
        return
    if args.segment_only:
        make_segment(args.reference)
        print("wrote segment")
        return
    fa, st = _load_reference(args.reference)
    if args.streaming_only:
        make_streaming(fa, st)
        print("wrote streaming")
        return
    for c in CASES:
        if args.only and c["name"] != args.only:
            continue
        make_case(fa, st, c)
        print("wrote", c["name"])
    if not args.only:
        make_misc(fa, st)
        make_streaming(fa, st)
        make_segment(args.reference)
        make_selections(fa)
        print("wrote misc, streaming, segment, selections_full")


if __name__ == "__main__":
    main()
