"""The reference benchmark's CSV, from the GPU path.

    python -m streaming_attention_b200.bench_csv --sweep-n 256 512 1024 --d 32 --dv 32 \\
        --degree 2 --block-size 128 --out results.csv

Writes one row per N with the columns of benchmark_attention.py (:205-229) so
that tooling reading the reference's CSV keeps working:

* ``article_*_ms``: ``fast_article_causal_attention`` on the GPU (the reference
  times its per-token streaming driver there; both compute the same
  approximation family, and this is the path the library provides);
* ``classical_*_ms``: exact causal attention, ``classical_causal_attention``
  (the reference's torch formula, run on the same device);
* ``rel_l2`` / ``max_abs`` / ``mean_abs``: article against classical;
* ``article_*_state_bytes``, ``article_max_coreset_items``: the streaming
  state of ``ArticleStreamingAttention`` fed every key (benchmark_attention.py
  :104-135), from the GPU streaming class;
* ``classical_kv_bytes`` / ``classical_naive_scores_bytes``: as the reference.

Inputs follow the reference's ``make_data`` (:70-101) on the CPU generator,
then move to the GPU.  Timing: median and best of ``--repeats`` wall-clock
runs after one warm-up, synchronised, as in the reference's ``time_call``.
"""

from __future__ import annotations

import argparse
import csv
import math
import statistics
import time
from typing import List, Tuple

import torch

from .fast import classical_causal_attention, fast_article_causal_attention, safe_relative_l2
from .streaming import ArticleStreamingAttention

COLUMNS = ["n", "d", "dv", "degree", "block_size", "compressor", "data", "radius", "scale", "device", "dtype",
           "rel_l2", "max_abs", "mean_abs", "classical_median_ms", "classical_best_ms", "article_median_ms",
           "article_best_ms", "article_final_state_bytes", "article_max_state_bytes", "article_max_coreset_items",
           "classical_kv_bytes", "classical_naive_scores_bytes"]


def make_data(n: int, d: int, dv: int, *, radius: float, data: str, seed: int):
    """benchmark_attention.py:70-101 on the CPU generator."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, d, generator=g)
    k = torch.randn(n, d, generator=g)
    v = torch.randn(n, dv, generator=g)
    if data == "unit_ball":
        qn = torch.clamp(torch.linalg.vector_norm(q, dim=-1, keepdim=True), min=1e-12)
        kn = torch.clamp(torch.linalg.vector_norm(k, dim=-1, keepdim=True), min=1e-12)
        rq = torch.rand(n, 1, generator=g).pow(1.0 / d) * radius
        rk = torch.rand(n, 1, generator=g).pow(1.0 / d) * radius
        q, k = q / qn * rq, k / kn * rk
    elif data == "unit_sphere":
        q = q / torch.clamp(torch.linalg.vector_norm(q, dim=-1, keepdim=True), min=1e-12) * radius
        k = k / torch.clamp(torch.linalg.vector_norm(k, dim=-1, keepdim=True), min=1e-12) * radius
    elif data != "normal":
        raise ValueError("data must be one of {'unit_ball', 'unit_sphere', 'normal'}")
    return q, k, v


def time_call(fn, repeats: int, device: torch.device) -> Tuple[float, float]:
    fn()
    torch.cuda.synchronize(device)
    times: List[float] = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize(device)
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times), min(times)


def state_bytes(k: torch.Tensor, v: torch.Tensor, *, degree: int, block_size: int, scale: float, compressor: str,
                seed: int, device: torch.device) -> Tuple[int, int, int]:
    """(final, max) state bytes and max coreset items over the stream
    (benchmark_attention.py:104-135)."""
    att = ArticleStreamingAttention(k.shape[-1], v.shape[-1], degree=degree, block_size=block_size, scale=scale,
                                    compressor=compressor, device=device, seed=seed)
    kd, vd = k.to(device), v.to(device)
    max_b = max_i = 0
    for i in range(k.shape[0]):
        att.update(kd[i], vd[i])
        max_b = max(max_b, att.state_size_bytes(include_feature_map=False))
        max_i = max(max_i, att.items()[2].numel())
    return att.state_size_bytes(include_feature_map=False), max_b, max_i


def run_one(args, n: int, device: torch.device) -> dict:
    scale = args.scale if args.scale is not None else (1.0 / math.sqrt(args.d) if args.standard_scale else 1.0)
    q, k, v = make_data(n, args.d, args.dv, radius=args.radius, data=args.data, seed=args.seed)
    qd, kd, vd = q.to(device), k.to(device), v.to(device)
    kw = dict(degree=args.degree, block_size=args.block_size, scale=scale, compressor=args.compressor, seed=args.seed)
    with torch.no_grad():
        exact = classical_causal_attention(qd, kd, vd, scale=scale)
        approx = fast_article_causal_attention(qd, kd, vd, **kw)
        rel = safe_relative_l2(approx, exact)
        diff = (approx - exact).abs()
    cm, cb = time_call(lambda: classical_causal_attention(qd, kd, vd, scale=scale), args.repeats, device)
    am, ab = time_call(lambda: fast_article_causal_attention(qd, kd, vd, **kw), args.repeats, device)
    fb, mb, mi = state_bytes(k, v, degree=args.degree, block_size=max(args.block_size, 2), scale=scale,
                             compressor=args.compressor, seed=args.seed, device=device)
    return {"n": n, "d": args.d, "dv": args.dv, "degree": args.degree, "block_size": args.block_size,
            "compressor": args.compressor, "data": args.data, "radius": args.radius, "scale": scale,
            "device": str(device), "dtype": "float32", "rel_l2": rel, "max_abs": diff.max().item(),
            "mean_abs": diff.mean().item(), "classical_median_ms": cm, "classical_best_ms": cb,
            "article_median_ms": am, "article_best_ms": ab, "article_final_state_bytes": fb,
            "article_max_state_bytes": mb, "article_max_coreset_items": mi,
            "classical_kv_bytes": n * (args.d + args.dv) * 4, "classical_naive_scores_bytes": n * n * 4}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--sweep-n", type=int, nargs="+", default=[256, 512, 1024])
    ap.add_argument("--d", type=int, default=32)
    ap.add_argument("--dv", type=int, default=32)
    ap.add_argument("--degree", type=int, default=2)
    ap.add_argument("--block-size", type=int, default=128)
    ap.add_argument("--compressor", default="sorted_pair", choices=["sorted_pair", "random", "none"])
    ap.add_argument("--data", default="unit_ball", choices=["unit_ball", "unit_sphere", "normal"])
    ap.add_argument("--radius", type=float, default=1.0)
    ap.add_argument("--scale", type=float, default=None)
    ap.add_argument("--standard-scale", action="store_true", help="use 1/sqrt(d) when --scale is not given")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--out", default="benchmark_results.csv")
    return ap.parse_args(argv)


def main(argv=None) -> List[dict]:
    args = parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("the GPU benchmark needs a CUDA device")
    device = torch.device("cuda", torch.cuda.current_device())
    rows = [run_one(args, n, device) for n in args.sweep_n]
    with open(args.out, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=COLUMNS)
        w.writeheader()
        w.writerows(rows)
    return rows


if __name__ == "__main__":
    main()
