"""Benchmark: causal queries/s of the streaming Taylor-moment + block-coreset
attention forward on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3] [--impl ours|reference]

For N > 1 launch under torchrun (one rank per GPU, NCCL).  The headline
configuration (config 3 by default) splits its B*H sequences into N
contiguous shards with no communication (every sequence is independent).
Rank 0 prints one JSON line.

A step is one forward of the rank's shard.  ``value`` is timed with the
inputs resident in HBM; ``e2e`` times the public entry point from pinned host
buffers with the host->device copies of q, k, v and the device->host copy of
the output inside the timed region.  Inputs (>= 1.5 GB for the default
configuration) are larger than the 126 MB L2, so no flush is needed between
steps.

Extra keys of the same line (after the headline's timed region):
  ``kernels``         per-stage device times of the timed forward itself
                      (CUDA events recorded by sa_fast_attention between its
                      launches on the launching stream, sa_set_stage_events)
  ``configs``         configs 1, 2 and 4 at full size (heads sharded over the
                      ranks), with rel-L2 against exact attention
  ``nshard_config5``  config 5 (64 sequences of 262144 tokens): on one GPU the
                      single-device forward; on N GPUs the N-sharded forward
                      (zig-zag chunks, NCCL all-gather of moment states and
                      reps, device prefix scan) with in-run parity against
                      the single-device forward on two sequences

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/oracle.py in float32 numpy; the reference itself is a Python/torch
package that is not present on the GPU host) on bounded samples of the same
workload, with every host core.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "causal queries/sec (B·H·N/s)"
UNIT = "queries/s"
CLOCK_FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
# A tf32 tcgen05.mma of M = 128, N = 64, K = 8 issues every 32 cycles per SM
# when run back to back (measured on B200): 2*128*64*8 / 32 = 4096 flop/clk/SM.
RAW_TF32_FLOP_PER_CLK_PER_SM = 4096
STAGES = ("splits", "compress", "moments", "residual")


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 4, 5])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-exact", action="store_true",
                    help="skip the accuracy check against exact attention and the exact kernel's timing")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the extra keys (configs 1/2/4 and config 5)")
    ap.add_argument("--exact-only", action="store_true",
                    help="profiling aid: time only the exact flash kernel on the configuration's inputs")
    ap.add_argument("--cpu-sample-heads", type=int, default=0, help="heads in the CPU sample (0 = auto)")
    ap.add_argument("--bh", type=int, default=0,
                    help="profiling only: replace B*H by this many sequences (B=1) to make a small case")
    ap.add_argument("--profile-nshard", type=int, default=0, metavar="W",
                    help="profiling aid: config 5's 64 sequences at N = 2048 W, split along N into W shards "
                         "run in one process (the all-gather replaced by stacking), once")
    return ap.parse_args()


def bench_config(cfg_id: int, bh: int = 0) -> dict:
    from streaming_attention_b200 import workloads

    if bh:
        return workloads.config(cfg_id, B=1, H=bh)
    return workloads.config(cfg_id)


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def workload_name(c: dict, cfg_id: int) -> str:
    return (f"config{cfg_id}: B={c['B']} H={c['H']} N={c['N']} d={c['d']} dv={c['dv']} degree={c['degree']} "
            f"block_size={c['block_size']} compressor={c['compressor']} data={c['data']}")


def pair_count(n: int, bs: int, m_blk: int) -> int:
    """(query, rep-or-key) pairs the residual kernel evaluates for one sequence."""
    i = np.arange(n, dtype=np.int64)
    c = i // bs
    return int((c * m_blk + (i - c * bs + 1)).sum())


def algorithmic_work(c: dict) -> dict:
    """Per-sequence algorithmic flops / bytes of each kernel."""
    n, d, dv, bs = c["N"], c["d"], c["dv"], c["block_size"]
    t = c["degree"]
    F = sum(1 if l == 0 else math.comb(d + l - 1, l) for l in range(t + 1))
    nc = (n - 1) // bs
    m_blk = bs if c["compressor"] == "none" else (bs + 1) // 2
    pairs = pair_count(n, bs, m_blk)
    R = 0 if c["compressor"] == "none" else nc * m_blk
    return {
        "residual_flops": pairs * (2 * d + 2 * dv + 2),
        # phi_k^T [V, 1] over the keys of completed blocks plus phi_q . [S, s] for
        # every query: 2 F (dv + 1) flops each.  (The intra-block product of a
        # chunked scan, bs (F + dv + 1) per token, is not done here: the current
        # block is exact and belongs to the residual kernel.)
        "moment_flops": 2 * F * (dv + 1) * n + 2 * F * (dv + 1) * nc * bs,
        "compress_bytes": (nc * bs * d * 4 + R * (d + dv) * 4 + R * (d + dv + 2) * 4
                           + nc * (d + bs // 2) * 4) if R else 0,
        "pairs": pairs,
        "features": F,
    }


def launches_per_forward(c: dict) -> int:
    """Kernels sa_fast_attention launches for config c: the k / v operand
    splits, the compressor and the split of its rep values, the moment scan,
    the residual (tensor-core shapes; the CUDA-core shapes launch fewer)."""
    d, dv, bs = c["d"], c["dv"], c["block_size"]
    tc = d <= 64 and dv <= 128 and bs % 4 == 0
    groups = dv <= 64 and d <= 128 and bs % 4 == 0
    compress = c["compressor"] != "none" and c["N"] > bs
    n = (1 if tc else 0) + (1 if (tc or groups) else 0)
    n += (1 + (1 if tc else 0)) if compress else 0
    return n + 2


class ClockSampler:
    """nvidia-smi samples of this GPU's clocks while the timed region runs
    (written to a temporary file, summarised into the JSON line)."""

    def __init__(self, device_index: int):
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix=f"sa_clocks_{device_index}_", suffix=".csv")
        os.close(fd)
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            uuid = None
        self.uuid = uuid

    def __enter__(self):
        try:
            cmd = ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        try:
            rows = [r.split(", ") for r in open(self.path).read().strip().splitlines() if r.count(",") >= 9]
        except Exception:
            rows = []
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[6 + j].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def profiled_traffic(cfg_id: int) -> dict:
    """DRAM bytes per launch of each kernel, from the ncu summary committed for
    this workload (profiles/traffic_config<N>.txt: `kernel bytes` lines)."""
    path = os.path.join(ROOT, "profiles", f"traffic_config{cfg_id}.txt")
    out = {}
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                out[parts[0]] = float(parts[1])
    except OSError:
        pass
    return out


def roofline_peaks() -> dict:
    """Fixed denominators: HBM and dense bf16 from MEASURED_PEAKS.json (the
    driver's copy and cuBLAS measurements on this pool), dense TF32 as half of
    the bf16 rate, and the ceiling of an fp32-accurate 3xTF32 product (three
    TF32 MMAs per product) as a third of that."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
    except Exception:
        p = {}
    if "bf16_tflops" in p:
        bf16, src = float(p["bf16_tflops"]), "of measured"
    else:
        bf16, src = 1590.0, "of fallback"
    hbm = float(p.get("hbm_gbs", 6650.0))
    return {"bf16_tflops": bf16, "tf32_tflops": bf16 / 2, "x3tf32_tflops": bf16 / 6, "hbm_gbs": hbm,
            "source": src, "hbm_source": "of measured" if "hbm_gbs" in p else "of fallback"}


def raw_tf32_tflops(sm_mhz) -> float:
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    mhz = sm_mhz or 1965.0
    return RAW_TF32_FLOP_PER_CLK_PER_SM * sms * mhz * 1e6 / 1e12


def reduce_max(ms: float, world: int, dev) -> float:
    if world == 1:
        return ms
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, dev) -> None:
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)


def timed(fn, steps: int, warmup: int, world: int, dev) -> float:
    """ms per call of fn() on the current stream, max over ranks."""
    for _ in range(warmup):
        fn()
    barrier(world, dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        fn()
    t1.record()
    barrier(world, dev)
    return reduce_max(t0.elapsed_time(t1), world, dev) / steps


def rel_l2_over_ranks(out: torch.Tensor, exact: torch.Tensor, world: int) -> dict:
    sums = torch.stack([(out - exact).double().pow(2).sum(), exact.double().pow(2).sum(),
                        (out - exact).abs().max().double()])
    if world > 1:
        torch.distributed.all_reduce(sums[:2])
        torch.distributed.all_reduce(sums[2:], op=torch.distributed.ReduceOp.MAX)
    return {"rel_l2_vs_exact": math.sqrt(float(sums[0]) / max(float(sums[1]), 1e-300)),
            "max_abs_vs_exact": float(sums[2])}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

class Forward:
    """The fused forward (sa_fast_attention) of one rank's sequences, inputs
    resident in HBM, with its draw tables and workspace made once."""

    def __init__(self, c, q3, k3, v3, head_range, dev):
        from streaming_attention_b200 import _lib, draws
        self.lib = _lib.load()
        self.c = c
        self.q3, self.k3, self.v3 = q3, k3, v3
        bh, n, d = q3.shape
        self.bh, self.n, self.d, self.dv = bh, n, d, v3.shape[-1]
        self.scale = float(1.0 / math.sqrt(d) if c["scale"] is None else c["scale"])
        self.comp = _lib.COMPRESSORS[c["compressor"]]
        self.tables = draws.draw_tables(seed=0, batch=c["B"], heads=c["H"], n=n, d=d, block_size=c["block_size"],
                                        compressor=c["compressor"], device=dev, head_range=head_range)
        self.out = torch.empty(bh, n, self.dv, device=dev)
        import ctypes
        fb = ctypes.c_size_t(0)
        _lib.check(self.lib.sa_fast_attention_workspace_size(bh, n, d, self.dv, c["degree"], c["block_size"],
                                                             self.comp, ctypes.byref(fb)), "workspace size")
        self.ws = torch.empty(max(int(fb.value), 256), device=dev, dtype=torch.uint8)
        self.launches = launches_per_forward(c)

    def __call__(self):
        from streaming_attention_b200 import _lib
        c, t = self.c, self.tables
        ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
        stream = torch.cuda.current_stream().cuda_stream
        _lib.check(self.lib.sa_fast_attention(
            self.q3.data_ptr(), self.k3.data_ptr(), self.v3.data_ptr(), self.bh, self.n, self.d, self.dv,
            self.c["degree"], self.c["block_size"], self.scale, self.comp, ptr(t.dirs), ptr(t.coins), ptr(t.perms),
            1e-12, self.out.data_ptr(), None, self.ws.data_ptr(), self.ws.numel(), stream), "sa_fast_attention")

    def stage_times(self, steps: int) -> dict:
        """Device time of each stage of the fused forward, from CUDA events that
        sa_fast_attention records between its launches on the launching stream."""
        import ctypes
        per = {k: [] for k in STAGES}
        for _ in range(steps):
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            for e in evs:   # torch creates the CUDA event at its first record
                e.record()
            handles = (ctypes.c_void_p * 5)(*[ctypes.c_void_p(e.cuda_event) for e in evs])
            self.lib.sa_set_stage_events(handles, 5)
            try:
                self()
            finally:
                self.lib.sa_set_stage_events(None, 0)
            torch.cuda.synchronize()
            for j, k in enumerate(STAGES):
                per[k].append(evs[j].elapsed_time(evs[j + 1]))
        return {k: statistics.mean(v) for k, v in per.items()}


def kernel_table(c: dict, stage_ms: dict, per: int, peaks: dict, sm_mhz) -> dict:
    work = algorithmic_work(c)
    total = sum(stage_ms.values())
    raw = raw_tf32_tflops(sm_mhz)
    out = {}
    for k, ms in stage_ms.items():
        out[k] = {"ms": ms, "share": ms / total if total else None}
    for name, key in (("moments", "moment_flops"), ("residual", "residual_flops")):
        if stage_ms.get(name, 0) > 0:
            tfl = work[key] * per / (stage_ms[name] / 1e3) / 1e12
            out[name].update({"tflops": tfl, "bound": "tensor (3xTF32)",
                              "frac_3xtf32": tfl / peaks["x3tf32_tflops"],
                              "frac_tf32": tfl / peaks["tf32_tflops"],
                              "frac_3xtf32_raw_rate": 3 * tfl / raw})
    if stage_ms.get("compress", 0) > 0 and work["compress_bytes"]:
        gbs = work["compress_bytes"] * per / (stage_ms["compress"] / 1e3) / 1e9
        out["compress"].update({"gbs": gbs, "bound": "hbm", "frac_hbm": gbs / peaks["hbm_gbs"],
                                "includes": "the compressor and the split of its rep values"})
    out["splits"]["includes"] = "tf32 hi/lo splits of k (rows) and v (transposed)"
    return out


def run_ours(args, rank, world, dev):
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import workloads

    c = bench_config(args.config, args.bh)
    bh_total = c["B"] * c["H"]
    if bh_total % world:
        raise SystemExit(f"B*H={bh_total} does not split over {world} GPUs")
    per = bh_total // world
    h0, h1 = rank * per, (rank + 1) * per
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda", heads=(h0, h1))
    q3, k3, v3 = q.reshape(per, c["N"], c["d"]), k.reshape(per, c["N"], c["d"]), v.reshape(per, c["N"], c["dv"])
    fwd = Forward(c, q3, k3, v3, (h0, h1), dev)
    peaks = roofline_peaks()

    # the headline: the fused entry point, inputs resident in HBM
    for _ in range(args.warmup):
        fwd()
    barrier(world, dev)
    with ClockSampler(dev.index) as clk:
        barrier(world, dev)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            fwd()
        t1.record()
        barrier(world, dev)
    ms_max = reduce_max(t0.elapsed_time(t1), world, dev)
    clocks = clk.summary()
    # per-stage device times of the same fused forward
    stage_ms = fwd.stage_times(max(3, min(args.steps, 10)))

    # end to end through the public entry point, from pinned host buffers
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        hout = torch.empty(q.shape[:-1] + (c["dv"],), dtype=torch.float32).pin_memory()
        kw = dict(degree=c["degree"], block_size=c["block_size"], scale=c["scale"], compressor=c["compressor"],
                  seed=0)
        grid = (c["B"], c["H"], c["N"])

        def e2e_step():
            # the public entry point takes the pinned host tensors as they are and
            # returns the output on the host (chunked, copies overlapping kernels)
            if per == bh_total:
                o = sa.fast_article_causal_attention(hq.view(*grid, c["d"]), hk.view(*grid, c["d"]),
                                                     hv.view(*grid, c["dv"]), **kw)
            else:
                o = sa.fast.fast_article_causal_attention_shard(hq, hk, hv, head_range=(h0, h1), batch=c["B"],
                                                                heads=c["H"], **kw)
            assert o.device.type == "cpu" and o.shape[-1] == c["dv"]

        e2e_ms = timed(e2e_step, args.steps, max(1, args.warmup), world, dev)
        e2e = {"value": bh_total * c["N"] / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * 4 * world),
               "d2h_bytes_per_step": int(hout.numel() * 4 * world), "ms_per_step": e2e_ms}
        del hq, hk, hv, hout

    # the metric's accuracy part: the timed output against exact causal
    # attention (this library's fp32-accurate flash kernel) on the same inputs,
    # over every rank's heads; and that exact kernel timed on them as a comparator
    accuracy = exact = None
    if not args.no_exact:
        fwd()
        exact_out = sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=fwd.scale)[0]
        accuracy = rel_l2_over_ranks(fwd.out, exact_out, world)
        accuracy["exact"] = "causal softmax attention, triton_flash_causal_attention (3xTF32 tensor cores)"
        del exact_out
        x_ms = timed(lambda: sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=fwd.scale),
                     max(1, min(args.steps, 5)), 2, world, dev)
        exact = {"value": bh_total * c["N"] / (x_ms / 1e3), "unit": UNIT, "ms_per_step": x_ms,
                 "what": "exact causal attention on the same inputs (the comparator, not the headline)"}

    out = None
    if rank == 0:
        work = algorithmic_work(c)
        kernels = kernel_table(c, stage_ms, per, peaks, clocks.get("sm_mhz"))
        dominant = max(STAGES, key=lambda s: stage_ms.get(s, 0.0))
        traffic = {k_: v_ * per / bh_total for k_, v_ in profiled_traffic(args.config).items()} if not args.bh else {}
        if dominant in ("compress", "splits"):
            roof = {"bound": "hbm", "achieved": kernels[dominant].get("gbs"), "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peaks['hbm_source']})"}
        else:
            roof = {"bound": "tensor", "achieved": kernels[dominant]["tflops"], "peak": peaks["x3tf32_tflops"],
                    "unit": "TFLOP/s",
                    "peak_source": (f"3xTF32 ceiling: a third of dense TF32, which is half the dense bf16 rate "
                                    f"{peaks['bf16_tflops']} TFLOP/s {peaks['source']} (MEASURED_PEAKS.json)"),
                    "frac_tf32": kernels[dominant]["frac_tf32"],
                    "frac_3xtf32_raw_rate": kernels[dominant]["frac_3xtf32_raw_rate"],
                    "raw_rate_note": "raw tcgen05 tf32 MMA rate (4096 flop/clk/SM, measured) at the sampled "
                                     "median SM clock; its third is the 3xTF32 ceiling of the hardware"}
        roof["frac"] = roof["achieved"] / roof["peak"] if roof.get("achieved") and roof["peak"] else None
        roof["kernel"] = dominant
        roof["traffic"] = traffic.get(dominant)
        roof["algorithmic_per_launch"] = (work["compress_bytes"] if dominant == "compress"
                                          else work["moment_flops" if dominant == "moments" else "residual_flops"]) * per
        roof["kernel_ms"] = stage_ms[dominant]
        value = bh_total * c["N"] * args.steps / (ms_max / 1e3)
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, CUDA generator)",
            "config": {"workload": workload_name(c, args.config), "B": c["B"], "H": c["H"], "N": c["N"],
                       "d": c["d"], "dv": c["dv"], "degree": c["degree"], "block_size": c["block_size"],
                       "compressor": c["compressor"], "parallelism": f"heads sharded over {world} GPU(s)",
                       "l2": "inputs larger than L2 (no flush needed)"},
            "roofline": roof, "kernels": kernels,
            "e2e": e2e, "gpu_launches": fwd.launches * args.steps, "accuracy": accuracy, "exact_attention": exact,
            "clocks": clocks, "peaks": peaks,
        }
    del fwd, q, k, v, q3, k3, v3
    torch.cuda.empty_cache()
    return out, c


def run_exact_only(args, rank, world, dev):
    """Profiling aid: the exact flash kernel alone on the configuration's inputs."""
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import workloads

    c = bench_config(args.config, args.bh)
    per = c["B"] * c["H"] // world
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda",
                                    heads=(rank * per, (rank + 1) * per))
    s = workloads.attention_scale(c)
    q3, k3, v3 = (x.reshape(per, c["N"], -1) for x in (q, k, v))
    ms = timed(lambda: sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=s),
               args.steps, args.warmup, world, dev)
    if rank != 0:
        return None
    return {"metric": "exact causal attention, queries/s", "value": c["B"] * c["H"] * c["N"] / (ms / 1e3),
            "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "config": {"workload": workload_name(c, args.config)}, "what": "triton_flash_causal_attention only"}


def run_profile_nshard(world_emulated: int, dev):
    """Profiling aid: the N-sharded arithmetic of config 5 (64 sequences) at
    N = 2048 W on one GPU, every shard in one process, so that a single-GPU
    profiler sees the shard kernels, the state prefix scan over up to W - 1
    earlier states (45 MB each) among them."""
    from streaming_attention_b200 import nshard, workloads

    c = workloads.config(5, N=2048 * world_emulated)
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda")
    kw = dict(degree=c["degree"], block_size=c["block_size"], scale=c["scale"], compressor=c["compressor"], seed=0)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    nshard.nshard_emulate(q, k, v, world=world_emulated, **kw)
    t1.record()
    torch.cuda.synchronize(dev)
    return {"what": "config 5 N-sharded arithmetic, shards emulated in one process", "N": c["N"],
            "shards": world_emulated, "ms": t0.elapsed_time(t1)}


def run_extra_config(cfg_id: int, rank: int, world: int, dev, steps: int, warmup: int):
    """One of configs 1, 2, 4 at full size, heads sharded over the ranks (config
    1 is a single sequence: measured on one GPU only)."""
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import workloads

    c = bench_config(cfg_id)
    bh_total = c["B"] * c["H"]
    if bh_total % world:
        return {"skipped": f"B*H={bh_total} does not split over {world} GPUs"}
    per = bh_total // world
    h0, h1 = rank * per, (rank + 1) * per
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda", heads=(h0, h1))
    q3, k3, v3 = (x.reshape(per, c["N"], -1) for x in (q, k, v))
    fwd = Forward(c, q3, k3, v3, (h0, h1), dev)
    ms = timed(fwd, steps, warmup, world, dev)
    stage_ms = fwd.stage_times(3)
    exact_out = sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=fwd.scale)[0]
    acc = rel_l2_over_ranks(fwd.out, exact_out, world)
    res = None
    if rank == 0:
        peaks = roofline_peaks()
        res = {"workload": workload_name(c, cfg_id), "value": bh_total * c["N"] / (ms / 1e3), "unit": UNIT,
               "ms_per_step": ms, "steps": steps, "warmup": warmup,
               "parallelism": f"heads sharded over {world} GPU(s)",
               "kernels": kernel_table(c, stage_ms, per, peaks, None), **acc}
    del fwd, q, k, v, q3, k3, v3, exact_out
    torch.cuda.empty_cache()
    return res


def run_config5(rank: int, world: int, dev, steps: int, warmup: int):
    """Config 5: 64 sequences of 262144 tokens.  One GPU: the single-device
    forward.  N GPUs: every sequence split along N into 2N zig-zag chunks
    (NCCL all-gather of moment states and reps, device prefix scan), with
    parity against the single-device forward on sequences 0 and 63."""
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import fast, nshard, workloads

    c = bench_config(5)
    N, bh = c["N"], c["B"] * c["H"]
    kw = dict(degree=c["degree"], block_size=c["block_size"], scale=c["scale"], compressor=c["compressor"], seed=0)
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda")
    s = workloads.attention_scale(c)
    sample = (0, bh - 1)
    if world == 1:
        out_holder = {}

        def step():
            out_holder["o"] = sa.fast_article_causal_attention(q, k, v, **kw)

        ms = timed(step, steps, warmup, world, dev)
        o = out_holder.pop("o")
        exact = sa.triton_flash_causal_attention(q[:, list(sample)], k[:, list(sample)], v[:, list(sample)],
                                                 scale=s)
        acc = rel_l2_over_ranks(o[:, list(sample)], exact, 1)
        del o, exact
        res = {"workload": workload_name(c, 5), "value": bh * N / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
               "steps": steps, "warmup": warmup, "n_gpus": 1, "parallelism": "single device (no N split)",
               "accuracy_sequences": list(sample), **acc}
    else:
        chunks = nshard.owned_chunks(rank, world, "zigzag")
        L = N // (2 * world)
        qs, ks, vs = (torch.cat([x[:, :, j * L:(j + 1) * L] for j in chunks], dim=2).contiguous() for x in (q, k, v))
        holder = {}

        def step():
            holder["r"] = nshard.fast_article_causal_attention_nshard(qs, ks, vs, rank=rank, world=world,
                                                                      return_rep_idx=True, **kw)

        ms = timed(step, steps, warmup, world, dev)
        out_sh, idx_sh = holder.pop("r")
        # parity on the sampled sequences: gather their output chunks and rep
        # indices from every rank (padded to a common size), rebuild them in
        # chunk order on rank 0 and compare with the single-device forward
        m_blk = (c["block_size"] + 1) // 2
        rows_chunk = (L // c["block_size"]) * m_blk
        o_part = out_sh[0, list(sample)].contiguous()                         # [2, 2L, dv]
        i_part = torch.full((2, len(chunks), rows_chunk), -1, device=dev, dtype=torch.int32)
        for slot, ix in enumerate(idx_sh):
            if ix is not None:
                i_part[:, slot, :ix.shape[1]] = ix[list(sample)]
        o_all = [torch.empty_like(o_part) for _ in range(world)]
        i_all = [torch.empty_like(i_part) for _ in range(world)]
        torch.distributed.all_gather(o_all, o_part)
        torch.distributed.all_gather(i_all, i_part)
        res = None
        if rank == 0:
            o_full = torch.empty(2, N, c["dv"], device=dev)
            i_full = []
            owner = {}
            for r in range(world):
                for slot, j in enumerate(nshard.owned_chunks(r, world, "zigzag")):
                    owner[j] = (r, slot)
            for j in range(2 * world):
                r, slot = owner[j]
                o_full[:, j * L:(j + 1) * L] = o_all[r][:, slot * L:(slot + 1) * L]
                i_full.append(i_all[r][:, slot])
            i_full = torch.cat(i_full, dim=1)
            rel, idx_equal = [], True
            for t, hsel in enumerate(sample):
                ref, ridx = fast._run(q[0, hsel][None].contiguous(), k[0, hsel][None].contiguous(),
                                      v[0, hsel][None].contiguous(), batch=1, heads=bh, degree=c["degree"],
                                      block_size=c["block_size"], scale=s, compressor=c["compressor"], seed=0,
                                      eps=1e-12, want_rep_idx=True, head_range=(hsel, hsel + 1))
                rel.append(float(torch.linalg.vector_norm((o_full[t] - ref[0]).double())
                                 / torch.linalg.vector_norm(ref[0].double())))
                got = i_full[t][i_full[t] >= 0]
                idx_equal = idx_equal and torch.equal(got, ridx[0])
            res = {"workload": workload_name(c, 5), "value": bh * N / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
                   "steps": steps, "warmup": warmup, "n_gpus": world,
                   "parallelism": f"N sharded over {world} GPUs in zig-zag chunk pairs: NCCL all-gather of "
                                  "moment states and reps, device prefix scan",
                   "parity": {"sequences": list(sample), "rel_l2_vs_single_device": max(rel),
                              "rep_idx_equal": bool(idx_equal), "tolerance": 1e-5,
                              "ok": bool(max(rel) <= 1e-5 and idx_equal)}}
        del out_sh, idx_sh, qs, ks, vs
    del q, k, v
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# CPU: the oracle port (the reference's algorithm in float32 numpy)
# ---------------------------------------------------------------------------

def host_cpu() -> dict:
    """Host cores the CPU runs may use, and what they are."""
    try:
        avail = len(os.sched_getaffinity(0))
    except Exception:
        avail = os.cpu_count() or 1
    try:
        import psutil
        phys = psutil.cpu_count(logical=False) or avail
    except Exception:
        phys = avail
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"nproc": os.cpu_count(), "available": avail, "physical": phys, "model": model,
            "threads": max(1, min(avail, phys))}


def set_cpu_threads(n: int) -> None:
    """Every host thread pool (torch and numpy's BLAS) to n threads; torchrun
    sets OMP_NUM_THREADS=1 for its workers, which this overrides."""
    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(limits=n)
    except Exception:
        pass


def cpu_sample(c: dict, heads: int, seed: int = 0):
    """Run the oracle port (float32) on `heads` sequences of config c; returns seconds."""
    from oracle import oracle as O
    from streaming_attention_b200 import workloads

    q, k, v = workloads.make_inputs(c, seed=seed, generator_device="cpu", heads=(0, heads))
    q, k, v = q.numpy(), k.numpy(), v.numpy()
    t0 = time.perf_counter()
    for h in range(heads):
        O.fast_attention_single(q[h], k[h], v[h], degree=c["degree"], block_size=c["block_size"], scale=c["scale"],
                                compressor=c["compressor"], seed=h, dtype=np.float32)
    return time.perf_counter() - t0


def auto_sample_heads(c: dict, budget_s: float) -> int:
    """Heads whose CPU time is about budget_s (at least one)."""
    one = cpu_sample(c, 1)
    return max(1, min(c["B"] * c["H"], int(budget_s / max(one, 1e-3))))


def run_reference(args, rank, world):
    if rank != 0:
        return None
    cpu = host_cpu()
    set_cpu_threads(cpu["threads"])
    c = bench_config(args.config, args.bh)
    heads = args.cpu_sample_heads or auto_sample_heads(c, 2.0)
    for _ in range(args.warmup):
        cpu_sample(c, heads)
    times = [cpu_sample(c, heads) for _ in range(args.steps)]
    per_step = statistics.mean(times)
    value = heads * c["N"] / per_step
    sample = f"{heads} of {c['B'] * c['H']} sequences (full N={c['N']}) per step"
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, CPU generator)",
        "config": {"workload": workload_name(c, args.config)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu["threads"], "kind": "port", "sample": sample,
                         "host": cpu},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------

def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        if args.exact_only:
            line = run_exact_only(args, rank, world, dev)
            if rank == 0:
                print(json.dumps(line), flush=True)
            return
        if args.profile_nshard:
            line = run_profile_nshard(args.profile_nshard, dev)
            if rank == 0:
                print(json.dumps(line), flush=True)
            return
        line, c = run_ours(args, rank, world, dev)
        if not args.no_extra and not args.bh:
            xs, xw = max(1, min(args.steps, 5)), max(1, min(args.warmup, 3))
            configs = {}
            for cfg_id in (1, 2, 4):
                if cfg_id == args.config:
                    continue
                if cfg_id == 1 and world > 1:
                    configs["config1"] = {"skipped": "a single sequence: measured on one GPU"}
                    continue
                configs[f"config{cfg_id}"] = run_extra_config(cfg_id, rank, world, dev, xs, xw)
            c5 = run_config5(rank, world, dev, max(1, min(args.steps, 3)), max(1, min(args.warmup, 2)))
            if rank == 0:
                line["configs"] = configs
                line["nshard_config5"] = c5
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                cpu = host_cpu()
                set_cpu_threads(cpu["threads"])
                heads = args.cpu_sample_heads or auto_sample_heads(c, 10.0)
                secs = cpu_sample(c, heads)
                line["cpu_baseline"] = {"value": heads * c["N"] / secs, "unit": UNIT, "cores": cpu["threads"],
                                        "kind": "port", "host": cpu,
                                        "sample": f"{heads} of {c['B'] * c['H']} sequences (full N={c['N']}), "
                                                  "oracle/oracle.py in float32"}
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
