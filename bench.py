"""Benchmark: causal queries/s of the streaming Taylor-moment + block-coreset
attention forward on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3] [--impl ours|reference]

For N > 1 launch under torchrun (one rank per GPU, NCCL); the B*H sequences
of the configuration are split into N contiguous shards with no
communication (every sequence is independent).  Rank 0 prints one JSON line.

A step is one forward of the rank's shard.  ``value`` is timed with the
inputs resident in HBM; ``e2e`` times the public entry point from pinned host
buffers with the host->device copies of q, k, v and the device->host copy of
the output inside the timed region.  Inputs (>= 1.5 GB for the default
configuration) are larger than the 126 MB L2, so no flush is needed between
steps.

``--impl reference`` times the CPU restatement of the reference algorithm
(oracle/oracle.py in float32 numpy; the reference itself is a Python/torch
package that is not present on the GPU host) on bounded samples of the same
workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
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
    ap.add_argument("--cpu-sample-heads", type=int, default=0, help="heads in the CPU sample (0 = auto)")
    ap.add_argument("--bh", type=int, default=0,
                    help="profiling only: replace B*H by this many sequences (B=1) to make a small case")
    return ap.parse_args()


def bench_config(args) -> dict:
    from streaming_attention_b200 import workloads

    if args.bh:
        return workloads.config(args.config, B=1, H=args.bh)
    return workloads.config(args.config)


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


class ClockSampler:
    """nvidia-smi samples of this GPU's clocks while the timed region runs."""

    def __init__(self, device_index: int):
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_rank{device_index}.csv")
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
        except Exception:
            uuid = None
        self.uuid = uuid

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
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
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[6 + j].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def tf32_gemm_peak_tflops(dev: torch.device) -> float:
    """Dense TF32 tensor-core throughput of this GPU, measured as a cuBLAS TF32
    GEMM (8192^3, best of 5): the denominator of the tensor-core kernels."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        a = torch.randn(n, n, device=dev)
        b = torch.randn(n, n, device=dev)
        c = a @ b
        best = float("inf")
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.mm(a, b, out=c)
            e1.record()
            torch.cuda.synchronize(dev)
            best = min(best, e0.elapsed_time(e1) / 1e3)
        del a, b, c
        return 2.0 * n ** 3 / best / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


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


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return {}


_FMA_SRC = r"""
extern "C" __global__ void fma_probe(float* out, int iters) {
  float a0 = threadIdx.x * 1e-7f, a1 = a0 + 1e-6f, a2 = a0 + 2e-6f, a3 = a0 + 3e-6f;
  float a4 = a0 + 4e-6f, a5 = a0 + 5e-6f, a6 = a0 + 6e-6f, a7 = a0 + 7e-6f;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      a0 = fmaf(a0, 0.9999f, 1e-7f); a1 = fmaf(a1, 0.9999f, 1e-7f);
      a2 = fmaf(a2, 0.9999f, 1e-7f); a3 = fmaf(a3, 0.9999f, 1e-7f);
      a4 = fmaf(a4, 0.9999f, 1e-7f); a5 = fmaf(a5, 0.9999f, 1e-7f);
      a6 = fmaf(a6, 0.9999f, 1e-7f); a7 = fmaf(a7, 0.9999f, 1e-7f);
    }
  }
  out[blockIdx.x * blockDim.x + threadIdx.x] = a0 + a1 + a2 + a3 + a4 + a5 + a6 + a7;
}
"""


def fp32_fma_peak_tflops(dev: torch.device) -> float:
    """FP32 FMA-pipe throughput of this GPU, measured with a small NVRTC-compiled
    kernel (8 independent FMA chains per thread, all SMs full)."""
    from cuda.bindings import driver, nvrtc

    prog = nvrtc.nvrtcCreateProgram(_FMA_SRC.encode(), b"fma_probe.cu", 0, [], [])[1]
    opts = [b"--gpu-architecture=sm_100a"]
    if nvrtc.nvrtcCompileProgram(prog, len(opts), opts)[0] != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        return float("nan")
    size = nvrtc.nvrtcGetCUBINSize(prog)[1]
    cubin = b" " * size
    nvrtc.nvrtcGetCUBIN(prog, cubin)
    torch.cuda.synchronize(dev)
    mod = driver.cuModuleLoadData(cubin)[1]
    fn = driver.cuModuleGetFunction(mod, b"fma_probe")[1]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    blocks, threads, iters = sms * 8, 256, 4096
    out = torch.empty(blocks * threads, device=dev)
    import ctypes
    p_out = ctypes.c_void_p(out.data_ptr())
    p_it = ctypes.c_int(iters)
    args = (ctypes.c_void_p * 2)(ctypes.addressof(p_out), ctypes.addressof(p_it))
    stream = torch.cuda.current_stream(dev).cuda_stream
    best = float("inf")
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        driver.cuLaunchKernel(fn, blocks, 1, 1, threads, 1, 1, 0, stream, ctypes.addressof(args), 0)
        e1.record()
        torch.cuda.synchronize(dev)
        best = min(best, e0.elapsed_time(e1) / 1e3)
    driver.cuModuleUnload(mod)
    flops = blocks * threads * iters * 16 * 8 * 2
    return flops / best / 1e12


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

class Staged:
    """The forward as its three C-ABI launches, with CUDA events between them
    so every kernel's device time is measured on the launching stream."""

    def __init__(self, sa_lib, c, q3, k3, v3, head_range, dev):
        from streaming_attention_b200 import draws
        self.lib = sa_lib
        self.c = c
        self.q3, self.k3, self.v3 = q3, k3, v3
        bh, n, d = q3.shape
        dv = v3.shape[-1]
        self.bh, self.n, self.d, self.dv = bh, n, d, dv
        self.scale = float(1.0 / math.sqrt(d) if c["scale"] is None else c["scale"])
        self.comp = {"none": 0, "sorted_pair": 1, "random": 2}[c["compressor"]]
        self.tables = draws.draw_tables(seed=0, batch=c["B"], heads=c["H"], n=n, d=d, block_size=c["block_size"],
                                        compressor=c["compressor"], device=dev, head_range=head_range)
        nc = self.tables.completed_blocks
        m = self.tables.reps_per_block
        R = nc * m if self.comp else 0
        self.R = R
        self.low = torch.empty(bh, n, dv + 1, device=dev)
        self.out = torch.empty(bh, n, dv, device=dev)
        self.rep_idx = torch.empty(bh, max(R, 1), device=dev, dtype=torch.int32)
        self.rk = torch.empty(bh, max(R, 1), d, device=dev)
        self.rv = torch.empty(bh, max(R, 1), dv, device=dev)
        self.rw = torch.empty(bh, max(R, 1), device=dev)
        import ctypes
        nbytes = ctypes.c_size_t(0)
        sa_lib.sa_residual_combine_workspace_size(bh, n, d, dv, c["block_size"], self.comp, ctypes.byref(nbytes))
        self.res_ws = torch.empty(max(int(nbytes.value), 256), device=dev, dtype=torch.uint8)
        mb = ctypes.c_size_t(0)
        sa_lib.sa_low_moments_workspace_size(bh, n, d, dv, c["degree"], c["block_size"], ctypes.byref(mb))
        self.mom_ws = torch.empty(max(int(mb.value), 256), device=dev, dtype=torch.uint8)
        self.times = {"compress": [], "moments": [], "residual": []}
        # the fused entry point (the timed `value`)
        fb = ctypes.c_size_t(0)
        sa_lib.sa_fast_attention_workspace_size(bh, n, d, dv, c["degree"], c["block_size"], self.comp,
                                                ctypes.byref(fb))
        self.ws = torch.empty(max(int(fb.value), 256), device=dev, dtype=torch.uint8)
        tc = int(nbytes.value) > 0
        # kernels per fused forward: (split k, split v,) compress, moments, residual
        self.launches = (2 if tc else 0) + (1 if R else 0) + 2

    def fused(self, stream):
        from streaming_attention_b200 import _lib
        c, t = self.c, self.tables
        ptr = lambda x: None if x is None else x.data_ptr()  # noqa: E731
        _lib.check(self.lib.sa_fast_attention(
            self.q3.data_ptr(), self.k3.data_ptr(), self.v3.data_ptr(), self.bh, self.n, self.d, self.dv,
            c["degree"], c["block_size"], self.scale, self.comp, ptr(t.dirs), ptr(t.coins), ptr(t.perms), 1e-12,
            self.out.data_ptr(), None, self.ws.data_ptr(), self.ws.numel(), stream), "sa_fast_attention")

    def step(self, stream, record=False):
        from streaming_attention_b200 import _lib
        c, t = self.c, self.tables
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            ev[0].record()
        if self.R:
            _lib.check(self.lib.sa_compress_blocks(
                self.k3.data_ptr(), self.v3.data_ptr(), self.bh, self.n, self.d, self.dv, c["block_size"],
                self.comp, t.dirs.data_ptr() if t.dirs is not None else None,
                t.coins.data_ptr() if t.coins is not None else None,
                t.perms.data_ptr() if t.perms is not None else None, self.rep_idx.data_ptr(), self.rk.data_ptr(),
                self.rv.data_ptr(), self.rw.data_ptr(), stream), "compress")
        if record:
            ev[1].record()
        _lib.check(self.lib.sa_low_moments(self.q3.data_ptr(), self.k3.data_ptr(), self.v3.data_ptr(), self.bh,
                                           self.n, self.d, self.dv, c["degree"], c["block_size"], self.scale,
                                           self.low.data_ptr(), self.mom_ws.data_ptr(), self.mom_ws.numel(),
                                           stream), "moments")
        if record:
            ev[2].record()
        rk = self.rk if self.R else self.k3
        rv = self.rv if self.R else self.v3
        _lib.check(self.lib.sa_residual_combine(
            self.q3.data_ptr(), self.k3.data_ptr(), self.v3.data_ptr(), rk.data_ptr(), rv.data_ptr(),
            self.rw.data_ptr() if self.R else None, self.low.data_ptr(), self.bh, self.n, self.d, self.dv,
            c["degree"], c["block_size"], self.comp, self.scale, 1e-12, self.out.data_ptr(), self.res_ws.data_ptr(),
            self.res_ws.numel(), stream), "residual")
        if record:
            ev[3].record()
        return ev

    def collect(self, evs):
        for ev in evs:
            self.times["compress"].append(ev[0].elapsed_time(ev[1]))
            self.times["moments"].append(ev[1].elapsed_time(ev[2]))
            self.times["residual"].append(ev[2].elapsed_time(ev[3]))


def run_nshard(args, rank, world, dev):
    """Config 5 over several GPUs: every sequence split along N (rank r holds
    tokens [r N/P, (r+1) N/P) of all sequences); each step is one collective
    sharded forward (local scan, NCCL all-gather of states and reps, device
    prefix scan, residual)."""
    from streaming_attention_b200 import nshard, workloads

    c = bench_config(args)
    N, P = c["N"], world
    chunks = nshard.owned_chunks(rank, world, "zigzag")
    L = N // (P * len(chunks))
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda")
    q, k, v = (torch.cat([x[:, :, j * L:(j + 1) * L] for j in chunks], dim=2).contiguous() for x in (q, k, v))
    torch.cuda.empty_cache()
    kw = dict(degree=c["degree"], block_size=c["block_size"], scale=c["scale"], compressor=c["compressor"], seed=0)

    def step():
        return nshard.fast_article_causal_attention_nshard(q, k, v, rank=rank, world=world, **kw)

    def barrier():
        torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    with ClockSampler(dev.index) as clk:
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        barrier()
    ms_max = reduce_max(t0.elapsed_time(t1), world, dev)
    out = None
    if rank == 0:
        work = algorithmic_work(c)
        flops = (work["moment_flops"] + work["residual_flops"]) * c["B"] * c["H"]
        tf32_peak = tf32_gemm_peak_tflops(dev)
        achieved = flops * args.steps / (ms_max / 1e3) / 1e12 / world
        out = {
            "metric": METRIC, "value": c["B"] * c["H"] * N * args.steps / (ms_max / 1e3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, CUDA generator)",
            "config": {"workload": workload_name(c, args.config), "B": c["B"], "H": c["H"], "N": N, "d": c["d"],
                       "dv": c["dv"], "degree": c["degree"], "block_size": c["block_size"],
                       "compressor": c["compressor"],
                       "parallelism": f"N sharded over {world} GPU(s) in zig-zag chunk pairs: NCCL all-gather "
                                      "of moment states and reps",
                       "l2": "inputs larger than L2 (no flush needed)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s",
                         "frac": achieved / tf32_peak, "frac_3xtf32": 3 * achieved / tf32_peak,
                         "kernel": "whole sharded forward, per GPU", "traffic": None,
                         "peak_source": "measured cuBLAS TF32 GEMM (8192^3) in this run"},
            "e2e": None, "gpu_launches": None, "clocks": clk.summary(),
        }
    return out, c


def run_ours(args, rank, world, dev):
    import streaming_attention_b200 as sa
    from streaming_attention_b200 import _lib, workloads

    c = bench_config(args)
    bh_total = c["B"] * c["H"]
    if bh_total % world:
        raise SystemExit(f"B*H={bh_total} does not split over {world} GPUs")
    per = bh_total // world
    h0, h1 = rank * per, (rank + 1) * per
    q, k, v = workloads.make_inputs(c, seed=0, device=dev, generator_device="cuda", heads=(h0, h1))
    q3, k3, v3 = q.reshape(per, c["N"], c["d"]), k.reshape(per, c["N"], c["d"]), v.reshape(per, c["N"], c["dv"])
    lib = _lib.load()
    st = Staged(lib, c, q3, k3, v3, (h0, h1), dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    # the headline: the fused entry point, inputs resident in HBM
    for _ in range(args.warmup):
        st.fused(stream)
    barrier()
    with ClockSampler(dev.index) as clk:
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            st.fused(stream)
        t1.record()
        barrier()
    ms = t0.elapsed_time(t1)
    ms_max = reduce_max(ms, world, dev)
    # per-kernel device times: the same kernels through the staged entry points,
    # CUDA events between the launches on the launching stream
    for _ in range(max(1, args.warmup)):
        st.step(stream)
    barrier()
    evs = [st.step(stream, record=True) for _ in range(args.steps)]
    barrier()
    st.collect(evs)

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

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(args.steps):
            e2e_step()
        a1.record()
        barrier()
        e2e_ms = reduce_max(a0.elapsed_time(a1), world, dev)
        e2e = {"value": bh_total * c["N"] * args.steps / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": int((hq.numel() + hk.numel() + hv.numel()) * 4 * world),
               "d2h_bytes_per_step": int(hout.numel() * 4 * world), "ms_per_step": e2e_ms / args.steps}

    # the metric's accuracy part: the timed output against exact causal
    # attention (this library's fp32-accurate flash kernel) on the same inputs,
    # over every rank's heads; and that exact kernel timed on them as a comparator
    accuracy = exact = None
    if not args.no_exact:
        st.fused(stream)
        exact_out = sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=st.scale)[0]
        sums = torch.stack([(st.out - exact_out).double().pow(2).sum(), exact_out.double().pow(2).sum(),
                            (st.out - exact_out).abs().max().double()])
        if world > 1:
            torch.distributed.all_reduce(sums[:2])
            torch.distributed.all_reduce(sums[2:], op=torch.distributed.ReduceOp.MAX)
        accuracy = {"rel_l2_vs_exact": math.sqrt(float(sums[0]) / max(float(sums[1]), 1e-300)),
                    "max_abs_vs_exact": float(sums[2]),
                    "exact": "causal softmax attention, triton_flash_causal_attention (3xTF32 tensor cores)"}
        del exact_out
        for _ in range(2):
            sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=st.scale)
        barrier()
        x0 = torch.cuda.Event(enable_timing=True)
        x1 = torch.cuda.Event(enable_timing=True)
        x_steps = max(1, min(args.steps, 5))
        x0.record()
        for _ in range(x_steps):
            sa.triton_flash_causal_attention(q3[None], k3[None], v3[None], scale=st.scale)
        x1.record()
        barrier()
        x_ms = reduce_max(x0.elapsed_time(x1), world, dev) / x_steps
        exact = {"value": bh_total * c["N"] / (x_ms / 1e3), "unit": UNIT, "ms_per_step": x_ms, "steps": x_steps,
                 "what": "exact causal attention on the same inputs (the comparator, not the headline)"}

    out = None
    if rank == 0:
        work = algorithmic_work(c)
        avg = {k_: statistics.mean(v_) for k_, v_ in st.times.items() if v_}
        dominant = max(avg, key=avg.get)
        peaks = measured_peaks()
        try:
            fma_peak = fp32_fma_peak_tflops(dev)
        except Exception as exc:  # the probe is a measurement aid only
            print(f"fp32 probe failed: {exc!r}", file=sys.stderr)
            fma_peak = float("nan")
        tf32_peak = tf32_gemm_peak_tflops(dev)
        hbm_peak = peaks.get("hbm_gbs", 6650.0)
        # full-size bytes per launch at one GPU; a rank's launch covers per / bh_total of it
        traffic = {k_: v_ * per / bh_total for k_, v_ in profiled_traffic(args.config).items()} if not args.bh else {}
        # The contractions of both tensor-core kernels run on the TF32 tensor pipe
        # with a 3xTF32 split (hi*hi + hi*lo + lo*hi per fp32 product), so their
        # ceiling for fp32-accurate work is a third of the TF32 rate; both
        # fractions are given.
        kernels = {}
        for name, t_ in avg.items():
            kernels[name] = {"ms": t_, "share": t_ / sum(avg.values())}
        for name, key in (("moments", "moment_flops"), ("residual", "residual_flops")):
            tfl = work[key] * per / (avg[name] / 1e3) / 1e12
            kernels[name].update({"tflops": tfl, "frac_tf32": tfl / tf32_peak,
                                  "frac_3xtf32": 3.0 * tfl / tf32_peak})
        kernels["residual"]["frac_fp32_fma"] = kernels["residual"]["tflops"] / fma_peak
        if "compress" in avg and avg["compress"] > 0:
            kernels["compress"]["gbs"] = work["compress_bytes"] * per / (avg["compress"] / 1e3) / 1e9
            kernels["compress"]["frac_hbm"] = kernels["compress"]["gbs"] / hbm_peak
        if dominant == "compress":
            roof = {"bound": "hbm", "achieved": kernels["compress"]["gbs"], "peak": hbm_peak, "unit": "GB/s",
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured copy)"}
        else:
            roof = {"bound": "tensor", "achieved": kernels[dominant]["tflops"], "peak": tf32_peak, "unit": "TFLOP/s",
                    "peak_source": "measured cuBLAS TF32 GEMM (8192^3) in this run; bf16 of measured "
                                   f"{peaks.get('bf16_tflops')} TFLOP/s for context",
                    "frac_3xtf32": kernels[dominant]["frac_3xtf32"]}
        roof["frac"] = roof["achieved"] / roof["peak"] if roof["peak"] else None
        roof["kernel"] = dominant
        roof["traffic"] = traffic.get(dominant)
        roof["algorithmic_per_launch"] = (work["compress_bytes"] if dominant == "compress"
                                          else work["moment_flops" if dominant == "moments" else "residual_flops"]) * per
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
            "e2e": e2e, "gpu_launches": st.launches * args.steps, "accuracy": accuracy, "exact_attention": exact,
            "clocks": clk.summary(), "fp32_fma_peak_tflops": fma_peak, "tf32_gemm_peak_tflops": tf32_peak,
        }
    return out, c


def reduce_max(ms: float, world: int, dev) -> float:
    if world == 1:
        return ms
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU: the oracle port (the reference's algorithm in float32 numpy)
# ---------------------------------------------------------------------------

def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        info = threadpool_info()
        return max([i.get("num_threads", 1) for i in info] or [1])
    except Exception:
        return os.cpu_count() or 1


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
    from streaming_attention_b200 import workloads

    if rank != 0:
        return None
    c = bench_config(args)
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
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu_threads(), "kind": "port", "sample": sample},
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
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    try:
        if args.config == 5 and world > 1:
            line, c = run_nshard(args, rank, world, dev)
        else:
            line, c = run_ours(args, rank, world, dev)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                heads = args.cpu_sample_heads or auto_sample_heads(c, 10.0)
                secs = cpu_sample(c, heads)
                line["cpu_baseline"] = {"value": heads * c["N"] / secs, "unit": UNIT, "cores": cpu_threads(),
                                        "kind": "port",
                                        "sample": f"{heads} of {c['B'] * c['H']} sequences (full N={c['N']}), "
                                                  "oracle/oracle.py in float32"}
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
