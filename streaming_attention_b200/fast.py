"""Drop-in GPU entry points of the reference fast path.

Mirrors ``fast_article_attention.py`` of PositiveLoss/streaming-attention:
same names, keyword arguments, argument checks and messages, return types and
``FastArticleStats`` fields.  All arithmetic runs in the sm_100a kernels of
libsa_b200.so (compressor, block-granular moment scan, residual + combine);
this module only validates, lays tensors out contiguously, builds the
compressor's draw tables and calls the C ABI.  There is no CPU compute path:
CUDA tensors run in place; host (CPU) tensors, as the reference takes them,
are streamed through the GPU in chunks with the copies overlapping the
kernels, and the result comes back on the host; without a CUDA device, or
without the library, the call raises.
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Optional, Tuple, Union

import torch

from . import _lib
from .draws import DrawTables, completed_blocks, draw_tables

Tensor = torch.Tensor

__all__ = [
    "FastArticleStats", "fast_article_causal_attention", "fast_article_causal_attention_single",
    "num_taylor_features", "exp_taylor", "safe_relative_l2", "classical_causal_attention",
    "build_completed_block_reps", "BlockReps",
]


@dataclass(frozen=True)
class FastArticleStats:
    """Field-for-field copy of fast_article_attention.py:293-301."""
    degree: int
    block_size: int
    feature_count: int
    coreset_items: int
    approx_streaming_state_bytes: int
    scratch_low_prefix_bytes: int
    scratch_residual_matrix_bytes: int


@dataclass(frozen=True)
class BlockReps:
    """Reps of the completed blocks (fast_article_attention.py:304-309) plus the
    selected global token indices."""
    keys: Tensor
    values: Tensor
    weights: Tensor
    active_from: Tensor
    indices: Tensor


def _attention_scale(scale: Optional[float], dim: int) -> float:
    """fast_article_attention.py:76-77."""
    return float(1.0 / math.sqrt(dim) if scale is None else scale)


def num_taylor_features(dim: int, degree: int) -> int:
    """Feature count through ``degree`` (fast_article_attention.py:137-148),
    extended to degree 3 (streaming_taylor_coreset_attention.py:155-164)."""
    if degree < 0:
        raise ValueError("degree must be non-negative")
    if degree > _lib.MAX_DEGREE:
        raise NotImplementedError(f"this implementation supports degree 0, 1, 2 or 3 (got {degree})")
    total = 1
    for l in range(1, degree + 1):
        total += math.comb(dim + l - 1, l)
    return total


def exp_taylor(logits: Tensor, degree: int) -> Tensor:
    """Elementwise sum_{r<=degree} logits**r / r! (fast_article_attention.py:95-104).
    A small helper kept for API parity; it is not on the kernel path."""
    if degree < 0:
        raise ValueError("degree must be non-negative")
    out = torch.ones_like(logits)
    term = torch.ones_like(logits)
    for r in range(1, degree + 1):
        term = term * logits / float(r)
        out = out + term
    return out


def safe_relative_l2(a: Tensor, b: Tensor, eps: float = 1e-12) -> float:
    """fast_article_attention.py:107-108."""
    return (torch.linalg.vector_norm(a - b) / torch.clamp(torch.linalg.vector_norm(b), min=eps)).item()


@torch.no_grad()
def classical_causal_attention(q: Tensor, k: Tensor, v: Tensor, *, scale: Optional[float] = None) -> Tensor:
    """Exact causal softmax attention for [..., N, D] tensors (fast_article_attention.py:116-129,
    streaming_taylor_coreset_attention.py:624-638).  A torch helper for comparisons, not the
    product path."""
    if q.shape[:-1] != k.shape[:-1] or v.shape[:-1] != k.shape[:-1]:
        raise ValueError("q and k must match, and v must have the same sequence length")
    s = _attention_scale(scale, q.shape[-1])
    logits = torch.matmul(q, k.transpose(-1, -2)) * s
    n = q.shape[-2]
    mask = torch.ones(n, n, device=q.device, dtype=torch.bool).tril()
    logits = logits.masked_fill(~mask, float("-inf"))
    return torch.matmul(torch.softmax(logits, dim=-1), v)


# ---------------------------------------------------------------------------
# argument checks (mirror the reference's order and messages)
# ---------------------------------------------------------------------------

def _check_single(q: Tensor, k: Tensor, v: Tensor, query_chunk_size: int, block_size: int) -> None:
    """fast_article_attention.py:552-561."""
    if q.ndim != 2 or k.ndim != 2 or v.ndim != 2:
        raise ValueError("q,k,v must have shapes [N,D], [N,D], [N,Dv]")
    if q.shape != k.shape:
        raise ValueError(f"q and k must have the same shape, got {tuple(q.shape)} and {tuple(k.shape)}")
    if v.shape[0] != k.shape[0]:
        raise ValueError("v must have the same sequence length as q/k")
    if query_chunk_size <= 0:
        raise ValueError("query_chunk_size must be positive")
    if block_size <= 0:
        raise ValueError("block_size must be positive")


def _check_modes(n: int, block_size: int, degree: int, compressor: str, low_mode: str) -> None:
    if low_mode not in ("auto", "stream", "prefix"):
        raise ValueError("mode must be one of {'auto', 'stream', 'prefix'}")  # :285
    if degree > _lib.MAX_DEGREE:
        raise NotImplementedError(f"this implementation supports degree 0, 1, 2 or 3 (got {degree})")
    if degree < 0 and n > 0:
        raise ValueError("degree must be non-negative")  # exp_taylor, :97-98
    # the reference rejects an unknown compressor only once a completed block
    # reaches _compress_one_completed_block (:361)
    if compressor not in _lib.COMPRESSORS and completed_blocks(n, block_size) > 0:
        raise ValueError("compressor must be one of {'sorted_pair', 'random', 'none'}")


def _check_dtype(t: Tensor) -> None:
    if not t.dtype.is_floating_point:
        raise ValueError(f"unsupported dtype {t.dtype}: the kernels compute in float32 "
                         "(float32, float64, float16 and bfloat16 inputs are accepted)")


def _check_device(*ts: Tensor) -> torch.device:
    dev = ts[0].device
    if dev.type != "cuda":
        raise ValueError("the B200 kernels need CUDA tensors; move q, k, v to a CUDA device")
    for t in ts:
        if t.device != dev:
            raise ValueError("q, k and v must be on the same device")
        _check_dtype(t)
    return dev


def _stats(n: int, dim: int, dv: int, degree: int, block_size: int, compressor: str, low_mode: str,
           query_chunk_size: int, elem: int, device_type: str = "cuda") -> FastArticleStats:
    """fast_article_attention.py:580-631 for one sequence whose inputs live on
    ``device_type``: ``low_mode="auto"`` resolves to "prefix" for CUDA inputs and
    to "stream" for host inputs, as the reference resolves it (:616)."""
    F = num_taylor_features(dim, degree)
    if compressor == "none":
        items = n
        resid = min(query_chunk_size, n) * n * elem
    else:
        m = (block_size + 1) // 2
        items = completed_blocks(n, block_size) * m
        block_scratch = 0
        for s0 in range(0, n, block_size):
            b = min(s0 + block_size, n) - s0
            block_scratch = max(block_scratch, b * b * elem)
        resid = max(min(query_chunk_size, n) * max(items, 1) * elem, block_scratch)
    approx = F * (1 + dv) * elem + items * (dim + dv + 1) * elem + min(block_size, n) * (dim + dv) * elem
    if low_mode == "auto":
        resolved = "prefix" if device_type == "cuda" else "stream"
    else:
        resolved = low_mode
    low_bytes = F * (1 + dv) * elem if resolved == "stream" else n * F * (1 + dv) * elem
    return FastArticleStats(degree, block_size, F, items, int(approx), int(low_bytes), int(resid))


# ---------------------------------------------------------------------------
# the launch
# ---------------------------------------------------------------------------

def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _run(q3: Tensor, k3: Tensor, v3: Tensor, *, batch: int, heads: int, degree: int, block_size: int,
         scale: float, compressor: str, seed: int, eps: float, want_rep_idx: bool = False,
         head_range: Optional[Tuple[int, int]] = None, out: Optional[Tensor] = None):
    """Forward of bh = q3.shape[0] sequences (contiguous float32 [bh, n, *]).

    head_range selects which flattened (b, h) sequences of the full B*H grid the
    rows of q3 are (their seeds are seed + b*H + h)."""
    bh, n, d = q3.shape
    dv = v3.shape[-1]
    dev = q3.device
    comp = _lib.COMPRESSORS.get(compressor, _lib.COMPRESSORS["sorted_pair"])
    if out is None:
        out = torch.empty(bh, n, dv, device=dev, dtype=torch.float32)
    if bh == 0 or n == 0:
        return out, None
    hr = head_range if head_range is not None else (0, bh)
    tables: DrawTables = draw_tables(seed=seed, batch=batch, heads=heads, n=n, d=d, block_size=block_size,
                                     compressor=compressor if compressor in _lib.COMPRESSORS else "sorted_pair",
                                     device=dev, head_range=hr)
    nc = tables.completed_blocks
    rep_idx = None
    if want_rep_idx and compressor != "none" and nc > 0:
        rep_idx = torch.empty(bh, nc * tables.reps_per_block, device=dev, dtype=torch.int32)
    lib = _lib.load()
    nbytes = _lib.ctypes.c_size_t(0)
    _lib.check(lib.sa_fast_attention_workspace_size(bh, n, d, dv, degree, block_size, comp,
                                                    _lib.ctypes.byref(nbytes)), "sa_fast_attention_workspace_size")
    ws = torch.empty(max(int(nbytes.value), 256), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.sa_fast_attention(
            q3.data_ptr(), k3.data_ptr(), v3.data_ptr(), bh, n, d, dv, degree, block_size, float(scale), comp,
            _ptr(tables.dirs), _ptr(tables.coins), _ptr(tables.perms), float(eps), out.data_ptr(),
            _ptr(rep_idx), ws.data_ptr(), ws.numel(), stream), "sa_fast_attention")
        if _CHECK_STATUS:
            check_device_status(ws)
    return out, rep_idx


_CHECK_STATUS = os.environ.get("SA_CHECK_STATUS", "0") == "1"

# bytes of q, k, v moved per chunk of the host path (about 4 chunks at config 3)
_HOST_CHUNK_BYTES = int(os.environ.get("SA_HOST_CHUNK_BYTES", str(384 << 20)))


# device slots (q, k, v and output buffers of one chunk) and compute streams of the host path
_HOST_SLOTS = 4
_HOST_COMPUTE_STREAMS = 3
_HOST_STREAMS: dict = {}


def _host_streams(dev: torch.device):
    """The host path's streams on `dev` (host->device copies, device->host
    copies, compute), made once per device.  Fresh streams on every call would
    come from torch's rotating stream pool, and the caching allocator keeps the
    blocks freed on one stream for that stream alone: every call would then
    allocate its workspaces anew (and, once device memory fills, release the
    cache with a device-wide synchronisation)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    got = _HOST_STREAMS.get(idx)
    if got is None:
        got = (torch.cuda.Stream(dev), torch.cuda.Stream(dev),
               [torch.cuda.Stream(dev) for _ in range(_HOST_COMPUTE_STREAMS)])
        _HOST_STREAMS[idx] = got
    return got


def _chunk_plan(bh: int, base: int) -> list:
    """Sequences per chunk of the host path: full chunks of `base` while more
    than two are left, then chunks of half the rest (at least base / 8), so that
    the last chunk's kernels and copy-back -- the part no later copy hides --
    are short."""
    sizes, rem, low = [], bh, max(1, base // 8)
    while rem > 0:
        c = base if rem > 2 * base else max(low, -(-rem // 2))
        c = min(c, rem)
        sizes.append(c)
        rem -= c
    return sizes


def _run_host(q3: Tensor, k3: Tensor, v3: Tensor, *, batch: int, heads: int, degree: int, block_size: int,
              scale: float, compressor: str, seed: int, eps: float, head_range: Optional[Tuple[int, int]] = None,
              device: Optional[torch.device] = None) -> Tensor:
    """Forward of host-resident sequences (contiguous float32 [bh, n, *] CPU
    tensors) on the GPU.  The sequences go through in chunks (_chunk_plan):
    chunk i's host->device copy, its kernels and its device->host copy run on
    separate streams, so the copies of one chunk overlap the kernels of its
    neighbours and the two copy directions overlap each other; chunks take
    turns over four device slots and three compute streams, which lets the
    short tail chunks (whose moment scans are latency-bound: one CTA scans a
    whole sequence) run side by side with the chunk before them.  The streams
    are the device's own persistent set (_host_streams), so the caching
    allocator reuses the kernels' workspaces from one call to the next.
    The chunks' forwards run with the moment-scan fork off
    (sa_set_moment_fork): overlapping chunks already fill the SMs a lone
    moment scan leaves idle, and a later chunk's scan at the fork's higher
    priority would delay the earlier chunk's residual and copy-back.
    Pinned inputs give asynchronous copies; the output is a pinned CPU
    tensor."""
    bh, n, d = q3.shape
    dv = v3.shape[-1]
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    out = torch.empty(bh, n, dv, dtype=torch.float32, pin_memory=True)
    if bh == 0 or n == 0:
        return out
    g0 = head_range[0] if head_range is not None else 0
    per_seq = n * (2 * d + dv) * 4
    chunk = max(1, min(bh, _HOST_CHUNK_BYTES // max(per_seq, 1)))
    bounds, s0 = [], 0
    for c in _chunk_plan(bh, chunk):
        bounds.append((s0, s0 + c))
        s0 += c
    lib = _lib.load()
    fork_was = lib.sa_moment_fork_enabled()
    lib.sa_set_moment_fork(0)
    try:
        _stream_chunks(q3, k3, v3, out, bounds, chunk, batch=batch, heads=heads, degree=degree,
                       block_size=block_size, scale=scale, compressor=compressor, seed=seed, eps=eps, g0=g0, dev=dev)
    finally:
        lib.sa_set_moment_fork(fork_was)
    return out


def _stream_chunks(q3: Tensor, k3: Tensor, v3: Tensor, out: Tensor, bounds: list, chunk: int, *, batch: int,
                   heads: int, degree: int, block_size: int, scale: float, compressor: str, seed: int, eps: float,
                   g0: int, dev: torch.device) -> None:
    """The chunk loop of _run_host: copies in, kernels, copies out."""
    bh, n, d = q3.shape
    dv = v3.shape[-1]
    with torch.cuda.device(dev):
        main = torch.cuda.current_stream(dev)
        h2d, d2h, comp = _host_streams(dev)
        for s_ in (h2d, d2h, *comp):
            s_.wait_stream(main)
        nslot = min(_HOST_SLOTS, len(bounds))
        dq = [torch.empty(chunk, n, d, device=dev) for _ in range(nslot)]
        dk = [torch.empty(chunk, n, d, device=dev) for _ in range(nslot)]
        dvv = [torch.empty(chunk, n, dv, device=dev) for _ in range(nslot)]
        dout = [torch.empty(chunk, n, dv, device=dev) for _ in range(nslot)]
        in_ready = [torch.cuda.Event() for _ in range(nslot)]
        computed = [torch.cuda.Event() for _ in range(nslot)]
        copied_out = [torch.cuda.Event() for _ in range(nslot)]
        for i, (s0, s1) in enumerate(bounds):
            slot, cnt = i % nslot, s1 - s0
            if i >= nslot:   # the slot's inputs are free once chunk i - nslot's kernels are done
                h2d.wait_event(computed[slot])
            with torch.cuda.stream(h2d):
                dq[slot][:cnt].copy_(q3[s0:s1], non_blocking=True)
                dk[slot][:cnt].copy_(k3[s0:s1], non_blocking=True)
                dvv[slot][:cnt].copy_(v3[s0:s1], non_blocking=True)
                in_ready[slot].record(h2d)
            cs = comp[i % len(comp)]
            cs.wait_event(in_ready[slot])
            if i >= nslot:   # and its output once chunk i - nslot has been copied back
                cs.wait_event(copied_out[slot])
            with torch.cuda.stream(cs):
                _run(dq[slot][:cnt], dk[slot][:cnt], dvv[slot][:cnt], batch=batch, heads=heads, degree=degree,
                     block_size=block_size, scale=scale, compressor=compressor, seed=seed, eps=eps,
                     head_range=(g0 + s0, g0 + s1), out=dout[slot][:cnt])
                computed[slot].record(cs)
            d2h.wait_event(computed[slot])
            with torch.cuda.stream(d2h):
                out[s0:s1].copy_(dout[slot][:cnt], non_blocking=True)
                copied_out[slot].record(d2h)
        d2h.synchronize()
        for s_ in (h2d, *comp):
            s_.synchronize()


def _host_inputs(*ts: Tensor) -> bool:
    """True when q, k, v all live on the host (the kernels still run on the
    GPU: without a CUDA device this raises)."""
    if not all(t.device.type == "cpu" for t in ts):
        return False
    if not torch.cuda.is_available():
        raise ValueError("the B200 kernels need a CUDA device; none is available")
    for t in ts:
        _check_dtype(t)
    return True


def check_device_status(workspace: Tensor) -> None:
    """Read the launch status word (the first 4 bytes of the workspace) through
    sa_workspace_status: the tensor-core kernels bound every wait and record a
    nonzero code there when one gives up (raised here as SAError).
    Synchronises the current stream."""
    with torch.cuda.device(workspace.device):
        rc = _lib.load().sa_workspace_status(workspace.data_ptr(),
                                             torch.cuda.current_stream(workspace.device).cuda_stream)
    _lib.check(rc, "device status")


def _as_f32(t: Tensor) -> Tensor:
    return t.to(torch.float32).contiguous()


@torch.no_grad()
def fast_article_causal_attention_single(
    q: Tensor, k: Tensor, v: Tensor, *, degree: int = 2, block_size: int = 128, scale: Optional[float] = None,
    compressor: str = "sorted_pair", seed: int = 0, query_chunk_size: int = 2048, low_mode: str = "auto",
    denominator_eps: float = 1e-12, return_stats: bool = False,
) -> Union[Tensor, Tuple[Tensor, FastArticleStats]]:
    """Approximate causal attention for one [N,D] sequence
    (fast_article_attention.py:522-631).  ``query_chunk_size`` and ``low_mode``
    are validated as in the reference and only affect the reported stats."""
    _check_single(q, k, v, query_chunk_size, block_size)
    n, dim = q.shape
    _check_modes(n, block_size, degree, compressor, low_mode)
    s = _attention_scale(scale, dim)
    kw = dict(batch=1, heads=1, degree=degree, block_size=block_size, scale=s, compressor=compressor, seed=seed,
              eps=denominator_eps)
    if _host_inputs(q, k, v):
        out = _run_host(_as_f32(q)[None], _as_f32(k)[None], _as_f32(v)[None], **kw)
    else:
        _check_device(q, k, v)
        out, _ = _run(_as_f32(q)[None], _as_f32(k)[None], _as_f32(v)[None], **kw)
    out = out[0].to(q.dtype)
    if not return_stats:
        return out
    return out, _stats(n, dim, v.shape[-1], degree, block_size, compressor, low_mode, query_chunk_size,
                       q.element_size(), q.device.type)


@torch.no_grad()
def fast_article_causal_attention(
    q: Tensor, k: Tensor, v: Tensor, *, degree: int = 2, block_size: int = 128, scale: Optional[float] = None,
    compressor: str = "sorted_pair", seed: int = 0, query_chunk_size: int = 2048, low_mode: str = "auto",
    denominator_eps: float = 1e-12, return_stats: bool = False,
) -> Union[Tensor, Tuple[Tensor, FastArticleStats]]:
    """Approximate causal attention for [N,D] or [B,H,N,D] tensors
    (fast_article_attention.py:634-719).  Sequence (b, h) uses seed
    ``seed + b*H + h`` (:693).  All B*H sequences run in one set of kernel
    launches."""
    if q.ndim == 2:
        return fast_article_causal_attention_single(
            q, k, v, degree=degree, block_size=block_size, scale=scale, compressor=compressor, seed=seed,
            query_chunk_size=query_chunk_size, low_mode=low_mode, denominator_eps=denominator_eps,
            return_stats=return_stats)
    if q.ndim != 4:
        raise ValueError("q/k/v must be [N,D] or [B,H,N,D]")
    if q.shape != k.shape:
        raise ValueError("q and k must have identical shape [B,H,N,D]")
    if v.shape[:3] != q.shape[:3]:
        raise ValueError("v must have shape [B,H,N,Dv]")
    bsz, heads, n, dim = q.shape
    dv = v.shape[-1]
    if bsz * heads > 0:
        if v.ndim != 4:
            raise ValueError("q,k,v must have shapes [N,D], [N,D], [N,Dv]")
        if query_chunk_size <= 0:
            raise ValueError("query_chunk_size must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        _check_modes(n, block_size, degree, compressor, low_mode)
    bh = bsz * heads
    s = _attention_scale(scale, dim)
    args3 = (_as_f32(q).reshape(bh, n, dim), _as_f32(k).reshape(bh, n, dim), _as_f32(v).reshape(bh, n, dv))
    kw = dict(batch=bsz, heads=heads, degree=degree, block_size=block_size, scale=s, compressor=compressor,
              seed=seed, eps=denominator_eps)
    if _host_inputs(q, k, v):
        # host tensors: streamed through the GPU in chunks, copies overlapping the kernels
        out3 = _run_host(*args3, **kw)
    else:
        _check_device(q, k, v)
        out3, _ = _run(*args3, **kw)
    out = out3.reshape(bsz, heads, n, dv).to(q.dtype)
    if not return_stats:
        return out
    if bh == 0:
        stats = FastArticleStats(degree, block_size, num_taylor_features(dim, degree), 0, 0, 0, 0)
    else:
        stats = _stats(n, dim, dv, degree, block_size, compressor, low_mode, query_chunk_size, q.element_size(),
                       q.device.type)
    return out, stats


@torch.no_grad()
def fast_article_causal_attention_shard(
    q: Tensor, k: Tensor, v: Tensor, *, head_range: Tuple[int, int], batch: int, heads: int, degree: int = 2,
    block_size: int = 128, scale: Optional[float] = None, compressor: str = "sorted_pair", seed: int = 0,
    denominator_eps: float = 1e-12,
) -> Tensor:
    """Forward of the flattened sequences ``head_range = [h0, h1)`` of a
    [batch, heads] grid, for one rank of a head-sharded multi-GPU run.
    q, k, v hold just those sequences ([h1-h0, ..., N, D] with any middle
    shape); sequence f = b*heads + h uses seed ``seed + f`` exactly as in the
    unsharded call, so the union of the shards equals the full result."""
    h0, h1 = head_range
    cnt = h1 - h0
    n, dim = q.shape[-2], q.shape[-1]
    dv = v.shape[-1]
    if q.numel() != cnt * n * dim or k.shape != q.shape or v.numel() != cnt * n * dv:
        raise ValueError("q/k/v must hold exactly the sequences of head_range")
    if not (0 <= h0 <= h1 <= batch * heads):
        raise ValueError("head_range outside the [batch, heads] grid")
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    _check_modes(n, block_size, degree, compressor, "auto")
    s = _attention_scale(scale, dim)
    args3 = (_as_f32(q).reshape(cnt, n, dim), _as_f32(k).reshape(cnt, n, dim), _as_f32(v).reshape(cnt, n, dv))
    kw = dict(batch=batch, heads=heads, degree=degree, block_size=block_size, scale=s, compressor=compressor,
              seed=seed, eps=denominator_eps, head_range=head_range)
    if _host_inputs(q, k, v):
        out3 = _run_host(*args3, **kw)
    else:
        _check_device(q, k, v)
        out3, _ = _run(*args3, **kw)
    return out3.reshape(q.shape[:-1] + (dv,)).to(q.dtype)


@torch.no_grad()
def build_completed_block_reps(k: Tensor, v: Tensor, *, block_size: int, compressor: str, seed: int) -> BlockReps:
    """GPU restatement of _build_completed_block_reps (fast_article_attention.py:364-434)
    for one [N,D] sequence: the reps, weights, active_from, and the selected token indices."""
    if block_size <= 0:
        raise ValueError("block_size must be positive")
    dev = _check_device(k, v)
    n, d = k.shape
    dv = v.shape[-1]
    if compressor == "none":
        pos = torch.arange(n, device=dev)
        return BlockReps(k, v, torch.ones(n, device=dev, dtype=k.dtype), pos, pos.to(torch.int32))
    nc = completed_blocks(n, block_size)
    if nc > 0 and compressor not in _lib.COMPRESSORS:
        raise ValueError("compressor must be one of {'sorted_pair', 'random', 'none'}")
    m = (block_size + 1) // 2
    R = nc * m
    k3, v3 = _as_f32(k)[None], _as_f32(v)[None]
    idx = torch.empty(1, R, device=dev, dtype=torch.int32)
    rk = torch.empty(1, R, d, device=dev)
    rv = torch.empty(1, R, dv, device=dev)
    rw = torch.empty(1, R, device=dev)
    if R > 0:
        t = draw_tables(seed=seed, batch=1, heads=1, n=n, d=d, block_size=block_size, compressor=compressor,
                        device=dev)
        with torch.cuda.device(dev):
            _lib.call("sa_compress_blocks", k3.data_ptr(), v3.data_ptr(), 1, n, d, dv, block_size,
                      _lib.COMPRESSORS[compressor], _ptr(t.dirs), _ptr(t.coins), _ptr(t.perms), idx.data_ptr(),
                      rk.data_ptr(), rv.data_ptr(), rw.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    active = ((torch.arange(R, device=dev) // m + 1) * block_size).to(torch.long)
    return BlockReps(rk[0].to(k.dtype), rv[0].to(v.dtype), rw[0].to(k.dtype), active, idx[0])
