"""One long sequence split along N over several GPUs (one process per GPU).

The reference computes every sequence on one device.  For sequences too long
for that (config 5: 64 sequences of 262144 tokens), rank r of P holds the
contiguous token range [r L, (r + 1) L) of every sequence, L = N / P a whole
number of blocks, and the forward runs in three steps:

1. ``sa_shard_begin``: split the local k, v; compress the shard's completed
   blocks with the draws of their *global* block ids (the draw stream is
   sequential per sequence, so every rank replays the same stream and takes
   its slice); run the moment scan over the shard, which also yields the
   shard's moment state T_r (every local block folded in).
2. exchange: all-gather T_r and the raw reps (NCCL over NVLink between
   processes); each rank keeps the states of the ranks before it and the reps
   of ranks 0..r in global block order.
3. ``sa_shard_end``: a device kernel forms the exclusive prefix sum of the
   earlier states; a frozen moment pass adds phi_q . (earlier state) to every
   local query; the residual runs over the reps of all earlier blocks (global
   block offset) and the exact current block, and divides.

With ``layout="zigzag"`` (the default) the sequence is cut into 2P chunks and
rank r holds chunks r and 2P - 1 - r: the residual work of a chunk grows with
the reps before it, so pairing an early with a late chunk evens the ranks out.
Each chunk is a shard of the 2P-way split; the exchange gathers all chunks.

The moment sums are linear in the state, so the local and the earlier-shard
parts are two sets of partial slices that the residual epilogue adds.  The
result equals the single-GPU forward up to the association of the fp32
state sums (well inside the 1e-5 tolerance); coreset selections are the same.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from . import _lib
from .draws import completed_blocks, draw_tables
from .fast import _attention_scale, _as_f32, _check_device, _check_modes, _ptr

Tensor = torch.Tensor

__all__ = ["ShardPlan", "shard_plan", "owned_chunks", "exchange", "fast_article_causal_attention_nshard",
           "nshard_emulate"]


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    t0: int            # first global token of the shard
    length: int        # tokens per shard (L)
    c_off: int         # global index of the shard's first block
    n_compress: int    # blocks of the shard that are compressed (completed blocks)
    reps_per_rank: int  # rows per sequence each rank contributes to the exchange (Rb)
    m_blk: int         # reps per block (bs for compressor none)


def shard_plan(n_total: int, world: int, rank: int, block_size: int, compressor: str) -> ShardPlan:
    """Token range, block offset and exchange sizes of one rank."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("rank must lie in [0, world)")
    if n_total % world:
        raise ValueError(f"sequence length {n_total} does not split into {world} equal shards")
    L = n_total // world
    if L % block_size:
        raise ValueError(f"shard length {L} is not a whole number of blocks of {block_size}")
    nbl = L // block_size
    c_off = rank * nbl
    if compressor == "none":
        return ShardPlan(rank, world, rank * L, L, c_off, 0, L, block_size)
    m = (block_size + 1) // 2
    n_compress = max(0, min(nbl, completed_blocks(n_total, block_size) - c_off))
    return ShardPlan(rank, world, rank * L, L, c_off, n_compress, nbl * m, m)


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


class _Shard:
    """The two C-ABI calls of one shard, with their shared workspace."""

    def __init__(self, q3: Tensor, k3: Tensor, v3: Tensor, plan: ShardPlan, *, batch: int, heads: int,
                 degree: int, block_size: int, scale: float, compressor: str, seed: int, eps: float,
                 head_range: Optional[Tuple[int, int]] = None):
        self.q3, self.k3, self.v3, self.plan = q3, k3, v3, plan
        self.bh, self.n, self.d = q3.shape
        self.dv = v3.shape[-1]
        self.degree, self.bs, self.scale, self.eps = degree, block_size, scale, eps
        self.compressor = compressor
        self.comp = _lib.COMPRESSORS[compressor]
        self.dev = q3.device
        self.lib = _lib.load()
        floats = _lib.ctypes.c_int64(0)
        _lib.check(self.lib.sa_shard_state_floats(self.bh, self.d, self.dv, degree, _lib.ctypes.byref(floats)),
                   "sa_shard_state_floats")
        self.state_floats = int(floats.value)
        rep_rows = (plan.rank + 1) * plan.reps_per_rank
        nbytes = _lib.ctypes.c_size_t(0)
        _lib.check(self.lib.sa_shard_workspace_size(self.bh, self.n, self.d, self.dv, degree, block_size, rep_rows,
                                                    _lib.ctypes.byref(nbytes)), "sa_shard_workspace_size")
        self.ws = torch.empty(max(int(nbytes.value), 256), device=self.dev, dtype=torch.uint8)
        self.tables = None
        if compressor != "none" and plan.n_compress > 0:
            full = draw_tables(seed=seed, batch=batch, heads=heads, n=plan.world * plan.length, d=self.d,
                               block_size=block_size, compressor=compressor, device=self.dev, head_range=head_range)
            c0, c1 = plan.c_off, plan.c_off + plan.n_compress
            cut = lambda t: None if t is None else t[:, c0:c1].contiguous()  # noqa: E731
            self.tables = (cut(full.dirs), cut(full.coins), cut(full.perms))

    def begin(self) -> Tuple[Tensor, Tensor, Tensor, Tensor, Optional[Tensor]]:
        """Local step: (state [S], rep_k [bh, Rb, d], rep_v [bh, Rb, dv], rep_w [bh, Rb], rep_idx)."""
        p = self.plan
        f32 = dict(device=self.dev, dtype=torch.float32)
        state = torch.empty(self.state_floats, **f32)
        rows = p.n_compress * p.m_blk
        rk = torch.empty(self.bh, rows, self.d, **f32)
        rv = torch.empty(self.bh, rows, self.dv, **f32)
        rw = torch.empty(self.bh, rows, **f32)
        ridx = torch.empty(self.bh, rows, device=self.dev, dtype=torch.int32)
        dirs, coins, perms = self.tables if self.tables is not None else (None, None, None)
        with torch.cuda.device(self.dev):
            _lib.check(self.lib.sa_shard_begin(
                self.q3.data_ptr(), self.k3.data_ptr(), self.v3.data_ptr(), self.bh, self.n, self.d, self.dv,
                self.degree, self.bs, float(self.scale), self.comp, _ptr(dirs), _ptr(coins), _ptr(perms),
                p.n_compress, p.c_off, state.data_ptr(), _ptr(rk) if rows else None, _ptr(rv) if rows else None,
                _ptr(rw) if rows else None, _ptr(ridx) if rows else None, self.ws.data_ptr(), self.ws.numel(),
                _stream(self.dev)), "sa_shard_begin")
        if self.compressor == "none":   # every earlier token is a rep of weight 1
            return state, self.k3, self.v3, torch.ones(self.bh, p.length, **f32), None
        if rows < p.reps_per_rank:       # the sequence's last block is not completed: pad the exchange
            pad = p.reps_per_rank - rows
            rk = torch.cat([rk, torch.zeros(self.bh, pad, self.d, **f32)], 1)
            rv = torch.cat([rv, torch.zeros(self.bh, pad, self.dv, **f32)], 1)
            rw = torch.cat([rw, torch.zeros(self.bh, pad, **f32)], 1)
        return state, rk, rv, rw, ridx

    def end(self, states_before: Tensor, rk: Tensor, rv: Tensor, rw: Tensor, out: Tensor) -> Tensor:
        """Global step, after the exchange: states_before [r, S] of ranks < r;
        rk / rv / rw [bh, (r + 1) Rb, *] the reps of ranks 0..r in block order."""
        p = self.plan
        rows = rk.shape[1]
        with torch.cuda.device(self.dev):
            _lib.check(self.lib.sa_shard_end(
                self.q3.data_ptr(), self.k3.data_ptr(), self.v3.data_ptr(), self.bh, self.n, self.d, self.dv,
                self.degree, self.bs, float(self.scale), self.comp, float(self.eps),
                states_before.data_ptr() if p.rank > 0 else None, p.rank, p.c_off, rk.data_ptr(), rv.data_ptr(),
                rw.data_ptr(), rows, out.data_ptr(), self.ws.data_ptr(), self.ws.numel(), _stream(self.dev)),
                "sa_shard_end")
        return out


def _assemble(parts: Sequence[Tensor]) -> Tensor:
    """Reps of ranks 0..r ([bh, Rb, *] each) as [bh, (r + 1) Rb, *], block order."""
    return torch.cat(list(parts), dim=1).contiguous()


def exchange(state: Tensor, rk: Tensor, rv: Tensor, rw: Tensor, rank: int, world: int,
             group=None) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    """All-gather the shard states and reps over a torch.distributed group (NCCL
    for CUDA tensors); returns (states of ranks < rank [rank, S], and the reps
    of ranks 0..rank assembled in block order)."""
    import torch.distributed as dist

    def gather(t: Tensor) -> List[Tensor]:
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous(), group=group)
        return parts

    states = gather(state)
    ks, vs, ws = gather(rk), gather(rv), gather(rw)
    before = torch.stack(states[:rank]) if rank > 0 else state.new_empty(0, state.numel())
    return before.contiguous(), _assemble(ks[:rank + 1]), _assemble(vs[:rank + 1]), _assemble(ws[:rank + 1])


def owned_chunks(rank: int, world: int, layout: str = "zigzag") -> List[int]:
    """Chunk indices a rank holds.  "contiguous": chunk r of a world-way split.
    "zigzag": chunks r and 2 world - 1 - r of a 2 world-way split, so that every
    rank gets one early and one late chunk (the residual work of a chunk grows
    with the number of reps before it) and the ranks finish together."""
    if layout == "contiguous":
        return [rank]
    if layout == "zigzag":
        return [rank, 2 * world - 1 - rank]
    raise ValueError("layout must be 'contiguous' or 'zigzag'")


def _prep(q: Tensor, k: Tensor, v: Tensor):
    if q.ndim != 4 or k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError("q/k/v must be [B,H,L,D], [B,H,L,D], [B,H,L,Dv] shards")
    B, H, L, d = q.shape
    return B, H, L, d, v.shape[-1]


@torch.no_grad()
def fast_article_causal_attention_nshard(
    q: Tensor, k: Tensor, v: Tensor, *, rank: int, world: int, group=None, layout: str = "zigzag", degree: int = 2,
    block_size: int = 128, scale: Optional[float] = None, compressor: str = "sorted_pair", seed: int = 0,
    denominator_eps: float = 1e-12, return_rep_idx: bool = False,
):
    """This rank's part of fast_article_causal_attention over [B, H, N, *]
    sequences split along N.  q, k, v hold the rank's chunks (see
    ``owned_chunks``) concatenated along N in that order; the result is the
    matching [B, H, len, Dv] slice of the output.  Every rank of ``group``
    calls it collectively.  With ``return_rep_idx`` it also returns, per owned
    chunk in the same order, the global token indices [B*H, rows] of the reps
    that chunk's blocks kept (None for compressor none)."""
    B, H, Lr, d, dv = _prep(q, k, v)
    _check_device(q, k, v)
    chunks = owned_chunks(rank, world, layout)
    nv = world * len(chunks)                     # chunks of the whole sequence
    if Lr % len(chunks):
        raise ValueError("the rank's tokens do not split into its chunks")
    L = Lr // len(chunks)
    _check_modes(L * nv, block_size, degree, compressor, "auto")
    if compressor not in _lib.COMPRESSORS:
        raise ValueError("compressor must be one of {'sorted_pair', 'random', 'none'}")
    bh = B * H
    s = _attention_scale(scale, d)
    shards = []
    for i, j in enumerate(chunks):
        sl = slice(i * L, (i + 1) * L)
        f = lambda x: _as_f32(x[:, :, sl]).reshape(bh, L, -1)  # noqa: E731
        shards.append(_Shard(f(q), f(k), f(v), shard_plan(L * nv, nv, j, block_size, compressor), batch=B,
                             heads=H, degree=degree, block_size=block_size, scale=s, compressor=compressor,
                             seed=seed, eps=denominator_eps))
    begun = [sh.begin() for sh in shards]
    # all-gather every rank's chunks, then index them by chunk
    import torch.distributed as dist

    def gather(t: Tensor) -> List[Tensor]:
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous(), group=group)
        return parts

    per = [gather(torch.stack([b[x] for b in begun])) for x in range(4)]   # state, rep_k, rep_v, rep_w
    owner = {}
    for r in range(world):
        for slot, j in enumerate(owned_chunks(r, world, layout)):
            owner[j] = (r, slot)
    by_chunk = [[per[x][owner[j][0]][owner[j][1]] for j in range(nv)] for x in range(4)]
    outs = []
    for sh, j in zip(shards, chunks):
        before = (torch.stack(by_chunk[0][:j]) if j > 0 else by_chunk[0][0].new_empty(0, sh.state_floats))
        out = torch.empty(bh, L, dv, device=q.device, dtype=torch.float32)
        outs.append(sh.end(before.contiguous(), _assemble(by_chunk[1][:j + 1]), _assemble(by_chunk[2][:j + 1]),
                           _assemble(by_chunk[3][:j + 1]), out))
    full = torch.cat(outs, dim=1).reshape(B, H, Lr, dv).to(q.dtype)
    if return_rep_idx:
        return full, [b[4] for b in begun]
    return full


@torch.no_grad()
def nshard_emulate(q: Tensor, k: Tensor, v: Tensor, *, world: int, degree: int = 2, block_size: int = 128,
                   scale: Optional[float] = None, compressor: str = "sorted_pair", seed: int = 0,
                   denominator_eps: float = 1e-12, return_rep_idx: bool = False):
    """Every rank of a world-way N split run in one process on one GPU, with
    the all-gather replaced by stacking: the sharded arithmetic without NCCL.
    q, k, v are the full [B, H, N, *] tensors; returns the full output."""
    B, H, N, d = q.shape
    dv = v.shape[-1]
    _check_device(q, k, v)
    _check_modes(N, block_size, degree, compressor, "auto")
    s = _attention_scale(scale, d)
    shards, begun = [], []
    for r in range(world):
        plan = shard_plan(N, world, r, block_size, compressor)
        sl = slice(plan.t0, plan.t0 + plan.length)
        f = lambda x: _as_f32(x[:, :, sl]).reshape(B * H, plan.length, -1)  # noqa: E731
        sh = _Shard(f(q), f(k), f(v), plan, batch=B, heads=H, degree=degree, block_size=block_size, scale=s,
                    compressor=compressor, seed=seed, eps=denominator_eps)
        shards.append(sh)
        begun.append(sh.begin())
    outs = []
    for r, sh in enumerate(shards):
        before = torch.stack([b[0] for b in begun[:r]]) if r > 0 else begun[0][0].new_empty(0, sh.state_floats)
        rk = _assemble([b[1] for b in begun[:r + 1]])
        rv = _assemble([b[2] for b in begun[:r + 1]])
        rw = _assemble([b[3] for b in begun[:r + 1]])
        out = torch.empty(B * H, sh.plan.length, dv, device=q.device, dtype=torch.float32)
        outs.append(sh.end(before.contiguous(), rk, rv, rw, out))
    full = torch.cat(outs, dim=1).reshape(B, H, N, dv).to(q.dtype)
    if return_rep_idx:
        idx = [b[4] for b in begun if b[4] is not None and b[4].numel()]
        return full, (torch.cat(idx, dim=1) if idx else None)
    return full
