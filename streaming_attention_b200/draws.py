"""Host draw tables: the random inputs of the block coreset compressor.

The reference draws, per sequence, from a CPU-or-device ``torch.Generator``
seeded with ``seed + b*H + h`` (fast_article_attention.py:395-396, :693) and,
for every completed block in order, either

* sorted_pair (block of more than 2 keys): ``randn(d)`` normalised to a unit
  direction, then ``rand(block_size // 2)`` pair coins (:339-348), or
* random (and sorted_pair blocks of <= 2 keys): ``randperm(block_size)[:m]``
  (:326-337).

This module replays exactly those calls on a CPU generator and packs the
results into dense tables that the GPU compressor reads:

    dirs  [bh, nc, d]          float32
    coins [bh, nc, bs // 2]    float32
    perms [bh, nc, m]          int32

(nc = (n - 1) // bs completed blocks, m = (bs + 1) // 2).  The tables depend
only on (seed, B, H, n, d, bs, compressor) -- never on the data -- so they are
cached per device, like any other set-up state.  Parity is against the
reference run on CPU: a CUDA generator draws a different stream.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch


@dataclass
class DrawTables:
    dirs: Optional[torch.Tensor]
    coins: Optional[torch.Tensor]
    perms: Optional[torch.Tensor]
    completed_blocks: int
    reps_per_block: int


def completed_blocks(n: int, block_size: int) -> int:
    """Blocks [s, s+bs) with a later query (fast_article_attention.py:403-407)."""
    return (n - 1) // block_size if n > 0 else 0


def _head_draws(seed: int, nc: int, d: int, bs: int, compressor: str):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    m = (bs + 1) // 2
    use_perm = compressor == "random" or bs <= 2
    if use_perm:
        perms = torch.empty(nc, m, dtype=torch.int32)
        for c in range(nc):
            perms[c] = torch.randperm(bs, generator=g)[:m].to(torch.int32)
        return None, None, perms
    dirs = torch.empty(nc, d, dtype=torch.float32)
    coins = torch.empty(nc, bs // 2, dtype=torch.float32)
    for c in range(nc):
        direction = torch.randn(d, generator=g, dtype=torch.float32)
        dirs[c] = direction / torch.clamp(torch.linalg.vector_norm(direction), min=1e-12)
        coins[c] = torch.rand(bs // 2, generator=g, dtype=torch.float32)
    return dirs, coins, None


_cache: Dict[Tuple, DrawTables] = {}
_cache_lock = threading.Lock()
_CACHE_MAX = 16


def draw_tables(*, seed: int, batch: int, heads: int, n: int, d: int, block_size: int, compressor: str,
                device: torch.device, head_range: Optional[Tuple[int, int]] = None,
                cache: bool = True) -> DrawTables:
    """Draw tables for sequences ``head_range = [h0, h1)`` of the flattened
    B*H axis (all of them by default), on ``device``."""
    bh = batch * heads
    h0, h1 = head_range if head_range is not None else (0, bh)
    nc = completed_blocks(n, block_size)
    m = (block_size + 1) // 2
    if compressor == "none" or nc == 0 or h1 <= h0:
        return DrawTables(None, None, None, nc, block_size if compressor == "none" else m)
    key = (int(seed), batch, heads, n, d, block_size, compressor, h0, h1, str(device))
    if cache:
        with _cache_lock:
            hit = _cache.get(key)
        if hit is not None:
            return hit
    use_perm = compressor == "random" or block_size <= 2
    cnt = h1 - h0
    dirs = None if use_perm else torch.empty(cnt, nc, d, dtype=torch.float32)
    coins = None if use_perm else torch.empty(cnt, nc, block_size // 2, dtype=torch.float32)
    perms = torch.empty(cnt, nc, m, dtype=torch.int32) if use_perm else None
    for idx in range(cnt):
        flat = h0 + idx
        b, h = divmod(flat, heads)
        dd, cc, pp = _head_draws(seed + b * heads + h, nc, d, block_size, compressor)
        if use_perm:
            perms[idx] = pp
        else:
            dirs[idx] = dd
            coins[idx] = cc
    pin = device.type == "cuda"

    def to_dev(t):
        if t is None:
            return None
        if pin:
            t = t.pin_memory()
        return t.to(device, non_blocking=True)

    tables = DrawTables(to_dev(dirs), to_dev(coins), to_dev(perms), nc, m)
    if cache:
        with _cache_lock:
            if len(_cache) >= _CACHE_MAX:
                _cache.pop(next(iter(_cache)))
            _cache[key] = tables
    return tables


def clear_cache() -> None:
    with _cache_lock:
        _cache.clear()
