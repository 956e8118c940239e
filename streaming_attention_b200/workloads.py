"""The benchmark configurations and their seeded synthetic inputs.

The five configurations are the ones the project is measured on (one head of
the reference CLI's default, the exact-decomposition check, a transformer
shape, degree 3, and a long single sequence).  Inputs follow the reference
generators: q, k, v drawn in that order from one seeded generator, then
``unit_ball`` rescales q and k to random radii r*U^(1/d) (drawing rq then rk),
``unit_sphere`` normalises them to a fixed radius, ``normal`` keeps N(0, 1)
(fast_article_attention.py:727-758; the batched variant draws [B,H,N,*]
tensors in the same order).  Generating on a CUDA generator gives the same
distributions with different values; parity against the reference's own
fixtures always uses the CPU generator.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

CONFIGS: Dict[int, dict] = {
    1: dict(B=1, H=1, N=1024, d=32, dv=32, degree=2, block_size=128, scale=1.0, compressor="sorted_pair",
            data="unit_ball", radius=1.0),
    2: dict(B=4, H=8, N=4096, d=64, dv=64, degree=2, block_size=256, scale=None, compressor="none",
            data="normal", radius=1.0),
    3: dict(B=8, H=32, N=8192, d=64, dv=64, degree=2, block_size=128, scale=None, compressor="sorted_pair",
            data="unit_sphere", radius=4.0),
    4: dict(B=4, H=16, N=32768, d=16, dv=64, degree=3, block_size=256, scale=1.0, compressor="random",
            data="unit_ball", radius=1.0),
    5: dict(B=1, H=64, N=262144, d=64, dv=64, degree=2, block_size=256, scale=None, compressor="sorted_pair",
            data="normal", radius=1.0),
}


def config(cfg_id: int, **overrides) -> dict:
    c = dict(CONFIGS[cfg_id])
    c.update(overrides)
    return c


def attention_scale(c: dict) -> float:
    return float(1.0 / math.sqrt(c["d"]) if c["scale"] is None else c["scale"])


@torch.no_grad()
def make_inputs(c: dict, *, seed: int = 0, device: Optional[torch.device] = None,
                generator_device: str = "cpu", heads: Optional[Tuple[int, int]] = None):
    """Seeded q, k, v of shape [B, H, N, d|dv] (float32) for config dict c.

    heads=(h0, h1) draws only a contiguous slice of the flattened B*H axis
    (each sequence then gets its own generator seeded with seed + flat index),
    which lets a rank generate just its shard."""
    B, H, N, d, dv = c["B"], c["H"], c["N"], c["d"], c["dv"]
    gdev = torch.device(generator_device)
    dev = device if device is not None else gdev

    def draw(shape, g):
        q = torch.randn(*shape, d, device=gdev, generator=g)
        k = torch.randn(*shape, d, device=gdev, generator=g)
        v = torch.randn(*shape, dv, device=gdev, generator=g)
        if c["data"] == "unit_ball":
            qn = torch.clamp(torch.linalg.vector_norm(q, dim=-1, keepdim=True), min=1e-12)
            kn = torch.clamp(torch.linalg.vector_norm(k, dim=-1, keepdim=True), min=1e-12)
            rq = torch.rand(*shape, 1, device=gdev, generator=g).pow(1.0 / d) * c["radius"]
            rk = torch.rand(*shape, 1, device=gdev, generator=g).pow(1.0 / d) * c["radius"]
            q = q / qn * rq
            k = k / kn * rk
        elif c["data"] == "unit_sphere":
            q = q / torch.clamp(torch.linalg.vector_norm(q, dim=-1, keepdim=True), min=1e-12) * c["radius"]
            k = k / torch.clamp(torch.linalg.vector_norm(k, dim=-1, keepdim=True), min=1e-12) * c["radius"]
        elif c["data"] != "normal":
            raise ValueError("data must be one of {'unit_ball', 'unit_sphere', 'normal'}")
        return q, k, v

    if heads is None:
        g = torch.Generator(device=gdev)
        g.manual_seed(seed)
        q, k, v = draw((B, H, N), g)
        return q.to(dev), k.to(dev), v.to(dev)
    h0, h1 = heads
    qs, ks, vs = [], [], []
    for flat in range(h0, h1):
        g = torch.Generator(device=gdev)
        g.manual_seed(seed * 1_000_003 + flat)
        q, k, v = draw((1, N), g)
        qs.append(q)
        ks.append(k)
        vs.append(v)
    cat = lambda xs: torch.cat(xs, 0).to(dev)  # noqa: E731
    return cat(qs), cat(ks), cat(vs)
