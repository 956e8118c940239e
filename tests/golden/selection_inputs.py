"""Key rows for the full-size coreset selection pins (selections_full.npz).

The pins compare the GPU compressor with the reference's own
``_build_completed_block_reps`` (fast_article_attention.py:364-434) on every
completed block of full-length, config-shaped sequences.  The fixture stores
only the selections (block-local indices) and a SHA-256 of each sequence's
keys; the keys themselves are regenerated here, at fixture time and at test
time, so they must come out bit-identical on any host:

* the draws are ``torch.randn`` on a CPU generator (the same call the
  compressor's direction draws use, which the other fixtures already pin);
* config 3's rows are put on the sphere of radius sqrt(d) / 2 = 4 in float64
  numpy with a fixed sequential sum of squares, a correctly rounded square
  root and division, and one rounding to float32 (no library reduction whose
  order could depend on the host's vector width);
* config 4 (random compressor: the selection does not depend on the keys) and
  config 5 (N(0, 1) keys) use the raw draws.

Only the keys matter for a selection; values are not generated.
"""

from __future__ import annotations

import hashlib

import numpy as np
import torch

# (B, H, N, d, block_size, compressor) of the configurations, and the heads pinned
CONFIGS = {
    3: dict(B=8, H=32, N=8192, d=64, bs=128, compressor="sorted_pair", heads=list(range(256))),
    4: dict(B=4, H=16, N=32768, d=16, bs=256, compressor="random", heads=list(range(64))),
    5: dict(B=1, H=64, N=262144, d=64, bs=256, compressor="sorted_pair", heads=[0, 63]),
}
_SEED_BASE = {3: 3_000_000, 4: 4_000_000, 5: 5_000_000}


def keys_for(cfg_id: int, head: int) -> np.ndarray:
    """float32 [N, d] keys of sequence `head` (flattened b*H + h) of config `cfg_id`."""
    c = CONFIGS[cfg_id]
    g = torch.Generator(device="cpu")
    g.manual_seed(_SEED_BASE[cfg_id] + head)
    k = torch.randn(c["N"], c["d"], generator=g, dtype=torch.float32).numpy()
    if cfg_id != 3:
        return np.ascontiguousarray(k)
    k64 = k.astype(np.float64)
    ss = np.zeros(k64.shape[0], np.float64)
    for a in range(k64.shape[1]):          # fixed order: one IEEE add per column
        ss = ss + k64[:, a] * k64[:, a]
    radius = np.sqrt(float(c["d"])) * 0.5  # 4.0 exactly
    return np.ascontiguousarray((k64 / np.sqrt(ss)[:, None] * radius).astype(np.float32))


def keys_digest(k: np.ndarray) -> np.ndarray:
    """SHA-256 of the key bytes, as 32 uint8."""
    return np.frombuffer(hashlib.sha256(np.ascontiguousarray(k, dtype=np.float32).tobytes()).digest(),
                         dtype=np.uint8).copy()
