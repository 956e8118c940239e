"""Streaming (decode) attention on the GPU: the reference's
``ArticleStreamingAttention`` (streaming_taylor_coreset_attention.py:523-616).

Same constructor arguments, ``update(key, value)``, ``query(query,
return_stats=...)``, ``state_size_bytes`` and ``length``.  The state is held in
device buffers: the Taylor moment sketch (num [F, dv], den [F], fp32), the
pending block of raw keys / values, and the merge-and-reduce levels.  Every
token costs one moment-update launch and two small copies; a full block
costs one compression launch (plus one per carry), a query two launches.
The arithmetic is in libsa_b200.so (``sa_stream_*``); this module keeps the
level structure (a binary carry, :386-403) and draws the compressor's random
numbers from a CPU ``torch.Generator`` seeded with ``seed``, in the
reference's order (randn(dim) then rand(n // 2) for sorted_pair, randperm(n)
for random or blocks of <= 2 items, :414-470): the same stream the reference
draws on CPU.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Tuple, Union

import torch

from . import _lib

Tensor = torch.Tensor

__all__ = ["ArticleStreamingAttention", "AttentionQueryStats"]

_DTYPES = {
    "float32": torch.float32, "fp32": torch.float32, "float": torch.float32,
    "float64": torch.float64, "fp64": torch.float64, "double": torch.float64,
    "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
    "float16": torch.float16, "fp16": torch.float16, "half": torch.float16,
}


def _resolve_dtype(dtype: Union[str, torch.dtype]) -> torch.dtype:
    """streaming_taylor_coreset_attention.py:45-69."""
    if isinstance(dtype, torch.dtype):
        return dtype
    key = str(dtype).lower()
    if key not in _DTYPES:
        raise ValueError(f"Unsupported dtype {dtype!r}. Use one of {sorted(_DTYPES)}")
    return _DTYPES[key]


@dataclass
class AttentionQueryStats:
    """Field-for-field copy of streaming_taylor_coreset_attention.py:513-520."""
    denominator: float
    low_denominator: float
    tail_denominator: float
    coreset_items: int
    state_bytes: int


@dataclass
class _Items:
    keys: Tensor      # [m, d] float32, device
    values: Tensor    # [m, dv]
    weights: Tensor   # [m]

    @property
    def size(self) -> int:
        return int(self.weights.numel())


class ArticleStreamingAttention:
    """Streaming causal attention via Taylor moments + a merge-and-reduce
    residual coreset, on the GPU.  Call ``update(k_t, v_t)`` then
    ``query(q_t)`` for causal self-attention that includes the current token."""

    def __init__(self, dim: int, value_dim: int, *, degree: int = 2, block_size: int = 128,
                 scale: Optional[float] = None, compressor: str = "sorted_pair",
                 device: Optional[Union[str, torch.device]] = None, dtype: Union[str, torch.dtype] = torch.float32,
                 seed: int = 0, max_monomials: int = 5_000_000, denominator_eps: float = 1e-12) -> None:
        # the reference's checks, in its order: feature map (:137-161), then coreset (:359-360)
        if dim <= 0:
            raise ValueError("dim must be positive")
        if degree < 0:
            raise ValueError("degree must be non-negative")
        total = 0
        for l in range(degree + 1):
            total += 1 if l == 0 else math.comb(dim + l - 1, l)
            if total > max_monomials:
                raise ValueError(
                    f"Requested Taylor feature map has {total:,} monomials through degree {l}, "
                    f"exceeding max_monomials={max_monomials:,}. Lower --degree/--d or raise the limit.")
        if degree > _lib.MAX_DEGREE:
            raise NotImplementedError(f"this implementation supports degree 0, 1, 2 or 3 (got {degree})")
        self.dtype = _resolve_dtype(dtype)
        if block_size < 2:
            raise ValueError("block_size must be at least 2")
        # the state and the arithmetic are float32 whatever ``dtype`` is; outputs
        # are returned in ``dtype`` and state sizes are counted in it
        self.dim = int(dim)
        self.value_dim = int(value_dim)
        self.degree = int(degree)
        self.scale = float(1.0 / math.sqrt(dim) if scale is None else scale)
        self.block_size = int(block_size)
        self.compressor = str(compressor)
        self.seed = int(seed)
        self.denominator_eps = float(denominator_eps)
        if device is None:
            if not torch.cuda.is_available():
                raise ValueError("the B200 kernels need a CUDA device; none is available")
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the streaming state lives on a CUDA device; pass device='cuda'")
        self.features = total
        self._lib = _lib.load()
        f32 = dict(device=self.device, dtype=torch.float32)
        self._num = torch.zeros(total, value_dim, **f32)
        self._den = torch.zeros(total, **f32)
        self._bk = torch.empty(block_size, dim, **f32)
        self._bv = torch.empty(block_size, value_dim, **f32)
        self._nbuf = 0
        self.levels: List[Optional[_Items]] = []
        self._packed = _Items(torch.empty(0, dim, **f32), torch.empty(0, value_dim, **f32), torch.empty(0, **f32))
        self._generator = torch.Generator(device="cpu")
        self._generator.manual_seed(self.seed)
        self._length = 0
        self.num_compressions = 0
        nbytes = _lib.ctypes.c_size_t(0)
        _lib.check(self._lib.sa_stream_query_workspace_size(dim, value_dim, degree, _lib.ctypes.byref(nbytes)),
                   "sa_stream_query_workspace_size")
        self._ws = torch.empty(max(int(nbytes.value), 16), device=self.device, dtype=torch.uint8)
        self._out = torch.empty(value_dim, **f32)
        self._dens = torch.empty(3, **f32)

    # ------------------------------------------------------------------ state
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def _vec(self, x: Tensor, n: int, what: str) -> Tensor:
        x = x.to(device=self.device)
        if x.shape != (n,):
            raise ValueError(f"{what} must have shape [{n}], got {tuple(x.shape)}")
        return x.to(torch.float32).contiguous()

    def _compress(self, block: _Items) -> _Items:
        """MergeReduceCoreset._compress (:414-470) with the reference's draws."""
        if self.compressor == "none" or block.size <= 1:
            return block
        if self.compressor not in ("random", "sorted_pair"):
            raise ValueError("compressor must be one of {'sorted_pair', 'random', 'none'}")
        n = block.size
        m = (n + 1) // 2
        g = self._generator
        direction = coins = perm = None
        if self.compressor == "random" or n <= 2:
            perm = torch.randperm(n, generator=g)[:m].to(torch.int32).to(self.device)
            comp = _lib.COMPRESSORS["random"]
        else:
            d = torch.randn(self.dim, generator=g, dtype=torch.float32)
            d = d / torch.clamp(torch.linalg.vector_norm(d), min=1e-12)
            u = torch.rand(n // 2, generator=g, dtype=torch.float32)
            direction, coins = d.to(self.device), u.to(self.device)
            comp = _lib.COMPRESSORS["sorted_pair"]
        f32 = dict(device=self.device, dtype=torch.float32)
        out = _Items(torch.empty(m, self.dim, **f32), torch.empty(m, self.value_dim, **f32), torch.empty(m, **f32))
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        with torch.cuda.device(self.device):
            _lib.check(self._lib.sa_stream_compress(
                block.keys.data_ptr(), block.values.data_ptr(), block.weights.data_ptr(), n, self.dim,
                self.value_dim, comp, ptr(direction), ptr(coins), ptr(perm), out.keys.data_ptr(),
                out.values.data_ptr(), out.weights.data_ptr(), self._stream()), "sa_stream_compress")
        self.num_compressions += 1
        return out

    def _insert_level(self, level: int, block: _Items) -> None:
        """Binary carry (:386-403): an occupied level merges (old items first)
        and the compressed merge moves one level up."""
        while len(self.levels) <= level:
            self.levels.append(None)
        if self.levels[level] is None:
            self.levels[level] = block
            return
        old = self.levels[level]
        merged = _Items(torch.cat([old.keys, block.keys]), torch.cat([old.values, block.values]),
                        torch.cat([old.weights, block.weights]))
        self.levels[level] = None
        self._insert_level(level + 1, self._compress(merged))

    def _repack(self) -> None:
        parts = [b for b in self.levels if b is not None and b.size > 0]
        if parts:
            self._packed = _Items(torch.cat([b.keys for b in parts]), torch.cat([b.values for b in parts]),
                                  torch.cat([b.weights for b in parts]))
        else:
            self._packed = _Items(self._packed.keys[:0], self._packed.values[:0], self._packed.weights[:0])

    # ------------------------------------------------------------------ API
    @torch.no_grad()
    def update(self, key: Tensor, value: Tensor) -> None:
        """TaylorMomentSketch.update + MergeReduceCoreset.append (:262-279, :374-384)."""
        k = self._vec(key, self.dim, "key")
        v = self._vec(value, self.value_dim, "value")
        with torch.cuda.device(self.device):
            _lib.check(self._lib.sa_stream_update(k.data_ptr(), v.data_ptr(), self.dim, self.value_dim, self.degree,
                                                  1.0, self._num.data_ptr(), self._den.data_ptr(), self._stream()),
                       "sa_stream_update")
        self._bk[self._nbuf].copy_(k)
        self._bv[self._nbuf].copy_(v)
        self._nbuf += 1
        self._length += 1
        if self._nbuf >= self.block_size:
            block = _Items(self._bk.clone(), self._bv.clone(),
                           torch.ones(self.block_size, device=self.device, dtype=torch.float32))
            self._nbuf = 0
            self._insert_level(0, self._compress(block))
            self._repack()

    @torch.no_grad()
    def query(self, query: Tensor, *, return_stats: bool = False) -> Union[Tensor, Tuple[Tensor, AttentionQueryStats]]:
        """ArticleStreamingAttention.query (:572-606)."""
        q = self._vec(query, self.dim, "query")
        lv = self._packed
        with torch.cuda.device(self.device):
            _lib.check(self._lib.sa_stream_query(
                q.data_ptr(), self.dim, self.value_dim, self.degree, self.scale, self._num.data_ptr(),
                self._den.data_ptr(), self._bk.data_ptr(), self._bv.data_ptr(), self._nbuf, lv.keys.data_ptr(),
                lv.values.data_ptr(), lv.weights.data_ptr(), lv.size, self.denominator_eps, self._out.data_ptr(),
                self._dens.data_ptr(), self._ws.data_ptr(), self._ws.numel(), self._stream()), "sa_stream_query")
        out = self._out.to(self.dtype, copy=True)
        if not return_stats:
            return out
        den, low, tail = (float(x) for x in self._dens.cpu())
        return out, AttentionQueryStats(den, low, tail, self._nbuf + lv.size,
                                        self.state_size_bytes(include_feature_map=False))

    def items(self) -> Tuple[Tensor, Tensor, Tensor]:
        """The residual items in the reference's order (pending block with
        weight 1, then levels 0, 1, ...; MergeReduceCoreset.items :472-491)."""
        n = self._nbuf
        ones = torch.ones(n, device=self.device, dtype=torch.float32)
        lv = self._packed
        return (torch.cat([self._bk[:n], lv.keys]), torch.cat([self._bv[:n], lv.values]),
                torch.cat([ones, lv.weights]))

    def state_size_bytes(self, *, include_feature_map: bool = False) -> int:
        """Bytes of the reference's state in ``dtype`` (:608-609, :290-296, :496-506)."""
        e = torch.empty(0, dtype=self.dtype).element_size()
        total = self.features * (1 + self.value_dim) * e
        total += self._nbuf * (self.dim + self.value_dim) * e
        for b in self.levels:
            if b is not None:
                total += b.size * (self.dim + self.value_dim + 1) * e
        if include_feature_map:   # SymmetricTaylorFeatureMap.bytes(include_indices=True), :218-226
            for l in range(1, self.degree + 1):
                total += math.comb(self.dim + l - 1, l) * l * 8
            total += self.features * e
        return int(total)

    @property
    def length(self) -> int:
        return self._length
