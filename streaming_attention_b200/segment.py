"""Drop-in GPU entry points of the reference's fused segment-mean variant.

Mirrors ``triton_article_attention.py`` of PositiveLoss/streaming-attention:
``triton_article_causal_attention``, ``build_segment_mean_coreset``,
``TritonArticleStats``, ``triton_flash_causal_attention`` (exact causal
attention, the comparator) and ``torch_classical_causal_attention`` keep the
reference's names, keyword arguments, argument checks (order and messages),
return types and stats fields.  The arithmetic runs in libsa_b200.so: the
segment-mean kernel, then the same block-granular moment scan and tensor-core
residual as the fast path, with reps of weight ``compress_stride`` and the exp
argument capped at 80 (triton_article_attention.py:331-333, :359).

The reference's Triton tile arguments (``block_m``, ``block_n``, ``block_r``,
``value_block``) are accepted and ignored: the tiles here are fixed by the
sm_100a kernels.  Value widths above 128 (the reference allows 256) run as
column slices of at most 128 through the same kernels.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple, Union

import torch

from . import _lib
from . import fast as _fast

Tensor = torch.Tensor

__all__ = ["TritonArticleStats", "build_segment_mean_coreset", "triton_article_causal_attention",
           "triton_flash_causal_attention", "torch_classical_causal_attention"]

_MAX_VALUE_SLICE = 128


@dataclass(frozen=True)
class TritonArticleStats:
    """Field-for-field copy of triton_article_attention.py:172-181."""
    degree: int
    block_size: int
    compress_stride: int
    coreset_items_per_sequence: int
    coreset_bytes_per_sequence: int
    kv_bytes_per_sequence: int
    score_matrix_bytes_per_sequence: int
    output_bytes_per_sequence: int


def _attention_scale(scale: Optional[float], dim: int) -> float:
    """triton_article_attention.py:96-97."""
    return float(1.0 / math.sqrt(dim) if scale is None else scale)


def _require_cuda(*tensors: Tensor) -> None:
    """triton_article_attention.py:80-83."""
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("the B200 kernels require CUDA tensors")


def _flatten_bh_qkv(q: Tensor, k: Tensor, v: Tensor) -> Tuple[Tensor, Tensor, Tensor, Tuple[int, ...], bool]:
    """Contiguous [BH,N,D], [BH,N,D], [BH,N,Dv] views (triton_article_attention.py:146-162)."""
    if q.shape != k.shape:
        raise ValueError(f"q and k must match, got {tuple(q.shape)} and {tuple(k.shape)}")
    if q.ndim == 2:
        if v.ndim != 2 or v.shape[0] != q.shape[0]:
            raise ValueError("for [N,D] q/k, v must be [N,Dv]")
        return q[None].contiguous(), k[None].contiguous(), v[None].contiguous(), tuple(q.shape), False
    if q.ndim == 4:
        if v.ndim != 4 or v.shape[:3] != q.shape[:3]:
            raise ValueError("for [B,H,N,D] q/k, v must be [B,H,N,Dv]")
        b, h, n, d = q.shape
        return (q.contiguous().view(b * h, n, d), k.contiguous().view(b * h, n, d),
                v.contiguous().view(b * h, n, v.shape[-1]), tuple(q.shape), True)
    raise ValueError("q/k/v must be [N,D] or [B,H,N,D]")


def _unflatten_output(out3: Tensor, original_q_shape: Tuple[int, ...], had_bh: bool) -> Tensor:
    if not had_bh:
        return out3[0]
    b, h, n, _ = original_q_shape
    return out3.view(b, h, n, out3.shape[-1])


def _kernel_dtype(t: Tensor) -> Tensor:
    """The reference computes in float32 from float16 / bfloat16 / float32
    inputs and converts anything else to float32 first (:507-512)."""
    if t.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return t.float()
    return t


def _rep_code(t: Tensor) -> int:
    return _lib.REP_DTYPES[str(t.dtype).replace("torch.", "")]


def _check_segment_args(degree: int, block_size: int, compress_stride: int) -> None:
    """triton_article_attention.py:487-492 (and :220-223)."""
    if degree not in (0, 1, 2):
        raise NotImplementedError("Triton article kernel currently supports degree 0, 1, or 2")
    if block_size <= 0 or compress_stride <= 0:
        raise ValueError("block_size and compress_stride must be positive")
    if block_size % compress_stride != 0:
        raise ValueError("block_size must be divisible by compress_stride")


@torch.no_grad()
def build_segment_mean_coreset(k_bhn: Tensor, v_bhn: Tensor, *, block_size: int,
                               compress_stride: int) -> Tuple[Tensor, Tensor, int]:
    """Deterministic reps of the completed blocks (triton_article_attention.py:190-245):
    rep_k [BH,R,D] and rep_v [BH,R,Dv] in the dtypes of k and v, and
    reps_per_block = block_size // compress_stride.  Each rep is the mean of
    compress_stride adjacent tokens; only blocks a later query reads are kept.
    The means are taken in float32 (a float64 input gets float32 means)."""
    if k_bhn.ndim != 3 or v_bhn.ndim != 3:
        raise ValueError("k_bhn and v_bhn must be [BH,N,D] and [BH,N,Dv]")
    if k_bhn.shape[:2] != v_bhn.shape[:2]:
        raise ValueError("k_bhn and v_bhn must have the same [BH,N]")
    if block_size <= 0 or compress_stride <= 0:
        raise ValueError("block_size and compress_stride must be positive")
    if block_size % compress_stride != 0:
        raise ValueError("for the Triton kernel, block_size must be divisible by compress_stride")
    _require_cuda(k_bhn, v_bhn)
    bh, n, dim = k_bhn.shape
    dv = v_bhn.shape[-1]
    m = block_size // compress_stride
    nc = max(0, (n - 1) // block_size)
    dev = k_bhn.device
    if nc == 0:
        return (torch.empty(bh, 0, dim, device=dev, dtype=k_bhn.dtype),
                torch.empty(bh, 0, dv, device=dev, dtype=v_bhn.dtype), m)
    k32 = k_bhn.to(torch.float32).contiguous()
    v32 = v_bhn.to(torch.float32).contiguous()
    R = nc * m
    rk = torch.empty(bh, R, dim, device=dev)
    rv = torch.empty(bh, R, dv, device=dev)
    kc = _rep_code(k_bhn) if k_bhn.dtype in (torch.float16, torch.bfloat16) else 0
    vc = _rep_code(v_bhn) if v_bhn.dtype in (torch.float16, torch.bfloat16) else 0
    with torch.cuda.device(dev):
        _lib.call("sa_segment_mean_reps", k32.data_ptr(), v32.data_ptr(), bh, n, dim, dv, block_size,
                  compress_stride, kc, vc, rk.data_ptr(), rv.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    return rk.to(k_bhn.dtype), rv.to(v_bhn.dtype), m


def _forward(q3: Tensor, k3: Tensor, v3: Tensor, *, degree: int, block_size: int, compress_stride: int,
             scale: float, eps: float, key_code: int, value_code: int) -> Tensor:
    """One launch sequence over contiguous float32 [bh, n, *] tensors, dv <= 128."""
    bh, n, d = q3.shape
    dv = v3.shape[-1]
    dev = q3.device
    out = torch.empty(bh, n, dv, device=dev, dtype=torch.float32)
    if bh == 0 or n == 0:
        return out
    lib = _lib.load()
    nbytes = _lib.ctypes.c_size_t(0)
    _lib.check(lib.sa_article_segment_mean_workspace_size(bh, n, d, dv, degree, block_size, compress_stride,
                                                          _lib.ctypes.byref(nbytes)),
               "sa_article_segment_mean_workspace_size")
    ws = torch.empty(max(int(nbytes.value), 256), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.sa_article_segment_mean(
            q3.data_ptr(), k3.data_ptr(), v3.data_ptr(), bh, n, d, dv, degree, block_size, compress_stride,
            float(scale), key_code, value_code, float(eps), out.data_ptr(), ws.data_ptr(), ws.numel(), stream),
            "sa_article_segment_mean")
        if _fast._CHECK_STATUS:
            _fast.check_device_status(ws)
    return out


@torch.no_grad()
def triton_article_causal_attention(
    q: Tensor, k: Tensor, v: Tensor, *, degree: int = 2, block_size: int = 128, compress_stride: int = 2,
    scale: Optional[float] = None, block_m: int = 16, block_n: int = 64, block_r: int = 64,
    value_block: Optional[int] = None, denominator_eps: float = 1.0e-12,
    output_dtype: Optional[torch.dtype] = torch.float32, return_stats: bool = False,
) -> Union[Tensor, Tuple[Tensor, TritonArticleStats]]:
    """Approximate causal attention with segment-mean reps of the completed
    blocks (triton_article_attention.py:448-578) for [N,D] or [B,H,N,D]
    tensors on a CUDA device.  ``compress_stride=1`` keeps every earlier key
    and matches exact softmax attention up to roundoff."""
    _require_cuda(q, k, v)
    _check_segment_args(degree, block_size, compress_stride)
    q3, k3, v3, original_shape, had_bh = _flatten_bh_qkv(q, k, v)
    bh, n, dim = q3.shape
    dv = v3.shape[-1]
    if dim > 128:
        raise ValueError("this compact kernel supports D <= 128; increase BLOCK_D logic for larger heads")
    if dv > 256:
        raise ValueError("this compact kernel supports Dv <= 256")
    q3, k3, v3 = _kernel_dtype(q3), _kernel_dtype(k3), _kernel_dtype(v3)
    key_code = _rep_code(k3)
    value_code = _rep_code(v3)
    s = _attention_scale(scale, dim)
    qf, kf, vf = (t.to(torch.float32).contiguous() for t in (q3, k3, v3))
    kw = dict(degree=degree, block_size=block_size, compress_stride=compress_stride, scale=s, eps=denominator_eps,
              key_code=key_code, value_code=value_code)
    if dv <= _MAX_VALUE_SLICE:
        out3 = _forward(qf, kf, vf, **kw)
    else:
        out3 = torch.cat([_forward(qf, kf, vf[..., a:a + _MAX_VALUE_SLICE].contiguous(), **kw)
                          for a in range(0, dv, _MAX_VALUE_SLICE)], -1)
    out_dtype = output_dtype or torch.float32
    out = _unflatten_output(out3.to(out_dtype), original_shape, had_bh)
    if not return_stats:
        return out
    r = max(0, (n - 1) // block_size) * (block_size // compress_stride)
    elem_kv = q3.element_size()
    elem_out = torch.empty((), dtype=out_dtype).element_size()
    stats = TritonArticleStats(
        degree=degree, block_size=block_size, compress_stride=compress_stride,
        coreset_items_per_sequence=int(r), coreset_bytes_per_sequence=int(r * (dim + dv) * elem_kv),
        kv_bytes_per_sequence=int(n * (dim + dv) * elem_kv), score_matrix_bytes_per_sequence=int(n * n * elem_kv),
        output_bytes_per_sequence=int(n * dv * elem_out))
    return out, stats


@torch.no_grad()
def triton_flash_causal_attention(
    q: Tensor, k: Tensor, v: Tensor, *, scale: Optional[float] = None, block_m: int = 16, block_n: int = 64,
    value_block: Optional[int] = None, output_dtype: Optional[torch.dtype] = torch.float32,
) -> Tensor:
    """Exact causal softmax attention for [N,D] or [B,H,N,D] tensors on a CUDA
    device (triton_article_attention.py:580-637): online softmax, fp32
    accumulation, out = acc / max(l, 1e-20).  Runs on the tensor cores (3xTF32)
    for D <= 64 and Dv <= 128, on the CUDA cores otherwise."""
    _require_cuda(q, k, v)
    q3, k3, v3, original_shape, had_bh = _flatten_bh_qkv(q, k, v)
    bh, n, dim = q3.shape
    dv = v3.shape[-1]
    if dim > 128:
        raise ValueError("this compact kernel supports D <= 128")
    if dv > 256:
        raise ValueError("this compact kernel supports Dv <= 256")
    s = _attention_scale(scale, dim)
    qf, kf, vf = (t.to(torch.float32).contiguous() for t in (q3, k3, v3))
    dev = qf.device
    out3 = torch.empty(bh, n, dv, device=dev, dtype=torch.float32)
    if bh > 0 and n > 0:
        lib = _lib.load()
        nbytes = _lib.ctypes.c_size_t(0)
        _lib.check(lib.sa_flash_causal_attention_workspace_size(bh, n, dim, dv, _lib.ctypes.byref(nbytes)),
                   "sa_flash_causal_attention_workspace_size")
        ws = torch.empty(max(int(nbytes.value), 256), device=dev, dtype=torch.uint8)
        with torch.cuda.device(dev):
            _lib.check(lib.sa_flash_causal_attention(
                qf.data_ptr(), kf.data_ptr(), vf.data_ptr(), bh, n, dim, dv, float(s), out3.data_ptr(),
                ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream), "sa_flash_causal_attention")
            if _fast._CHECK_STATUS and nbytes.value:
                _fast.check_device_status(ws)
    return _unflatten_output(out3.to(output_dtype or torch.float32), original_shape, had_bh)


@torch.no_grad()
def torch_classical_causal_attention(q: Tensor, k: Tensor, v: Tensor, *, scale: Optional[float] = None) -> Tensor:
    """Exact causal softmax attention for [N,D] or [B,H,N,D] tensors
    (triton_article_attention.py:123-143).  A torch helper for comparisons, not
    the product path."""
    if q.shape != k.shape:
        raise ValueError("q and k must have identical shape")
    if q.ndim == 2:
        n, dim = q.shape
    elif q.ndim == 4:
        if v.shape[:3] != q.shape[:3]:
            raise ValueError("v must have shape [B,H,N,Dv]")
        n, dim = q.shape[2], q.shape[3]
    else:
        raise ValueError("q/k/v must be [N,D] or [B,H,N,D]")
    s = _attention_scale(scale, dim)
    logits = torch.matmul(q, k.transpose(-1, -2)) * s
    mask = torch.ones(n, n, device=q.device, dtype=torch.bool).tril()
    logits = logits.masked_fill(~mask, float("-inf"))
    return torch.matmul(torch.softmax(logits, dim=-1), v)
