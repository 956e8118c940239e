"""The N-sharded forward (one long sequence split over ranks) against the
unsharded forward on the same GPU: all ranks emulated in one process (the
all-gather replaced by stacking), and over NCCL when two GPUs are present.

Bars: outputs within 1e-5 relative L2 of the single-device forward (the fp32
moment states are summed in a different association); coreset selections
(global token indices) bit-exact."""

import os
import socket

import pytest
import torch

import streaming_attention_b200 as sa
from oracle import oracle as O
from streaming_attention_b200 import fast, nshard, workloads

pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


CASES = [
    ("cfg5_shape_w2", 5, dict(B=1, H=3, N=2048), 2),
    ("cfg5_shape_w4", 5, dict(B=1, H=2, N=4096), 4),
    ("cfg3_shape_w4", 3, dict(B=1, H=2, N=2048, block_size=128), 4),
    ("cfg4_deg3_random_w2", 4, dict(B=1, H=2, N=2048), 2),
    ("none_w2", 2, dict(B=1, H=2, N=1024), 2),
]


@pytest.mark.parametrize("label,cfg,over,world", CASES, ids=[c[0] for c in CASES])
def test_sharded_forward_matches_single_device(label, cfg, over, world, dev):
    c = workloads.config(cfg, **over)
    q, k, v = workloads.make_inputs(c, seed=2, device=dev)
    kw = dict(degree=c["degree"], block_size=c["block_size"], scale=c["scale"], compressor=c["compressor"], seed=5)
    ref = sa.fast_article_causal_attention(q, k, v, **kw)
    out, ridx = nshard.nshard_emulate(q, k, v, world=world, return_rep_idx=True, **kw)
    err = O.relative_l2(out.cpu().numpy(), ref.cpu().numpy())
    assert err < TOL, f"{label}: rel L2 {err:.3e}"
    if c["compressor"] != "none":
        B, H, N, d = q.shape
        _, ref_idx = fast._run(q.reshape(B * H, N, d), k.reshape(B * H, N, d), v.reshape(B * H, N, -1), batch=B,
                               heads=H, degree=c["degree"], block_size=c["block_size"],
                               scale=workloads.attention_scale(c), compressor=c["compressor"], seed=5, eps=1e-12,
                               want_rep_idx=True)
        assert torch.equal(ridx, ref_idx)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, q, k, v, kw, results):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        d = torch.device("cuda", rank)
        for layout in ("contiguous", "zigzag"):
            chunks = nshard.owned_chunks(rank, world, layout)
            L = q.shape[2] // (world * len(chunks))
            pick = lambda x: torch.cat([x[:, :, j * L:(j + 1) * L] for j in chunks], dim=2).to(d)  # noqa: E731
            out = nshard.fast_article_causal_attention_nshard(pick(q), pick(k), pick(v), rank=rank, world=world,
                                                              layout=layout, **kw)
            results[(rank, layout)] = (chunks, out.cpu())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_forward_over_nccl(dev):
    import torch.multiprocessing as mp
    c = workloads.config(5, B=1, H=2, N=2048)
    q, k, v = workloads.make_inputs(c, seed=3)
    kw = dict(degree=2, block_size=256, compressor="sorted_pair", seed=1)
    ref = sa.fast_article_causal_attention(q.to(dev), k.to(dev), v.to(dev), **kw).cpu()
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_nccl_rank, args=(2, _free_port(), q, k, v, kw, results), nprocs=2, join=True)
        for layout in ("contiguous", "zigzag"):
            parts = {}
            for r in range(2):
                chunks, out = results[(r, layout)]
                L = out.shape[2] // len(chunks)
                for i, j in enumerate(chunks):
                    parts[j] = out[:, :, i * L:(i + 1) * L]
            full = torch.cat([parts[j] for j in sorted(parts)], dim=2)
            assert O.relative_l2(full.numpy(), ref.numpy()) < TOL, layout
