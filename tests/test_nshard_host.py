"""Host logic of the N-sharded forward on CPU: the shard plan, and the
exchange over a world-size-2 gloo group (two processes on this host)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from streaming_attention_b200 import nshard


def test_shard_plan_splits_blocks_and_reps():
    p = [nshard.shard_plan(4096, 4, r, 256, "sorted_pair") for r in range(4)]
    assert [x.t0 for x in p] == [0, 1024, 2048, 3072]
    assert [x.c_off for x in p] == [0, 4, 8, 12]
    # 15 completed blocks in all: the last shard's last block completes nothing later
    assert [x.n_compress for x in p] == [4, 4, 4, 3]
    assert all(x.reps_per_rank == 4 * 128 for x in p)
    none = nshard.shard_plan(1024, 2, 1, 64, "none")
    assert (none.n_compress, none.reps_per_rank, none.m_blk) == (0, 512, 64)
    with pytest.raises(ValueError, match="equal shards"):
        nshard.shard_plan(1000, 3, 0, 8, "sorted_pair")
    with pytest.raises(ValueError, match="whole number of blocks"):
        nshard.shard_plan(1024, 2, 0, 100, "sorted_pair")
    with pytest.raises(ValueError, match="rank"):
        nshard.shard_plan(1024, 2, 2, 64, "sorted_pair")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _exchange_rank(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bh, rb, d = 2, 3, 4
        state = torch.full((5,), float(rank + 1))
        rk = torch.arange(bh * rb * d, dtype=torch.float32).reshape(bh, rb, d) + 100 * rank
        rv = rk[..., :2] * 2
        rw = torch.full((bh, rb), float(rank))
        before, ka, va, wa = nshard.exchange(state, rk, rv, rw, rank, world)
        results[rank] = (before.clone(), ka.clone(), va.clone(), wa.clone())
    finally:
        dist.destroy_process_group()


def test_exchange_over_a_two_rank_gloo_group():
    world = 2
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_exchange_rank, args=(world, _free_port(), results), nprocs=world, join=True)
        r0, r1 = results[0], results[1]
    # rank 0 sees no earlier state and only its own reps
    assert r0[0].shape == (0, 5)
    assert r0[1].shape == (2, 3, 4) and torch.equal(r0[3], torch.zeros(2, 3))
    # rank 1: the state of rank 0, the reps of ranks 0 then 1 per sequence
    assert torch.equal(r1[0], torch.ones(1, 5))
    base = torch.arange(24, dtype=torch.float32).reshape(2, 3, 4)
    assert torch.equal(r1[1], torch.cat([base, base + 100], dim=1))
    assert torch.equal(r1[3], torch.cat([torch.zeros(2, 3), torch.ones(2, 3)], dim=1))


def test_zigzag_ownership_covers_every_chunk_once():
    for world in (1, 2, 4, 8):
        owned = [j for r in range(world) for j in nshard.owned_chunks(r, world, "zigzag")]
        assert sorted(owned) == list(range(2 * world))
        assert nshard.owned_chunks(1, 4, "contiguous") == [1]
    with pytest.raises(ValueError, match="layout"):
        nshard.owned_chunks(0, 2, "striped")


# ---------------------------------------------------------------------------
# failure detection: a rank that is gone before the exchange
# ---------------------------------------------------------------------------

def _failing_rank(rank, world, port, how, results):
    """Rank 1 leaves (or raises) after joining the group and before the
    exchange; rank 0 runs the exchange and records how it ended."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        results[1] = "left"
        if how == "raise":
            raise RuntimeError("rank 1 failed before the exchange")
        return          # leaves between steps: none of its collectives is in flight
    state = torch.ones(5)
    rk = torch.zeros(2, 3, 4)
    t0 = time.monotonic()
    try:
        nshard.exchange(state, rk, rk[..., :2], torch.zeros(2, 3), rank, world)
        results[0] = ("completed", time.monotonic() - t0, "")
    except Exception as exc:   # the survivor must get an error, not hang
        results[0] = ("raised", time.monotonic() - t0, f"{type(exc).__name__}: {exc}"[:300])


@pytest.mark.timeout(180)
@pytest.mark.parametrize("how", ["exit", "raise"])
def test_exchange_fails_with_an_error_when_a_rank_is_gone(how):
    ctx = mp.get_context("spawn")
    port = _free_port()
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_failing_rank, args=(r, 2, port, how, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=150)
        alive = [p.is_alive() for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        res = dict(results)
    assert not any(alive), "a rank hung"
    assert res.get(1) == "left"
    outcome, secs, msg = res[0]
    assert outcome == "raised", f"the exchange finished without the other rank: {outcome}"
    # within the process group's 5 s timeout (plus start-up slack), not after a hang
    assert secs < 60, (secs, msg)
