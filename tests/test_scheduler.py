"""CPU tests of the stream scheduler: partitioning, the 2-rank (gloo) shard run
with the reporting gather, and a rank that fails on the host."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from mockbird_b200.scheduler import partition_streams


def test_equal_blocks_cover_every_stream_once():
    for total, world in [(64, 1), (64, 2), (64, 8), (4096, 8), (5, 8), (0, 4), (13, 4)]:
        shards = partition_streams(total, world)
        ids = np.concatenate([s.streams for s in shards]) if total else np.array([])
        assert sorted(ids.tolist()) == list(range(total))
        counts = [s.count for s in shards]
        assert max(counts) - min(counts) <= 1
        for s in shards:  # contiguous, ascending
            assert np.all(np.diff(s.streams) == 1)


def test_length_balanced_partition():
    rng = np.random.default_rng(0)
    lengths = rng.integers(1, 4097, size=4096)
    shards = partition_streams(4096, 8, lengths)
    ids = np.concatenate([s.streams for s in shards])
    assert sorted(ids.tolist()) == list(range(4096))
    loads = [int(lengths[s.streams].sum()) for s in shards]
    assert max(loads) / min(loads) < 1.01
    assert {s.count for s in shards} == {512}


def test_bad_arguments():
    with pytest.raises(ValueError):
        partition_streams(4, 0)
    with pytest.raises(ValueError):
        partition_streams(4, 2, lengths=[1, 2, 3])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shard_worker(rank, world, port, total, q):
    """Each rank runs the (CPU oracle) decode of its own streams, then gathers reports."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from mockbird_b200.scheduler import gather_reports, init_group, max_over_ranks
    import oracle

    dist = init_group("gloo", timeout_s=30)
    shard = partition_streams(total, world)[rank]
    ring = oracle.Ring(layers=1, streams=total, heads=12, capacity=16, dtype="f32", wrap=True)
    rng = np.random.default_rng(100 + rank)
    csum = 0.0
    for pos in range(20):
        qkv = rng.standard_normal((shard.count, 3 * 768)).astype(np.float32)
        ctx, _ = ring.append_attend(0, shard.streams, [pos] * shard.count, qkv)
        csum += float(ctx.astype(np.float64).sum())
    reports = gather_reports({"rank": rank, "streams": shard.count, "checksum": csum})
    slow = max_over_ranks(float(rank + 1))
    q.put((rank, reports, slow, shard.streams.tolist()))
    dist.destroy_process_group()


def test_two_rank_shards_gather_reports():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, 6, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    owned = sorted(results[0][3] + results[1][3])
    assert owned == list(range(6))
    for rank, reports, slow, _ in results:
        assert [int(r["rank"]) for r in reports] == [0, 1]
        assert [int(r["streams"]) for r in reports] == [3, 3]
        assert slow == 2.0


def _failing_worker(rank, world, port, q):
    """Rank 1 raises before the reporting gather; rank 0 must get an error, not hang."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from mockbird_b200.scheduler import gather_reports, init_group

    dist = init_group("gloo", timeout_s=10)
    if rank == 1:
        q.put((rank, "raised"))
        raise SystemExit(3)
    try:
        gather_reports({"rank": rank})
        q.put((rank, "no error"))
    except Exception as e:  # the peer is gone: the collective fails within the timeout
        q.put((rank, "error: " + type(e).__name__))
    dist.destroy_process_group()


def test_rank_failure_surfaces_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert out[1] == "raised"
    assert out[0].startswith("error"), out[0]
    assert procs[1].exitcode == 3


def _balance_worker(rank, world, port, q):
    """Each rank computes its own share of BASELINE config 5's length-balanced split
    (4096 streams over 8 shards, seeded lengths U[1, 4096]); the ranks gather their
    shards' total live lengths and stream counts."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from mockbird_b200.scheduler import gather_reports, init_group

    dist = init_group("gloo", timeout_s=30)
    lengths = np.random.default_rng(0).integers(1, 4097, size=4096)
    shards = partition_streams(4096, 8, lengths)
    mine = [shards[i] for i in range(rank, 8, world)]  # this rank's 4 of the 8 shards
    reports = [gather_reports({"shard": sh.rank, "load": int(lengths[sh.streams].sum()), "count": sh.count})
               for sh in mine]
    q.put((rank, [r for rep in reports for r in rep], int(lengths.max())))
    dist.destroy_process_group()


def test_two_rank_config5_length_balance():
    """Run as 2 gloo ranks: config 5's 8 shards each carry the same number of
    streams (512) and their total live lengths differ by less than the longest
    stream's length (one stream's worth of imbalance at most)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_balance_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict((r, (reps, mx)) for r, reps, mx in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0][0] == results[1][0]  # both ranks saw every shard's report
    reps, longest = results[0]
    by_shard = {int(r["shard"]): r for r in reps}
    assert sorted(by_shard) == list(range(8))
    loads = [by_shard[i]["load"] for i in range(8)]
    assert {int(by_shard[i]["count"]) for i in range(8)} == {512}
    assert max(loads) - min(loads) <= longest
