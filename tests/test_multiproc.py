"""Row sharding and max-over-ranks timing with world_size 2 on gloo (CPU)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, B, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "omni.js_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from minisample.sharding import max_over_ranks, row_shard, sum_over_ranks

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        r0, r1 = row_shard(B, world, rank)
        got = [None] * world
        dist.all_gather_object(got, (r0, r1))
        t = max_over_ranks(1.0 + rank)
        rows = sum_over_ranks(r1 - r0)
        q.put((rank, got, t, rows))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [512, 7, 1])
def test_row_shards_cover_batch_once_and_time_is_max(B):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, shards, t, rows in res:
        assert t == 2.0
        assert rows == B
        covered = []
        for r0, r1 in shards:
            covered += list(range(r0, r1))
        assert covered == list(range(B))


def test_row_shard_rejects_bad_arguments():
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "omni.js_b200"))
    from minisample.sharding import row_shard

    with pytest.raises(ValueError):
        row_shard(4, 0, 0)
    with pytest.raises(ValueError):
        row_shard(4, 2, 2)
    assert row_shard(5, 4, 3) == (5, 5)


def _shard_worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "omni.js_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from minisample.sharding import col_shard, exchange_records, gather_rows

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        B, R, V = 5, 8, 11
        # record of (row r, shard s) = bytes r*16 + s, then a marker
        rec = torch.zeros((B, R), dtype=torch.uint8)
        for r in range(B):
            rec[r, 0] = r * 16 + rank
            rec[r, 1] = 200 + rank
        recs, Bb = exchange_records(rec)
        c0, c1 = col_shard(V, world, rank)
        full = torch.arange(3 * V, dtype=torch.float32).view(3, V)
        rows = gather_rows(full[:, c0:c1].contiguous())
        q.put((rank, Bb, recs.numpy().tolist(), bool(torch.equal(rows, full)), (c0, c1)))
    finally:
        dist.destroy_process_group()


def test_vocab_shard_exchange_and_row_gather():
    """Each rank gets every shard's record of its own row block, in shard
    order; the column shards of a row reassemble in rank order."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cols = []
    for rank, Bb, recs, same, (c0, c1) in res:
        assert Bb == 3 and same
        cols += list(range(c0, c1))
        for j in range(Bb):
            r = rank * Bb + j
            for s in range(world):
                if r < 5:
                    assert recs[j][s][0] == r * 16 + s and recs[j][s][1] == 200 + s
                else:
                    assert recs[j][s][0] == 0  # padding rows past B
    assert cols == list(range(11))
