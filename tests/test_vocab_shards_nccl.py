"""Vocabulary sharding over two GPUs: one process per GPU holding a column
shard, records exchanged by NCCL all-to-all, ids all-gathered; checked against
the oracle on the whole rows.  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "omni.js_b200"))
    import datetime

    import torch
    import torch.distributed as dist

    from minisample import Sampler, workloads as W
    from minisample.sharding import col_shard, sample_vocab_sharded

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", rank)
        w = W.WORKLOADS["vocab_sharded"]
        B = 16
        X = W.logits_np(w, 4, B=B)
        hist, off = W.history_np(w, 4, B=B)
        u = W.uniforms(4, B)
        c0, c1 = col_shard(w.V, world, rank)
        xs = torch.from_numpy(np.ascontiguousarray(X[:, c0:c1])).to(dev)
        with Sampler([rank]) as s:
            ids = sample_vocab_sharded(s, xs, c0, w.V, w.params, torch.from_numpy(u).to(dev),
                                       torch.from_numpy(hist).to(dev), torch.from_numpy(off).to(dev))
            torch.cuda.synchronize()
        q.put((rank, ids.cpu().numpy().tolist()))
    finally:
        dist.destroy_process_group()


def test_two_gpu_vocab_shards_match_oracle(oracle):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from minisample import workloads as W
    from test_parity_gpu import BOUNDARY, params

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0] == res[1]
    w = W.WORKLOADS["vocab_sharded"]
    B = 16
    X = W.logits_np(w, 4, B=B)
    hist, off = W.history_np(w, 4, B=B)
    u = W.uniforms(4, B)
    ids_r, d_r = oracle.sample_batch(X, hist, off, params(oracle, w.params), u, cand_cap=8)
    for r in range(B):
        if res[0][r] != ids_r[r]:
            assert d_r["margin_draw"][r] < BOUNDARY or d_r["margin_cut"][r] < BOUNDARY, r
