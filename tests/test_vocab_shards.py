"""Vocabulary sharding on one GPU: the G shards' records are computed on column
views of the same logits and stacked as the all-to-all would deliver them,
then merged; the ids are checked against the oracle on the whole rows with
the tolerances of test_parity_gpu."""
import numpy as np
import pytest

from test_parity_gpu import check, params

pytestmark = pytest.mark.gpu


def _merge_sharded(sampler, X, sp, G, u, hist=None, off=None, cap=64):
    import torch

    from minisample.sharding import col_shard

    dev = torch.device("cuda", 0)
    B, V = X.shape
    xd = torch.from_numpy(X).to(dev)
    hd = od = None
    if off is not None:
        hd = torch.from_numpy(np.ascontiguousarray(hist if len(hist) else np.zeros(1), np.int32)).to(dev)
        od = torch.from_numpy(np.ascontiguousarray(off, np.int64)).to(dev)
    recs = []
    for g in range(G):
        c0, c1 = col_shard(V, G, g)
        recs.append(sampler.shard_records(xd[:, c0:c1], V, c0, sp, hd, od))
    R = torch.stack(recs, dim=1).contiguous()
    ud = torch.from_numpy(np.ascontiguousarray(u, np.float64)).to(dev)
    ids, d = sampler.merge_records(R, V, sp, u=ud, diag=True, cand_cap=cap)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), {k: v.cpu().numpy() for k, v in d.items()}


def _workload(name, B, seed=3):
    from minisample import workloads as W

    w = W.WORKLOADS[name]
    X = W.logits_np(w, seed, B=B)
    hist, off = W.history_np(w, seed, B=B)
    return w, X, hist, off, W.uniforms(seed, B)


@pytest.mark.parametrize("G", [2, 3, 8])
@pytest.mark.parametrize("name", ["vocab_sharded", "gemma_b512", "llama3_b64", "llama3_b64_greedy", "gpt2_b1"])
def test_sharded_merge_matches_oracle(oracle, sampler, name, G):
    w, X, hist, off, u = _workload(name, 12 if name != "gpt2_b1" else 6)
    ids_g, d_g = _merge_sharded(sampler, X, w.params, G, u, hist, off)
    ids_r, d_r = oracle.sample_batch(X, hist, off, params(oracle, w.params), u, cand_cap=64)
    assert not np.any(d_g["row_flags"] & 0x10), d_g["row_flags"]
    check(ids_r, d_r, ids_g, d_g, w.params, f"{name} G={G}")


def test_sharded_edge_rows(oracle, sampler):
    """A shard of -inf, a NaN in one shard, a row of -inf, the maximum in the
    last shard, a huge boost inside one shard."""
    from minisample import SampleParams

    rng = np.random.default_rng(9)
    B, V, G = 6, 70000, 4
    X = rng.normal(0.0, 1.5, (B, V)).astype(np.float32)
    X[0, : V // 4] = -np.inf
    X[1, 40000] = np.nan
    X[2, :] = -np.inf
    X[3, -1] = 30.0
    X[4, 12345] = 25.0
    sp = SampleParams(True, 0.8, 50, 0.9, 1.0)
    u = rng.random(B)
    ids_g, d_g = _merge_sharded(sampler, X, sp, G, u)
    ids_r, d_r = oracle.sample_batch(X, None, None, params(oracle, sp), u, cand_cap=64)
    assert not np.any(d_g["row_flags"] & 0x10), d_g["row_flags"]
    check(ids_r, d_r, ids_g, d_g, sp, "edge rows", max_boundary_frac=0.34)


def test_sharded_ties_are_unsettled_or_exact(oracle, sampler):
    """Rows of equal logits tie everywhere: the merge either settles them
    exactly or reports them (-1, MS_ROW_UNSETTLED), never a wrong id; the
    reported ones match the oracle through the whole-row path."""
    from minisample import SampleParams

    B, V, G = 4, 40000, 4
    X = np.zeros((B, V), np.float32)
    X[1, ::7] = 1.0
    X[2, :] = np.repeat(np.arange(V // 100, dtype=np.float32), 100)[:V] * 1e-3
    X[3, 5:] = -1.0
    sp = SampleParams(True, 1.0, 20, 0.9, 1.0)
    u = np.array([0.1, 0.5, 0.9, 0.3])
    ids_g, d_g = _merge_sharded(sampler, X, sp, G, u)
    ids_r, d_r = oracle.sample_batch(X, None, None, params(oracle, sp), u, cand_cap=64)
    for r in range(B):
        if d_g["row_flags"][r] & 0x10:
            assert ids_g[r] == -1
            ids_w = sampler.sample(X[r:r + 1], sp, u=u[r:r + 1])
            assert ids_w[0] == ids_r[r]
        else:
            assert ids_g[r] == ids_r[r], (r, ids_g[r], ids_r[r])


def test_shard_record_bytes_and_errors(sampler):
    from minisample import SampleParams, record_bytes
    from minisample._native import MiniSampleError

    assert record_bytes(1000, SampleParams(False)) == 32
    assert record_bytes(1000, SampleParams(True, 0.9, 50, 0.9, 1.0)) == 32 + (50 + 32) * 16
    with pytest.raises(MiniSampleError):
        record_bytes(1000, SampleParams(True, 0.9, 0, 0.9, 1.0))  # top_k off: whole-row path only
