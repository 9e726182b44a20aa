"""GPU parity: libminisample (through the C ABI) against the oracle on the same
seeded inputs.

Tolerances (the sampler's contract):
  * penalised logits (the reference's `work` after the penalty), the
    tempered max and the candidate ids / order: bit-exact;
  * probabilities: within 1e-5 relative;
  * sampled ids: identical, except rows whose draw r, or whose running top-p
    sum, lies within 1e-6 of a cumulative-probability boundary in the oracle;
    those rows are counted and reported, and must stay rare.
"""
import json
import os
import time

import numpy as np
import pytest

from test_oracle import KAT

pytestmark = pytest.mark.gpu

BOUNDARY = 1e-6
PROB_RTOL = 1e-5


def params(oracle, sp):
    return oracle.make_params(sp.do_sample, sp.temperature, sp.top_k, sp.top_p, sp.repetition_penalty)


def run_both(oracle, sampler, X, sp, u=None, hist=None, off=None, cap=64, pen=True):
    ids_r, d_r = oracle.sample_batch(X, hist, off, params(oracle, sp), u, cand_cap=cap, want_pen=pen)
    ids_g, d_g = sampler.sample(X, sp, u=u, hist=hist, hist_off=off, diag="pen" if pen else True, cand_cap=cap)
    return ids_r, d_r, ids_g, d_g


def check(ids_r, d_r, ids_g, d_g, sp, label="", cap=64, max_boundary_frac=0.02):
    """Compare one batch; returns the rows whose id differs within the
    boundary tolerance.  A row near a boundary still has its candidate list
    compared up to the shorter of the two cuts."""
    B = len(ids_r)
    tolerated = []
    greedy = (not sp.do_sample) or sp.temperature <= 1e-4
    for r in range(B):
        near_draw = d_r["margin_draw"][r] < BOUNDARY
        near_cut = d_r["margin_cut"][r] < BOUNDARY
        near = near_draw or near_cut
        if ids_r[r] != ids_g[r]:
            assert near and not greedy, (
                f"{label} row {r}: gpu {ids_g[r]} oracle {ids_r[r]} "
                f"margins draw={d_r['margin_draw'][r]:.3g} cut={d_r['margin_cut'][r]:.3g} "
                f"flags={d_g['row_flags'][r]}")
            tolerated.append(r)
        if greedy or d_r["nan_path"][r]:
            continue
        # tempered max is an fp32 value in both
        assert d_g["row_max"][r] == d_r["mx"][r], (label, r)
        assert abs(d_g["row_sum"][r] - d_r["sum"][r]) <= 1e-6 * d_r["sum"][r], (label, r)
        n = int(d_r["n_cand"][r])
        if not near_cut:
            assert d_g["n_cand"][r] == n, (label, r, d_g["n_cand"][r], n)
            assert abs(d_g["total"][r] - d_r["total"][r]) <= 1e-6 * max(d_r["total"][r], 1e-30), (label, r)
        if "cand_ids" in d_g:
            n = min(n, int(d_g["n_cand"][r]), cap)
            np.testing.assert_array_equal(d_g["cand_ids"][r, :n], d_r["cand_ids"][r, :n], err_msg=f"{label} r{r}")
            np.testing.assert_allclose(d_g["cand_probs"][r, :n], d_r["cand_probs"][r, :n], rtol=PROB_RTOL,
                                       err_msg=f"{label} r{r}")
    if "pen_logits" in d_g and "pen_logits" in d_r:
        ga, ra = np.ascontiguousarray(d_g["pen_logits"]), np.ascontiguousarray(d_r["pen_logits"])
        diff = (ga.view(np.uint32) != ra.view(np.uint32)) & ~(np.isnan(ga) & np.isnan(ra))
        bad = np.argwhere(diff)
        assert bad.shape[0] == 0, f"{label}: {bad.shape[0]} penalised logits differ, first {bad[:3].tolist()}"
    frac = len(tolerated) / max(B, 1)
    assert frac <= max_boundary_frac, f"{label}: {len(tolerated)}/{B} boundary rows"
    return tolerated


def report(name, **kv):
    """Parity figures of a full-size case: printed, and appended as a JSON line
    to $MS_PARITY_REPORT when that is set."""
    line = dict(case=name, **kv)
    print(json.dumps(line))
    path = os.environ.get("MS_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(line) + "\n")


# ------------------------------------------------------------------ known answers
@pytest.mark.parametrize("case", KAT, ids=[c["name"] for c in KAT])
def test_known_answers_on_gpu(sampler, case):
    from minisample import SampleParams

    p = case["params"]
    sp = SampleParams(bool(p["do_sample"]), p["temperature"], int(p["top_k"]), p["top_p"], p["repetition_penalty"])
    x = case["logits"].reshape(1, -1)
    hist = np.array(case["hist"], np.int32) if case["hist"] else None
    off = np.array([0, len(case["hist"])], np.int64) if case["hist"] else None
    ids = sampler.sample(x, sp, u=np.array([case["u"]]), hist=hist, hist_off=off)
    assert int(ids[0]) == case["expected_id"], case["why"]


# ------------------------------------------------------------------ edge shapes
EDGE_V = [1, 2, 3, 5, 31, 33, 4097, 16384, 16385, 50257]


def edge_params():
    from minisample import SampleParams

    return {
        "greedy": SampleParams(False, 1.0, 50, 0.95, 1.3),
        "topk5": SampleParams(True, 0.8, 5, 0.95, 1.1),
        "topk50_nop": SampleParams(True, 1.3, 50, 0.0, 1.0),
        "full_topp": SampleParams(True, 1.0, 0, 0.9, 1.0),
        "full_nopen_nop": SampleParams(True, 0.6, 0, 1.0, 1.0),
        "k_ge_V": SampleParams(True, 1.0, 1 << 20, 0.8, 1.2),
        "k300": SampleParams(True, 0.9, 300, 0.95, 1.2),
        "topp_neg": SampleParams(True, 1.0, 40, -0.5, 1.0),
    }


@pytest.mark.parametrize("V", EDGE_V)
@pytest.mark.parametrize("pname", list(edge_params().keys()))
def test_edge_shapes(oracle, sampler, V, pname):
    sp = edge_params()[pname]
    rng = np.random.default_rng(V * 31 + len(pname))
    for B in (1, 3):
        X = rng.normal(0, 2, (B, V)).astype(np.float32)
        H = 12
        hist = rng.integers(-3, V + 3, B * H).astype(np.int32)  # out-of-range ids are no-ops
        hist[::5] = hist[0]                                       # duplicates count once
        off = np.arange(0, (B + 1) * H, H, dtype=np.int64)
        u = rng.random(B)
        u[0] = 0.0
        ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, sp, u, hist, off)
        check(ids_r, d_r, ids_g, d_g, sp, f"V{V} B{B} {pname}", max_boundary_frac=0.34)


def test_u_near_one_and_zero(oracle, sampler):
    from minisample import SampleParams

    sp = SampleParams(True, 0.8, 50, 0.95, 1.0)
    rng = np.random.default_rng(1)
    X = rng.normal(0, 2, (6, 4097)).astype(np.float32)
    u = np.array([0.0, 1e-300, 0.5, 1 - 2**-32, 0.999999, 0.25])
    ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, sp, u)
    check(ids_r, d_r, ids_g, d_g, sp, "u-extremes")


def test_nan_inf_rows(oracle, sampler):
    from minisample import SampleParams

    rng = np.random.default_rng(2)
    V = 20000
    X = rng.normal(0, 1, (6, V)).astype(np.float32)
    X[0, 777] = np.nan
    X[1, 19999] = np.inf
    X[2, :] = -np.inf
    X[3, :100] = -np.inf
    X[4, 0] = np.nan
    for sp in (SampleParams(True, 0.7, 30, 0.9, 1.0), SampleParams(True, 1.0, 0, 0.9, 1.0),
               SampleParams(False, 1.0, 30, 0.9, 1.0)):
        ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, sp, rng.random(6))
        np.testing.assert_array_equal(ids_g, ids_r)


def test_ties_and_constant_rows(oracle, sampler):
    """Heavy ties: quantised logits, a constant row (every element a candidate,
    chunk lists overflow), and ties straddling the top-k boundary."""
    from minisample import SampleParams

    rng = np.random.default_rng(3)
    V = 40000
    X = np.round(rng.normal(0, 1, (5, V)) * 4).astype(np.float32) / 4
    X[1] = 0.5
    X[2, :] = -3.0
    X[2, rng.choice(V, 70, replace=False)] = 2.0      # 70 tied maxima, top_k 64
    X[3] = np.float32(1e-3) * rng.integers(0, 3, V).astype(np.float32)
    for sp in (SampleParams(True, 1.0, 64, 0.9, 1.0), SampleParams(True, 0.9, 10, 1.0, 1.0),
               SampleParams(True, 1.0, 0, 0.5, 1.0), SampleParams(False)):
        u = rng.random(5)
        ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, sp, u)
        check(ids_r, d_r, ids_g, d_g, sp, f"ties k{sp.top_k}", max_boundary_frac=0.2)


def test_row_stride_and_device_pointers(oracle, sampler):
    import torch
    from minisample import SampleParams

    sp = SampleParams(True, 0.9, 64, 0.9, 1.2)
    rng = np.random.default_rng(4)
    V, B = 70001, 4
    big = rng.normal(0, 2, (B, V + 15)).astype(np.float32)
    X = big[:, :V]                                     # row stride V+15 (unaligned rows)
    hist = rng.integers(0, V, B * 50).astype(np.int32)
    off = np.arange(0, (B + 1) * 50, 50, dtype=np.int64)
    u = rng.random(B)
    ids_host = sampler.sample(X, sp, u=u, hist=hist, hist_off=off)
    ids_r, _ = oracle.sample_batch(np.ascontiguousarray(X), hist, off, params(oracle, sp), u)
    np.testing.assert_array_equal(ids_host, ids_r)
    tX = torch.from_numpy(big).cuda()[:, :V]
    ids_dev = sampler.sample(tX, sp, u=torch.from_numpy(u).cuda(), hist=torch.from_numpy(hist).cuda(),
                             hist_off=torch.from_numpy(off).cuda())
    np.testing.assert_array_equal(ids_dev.cpu().numpy(), ids_r)


# ------------------------------------------------------------------ benchmark workloads
def _workload(name, B, seed=11):
    from minisample import workloads as W

    w = W.WORKLOADS[name]
    X = W.logits_np(w, seed, B=B)
    hist, off = W.history_np(w, seed, B=B)
    u = W.uniforms(seed, B)
    return w, X, hist, off, u


@pytest.mark.parametrize("name", ["llama3_b64_greedy", "llama3_b64", "qwen2_b256", "gemma_b512", "vocab_sharded"])
def test_workload_parity_full_batch(oracle, sampler, name):
    """Every row of the workload's full batch against the oracle: ids,
    penalised logits (bit-exact), row max and sum, candidate lists (for
    whole-vocabulary rows too), n_cand and total; the boundary rows are
    reported."""
    from minisample import workloads as W

    w = W.WORKLOADS[name]
    w_, X, hist, off, u = _workload(name, w.B, seed=5)
    t0 = time.time()
    ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, w.params, u, hist, off)
    tol = check(ids_r, d_r, ids_g, d_g, w.params, name)
    flags = d_g["row_flags"]
    report(name, rows=int(w.B), vocab=int(w.V), boundary_rows=len(tol), boundary_frac=len(tol) / w.B,
           id_mismatch=int(np.sum(ids_r != ids_g)), fullvocab_rows=int(np.sum((flags & 0x4) != 0)),
           slowpath_rows=int(np.sum((flags & 0x8) != 0)), seconds=round(time.time() - t0, 1))


@pytest.mark.parametrize("name,B", [("gpt2_b1", 16), ("llama3_b64", 16), ("gemma_b512", 16)])
def test_topk_rows_stay_on_candidate_path(oracle, sampler, name, B):
    """Rows with top_k <= 256 on these distributions are finalized from the
    chunk candidates, without the exact rescan (row flag 0x8), including a
    vocabulary whose last chunk is short (50257 = 3 * 16384 + 1105)."""
    w, X, hist, off, u = _workload(name, B)
    ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, w.params, u, hist, off)
    check(ids_r, d_r, ids_g, d_g, w.params, name)
    slow = int(np.sum((d_g["row_flags"] & 0x8) != 0))
    assert slow == 0, f"{name}: {slow}/{B} rows took the rescan"


@pytest.mark.parametrize("tail", [1, 63, 64, 65, 700, 1105, 2047, 2048, 2049])
@pytest.mark.parametrize("k", [50, 256])
def test_short_last_chunk(oracle, sampler, tail, k):
    """Rows of 2 full chunks plus a short one, against the oracle."""
    from minisample import SampleParams

    rng = np.random.default_rng(tail * 7 + k)
    V = 2 * 16384 + tail
    X = rng.normal(0.0, 2.0, (6, V)).astype(np.float32)
    X[1, -tail:] += 6.0          # the short chunk holds the largest logits
    X[2, : 2 * 16384] = -np.inf  # only the short chunk is finite
    sp = SampleParams(True, 0.8, k, 0.9, 1.0)
    u = rng.random(6)
    ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, sp, u)
    check(ids_r, d_r, ids_g, d_g, sp, f"tail {tail} k {k}", max_boundary_frac=0.34)
    if k == 50 and tail >= 700:  # a short last chunk still bounds its candidates
        assert not d_g["row_flags"][0] & 0x8, d_g["row_flags"]


def test_gpt2_b1_generation_loop(oracle, sampler):
    """256 single-row steps, history = 64 prior ids + ids sampled so far; the
    penalty starts once something was generated (src/generation.js:73)."""
    from minisample import workloads as W

    w = W.WORKLOADS["gpt2_b1"]
    rng = np.random.default_rng(21)
    prior = rng.integers(0, w.V, 64).astype(np.int32)
    us = W.mulberry32(2024, w.steps)
    generated = []  # the oracle's ids drive the history of both sides
    tolerated = 0
    for step in range(w.steps):
        x = W.logits_np(w, 1000 + step, B=1)
        h = np.concatenate([prior, np.array(generated, np.int32)]) if generated else None
        r_id, d = oracle.pick_token(x[0], h, params(oracle, w.params), us[step])
        g_id = int(sampler.sample(x, w.params, u=us[step:step + 1], hist=h,
                                  hist_off=None if h is None else np.array([0, len(h)], np.int64))[0])
        if r_id != g_id:
            assert d["margin_draw"] < BOUNDARY or d["margin_cut"] < BOUNDARY, step
            tolerated += 1
        generated.append(r_id)
    assert tolerated <= 2


def test_gemma_b512_rows_mostly_on_candidate_path(oracle, sampler):
    """The headline workload's rows are settled from the chunk candidates: at
    most a handful take the exact rescan."""
    w, X, hist, off, u = _workload("gemma_b512", 512, seed=5)
    ids_g, d_g = sampler.sample(X, w.params, u=u, hist=hist, hist_off=off, diag=True)
    slow = int(np.sum((d_g["row_flags"] & 0x8) != 0))
    assert slow <= 8, slow


def test_repeatable(sampler):
    w, X, hist, off, u = _workload("gemma_b512", 16)
    a = sampler.sample(X, w.params, u=u, hist=hist, hist_off=off)
    b = sampler.sample(X, w.params, u=u, hist=hist, hist_off=off)
    np.testing.assert_array_equal(a, b)


def test_default_stream_ordering(sampler):
    """A device call on torch's default stream without MS_SYNC must stay ordered
    with the next torch operation on that stream (the wrapper names the legacy
    default stream explicitly; a NULL stream would mean the library's own)."""
    import torch

    from minisample import workloads as W

    w = W.WORKLOADS["gemma_b512"]
    dev = torch.device("cuda", 0)
    x = W.logits_torch(w, 2, dev, B=256)
    h, o = W.history_np(w, 2, B=256)
    hd, od = torch.from_numpy(h).to(dev), torch.from_numpy(o).to(dev)
    u = torch.from_numpy(W.uniforms(2, 256)).to(dev)
    ref = sampler.sample(x, w.params, u=u, hist=hd, hist_off=od).clone()
    for _ in range(3):
        out = torch.full((256,), -1, dtype=torch.int32, device=dev)
        sampler.sample(x, w.params, u=u, hist=hd, hist_off=od, out=out, sync=False)
        got = out.clone()  # queued right behind the sampler's kernels
        assert torch.equal(got, ref)


@pytest.mark.parametrize("pen", [0.5, 0.8, 1.2, 3.0])
@pytest.mark.parametrize("H", [40, 2500, 5000])
def test_penalty_edge_histories(oracle, sampler, pen, H):
    """The repetition penalty on top-k calls: rows where it lowers the maximum
    (pen > 1), raises low values above the candidates (pen < 1), hits every top
    candidate, or repeats ids; short and long histories, including ids outside
    the vocabulary."""
    from minisample import SampleParams

    rng = np.random.default_rng(int(pen * 100) + H)
    B, V = 6, 70000
    X = rng.normal(0.0, 2.0, (B, V)).astype(np.float32)
    X[3] = np.float32(-5.0)  # a row of equal values with a few peaks
    X[3, rng.choice(V, 50, replace=False)] = np.float32(4.0)
    rows = []
    for r in range(B):
        h = rng.integers(-2, V + 2, H)
        if r == 1:  # the row's largest logits are all in the history
            h[: min(H, 300)] = np.argsort(-X[r])[: min(H, 300)]
        if r == 2:  # low values that a penalty < 1 lifts toward the top
            h[: min(H, 200)] = np.argsort(X[r])[: min(H, 200)]
        h[::7] = h[0]  # repeats count once
        rows.append(h.astype(np.int32))
    hist = np.concatenate(rows)
    off = np.arange(0, (B + 1) * H, H, dtype=np.int64)
    u = rng.random(B)
    for sp in (SampleParams(True, 0.9, 64, 0.9, pen), SampleParams(True, 1.3, 8, 1.0, pen)):
        ids_r, d_r, ids_g, d_g = run_both(oracle, sampler, X, sp, u, hist, off)
        check(ids_r, d_r, ids_g, d_g, sp, f"pen {pen} H {H} k {sp.top_k}", max_boundary_frac=0.34)
