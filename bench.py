#!/usr/bin/env python
"""Sampler benchmark: sampled rows/s of the B200 sampler on one of the synthetic
sampling workloads (default gemma_b512: batch 512 x vocab 262144, T 0.9,
top_k 64, top_p 0.9, repetition penalty 1.2 over a 2048-id history).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--workload NAME]
                  [--weak] [--no-vocab-shards]

One process per GPU (torchrun for N > 1).  Rows are independent, so the
workload's batch is split over the ranks in contiguous row blocks with no
collective ("strong" scaling: 64 rows per GPU at N = 8 for gemma_b512); the
line also carries the weak figure (every rank samples a whole batch) as
`weak`.  --weak makes the weak figure the headline.  The vocab_sharded
workload at N > 1 splits the vocabulary instead (each rank holds V/N columns of
every row; shard records, an NCCL all-to-all, a merge and an all-gather of
the ids per step).  Prints ONE JSON line on rank 0.

  value      rows/s over all ranks, logits already in HBM, device-timed (CUDA
             events on the sampler's stream, max over ranks)
  e2e        the same metric through the public host-pointer call: pinned host
             logits copied in, ids copied out, every step
  roofline   algorithmic bytes (4 * V per row, logits read once) per launch of
             the dominant chunk kernel / its event-timed duration, against the
             measured HBM copy bandwidth
  parity     32 rows of the last timed step checked against the oracle
  cpu_baseline  the oracle port of src/generation.js on the host cores (a
             bounded sample of the same rows)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "omni.js_b200"))

L2_BYTES = 126 * 1024 * 1024
VERIFY_ROWS = 32


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="minisample", choices=["minisample", "reference"])
    ap.add_argument("--workload", default="gemma_b512")
    ap.add_argument("--weak", action="store_true", help="every rank samples a whole batch (headline = weak)")
    ap.add_argument("--no-vocab-shards", action="store_true", help="vocab_sharded workload: split rows instead")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--rows", type=int, default=0,
                    help="one GPU: sample only the first ROWS rows of the batch (a smaller case of the same "
                         "kernels, for profiling captures); the line's config says so")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic(workload):
    """DRAM bytes per chunk-kernel launch from a committed ncu summary (or None)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    return d.get(workload)


# ---------------------------------------------------------------- clocks
REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
           ("sw_power_cap", 0x4))


class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled from a thread in
    this process (NVML, every ~0.5 ms) so that even a timed region of a few
    milliseconds holds samples.  Falls back to `nvidia-smi -lms 50`."""

    def __init__(self, device_index):
        self.dev = device_index
        self.samples = []
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def _uuid(self):
        import torch

        try:
            u = str(torch.cuda.get_device_properties(self.dev).uuid)
            return u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            return None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = self._uuid()
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid) if uuid else pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def run():
                while not self._stop.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:
                        break
                    self.samples.append((time.time(), float(sm), float(mx), int(rs)))
                    time.sleep(0.0005)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
            return
        except Exception:
            self._thread = None
        fields = ("timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.active")
        sel = ["-i", self._uuid()] if self._uuid() else []
        try:
            self._proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                           "-lms", "50"] + sel, stdout=subprocess.PIPE,
                                          stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._proc = None

    def stop(self, t0=None, t1=None):
        """Median SM clock and clock-event reasons of the samples taken between
        wall times t0 and t1 (all samples if none fall inside)."""
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
            src = "nvml"
        elif self._proc is not None:
            self._proc.terminate()
            try:
                text, _ = self._proc.communicate(timeout=5)
            except Exception:
                self._proc.kill()
                text = ""
            import datetime

            for line in text.splitlines():
                f = [c.strip() for c in line.split(",")]
                try:
                    ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    self.samples.append((ts, float(f[1]), float(f[2]), int(f[3], 16)))
                except (ValueError, IndexError):
                    continue
            src = "nvidia-smi"
        else:
            return None
        if not self.samples:
            return None
        inside = [x for x in self.samples if t0 is not None and t0 <= x[0] <= t1]
        use = inside or self.samples
        reasons = set()
        for x in use:
            reasons |= {nm for nm, bit in REASONS if x[3] & bit}
        return {"sm_mhz": statistics.median(x[1] for x in use), "sm_max_mhz": max(x[2] for x in use),
                "samples": len(use), "in_window": bool(inside), "source": src, "reasons": sorted(reasons)}


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's CPU sampler (the oracle port of src/generation.js; no
    JavaScript engine exists on these machines) on the host cores, rank 0
    only.  Each step samples the workload's whole batch when the run fits in
    a few minutes, else a fixed sample of its rows (stated in the line)."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ms_oracle
    from minisample import workloads as W

    w = W.WORKLOADS[args.workload]
    cores = os.cpu_count() or 1
    p = ms_oracle.make_params(w.params.do_sample, w.params.temperature, w.params.top_k, w.params.top_p,
                              w.params.repetition_penalty)
    probe = min(w.B, 2 * cores)
    Xp = W.logits_np(w, args.seed, B=probe)
    hp, op = W.history_np(w, args.seed, B=probe)
    t0 = time.perf_counter()
    ms_oracle.sample_batch(Xp, hp, op, p, W.uniforms(args.seed, probe), nthreads=cores, want_diag=False)
    rate = probe / max(time.perf_counter() - t0, 1e-6)
    budget_s = 150.0
    rows = int(min(w.B, max(probe, rate * budget_s / max(1, args.steps + args.warmup))))
    X = Xp if rows == probe else W.logits_np(w, args.seed, B=rows)
    hist, off = (hp, op) if rows == probe else W.history_np(w, args.seed, B=rows)
    u = W.uniforms(args.seed, rows)
    for _ in range(args.warmup):
        ms_oracle.sample_batch(X, hist, off, p, u, nthreads=cores, want_diag=False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ms_oracle.sample_batch(X, hist, off, p, u, nthreads=cores, want_diag=False)
    dt = (time.perf_counter() - t0) / args.steps
    value = rows / dt
    whole = rows == w.B
    sample = (f"the whole batch of {w.B} rows per step" if whole else
              f"{rows} of the batch's {w.B} rows per step") + f" ({w.V} vocab), {cores} threads, oracle port"
    cfg = workload_config(w, rows if not whole else w.B, 1, rows)
    cfg["parallelism"] = f"{cores} host threads over rows"
    line = {
        "impl": "reference",
        "metric": "sampled rows/sec at batch x vocab",
        "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f64-on-f32", "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(w, b_rank, world, global_batch, parallelism=None):
    return {
        "workload": w.name, "batch_per_gpu": b_rank, "global_batch": global_batch,
        "vocab": w.V, "history_per_row": w.hist_len, "temperature": w.params.temperature,
        "top_k": w.params.top_k, "top_p": w.params.top_p, "repetition_penalty": w.params.repetition_penalty,
        "do_sample": w.params.do_sample,
        "parallelism": parallelism or f"rows split over {world} GPU(s), no collective",
    }


# ---------------------------------------------------------------- our arm: helpers
def verify_rows(w, X_dev, hist_np, off_np, u_np, ids_dev, rows=VERIFY_ROWS):
    """Checks the first `rows` ids of a timed step against the oracle on the
    same bytes (ids may differ only where the oracle's draw or top-p sum lies
    within 1e-6 of a cumulative boundary)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ms_oracle

    n = min(rows, X_dev.shape[0])
    X = X_dev[:n].cpu().numpy()
    hs = os_ = None
    if hist_np is not None:
        hs, os_ = hist_np[: off_np[n]], off_np[: n + 1]
    p = ms_oracle.make_params(w.params.do_sample, w.params.temperature, w.params.top_k, w.params.top_p,
                              w.params.repetition_penalty)
    ref, d = ms_oracle.sample_batch(X, hs, os_, p, u_np[:n])
    got = ids_dev[:n].cpu().numpy()
    miss = [r for r in range(n) if got[r] != ref[r]]
    boundary = [r for r in miss if d["margin_draw"][r] < 1e-6 or d["margin_cut"][r] < 1e-6]
    return {"rows_checked": n, "id_mismatch": len(miss), "boundary_rows": len(boundary),
            "verified": len(miss) == len(boundary)}


def max_over_ranks(vals, dev, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return list(vals)
    t = torch.tensor(list(vals), dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def sum_over_ranks(v, dev, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return float(v)
    t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
    dist.all_reduce(t)
    return float(t[0])


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def time_rows(args, w, b_rank, seed, dev, world, local_rank, sampler, clocks=None, verify=False):
    """Device-timed sampling of b_rank rows per step on this rank.  Returns a
    dict of per-rank figures (not yet reduced over ranks)."""
    import torch

    from minisample import workloads as W

    row_bytes = w.V * 4
    out = {"b_rank": b_rank, "ms": 0.0, "chunk_ms": 0.0, "fin_ms": 0.0, "launches": 0, "nbuf": 0,
           "clk": None, "parity": None}
    # every rank takes the same collective steps, also with no rows
    nbuf = max(1, -(-2 * L2_BYTES // max(1, b_rank * row_bytes))) if b_rank else 0
    xs = [W.logits_torch(w, seed + i, dev, B=b_rank) for i in range(nbuf)]
    hist_np, off_np = W.history_np(w, seed, B=b_rank) if b_rank else (None, None)
    u_np = W.uniforms(seed, b_rank)
    h_d = o_d = None
    if hist_np is not None:
        h_d = torch.from_numpy(hist_np).to(dev)
        o_d = torch.from_numpy(off_np).to(dev)
    u_d = torch.from_numpy(u_np).to(dev)
    ids = torch.empty(b_rank, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)

    def step(i, profile=False):
        if b_rank:
            sampler.sample(xs[i % nbuf], w.params, u=u_d, hist=h_d, hist_off=o_d, out=ids, sync=False,
                           stream=stream, profile=profile)

    for i in range(args.warmup):
        step(i)
    stream.synchronize()
    sampler.profile_read()
    barrier(world)
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
        time.sleep(0.3)  # the sampler's first samples
    w0 = time.time()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    # every 8th step records kernel events (an event between the two kernels
    # keeps the finalize from starting early, so not every step carries one)
    n0 = sampler.launch_count()
    e0.record(stream)
    for i in range(args.steps):
        step(i, profile=(i % 8 == 0))
    e1.record(stream)
    stream.synchronize()
    w1 = time.time()
    if clocks is not None:
        out["clk"] = clocks.stop(w0, w1)
    barrier(world)
    out["ms"] = e0.elapsed_time(e1) / args.steps
    out["launches"] = sampler.launch_count() - n0
    chunk_ms, fin_ms, calls = sampler.profile_read()
    out["chunk_ms"] = chunk_ms / max(calls, 1)
    out["fin_ms"] = fin_ms / max(calls, 1)
    out["nbuf"] = nbuf
    if verify and b_rank:
        out["parity"] = verify_rows(w, xs[(args.steps - 1) % nbuf], hist_np, off_np, u_np, ids)
    out["xs0"] = xs[0] if b_rank else None
    out["hist_np"], out["off_np"], out["u_np"] = hist_np, off_np, u_np
    return out


def time_e2e(args, w, r, sampler, world):
    """End to end through the host-pointer call: pinned host logits in, ids
    out, every step."""
    import numpy as np

    b_rank = r["b_rank"]
    if not b_rank:
        barrier(world)
        barrier(world)
        return 0.0, 0, 0
    x_np = r["xs0"].cpu().pin_memory().numpy()
    hist_np, off_np, u_np = r["hist_np"], r["off_np"], r["u_np"]
    ids_h = np.empty(b_rank, np.int32)
    sampler.sample(x_np, w.params, u=u_np, hist=hist_np, hist_off=off_np, out=ids_h)
    barrier(world)
    t0 = time.perf_counter()
    n = max(1, args.e2e_steps)
    for _ in range(n):
        sampler.sample(x_np, w.params, u=u_np, hist=hist_np, hist_off=off_np, out=ids_h)
    e2e_s = (time.perf_counter() - t0) / n
    barrier(world)
    h2d = x_np.nbytes + (hist_np.nbytes + off_np.nbytes if hist_np is not None else 0) + u_np.nbytes
    return e2e_s, int(h2d), int(ids_h.nbytes)


def cpu_baseline(w, r):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ms_oracle

    cores = os.cpu_count() or 1
    b_rank = r["b_rank"]
    rows = min(b_rank, max(8, 2 * cores))
    Xs = r["xs0"][:rows].cpu().numpy()
    hs = os_ = None
    if r["hist_np"] is not None:
        hs, os_ = r["hist_np"][: r["off_np"][rows]], r["off_np"][: rows + 1]
    p = ms_oracle.make_params(w.params.do_sample, w.params.temperature, w.params.top_k, w.params.top_p,
                              w.params.repetition_penalty)
    n_done, t_cpu = 0, 0.0
    while t_cpu < 8.0 and n_done < 16 * rows:
        t0 = time.perf_counter()
        ms_oracle.sample_batch(Xs, hs, os_, p, r["u_np"][:rows], nthreads=cores, want_diag=False)
        t_cpu += time.perf_counter() - t0
        n_done += rows
    return {"value": n_done / t_cpu, "unit": "rows/s", "cores": cores, "kind": "port",
            "sample": f"{rows} rows of the same logits, repeated {n_done // rows}x, {cores} threads"}


# ---------------------------------------------------------------- our arm: row split
def run_ours(args, rank, world, local_rank):
    import torch

    from minisample import Sampler
    from minisample import workloads as W
    from minisample.sharding import row_shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = W.WORKLOADS[args.workload]
    sampler = Sampler()
    if args.weak:
        b_rank = w.B
    else:
        r0, r1 = row_shard(w.B, world, rank)
        b_rank = r1 - r0
    if args.rows > 0 and world == 1:
        b_rank = min(b_rank, args.rows)
    seed = args.seed + 7919 * rank
    clocks = ClockSampler(local_rank)
    r = time_rows(args, w, b_rank, seed, dev, world, local_rank, sampler, clocks=clocks,
                  verify=not args.no_verify and rank == 0)
    ms_max, chunk_max = max_over_ranks([r["ms"], r["chunk_ms"]], dev, world)
    rows_total = sum_over_ranks(b_rank, dev, world)
    value = rows_total / (ms_max / 1e3)
    launches = int(sum_over_ranks(r["launches"], dev, world))

    weak = None
    if world > 1 and not args.weak:  # the weak figure beside the strong one
        rw = time_rows(args, w, w.B, seed + 104729, dev, world, local_rank, sampler)
        wms, = max_over_ranks([rw["ms"]], dev, world)
        weak = {"value": w.B * world / (wms / 1e3), "ms_per_step": wms, "batch_per_gpu": w.B,
                "global_batch": w.B * world}
        del rw

    e2e_s, h2d, d2h = time_e2e(args, w, r, sampler, world)
    e2e_s, = max_over_ranks([e2e_s], dev, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, r)

    peak, peak_src = measured_peaks()
    bytes_launch = float(b_rank) * w.V * 4
    achieved = bytes_launch / (r["chunk_ms"] / 1e3) / 1e9 if r["chunk_ms"] > 0 else 0.0
    scaling = "weak" if args.weak else "strong"
    gb = w.B * world if args.weak else w.B
    if args.rows > 0 and world == 1:
        gb = b_rank
    line = {
        "metric": "sampled rows/sec at batch x vocab",
        "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(workload_config(w, b_rank, world, gb),
                       l2=f"inputs larger than L2: {r['nbuf']} rotating buffer(s) of "
                          f"{b_rank * w.V * 4 / 2**20:.0f} MiB per GPU"),
        "tokens_per_s": value,
        "step_hbm_gbs": rows_total * w.V * 4 / (ms_max / 1e3) / 1e9,
        "kernel_ms": {"chunk": r["chunk_ms"], "finalize": r["fin_ms"], "chunk_max_over_ranks": chunk_max},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": committed_traffic(w.name) if b_rank == w.B else None,
                     "note": f"peak {peak_src}; chunk kernel on rank 0, {b_rank}x{w.V}x4 B per launch"},
        "e2e": {"value": rows_total / e2e_s if e2e_s > 0 else 0.0, "unit": "rows/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": r["clk"],
        "parity": r["parity"],
    }
    if weak is not None:
        line["weak"] = weak
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)
    sampler.close()


# ---------------------------------------------------------------- our arm: vocabulary shards
def run_vocab_sharded(args, rank, world, local_rank):
    """Config 5: every rank holds V/world columns of all rows; per step the
    shard records, an NCCL all-to-all of the records, the merge of a block of
    rows, and an all-gather of the ids."""
    import numpy as np
    import torch

    from minisample import Sampler
    from minisample import workloads as W
    from minisample.sharding import col_shard, resolve_unsettled, sample_vocab_sharded

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = W.WORKLOADS[args.workload]
    B, V = w.B, w.V
    c0, c1 = col_shard(V, world, rank)
    sampler = Sampler()
    nbuf = max(1, -(-2 * L2_BYTES // max(1, B * (c1 - c0) * 4)))
    xs = []
    for i in range(nbuf):  # the same global logits on every rank; keep this rank's columns
        full = W.logits_torch(w, args.seed + i, dev, B=B)
        xs.append(full[:, c0:c1].contiguous())
        del full
    hist_np, off_np = W.history_np(w, args.seed, B=B)
    h_d = torch.from_numpy(hist_np).to(dev)
    o_d = torch.from_numpy(off_np).to(dev)
    u_np = W.uniforms(args.seed, B)
    u_d = torch.from_numpy(u_np).to(dev)

    def step(i, resolve=False):
        return sample_vocab_sharded(sampler, xs[i % nbuf], c0, V, w.params, u_d, h_d, o_d, resolve=resolve)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    w0 = time.time()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n0 = sampler.launch_count()
    e0.record()
    ids = None
    for i in range(args.steps):
        ids = step(i)
    e1.record()
    torch.cuda.synchronize()
    w1 = time.time()
    clk = clocks.stop(w0, w1)
    barrier(world)
    ms = e0.elapsed_time(e1) / args.steps
    launches = sampler.launch_count() - n0
    unsettled = int((ids < 0).sum().item())
    ids = resolve_unsettled(sampler, ids, xs[(args.steps - 1) % nbuf], w.params, u_d, h_d, o_d)
    ms_max, = max_over_ranks([ms], dev, world)
    launches = int(sum_over_ranks(launches, dev, world))
    value = B / (ms_max / 1e3)
    parity = None
    if not args.no_verify:
        # rank 0 checks 32 whole rows, gathered from the shards, against the oracle
        from minisample.sharding import gather_rows

        rows = gather_rows(xs[(args.steps - 1) % nbuf][:VERIFY_ROWS], None)
        if rank == 0:
            parity = verify_rows(w, rows, hist_np, off_np, u_np, ids)
        barrier(world)

    # end to end: this rank's pinned host shard in, ids out, every step
    x_host = xs[0].cpu().pin_memory()
    x_dev = torch.empty_like(xs[0])
    barrier(world)
    t0 = time.perf_counter()
    n = max(1, args.e2e_steps)
    for _ in range(n):
        x_dev.copy_(x_host, non_blocking=True)
        out = sample_vocab_sharded(sampler, x_dev, c0, V, w.params, u_d, h_d, o_d, resolve=True).cpu()
    e2e_s = (time.perf_counter() - t0) / n
    barrier(world)
    e2e_s, = max_over_ranks([e2e_s], dev, world)
    del out
    peak, peak_src = measured_peaks()
    bytes_rank = float(B) * (c1 - c0) * 4
    line = {
        "metric": "sampled rows/sec at batch x vocab",
        "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": dict(workload_config(w, B, world, B,
                                       f"vocabulary split over {world} GPU(s): {c1 - c0} columns per GPU; "
                                       "NCCL all-to-all of shard records + all-gather of ids"),
                       l2=f"inputs larger than L2: {nbuf} rotating buffer(s) of {bytes_rank / 2**20:.0f} MiB"),
        "tokens_per_s": value,
        "roofline": {"bound": "hbm", "achieved": bytes_rank / (ms_max / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": bytes_rank / (ms_max / 1e3) / 1e9 / peak, "traffic": None,
                     "note": f"peak {peak_src}; whole step per GPU (shard kernels + exchange), "
                             f"{B}x{c1 - c0}x4 B per GPU"},
        "e2e": {"value": B / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": int(x_host.numel() * 4),
                "d2h_bytes_per_step": int(B * 4)},
        "gpu_launches": launches,
        "unsettled_rows_last_step": unsettled,
        "clocks": clk,
        "parity": parity,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    sampler.close()


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "vocab_sharded" and world > 1 and not args.no_vocab_shards:
            run_vocab_sharded(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
