#!/usr/bin/env python
"""Sampler benchmark: sampled rows/s of the fused B200 sampler on one of the
synthetic sampling workloads (default gemma_b512: batch 512 x vocab 262144,
T 0.9, top_k 64, top_p 0.9, repetition penalty 1.2 over a 2048-id history).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--workload NAME]

One process per GPU (torchrun for N > 1).  Rows are independent, so every rank
samples its own batch with no collective ("weak" scaling; --strong splits one
global batch instead).  Prints ONE JSON line on rank 0.

  value      rows/s over all ranks, logits already in HBM, device-timed (CUDA
             events on the sampler's stream, max over ranks)
  e2e        the same metric through the public host-pointer call: pinned host
             logits copied in, ids copied out, every step
  roofline   algorithmic bytes (4 * V per row, logits read once) per launch of
             the dominant chunk kernel / its event-timed duration, against the
             measured HBM copy bandwidth
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
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "omni.js_b200"))

L2_BYTES = 126 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="minisample", choices=["minisample", "reference"])
    ap.add_argument("--workload", default="gemma_b512")
    ap.add_argument("--strong", action="store_true", help="split one global batch over the ranks")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=1234)
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
class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.out = None

    def start(self):
        import torch

        sel = []
        try:
            uuid = str(torch.cuda.get_device_properties(self.dev).uuid)
            sel = ["-i", uuid if uuid.startswith("GPU-") else "GPU-" + uuid]
        except Exception:
            sel = []
        try:
            self.out = open(os.devnull, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"] + sel, stdout=subprocess.PIPE, stderr=self.out, text=True)
        except Exception:
            self.proc = None

    def stop(self, t0=None, t1=None):
        """Median SM clock and throttle reasons of the samples taken between
        wall times t0 and t1 (all samples if none fall inside)."""
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            text, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            text = ""
        import datetime

        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        samples = []
        for line in text.splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                sm, mx = float(f[2]), float(f[3])
            except ValueError:
                continue
            rs = {nm for nm, v in zip(names, f[6:10]) if v.lower().startswith("active")}
            samples.append((ts, sm, mx, rs))
        if not samples:
            return None
        inside = [x for x in samples if t0 is not None and t0 <= x[0] <= t1] or samples
        reasons = set()
        for x in inside:
            reasons |= x[3]
        return {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": max(x[2] for x in inside),
                "samples": len(inside), "in_window": len(inside) < len(samples) or t0 is None,
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's CPU sampler (the oracle port of src/generation.js; the
    JS itself cannot run on this machine) on the host cores, rank 0 only."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import ms_oracle
    from minisample import workloads as W

    w = W.WORKLOADS[args.workload]
    cores = os.cpu_count() or 1
    rows = max(2 * cores, 8)
    X = W.logits_np(w, args.seed, B=rows)
    hist, off = W.history_np(w, args.seed, B=rows)
    u = W.uniforms(args.seed, rows)
    p = ms_oracle.make_params(w.params.do_sample, w.params.temperature, w.params.top_k, w.params.top_p,
                              w.params.repetition_penalty)
    for _ in range(args.warmup):
        ms_oracle.sample_batch(X, hist, off, p, u, nthreads=cores, want_diag=False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ms_oracle.sample_batch(X, hist, off, p, u, nthreads=cores, want_diag=False)
    dt = (time.perf_counter() - t0) / args.steps
    value = rows / dt
    sample = f"{rows} rows of {args.workload} per step ({w.V} vocab), {cores} threads, oracle port"
    line = {
        "impl": "reference",
        "metric": "sampled rows/sec at batch x vocab",
        "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f64-on-f32", "data": "synthetic",
        "config": workload_config(w, w.B, world, args.strong),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(w, b_rank, world, strong):
    return {
        "workload": w.name, "batch_per_gpu": b_rank, "global_batch": b_rank * world if not strong else w.B,
        "vocab": w.V, "history_per_row": w.hist_len, "temperature": w.params.temperature,
        "top_k": w.params.top_k, "top_p": w.params.top_p, "repetition_penalty": w.params.repetition_penalty,
        "do_sample": w.params.do_sample, "parallelism": f"row-sharded x{world}, no collective",
    }


# ---------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist

    from minisample import Sampler
    from minisample import workloads as W

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = W.WORKLOADS[args.workload]
    b_rank = w.B
    if args.strong:
        b_rank = (w.B + world - 1) // world
        b_rank = max(0, min(b_rank, w.B - rank * b_rank))
    seed = args.seed + 7919 * rank
    row_bytes = w.V * 4
    nbuf = max(1, -(-2 * L2_BYTES // max(1, b_rank * row_bytes)))  # rotate inputs past L2
    xs = [W.logits_torch(w, seed + i, dev, B=b_rank) for i in range(nbuf)]
    hist_np, off_np = W.history_np(w, seed, B=b_rank)
    u_np = W.uniforms(seed, b_rank)
    h_d = o_d = None
    if hist_np is not None:
        h_d = torch.from_numpy(hist_np).to(dev)
        o_d = torch.from_numpy(off_np).to(dev)
    u_d = torch.from_numpy(u_np).to(dev)
    ids = torch.empty(b_rank, dtype=torch.int32, device=dev)
    sampler = Sampler()
    stream = torch.cuda.Stream(dev)

    def step(i, profile=False):
        sampler.sample(xs[i % nbuf], w.params, u=u_d, hist=h_d, hist_off=o_d, out=ids, sync=False,
                       stream=stream, profile=profile)

    def barrier():
        if world > 1:
            dist.barrier()

    for i in range(args.warmup):
        step(i)
    stream.synchronize()
    sampler.profile_read()

    clocks = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.5)  # the sampler's first samples
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
    clk = clocks.stop(w0, w1)
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    launches = sampler.launch_count() - n0
    chunk_ms, fin_ms, calls = sampler.profile_read()
    chunk_ms /= max(calls, 1)
    fin_ms /= max(calls, 1)
    if world > 1:
        t = torch.tensor([ms, chunk_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max, chunk_max = float(t[0]), float(t[1])
        tot = torch.tensor([float(b_rank)], dtype=torch.float64, device=dev)
        dist.all_reduce(tot)
        rows_total = float(tot[0])
    else:
        ms_max, chunk_max, rows_total = ms, chunk_ms, float(b_rank)
    value = rows_total / (ms_max / 1e3)

    # ---- end to end through the host-pointer call (pinned host buffers)
    x_host = xs[0].cpu().pin_memory()
    x_np = x_host.numpy()
    e2e_steps = max(1, args.e2e_steps)
    ids_h = np.empty(b_rank, np.int32)
    sampler.sample(x_np, w.params, u=u_np, hist=hist_np, hist_off=off_np, out=ids_h)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        sampler.sample(x_np, w.params, u=u_np, hist=hist_np, hist_off=off_np, out=ids_h)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    barrier()
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t[0])
    ref_ids = ids.cpu().numpy()  # last device result (same logits buffer index may differ)
    del ref_ids
    h2d = x_np.nbytes + (hist_np.nbytes + off_np.nbytes if hist_np is not None else 0) + u_np.nbytes
    d2h = ids_h.nbytes

    # ---- CPU baseline (rank 0, N = 1): oracle on a bounded sample of the same rows
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import ms_oracle

        cores = os.cpu_count() or 1
        rows = min(b_rank, max(8, 2 * cores))
        Xs = xs[0][:rows].cpu().numpy()
        hs = os_ = None
        if hist_np is not None:
            hs = hist_np[: off_np[rows]]
            os_ = off_np[: rows + 1]
        p = ms_oracle.make_params(w.params.do_sample, w.params.temperature, w.params.top_k, w.params.top_p,
                                  w.params.repetition_penalty)
        n_done, t_cpu = 0, 0.0
        while t_cpu < 8.0 and n_done < 16 * rows:
            t0 = time.perf_counter()
            ms_oracle.sample_batch(Xs, hs, os_, p, u_np[:rows], nthreads=cores, want_diag=False)
            t_cpu += time.perf_counter() - t0
            n_done += rows
        cpu = {"value": n_done / t_cpu, "unit": "rows/s", "cores": cores, "kind": "port",
               "sample": f"{rows} rows of the same logits, repeated {n_done // rows}x, {cores} threads"}

    peak, peak_src = measured_peaks()
    bytes_launch = float(b_rank) * w.V * 4
    achieved = bytes_launch / (chunk_ms / 1e3) / 1e9 if chunk_ms > 0 else 0.0
    traffic = committed_traffic(w.name)
    line = {
        "metric": "sampled rows/sec at batch x vocab",
        "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong" if args.strong else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(workload_config(w, b_rank, world, args.strong),
                       l2=f"inputs larger than L2: {nbuf} rotating buffer(s) of {b_rank * row_bytes / 2**20:.0f} MiB"),
        "tokens_per_s": value,
        "step_hbm_gbs": bytes_launch * world / (ms_max / 1e3) / 1e9 if not args.strong else None,
        "kernel_ms": {"chunk": chunk_ms, "finalize": fin_ms},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "note": f"peak {peak_src}; chunk kernel, {b_rank}x{w.V}x4 B per launch"},
        "e2e": {"value": rows_total / e2e_s, "unit": "rows/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
