"""Seeded synthetic sampling workloads with the five shapes of the sampler benchmark.

The reference publishes no benchmark and uses no dataset; these generators
stand in with the stated shapes and value distributions:

  gpt2_b1        B=1,    V=50257   N(0, 2.5^2) + 5 ids boosted by +8; 64-id history
                                   T 0.8, top_k 50, top_p 0.95, penalty 1.1; 256 steps
  llama3_b64     B=64,   V=128256  Zipf-like -1.1*ln(rank) + N(0, 0.5^2); 256-id history
                                   greedy, and T 0.7, top_k 40, top_p 0.9, penalty 1.15
  qwen2_b256     B=256,  V=151936  50% flat N(0,1) rows, 50% peaked (one id +12); no history
                                   T 1.0, top_k 0, top_p 0.95
  gemma_b512     B=512,  V=262144  Zipf-like; 2048-id history, 10% repeats
                                   T 0.9, top_k 64, top_p 0.9, penalty 1.2
  vocab_sharded  B=1024, V=262144  Zipf-like, split into G vocab shards; 512-id history
                                   T 0.8, top_k 50, top_p 0.9, penalty 1.1

Uniforms are mulberry32(seed) draws k / 2^32 (test/synth.mjs:10-17), one per
sampled row in row order.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .sampler import SampleParams


@dataclass(frozen=True)
class Workload:
    name: str
    B: int
    V: int
    params: SampleParams
    hist_len: int
    kind: str            # "normal_boost" | "zipf" | "flat_peaked"
    repeat_frac: float = 0.0
    steps: int = 1


WORKLOADS = {
    "gpt2_b1": Workload("gpt2_b1", 1, 50257, SampleParams(True, 0.8, 50, 0.95, 1.1), 64, "normal_boost",
                        steps=256),
    "llama3_b64_greedy": Workload("llama3_b64_greedy", 64, 128256, SampleParams(False, 1.0, 50, 0.95, 1.15),
                                  256, "zipf"),
    "llama3_b64": Workload("llama3_b64", 64, 128256, SampleParams(True, 0.7, 40, 0.9, 1.15), 256, "zipf"),
    "qwen2_b256": Workload("qwen2_b256", 256, 151936, SampleParams(True, 1.0, 0, 0.95, 1.0), 0, "flat_peaked"),
    "gemma_b512": Workload("gemma_b512", 512, 262144, SampleParams(True, 0.9, 64, 0.9, 1.2), 2048, "zipf",
                           repeat_frac=0.1),
    "vocab_sharded": Workload("vocab_sharded", 1024, 262144, SampleParams(True, 0.8, 50, 0.9, 1.1), 512, "zipf"),
}


# ---------------------------------------------------------------- mulberry32
def mulberry32_u32(seed: int, n: int) -> np.ndarray:
    """n raw mulberry32 outputs; the state after k calls is seed + k*0x6d2b79f5."""
    a = (np.uint64(seed & 0xFFFFFFFF) + np.arange(1, n + 1, dtype=np.uint64) * np.uint64(0x6D2B79F5)) & np.uint64(
        0xFFFFFFFF)
    a = a.astype(np.uint32)
    with np.errstate(over="ignore"):
        t = (a ^ (a >> np.uint32(15))) * (a | np.uint32(1))
        t = (t + (t ^ (t >> np.uint32(7))) * (t | np.uint32(61))) ^ t
        return t ^ (t >> np.uint32(14))


def mulberry32(seed: int, n: int) -> np.ndarray:
    return mulberry32_u32(seed, n).astype(np.float64) / 4294967296.0


# ---------------------------------------------------------------- logits (numpy)
def zipf_rows(rng: np.random.Generator, B: int, V: int) -> np.ndarray:
    out = np.empty((B, V), np.float32)
    for r in range(B):
        ranks = rng.permutation(V).astype(np.float64) + 1.0
        out[r] = (-1.1 * np.log(ranks) + rng.normal(0.0, 0.5, V)).astype(np.float32)
    return out


def flat_peaked_rows(rng: np.random.Generator, B: int, V: int) -> np.ndarray:
    out = rng.normal(0.0, 1.0, (B, V)).astype(np.float32)
    peaked = rng.random(B) < 0.5
    for r in np.nonzero(peaked)[0]:
        out[r, rng.integers(0, V)] += np.float32(12.0)
    return out


def normal_boost_rows(rng: np.random.Generator, B: int, V: int) -> np.ndarray:
    out = rng.normal(0.0, 2.5, (B, V)).astype(np.float32)
    for r in range(B):
        out[r, rng.choice(V, 5, replace=False)] += np.float32(8.0)
    return out


def logits_np(w: Workload, seed: int, B: int | None = None) -> np.ndarray:
    rng = np.random.default_rng(seed)
    B = w.B if B is None else B
    if w.kind == "zipf":
        return zipf_rows(rng, B, w.V)
    if w.kind == "flat_peaked":
        return flat_peaked_rows(rng, B, w.V)
    return normal_boost_rows(rng, B, w.V)


def history_np(w: Workload, seed: int, B: int | None = None, H: int | None = None):
    """CSR history (ids int32, offsets int64[B+1]); ids uniform over V, with
    `repeat_frac` of the positions repeating an earlier entry of the row."""
    B = w.B if B is None else B
    H = w.hist_len if H is None else H
    if H == 0:
        return None, None
    rng = np.random.default_rng(seed + 7777)
    ids = rng.integers(0, w.V, (B, H)).astype(np.int32)
    if w.repeat_frac > 0:
        rep = rng.random((B, H)) < w.repeat_frac
        rep[:, 0] = False
        rows, cols = np.nonzero(rep)
        src = (rng.random(rows.shape[0]) * cols).astype(np.int64)
        ids[rows, cols] = ids[rows, src]
    off = np.arange(0, (B + 1) * H, H, dtype=np.int64)
    return ids.reshape(-1), off


def uniforms(seed: int, B: int) -> np.ndarray:
    return mulberry32(seed, B)


# ---------------------------------------------------------------- logits (torch, on device)
def logits_torch(w: Workload, seed: int, device, B: int | None = None):
    """The same distributions generated on the GPU (for full-size benchmarks)."""
    import torch

    B = w.B if B is None else B
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if w.kind == "zipf":
        out = torch.empty((B, w.V), dtype=torch.float32, device=device)
        step = max(1, (1 << 26) // w.V)
        for r0 in range(0, B, step):
            r1 = min(B, r0 + step)
            ranks = torch.argsort(torch.rand((r1 - r0, w.V), generator=g, device=device), dim=1).to(torch.float64) + 1
            noise = torch.randn((r1 - r0, w.V), generator=g, device=device, dtype=torch.float64) * 0.5
            out[r0:r1] = (-1.1 * torch.log(ranks) + noise).to(torch.float32)
        return out
    if w.kind == "flat_peaked":
        out = torch.randn((B, w.V), generator=g, device=device, dtype=torch.float32)
        peaked = torch.rand(B, generator=g, device=device) < 0.5
        ids = torch.randint(0, w.V, (B,), generator=g, device=device)
        rows = torch.nonzero(peaked).flatten()
        out[rows, ids[rows]] += 12.0
        return out
    out = torch.randn((B, w.V), generator=g, device=device, dtype=torch.float32) * 2.5
    ids = torch.randint(0, w.V, (B, 5), generator=g, device=device)
    out.scatter_add_(1, ids, torch.full((B, 5), 8.0, device=device))
    return out
