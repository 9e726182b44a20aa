"""minisample — B200 token sampler for mini.js (src/generation.js pickToken) behind libminisample.

  Sampler / SampleParams   batched sampling through the C ABI (include/minisample.h)
  generation               normalize_options / pick_token / generate_tokens mirroring
                           src/generation.js on the 'cuda' backend
  workloads                seeded synthetic logits of the benchmark shapes
  sharding                 row shards, and vocabulary shards exchanging records over NCCL
"""
from ._native import LIB_PATH, MiniSampleError, load  # noqa: F401
from .sampler import SampleParams, Sampler, record_bytes, scratch_bytes  # noqa: F401

__all__ = ["Sampler", "SampleParams", "MiniSampleError", "load", "scratch_bytes", "record_bytes", "LIB_PATH"]
