"""Host mirror of mini.js's generation API (src/generation.js) on the CUDA sampler.

Same names (snake_case), option normalisation, stopping rules and uniform-draw
discipline as the reference, so a caller switching from the JS sampler finds
the same behaviour:

  normalize_options  src/generation.js:57-68  (`??` keeps 0 / False, defaults
                     only None)
  pick_token         src/generation.js:71-81  (penalty only once something was
                     generated; one uniform per sampled step, none when greedy)
  generate_tokens    src/generation.js:97-114 (onToken(id, n) returning False
                     stops; EOS stops after it is appended)
  generate_async     src/generation.js:121-142

The backend is 'cuda' (libminisample).  Selecting it fails loudly when the
library or a GPU is missing; there is no CPU fallback on this path.
"""
from __future__ import annotations

import asyncio
import random as _random

import numpy as np

from .sampler import SampleParams, Sampler

_ACTIVE = None      # 'cuda' or None
_SAMPLER = None


def set_backend(name: str) -> str:
    """Select the sampler backend; only 'cuda' lives here (src/tensor.js:15-20)."""
    global _ACTIVE, _SAMPLER
    if name != "cuda":
        raise ValueError(f"[minisample] unknown backend: {name}")
    if _SAMPLER is None:
        _SAMPLER = Sampler()
    _ACTIVE = "cuda"
    return _ACTIVE


def current_backend() -> str:
    if _ACTIVE is None:
        set_backend("cuda")
    return _ACTIVE


def _sampler() -> Sampler:
    current_backend()
    return _SAMPLER


def _first(*vals, default):
    for v in vals:
        if v is not None:
            return v
    return default


def normalize_options(options: dict | None) -> dict:
    o = options or {}
    return {
        "max_new_tokens": _first(o.get("maxNewTokens"), o.get("max_new_tokens"), default=50),
        "do_sample": _first(o.get("doSample"), o.get("do_sample"), default=True),
        "temperature": _first(o.get("temperature"), default=1.0),
        "top_k": _first(o.get("topK"), o.get("top_k"), default=50),
        "top_p": _first(o.get("topP"), o.get("top_p"), default=0.95),
        "repetition_penalty": _first(o.get("repetitionPenalty"), o.get("repetition_penalty"), default=1.0),
        "eos_token_id": _first(o.get("eosTokenId"), o.get("eos_token_id"), default=None),
        "on_token": o.get("onToken") or o.get("on_token") or None,
    }


def params_of(opts: dict) -> SampleParams:
    return SampleParams(bool(opts["do_sample"]), float(opts["temperature"]), int(opts["top_k"]),
                        float(opts["top_p"]), float(opts["repetition_penalty"]))


def is_greedy(opts: dict) -> bool:
    return (not opts["do_sample"]) or float(opts["temperature"]) <= 0.0001


def pick_token(last_logits, generated, input_ids, opts, rand=_random.random):
    """Next id from one row of logits; returns [id, True] like the reference."""
    row = np.ascontiguousarray(np.asarray(last_logits, dtype=np.float32).reshape(1, -1))
    hist = hist_off = None
    if len(generated):
        h = np.asarray(list(input_ids) + list(generated), dtype=np.int64)
        # ids beyond int32 can never index the vocabulary: they are no-ops
        h = np.where((h < 0) | (h > 2**31 - 1), -1, h).astype(np.int32)
        hist = h
        hist_off = np.array([0, h.shape[0]], dtype=np.int64)
    u = None if is_greedy(opts) else np.array([rand()], dtype=np.float64)
    ids = _sampler().sample(row, params_of(opts), u=u, hist=hist, hist_off=hist_off)
    return [int(ids[0]), True]


def last_token_logits(model, input_ids, cache):
    """src/generation.js:83-90: the last row of model.forward(..., last_only=True)."""
    logits = np.asarray(model.forward(input_ids, cache=cache, last_only=True), dtype=np.float32)
    if logits.ndim == 2:
        logits = logits[-1]
    return logits


def generate_tokens(model, input_ids, options=None, rand=_random.random):
    opts = normalize_options(options)
    cache = model.make_cache()
    try:
        generated = []
        last = last_token_logits(model, input_ids, cache)
        for step in range(int(opts["max_new_tokens"])):
            next_id, _ = pick_token(last, generated, input_ids, opts, rand)
            generated.append(next_id)
            if opts["on_token"] and opts["on_token"](next_id, step + 1) is False:
                break
            if opts["eos_token_id"] is not None and next_id == opts["eos_token_id"]:
                break
            last = last_token_logits(model, [next_id], cache)
        return generated
    finally:
        model.dispose_cache(cache)


async def generate_async(model, input_ids, options=None, rand=_random.random):
    opts = normalize_options(options)
    tick = (options or {}).get("tick")
    cache = model.make_cache()
    try:
        generated = []
        last = last_token_logits(model, input_ids, cache)
        for step in range(int(opts["max_new_tokens"])):
            next_id, _ = pick_token(last, generated, input_ids, opts, rand)
            generated.append(next_id)
            if opts["on_token"] and opts["on_token"](next_id, step + 1) is False:
                break
            if opts["eos_token_id"] is not None and next_id == opts["eos_token_id"]:
                break
            if tick:
                await tick()
            else:
                await asyncio.sleep(0)
            last = last_token_logits(model, [next_id], cache)
        return generated
    finally:
        model.dispose_cache(cache)


def generate_tokens_batch(model, input_ids_batch, options=None, rands=None):
    """B sequences at once: one sampler call per step over the rows still
    running, each row with the rules of generate_tokens (the reference's
    roadmap item of batched generation, README.md:232; per row
    src/generation.js:97-114).  onToken(row, id, n) returning False stops that
    row; EOS stops a row after it is appended.  rands[i] draws row i's
    uniforms (one per sampled step of that row, none when greedy), so row i
    gets the ids generate_tokens would give it with rands[i].  `model` is one
    model for every row, or a list of one per row."""
    opts = normalize_options(options)
    B = len(input_ids_batch)
    models = model if isinstance(model, (list, tuple)) else [model] * B
    rands = rands if rands is not None else [_random.random] * B
    on_token = opts["on_token"]
    greedy = is_greedy(opts)
    params = params_of(opts)
    caches = [models[i].make_cache() for i in range(B)]
    try:
        generated = [[] for _ in range(B)]
        last = [last_token_logits(models[i], input_ids_batch[i], caches[i]) for i in range(B)]
        active = list(range(B))
        for step in range(int(opts["max_new_tokens"])):
            if not active:
                break
            X = np.ascontiguousarray(np.stack([last[i] for i in active]).astype(np.float32))
            hs, offs = [], [0]
            for i in active:
                if generated[i]:  # the penalty starts once the row generated something
                    h = np.asarray(list(input_ids_batch[i]) + generated[i], dtype=np.int64)
                    hs.append(np.where((h < 0) | (h > 2**31 - 1), -1, h).astype(np.int32))
                offs.append(offs[-1] + (hs[-1].shape[0] if generated[i] else 0))
            hist = np.concatenate(hs) if hs else np.zeros(0, np.int32)
            hist_off = np.asarray(offs, dtype=np.int64)
            u = None if greedy else np.array([rands[i]() for i in active], dtype=np.float64)
            ids = _sampler().sample(X, params, u=u, hist=hist, hist_off=hist_off)
            still = []
            for j, i in enumerate(active):
                nid = int(ids[j])
                generated[i].append(nid)
                if on_token and on_token(i, nid, step + 1) is False:
                    continue
                if opts["eos_token_id"] is not None and nid == opts["eos_token_id"]:
                    continue
                still.append(i)
            active = still
            for i in active:
                if step + 1 < int(opts["max_new_tokens"]):
                    last[i] = last_token_logits(models[i], [generated[i][-1]], caches[i])
        return generated
    finally:
        for i in range(B):
            models[i].dispose_cache(caches[i])


class DeviceHistory:
    """A batch's penalty histories kept on the GPU (ms_history_append).  Row r
    holds its prompt and generated ids in hist[r, :lens[r]] and -1 after them
    (the penalty ignores ids outside the vocabulary), so (hist, off) is a
    ready CSR history for the sampler.  The prompts are uploaded once; each
    step appends the sampled ids on the device (src/generation.js:73-74, 105)."""

    def __init__(self, input_ids_batch, cap: int, device):
        import torch

        B = len(input_ids_batch)
        h = np.full((B, cap), -1, np.int32)
        lens = np.zeros(B, np.int32)
        for i, ids in enumerate(input_ids_batch):
            a = np.asarray(list(ids), dtype=np.int64)[:cap]
            h[i, : a.shape[0]] = np.where((a < 0) | (a > 2**31 - 1), -1, a).astype(np.int32)
            lens[i] = a.shape[0]
        self.hist = torch.from_numpy(h).to(device)
        self.lens = torch.from_numpy(lens).to(device)
        self.off = torch.arange(0, (B + 1) * cap, cap, dtype=torch.int64, device=device)
        self.upload_bytes = h.nbytes + lens.nbytes + self.off.numel() * 8

    def append(self, sampler: Sampler, ids) -> None:
        sampler.history_append(self.hist, self.lens, ids)


def generate_tokens_device(model, input_ids_batch, options=None, rands=None):
    """Batched generation with the logits and the penalty history on the GPU.

    model.forward_batch(last_ids, caches) returns the [B, V] fp32 CUDA logits of
    the next step for every row (last_ids is None for the prompts; the logits
    come from the model's lm head on the device, so no logits cross the host
    link); model.make_cache() / dispose_cache(cache) as in generate_tokens.  Each
    step samples on the device, appends the ids to the device history, and
    copies only the B ids back for the onToken / EOS rules, which are those of
    generate_tokens_batch (per row, src/generation.js:97-114).  Rows that
    stopped keep a slot in the batch; their ids are ignored and draw no
    uniform.  Returns the generated ids of each row."""
    import torch

    opts = normalize_options(options)
    B = len(input_ids_batch)
    rands = rands if rands is not None else [_random.random] * B
    on_token = opts["on_token"]
    greedy = is_greedy(opts)
    params = params_of(opts)
    steps = int(opts["max_new_tokens"])
    s = _sampler()
    caches = [model.make_cache() for _ in range(B)]
    try:
        logits = model.forward_batch(None, caches)
        dev = logits.device
        cap = max(len(list(x)) for x in input_ids_batch) + max(steps, 1)
        H = DeviceHistory(input_ids_batch, cap, dev)
        ids_d = torch.empty(B, dtype=torch.int32, device=dev)
        generated = [[] for _ in range(B)]
        active = [True] * B
        for step in range(steps):
            if not any(active):
                break
            u = None
            if not greedy:
                u = torch.tensor([rands[i]() if active[i] else 0.0 for i in range(B)], dtype=torch.float64,
                                 device=dev)
            # the penalty starts once something was generated (src/generation.js:73)
            hist = (H.hist.view(-1), H.off) if step > 0 else (None, None)
            s.sample(logits, params, u=u, hist=hist[0], hist_off=hist[1], out=ids_d, sync=False)
            H.append(s, ids_d)
            ids = ids_d.cpu().numpy()
            for i in range(B):
                if not active[i]:
                    continue
                nid = int(ids[i])
                generated[i].append(nid)
                if on_token and on_token(i, nid, step + 1) is False:
                    active[i] = False
                elif opts["eos_token_id"] is not None and nid == opts["eos_token_id"]:
                    active[i] = False
            if step + 1 < steps and any(active):
                logits = model.forward_batch([int(x) for x in ids], caches)
        return generated
    finally:
        for c in caches:
            model.dispose_cache(c)
