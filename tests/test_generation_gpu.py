"""generate_tokens / generate_async (src/generation.js:97-142) on the 'cuda'
sampler with a stub model, against the same loop driven by the oracle: the
same ids, the same stopping rules (onToken returning false stops after the
call; EOS stops after it is appended), one uniform per sampled step and none
when greedy, penalty only once something was generated."""
import asyncio

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V = 5003


class StubModel:
    """model.forward(ids, cache, last_only) -> [1, V] logits that depend on the
    step and on the last id fed, as a real decoder's would."""

    def __init__(self, seed):
        self.seed = seed
        self.disposed = 0

    def make_cache(self):
        return {"step": 0}

    def dispose_cache(self, cache):
        self.disposed += 1

    def forward(self, ids, cache=None, last_only=True):
        rng = np.random.default_rng((self.seed, cache["step"], int(ids[-1])))
        cache["step"] += 1
        x = rng.normal(0.0, 2.0, (1, V)).astype(np.float32)
        x[0, rng.integers(0, V, 4)] += 6.0
        return x


def _mulberry(seed):
    from minisample.workloads import mulberry32

    seq = iter(mulberry32(seed, 1000))
    calls = []

    def rand():
        calls.append(1)
        return float(next(seq))

    return rand, calls


def _oracle_loop(oracle, model, input_ids, opts, rand):
    from test_parity_gpu import params

    from minisample.generation import is_greedy, normalize_options, params_of

    o = normalize_options(opts)
    p = params(oracle, params_of(o))
    cache = model.make_cache()
    gen = []
    last = model.forward(input_ids, cache)[-1]
    for step in range(int(o["max_new_tokens"])):
        hist = np.array(list(input_ids) + gen, np.int32) if gen else None
        u = 0.0 if is_greedy(o) else rand()
        nid, _ = oracle.pick_token(last, hist, p, u)
        gen.append(int(nid))
        if o["on_token"] and o["on_token"](int(nid), step + 1) is False:
            break
        if o["eos_token_id"] is not None and nid == o["eos_token_id"]:
            break
        last = model.forward([int(nid)], cache)[-1]
    return gen


CASES = [
    {"maxNewTokens": 24, "temperature": 0.8, "topK": 50, "topP": 0.95, "repetitionPenalty": 1.3},
    {"max_new_tokens": 16, "do_sample": False, "repetition_penalty": 1.5},
    {"maxNewTokens": 20, "temperature": 1.0, "topK": 0, "topP": 0.9},
    {"maxNewTokens": 12, "doSample": True, "temperature": 0.0001},  # greedy by temperature
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_generate_tokens_matches_oracle_loop(oracle, case):
    from minisample.generation import generate_tokens, set_backend

    set_backend("cuda")
    opts = CASES[case]
    r1, c1 = _mulberry(77 + case)
    r2, c2 = _mulberry(77 + case)
    got = generate_tokens(StubModel(case), [1, 2, 3, 2], opts, rand=r1)
    want = _oracle_loop(oracle, StubModel(case), [1, 2, 3, 2], opts, rand=r2)
    assert got == want
    assert len(c1) == len(c2)  # the same number of uniforms drawn
    greedy = opts.get("do_sample", opts.get("doSample", True)) is False or opts.get("temperature", 1.0) <= 0.0001
    assert len(c1) == (0 if greedy else len(got))


def test_on_token_false_stops_and_eos_is_appended(oracle):
    from minisample.generation import generate_tokens, set_backend

    set_backend("cuda")
    seen = []

    def on_token(tid, n):
        seen.append((tid, n))
        return n < 3

    model = StubModel(11)
    got = generate_tokens(model, [5], {"maxNewTokens": 30, "onToken": on_token}, rand=_mulberry(5)[0])
    assert len(got) == 3 and [n for _, n in seen] == [1, 2, 3]
    assert model.disposed == 1
    # EOS: stop right after the EOS id is appended (use the 2nd greedy id as EOS)
    greedy = generate_tokens(StubModel(12), [5], {"maxNewTokens": 8, "doSample": False})
    eos = greedy[1]
    got = generate_tokens(StubModel(12), [5], {"maxNewTokens": 8, "doSample": False, "eosTokenId": eos})
    assert got == greedy[: greedy.index(eos) + 1]


def test_generate_async_equals_sync(oracle):
    from minisample.generation import generate_async, generate_tokens, set_backend

    set_backend("cuda")
    opts = CASES[0]
    a = generate_tokens(StubModel(3), [9, 9], opts, rand=_mulberry(1)[0])
    ticks = []

    async def tick():
        ticks.append(1)

    b = asyncio.run(generate_async(StubModel(3), [9, 9], dict(opts, tick=tick), rand=_mulberry(1)[0]))
    assert a == b
    assert len(ticks) == len(b) - 1 or len(ticks) == len(b)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_generate_tokens_batch_matches_oracle_loop(oracle, case):
    """Row i of the batched loop equals the oracle's generation loop on row i
    with the same uniform stream; a row that hits EOS or onToken=false stops
    alone."""
    from minisample.generation import generate_tokens_batch, set_backend

    set_backend("cuda")
    opts = dict(CASES[case])
    inputs = [[1, 2, 3], [7], [4, 4, 4, 4], [9, 8]]
    per_row = [_oracle_loop(oracle, StubModel(40 + i), inputs[i], opts, _mulberry(60 + i)[0])
               for i in range(len(inputs))]
    eos = per_row[1][2]  # makes row 1 stop at its third id (and any other row that draws it)
    stop_at = {3: 2}     # row 3 stops after its second id

    def on_token(row, tid, n):
        return not (row in stop_at and n >= stop_at[row])

    opts_b = dict(opts, eosTokenId=eos, onToken=on_token)
    got = generate_tokens_batch([StubModel(40 + i) for i in range(len(inputs))], inputs, opts_b,
                                rands=[_mulberry(60 + i)[0] for i in range(len(inputs))])
    for i in range(len(inputs)):
        want = per_row[i]
        if eos in want:
            want = want[: want.index(eos) + 1]
        if i in stop_at:
            want = want[: stop_at[i]]
        assert got[i] == want, (i, got[i], want)


class StubDeviceModel:
    """The batched, device-resident counterpart of StubModel: forward_batch
    returns the [B, V] CUDA logits whose row i equals StubModel(seeds[i])'s
    output for the same step and last id."""

    def __init__(self, seeds, input_ids_batch):
        self.rows = [StubModel(sd) for sd in seeds]
        self.inputs = input_ids_batch
        self.host_caches = None

    def make_cache(self):
        return {}

    def dispose_cache(self, cache):
        pass

    def forward_batch(self, last_ids, caches):
        import torch

        if last_ids is None:
            self.host_caches = [m.make_cache() for m in self.rows]
            xs = [m.forward(list(self.inputs[i]), self.host_caches[i]) for i, m in enumerate(self.rows)]
        else:
            xs = [m.forward([last_ids[i]], self.host_caches[i]) for i, m in enumerate(self.rows)]
        return torch.from_numpy(np.concatenate(xs)).cuda()


@pytest.mark.parametrize("case", [0, 1, 2])
def test_generate_tokens_device_matches_oracle_loop(oracle, case):
    """Logits and penalty history on the GPU (ms_history_append): each row's
    ids equal the oracle's generation loop on that row with the same uniform
    stream, with per-row EOS / onToken stops."""
    from minisample.generation import generate_tokens_device, set_backend

    set_backend("cuda")
    opts = dict(CASES[case])
    inputs = [[1, 2, 3], [7], [4, 4, 4, 4], [9, 8]]
    per_row = [_oracle_loop(oracle, StubModel(80 + i), inputs[i], opts, _mulberry(90 + i)[0])
               for i in range(len(inputs))]
    eos = per_row[1][2]
    stop_at = {3: 2}

    def on_token(row, tid, n):
        return not (row in stop_at and n >= stop_at[row])

    opts_b = dict(opts, eosTokenId=eos, onToken=on_token)
    got = generate_tokens_device(StubDeviceModel([80 + i for i in range(len(inputs))], inputs), inputs, opts_b,
                                 rands=[_mulberry(90 + i)[0] for i in range(len(inputs))])
    for i in range(len(inputs)):
        want = per_row[i]
        if eos in want:
            want = want[: want.index(eos) + 1]
        if i in stop_at:
            want = want[: stop_at[i]]
        assert got[i] == want, (i, got[i], want)


def test_history_append_rows():
    """ms_history_append writes each id after the row's last one, skips -1 and
    full rows."""
    import torch

    from minisample.generation import DeviceHistory, set_backend, _sampler

    set_backend("cuda")
    H = DeviceHistory([[5, 6], [], [1, 2, 3]], 3, torch.device("cuda", 0))
    ids = torch.tensor([7, 8, 9], dtype=torch.int32, device="cuda")
    H.append(_sampler(), ids)
    H.append(_sampler(), torch.tensor([-1, 10, 11], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert H.hist.cpu().numpy().tolist() == [[5, 6, 7], [8, 10, -1], [1, 2, 3]]
    assert H.lens.cpu().numpy().tolist() == [3, 2, 3]
