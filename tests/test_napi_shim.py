"""The N-API shim (omni.js_b200/csrc/napi_minisample.c) built against the small
N-API runtime in tests/napi_fake/ and driven from Python: argument checks,
thrown errors, promise settlement of sampleAsync, and on the GPU the ids of
sample / sampleAsync against the oracle (mini.js's pickToken,
src/generation.js:71-81, through the binding a JS caller uses).  The image has
no Node runtime, so this is where the shim's C code runs."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "omni.js_b200", "minisample")

F32P = ctypes.POINTER(ctypes.c_float)
I32P = ctypes.POINTER(ctypes.c_int32)
F64P = ctypes.POINTER(ctypes.c_double)


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    import minisample._native  # noqa: F401  (checks the library exists)

    out = str(tmp_path_factory.mktemp("napi") / "libnapifake.so")
    cmd = ["gcc", "-O1", "-Wall", "-Wextra", "-Werror", "-fPIC", "-shared",
           "-I" + os.path.join(ROOT, "tests", "napi_fake"), "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "napi_fake", "fake_napi.c"),
           os.path.join(ROOT, "omni.js_b200", "csrc", "napi_minisample.c"),
           "-L" + PKG, "-lminisample", "-Wl,-rpath," + PKG, "-lpthread", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    L = ctypes.CDLL(out)
    common = [F32P, ctypes.c_size_t, ctypes.c_double, ctypes.c_double, I32P, ctypes.c_size_t, I32P,
              ctypes.c_size_t, F64P, ctypes.c_int, F64P, ctypes.c_size_t]
    L.fake_sample.argtypes = common + [I32P, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
    L.fake_sample.restype = ctypes.c_int
    L.fake_sample_async.argtypes = common + [ctypes.c_char_p, ctypes.c_size_t]
    L.fake_sample_async.restype = ctypes.c_void_p
    L.fake_promise.argtypes = [ctypes.c_void_p, I32P, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
    L.fake_promise.restype = ctypes.c_int
    L.fake_set_deferred_start.argtypes = [ctypes.c_int]
    assert L.fake_load() == 3  # sample, sampleAsync, status
    yield L
    L.fake_reset()


class Call:
    """One call's arguments, kept alive while the shim may read them."""

    KEYS = ("doSample", "temperature", "topK", "topP", "repetitionPenalty")

    def __init__(self, X, B=None, V=None, hist=None, off=None, opts=None, u=None):
        self.X = None if X is None else np.ascontiguousarray(X, np.float32)
        self.B = B if B is not None else self.X.shape[0]
        self.V = V if V is not None else self.X.shape[1]
        self.hist = None if hist is None else np.ascontiguousarray(hist, np.int32)
        self.off = None if off is None else np.ascontiguousarray(off, np.int32)
        self.u = None if u is None else np.ascontiguousarray(u, np.float64)
        opts = opts or {}
        self.opts = np.array([float(opts.get(k, 0)) for k in self.KEYS], np.float64)
        self.mask = sum(1 << i for i, k in enumerate(self.KEYS) if k in opts)
        self.err = ctypes.create_string_buffer(600)

    def args(self):
        def p(a, t):
            return None if a is None else a.ctypes.data_as(t)

        def n(a):
            return 0 if a is None else a.size

        return [p(self.X, F32P), n(self.X), float(self.B), float(self.V), p(self.hist, I32P), n(self.hist),
                p(self.off, I32P), n(self.off), self.opts.ctypes.data_as(F64P), self.mask, p(self.u, F64P), n(self.u)]

    def sample(self, L):
        out = np.zeros(max(int(self.B), 1), np.int32)
        n = L.fake_sample(*self.args(), out.ctypes.data_as(I32P), out.size, self.err, 600)
        return (out[:n] if n >= 0 else None), self.err.value.decode()

    def sample_async(self, L):
        self.promise = L.fake_sample_async(*self.args(), self.err, 600)
        return self.promise, self.err.value.decode()

    def settled(self, L):
        out = np.zeros(max(int(self.B), 1), np.int32)
        n = L.fake_promise(self.promise, out.ctypes.data_as(I32P), out.size, self.err, 600)
        return (out[:n] if n >= 0 else n), self.err.value.decode()


def _rows(seed=3, B=6, V=50000):
    rng = np.random.default_rng(seed)
    return rng.normal(0.0, 2.5, (B, V)).astype(np.float32), rng.random(B)


OPTS = {"doSample": 1, "temperature": 0.8, "topK": 40, "topP": 0.9, "repetitionPenalty": 1.3}


def test_status_reports_the_abi(shim):
    from minisample import _native as N

    assert shim.fake_status_abi() == N.ABI_VERSION


@pytest.mark.parametrize("case,kind,text", [
    ("logits_not_typed", "TypeError", "Float32Array of B*V"),
    ("logits_short", "TypeError", "Float32Array of B*V"),
    ("B_zero", "TypeError", "Float32Array of B*V"),
    ("uniforms_short", "TypeError", "uniforms must have B entries"),
    ("offsets_count", "TypeError", "B+1 entries"),
    ("offsets_descend", "RangeError", "must ascend"),
    ("offsets_past_history", "RangeError", "must ascend"),
    ("offsets_negative", "RangeError", "must ascend"),
])
def test_async_argument_errors_throw_synchronously(shim, case, kind, text):
    X, u = _rows(B=3, V=1000)
    h = np.arange(10, dtype=np.int32)
    c = {
        "logits_not_typed": Call(None, B=3, V=1000, opts=OPTS, u=u),
        "logits_short": Call(X[:, :999], B=3, V=1000, opts=OPTS, u=u),
        "B_zero": Call(X, B=0, opts=OPTS, u=u),
        "uniforms_short": Call(X, opts=OPTS, u=u[:2]),
        "offsets_count": Call(X, hist=h, off=[0, 2, 4], opts=OPTS, u=u),
        "offsets_descend": Call(X, hist=h, off=[0, 5, 3, 10], opts=OPTS, u=u),
        "offsets_past_history": Call(X, hist=h, off=[0, 2, 4, 11], opts=OPTS, u=u),
        "offsets_negative": Call(X, hist=h, off=[-1, 2, 4, 10], opts=OPTS, u=u),
    }[case]
    p, err = c.sample_async(shim)
    assert p is None
    assert err.startswith(kind + ": minisample.sample") and text in err, err
    shim.fake_reset()


def test_without_a_gpu_calls_fail_loudly(shim):
    import torch

    if torch.cuda.is_available():
        pytest.skip("this machine has a GPU: the GPU tests below cover the calls")
    X, u = _rows(B=2, V=1000)
    ids, err = Call(X, opts=OPTS, u=u).sample(shim)
    assert ids is None and "no CUDA device" in err
    c = Call(X, opts=OPTS, u=u)
    p, _ = c.sample_async(shim)
    assert p is not None
    assert shim.fake_drain() == 1
    res, err = c.settled(shim)
    assert res == -1 and "no CUDA device" in err, err
    shim.fake_reset()


def _oracle_ids(oracle, X, opts, u, hist=None, off=None):
    p = oracle.make_params(bool(opts.get("doSample", 1)), opts.get("temperature", 1.0), int(opts.get("topK", 50)),
                           opts.get("topP", 0.95), opts.get("repetitionPenalty", 1.0))
    ids, _ = oracle.sample_batch(X, hist, None if off is None else np.asarray(off, np.int64), p, u)
    return ids


@pytest.mark.gpu
@pytest.mark.parametrize("opts", [OPTS, {"doSample": 0}, {}, {"temperature": 1.1, "topK": 0, "topP": 0.5}])
def test_sample_and_sample_async_match_the_oracle(shim, oracle, opts):
    X, u = _rows(7, B=6, V=50000)
    rng = np.random.default_rng(8)
    lens = rng.integers(0, 300, 6)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    hist = rng.integers(-5, 50010, int(off[-1])).astype(np.int32)
    greedy = "doSample" in opts and not opts["doSample"]
    uu = None if greedy else u
    want = _oracle_ids(oracle, X, opts, uu, hist, off)
    ids, err = Call(X, hist=hist, off=off, opts=opts, u=uu).sample(shim)
    assert ids is not None, err
    np.testing.assert_array_equal(ids, want)
    c = Call(X, hist=hist, off=off, opts=opts, u=uu)
    p, err = c.sample_async(shim)
    assert p is not None, err
    assert shim.fake_drain() == 1
    res, err = c.settled(shim)
    assert not isinstance(res, int), err
    np.testing.assert_array_equal(res, want)
    shim.fake_reset()


@pytest.mark.gpu
def test_sample_async_reads_a_copy_of_its_inputs(shim, oracle):
    """The worker runs after the JS arrays changed: the ids are those of the
    arrays at call time."""
    X, u = _rows(9, B=4, V=30000)
    want = _oracle_ids(oracle, X, OPTS, u)
    c = Call(X, opts=OPTS, u=u)
    shim.fake_set_deferred_start(1)
    try:
        p, err = c.sample_async(shim)
        assert p is not None, err
        assert c.settled(shim)[0] == -2  # pending until drained
        c.X[:] = -c.X  # the caller reuses its buffers
        c.u[:] = 0.999
        assert shim.fake_drain() == 1
    finally:
        shim.fake_set_deferred_start(0)
    res, err = c.settled(shim)
    assert not isinstance(res, int), err
    np.testing.assert_array_equal(res, want)
    shim.fake_reset()


@pytest.mark.gpu
def test_concurrent_async_calls_each_settle_correctly(shim, oracle):
    """Eight sampleAsync calls in flight at once (eight worker threads sharing
    the async context under its lock), next to synchronous calls on the JS
    thread's own context."""
    calls, wants = [], []
    for i in range(8):
        X, u = _rows(20 + i, B=3 + i, V=20000 + 997 * i)
        wants.append(_oracle_ids(oracle, X, OPTS, u))
        calls.append(Call(X, opts=OPTS, u=u))
    for c in calls:
        p, err = c.sample_async(shim)
        assert p is not None, err
    X, u = _rows(40, B=5, V=40000)
    ids, err = Call(X, opts=OPTS, u=u).sample(shim)
    np.testing.assert_array_equal(ids, _oracle_ids(oracle, X, OPTS, u))
    assert shim.fake_drain() == 8
    for c, w in zip(calls, wants):
        res, err = c.settled(shim)
        assert not isinstance(res, int), err
        np.testing.assert_array_equal(res, w)
    shim.fake_reset()


@pytest.mark.gpu
def test_library_errors_reject_the_promise(shim):
    """A sampled call without uniforms passes the shim's checks (uniforms are
    optional for greedy calls) and fails in ms_sample: sample throws and
    sampleAsync rejects, with the library's message."""
    X, _ = _rows(B=2, V=1000)
    ids, err = Call(X, opts=OPTS).sample(shim)
    assert ids is None and err.startswith("Error: ms_sample"), err
    c = Call(X, opts=OPTS)
    p, err = c.sample_async(shim)
    assert p is not None, err
    shim.fake_drain()
    res, err = c.settled(shim)
    assert res == -1 and err.startswith("ms_sample"), err
    shim.fake_reset()

