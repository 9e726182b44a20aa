"""Failure paths on the GPU, made without a GPU fault: a bounded kernel wait
that runs out (ms_debug_inject makes one chunk CTA wait a few thousand cycles
on an mbarrier nothing completes; no copy is in flight against it), an
allocation that fails, and invalid arguments.  Each is followed by a good
call on the same context, which must be unaffected.  Also the exact-term exp
against the oracle's, bit for bit."""
import ctypes

import numpy as np
import pytest

from test_parity_gpu import params

pytestmark = pytest.mark.gpu


def _small(seed=1, B=4, V=40000):
    from minisample import SampleParams

    rng = np.random.default_rng(seed)
    X = rng.normal(0.0, 2.0, (B, V)).astype(np.float32)
    return X, SampleParams(True, 0.8, 40, 0.9, 1.0), rng.random(B)


def test_wait_timeout_fails_the_call_and_the_next_call_is_clean(oracle):
    import torch

    from minisample import Sampler
    from minisample import _native as N

    X, sp, u = _small()
    ref, _ = oracle.sample_batch(X, None, None, params(oracle, sp), u)
    with Sampler() as s:
        # synchronous host call: MS_ERR_TIMEOUT
        s.inject(N.MS_INJECT_WAIT, 4000)
        with pytest.raises(N.MiniSampleError) as e:
            s.sample(X, sp, u=u)
        assert e.value.code == N.MS_ERR_TIMEOUT
        np.testing.assert_array_equal(s.sample(X, sp, u=u), ref)
        # asynchronous device call: the rows come back -1 (MS_ROW_TIMEOUT); in
        # this small top-k call, which finalizes each row as its chunks finish,
        # always row 0 (whose wait ran out), and any row finalized after it;
        # the others keep their correct ids
        xd, ud = torch.from_numpy(X).cuda(), torch.from_numpy(u).cuda()
        s.inject(N.MS_INJECT_WAIT, 4000)
        ids, d = s.sample(xd, sp, u=ud, sync=False, diag=True)
        torch.cuda.synchronize()
        ids = ids.cpu().numpy()
        timed = (d["row_flags"].cpu().numpy() & N.MS_ROW_TIMEOUT) != 0
        assert timed[0]
        assert np.all(ids[timed] == -1)
        np.testing.assert_array_equal(ids[~timed], ref[~timed])
        # the next asynchronous call is unaffected, and so is a synchronous one
        ids = s.sample(xd, sp, u=ud, sync=False)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ids.cpu().numpy(), ref)
        np.testing.assert_array_equal(s.sample(xd, sp, u=ud, sync=True).cpu().numpy(), ref)
        # device call with MS_SYNC reports the timeout too
        s.inject(N.MS_INJECT_WAIT, 4000)
        with pytest.raises(N.MiniSampleError) as e:
            s.sample(xd, sp, u=ud, sync=True)
        assert e.value.code == N.MS_ERR_TIMEOUT
        np.testing.assert_array_equal(s.sample(X, sp, u=u), ref)


def test_wait_timeout_with_a_finalize_grid(oracle):
    """Top-k calls of more than 16 rows finalize in a second grid, after every
    chunk: a wait that ran out leaves every row of the call at -1."""
    import torch

    from minisample import Sampler
    from minisample import _native as N

    X, sp, u = _small(6, B=24)
    ref, _ = oracle.sample_batch(X, None, None, params(oracle, sp), u)
    with Sampler() as s:
        xd, ud = torch.from_numpy(X).cuda(), torch.from_numpy(u).cuda()
        s.inject(N.MS_INJECT_WAIT, 4000)
        ids, d = s.sample(xd, sp, u=ud, sync=False, diag=True)
        torch.cuda.synchronize()
        assert ids.cpu().numpy().tolist() == [-1] * X.shape[0]
        assert np.all(d["row_flags"].cpu().numpy() & N.MS_ROW_TIMEOUT)
        np.testing.assert_array_equal(s.sample(X, sp, u=u), ref)


def test_wait_timeout_greedy_rows():
    """Greedy calls finalize inside the chunk kernel: the stalled row is -1."""
    from minisample import SampleParams, Sampler
    from minisample import _native as N

    X, _, _ = _small(2)
    sp = SampleParams(False)
    with Sampler() as s:
        want = s.sample(X, sp)
        s.inject(N.MS_INJECT_WAIT, 4000)
        with pytest.raises(N.MiniSampleError) as e:
            s.sample(X, sp)
        assert e.value.code == N.MS_ERR_TIMEOUT
        np.testing.assert_array_equal(s.sample(X, sp), want)
        np.testing.assert_array_equal(want, np.argmax(X, axis=1))


def test_injected_allocation_failure_then_recovery(oracle):
    from minisample import Sampler
    from minisample import _native as N

    X, sp, u = _small(3)
    ref, _ = oracle.sample_batch(X, None, None, params(oracle, sp), u)
    with Sampler() as s:  # a fresh context: the first call allocates
        s.inject(N.MS_INJECT_ALLOC, 1)
        with pytest.raises(N.MiniSampleError) as e:
            s.sample(X, sp, u=u)
        assert e.value.code == N.MS_ERR_OOM
        assert "injected" in str(e.value)
        np.testing.assert_array_equal(s.sample(X, sp, u=u), ref)


def test_invalid_arguments_are_rejected(oracle):
    from minisample import Sampler
    from minisample import _native as N

    X, sp, u = _small(4)
    L = N.load()
    ref, _ = oracle.sample_batch(X, None, None, params(oracle, sp), u)
    with Sampler() as s:
        ctx = s._ctx
        p = sp.to_c()
        out = np.zeros(4, np.int32)
        x, uu, o = X.ctypes.data, u.ctypes.data, out.ctypes.data
        hist = np.zeros(4, np.int32)
        cases = [
            (x, 4, 0, 40000, None, None, uu, o, None, N.MS_HOST_PTRS),            # V < 1
            (x, 4, 40000, 39999, None, None, uu, o, None, N.MS_HOST_PTRS),        # ld < V
            (x, -1, 40000, 40000, None, None, uu, o, None, N.MS_HOST_PTRS),       # B < 0
            (x, 4, 40000, 40000, None, None, uu, o, None, 0),                     # no pointer kind
            (x, 4, 40000, 40000, None, None, uu, o, None, N.MS_HOST_PTRS | N.MS_DEVICE_PTRS),
            (x, 4, 40000, 40000, None, np.arange(5, dtype=np.int64).ctypes.data, uu, o, None,
             N.MS_HOST_PTRS),                                                     # hist_off without hist
            (x, 4, 40000, 40000, hist.ctypes.data, np.array([0, 2, 1, 3, 4], np.int64).ctypes.data, uu, o,
             None, N.MS_HOST_PTRS),                                               # offsets not ascending
            (x, 4, 40000, 40000, None, None, None, o, None, N.MS_HOST_PTRS),      # sampled rows need u
            (None, 4, 40000, 40000, None, None, uu, o, None, N.MS_HOST_PTRS),     # NULL logits
            (x, 4, 2**31, 2**31, None, None, uu, o, None, N.MS_HOST_PTRS),        # V beyond the limit
        ]
        for i, (xp, B, V, ld, hp, op, up, outp, dg, fl) in enumerate(cases):
            rc = L.ms_sample(ctx, xp, B, V, ld, hp, op, ctypes.byref(p), up, outp, dg, fl, None)
            assert rc == N.MS_ERR_ARG, (i, rc)
            assert L.ms_last_error(ctx).decode().startswith("ms_sample"), i
        D = N.MsDiag()
        D.cand_cap = -1
        assert L.ms_sample(ctx, x, 4, 40000, 40000, None, None, ctypes.byref(p), uu, o, ctypes.byref(D),
                           N.MS_HOST_PTRS, None) == N.MS_ERR_ARG
        D.cand_cap = 0
        pen = np.zeros((4, 10), np.float32)
        D.pen_logits, D.pen_ld = pen.ctypes.data, 10
        assert L.ms_sample(ctx, x, 4, 40000, 40000, None, None, ctypes.byref(p), uu, o, ctypes.byref(D),
                           N.MS_HOST_PTRS, None) == N.MS_ERR_ARG
        assert L.ms_debug_inject(ctx, 99, 1) == N.MS_ERR_ARG
        np.testing.assert_array_equal(s.sample(X, sp, u=u), ref)


def test_device_exact_exp_equals_oracle_exp(oracle):
    """The GPU's exact-term exp (fdlibm's method) against the oracle's, bit for bit."""
    import torch

    from minisample import _native as N

    rng = np.random.default_rng(5)
    x = np.concatenate([-rng.exponential(4.0, 1 << 20), rng.uniform(-746.0, 710.0, 1 << 16),
                        -rng.uniform(0.0, 0.7, 1 << 16),
                        np.array([0.0, -0.0, 1.0, -1e-30, 2.0**-28, -745.13, -745.2, 709.78, np.inf, -np.inf])])
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    rc = N.load().ms_debug_exp(xd.data_ptr(), yd.data_ptr(), x.shape[0], None)
    assert rc == N.MS_OK
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    oracle.set_exp(libc=False)
    L = oracle.lib()
    want = np.array([L.msref_exp(float(v)) for v in x])
    bad = np.nonzero(y.view(np.uint64) != want.view(np.uint64))[0]
    assert bad.size == 0, [(x[i], y[i], want[i]) for i in bad[:5]]
