"""ORACLE — test infrastructure only (the checker, never the product).

ctypes wrapper of oracle/ms_oracle.c, the C restatement of mini.js's sampler
(src/generation.js:9-81).  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg import this module.

Math.exp is V8's (a restatement of fdlibm's exp, the method V8 ports); the C
library's exp can be selected with set_exp(libc=True) for comparisons.
Parity is pinned to the reference's arithmetic, not to a run of the reference
(no JavaScript engine exists on these machines; the reference's tests pin no
sampled value): tests/golden/ holds known-answer cases derived by hand from the
JS source, and an independent restatement of fdlibm's exp checks the oracle's.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmsoracle.so")
_lib = None


class Params(ctypes.Structure):
    """Same layout as ms_params in include/minisample.h."""

    _fields_ = [
        ("do_sample", ctypes.c_int32),
        ("temperature", ctypes.c_double),
        ("top_k", ctypes.c_int32),
        ("top_p", ctypes.c_double),
        ("repetition_penalty", ctypes.c_double),
    ]


class RowDiag(ctypes.Structure):
    """Same layout as msref_row_diag in oracle/ms_oracle.c."""

    _fields_ = [
        ("mx", ctypes.c_double),
        ("sum", ctypes.c_double),
        ("greedy", ctypes.c_int32),
        ("nan_path", ctypes.c_int32),
        ("n_topk", ctypes.c_int64),
        ("n_cand", ctypes.c_int64),
        ("total", ctypes.c_double),
        ("r", ctypes.c_double),
        ("draw_pos", ctypes.c_int64),
        ("margin_draw", ctypes.c_double),
        ("margin_cut", ctypes.c_double),
        ("cand_cap", ctypes.c_int32),
        ("cand_ids", ctypes.POINTER(ctypes.c_int32)),
        ("cand_probs", ctypes.POINTER(ctypes.c_float)),
    ]


def build() -> str:
    """Compile the oracle library with oracle/Makefile; returns its path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.msref_mulberry32_u32.restype = ctypes.c_uint32
        L.msref_mulberry32_u32.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        L.msref_mulberry32.restype = ctypes.c_double
        L.msref_mulberry32.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
        L.msref_pick_token.restype = ctypes.c_int32
        L.msref_pick_token.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
            ctypes.POINTER(Params), ctypes.c_double, ctypes.POINTER(RowDiag),
            ctypes.c_void_p, ctypes.c_void_p,
        ]
        L.msref_sample_batch.restype = ctypes.c_int
        L.msref_sample_batch.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(Params), ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
        ]
        L.msref_set_exp.restype = None
        L.msref_set_exp.argtypes = [ctypes.c_int]
        L.msref_exp.restype = ctypes.c_double
        L.msref_exp.argtypes = [ctypes.c_double]
        L.msref_terms_both.restype = None
        L.msref_terms_both.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_void_p,
                                       ctypes.c_void_p]
        L.msref_row_diag_size.restype = ctypes.c_int
        assert L.msref_row_diag_size() == ctypes.sizeof(RowDiag), "RowDiag layout mismatch"
        _lib = L
    return _lib


def set_exp(libc: bool = False) -> None:
    """Math.exp as V8 computes it (default), or the C library's exp."""
    lib().msref_set_exp(1 if libc else 0)


def js_exp(x: float) -> float:
    """The oracle's Math.exp (whichever set_exp selected)."""
    return lib().msref_exp(float(x))


def terms_both(xs, mx: float):
    """fp32(exp(x - mx)) for every x with V8's exp and with the C library's."""
    xs = np.ascontiguousarray(xs, dtype=np.float32)
    a = np.empty(xs.shape[0], np.float32)
    b = np.empty(xs.shape[0], np.float32)
    lib().msref_terms_both(xs.ctypes.data, xs.shape[0], float(mx), a.ctypes.data, b.ctypes.data)
    return a, b


def make_params(do_sample=True, temperature=1.0, top_k=50, top_p=0.95, repetition_penalty=1.0):
    return Params(int(bool(do_sample)), float(temperature), int(top_k), float(top_p),
                  float(repetition_penalty))


def mulberry32(seed: int, n: int) -> np.ndarray:
    """n draws of mulberry32(seed) as doubles k / 2**32 (test/synth.mjs:10-17)."""
    st = ctypes.c_uint32(seed & 0xFFFFFFFF)
    L = lib()
    return np.array([L.msref_mulberry32(ctypes.byref(st)) for _ in range(n)], dtype=np.float64)


def _ptr(a):
    return None if a is None else a.ctypes.data


def pick_token(row, hist=None, params=None, u=0.0, cand_cap=0, want_arrays=False):
    """pickToken on one row.  Returns (id, diag dict[, work, probs])."""
    row = np.ascontiguousarray(row, dtype=np.float32)
    V = row.shape[0]
    h = None if hist is None or len(hist) == 0 else np.ascontiguousarray(hist, dtype=np.int32)
    H = 0 if h is None else h.shape[0]
    p = params if params is not None else make_params()
    d = RowDiag()
    ids = probs_c = None
    if cand_cap > 0:
        ids = np.zeros(cand_cap, np.int32)
        probs_c = np.zeros(cand_cap, np.float32)
        d.cand_cap = cand_cap
        d.cand_ids = ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
        d.cand_probs = probs_c.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    work = np.zeros(V, np.float32) if want_arrays else None
    probs = np.zeros(V, np.float32) if want_arrays else None
    tid = lib().msref_pick_token(row.ctypes.data, V, _ptr(h), H, ctypes.byref(p), float(u),
                                 ctypes.byref(d), _ptr(work), _ptr(probs))
    out = _diag_dict(d)
    if cand_cap > 0:
        n = min(out["n_cand"], cand_cap)
        out["cand_ids"] = ids[:n].copy()
        out["cand_probs"] = probs_c[:n].copy()
    if want_arrays:
        return int(tid), out, work, probs
    return int(tid), out


def _diag_dict(d: RowDiag) -> dict:
    return {k: getattr(d, k) for k in ("mx", "sum", "greedy", "nan_path", "n_topk", "n_cand",
                                       "total", "r", "draw_pos", "margin_draw", "margin_cut")}


def sample_batch(logits, hist=None, hist_off=None, params=None, u=None, nthreads=None,
                 cand_cap=0, want_diag=True, want_pen=False):
    """B independent pickToken calls.  Returns (ids[B], diag dict of arrays or None);
    with want_pen the diag also holds "pen_logits" [B, V], each row's `work`
    after the repetition penalty (src/generation.js:72-75)."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    B, V = logits.shape
    p = params if params is not None else make_params()
    hist_a = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
    off_a = None if hist_off is None else np.ascontiguousarray(hist_off, dtype=np.int64)
    if hist_a is not None and hist_a.size == 0:
        hist_a = np.zeros(1, np.int32)
    u_a = None if u is None else np.ascontiguousarray(u, dtype=np.float64)
    out = np.zeros(B, np.int32)
    diags = (RowDiag * B)() if want_diag else None
    cids = cps = None
    if want_diag and cand_cap > 0:
        cids = np.zeros((B, cand_cap), np.int32)
        cps = np.zeros((B, cand_cap), np.float32)
        for r in range(B):
            diags[r].cand_cap = cand_cap
            diags[r].cand_ids = cids[r].ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
            diags[r].cand_probs = cps[r].ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    pen = np.empty((B, V), np.float32) if want_pen else None
    rc = lib().msref_sample_batch(logits.ctypes.data, B, V, V, _ptr(hist_a), _ptr(off_a),
                                  ctypes.byref(p), _ptr(u_a), out.ctypes.data,
                                  ctypes.cast(diags, ctypes.c_void_p) if diags is not None else None,
                                  int(nthreads), _ptr(pen))
    if rc != 0:
        raise RuntimeError("oracle batch failed")
    if not want_diag:
        return out, None
    dd = {k: np.array([getattr(diags[r], k) for r in range(B)]) for k in
          ("mx", "sum", "greedy", "nan_path", "n_topk", "n_cand", "total", "r", "draw_pos",
           "margin_draw", "margin_cut")}
    if cand_cap > 0:
        dd["cand_ids"] = cids
        dd["cand_probs"] = cps
    if want_pen:
        dd["pen_logits"] = pen
    return out, dd
