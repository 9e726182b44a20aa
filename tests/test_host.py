"""Host-side checks that need no GPU: the C ABI library, struct layouts, the
generation-option mirror and the workload generators."""
import ctypes
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "minisample.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\**\s*(ms_\w+)\s*\(", src, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    from minisample import _native

    L = _native.load()
    decl = declared_functions()
    assert set(decl) == set(_native.EXPORTED), decl
    for name in decl:
        assert hasattr(L, name), name
    assert L.ms_version() == _native.ABI_VERSION
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    for name in decl:
        assert re.search(rf"\bT {name}$", out, flags=re.M), name


def test_struct_layouts_match_header():
    """Compile a probe against include/minisample.h and compare with ctypes."""
    from minisample._native import MsDiag, MsParams

    code = r'''
#include <stdio.h>
#include <stddef.h>
#include "minisample.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu\n", sizeof(ms_params), offsetof(ms_params, temperature),
         offsetof(ms_params, top_k), offsetof(ms_params, top_p), offsetof(ms_params, repetition_penalty),
         sizeof(ms_diag));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(code)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        vals = [int(v) for v in subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()]
    assert vals == [ctypes.sizeof(MsParams), MsParams.temperature.offset, MsParams.top_k.offset,
                    MsParams.top_p.offset, MsParams.repetition_penalty.offset, ctypes.sizeof(MsDiag)]


def test_ms_create_without_gpu_reports_state_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from minisample import _native

    L = _native.load()
    ctx = ctypes.c_void_p()
    assert L.ms_create(ctypes.byref(ctx), None, 0) == _native.MS_ERR_STATE
    assert L.ms_last_error(None) == b"null context"
    assert L.ms_sample(None, None, 1, 1, 1, None, None, None, None, None, None, 1, None) == _native.MS_ERR_ARG


def test_scratch_bytes_formula():
    from minisample import SampleParams, scratch_bytes

    p = SampleParams(True, 0.9, 64, 0.9, 1.2)
    b = scratch_bytes(512, 262144, p)
    # 16 chunks/row: stats 32 B, 512 candidate slots of 8 B; penalty bitmap V/8 B per row
    expect = 512 * 16 * 32 + 512 * 16 * 512 * 8 + 512 * 262144 // 8
    assert expect <= b <= expect + 4096
    g = scratch_bytes(512, 262144, SampleParams(False))
    assert g < b


def test_normalize_options_keeps_falsy_values():
    from minisample.generation import normalize_options

    d = normalize_options({})
    assert d["max_new_tokens"] == 50 and d["do_sample"] is True and d["temperature"] == 1.0
    assert d["top_k"] == 50 and d["top_p"] == 0.95 and d["repetition_penalty"] == 1.0
    assert d["eos_token_id"] is None and d["on_token"] is None
    d = normalize_options({"do_sample": False, "top_k": 0, "topP": 0, "temperature": 0,
                           "repetitionPenalty": 1.3, "repetition_penalty": 2.0, "eos_token_id": 0})
    assert d["do_sample"] is False and d["top_k"] == 0 and d["top_p"] == 0 and d["temperature"] == 0
    assert d["repetition_penalty"] == 1.3  # camelCase wins, as `a ?? b`
    assert d["eos_token_id"] == 0


def test_workload_generators_shapes_and_determinism():
    from minisample import workloads as W

    w = W.WORKLOADS["gemma_b512"]
    a = W.logits_np(w, 3, B=2)
    b = W.logits_np(w, 3, B=2)
    assert a.shape == (2, 262144) and a.dtype == np.float32
    np.testing.assert_array_equal(a, b)
    h, off = W.history_np(w, 3, B=4)
    assert off.tolist() == [0, 2048, 4096, 6144, 8192]
    assert h.min() >= 0 and h.max() < w.V
    rep = np.mean([len(h[off[r]:off[r + 1]]) - len(set(h[off[r]:off[r + 1]].tolist())) for r in range(4)])
    assert 100 < rep < 330  # about 10% of 2048 positions repeat an earlier id
    z = W.logits_np(W.WORKLOADS["qwen2_b256"], 1, B=64)
    assert (z.max(axis=1) > 9).sum() > 10  # peaked rows exist


def test_argument_checks_that_need_no_gpu():
    """Size and pointer checks that run before any CUDA call: the allocation-free
    entry point, the scratch sizing, the shard record sizing and the test
    hooks."""
    from minisample import SampleParams
    from minisample import _native as N

    L = N.load()
    p = SampleParams(True, 0.9, 64, 0.9, 1.2).to_c()
    g = SampleParams(False).to_c()
    dummy = ctypes.c_void_p(16)  # never dereferenced: every call below is rejected first
    call = L.ms_sample_noalloc
    assert call(dummy, 4, 0, 1, None, None, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_ARG      # V < 1
    assert call(dummy, 4, 100, 99, None, None, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_ARG   # ld < V
    assert call(dummy, -1, 100, 100, None, None, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_ARG
    assert call(dummy, 4, 2**31, 2**31, None, None, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_ARG
    assert call(None, 4, 100, 100, None, None, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_ARG
    assert call(dummy, 4, 100, 100, None, dummy, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_ARG  # off w/o hist
    assert call(dummy, 4, 100, 100, None, None, ctypes.byref(p), None, dummy, None) == N.MS_ERR_ARG    # needs u
    assert call(dummy, 4, 100, 100, None, None, None, dummy, dummy, None) == N.MS_ERR_ARG
    assert call(dummy, 0, 100, 100, None, None, ctypes.byref(g), None, dummy, None) == N.MS_OK         # B = 0
    # 512 x 262144 with top-k needs ~50 MiB of scratch: beyond the fixed array
    assert call(dummy, 512, 262144, 262144, None, None, ctypes.byref(p), dummy, dummy, None) == N.MS_ERR_SCRATCH
    out = ctypes.c_int64()
    assert L.ms_scratch_bytes(-1, 100, ctypes.byref(p), ctypes.byref(out)) == N.MS_ERR_ARG
    assert L.ms_scratch_bytes(4, 0, ctypes.byref(p), ctypes.byref(out)) == N.MS_ERR_ARG
    assert L.ms_scratch_bytes(4, 100, None, ctypes.byref(out)) == N.MS_ERR_ARG
    assert L.ms_shard_record_bytes(0, ctypes.byref(p), ctypes.byref(out)) == N.MS_ERR_ARG
    assert L.ms_debug_inject(None, N.MS_INJECT_WAIT, 10) == N.MS_ERR_ARG
    assert L.ms_debug_exp(None, None, -1, None) == N.MS_ERR_ARG
    assert L.ms_debug_exp(None, None, 0, None) == N.MS_OK
    for fn in (L.ms_destroy, L.ms_launch_count):
        assert (fn(None) if fn is L.ms_destroy else fn(None, ctypes.byref(out))) == N.MS_ERR_ARG
