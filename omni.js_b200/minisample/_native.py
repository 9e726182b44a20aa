"""ctypes binding of libminisample (include/minisample.h).

The library is built in-tree (omni.js_b200/csrc/build.sh) next to this file.
Loading fails loudly when it is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libminisample.so")

MS_OK = 0
MS_ERR_ARG = -1
MS_ERR_CUDA = -2
MS_ERR_NCCL = -3
MS_ERR_TIMEOUT = -4
MS_ERR_OOM = -5
MS_ERR_STATE = -6
MS_ERR_SCRATCH = -7

MS_NOALLOC_SCRATCH_BYTES = 8 << 20

MS_HOST_PTRS = 0x1
MS_DEVICE_PTRS = 0x2
MS_ROW_SHARDED = 0x4
MS_SYNC = 0x8
MS_PROFILE = 0x10

MS_ROW_GREEDY = 0x1
MS_ROW_NAN = 0x2
MS_ROW_FULLVOCAB = 0x4
MS_ROW_SLOWPATH = 0x8
MS_ROW_UNSETTLED = 0x10
MS_ROW_TIMEOUT = 0x20

MS_INJECT_WAIT = 1
MS_INJECT_ALLOC = 2
ABI_VERSION = 2

ERROR_NAMES = {
    MS_ERR_ARG: "MS_ERR_ARG", MS_ERR_CUDA: "MS_ERR_CUDA", MS_ERR_NCCL: "MS_ERR_NCCL",
    MS_ERR_TIMEOUT: "MS_ERR_TIMEOUT", MS_ERR_OOM: "MS_ERR_OOM", MS_ERR_STATE: "MS_ERR_STATE",
    MS_ERR_SCRATCH: "MS_ERR_SCRATCH",
}

# Every symbol include/minisample.h declares.
EXPORTED = ("ms_version", "ms_create", "ms_destroy", "ms_last_error", "ms_sample", "ms_profile_read",
            "ms_scratch_bytes", "ms_sample_noalloc", "ms_launch_count", "ms_shard_record_bytes",
            "ms_shard_records", "ms_merge_records", "ms_debug_inject", "ms_debug_exp", "ms_history_append")


class MsParams(ctypes.Structure):
    _fields_ = [
        ("do_sample", ctypes.c_int32),
        ("temperature", ctypes.c_double),
        ("top_k", ctypes.c_int32),
        ("top_p", ctypes.c_double),
        ("repetition_penalty", ctypes.c_double),
    ]


class MsDiag(ctypes.Structure):
    _fields_ = [
        ("cand_cap", ctypes.c_int32),
        ("cand_ids", ctypes.c_void_p),
        ("cand_probs", ctypes.c_void_p),
        ("n_cand", ctypes.c_void_p),
        ("row_max", ctypes.c_void_p),
        ("row_sum", ctypes.c_void_p),
        ("total", ctypes.c_void_p),
        ("row_flags", ctypes.c_void_p),
        ("pen_logits", ctypes.c_void_p),
        ("pen_ld", ctypes.c_int64),
    ]


class MiniSampleError(RuntimeError):
    """A libminisample call returned a negative status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {message}")
        self.code = code


_lib = None


def load(path: str | None = None):
    """Load libminisample (once).  Raises when the library is not built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise ImportError(f"libminisample is not built ({p}); run omni.js_b200/csrc/build.sh")
    L = ctypes.CDLL(p)
    L.ms_version.restype = ctypes.c_int
    L.ms_version.argtypes = []
    L.ms_create.restype = ctypes.c_int
    L.ms_create.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_int]
    L.ms_destroy.restype = ctypes.c_int
    L.ms_destroy.argtypes = [ctypes.c_void_p]
    L.ms_last_error.restype = ctypes.c_char_p
    L.ms_last_error.argtypes = [ctypes.c_void_p]
    L.ms_sample.restype = ctypes.c_int
    L.ms_sample.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(MsParams), ctypes.c_void_p,
        ctypes.c_void_p, ctypes.POINTER(MsDiag), ctypes.c_int, ctypes.c_void_p,
    ]
    L.ms_profile_read.restype = ctypes.c_int
    L.ms_profile_read.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(ctypes.c_int64)]
    L.ms_shard_record_bytes.restype = ctypes.c_int
    L.ms_shard_record_bytes.argtypes = [ctypes.c_int64, ctypes.POINTER(MsParams), ctypes.POINTER(ctypes.c_int64)]
    L.ms_shard_records.restype = ctypes.c_int
    L.ms_shard_records.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(MsParams), ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_void_p,
    ]
    L.ms_merge_records.restype = ctypes.c_int
    L.ms_merge_records.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(MsParams),
        ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(MsDiag), ctypes.c_int64, ctypes.c_void_p,
    ]
    L.ms_launch_count.restype = ctypes.c_int
    L.ms_launch_count.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]
    L.ms_scratch_bytes.restype = ctypes.c_int
    L.ms_scratch_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(MsParams),
                                   ctypes.POINTER(ctypes.c_int64)]
    L.ms_history_append.restype = ctypes.c_int
    L.ms_history_append.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_void_p, ctypes.c_void_p]
    L.ms_debug_exp.restype = ctypes.c_int
    L.ms_debug_exp.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
    L.ms_debug_inject.restype = ctypes.c_int
    L.ms_debug_inject.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64]
    L.ms_sample_noalloc.restype = ctypes.c_int
    L.ms_sample_noalloc.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.POINTER(MsParams), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
    ]
    if path is None:
        _lib = L
    return L
