"""Batched sampler over libminisample: one call samples one id per logits row.

Host arrays (numpy) go through MS_HOST_PTRS: the library copies them in,
samples on the GPU and copies the ids out.  CUDA tensors (torch) go through
MS_DEVICE_PTRS on the tensor's stream, with no host copies.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _native as N


@dataclass
class SampleParams:
    """The normalised options of src/generation.js:57-68 that reach the sampler."""

    do_sample: bool = True
    temperature: float = 1.0
    top_k: int = 50
    top_p: float = 0.95
    repetition_penalty: float = 1.0

    def to_c(self) -> N.MsParams:
        return N.MsParams(int(bool(self.do_sample)), float(self.temperature), int(self.top_k),
                          float(self.top_p), float(self.repetition_penalty))


def _stream_handle(st):
    """The C ABI reads a NULL stream as the context's own stream.  torch's
    default stream has handle 0 (CUDA's legacy default stream), so it is named
    explicitly as cudaStreamLegacy (handle 1): the work then stays ordered with
    the caller's other work on that stream."""
    return ctypes.c_void_p(st.cuda_stream or 1)


def _is_torch(x) -> bool:
    return type(x).__module__.startswith("torch")


class Sampler:
    """A libminisample context on one or more CUDA devices (the 'cuda' sampler backend)."""

    def __init__(self, devices=None):
        self._L = N.load()
        self._ctx = ctypes.c_void_p()
        if devices:
            arr = (ctypes.c_int * len(devices))(*devices)
            rc = self._L.ms_create(ctypes.byref(self._ctx), arr, len(devices))
        else:
            rc = self._L.ms_create(ctypes.byref(self._ctx), None, 0)
        if rc != N.MS_OK:
            raise N.MiniSampleError(rc, "ms_create failed (no CUDA device?)")
        self.devices = list(devices) if devices else None

    def close(self):
        if self._ctx:
            self._L.ms_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc):
        if rc != N.MS_OK:
            raise N.MiniSampleError(rc, self._L.ms_last_error(self._ctx).decode())

    def sample(self, logits, params: SampleParams, u=None, hist=None, hist_off=None,
               diag: bool = False, cand_cap: int = 0, row_sharded: bool = False, out=None,
               sync: bool = True, stream=None, profile: bool = False):
        """Sample one id per row of `logits` [B, V] (fp32).

        hist / hist_off: CSR id history per row (int32 ids, int64 offsets [B+1]).
        u: [B] float64 uniforms in [0, 1), used by sampled rows only.
        Returns int32 ids [B] (numpy for host input, torch for device input), or
        (ids, diag_dict) when diag is true.
        """
        if _is_torch(logits) and logits.is_cuda:
            return self._sample_device(logits, params, u, hist, hist_off, diag, cand_cap, out, sync, stream,
                                       profile)
        return self._sample_host(logits, params, u, hist, hist_off, diag, cand_cap, row_sharded, out, profile)

    def profile_read(self):
        """(chunk_kernel_ms, finalize_ms, calls) summed over MS_PROFILE calls since the last read."""
        a, b, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int64()
        self._check(self._L.ms_profile_read(self._ctx, ctypes.byref(a), ctypes.byref(b), ctypes.byref(n)))
        return a.value, b.value, n.value

    def history_append(self, hist, lens, ids, stream=None) -> None:
        """Appends ids[r] to row r of a device history ([B, cap] int32, -1 in unused
        slots) and bumps lens[r] (ms_history_append)."""
        import torch

        B, cap = hist.shape
        st = stream if stream is not None else torch.cuda.current_stream(hist.device)
        with torch.cuda.device(hist.device):
            self._check(self._L.ms_history_append(self._ctx, hist.data_ptr(), lens.data_ptr(), B, cap, ids.data_ptr(),
                                                  _stream_handle(st)))

    def inject(self, what: int, arg: int) -> None:
        """Failure injection for the next call (ms_debug_inject): N.MS_INJECT_WAIT
        with a cycle count, or N.MS_INJECT_ALLOC."""
        self._check(self._L.ms_debug_inject(self._ctx, int(what), int(arg)))

    def launch_count(self) -> int:
        """Kernels this context has launched since it was created."""
        n = ctypes.c_int64()
        self._check(self._L.ms_launch_count(self._ctx, ctypes.byref(n)))
        return n.value

    # ------------------------------------------------------------------ host
    def _sample_host(self, logits, params, u, hist, hist_off, diag, cand_cap, row_sharded, out, profile=False):
        if _is_torch(logits):
            logits = logits.numpy()
        x = np.asarray(logits)
        if x.dtype != np.float32 or x.ndim != 2:
            raise ValueError("logits must be a [B, V] float32 array")
        if x.strides[1] != 4 or x.strides[0] % 4:
            x = np.ascontiguousarray(x)
        B, V = x.shape
        ld = x.strides[0] // 4
        h = ho = None
        if hist_off is not None:
            ho = np.ascontiguousarray(hist_off, dtype=np.int64)
            h = np.ascontiguousarray(hist if hist is not None and len(hist) else np.zeros(1), dtype=np.int32)
            if ho.shape[0] != B + 1:
                raise ValueError("hist_off must have B+1 entries")
        ua = None if u is None else np.ascontiguousarray(u, dtype=np.float64)
        if ua is not None and ua.shape[0] < B:
            raise ValueError("u must have B entries")
        ids = out if out is not None else np.empty(B, np.int32)
        D, keep = self._host_diag(B, V, diag, cand_cap)
        p = params.to_c()
        flags = N.MS_HOST_PTRS | (N.MS_ROW_SHARDED if row_sharded else 0) | (N.MS_PROFILE if profile else 0)
        rc = self._L.ms_sample(self._ctx, x.ctypes.data, B, V, ld,
                               None if h is None else h.ctypes.data,
                               None if ho is None else ho.ctypes.data, ctypes.byref(p),
                               None if ua is None else ua.ctypes.data, ids.ctypes.data,
                               ctypes.byref(D) if D is not None else None, flags, None)
        self._check(rc)
        if diag:
            return ids, keep
        return ids

    @staticmethod
    def _host_diag(B, V, diag, cand_cap):
        """diag: False, True (row diagnostics), or "pen" (also the penalised
        logits [B, V])."""
        if not diag:
            return None, None
        keep = {
            "n_cand": np.zeros(B, np.int32), "row_max": np.zeros(B, np.float64),
            "row_sum": np.zeros(B, np.float64), "total": np.zeros(B, np.float64),
            "row_flags": np.zeros(B, np.int32),
        }
        D = N.MsDiag()
        if diag == "pen":
            keep["pen_logits"] = np.zeros((B, V), np.float32)
            D.pen_logits = keep["pen_logits"].ctypes.data
            D.pen_ld = V
        D.cand_cap = int(cand_cap)
        if cand_cap > 0:
            keep["cand_ids"] = np.full((B, cand_cap), -1, np.int32)
            keep["cand_probs"] = np.zeros((B, cand_cap), np.float32)
            D.cand_ids = keep["cand_ids"].ctypes.data
            D.cand_probs = keep["cand_probs"].ctypes.data
        for k in ("n_cand", "row_max", "row_sum", "total", "row_flags"):
            setattr(D, k, keep[k].ctypes.data)
        return D, keep

    # ------------------------------------------------------------------ device
    def _sample_device(self, logits, params, u, hist, hist_off, diag, cand_cap, out, sync, stream, profile=False):
        import torch

        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("logits must be a [B, V] float32 CUDA tensor with unit column stride")
        B, V = logits.shape
        dev = logits.device
        ld = logits.stride(0)
        ids = out if out is not None else torch.empty(B, dtype=torch.int32, device=dev)
        hp = hop = None
        if hist_off is not None:
            hop = hist_off.data_ptr()
            hp = hist.data_ptr()
        up = None if u is None else u.data_ptr()
        D = None
        keep = None
        if diag:
            keep = {
                "n_cand": torch.zeros(B, dtype=torch.int32, device=dev),
                "row_max": torch.zeros(B, dtype=torch.float64, device=dev),
                "row_sum": torch.zeros(B, dtype=torch.float64, device=dev),
                "total": torch.zeros(B, dtype=torch.float64, device=dev),
                "row_flags": torch.zeros(B, dtype=torch.int32, device=dev),
            }
            D = N.MsDiag()
            if diag == "pen":
                keep["pen_logits"] = torch.zeros((B, V), dtype=torch.float32, device=dev)
                D.pen_logits = keep["pen_logits"].data_ptr()
                D.pen_ld = V
            D.cand_cap = int(cand_cap)
            if cand_cap > 0:
                keep["cand_ids"] = torch.full((B, cand_cap), -1, dtype=torch.int32, device=dev)
                keep["cand_probs"] = torch.zeros((B, cand_cap), dtype=torch.float32, device=dev)
                D.cand_ids = keep["cand_ids"].data_ptr()
                D.cand_probs = keep["cand_probs"].data_ptr()
            for k in ("n_cand", "row_max", "row_sum", "total", "row_flags"):
                setattr(D, k, keep[k].data_ptr())
        st = stream if stream is not None else torch.cuda.current_stream(dev)
        p = params.to_c()
        flags = N.MS_DEVICE_PTRS | (N.MS_SYNC if sync else 0) | (N.MS_PROFILE if profile else 0)
        with torch.cuda.device(dev):
            rc = self._L.ms_sample(self._ctx, logits.data_ptr(), B, V, ld, hp, hop, ctypes.byref(p), up,
                                   ids.data_ptr(), ctypes.byref(D) if D is not None else None, flags,
                                   _stream_handle(st))
        self._check(rc)
        if diag:
            return ids, keep
        return ids


    # ------------------------------------------------------------------ vocabulary shards
    def shard_records(self, logits, V: int, col0: int, params: SampleParams, hist=None, hist_off=None,
                      records=None, stream=None):
        """Row records of one vocabulary shard: `logits` is the [B, cols] fp32 CUDA
        view of columns [col0, col0 + cols) (row stride >= cols); hist / hist_off
        hold global ids.  Returns a [B, rec_bytes] uint8 CUDA tensor."""
        import torch

        if logits.dtype != torch.float32 or logits.dim() != 2 or logits.stride(1) != 1:
            raise ValueError("logits must be a [B, cols] float32 CUDA tensor with unit column stride")
        B, cols = logits.shape
        R = record_bytes(V, params)
        if records is None:
            records = torch.empty((B, R), dtype=torch.uint8, device=logits.device)
        st = stream if stream is not None else torch.cuda.current_stream(logits.device)
        p = params.to_c()
        hp = hop = None
        if hist_off is not None:
            hp, hop = hist.data_ptr(), hist_off.data_ptr()
        with torch.cuda.device(logits.device):
            rc = self._L.ms_shard_records(self._ctx, logits.data_ptr(), B, V, col0, cols, logits.stride(0), hp, hop,
                                          ctypes.byref(p), records.data_ptr(), R, _stream_handle(st))
        self._check(rc)
        return records

    def merge_records(self, records, V: int, params: SampleParams, u=None, out=None, diag: bool = False,
                      cand_cap: int = 0, stream=None):
        """Ids from the [B, G, rec_bytes] records of each row's G shards (in shard
        order).  Unsettled rows get -1 (row flag MS_ROW_UNSETTLED)."""
        import torch

        B, G, R = records.shape
        dev = records.device
        ids = out if out is not None else torch.empty(B, dtype=torch.int32, device=dev)
        D = keep = None
        if diag:
            keep = {
                "n_cand": torch.zeros(B, dtype=torch.int32, device=dev),
                "row_max": torch.zeros(B, dtype=torch.float64, device=dev),
                "row_sum": torch.zeros(B, dtype=torch.float64, device=dev),
                "total": torch.zeros(B, dtype=torch.float64, device=dev),
                "row_flags": torch.zeros(B, dtype=torch.int32, device=dev),
            }
            D = N.MsDiag()
            D.cand_cap = int(cand_cap)
            if cand_cap > 0:
                keep["cand_ids"] = torch.full((B, cand_cap), -1, dtype=torch.int32, device=dev)
                keep["cand_probs"] = torch.zeros((B, cand_cap), dtype=torch.float32, device=dev)
                D.cand_ids = keep["cand_ids"].data_ptr()
                D.cand_probs = keep["cand_probs"].data_ptr()
            for k in ("n_cand", "row_max", "row_sum", "total", "row_flags"):
                setattr(D, k, keep[k].data_ptr())
        st = stream if stream is not None else torch.cuda.current_stream(dev)
        p = params.to_c()
        with torch.cuda.device(dev):
            rc = self._L.ms_merge_records(self._ctx, records.data_ptr(), B, G, V, ctypes.byref(p),
                                          None if u is None else u.data_ptr(), ids.data_ptr(),
                                          ctypes.byref(D) if D is not None else None, R,
                                          _stream_handle(st))
        self._check(rc)
        if diag:
            return ids, keep
        return ids


def record_bytes(V: int, params: SampleParams) -> int:
    """Bytes of one row's shard record (ms_shard_record_bytes)."""
    L = N.load()
    out = ctypes.c_int64()
    p = params.to_c()
    rc = L.ms_shard_record_bytes(V, ctypes.byref(p), ctypes.byref(out))
    if rc != N.MS_OK:
        raise N.MiniSampleError(rc, "ms_shard_record_bytes: these params are not supported vocab-sharded")
    return out.value


def scratch_bytes(B: int, V: int, params: SampleParams) -> int:
    L = N.load()
    out = ctypes.c_int64()
    p = params.to_c()
    rc = L.ms_scratch_bytes(B, V, ctypes.byref(p), ctypes.byref(out))
    if rc != N.MS_OK:
        raise N.MiniSampleError(rc, "ms_scratch_bytes failed")
    return out.value
