"""Python mirror of rust-llama's sampler API over the C ABI (libllamars_sampler.so).

  SamplingParams        src/sampler.rs:3-26   (same fields and defaults)
  Sampler(seed)         src/sampler.rs:28-37  (state = seed | 1)
  Sampler.sample(...)   src/sampler.rs:56     (one row: host logits, params, recent -> token)
  BatchSampler          many independent samplers, one per row, one GPU

The reference panics (aborts) when a probability is NaN (sampler.rs:129/132); here
that row raises SamplerPanic (single row) or reports LRS_E_NAN (batched).  Nothing
falls back to CPU code: if the CUDA library is missing the import fails loudly.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from .workloads import PARAMS_DTYPE

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libllamars_sampler.so")

LRS_OK = 0
LRS_E_INVALID = -1
LRS_E_NAN = -2
LRS_E_CUDA = -3
LRS_E_NOMEM = -4
LRS_E_TIMEOUT = -5
LRS_E_NCCL = -6
LRS_E_INTERNAL = -7
TOKEN_NONE = 0xFFFFFFFF

ROW_INFO_DTYPE = np.dtype([
    ("status", "<i4"), ("token", "<u4"), ("path", "<u4"), ("k", "<u4"), ("cutoff", "<u4"),
    ("pos", "<u4"), ("max", "<f4"), ("sum_exp", "<f4"), ("surv_sum", "<f4"), ("r0", "<f4"),
    ("prob", "<f4"), ("n_cand", "<u4"), ("events", "<u4"), ("cycles", "<u4", (8,)),
    ("reserved", "<u4"),
])

# Every entry point declared in include/llamars_sampler.h.
EXPORTS = [
    "lrs_create", "lrs_destroy", "lrs_last_error", "lrs_seed_state", "lrs_set_state", "lrs_get_state",
    "lrs_set_params", "lrs_sample", "lrs_sample_device", "lrs_sampler_new", "lrs_sampler_free",
    "lrs_sampler_state", "lrs_sampler_sample", "lrs_sample_device_noalloc", "lrs_assemble_shards",
    "lrs_poll_error", "lrs_noalloc_poll_error", "lrs_test_wait_timeout", "lrs_history_append",
    "lrs_remap_tokens",
]


class SamplerError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (status {code})")
        self.code = code


class SamplerPanic(SamplerError):
    """The reference sampler would panic on this input (NaN probabilities)."""


_lib = None


def lib() -> ctypes.CDLL:
    """Load libllamars_sampler.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run llama.rs_b200/lrs/build.py (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        P, U32, U64, I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
        L.lrs_create.argtypes = [I, U32, U32, U32, ctypes.POINTER(P)]
        L.lrs_create.restype = I
        L.lrs_destroy.argtypes = [P]
        L.lrs_destroy.restype = I
        L.lrs_last_error.argtypes = [P]
        L.lrs_last_error.restype = ctypes.c_char_p
        L.lrs_seed_state.argtypes = [U64]
        L.lrs_seed_state.restype = U64
        for f in (L.lrs_set_state, L.lrs_get_state, L.lrs_set_params):
            f.argtypes = [P, P, U32]
            f.restype = I
        L.lrs_sample.argtypes = [P, P, I, U32, U32, U64, P, U64, P, P, P]
        L.lrs_sample.restype = I
        L.lrs_sample_device.argtypes = [P, P, U32, U32, U64, P, U64, P, P, P, P, P, P, P, P]
        L.lrs_sample_device.restype = I
        L.lrs_sample_device_noalloc.argtypes = [I, P, U32, U32, U64, P, U64, P, P, P, P, P, P, P]
        L.lrs_sample_device_noalloc.restype = I
        L.lrs_poll_error.argtypes = [P]
        L.lrs_poll_error.restype = I
        L.lrs_noalloc_poll_error.argtypes = [I, P]
        L.lrs_noalloc_poll_error.restype = I
        L.lrs_test_wait_timeout.argtypes = [P, ctypes.c_uint32, P]
        L.lrs_test_wait_timeout.restype = I
        L.lrs_assemble_shards.argtypes = [P, U32, U32, U32, P, U64, P]
        L.lrs_assemble_shards.restype = I
        L.lrs_history_append.argtypes = [P, P, U32, U32, P, U64, P, U32, P]
        L.lrs_history_append.restype = I
        L.lrs_remap_tokens.argtypes = [P, P, U32, P, U32, P, P]
        L.lrs_remap_tokens.restype = I
        L.lrs_sampler_new.argtypes = [U64, I]
        L.lrs_sampler_new.restype = P
        L.lrs_sampler_free.argtypes = [P]
        L.lrs_sampler_free.restype = None
        L.lrs_sampler_state.argtypes = [P]
        L.lrs_sampler_state.restype = U64
        L.lrs_sampler_sample.argtypes = [P, P, ctypes.c_size_t, P, P, ctypes.c_size_t, ctypes.POINTER(I)]
        L.lrs_sampler_sample.restype = U32
        _lib = L
    return _lib


@dataclass
class SamplingParams:
    """SamplingParams of src/sampler.rs:3-26 (defaults of sampler.rs:15-26)."""
    temperature: float = 0.7
    top_k: int = 40
    top_p: float = 0.95
    repetition_penalty: float = 1.1
    repeat_last_n: int = 64
    seed: int = 0x1234_5678_9ABC_DEF0

    def record(self) -> np.ndarray:
        p = np.zeros((), PARAMS_DTYPE)
        p["temperature"] = self.temperature
        p["top_k"] = self.top_k
        p["top_p"] = self.top_p
        p["repetition_penalty"] = self.repetition_penalty
        p["repeat_last_n"] = self.repeat_last_n
        return p


def _check(code: int, ctx=None):
    if code != LRS_OK:
        msg = lib().lrs_last_error(ctx).decode(errors="replace")
        if code == LRS_E_NAN:
            raise SamplerPanic(code, msg)
        raise SamplerError(code, msg)


class Sampler:
    """Sampler of src/sampler.rs:28-163: one generation stream on one GPU."""

    def __init__(self, seed: int, device: int = 0):
        self._h = lib().lrs_sampler_new(ctypes.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), device)

    @property
    def state(self) -> int:
        return int(lib().lrs_sampler_state(self._h))

    def sample(self, logits, params: SamplingParams, recent) -> int:
        x = np.ascontiguousarray(logits, np.float32).reshape(-1)
        r = np.ascontiguousarray(np.asarray(recent, np.uint32).reshape(-1))
        p = params.record() if isinstance(params, SamplingParams) else np.asarray(params, PARAMS_DTYPE).reshape(())
        p = np.ascontiguousarray(p)
        st = ctypes.c_int(0)
        tok = lib().lrs_sampler_sample(self._h, x.ctypes.data, x.size, p.ctypes.data, r.ctypes.data, r.size,
                                       ctypes.byref(st))
        if st.value != LRS_OK:
            msg = f"sampler row failed (status {st.value})"
            if st.value == LRS_E_NAN:
                raise SamplerPanic(st.value, "NaN probabilities (the reference sampler panics here)")
            raise SamplerError(st.value, msg)
        return int(tok)

    def close(self):
        if getattr(self, "_h", None):
            lib().lrs_sampler_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchSampler:
    """Independent samplers, one per row, on one GPU (a context of the C ABI)."""

    def __init__(self, max_rows: int, max_vocab: int, max_hist: int = 64, device: int = 0):
        h = ctypes.c_void_p()
        _check(lib().lrs_create(device, max_rows, max_vocab, max_hist, ctypes.byref(h)))
        self._h = h
        self.device = device
        self.max_rows, self.max_vocab, self.max_hist = max_rows, max_vocab, max_hist

    def set_params(self, params: np.ndarray):
        p = np.ascontiguousarray(params, PARAMS_DTYPE).reshape(-1)
        _check(lib().lrs_set_params(self._h, p.ctypes.data, p.size), self._h)

    def set_state(self, state):
        s = np.ascontiguousarray(state, np.uint64).reshape(-1)
        _check(lib().lrs_set_state(self._h, s.ctypes.data, s.size), self._h)

    def get_state(self, rows: int) -> np.ndarray:
        s = np.zeros(rows, np.uint64)
        _check(lib().lrs_get_state(self._h, s.ctypes.data, rows), self._h)
        return s

    def sample(self, logits: np.ndarray, n: int | None = None, hist=None, hist_len=None, probs: bool = False):
        """Host-buffer entry point (lrs_sample): returns tokens (and probabilities)."""
        x = np.ascontiguousarray(logits, np.float32)
        if x.ndim == 1:
            x = x.reshape(1, -1)
        rows, ld = x.shape
        n = ld if n is None else n
        h = hl = None
        hld = 0
        if hist is not None:
            h = np.ascontiguousarray(hist, np.uint32)
            hl = np.ascontiguousarray(hist_len, np.uint32)
            hld = h.shape[1]
        tok = np.zeros(rows, np.uint32)
        pr = np.zeros(rows, np.float32) if probs else None
        code = lib().lrs_sample(self._h, x.ctypes.data, 0, rows, n, ld, None if h is None else h.ctypes.data, hld,
                                None if hl is None else hl.ctypes.data, tok.ctypes.data,
                                None if pr is None else pr.ctypes.data)
        _check(code, self._h)
        return (tok, pr) if probs else tok

    def sample_device(self, logits, params, state, tokens, n=None, hist=None, hist_len=None, probs=None,
                      status=None, info=None, stream=None, ld=None, rows=None):
        """Device-buffer entry point (lrs_sample_device) on torch CUDA tensors; async.
        rows defaults to tokens.numel() (with ld == 0 every row reads logits row 0)."""
        rows = tokens.numel() if rows is None else rows
        n = logits.shape[1] if n is None else n
        ld = (logits.stride(0) if ld is None else ld)
        hld = hist.stride(0) if hist is not None else 0
        ptr = lambda t: None if t is None else t.data_ptr()
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(logits.device).cuda_stream
        code = lib().lrs_sample_device(self._h, logits.data_ptr(), rows, n, ld, ptr(hist), hld, ptr(hist_len),
                                       params.data_ptr(), state.data_ptr(), tokens.data_ptr(), ptr(probs),
                                       ptr(status), ptr(info), stream)
        _check(code, self._h)

    @staticmethod
    def history_append(tokens, hist, hist_len, status=None, eos=None, keep=None, stream=None, rows=None):
        """`recent.push(next)` of a batched generation loop on the device (lrs_history_append):
        appends each row's token (torch CUDA tensors, int32 views of the u32 ids) to its history
        row unless the row failed (status) or drew `eos`; a full row keeps its last `keep` ids
        (default half the row).  Async on `stream`."""
        rows = tokens.numel() if rows is None else rows
        hld = hist.stride(0)
        keep = hld // 2 if keep is None else keep
        eos = TOKEN_NONE if eos is None else eos
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(tokens.device).cuda_stream
        _check(lib().lrs_history_append(tokens.data_ptr(), None if status is None else status.data_ptr(), rows,
                                        eos, hist.data_ptr(), hld, hist_len.data_ptr(), keep, stream))

    @staticmethod
    def remap_tokens(tokens, id_map, out, status=None, stream=None, rows=None):
        """Pruned-vocabulary ids to the full vocabulary (lrs_remap_tokens): out[r] = id_map[tokens[r]]
        for rows sampled without error.  Async on `stream`."""
        rows = tokens.numel() if rows is None else rows
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(tokens.device).cuda_stream
        _check(lib().lrs_remap_tokens(tokens.data_ptr(), None if status is None else status.data_ptr(), rows,
                                      id_map.data_ptr(), id_map.numel(), out.data_ptr(), stream))

    def poll_error(self):
        """Waits for the last launch and raises the error it reported (lrs_poll_error)."""
        _check(lib().lrs_poll_error(self._h), self._h)

    def test_wait_timeout(self, bound_cycles: int, stream=None):
        """Enqueues the test of the bounded wait (lrs_test_wait_timeout): its wait runs out and
        the next call, or poll_error, reports LRS_E_TIMEOUT."""
        _check(lib().lrs_test_wait_timeout(self._h, bound_cycles, stream), self._h)

    def close(self):
        if getattr(self, "_h", None):
            lib().lrs_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
