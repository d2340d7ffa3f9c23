"""ctypes front end of the CPU oracle (oracle/sampler_ref.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by the
cpu_baseline / --impl reference legs of bench.py, never by the product library.
The oracle restates rust-llama src/sampler.rs:40-163 and src/ops.rs:397-419; see the
header of sampler_ref.cpp for what is pinned by the reference's own tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblrs_oracle.so")

# Same layout as lrs_params in include/llamars_sampler.h.
PARAMS_DTYPE = np.dtype([
    ("temperature", "<f4"), ("top_k", "<u4"), ("top_p", "<f4"),
    ("repetition_penalty", "<f4"), ("repeat_last_n", "<u4"), ("reserved", "<u4"),
])
# lrs_row_info followed by the oracle-only flags word.
ROW_INFO_FIELDS = [
    ("status", "<i4"), ("token", "<u4"), ("path", "<u4"), ("k", "<u4"), ("cutoff", "<u4"),
    ("pos", "<u4"), ("max", "<f4"), ("sum_exp", "<f4"), ("surv_sum", "<f4"), ("r0", "<f4"),
    ("prob", "<f4"), ("n_cand", "<u4"), ("events", "<u4"), ("cycles", "<u4", (8,)),
    ("reserved", "<u4"),
]
INFO_DTYPE = np.dtype(ROW_INFO_FIELDS + [("flags", "<u4"), ("pad", "<u4")])

FLAG_KTIE = 1
FLAG_DRAWTIE = 2
FLAG_CUTTIE = 4
UNPINNED = FLAG_KTIE | FLAG_DRAWTIE | FLAG_CUTTIE

_lib = None
_lock = threading.Lock()


def build() -> str:
    """Compile the oracle with its Makefile (g++, strict IEEE flags)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                build()
            L = ctypes.CDLL(LIB_PATH)
            P = ctypes.c_void_p
            L.lrs_ref_sample.restype = ctypes.c_uint32
            L.lrs_ref_sample.argtypes = [P, ctypes.c_size_t, P, P, ctypes.c_size_t, P, P]
            L.lrs_ref_sample_batch.restype = None
            L.lrs_ref_sample_batch.argtypes = [P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64,
                                               P, ctypes.c_uint64, P, P, P, P, P, ctypes.c_int]
            L.lrs_ref_seed_state.restype = ctypes.c_uint64
            L.lrs_ref_seed_state.argtypes = [ctypes.c_uint64]
            L.lrs_ref_next_u64.restype = ctypes.c_uint64
            L.lrs_ref_next_u64.argtypes = [P]
            L.lrs_ref_next_f32.restype = ctypes.c_float
            L.lrs_ref_next_f32.argtypes = [P]
            L.lrs_ref_softmax.restype = None
            L.lrs_ref_softmax.argtypes = [P, ctypes.c_size_t, P, P]
            L.lrs_ref_probs.restype = None
            L.lrs_ref_probs.argtypes = [P, ctypes.c_size_t, P, P, ctypes.c_size_t, P]
            L.lrs_ref_sizeof_info.restype = ctypes.c_size_t
            L.lrs_ref_sizeof_params.restype = ctypes.c_size_t
            assert L.lrs_ref_sizeof_info() == INFO_DTYPE.itemsize
            assert L.lrs_ref_sizeof_params() == PARAMS_DTYPE.itemsize
            _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def make_params(temperature=0.7, top_k=40, top_p=0.95, repetition_penalty=1.1,
                repeat_last_n=64, rows=None):
    """Build lrs_params records (scalars, or per-row arrays when rows is given)."""
    if rows is None:
        p = np.zeros((), PARAMS_DTYPE)
    else:
        p = np.zeros(rows, PARAMS_DTYPE)
    p["temperature"] = temperature
    p["top_k"] = top_k
    p["top_p"] = top_p
    p["repetition_penalty"] = repetition_penalty
    p["repeat_last_n"] = repeat_last_n
    return p


def seed_state(seed: int) -> int:
    """Sampler::new(seed).state (sampler.rs:33-37)."""
    return int(lib().lrs_ref_seed_state(ctypes.c_uint64(seed & (2**64 - 1))))


def next_u64(state: int) -> tuple[int, int]:
    """One xorshift64* step (sampler.rs:40-48): returns (output, new_state)."""
    s = np.array([state], np.uint64)
    out = lib().lrs_ref_next_u64(s.ctypes.data)
    return int(out), int(s[0])


def sample_one(logits: np.ndarray, params, recent, state: int):
    """Sampler{state}.sample(logits, params, recent) -> (token, info, new_state)."""
    x = np.ascontiguousarray(logits, np.float32)
    r = np.ascontiguousarray(np.asarray(recent, np.uint32).reshape(-1))
    p = np.ascontiguousarray(np.asarray(params, PARAMS_DTYPE).reshape(()))
    s = np.array([state], np.uint64)
    info = np.zeros((), INFO_DTYPE)
    tok = lib().lrs_ref_sample(x.ctypes.data, x.size, p.ctypes.data, r.ctypes.data, r.size,
                               s.ctypes.data, info.ctypes.data)
    return int(tok), info, int(s[0])


def sample_batch(logits: np.ndarray, n: int, hist: np.ndarray | None, hist_len: np.ndarray | None,
                 params: np.ndarray, state: np.ndarray, threads: int = 1):
    """Independent samplers per row.  logits (rows, ld) f32; hist (rows, hist_ld) u32.
    A single logits row with more than one parameter record is shared by every row
    (ld = 0), as the C ABI allows.

    Returns (tokens u32[rows], infos INFO_DTYPE[rows], new_state u64[rows])."""
    if logits.ndim == 2 and logits.shape[0] > 1 and logits.strides[0] == 0:
        logits = logits[:1]  # a broadcast row: share it instead of materialising every copy
    logits = np.ascontiguousarray(logits, np.float32)
    if logits.ndim == 1:
        logits = logits.reshape(1, -1)
    rows, ld = logits.shape[0], logits.shape[1]
    if rows == 1 and np.size(params) > 1:
        rows, ld = int(np.size(params)), 0
    if hist is not None:
        hist = np.ascontiguousarray(hist, np.uint32)
        hist_ld = hist.shape[1]
        hist_len = np.ascontiguousarray(hist_len, np.uint32)
    else:
        hist_ld = 0
    params = np.ascontiguousarray(params, PARAMS_DTYPE)
    st = np.array(state, np.uint64, copy=True)
    tokens = np.zeros(rows, np.uint32)
    infos = np.zeros(rows, INFO_DTYPE)
    lib().lrs_ref_sample_batch(logits.ctypes.data, rows, n, ld, _ptr(hist), hist_ld, _ptr(hist_len),
                               params.ctypes.data, st.ctypes.data, tokens.ctypes.data,
                               infos.ctypes.data, int(threads))
    return tokens, infos, st


def probs(logits: np.ndarray, params, recent) -> np.ndarray:
    """Probability vector after penalty, temperature and softmax (sampler.rs:72-119)."""
    x = np.ascontiguousarray(logits, np.float32)
    r = np.ascontiguousarray(np.asarray(recent, np.uint32).reshape(-1))
    p = np.ascontiguousarray(np.asarray(params, PARAMS_DTYPE).reshape(()))
    out = np.empty_like(x)
    lib().lrs_ref_probs(x.ctypes.data, x.size, p.ctypes.data, r.ctypes.data, r.size, out.ctypes.data)
    return out
