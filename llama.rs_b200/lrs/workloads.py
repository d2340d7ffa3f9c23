"""Seeded synthetic sampler workloads (no dataset exists for this path; the reference
measures nothing on the sampler, so these stand in with the shapes and value
distributions of the five benchmark configurations).

Every row is generated from its own numpy PCG64 stream seeded with (base_seed, row),
so any subset of rows can be regenerated identically (tests take small subsets of the
full-size configurations).  Values are computed in float64 and rounded to float32.

Configurations (rows x vocab, history window W):
  single    1 x 151,936, N(0,3), W=64, penalty 1.1, temp 0.8, top_k 40, top_p 0.95
  greedy    256 x 151,936, N(0,3), 10% of rows with the max planted at 2-4 positions
  mixed     1024 x 109,051, Gumbel(0,1) - 2.2*ln(rank) under a per-row permutation,
            temp U[0.5,1.5], top_k in {0,20,40,100}, top_p U[0.8,1.0], penalty U[1.0,1.3], W=64
  headline  the mixed parameter mix at 1024 x 151,936
  nucleus   4096 x 151,936, top_k 0, top_p 0.9, temp 1.0, even rows N(0,0.5),
            odd rows N(0,2) with +12 at one random index, penalty 1.2, W=1024
  vocab_sharded 64 x 151,936, rows alternate the mixed and nucleus generators,
            top_k 50, top_p 0.95, temp 0.7, penalty 1.0
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

PARAMS_DTYPE = np.dtype([
    ("temperature", "<f4"), ("top_k", "<u4"), ("top_p", "<f4"),
    ("repetition_penalty", "<f4"), ("repeat_last_n", "<u4"), ("reserved", "<u4"),
])

QWEN_VOCAB = 151_936
PRUNED_VOCAB = 109_051


@dataclass
class Workload:
    name: str
    logits: np.ndarray      # (rows, ld) float32, ld == vocab
    vocab: int
    hist: np.ndarray        # (rows, W) uint32
    hist_len: np.ndarray    # (rows,) uint32
    params: np.ndarray      # (rows,) PARAMS_DTYPE
    state: np.ndarray       # (rows,) uint64 PRNG states (seed | 1)

    @property
    def rows(self) -> int:
        return self.logits.shape[0]

    @property
    def window(self) -> int:
        return self.hist.shape[1]


def _rng(base: int, row: int) -> np.random.Generator:
    return np.random.default_rng([base, row])


def _zipf_row(rng, vocab):
    g = -np.log(-np.log(rng.random(vocab)))
    head = -2.2 * np.log(np.arange(1, vocab + 1, dtype=np.float64))
    x = np.empty(vocab, np.float64)
    x[rng.permutation(vocab)] = g + head
    return x.astype(np.float32)


def _mixed_params(rng, p):
    p["temperature"] = np.float32(rng.uniform(0.5, 1.5))
    p["top_k"] = (0, 20, 40, 100)[int(rng.integers(0, 4))]
    p["top_p"] = np.float32(rng.uniform(0.8, 1.0))
    p["repetition_penalty"] = np.float32(rng.uniform(1.0, 1.3))
    p["repeat_last_n"] = 64


def _state(seed: int) -> np.uint64:
    return np.uint64((seed | 1) & 0xFFFFFFFFFFFFFFFF)


def _alloc(name, rows, vocab, window):
    return Workload(name, np.empty((rows, vocab), np.float32), vocab,
                    np.zeros((rows, window), np.uint32), np.full(rows, window, np.uint32),
                    np.zeros(rows, PARAMS_DTYPE), np.zeros(rows, np.uint64))


def single(rows: int = 1) -> Workload:
    """Config 1: one row repeated `rows` times (the same logits and history)."""
    rng = np.random.default_rng(42)
    vocab, window = QWEN_VOCAB, 64
    x = (rng.standard_normal(vocab) * 3.0).astype(np.float32)
    h = rng.integers(0, vocab, window).astype(np.uint32)
    w = _alloc("single", rows, vocab, window)
    w.logits[:] = x
    w.hist[:] = h
    w.params["temperature"] = 0.8
    w.params["top_k"] = 40
    w.params["top_p"] = 0.95
    w.params["repetition_penalty"] = 1.1
    w.params["repeat_last_n"] = 64
    w.state[:] = _state(42)
    return w


def greedy(rows: int = 256, vocab: int = QWEN_VOCAB, row_ids=None) -> Workload:
    """Config 2: greedy argmax with planted ties in 10% of rows."""
    ids = np.arange(rows) if row_ids is None else np.asarray(row_ids)
    w = _alloc("greedy", len(ids), vocab, 0)
    for i, r in enumerate(ids):
        rng = _rng(2, int(r))
        x = rng.standard_normal(vocab) * 3.0
        if r % 10 == 3:
            m = x.max() + abs(rng.standard_normal()) + 0.5
            pos = rng.choice(vocab, size=int(rng.integers(2, 5)), replace=False)
            x[pos] = m
        w.logits[i] = x.astype(np.float32)
        w.state[i] = _state(1000 + int(r))
    w.params["temperature"] = 0.0
    w.params["top_k"] = 0
    w.params["top_p"] = 1.0
    w.params["repetition_penalty"] = 1.0
    w.params["repeat_last_n"] = 64
    return w


def mixed(rows: int = 1024, vocab: int = PRUNED_VOCAB, row_ids=None, name="mixed", base=3) -> Workload:
    """Config 3 (and the headline at vocab=151,936): Zipf-like rows, mixed parameters."""
    ids = np.arange(rows) if row_ids is None else np.asarray(row_ids)
    w = _alloc(name, len(ids), vocab, 64)
    for i, r in enumerate(ids):
        rng = _rng(base, int(r))
        w.logits[i] = _zipf_row(rng, vocab)
        w.hist[i] = rng.integers(0, vocab, 64).astype(np.uint32)
        _mixed_params(rng, w.params[i:i + 1])
        w.state[i] = _state(int(rng.integers(0, 2**63)))
    return w


def headline(rows: int = 1024, row_ids=None) -> Workload:
    """The metric's configuration: config-3 parameter mix at 1024 x 151,936."""
    return mixed(rows, QWEN_VOCAB, row_ids, name="headline", base=33)


def nucleus(rows: int = 4096, vocab: int = QWEN_VOCAB, row_ids=None, window: int = 1024) -> Workload:
    """Config 4: full-vocab nucleus stress (flat and spiked rows)."""
    ids = np.arange(rows) if row_ids is None else np.asarray(row_ids)
    w = _alloc("nucleus", len(ids), vocab, window)
    for i, r in enumerate(ids):
        rng = _rng(4, int(r))
        if r % 2 == 0:
            x = rng.standard_normal(vocab) * 0.5
        else:
            x = rng.standard_normal(vocab) * 2.0
            x[int(rng.integers(0, vocab))] += 12.0
        w.logits[i] = x.astype(np.float32)
        w.hist[i] = rng.integers(0, vocab, window).astype(np.uint32)
        w.state[i] = _state(int(rng.integers(0, 2**63)))
    w.params["temperature"] = 1.0
    w.params["top_k"] = 0
    w.params["top_p"] = 0.9
    w.params["repetition_penalty"] = 1.2
    w.params["repeat_last_n"] = window
    return w


def vocab_sharded(rows: int = 64, vocab: int = QWEN_VOCAB, row_ids=None) -> Workload:
    """Config 5: rows alternate the mixed and nucleus generators; global sampler params."""
    ids = np.arange(rows) if row_ids is None else np.asarray(row_ids)
    w = _alloc("vocab_sharded", len(ids), vocab, 64)
    for i, r in enumerate(ids):
        rng = _rng(5, int(r))
        if r % 2 == 0:
            w.logits[i] = _zipf_row(rng, vocab)
        elif r % 4 == 1:
            w.logits[i] = (rng.standard_normal(vocab) * 0.5).astype(np.float32)
        else:
            x = rng.standard_normal(vocab) * 2.0
            x[int(rng.integers(0, vocab))] += 12.0
            w.logits[i] = x.astype(np.float32)
        w.hist[i] = rng.integers(0, vocab, 64).astype(np.uint32)
        w.state[i] = _state(int(rng.integers(0, 2**63)))
    w.params["temperature"] = 0.7
    w.params["top_k"] = 50
    w.params["top_p"] = 0.95
    w.params["repetition_penalty"] = 1.0
    w.params["repeat_last_n"] = 64
    return w


CONFIGS = {
    "single": single,
    "greedy": greedy,
    "mixed": mixed,
    "headline": headline,
    "nucleus": nucleus,
    "vocab_sharded": vocab_sharded,
}


def xorshift_states(state: int, count: int) -> np.ndarray:
    """States after 0..count-1 draws of sampler.rs:40-48 from `state` (one u64 per draw)."""
    out = np.empty(count, np.uint64)
    x = int(state)
    m = 0xFFFFFFFFFFFFFFFF
    for i in range(count):
        out[i] = x
        x ^= x >> 12
        x ^= (x << 25) & m
        x ^= x >> 27
    return out
