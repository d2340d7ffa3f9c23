"""Second, independent restatement of rust-llama's sampler in pure Python (small inputs only).

Used to cross-check the C++ oracle (oracle/sampler_ref.cpp).  f32 arithmetic is
numpy float32 scalar arithmetic (one IEEE binary32 rounding per operation) and exp is
libm's expf called through ctypes, which is what Rust's f32::exp calls on
x86_64-linux-gnu.  Follows src/sampler.rs:40-163 and src/ops.rs:397-419 line by line;
equal probabilities are ordered by index (see the oracle's header on tie order).
"""
from __future__ import annotations

import ctypes
import ctypes.util

import numpy as np

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
F = np.float32
M64 = 0xFFFFFFFFFFFFFFFF


def expf(x) -> np.float32:
    return F(_libm.expf(float(x)))


def next_u64(state: int) -> tuple[int, int]:
    x = state
    x ^= x >> 12
    x ^= (x << 25) & M64
    x ^= x >> 27
    return (x * 0x2545F4914F6CDD1D) & M64, x


def next_f32(state: int) -> tuple[np.float32, int]:
    out, state = next_u64(state)
    return F(F(out >> 40) / F(1 << 24)), state


def sample(logits, temperature, top_k, top_p, penalty, last_n, recent, state):
    """Returns (token or None on panic, new_state, probs or None)."""
    with np.errstate(all="ignore"):
        x = [F(v) for v in logits]
        n = len(x)
        temperature, top_p, penalty = F(temperature), F(top_p), F(penalty)
        if n == 0:
            return 0, state, None
        if temperature <= 0 and penalty == F(1.0):
            best = 0
            for i in range(1, n):
                if x[i] > x[best]:
                    best = i
            return best, state, None
        probs = list(x)
        if penalty != F(1.0):
            start = 0 if last_n == 0 else max(len(recent) - last_n, 0)
            seen = []
            for t in recent[start:]:
                t = int(t)
                if t >= n or t in seen:
                    continue
                seen.append(t)
                probs[t] = F(probs[t] / penalty) if probs[t] > 0 else F(probs[t] * penalty)
        if temperature <= 0:
            best = 0
            for i in range(1, n):
                if probs[i] > probs[best]:
                    best = i
            return best, state, None
        inv_t = F(F(1.0) / temperature)
        probs = [F(p * inv_t) for p in probs]
        mx = probs[0]
        for v in probs[1:]:
            if v > mx:
                mx = v
        s = F(0.0)
        for i in range(n):
            probs[i] = expf(F(probs[i] - mx))
            s = F(s + probs[i])
        if s > 0:
            inv = F(F(1.0) / s)
            probs = [F(p * inv) for p in probs]
        if n >= 2 and any(np.isnan(p) for p in probs):
            return None, state, probs
        k = n if (top_k == 0 or top_k > n) else top_k
        idx = sorted(range(n), key=lambda i: (-float(probs[i]), i))[:k]
        cutoff = len(idx)
        if F(0.0) < top_p < F(1.0):
            cum = F(0.0)
            for pos, i in enumerate(idx):
                cum = F(cum + probs[i])
                if cum >= top_p:
                    cutoff = pos + 1
                    break
        idx = idx[:cutoff]
        tot = F(0.0)
        for i in idx:
            tot = F(tot + probs[i])
        if tot <= 0:
            return idx[0], state, probs
        u, state = next_f32(state)
        r = F(u * tot)
        for i in idx:
            r = F(r - probs[i])
            if r <= 0:
                return i, state, probs
        return idx[-1], state, probs
