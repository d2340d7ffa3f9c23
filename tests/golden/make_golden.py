"""Generates the golden fixtures of tests/golden/ from the CPU oracle.

The fixtures pin the oracle's outputs (tokens, PRNG states, softmax sums, token
probabilities, statuses) on small seeded inputs so that later changes to the oracle
or the GPU path are compared against fixed vectors.  Run from the repository root:
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "llama.rs_b200"))

import oracle as O  # noqa: E402
from lrs import workloads as W  # noqa: E402


def small_mixed():
    rows, n = 48, 3001
    w = W.mixed(rows, n, name="small_mixed", base=101)
    return w.logits, n, w.hist, w.hist_len, w.params, w.state


def small_edges():
    n, rows = 64, 16
    rng = np.random.default_rng(202)
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    x[1] = 1.5                                   # all equal
    x[2, 7] = np.nan                             # NaN -> panic row
    x[3, 0] = np.inf                             # +inf max -> panic row
    x[4] = -np.inf; x[4, 9] = 0.0                # -inf everywhere but one
    x[5] = np.round(x[5])                        # integer ties
    x[6, ::3] = x[6].max() + 1                   # planted max ties
    x[7] *= 1e-6                                 # nearly flat
    x[8] *= 40                                   # very peaked
    hist = rng.integers(0, n + 4, (rows, 16)).astype(np.uint32)
    hist_len = rng.integers(0, 17, rows).astype(np.uint32)
    p = O.make_params(rows=rows)
    p["temperature"] = [0.7, 1.0, 0.7, 0.7, 0.7, 1.3, 0.0, 0.9, 0.5, 1e-3, -1.0, 0.7, 2.0, 0.7, 0.7, 0.8]
    p["top_k"] = [40, 0, 5, 0, 3, 7, 0, 0, 2, 1, 0, 64, 65, 63, 10, 0]
    p["top_p"] = [0.95, 0.9, 1.0, 0.5, 0.99, 0.7, 1.0, 0.999, 0.5, 0.95, 1.0, 0.0, 1.0, 0.2, 1.0, 1e-7]
    p["repetition_penalty"] = [1.1, 1.2, 1.0, 1.0, 1.3, 1.1, 1.0, 0.0, 2.0, 1.1, 1.5, 1.0, 1.0, 1.1, 0.5, 1.1]
    p["repeat_last_n"] = [64, 0, 4, 64, 2, 64, 64, 1, 0, 64, 64, 64, 64, 3, 64, 64]
    state = (rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1))
    return x, n, hist, hist_len, p, state


def main():
    O.build()
    for name, fn in (("small_mixed", small_mixed), ("small_edges", small_edges)):
        logits, n, hist, hist_len, params, state = fn()
        tokens, infos, st = O.sample_batch(logits, n, hist, hist_len, params, state)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), logits=logits, n=n, hist=hist, hist_len=hist_len,
                            params=params, state=state, tokens=tokens, state_out=st, sum_exp=infos["sum_exp"],
                            prob=infos["prob"], status=infos["status"], cutoff=infos["cutoff"], pos=infos["pos"],
                            flags=infos["flags"])
        print(name, "rows", len(tokens), "statuses", np.unique(infos["status"]).tolist())


if __name__ == "__main__":
    main()
