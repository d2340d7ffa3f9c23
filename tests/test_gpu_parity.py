"""GPU parity: the CUDA sampler against the CPU oracle, bit for bit.

Every row's token, status, PRNG state, softmax max and sum, survivor sum, draw value,
cutoff, drawn position and token probability must equal the oracle's (the oracle
restates src/sampler.rs:40-163 and src/ops.rs:397-419).  Inputs are the seeded
synthetic configurations of lrs.workloads at reduced row counts, the golden fixtures,
and edge cases the reference's semantics single out.
"""
import os

import numpy as np
import pytest

import lrs
from lrs import workloads as W
import oracle as O
from gpu_util import compare, run_device, run_oracle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _check_workload(w, label, rows=None):
    gpu = run_device(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    ref = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    return compare(gpu, ref, label)


def test_reference_kats_single_row_api():
    # sampler.rs:181-206 through the Sampler drop-in (lrs_sampler_sample)
    gp = lambda pen, n: lrs.SamplingParams(temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=pen,
                                           repeat_last_n=n, seed=1)
    s = lrs.Sampler(1)
    lg = np.array([10.0, 1.0], np.float32)
    assert s.sample(lg, gp(2.0, 64), [0, 0, 0, 0]) == 0
    assert s.sample(lg, gp(20.0, 2), [7, 7, 0]) == 1
    assert s.sample(lg, gp(20.0, 2), [0, 7, 7]) == 0
    assert s.sample(lg, gp(1.0, 64), [0, 0, 0]) == 0


@pytest.mark.parametrize("name", ["small_mixed", "small_edges"])
def test_golden_fixtures(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    tok, infos, st, probs, status = run_device(z["logits"], int(z["n"]), z["hist"], z["hist_len"], z["params"],
                                               z["state"])
    np.testing.assert_array_equal(status, z["status"])
    np.testing.assert_array_equal(tok, z["tokens"])
    np.testing.assert_array_equal(st, z["state_out"])
    ok = z["status"] == 0
    np.testing.assert_array_equal(probs[ok].view(np.uint32), z["prob"][ok].view(np.uint32))


def test_headline_rows():
    w = W.headline(row_ids=range(0, 1024, 16))  # 64 rows of the metric's configuration
    assert _check_workload(w, "headline") == 64


def test_mixed_pruned_vocab_unaligned_rows():
    w = W.mixed(row_ids=range(0, 1024, 16))  # 109,051-wide rows: every other row is misaligned
    assert _check_workload(w, "mixed") == 64


def test_greedy_rows_with_planted_ties():
    w = W.greedy(row_ids=range(0, 256, 4))
    assert _check_workload(w, "greedy") == 64


def test_nucleus_stress_rows():
    w = W.nucleus(row_ids=range(0, 4096, 256))  # flat and spiked rows, window 1024
    assert _check_workload(w, "nucleus") == 16


def test_vocab_sharded_rows_unsharded():
    w = W.vocab_sharded(row_ids=range(0, 64, 4))
    assert _check_workload(w, "vocab_sharded") == 16


def test_single_row_stream_shared_logits():
    # Config 1: 2,000 successive draws on the same logits and history.  The GPU takes
    # them as 2,000 rows that share one logits row (ld = 0) with the per-draw states
    # precomputed; the oracle draws them one after the other.
    draws = 2000
    w = W.single(1)
    states = W.xorshift_states(int(w.state[0]), draws)
    params = np.repeat(w.params, draws)
    hist = np.repeat(w.hist, draws, axis=0)
    hl = np.repeat(w.hist_len, draws)
    tok, infos, st, probs, status = run_device(w.logits, w.vocab, hist, hl, params, states, ld=0)
    s = int(w.state[0])
    ref = []
    for i in range(draws):
        t, _, s = O.sample_one(w.logits[0], w.params[0], w.hist[0], s)
        ref.append(t)
    np.testing.assert_array_equal(tok, np.array(ref, np.uint32))
    assert (status == 0).all()


def _edge_rows(n, rows, rng):
    x = (rng.standard_normal((rows, n)) * 2).astype(np.float32)
    p = O.make_params(rows=rows)
    p["temperature"] = rng.choice([0.0, 0.5, 1.0, 1.7], rows)
    p["top_k"] = rng.choice([0, 1, 3, n, n + 1], rows)
    p["top_p"] = rng.choice([0.0, 0.3, 0.9, 1.0], rows)
    p["repetition_penalty"] = rng.choice([1.0, 1.2, 0.7], rows)
    p["repeat_last_n"] = rng.choice([0, 2, 64], rows)
    hist = rng.integers(0, n + 3, (rows, 12)).astype(np.uint32)
    hl = rng.integers(0, 13, rows).astype(np.uint32)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    return x, p, hist, hl, st


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 7, 31, 64, 255, 1000, 4097, 8195])
def test_small_vocab_fuzz(n):
    rng = np.random.default_rng(1000 + n)
    x, p, hist, hl, st = _edge_rows(n, 96, rng)
    gpu = run_device(x, n, hist, hl, p, st)
    ref = run_oracle(x, n, hist, hl, p, st)
    compare(gpu, ref, f"fuzz n={n}")


def test_special_values():
    n, rows = 151_936, 12
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    x[0] = 0.25                        # all equal: one bucket holds the whole row
    x[1, 100] = np.nan                 # NaN -> panic row
    x[2, 5] = np.inf                   # +inf -> panic row
    x[3, :] = -np.inf; x[3, 77] = 1.0  # one finite logit
    x[4] = np.round(x[4] * 4) / 4      # heavy ties
    x[5] *= 1e-5                       # nearly flat: nucleus ~ whole vocabulary
    p = O.make_params(rows=rows)
    p["temperature"] = [1.0, 0.7, 0.7, 0.9, 0.8, 1.0, 1e-30, 0.7, float("nan"), 0.7, 0.7, 0.7]
    p["top_k"] = [0, 40, 0, 0, 0, 0, 0, 0, 40, 0, 1, 0]
    p["top_p"] = [0.9, 0.95, 0.9, 0.99, 0.95, 0.5, 0.9, 1e-7, 0.9, 1.0, 0.9, 0.97]
    p["repetition_penalty"] = [1.0, 1.1, 1.0, 1.0, 1.1, 1.0, 1.0, 1.1, 1.0, 1.0, 0.0, 1.3]
    p["repeat_last_n"] = 64
    hist = rng.integers(0, n, (rows, 64)).astype(np.uint32)
    hl = np.full(rows, 64, np.uint32)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    gpu = run_device(x, n, hist, hl, p, st)
    ref = run_oracle(x, n, hist, hl, p, st)
    compare(gpu, ref, "special")


def test_padded_rows_and_no_history():
    rng = np.random.default_rng(9)
    rows, n, ld = 8, 5000, 5003
    buf = (rng.standard_normal((rows, ld)) * 3).astype(np.float32)
    p = O.make_params(0.8, 40, 0.95, 1.0, 64, rows=rows)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    empty = np.zeros((rows, 0), np.uint32)
    gpu = run_device(buf, n, empty, np.zeros(rows, np.uint32), p, st, ld=ld)
    ref = run_oracle(np.ascontiguousarray(buf[:, :n]), n, None, None, p, st)
    compare(gpu, ref, "padded")


def test_host_entry_point_matches_device_entry_point():
    w = W.headline(row_ids=range(5, 1024, 64))
    bs = lrs.BatchSampler(len(w.params), w.vocab, w.window)
    bs.set_params(w.params)
    bs.set_state(w.state)
    tok, probs = bs.sample(w.logits, hist=w.hist, hist_len=w.hist_len, probs=True)
    st = bs.get_state(len(w.params))
    rtok, rinfo, rst = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    np.testing.assert_array_equal(tok, rtok)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(probs.view(np.uint32), rinfo["prob"].view(np.uint32))
    bs.close()


def test_nan_row_raises_panic_error_single_row():
    s = lrs.Sampler(3)
    x = np.array([1.0, np.nan, 0.5], np.float32)
    with pytest.raises(lrs.SamplerPanic):
        s.sample(x, lrs.SamplingParams(), [])
    assert s.state == 3  # untouched
