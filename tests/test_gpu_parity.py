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


def test_many_short_rows_every_claim_key():
    # More rows than the ordering pass's block has threads and than the grid has CTAs,
    # so rows are claimed in cost order (every temperature band, both finishes, greedy
    # rows last), on short misaligned rows; the results must not depend on the order.
    rng = np.random.default_rng(11)
    rows, n, ld = 2500, 2003, 2005
    buf = (rng.standard_normal((rows, ld)) * 3).astype(np.float32)
    p = O.make_params(rows=rows)
    p["temperature"] = rng.choice(np.array([0.0, 0.05, 0.3, 0.5, 0.7, 0.9, 1.1, 1.3, 1.5, 2.5], np.float32), rows)
    p["top_k"] = rng.choice(np.array([0, 1, 40, 128, 200, n], np.uint32), rows)
    p["top_p"] = rng.choice(np.array([0.5, 0.9, 0.99, 1.0], np.float32), rows)
    p["repetition_penalty"] = rng.choice(np.array([1.0, 1.2], np.float32), rows)
    p["repeat_last_n"] = 64
    hist = rng.integers(0, n, (rows, 64)).astype(np.uint32)
    hl = rng.integers(0, 65, rows).astype(np.uint32)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    gpu = run_device(buf, n, hist, hl, p, st, ld=ld)
    ref = run_oracle(np.ascontiguousarray(buf[:, :n]), n, hist, hl, p, st)
    assert compare(gpu, ref, "many short rows") == rows



def test_regathered_nucleus_with_edge_elements():
    # Long misaligned rows whose 0.999 nucleus (about 7,000 high logits) is deeper than the
    # rank-limited list, so the finish gathers it again from the row; the unaligned head and
    # tail elements (outside the 16-byte-aligned tiles) are among the high ones and must be
    # gathered too, whatever the number of tiles.
    rng = np.random.default_rng(23)
    rows, n, ld = 4, 151_937, 151_941
    buf = np.full((rows, ld), -40.0, np.float32)
    for r in range(rows):
        hi = rng.choice(n, 7000, replace=False)
        buf[r, hi] = rng.uniform(0.0, 1.0, 7000).astype(np.float32)
        buf[r, [0, 1, 2, n - 3, n - 2, n - 1]] = rng.uniform(0.5, 1.0, 6).astype(np.float32)
    p = O.make_params(rows=rows, temperature=1.0, top_k=0, top_p=0.999, repetition_penalty=1.0)
    st = (np.arange(rows, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)) | np.uint64(1)
    gpu = run_device(buf, n, None, None, p, st, ld=ld)
    ref = run_oracle(np.ascontiguousarray(buf[:, :n]), n, None, None, p, st)
    assert compare(gpu, ref, "regathered nucleus") == rows
    infos = gpu[1]
    staged = infos["cycles"][:, 4] == 1
    assert staged.all()
    assert (infos["cycles"][:, 3] > 0).any(), "no row took the regather path"

def test_greedy_rows_with_planted_ties():
    w = W.greedy(row_ids=range(0, 256, 4))
    assert _check_workload(w, "greedy") == 64


def test_nucleus_stress_rows():
    w = W.nucleus(row_ids=range(0, 4096, 256))  # flat and spiked rows, window 1024
    assert _check_workload(w, "nucleus") == 16


def test_vocab_sharded_rows_unsharded():
    w = W.vocab_sharded(row_ids=range(0, 64, 4))
    assert _check_workload(w, "vocab_sharded") == 16


def _unpinned_rows(ref, label):
    """Rows whose token could depend on how Rust's select_nth_unstable orders equal
    probabilities (oracle flags KTIE / DRAWTIE / CUTTIE): counted, printed and required
    to be zero on the benchmark configurations, so that bit-exact agreement with the
    oracle is agreement with the reference (sampler.rs:122-162)."""
    flagged = int(((ref[1]["flags"] & O.UNPINNED) != 0).sum())
    print(f"{label}: {flagged} of {len(ref[0])} rows with an unpinned tie order")
    return flagged


def test_single_row_stream_shared_logits():
    # Config 1 in full: 10,000 successive draws on the same logits and history.  The GPU
    # takes them as 10,000 rows that share one logits row (ld = 0), each with the state
    # the stream has reached before it; every row's token, final state and intermediates
    # must equal the oracle's, and each row's final state must be the next row's start
    # state, so the GPU reproduces the whole token stream of Sampler::new(42).
    draws = 10_000
    w = W.single(1)
    states = W.xorshift_states(int(w.state[0]), draws)
    params = np.repeat(w.params, draws)
    hist = np.repeat(w.hist, draws, axis=0)
    hl = np.repeat(w.hist_len, draws)
    gpu = run_device(w.logits, w.vocab, hist, hl, params, states, ld=0)
    ref = O.sample_batch(w.logits, w.vocab, hist, hl, params, states, threads=os.cpu_count() or 8)
    assert compare(gpu, ref, "config 1 stream") == draws
    st = gpu[2]
    assert (st[:-1] == states[1:]).all()  # one next_u64 per draw: the stream continues row to row
    assert _unpinned_rows(ref, "config 1") == 0


def test_greedy_config_full():
    """Config 2 in full: all 256 greedy rows, planted ties included."""
    w = W.greedy()
    assert _check_workload(w, "config 2 full") == 256


def test_mixed_config_full():
    """Config 3 in full: all 1,024 rows of 109,051 (pruned vocabulary, misaligned rows)."""
    w = W.mixed()
    gpu = run_device(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    ref = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state, threads=os.cpu_count() or 8)
    assert compare(gpu, ref, "config 3 full") == 1024
    assert _unpinned_rows(ref, "config 3") == 0


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
    bs.poll_error()  # no launch error is pending
    bs.close()


def test_nan_row_raises_panic_error_single_row():
    s = lrs.Sampler(3)
    x = np.array([1.0, np.nan, 0.5], np.float32)
    with pytest.raises(lrs.SamplerPanic):
        s.sample(x, lrs.SamplingParams(), [])
    assert s.state == 3  # untouched


def test_headline_full_size():
    """Every row of the metric's configuration (1024 x 151,936), bit for bit."""
    w = W.headline()
    gpu = run_device(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    ref = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state, threads=os.cpu_count() or 8)
    assert compare(gpu, ref, "headline full") == 1024
    assert _unpinned_rows(ref, "headline") == 0


@pytest.mark.parametrize("block", range(4))
def test_nucleus_stress_config_full(block):
    """Config 4 in full (4096 x 151,936, window 1024), in four blocks of 1,024 rows so
    that the host holds one block at a time and the oracle finishes each in seconds."""
    w = W.nucleus(row_ids=range(block * 1024, (block + 1) * 1024))
    gpu = run_device(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    ref = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state, threads=os.cpu_count() or 8)
    assert compare(gpu, ref, f"config 4 block {block}") == 1024
    assert _unpinned_rows(ref, f"config 4 block {block}") == 0


def test_candidate_bound_edges():
    """Rows that stress the pass-1 candidate lists: the running max grows in every tile,
    the max sits in the last element, every element is a candidate (temperature 1e3),
    almost none is (temperature 0.02), and elements placed at the 18.1 bound."""
    n, rows = 151_936, 10
    rng = np.random.default_rng(21)
    i = np.arange(n, dtype=np.float64)
    x = np.empty((rows, n), np.float32)
    x[0] = i * 1e-4                                        # slow ramp: everything within 18.1
    x[1] = i * 4e-4                                        # steep ramp: early tiles far below the final max
    x[2] = rng.standard_normal(n); x[2, n - 1] = 30.0      # spike in the last element
    x[3] = rng.standard_normal(n) * 3                      # temperature 1e3 below
    x[4] = rng.standard_normal(n) * 3                      # temperature 0.02 below
    x[5] = -18.1 + rng.uniform(-0.02, 0.02, n); x[5, 0] = 0.0   # at the bound, max first
    x[6] = -18.1 + rng.uniform(-0.02, 0.02, n); x[6, n - 1] = 0.0  # at the bound, max last
    x[7] = -18.8 + rng.uniform(-0.02, 0.02, n); x[7, 1000] = 0.0
    x[8] = np.where(rng.random(n) < 0.02, rng.standard_normal(n), -40.0)  # sparse live elements
    x[9] = np.where((i // 1024) % 2 == 0, rng.standard_normal(n), -30.0)  # dense and empty tiles alternate
    p = O.make_params(rows=rows)
    p["temperature"] = [1.0, 1.0, 1.0, 1e3, 0.02, 1.0, 1.0, 1.0, 1.0, 1.3]
    p["top_k"] = [0, 0, 40, 0, 100, 0, 0, 20, 0, 0]
    p["top_p"] = [0.9, 1.0, 0.95, 0.999, 1.0, 1.0, 0.9, 1.0, 0.95, 0.97]
    p["repetition_penalty"] = [1.0, 1.1, 1.0, 1.2, 1.0, 1.0, 1.3, 1.0, 1.1, 1.0]
    p["repeat_last_n"] = 64
    hist = rng.integers(0, n, (rows, 64)).astype(np.uint32)
    hl = np.full(rows, 64, np.uint32)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    gpu = run_device(x, n, hist, hl, p, st)
    ref = run_oracle(x, n, hist, hl, p, st)
    compare(gpu, ref, "candidate bound")


def test_rows_longer_than_two_to_the_21():
    """n > 2^21 takes the wider candidate bound (18.8) and the global tile records."""
    n, rows = (1 << 21) + 4099, 3
    rng = np.random.default_rng(22)
    x = (rng.standard_normal((rows, n)) * 2).astype(np.float32)
    x[1] = (rng.standard_normal(n) * 0.3).astype(np.float32)  # flat: nucleus of ~ the whole row
    p = O.make_params(rows=rows)
    p["temperature"] = [1.0, 1.0, 0.7]
    p["top_k"] = [0, 0, 40]
    p["top_p"] = [0.9, 0.95, 0.9]
    hist = rng.integers(0, n, (rows, 64)).astype(np.uint32)
    hl = np.full(rows, 64, np.uint32)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    gpu = run_device(x, n, hist, hl, p, st)
    ref = run_oracle(x, n, hist, hl, p, st)
    compare(gpu, ref, "long rows")


def test_equal_probabilities_across_bucket_boundaries():
    """Elements whose d lies a few ulp either side of -1/32 share one probability; the
    draw must pick among them in index order (p desc, index asc), whatever side of the
    boundary each lies on."""
    n, rows = 4096, 96
    rng = np.random.default_rng(23)
    x = np.full((rows, n), -40.0, np.float32)
    base = np.float32(-0.03125)
    for r in range(rows):
        x[r, rng.integers(0, n)] = 0.0 if r % 3 else 0.5  # the max (and d = x - max)
        m = float(x[r].max())
        ids = rng.choice(n, 48, replace=False)
        for j, i in enumerate(ids):
            if x[r, i] != m:
                v = np.float32(m) + base
                steps = int(rng.integers(-24, 25))
                for _ in range(abs(steps)):
                    v = np.nextafter(v, np.float32(np.inf if steps > 0 else -np.inf), dtype=np.float32)
                x[r, i] = v
    p = O.make_params(rows=rows)
    p["temperature"] = 1.0
    p["top_k"] = 0
    p["top_p"] = np.where(np.arange(rows) % 2 == 0, 1.0, 0.5)
    p["repetition_penalty"] = 1.0
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    empty = np.zeros((rows, 0), np.uint32)
    gpu = run_device(x, n, empty, np.zeros(rows, np.uint32), p, st)
    ref = run_oracle(x, n, None, None, p, st)
    compare(gpu, ref, "bucket-boundary ties")


def test_pinned_host_rows_copied_in_pieces():
    """lrs_sample with pinned host rows (>= 512): copies overlapped with sampling, piece by piece."""
    import torch
    w = W.headline(row_ids=range(600))
    pinned = torch.from_numpy(w.logits).pin_memory().numpy()
    bs = lrs.BatchSampler(len(w.params), w.vocab, w.window)
    bs.set_params(w.params)
    bs.set_state(w.state)
    tok, probs = bs.sample(pinned, hist=w.hist, hist_len=w.hist_len, probs=True)
    st = bs.get_state(len(w.params))
    rtok, rinfo, rst = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    np.testing.assert_array_equal(tok, rtok)
    np.testing.assert_array_equal(st, rst)
    np.testing.assert_array_equal(probs.view(np.uint32), rinfo["prob"].view(np.uint32))
    bs.close()


def test_big_nucleus_rows():
    # Nuclei of 10^4 - 10^5 tokens, larger than any list: the big-nucleus stage buckets every
    # key of the row and walks the top-p sum and the draw over them.  Covered: top_k between
    # the list's capacity and the nucleus (the walk stops at k), penalties over a long window,
    # rows that start off 16-byte alignment, logits rounded to a coarse grid (runs of equal
    # probabilities: buckets of more than 512 keys are sorted by the block, a bucket longer
    # than a chunk sends the row to the persistent kernel), and a flat row with top_p near 1.
    rng = np.random.default_rng(41)
    rows, n, ld = 12, 151_936, 151_939
    buf = (rng.standard_normal((rows, ld)) * 0.5).astype(np.float32)
    buf[3] = np.round(buf[3] * 64) / 64      # about 250 distinct values: long runs of ties
    buf[4] = np.round(buf[4] * 512) / 512    # about 2,000 distinct values
    buf[5, 7] += 6.0                         # one high logit over a flat row
    buf[6] = (rng.standard_normal(ld) * 2).astype(np.float32)
    buf[6, 1234] += 12.0                     # config-4 spiked row
    p = O.make_params(1.0, 0, 0.9, 1.2, 1024, rows=rows)
    p["top_k"] = [0, 20_000, 9_000, 0, 0, 0, 0, 60_000, 0, 0, 0, 0]
    p["top_p"] = [0.9, 0.95, 0.97, 0.9, 0.9, 0.8, 0.9, 0.999, 0.5, 0.99, 0.9, 0.9]
    p["temperature"] = [1.0, 1.0, 1.3, 1.0, 0.9, 1.0, 1.0, 1.0, 1.0, 0.7, 1.5, 1.0]
    p["repetition_penalty"] = [1.2, 1.0, 1.2, 1.0, 1.2, 1.0, 1.2, 1.1, 1.3, 1.0, 0.8, 1.2]
    hist = rng.integers(0, n, (rows, 1024)).astype(np.uint32)
    hl = np.full(rows, 1024, np.uint32)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    # odd rows start 4 bytes past a 16-byte boundary (ld is odd)
    gpu = run_device(buf, n, hist, hl, p, st, ld=ld)
    ref = run_oracle(np.ascontiguousarray(buf[:, :n]), n, hist, hl, p, st)
    assert compare(gpu, ref, "big nuclei") == rows
    infos = gpu[1]
    big = (infos["cycles"][:, 4] == 1) & (infos["n_cand"] > 8192)  # (more keys than a list holds)
    assert big.sum() >= 8, f"only {int(big.sum())} rows took the big-nucleus stage"
