"""GPU: the state of a batched generation loop kept on the device.

A loop of the reference (model.rs:741-776, server.rs:166-191) samples a token, stops on the
end-of-sequence id, and otherwise pushes the token onto `recent`, which the next draw's
repetition penalty reads.  Here `recent` is a device history row extended by
lrs_history_append after each batched draw; every step's tokens and PRNG states are compared
with the oracle driven by host-side `recent` lists.  lrs_remap_tokens maps tokens sampled on
pruned rows back to the full vocabulary (prune.rs:187-195).
"""
import numpy as np
import pytest

import lrs
import oracle as O
from gpu_util import run_oracle

pytestmark = pytest.mark.gpu


def test_generation_loop_with_device_history():
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(77)
    rows, n, steps, hld, keep, eos = 16, 32_000, 60, 128, 48, 7
    # prompts of 20-100 ids: with up to 60 tokens appended, rows pass hld and are compacted
    prompts = [rng.integers(0, n, int(rng.integers(20, 101))).astype(np.uint32) for _ in range(rows)]
    p = O.make_params(0.9, 40, 0.95, 1.2, 32, rows=rows)
    p["temperature"] = rng.uniform(0.6, 1.4, rows)
    p["top_k"] = [0, 20, 40, 100] * 4
    p["top_p"] = rng.uniform(0.85, 1.0, rows)
    p["repetition_penalty"] = rng.uniform(1.05, 1.5, rows)
    p["repeat_last_n"] = [8, 16, 32, 48] * 4  # (at most keep: the window survives compaction)
    p["temperature"][3] = 0.0                 # a greedy row with a penalty
    state = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)

    bs = lrs.BatchSampler(rows, n, hld)
    hist = torch.zeros((rows, hld), dtype=torch.int32, device=dev)
    hlen = torch.zeros(rows, dtype=torch.int32, device=dev)
    for r, pr in enumerate(prompts):
        k = min(len(pr), hld)
        hist[r, :k] = torch.from_numpy(pr[-k:].view(np.int32))
        hlen[r] = k
    tp = torch.from_numpy(p.view(np.uint8)).to(dev)
    ts = torch.from_numpy(state.view(np.int64)).to(dev)
    tok = torch.zeros(rows, dtype=torch.int32, device=dev)
    sts = torch.zeros(rows, dtype=torch.int32, device=dev)

    recent = [list(pr) for pr in prompts]
    ref_state = state.copy()
    done = np.zeros(rows, bool)
    compacted = 0
    for step in range(steps):
        x = (rng.standard_normal((rows, n)) * 2.5).astype(np.float32)
        if step % 9 == 4:
            x[step % rows, eos] += 40.0  # one row meets its end of sequence
        bs.sample_device(torch.from_numpy(x).to(dev), tp, ts, tok, n=n, hist=hist, hist_len=hlen, status=sts)
        bs.history_append(tok, hist, hlen, status=sts, eos=eos, keep=keep)
        # the oracle on the host recent lists (full histories: its window is repeat_last_n)
        w = max(len(rc) for rc in recent)
        hh = np.zeros((rows, w), np.uint32)
        hl = np.zeros(rows, np.uint32)
        for r, rc in enumerate(recent):
            hh[r, :len(rc)] = rc
            hl[r] = len(rc)
        rtok, rinfo, rst = run_oracle(x, n, hh, hl, p, ref_state)
        gtok = tok.cpu().numpy().view(np.uint32)
        gst = ts.cpu().numpy().view(np.uint64)
        live = ~done
        assert (sts.cpu().numpy()[live] == 0).all()
        bad = np.nonzero(live & ((gtok != rtok) | (gst != rst)))[0]
        assert bad.size == 0, f"step {step}: rows {bad.tolist()} differ: gpu {gtok[bad]} oracle {rtok[bad]}"
        ref_state = rst.copy()
        for r in np.nonzero(live)[0]:
            if rtok[r] == eos:
                done[r] = True  # (the reference's loop stops here: the row is compared no more)
            else:
                if len(recent[r]) >= hld:
                    compacted += 1
                recent[r].append(int(rtok[r]))
    assert done.any() and compacted > 0
    # the device rows hold the tail of each live row's recent list
    gh = hist.cpu().numpy().view(np.uint32)
    gl = hlen.cpu().numpy()
    for r in np.nonzero(~done)[0]:
        assert gl[r] <= hld
        assert gh[r, :gl[r]].tolist() == recent[r][-int(gl[r]):]
    bs.close()


def test_pruned_vocab_remap():
    import torch
    dev = torch.device("cuda:0")
    rng = np.random.default_rng(78)
    rows, full, n = 64, 151_936, 10_000
    kept = np.sort(rng.choice(full, n, replace=False)).astype(np.uint32)  # pruned id t is full id kept[t]
    x = (rng.standard_normal((rows, n)) * 3).astype(np.float32)
    p = O.make_params(0.8, 40, 0.95, 1.0, 64, rows=rows)
    st = rng.integers(1, 2**62, rows).astype(np.uint64) | np.uint64(1)
    bs = lrs.BatchSampler(rows, n, 1)
    tok = torch.zeros(rows, dtype=torch.int32, device=dev)
    sts = torch.zeros(rows, dtype=torch.int32, device=dev)
    ts = torch.from_numpy(st.view(np.int64)).to(dev)
    bs.sample_device(torch.from_numpy(x).to(dev), torch.from_numpy(p.view(np.uint8)).to(dev), ts, tok, n=n,
                     status=sts)
    out = torch.zeros_like(tok)
    bs.remap_tokens(tok, torch.from_numpy(kept.view(np.int32)).to(dev), out, status=sts)
    rtok, _, _ = run_oracle(x, n, None, None, p, st)
    assert (out.cpu().numpy().view(np.uint32) == kept[rtok]).all()
    assert (tok.cpu().numpy().view(np.uint32) == rtok).all()
    bs.close()
