"""GPU test of lrs_sample_device_noalloc, the entry point for callers that cannot let the
library allocate device memory.  It must return exactly what lrs_sample_device returns
(tokens, probabilities, statuses and advanced PRNG states) on the same inputs, on two
calls in a row.  Kept in a file of its own that pytest collects last."""
import ctypes

import numpy as np
import pytest

import lrs
from lrs import workloads as W

pytestmark = pytest.mark.gpu


def _buffers(w, torch, dev):
    return dict(
        x=torch.from_numpy(w.logits).to(dev),
        h=torch.from_numpy(w.hist.view(np.int32)).to(dev),
        hl=torch.from_numpy(w.hist_len.view(np.int32)).to(dev),
        p=torch.from_numpy(w.params.view(np.uint8)).to(dev),
        s=torch.from_numpy(w.state.view(np.int64)).to(dev),
        t=torch.zeros(len(w.params), dtype=torch.int32, device=dev),
        pr=torch.zeros(len(w.params), dtype=torch.float32, device=dev),
        st=torch.zeros(len(w.params), dtype=torch.int32, device=dev),
    )


def test_no_alloc_entry_point_matches_context_entry_point():
    import torch
    dev = torch.device("cuda:0")
    # headline rows: top-k rows and top_k-off rows (the latter use the candidate scratch)
    w = W.headline(row_ids=range(0, 1024, 32))
    L = lrs.lib()
    bs = lrs.BatchSampler(len(w.params), w.vocab, w.window)
    a = _buffers(w, torch, dev)
    b = _buffers(w, torch, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rows, n = len(w.params), w.vocab
    for call in range(2):
        bs.sample_device(a["x"], a["p"], a["s"], a["t"], n=n, hist=a["h"], hist_len=a["hl"], probs=a["pr"],
                         status=a["st"], stream=stream)
        rc = L.lrs_sample_device_noalloc(0, b["x"].data_ptr(), rows, n, b["x"].stride(0), b["h"].data_ptr(),
                                         b["h"].stride(0), b["hl"].data_ptr(), b["p"].data_ptr(), b["s"].data_ptr(),
                                         b["t"].data_ptr(), b["pr"].data_ptr(), b["st"].data_ptr(), stream)
        assert rc == lrs.LRS_OK
        torch.cuda.synchronize()
        for key in ("t", "st", "s"):
            assert torch.equal(a[key], b[key]), (call, key)
        assert torch.equal(a["pr"].view(torch.int32), b["pr"].view(torch.int32)), call
    bs.close()


def test_no_alloc_after_a_wider_call_penalises_only_the_window():
    """A call at one vocabulary size, then penalised calls at smaller sizes: the shared
    scratch is laid out per size, so the later calls must not see the earlier call's data
    as window bits (they must equal lrs_sample_device bit for bit)."""
    import torch
    dev = torch.device("cuda:0")
    L = lrs.lib()
    stream = torch.cuda.current_stream(dev).cuda_stream
    for rows, n, call in ((40, 151_936, "wide, top_k off"), (40, 100_003, "narrower, penalised"),
                          (40, 60_000, "narrower again")):
        w = W.headline(row_ids=range(rows))
        w.logits = np.ascontiguousarray(w.logits[:, :n])
        w.vocab = n
        w.hist = (w.hist % n).astype(np.uint32)
        if call == "wide, top_k off":
            w.params["top_k"] = 0  # the path that fills the candidate-key scratch
        else:
            w.params["repetition_penalty"] = 1.25
        bs = lrs.BatchSampler(rows, n, w.window)
        a = _buffers(w, torch, dev)
        b = _buffers(w, torch, dev)
        bs.sample_device(a["x"], a["p"], a["s"], a["t"], n=n, hist=a["h"], hist_len=a["hl"], probs=a["pr"],
                         status=a["st"], stream=stream)
        rc = L.lrs_sample_device_noalloc(0, b["x"].data_ptr(), rows, n, b["x"].stride(0), b["h"].data_ptr(),
                                         b["h"].stride(0), b["hl"].data_ptr(), b["p"].data_ptr(), b["s"].data_ptr(),
                                         b["t"].data_ptr(), b["pr"].data_ptr(), b["st"].data_ptr(), stream)
        assert rc == lrs.LRS_OK
        assert L.lrs_noalloc_poll_error(0, stream) == lrs.LRS_OK
        torch.cuda.synchronize()
        for key in ("t", "st", "s"):
            assert torch.equal(a[key], b[key]), (call, key)
        assert torch.equal(a["pr"].view(torch.int32), b["pr"].view(torch.int32)), call
        bs.close()


def test_no_alloc_rejects_sizes_beyond_its_limit():
    L = lrs.lib()
    rc = L.lrs_sample_device_noalloc(0, 16, 1, 262144 + 1, 262145, None, 0, None, 16, 16, 16, None, None, None)
    assert rc == lrs.LRS_E_INVALID
    rc = L.lrs_sample_device_noalloc(0, 16, 1, 0, 0, None, 0, None, 16, 16, 16, None, None, None)
    assert rc == lrs.LRS_E_INVALID
