"""Helpers shared by the GPU tests: run a workload through the C ABI and compare it
with the CPU oracle field by field."""
from __future__ import annotations

import numpy as np

import lrs
import oracle as O

_samplers = {}


def batch_sampler(rows, vocab, hist):
    key = (rows, vocab, hist)
    bs = _samplers.get(key)
    if bs is None:
        for k in list(_samplers):
            _samplers.pop(k).close()
        bs = lrs.BatchSampler(rows, vocab, hist)
        _samplers[key] = bs
    return bs


def run_device(logits, n, hist, hist_len, params, state, ld=None):
    """lrs_sample_device on torch CUDA tensors; returns (tokens, infos, state, probs, status)."""
    import torch
    rows = logits.shape[0] if ld != 0 else len(params)
    dev = torch.device("cuda:0")
    x = torch.from_numpy(np.ascontiguousarray(logits)).to(dev)
    if ld is None:
        ld = x.stride(0)
    W = hist.shape[1] if hist is not None and hist.ndim == 2 else 0
    bs = batch_sampler(max(rows, 1), max(n, 1), max(W, 1))
    th = torch.from_numpy(np.ascontiguousarray(hist)).to(dev) if W else None
    thl = torch.from_numpy(np.ascontiguousarray(hist_len, np.uint32).view(np.int32)).to(dev) if W else None
    tp = torch.from_numpy(np.ascontiguousarray(params).view(np.uint8)).to(dev)
    ts = torch.from_numpy(np.ascontiguousarray(state, np.uint64).view(np.int64)).to(dev)
    tok = torch.zeros(rows, dtype=torch.int32, device=dev)
    prb = torch.zeros(rows, dtype=torch.float32, device=dev)
    sts = torch.zeros(rows, dtype=torch.int32, device=dev)
    inf = torch.zeros(rows * lrs.ROW_INFO_DTYPE.itemsize, dtype=torch.uint8, device=dev)
    bs.sample_device(x, tp, ts, tok, n=n, hist=th, hist_len=thl, probs=prb, status=sts, info=inf, ld=ld)
    torch.cuda.synchronize()
    infos = inf.cpu().numpy().view(lrs.ROW_INFO_DTYPE)
    return (tok.cpu().numpy().view(np.uint32), infos, ts.cpu().numpy().view(np.uint64),
            prb.cpu().numpy(), sts.cpu().numpy())


def run_oracle(logits, n, hist, hist_len, params, state, threads=8):
    return O.sample_batch(logits, n, hist if hist is not None and hist.size else None,
                          hist_len if hist is not None and hist.size else None, params, state, threads=threads)


def compare(gpu, ref, label="", check_info=True):
    """Bit-exact comparison of every output; returns the number of rows checked."""
    tok, infos, st, probs, status = gpu
    rtok, rinfo, rst = ref
    bad = np.nonzero((tok != rtok) | (status != rinfo["status"]) | (st != rst))[0]
    if bad.size:
        r = int(bad[0])
        raise AssertionError(f"{label}: {bad.size} rows differ; first row {r}: gpu token {tok[r]} status {status[r]} "
                             f"state {st[r]} info {infos[r]} | oracle token {rtok[r]} state {rst[r]} info {rinfo[r]}")
    if check_info:
        ok = rinfo["status"] == 0
        stoch = ok & (rinfo["path"] == 2)
        for f in ("sum_exp", "surv_sum", "r0", "max"):
            g = infos[f][stoch].view(np.uint32)
            o = rinfo[f][stoch].view(np.uint32)
            if not np.array_equal(g, o):
                r = int(np.nonzero(stoch)[0][np.nonzero(g != o)[0][0]])
                raise AssertionError(f"{label}: field {f} differs at row {r}: gpu {infos[r]} oracle {rinfo[r]}")
        for f in ("cutoff", "pos", "k"):
            if not np.array_equal(infos[f][stoch], rinfo[f][stoch]):
                r = int(np.nonzero(stoch)[0][np.nonzero(infos[f][stoch] != rinfo[f][stoch])[0][0]])
                raise AssertionError(f"{label}: field {f} differs at row {r}: gpu {infos[r]} oracle {rinfo[r]}")
        gp = probs[ok].view(np.uint32)
        op = rinfo["prob"][ok].view(np.uint32)
        if not np.array_equal(gp, op):
            r = int(np.nonzero(ok)[0][np.nonzero(gp != op)[0][0]])
            raise AssertionError(f"{label}: probability differs at row {r}: gpu {probs[r]} oracle {rinfo[r]}")
    return len(tok)
