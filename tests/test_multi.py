"""Multi-process host logic on CPU (gloo, world sizes 2 and 4) and the shard assembly kernel.

Row sharding: every rank samples its block of rows; the union over ranks must equal the
unsharded result.  Vocabulary sharding (config 5): every rank holds a column block; the
all-to-all plus assembly must rebuild each rank's own rows exactly, and after sampling them
and sharing the results every rank must hold the unsharded oracle's tokens and states.  A
rank that skips the exchange makes the other's exchange fail with LRS_E_TIMEOUT within its
deadline.  The CPU tests use the oracle as the sampler (no GPU); the `gpu` test drives
lrs_assemble_shards and the CUDA sampler on one device.
"""
import os
import socket

import numpy as np
import pytest

from lrs import sharded
from lrs import workloads as W


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    for p in (os.path.join(repo, "llama.rs_b200"), os.path.join(repo, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime

    import torch.distributed as dist

    import oracle as O
    from lrs import sharded as S
    from lrs import workloads as WL
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # row sharding: this rank's block of the headline rows
        w = WL.headline(row_ids=range(24))
        blk = S.row_block(w.rows, world, rank)
        sl = slice(blk.start, blk.stop)
        tok, info, st = O.sample_batch(w.logits[sl], w.vocab, w.hist[sl], w.hist_len[sl], w.params[sl],
                                       w.state[sl], threads=2)
        np.save(os.path.join(out_dir, f"rows_{rank}.npy"), np.stack([tok.astype(np.uint64), st]))
        # vocabulary sharding: columns of config 5 rows; each rank's own rows through the
        # all-to-all, sampled there, the results shared by an all-gather
        v = WL.vocab_sharded(row_ids=range(13))
        cols = S.shard_columns(v.vocab, world, rank)
        own = S.row_block(v.rows, world, rank)
        osl = slice(own.start, own.stop)
        full = S.owner_exchange_host(v.logits[:, cols], v.rows)
        np.save(os.path.join(out_dir, f"full_{rank}.npy"), full)
        tok2, _, st2 = O.sample_batch(full, v.vocab, v.hist[osl], v.hist_len[osl], v.params[osl], v.state[osl],
                                      threads=2)
        res = S.share_rows_host(np.stack([tok2.astype(np.uint64), st2], axis=1), v.rows)
        np.save(os.path.join(out_dir, f"vs_{rank}.npy"), res.T)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])  # (the vocabulary must split evenly: 151,936 = 4 x 37,984)
def test_row_and_vocab_sharding_gloo(tmp_path, oracle, world):
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    # rows: the union of the blocks is the unsharded batch
    w = W.headline(row_ids=range(24))
    tok, _, st = oracle.sample_batch(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state, threads=4)
    got = np.concatenate([np.load(tmp_path / f"rows_{r}.npy") for r in range(world)], axis=1)
    np.testing.assert_array_equal(got[0], tok.astype(np.uint64))
    np.testing.assert_array_equal(got[1], st)
    # vocabulary: every rank rebuilt its own rows, and holds the unsharded tokens and states
    v = W.vocab_sharded(row_ids=range(13))
    tok2, _, st2 = oracle.sample_batch(v.logits, v.vocab, v.hist, v.hist_len, v.params, v.state, threads=4)
    for r in range(world):
        own = sharded.row_block(v.rows, world, r)
        np.testing.assert_array_equal(np.load(tmp_path / f"full_{r}.npy").view(np.uint32),
                                      v.logits[own.start:own.stop].view(np.uint32))
        vs = np.load(tmp_path / f"vs_{r}.npy")
        np.testing.assert_array_equal(vs[0], tok2.astype(np.uint64))
        np.testing.assert_array_equal(vs[1], st2)



def _timeout_worker(rank, world, port, out_dir):
    import sys
    import time
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(here)
    if os.path.join(repo, "llama.rs_b200") not in sys.path:
        sys.path.insert(0, os.path.join(repo, "llama.rs_b200"))
    import datetime

    import torch.distributed as dist

    from lrs import sharded as S
    from lrs.sampler import SamplerError
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    if rank == 1:  # the failing rank: alive, but it never joins the exchange
        time.sleep(8.0)
        os._exit(0)
    shard = np.zeros((4, 8), np.float32)
    t = time.time()
    code = 0
    try:
        S.owner_exchange_host(shard, 4, deadline_s=1.5)
    except SamplerError as e:
        code = e.code
    with open(os.path.join(out_dir, "timeout.txt"), "w") as f:
        f.write(f"{code} {time.time() - t:.3f}")
    os._exit(0)  # (the group is unusable after a timed-out collective: no teardown)


def test_exchange_timeout_gloo_world2(tmp_path):
    import torch.multiprocessing as mp

    from lrs.sampler import LRS_E_TIMEOUT
    mp.start_processes(_timeout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    code, elapsed = open(tmp_path / "timeout.txt").read().split()
    assert int(code) == LRS_E_TIMEOUT
    assert float(elapsed) < 6.0  # (the deadline is 1.5 s; the skipping rank sleeps 8 s)

def test_row_block_partitions_rows():
    for rows in (1, 7, 1024, 4096):
        for world in (1, 2, 3, 8):
            blocks = [sharded.row_block(rows, world, r) for r in range(world)]
            assert sum(len(b) for b in blocks) == rows
            assert blocks[0].start == 0 and blocks[-1].stop == rows
            for a, b in zip(blocks, blocks[1:]):
                assert a.stop == b.start


def test_assemble_host_inverts_column_sharding():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 24)).astype(np.float32)
    for world in (1, 2, 3, 4):
        vs = 24 // world
        gathered = np.concatenate([x[:, g * vs:(g + 1) * vs].reshape(-1) for g in range(world)])
        np.testing.assert_array_equal(sharded.assemble_host(gathered, world, 5, vs), x)


@pytest.mark.gpu
def test_assemble_kernel_and_sampling_of_vocab_sharded_rows():
    """lrs_assemble_shards on a rank-major buffer of 4 shards, then the CUDA sampler."""
    import ctypes

    import torch

    import lrs
    from gpu_util import compare, run_oracle
    v = W.vocab_sharded(row_ids=range(16))
    world, vs = 4, v.vocab // 4
    dev = torch.device("cuda:0")
    gathered = torch.from_numpy(np.concatenate([v.logits[:, g * vs:(g + 1) * vs].reshape(-1)
                                                for g in range(world)])).to(dev)
    full = torch.empty(v.rows, v.vocab, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    code = lrs.lib().lrs_assemble_shards(ctypes.c_void_p(gathered.data_ptr()), world, v.rows, vs,
                                         ctypes.c_void_p(full.data_ptr()), v.vocab, ctypes.c_void_p(stream))
    assert code == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(full.cpu().numpy().view(np.uint32), v.logits.view(np.uint32))
    # the assembled rows through the sampler equal the unsharded oracle
    from gpu_util import run_device
    gpu = run_device(full.cpu().numpy(), v.vocab, v.hist, v.hist_len, v.params, v.state)
    ref = run_oracle(v.logits, v.vocab, v.hist, v.hist_len, v.params, v.state)
    compare(gpu, ref, "vocab_sharded assembled")
