"""Multi-GPU sampling: row replicas and vocabulary sharding.

Row sharding (configs 2-4 and the headline).  Rows are independent (one Sampler per
generation in the reference, sampler.rs:28-37), so rank r samples its own contiguous
block of rows, `row_block(rows, world, r)`, with its own BatchSampler: no collective.

Vocabulary sharding (config 5).  A tensor-parallel LM head leaves rank g holding columns
[g * Vs, (g + 1) * Vs) of every row.  The reference's softmax denominator is a sequential
f32 sum over the whole row in index order (ops.rs:408-411), which no combination of
per-shard partial sums reproduces bit for bit, so a row is sampled whole, on one rank: row
r belongs to the rank whose `row_block` holds it.  The exchange is one all-to-all (NCCL
over NVLink / NVSwitch on GPUs, gloo on CPUs) that sends each rank's columns of a row to
the row's owner only, so a rank receives (G - 1) / G of its own rows instead of every
rank's columns of every row; lrs_assemble_shards lays the owner's rows out and
lrs_sample_device samples them; one all-gather then gives every rank every row's token,
state and status.  Deadlines: on host buffers (gloo) each collective is waited for with a
deadline, and one that does not complete in time raises SamplerError with LRS_E_TIMEOUT (a
peer lost another way: LRS_E_NCCL); on GPUs the collectives stay stream-ordered (a host wait
would stall the launches behind them) and the process group's timeout, enforced by NCCL's
watchdog, bounds them.
"""
from __future__ import annotations

import ctypes

import numpy as np


def row_block(rows: int, world: int, rank: int) -> range:
    """Rows [start, stop) of `rank` when `rows` are split over `world` ranks in blocks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    return range(rows * rank // world, rows * (rank + 1) // world)


def shard_columns(vocab: int, world: int, rank: int) -> slice:
    """Columns of `rank` under vocabulary sharding (vocab must split evenly)."""
    if vocab % world:
        raise ValueError(f"vocab {vocab} does not split over {world} ranks")
    vs = vocab // world
    return slice(rank * vs, (rank + 1) * vs)


def assemble_host(gathered: np.ndarray, shards: int, rows: int, shard_n: int) -> np.ndarray:
    """Host form of lrs_assemble_shards: rank-major [g][row][col] -> rows [row][g*shard_n + col]."""
    return np.ascontiguousarray(gathered.reshape(shards, rows, shard_n).transpose(1, 0, 2).reshape(rows, -1))


def _wait(work, deadline_s: float, what: str) -> None:
    """Waits for an asynchronous collective; SamplerError(LRS_E_TIMEOUT) past the deadline."""
    import datetime

    from .sampler import LRS_E_NCCL, LRS_E_TIMEOUT, SamplerError
    try:
        done = work.wait(timeout=datetime.timedelta(seconds=deadline_s))
    except RuntimeError as e:
        import re
        timed_out = re.search(r"tim(ed|ing) ?out|timeout", str(e).lower()) is not None
        raise SamplerError(LRS_E_TIMEOUT if timed_out else LRS_E_NCCL, f"{what}: {str(e)[:200]}") from None
    if done is False:
        raise SamplerError(LRS_E_TIMEOUT, f"{what}: not complete after {deadline_s} s")


def owner_exchange_host(shard: np.ndarray, rows: int, group=None, deadline_s: float = 30.0) -> np.ndarray:
    """Config 5's exchange on host shards (gloo): rank g's shard (rows x Vs) in, the full rows of
    g's `row_block` out (len(block) x world * Vs), through one all-to-all."""
    import torch
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    vs = shard.shape[1]
    blocks = [row_block(rows, world, h) for h in range(world)]
    mine = len(blocks[rank])
    src = torch.from_numpy(np.ascontiguousarray(shard, np.float32)).reshape(-1)
    out = torch.empty(world * mine * vs, dtype=torch.float32)
    work = dist.all_to_all_single(out, src, output_split_sizes=[mine * vs] * world,
                                  input_split_sizes=[len(b) * vs for b in blocks], group=group, async_op=True)
    _wait(work, deadline_s, "config-5 exchange")
    return assemble_host(out.numpy(), world, mine, vs)


def share_rows_host(values: np.ndarray, rows: int, group=None, deadline_s: float = 30.0) -> np.ndarray:
    """Every rank's per-row results (its row_block) to every rank: one all-gather (gloo)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    blocks = [row_block(rows, world, h) for h in range(world)]
    width = max(len(b) for b in blocks)
    pad = np.zeros((width,) + values.shape[1:], values.dtype)
    pad[:len(values)] = values
    raw = torch.from_numpy(pad.reshape(width, -1).view(np.uint8))  # (as bytes: any element type)
    parts = [torch.empty_like(raw) for _ in range(world)]
    work = dist.all_gather(parts, raw, group=group, async_op=True)
    _wait(work, deadline_s, "config-5 results")
    shape = (-1,) + values.shape[1:]
    return np.concatenate([parts[h].numpy().view(values.dtype).reshape(shape)[:len(blocks[h])] for h in range(world)])


def gather_shards_host(shard: np.ndarray, group=None) -> np.ndarray:
    """All-gather of host shards (gloo): the rank-major buffer lrs_assemble_shards expects."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    t = torch.from_numpy(np.ascontiguousarray(shard))
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t, group=group)
    return torch.stack(parts).numpy().reshape(-1)


class VocabShardedSampler:
    """Config 5 on GPUs: sample rows whose columns are spread over the ranks of `group`; row r is
    sampled by the rank whose `row_block` holds it."""

    def __init__(self, rows: int, vocab: int, max_hist: int = 64, group=None, device: int = 0):
        import torch
        import torch.distributed as dist

        from .sampler import BatchSampler
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rows, self.vocab = rows, vocab
        self.shard_n = vocab // self.world
        if self.shard_n * self.world != vocab:
            raise ValueError(f"vocab {vocab} does not split over {self.world} ranks")
        self.blocks = [row_block(rows, self.world, h) for h in range(self.world)]
        self.mine = self.blocks[self.rank]
        self.width = max(len(b) for b in self.blocks)  # (rows of the largest block: the result slots)
        dev = torch.device("cuda", device)
        self.bs = BatchSampler(max(len(self.mine), 1), vocab, max_hist, device=device)
        self.recv = torch.empty(self.world * len(self.mine) * self.shard_n, dtype=torch.float32, device=dev)
        self.full = torch.empty(len(self.mine), vocab, dtype=torch.float32, device=dev)
        # per row of every rank's block: the state, then (token, status), then (probability, -) as
        # 64-bit words, so the results take one all-gather
        self.res = torch.zeros(self.world, 3, self.width, dtype=torch.int64, device=dev)
        self.res_st = self.res[:, 0]
        self.res_tok = self.res[:, 1].view(torch.int32).view(self.world, self.width, 2)[:, :, 0]
        self.res_sts = self.res[:, 1].view(torch.int32).view(self.world, self.width, 2)[:, :, 1]
        self.res_prb = self.res[:, 2].view(torch.float32).view(self.world, self.width, 2)[:, :, 0]

    def exchange_bytes(self) -> int:
        """Bytes this rank receives from its peers per step (the shards; the results are 16 B a row)."""
        return (self.world - 1) * len(self.mine) * self.shard_n * 4

    def exchange(self, shard, stream=None) -> None:
        """The exchange step: this rank's rows from every rank's columns, laid out whole."""
        import torch
        import torch.distributed as dist

        from .sampler import _check, lib
        flat = shard.contiguous().view(-1)
        mine = len(self.mine)
        if self.world > 1:
            work = dist.all_to_all_single(self.recv, flat, output_split_sizes=[mine * self.shard_n] * self.world,
                                          input_split_sizes=[len(b) * self.shard_n for b in self.blocks],
                                          group=self.group, async_op=True)
            work.wait()  # (stream-ordered: the process group's timeout bounds it)
        else:
            self.recv.copy_(flat)
        if stream is None:
            stream = torch.cuda.current_stream(self.full.device).cuda_stream
        if mine:
            code = lib().lrs_assemble_shards(ctypes.c_void_p(self.recv.data_ptr()), self.world, mine,
                                             self.shard_n, ctypes.c_void_p(self.full.data_ptr()), self.vocab,
                                             ctypes.c_void_p(stream))
            _check(code, None)

    def sample_owned(self, params, state, tokens, hist=None, hist_len=None, probs=None, status=None,
                     stream=None) -> None:
        """After exchange(): sample this rank's rows and share every row's results with every rank.
        params, state, tokens, ... cover all rows, as for lrs_sample_device."""
        import torch
        import torch.distributed as dist
        r0, r1 = self.mine.start, self.mine.stop
        rp = params.view(self.rows, -1)[r0:r1]
        if r1 > r0:
            m = r1 - r0
            st = self.res_st[self.rank, :m]
            st.copy_(state[r0:r1])
            tok = torch.empty(m, dtype=torch.int32, device=self.full.device)
            sts = torch.empty(m, dtype=torch.int32, device=self.full.device)
            prb = torch.empty(m, dtype=torch.float32, device=self.full.device)
            self.bs.sample_device(self.full, rp.reshape(-1), st, tok, n=self.vocab,
                                  hist=None if hist is None else hist[r0:r1],
                                  hist_len=None if hist_len is None else hist_len[r0:r1],
                                  probs=prb, status=sts, stream=stream)
            self.res_tok[self.rank, :m] = tok
            self.res_sts[self.rank, :m] = sts
            self.res_prb[self.rank, :m] = prb
        if self.world > 1:
            work = dist.all_gather_into_tensor(self.res.view(-1), self.res[self.rank].contiguous().view(-1),
                                               group=self.group, async_op=True)
            work.wait()
        for h, b in enumerate(self.blocks):
            n = len(b)
            if n == 0:
                continue
            tokens[b.start:b.stop] = self.res_tok[h, :n]
            state[b.start:b.stop] = self.res_st[h, :n]
            if status is not None:
                status[b.start:b.stop] = self.res_sts[h, :n]
            if probs is not None:
                probs[b.start:b.stop] = self.res_prb[h, :n]

    def sample(self, shard, params, state, tokens, hist=None, hist_len=None, probs=None, status=None,
               stream=None) -> None:
        """shard: (rows, vocab / world) float32 CUDA tensor of this rank's columns."""
        self.exchange(shard, stream)
        self.sample_owned(params, state, tokens, hist=hist, hist_len=hist_len, probs=probs, status=status,
                          stream=stream)

    def close(self) -> None:
        self.bs.close()
