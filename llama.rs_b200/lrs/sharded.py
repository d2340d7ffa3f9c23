"""Multi-GPU sampling: row replicas and vocabulary sharding.

Row sharding (configs 2-4 and the headline).  Rows are independent (one Sampler per
generation in the reference, sampler.rs:28-37), so rank r samples its own contiguous
block of rows, `row_block(rows, world, r)`, with its own BatchSampler: no collective.

Vocabulary sharding (config 5).  A tensor-parallel LM head leaves rank g holding columns
[g * Vs, (g + 1) * Vs) of every row.  The reference's softmax denominator is a sequential
f32 sum over the whole row in index order (ops.rs:408-411), which no combination of
per-shard partial sums reproduces bit for bit, so the exchange step moves the rows: one
all-gather of the shards (NCCL over NVLink / NVSwitch on GPUs, gloo on CPUs),
lrs_assemble_shards to lay the rows out, then lrs_sample_device.  Every rank samples every
row with the same PRNG states, so all ranks hold the same tokens without a second
collective.
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
    """Config 5 on GPUs: sample rows whose columns are spread over the ranks of `group`."""

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
        dev = torch.device("cuda", device)
        self.bs = BatchSampler(rows, vocab, max_hist, device=device)
        self.gathered = torch.empty(self.world * rows * self.shard_n, dtype=torch.float32, device=dev)
        self.full = torch.empty(rows, vocab, dtype=torch.float32, device=dev)

    def exchange(self, shard, stream=None) -> None:
        """The exchange step: all-gather the shards and lay out the full rows."""
        import torch
        import torch.distributed as dist

        from .sampler import _check, lib
        flat = shard.contiguous().view(-1)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, flat, group=self.group)
        else:
            self.gathered.copy_(flat)
        if stream is None:
            stream = torch.cuda.current_stream(self.full.device).cuda_stream
        code = lib().lrs_assemble_shards(ctypes.c_void_p(self.gathered.data_ptr()), self.world, self.rows,
                                         self.shard_n, ctypes.c_void_p(self.full.data_ptr()), self.vocab,
                                         ctypes.c_void_p(stream))
        _check(code, None)

    def sample(self, shard, params, state, tokens, hist=None, hist_len=None, probs=None, status=None,
               stream=None) -> None:
        """shard: (rows, vocab / world) float32 CUDA tensor of this rank's columns."""
        self.exchange(shard, stream)
        self.bs.sample_device(self.full, params, state, tokens, n=self.vocab, hist=hist, hist_len=hist_len,
                              probs=probs, status=status, stream=stream)

    def close(self) -> None:
        self.bs.close()
