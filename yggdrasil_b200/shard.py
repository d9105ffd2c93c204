"""Stream sharding over the GPUs of one box: one process per GPU, a full replica of the model on each, the streams
split into contiguous shards, no collective on the step path and one gather of the per-row results at the end.

The reference has no multi-device path (one stream per core, cpu/ygg.cpp; one device for the Triton backend,
yggdrasil/inference_triton.py); streams are independent, so a shard needs nothing from the others until the final
gather of the scores (float64 per row, tiny next to NVLink bandwidth).
"""
from __future__ import annotations

import numpy as np


def shard_rows(n_rows: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous shard; the first n_rows % world ranks take one row more."""
    if world < 1 or not 0 <= rank < world or n_rows < 0:
        raise ValueError(f"shard_rows({n_rows}, {rank}, {world})")
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_rows(local, n_rows: int, group=None):
    """Concatenate every rank's shard (shards in rank order, as shard_rows splits) on every rank.

    local: this rank's rows as a torch tensor (first dim = shard length) on the process group's device. Shards are
    padded to the largest shard for all_gather_into_tensor (NCCL wants equal sizes) and the padding is dropped."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    width = -(-n_rows // world)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    out = torch.empty((world * width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    parts = []
    for r in range(world):
        a, b = shard_rows(n_rows, r, world)
        parts.append(out[r * width: r * width + (b - a)])
    return torch.cat(parts)


class ShardedScorer:
    """score() over all rows of a batch with the rows split across the ranks of a process group.

    score_shard(tokens_shard) -> float64 bits of those rows (B200Yggdrasil.score on this rank's GPU in practice).
    Every rank passes the same full token array; each scores its shard and all ranks return all rows' bits."""

    def __init__(self, score_shard, group=None, device=None):
        self.score_shard, self.group, self.device = score_shard, group, device

    def score(self, tokens):
        import torch
        import torch.distributed as dist
        tokens = np.atleast_2d(np.asarray(tokens))
        rank, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        a, b = shard_rows(len(tokens), rank, world)
        bits = np.asarray(self.score_shard(tokens[a:b]), np.float64)
        if bits.shape != (b - a,):
            raise RuntimeError(f"rank {rank}: score of {b - a} rows returned shape {bits.shape}")
        t = torch.as_tensor(bits, device=self.device)
        return gather_rows(t, len(tokens), self.group).cpu().numpy()
