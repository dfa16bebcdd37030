"""Tensor-parallel combination of the attention share: one all-reduce over the ranks' devices.

Tensor parallelism splits the KV heads over the ranks; each rank records the share of its own heads.
The reference averages the ranks' shares on the host after copying each rank's table out over IPC
(RankedShareSource.read, observe/ranks.py:105-119: ``np.mean(shares, axis=0)``). Here every rank's
audit kernel leaves its normalised share [rows, width] on its own GPU, and ``allreduce_shares``
sums them with one NCCL all-reduce over NVLink and divides by the world size: the same mean, NaN
wherever any rank had no evidence. ``head_shard`` gives a rank its KV heads.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
import torch.distributed as dist


def head_shard(kv_heads: int, rank: int, world_size: int) -> range:
    """The KV heads of ``rank`` when ``kv_heads`` split evenly over ``world_size`` ranks."""
    if world_size <= 0 or kv_heads % world_size:
        raise ValueError(f"{kv_heads} KV heads do not split evenly over {world_size} ranks")
    per = kv_heads // world_size
    return range(rank * per, (rank + 1) * per)


def allreduce_shares(share: torch.Tensor, group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """In place: the mean over ranks of each rank's ``share`` (SUM all-reduce, then / world size)."""
    world = dist.get_world_size(group)
    if world > 1:
        dist.all_reduce(share, op=dist.ReduceOp.SUM, group=group)
        share.div_(world)
    return share


class RankedShareSource:
    """The attention share of a block averaged over the ranks' sources (reference ranks.py:105-119).

    For sources read in one process (each returning a [live_rows, width] array), the mean is taken
    over the ranks. Ranks in separate processes use ``allreduce_shares`` instead."""

    def __init__(self, sources: Sequence[object]) -> None:
        if not sources:
            raise ValueError("a ranked share source needs at least one rank")
        self.sources = list(sources)

    def read(self, live_rows: int, row_blocks: np.ndarray):
        shares = [source.read(live_rows, row_blocks) for source in self.sources]
        if isinstance(shares[0], torch.Tensor):
            return torch.stack(shares).mean(dim=0)
        return np.mean(shares, axis=0)
