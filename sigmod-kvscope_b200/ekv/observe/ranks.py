"""Tensor-parallel combination of the attention share: one all-reduce over the ranks' devices.

Tensor parallelism splits the KV heads over the ranks; each rank records the share of its own heads.
The reference averages the ranks' shares on the host after copying each rank's table out over IPC
(RankedShareSource.read, observe/ranks.py:105-119: ``np.mean(shares, axis=0)``). Here every rank's
audit kernel leaves its normalised share [rows, width] on its own GPU, and ``allreduce_shares``
averages them with one NCCL all-reduce over NVLink: the same mean, NaN wherever any rank had no
evidence. ``StepCombiner`` runs that all-reduce inside the step's CUDA graph, concurrently with the
next step's audit, on two alternating share buffers. ``head_shard`` gives a rank its KV heads.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

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
    """In place: the mean over ranks of each rank's ``share``.

    NCCL averages in the collective itself (one launch); backends without an averaging reduction
    (gloo) sum and then divide by the world size."""
    if not dist.is_initialized():
        return share  # one process: its shares are the mean
    world = dist.get_world_size(group)
    if world > 1:
        if dist.get_backend(group) == "nccl":
            dist.all_reduce(share, op=dist.ReduceOp.AVG, group=group)
        else:
            dist.all_reduce(share, op=dist.ReduceOp.SUM, group=group)
            share.div_(world)
    return share


class StepCombiner:
    """Audit steps whose shares are averaged over the ranks while the next step records.

    ``record()`` launches one audit step on the current stream with its shares written to the plane's
    current share buffer (``RecordingPlane.direct_shares``). Two CUDA graphs are captured, one per
    share buffer; graph ``p`` records a step into buffer ``p`` on the capture stream and, on a second
    stream joined before the graph ends, all-reduces buffer ``1 - p``: the previous step's shares. A
    step's combine therefore runs concurrently with the next step's record kernel, and it is complete
    when the next step's graph is. ``flush()`` combines the last step's shares (one all-reduce, eager).

    Every rank must call ``step`` and ``flush`` the same number of times, in the same order. The
    graphs hold NCCL work: ``release()`` them before the process group is destroyed. In a single process
    (no process group) there is nothing to combine, and the two graphs just alternate the share buffers,
    so one step's shares can be read out while the next step writes the other buffer.
    """

    def __init__(self, plane, record: Callable[[], None], group: dist.ProcessGroup | None = None) -> None:
        self.plane, self.group = plane, group
        first = plane.shares()
        self.buffers = [first, torch.full_like(first, float("nan"))]
        self.stream = torch.cuda.Stream()
        self.graphs: list[torch.cuda.CUDAGraph] = []
        self.steps = 0
        main = torch.cuda.current_stream()
        for p in (0, 1):
            plane.direct_shares(self.buffers[p])
            # one eager run outside the capture sets the kernels' one-time attributes and the
            # communicator's state for this buffer
            side = torch.cuda.Stream()
            side.wait_stream(main)
            with torch.cuda.stream(side):
                self._body(record, p)
            main.wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._body(record, p)
            self.graphs.append(graph)
        torch.cuda.synchronize()
        plane.direct_shares(self.buffers[0])

    def _body(self, record: Callable[[], None], p: int) -> None:
        here = torch.cuda.current_stream()
        self.stream.wait_stream(here)
        with torch.cuda.stream(self.stream):
            allreduce_shares(self.buffers[1 - p], self.group)
        record()
        here.wait_stream(self.stream)

    def step(self) -> None:
        """Replay one step: record into the next buffer, combine the previous step's."""
        self.graphs[self.steps % 2].replay()
        self.steps += 1

    def last(self) -> torch.Tensor:
        """The buffer of the last step replayed (combined once ``flush`` has run after it)."""
        return self.buffers[(self.steps - 1) % 2]

    def flush(self) -> torch.Tensor:
        """Combine the last step's shares (an eager all-reduce on the current stream) and return them."""
        return allreduce_shares(self.last(), self.group)

    def release(self) -> None:
        self.graphs.clear()


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
