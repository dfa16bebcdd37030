"""Tensor-parallel combination on CPU: two gloo ranks, each holding its own heads' shares.

The reference averages the ranks' shares on the host (RankedShareSource.read, observe/ranks.py:117-119);
ekv.observe.ranks.allreduce_shares does it with one all-reduce (NCCL on the GPUs, gloo here) and a
division by the world size. The result must equal the oracle's mean over ranks bit for bit, NaN
where any rank had no evidence; a rank that never joins makes the other's rendezvous fail on its
timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import shares as osh


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_shares(rank: int, rows: int = 5, width: int = 12) -> np.ndarray:
    """Each rank's normalised shares: a share vector per row, NaN rows where it has no evidence."""
    rng = np.random.default_rng(100 + rank)
    x = rng.dirichlet(np.full(width, 0.5), rows).astype(np.float32)
    x[rows - 1 - rank] = np.nan  # rank 0 lacks the last row, rank 1 the one before
    return x


def _worker(rank: int, world: int, port: int, out: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from ekv.observe.ranks import allreduce_shares, head_shard

    share = torch.from_numpy(rank_shares(rank))
    allreduce_shares(share)
    heads = list(head_shard(8, rank, world))
    np.savez(f"{out}.{rank}.npz", share=share.numpy(), heads=np.array(heads))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_combine_to_the_mean_over_ranks(tmp_path):
    port = free_port()
    out = str(tmp_path / "tp")
    mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    want = osh.mean_over_ranks([rank_shares(0), rank_shares(1)])
    got0 = np.load(f"{out}.0.npz")
    got1 = np.load(f"{out}.1.npz")
    for got in (got0, got1):
        assert np.array_equal(np.isnan(got["share"]), np.isnan(want))
        np.testing.assert_allclose(got["share"], want, rtol=1e-6, equal_nan=True)
    assert np.isnan(want[3]).all() and np.isnan(want[4]).all()
    assert got0["heads"].tolist() == [0, 1, 2, 3] and got1["heads"].tolist() == [4, 5, 6, 7]


def _lonely(port: int, out: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=timedelta(seconds=3))
        open(out, "w").write("joined")
    except Exception as exc:  # the rendezvous gives up on its timeout
        open(out, "w").write(type(exc).__name__)


def test_a_rank_that_never_joins_ends_the_rendezvous_with_an_error(tmp_path):
    port = free_port()
    out = str(tmp_path / "lonely.txt")
    ctx = mp.get_context("spawn")
    proc = ctx.Process(target=_lonely, args=(port, out))
    proc.start()
    proc.join(timeout=60)
    if proc.is_alive():
        proc.kill()
        pytest.fail("the rendezvous did not give up on its timeout")
    assert open(out).read() != "joined"


def test_head_shards_must_split_evenly():
    from ekv.observe.ranks import head_shard

    assert list(head_shard(8, 3, 4)) == [6, 7]
    with pytest.raises(ValueError):
        head_shard(8, 0, 3)


def test_ranked_share_source_is_the_mean_over_sources():
    from ekv.observe.ranks import RankedShareSource

    class Source:
        def __init__(self, rank):
            self.rank = rank

        def read(self, live_rows, row_blocks):
            return rank_shares(self.rank)[:live_rows].astype(np.float64)

    got = RankedShareSource([Source(0), Source(1)]).read(5, np.full(5, 12))
    want = np.mean([rank_shares(0).astype(np.float64), rank_shares(1).astype(np.float64)], axis=0)
    np.testing.assert_array_equal(got, want)
    with pytest.raises(ValueError):
        RankedShareSource([])
