"""Attention share of each block from the tile records the audit kernel writes, on the device.

Drop-in for observe/tile_shares.py of the reference: ``share_descriptor``, ``Aggregate``,
``normalize_tile_lse``, ``read_tile_lse`` and ``read_tile_rows`` keep their names, signatures and
exceptions. The table has two planes ``[2][layer][row][block][query_row]`` (plane 0 the tile max
``m``, plane 1 the tile sum ``l``); ``u = m + log(l) - log(tile_blocks)`` is the log weight of a
block, with the tile's weight split evenly over its blocks. Normalising ``u`` over the blocks of one
(layer, row, query row) gives that query's share per block; layers and query rows then average
(or max and rescale) into the row's share.

``normalize_tile_lse`` runs the sm_100a kernel ``ekv_normalize_log_weights``; ``table_shares``
runs ``ekv_normalize_tile_lse`` on a statistic table that is already on the device (the read path
of a controller on the same GPU), with no host round trip for the cells.
"""

from __future__ import annotations

import json
from typing import Literal

import numpy as np
import torch

from .. import _lib
from ..runtime.audit import runtime_dir

Aggregate = Literal["mean", "max"]
_AGGREGATES = {"mean": _lib.AGG_MEAN, "max": _lib.AGG_MAX}


def _pub_path(pid: int) -> str:
    return f"{runtime_dir()}/ekv_pass_{pid}.json"


def _json_lines(path: str) -> list[dict]:
    try:
        with open(path) as f:
            return [json.loads(line) for line in f if line.strip()]
    except FileNotFoundError:
        return []


def share_descriptor(pid: int) -> dict[str, int | str]:
    """The statistic block of process ``pid`` with the tile size of the kernel that records into it.

    Among several recording kernels the narrowest tile wins (the decode kernel's: an audit step
    decodes). Raises ``RuntimeError`` until a recording kernel has published (reference :26-52).
    """
    descriptors = _pub_path(pid)
    coverage = {
        int(item.get("host_va", 0) or 0): item for item in _json_lines(descriptors.replace("ekv_pass_", "ekv_coverage_"))
    }
    candidates = []
    for entry in _json_lines(descriptors):
        if not int(entry.get("tile_lse_dev", 0)):
            continue
        tile_blocks = int(coverage.get(int(entry["host_va"]), {}).get("attn_share_tile_blocks", 0))
        if tile_blocks:
            candidates.append({**entry, "attn_share_tile_blocks": tile_blocks})
    if not candidates:
        raise RuntimeError(f"process {pid} has not compiled a kernel that records the attention statistic")
    return min(candidates, key=lambda entry: int(entry["attn_share_tile_blocks"]))


def _check_aggregate(aggregate: str) -> None:
    if aggregate not in _AGGREGATES:
        raise ValueError(f"unknown aggregate {aggregate!r}")


def normalize_tile_lse(lse, row_blocks, tile_blocks: int, aggregate: Aggregate = "mean"):
    """The attention share per (row, block) from ``lse[layer, row, block, query_row]`` (u values).

    A partial last tile's weight goes back to the blocks that exist; cells at or past
    ``row_blocks[row]`` drop out. Each (layer, row, query row) with a finite value contributes a
    share vector summing to 1; ``mean`` averages them, ``max`` takes each block's largest share and
    rescales the row to sum to 1. A row with no finite value is NaN (reference :58-103).

    numpy in, numpy float64 out (as the reference); a CUDA tensor in, a float32 CUDA tensor out.
    """
    _check_aggregate(aggregate)
    on_device = isinstance(lse, torch.Tensor)
    if lse.ndim != 4:
        raise ValueError("lse must be [layers, rows, blocks, query_rows]")
    layers, rows, width, query_rows = (int(x) for x in lse.shape)
    rb_shape = tuple(row_blocks.shape)
    if rb_shape != (rows,) or tile_blocks < 1:
        raise ValueError("row_blocks must give one length per row, and tile_blocks must be positive")
    device = lse.device if on_device else torch.device("cuda", torch.cuda.current_device())
    u = (lse if on_device else torch.from_numpy(np.ascontiguousarray(lse))).to(device=device, dtype=torch.float32)
    u = u.contiguous()
    rb = torch.as_tensor(np.asarray(row_blocks.cpu() if isinstance(row_blocks, torch.Tensor) else row_blocks))
    rb = rb.clamp(min=-1, max=2**31 - 1).to(device=device, dtype=torch.int32)
    share = torch.empty(rows, width, dtype=torch.float32, device=device)
    if rows and width:
        rc = _lib.load().ekv_normalize_log_weights(
            u.data_ptr() if u.numel() else None, layers, rows, width, query_rows, rb.data_ptr(),
            int(tile_blocks), _AGGREGATES[aggregate], share.data_ptr(), None, _lib.current_stream(),
        )
        _lib.check(rc, "ekv_normalize_log_weights")
    if on_device:
        return share
    return share.cpu().numpy().astype(np.float64)


def table_shares(
    table: torch.Tensor,
    layers: int,
    row_ids,
    row_blocks,
    tile_blocks: int,
    aggregate: Aggregate = "mean",
    contributors: bool = False,
):
    """Shares [len(row_ids), width] (float32, device) straight from the statistic table.

    ``table`` is the device table [2, table_layers, rows, width, cell] (``RecordingPlane.table()``,
    or an IPC mapping of it); this is read_tile_rows followed by normalize_tile_lse without the copy.
    """
    _check_aggregate(aggregate)
    if table.ndim != 5 or table.shape[0] != 2 or table.dtype != torch.float32:
        raise ValueError("the table must be float32 [2, layers, rows, width, cell]")
    _, table_layers, rows, width, cell = (int(x) for x in table.shape)
    ids = torch.as_tensor(np.asarray(row_ids), dtype=torch.int32).to(table.device)
    rb = torch.as_tensor(np.asarray(row_blocks), dtype=torch.int64).clamp(-1, 2**31 - 1).to(torch.int32).to(table.device)
    if ids.shape != rb.shape:
        raise ValueError("row_ids and row_blocks must have one entry each per row read")
    share = torch.empty(len(ids), width, dtype=torch.float32, device=table.device)
    count = torch.empty(len(ids), dtype=torch.int32, device=table.device)
    rc = _lib.load().ekv_normalize_tile_lse(
        table.data_ptr(), table_layers, int(layers), rows, width, cell, ids.data_ptr(), rb.data_ptr(), len(ids),
        int(tile_blocks), _AGGREGATES[aggregate], share.data_ptr(), count.data_ptr(), _lib.current_stream(),
    )
    _lib.check(rc, "ekv_normalize_tile_lse")
    return (share, count) if contributors else share


def read_tile_lse(cuda, base, table_layers, layers, rows, width, group_rows, live_rows, tile_blocks) -> np.ndarray:
    """``u[layers, live_rows, width, group_rows]`` for the first ``live_rows`` rows (reference :106-126)."""
    return read_tile_rows(cuda, base, table_layers, layers, rows, width, group_rows, np.arange(live_rows), tile_blocks)


def read_tile_rows(cuda, base, table_layers, layers, rows, width, group_rows, row_ids, tile_blocks) -> np.ndarray:
    """``u`` for the ascending rows ``row_ids``, copied one run of adjacent rows per (plane, layer).

    ``cuda`` provides ``d2h_many([(address, nbytes), ...])`` (reference :129-173). This is the host
    copy protocol of a controller in another process; ``table_shares`` is the on-device read.
    """
    row_ids = np.asarray(row_ids)
    if np.any(np.diff(row_ids) <= 0):
        raise ValueError("row_ids must be ascending and distinct")
    row_bytes = width * group_rows * 4
    layer_bytes = rows * row_bytes
    plane_bytes = table_layers * layer_bytes
    runs: list[tuple[int, int]] = []
    for r in row_ids.tolist():
        if runs and runs[-1][0] + runs[-1][1] == r:
            runs[-1] = (runs[-1][0], runs[-1][1] + 1)
        else:
            runs.append((r, 1))
    requests = [
        (base + plane * plane_bytes + layer * layer_bytes + first * row_bytes, count * row_bytes)
        for plane in (0, 1)
        for layer in range(layers)
        for first, count in runs
    ]
    blobs = cuda.d2h_many(requests)
    per_plane = layers * len(runs)
    planes = [
        np.frombuffer(b"".join(blobs[p * per_plane : (p + 1) * per_plane]), dtype=np.float32).reshape(
            layers, len(row_ids), width, group_rows
        )
        for p in (0, 1)
    ]
    with np.errstate(divide="ignore"):  # a tile with no keys has l = 0: its weight is exp(-inf) = 0
        return planes[0] + np.log(planes[1]) - np.float32(np.log(tile_blocks))
