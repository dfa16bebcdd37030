"""Oracle of the exact-statistic normalisation -- TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``log_weights`` restates the arithmetic of read_tile_rows (observe/tile_shares.py:129-173):
``u = m + log(l) - log(tile_blocks)`` in float32 for the chosen rows and layers. ``normalize``
restates normalize_tile_lse (:58-103): the weight of a partial last tile is given back to the blocks
that exist, cells at or past the row's length drop out, each (layer, row, query row) with a finite
value becomes a share vector summing to 1, and the vectors are averaged (``mean``) or maxed and
rescaled (``max``); a row with no finite value is NaN. ``mean_over_ranks`` is RankedShareSource.read
(observe/ranks.py:117-119).
"""

from __future__ import annotations

import numpy as np


def log_weights(lse: np.ndarray, layers: int, row_ids: np.ndarray, tile_blocks: int) -> np.ndarray:
    """u[layers, len(row_ids), width, cell] from the table lse[2, table_layers, rows, width, cell]."""
    m = lse[0, :layers][:, row_ids]
    total = lse[1, :layers][:, row_ids]
    with np.errstate(divide="ignore", invalid="ignore"):
        return m + np.log(total) - np.float32(np.log(tile_blocks))


def normalize(u: np.ndarray, row_blocks: np.ndarray, tile_blocks: int, aggregate: str = "mean") -> np.ndarray:
    """share[rows, width] (float64) from u[layers, rows, width, query_rows]."""
    if aggregate not in ("mean", "max"):
        raise ValueError(f"unknown aggregate {aggregate!r}")
    if u.ndim != 4:
        raise ValueError("u must be [layers, rows, blocks, query_rows]")
    layers, rows, width, query_rows = u.shape
    row_blocks = np.asarray(row_blocks)
    if row_blocks.shape != (rows,) or tile_blocks < 1:
        raise ValueError("row_blocks must give one length per row, and tile_blocks must be positive")
    out = np.full((rows, width), np.nan)
    for r in range(rows):
        n = int(row_blocks[r])
        b = np.arange(width)
        # the partial last tile: its valid blocks share the whole tile weight (tile_shares.py:82-87)
        tail_start = (n // tile_blocks) * tile_blocks
        valid_tail = max(n - tail_start, 1)
        regain = np.where((n % tile_blocks != 0) & (b >= tail_start) & (b < n), np.log(tile_blocks / valid_tail), 0.0)
        x = np.where((b < n)[None, :, None], u[:, r].astype(np.float64), np.nan) + regain[None, :, None]
        finite = np.isfinite(x)
        acc = np.zeros(width)
        contributors = 0
        for layer in range(layers):
            for j in range(query_rows):
                f = finite[layer, :, j]
                if not f.any():
                    continue
                contributors += 1
                v = x[layer, :, j]
                w = np.where(f, np.exp(np.where(f, v, 0.0) - v[f].max()), 0.0)
                s = w / w.sum()
                acc = np.maximum(acc, s) if aggregate == "max" else acc + s
        if contributors == 0:
            continue  # no evidence: the row stays NaN (:103)
        if aggregate == "max":
            t = acc.sum()
            out[r] = acc / t if t > 0 else np.zeros(width)
        else:
            out[r] = acc / contributors
    return out


def normalize_rows(u: np.ndarray, row_blocks: np.ndarray, tile_blocks: int, aggregate: str = "mean") -> np.ndarray:
    """``normalize`` with each row's (layer, query row) share vectors computed at once.

    The same arithmetic (observe/tile_shares.py:82-103) in float64, vectorised over a row's layers and
    query rows instead of looping over them, for checks at full model sizes (80 layers x 64 query rows).
    The per-vector sums run in NumPy's order rather than one after another, a difference of a few units
    in the last place of float64; tests hold both forms to each other.
    """
    if aggregate not in ("mean", "max"):
        raise ValueError(f"unknown aggregate {aggregate!r}")
    if u.ndim != 4:
        raise ValueError("u must be [layers, rows, blocks, query_rows]")
    layers, rows, width, query_rows = u.shape
    row_blocks = np.asarray(row_blocks)
    if row_blocks.shape != (rows,) or tile_blocks < 1:
        raise ValueError("row_blocks must give one length per row, and tile_blocks must be positive")
    out = np.full((rows, width), np.nan)
    b = np.arange(width)
    for r in range(rows):
        n = int(row_blocks[r])
        tail_start = (n // tile_blocks) * tile_blocks
        valid_tail = max(n - tail_start, 1)
        regain = np.where((n % tile_blocks != 0) & (b >= tail_start) & (b < n), np.log(tile_blocks / valid_tail), 0.0)
        x = np.where((b < n)[None, :, None], u[:, r].astype(np.float64), np.nan) + regain[None, :, None]  # [L, W, Q]
        finite = np.isfinite(x)
        peak = np.where(finite, x, -np.inf).max(axis=1, keepdims=True)
        has = np.isfinite(peak)
        w = np.where(finite, np.exp(np.where(finite, x, 0.0) - np.where(has, peak, 0.0)), 0.0)
        total = w.sum(axis=1, keepdims=True)
        share = np.divide(w, total, out=np.zeros_like(w), where=total > 0)
        count = int(has.sum())
        if count == 0:
            continue  # no evidence: the row stays NaN (:103)
        if aggregate == "max":
            acc = share.max(axis=(0, 2))
            t = acc.sum()
            out[r] = acc / t if t > 0 else np.zeros(width)
        else:
            out[r] = share.sum(axis=(0, 2)) / count
    return out


def contributors(u: np.ndarray, row_blocks: np.ndarray, tile_blocks: int) -> np.ndarray:
    """The number of (layer, query row) pairs of each row with at least one finite cell."""
    layers, rows, width, query_rows = u.shape
    b = np.arange(width)
    inside = b[None, :] < np.asarray(row_blocks)[:, None]
    finite = np.isfinite(u) & inside[None, :, :, None]
    return finite.any(axis=2).sum(axis=(0, 2))


def mean_over_ranks(shares: list[np.ndarray]) -> np.ndarray:
    """The mean over tensor-parallel ranks; a NaN at any rank stays NaN (ranks.py:117-119)."""
    return np.mean(np.stack(shares), axis=0)
