"""Oracle of the audit kernel -- TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``tile_lse`` restates tile_lse_kernel (runtime/audit_kernel.py:34-109) and the launch that feeds it
(:224-265) in float32 numpy: for every selected row and every tile of ``tile_blocks * block_size``
tokens whose first token lies below the row's length, the tile max ``m`` and the tile sum
``l = sum(exp(score - m))`` of ``score = q . k * scale`` over the tile's tokens below the length,
stored in every block cell of the tile that starts below the length. ``heads`` > 1 records KV heads
``group .. group + heads - 1`` side by side in a cell (the all-heads mode); 1 is the reference.
"""

from __future__ import annotations

import numpy as np


def tile_lse(
    query: np.ndarray,
    keys: np.ndarray,
    table: np.ndarray,
    lens: np.ndarray,
    qrow: np.ndarray,
    select: np.ndarray,
    flag: int,
    lse: np.ndarray,
    scale: float,
    layer: int,
    group: int,
    block_size: int,
    tile_blocks: int,
    heads: int = 1,
) -> None:
    """Write one layer's cells into ``lse`` [2, layers, rows, width, heads*G] in place.

    query [tokens, q_heads, D] and keys [pool, block_size, kv_heads, D] of any float type are read
    as float32, as the reference kernel's dot accumulates in float32 (audit_kernel.py:93).
    """
    if not flag:  # the statistic is off: nothing is written (:64)
        return
    rows, width = table.shape
    q_cell = lse.shape[-1]
    group_rows = q_cell // heads
    tile_tokens = tile_blocks * block_size
    for row in range(rows):
        if not select[row]:
            continue
        length = int(lens[row])
        if length <= 0:
            continue
        n_tiles = -(-length // tile_tokens)
        pos = np.arange(n_tiles * tile_tokens)
        valid = pos < length
        block_col = np.minimum(pos // block_size, width - 1)
        ids = np.where(valid, table[row, block_col], 0)
        n_blocks = -(-length // block_size)
        for h in range(heads):
            kv = group + h
            q = np.asarray(query[int(qrow[row]), kv * group_rows : (kv + 1) * group_rows], dtype=np.float32)
            k = np.asarray(keys[ids, pos % block_size, kv], dtype=np.float32)  # [tokens, D]
            k[~valid] = 0.0
            score = (k @ q.T) * np.float32(scale)  # [tokens, G], as tl.dot(q, k^T) * scale (:93)
            score = np.where(valid[:, None], score, np.float32(-np.inf)).reshape(n_tiles, tile_tokens, -1)
            peak = score.max(axis=1)  # (:95)
            total = np.exp(score - peak[:, None, :]).sum(axis=1, dtype=np.float32)  # (:96)
            cells = slice(h * group_rows, (h + 1) * group_rows)
            blocks = np.arange(n_blocks)  # block_index * BLOCK_SIZE < length (:99)
            lse[0, layer, row, blocks, cells] = peak[blocks // tile_blocks]
            lse[1, layer, row, blocks, cells] = total[blocks // tile_blocks]


def new_table(layers: int, rows: int, width: int, cell: int) -> np.ndarray:
    """The statistic table as RecordingPlane allocates it: every cell NaN (audit_kernel.py:135-137)."""
    return np.full((2, layers, rows, width, cell), np.nan, dtype=np.float32)
