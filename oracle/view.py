"""Oracle of the block-table view -- TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``compact_block_table`` restates runtime/block_view.py:36-56 in numpy: block 0 and the last block
of the request are always kept, kept blocks come first in their original order and the other
positions follow in theirs (a stable partition), and the view length is the kept blocks times the
block size less the unfilled part of the last block (0 for an empty row). ``decode_keep`` restates
the keep algebra of DecodeView.build (:272-281).
"""

from __future__ import annotations

import numpy as np


def compact_block_table(table: np.ndarray, seq_lens: np.ndarray, keep: np.ndarray, block_size: int):
    """(view int32 [rows, width], view_lens int32 [rows])."""
    table = np.asarray(table, dtype=np.int32)
    seq_lens = np.asarray(seq_lens, dtype=np.int64)
    keep = np.asarray(keep).astype(bool)
    rows, width = table.shape
    view = np.empty_like(table)
    view_lens = np.zeros(rows, dtype=np.int32)
    for r in range(rows):
        blocks = int(-(-seq_lens[r] // block_size)) if seq_lens[r] > 0 else 0
        pos = np.arange(width)
        k = (keep[r] | (pos == 0) | (pos == blocks - 1)) & (pos < blocks)
        view[r] = np.concatenate([table[r, k], table[r, ~k]])
        if blocks > 0:
            last = int(seq_lens[r]) - (blocks - 1) * block_size
            view_lens[r] = (int(k.sum()) - 1) * block_size + last
    return view, view_lens


def decode_keep(committed: np.ndarray, full_rows: np.ndarray | None = None, released: np.ndarray | None = None):
    """The mask the view compacts: committed | full rows, then without released blocks."""
    keep = np.asarray(committed).astype(bool).copy()
    if full_rows is not None:
        keep |= np.asarray(full_rows).astype(bool)[:, None]
    if released is not None:
        keep &= ~np.asarray(released).astype(bool)
    return keep
