"""Oracle of the block-table view -- TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``compact_block_table`` restates runtime/block_view.py:36-56 in numpy: block 0 and the last block
of the request are always kept, kept blocks come first in their original order and the other
positions follow in theirs (a stable partition), and the view length is the kept blocks times the
block size less the unfilled part of the last block (0 for an empty row). ``decode_keep`` restates
the keep algebra of DecodeView.build (:272-281). ``slot_compact`` restates the SGLang CSR compaction
(runtime/sglang_compact.py:22-167); it is pinned to the reference's own kernels by
tests/golden/slot_cases.npz.
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


# ---- the SGLang CSR compaction (runtime/sglang_compact.py) --------------------------------------------

SLOT_COUNTS = 5  # blocks read, blocks a full read reads, read in audits, read untrimmed, read with no live policy


def slot_compact(indptr, slots, keep, audit, active: bool, n_real: int, n_rows: int, block_tokens: int):
    """SlotCompactor.compact (sglang_compact.py:131-167): (new indptr, the new list, new lengths, counter deltas).

    plan_kernel (:22-79): a row keeps its first and last block always, and every block when the policy is not
    live, when it is audited (``audit`` uint8 or None), or when it is a padding row (row >= n_real); only real
    rows read ``keep`` and count. gather_kernel (:82-104): position p of the new list comes from its row's kept
    block p // block_tokens (in order) at offset p % block_tokens.
    """
    indptr = np.asarray(indptr, dtype=np.int64)
    slots = np.asarray(slots)
    keep = np.asarray(keep).astype(bool)
    width = keep.shape[1]
    new_indptr = np.zeros(n_rows + 1, dtype=np.int64)
    lens = np.zeros(n_rows, dtype=np.int64)
    out = []
    counts = np.zeros(SLOT_COUNTS, dtype=np.int64)
    for row in range(n_rows):
        length = int(indptr[row + 1] - indptr[row])
        blocks = -(-length // block_tokens)
        real = row < n_real
        audited = audit is not None and real and bool(audit[row])
        whole = (not active) or audited or not real
        chosen = []
        for b in range(min(blocks, width)):
            k = real and bool(keep[row, b])
            if k or whole or b == 0 or b == blocks - 1:
                chosen.append(b)
        kept = len(chosen)
        new_length = (kept - 1) * block_tokens + length - (blocks - 1) * block_tokens if blocks > 0 else 0
        lens[row] = new_length
        new_indptr[row + 1] = new_indptr[row] + new_length
        for p in range(new_length):
            out.append(slots[indptr[row] + chosen[p // block_tokens] * block_tokens + p % block_tokens])
        if real:
            counts[0] += kept
            counts[1] += blocks
            counts[2] += kept * audited
            counts[3] += kept * (new_length == length and not audited and active)
    counts[4] = counts[0] * (1 - int(active))
    return new_indptr, np.asarray(out, dtype=slots.dtype), lens, counts
