"""Oracle of the controller's decide stage -- TEST INFRASTRUCTURE ONLY.

``Ledger`` restates the parts of observe/controller.py that turn audits into the committed keep mask:
the fold of an audit into the per-request shares (Controller._absorb_audit, :311-345: the length of
an audited request looked up by key, rows at or below the length cap not read, rows without evidence
skipped, NaN cells as 0, decay * old + (1 - decay) * new), the shares part of _forget_departed
(:347-359), and the keep mask of _allocate (:398-451) for measured shares with no released blocks,
through ``oracle.allocation.allocate``.
"""

from __future__ import annotations

import math

import numpy as np

from . import allocation as oalloc


def audit_row_blocks(audit_keys: np.ndarray, keys: np.ndarray, lengths: np.ndarray, cap_above_blocks: int):
    """(live, row_blocks) of an audit: rows up to the last audited one, each with its request's current
    length by key, 0 at or below the cap (controller.py:319-323)."""
    audit_keys = np.asarray(audit_keys, dtype=np.uint64)
    audited = np.flatnonzero(audit_keys)
    live = int(audited[-1]) + 1 if audited.size else 0
    current = {int(k): int(n) for k, n in zip(np.asarray(keys, dtype=np.uint64), lengths) if int(k)}
    row_blocks = np.array([current.get(int(audit_keys[row]), 0) for row in range(live)], dtype=np.int64)
    row_blocks[row_blocks <= cap_above_blocks] = 0
    return live, row_blocks


class Ledger:
    def __init__(self, width: int, decay: float) -> None:
        self.width = width
        self.decay = decay
        self.shares: dict[int, np.ndarray] = {}
        self.measured: dict[int, int] = {}

    def absorb(self, fresh: np.ndarray, audit_keys: np.ndarray, row_blocks: np.ndarray) -> None:
        """Fold rows [0, len(fresh)) of an audit (controller.py:332-345)."""
        for row in range(len(fresh)):
            key = int(audit_keys[row])
            if key == 0 or np.isnan(fresh[row]).all():
                continue
            new = np.nan_to_num(fresh[row], nan=0.0)
            old = self.shares.get(key)
            if old is not None:
                grown = np.zeros(max(len(old), len(new)))
                grown[: len(old)] = old
                shorter = np.zeros_like(grown)
                shorter[: len(new)] = new
                new = self.decay * grown + (1.0 - self.decay) * shorter
            self.shares[key] = new
            self.measured[key] = int(row_blocks[row])

    def forget(self, keys: np.ndarray) -> None:
        present = {int(k) for k in np.asarray(keys, dtype=np.uint64) if int(k)}
        for key in set(self.shares) - present:
            del self.shares[key], self.measured[key]

    def keep(self, keys, lengths, row_width: int, budget_fraction: float, objective: str, recent_blocks: int,
             cap_above_blocks: int, weight=None) -> np.ndarray:
        """The keep mask uint8 [rows, row_width] of Controller._allocate (controller.py:398-451)."""
        keys = np.asarray(keys, dtype=np.uint64)
        rows = len(keys)
        keep = np.ones((rows, row_width), dtype=np.uint8)
        measured = [r for r in range(rows)
                    if int(lengths[r]) > cap_above_blocks and int(keys[r]) and int(keys[r]) in self.shares]
        if not measured:
            return keep
        score_list, pinned_list, weights = [], [], []
        for r in measured:
            key = int(keys[r])
            n = min(int(lengths[r]), row_width)
            scores = np.zeros(n)
            have = self.shares[key][:n]
            scores[: len(have)] = have
            pinned = oalloc.controller_pins(n, recent_blocks, self.measured[key])
            score_list.append(scores)
            pinned_list.append(pinned)
            weights.append(1.0 if weight is None else float(weight(key)))
        total = sum(len(s) for s in score_list)
        floor = sum(int(p.sum()) for p in pinned_list)
        budget = max(floor, int(math.ceil(budget_fraction * total)))
        for r, mask in zip(measured, oalloc.allocate(score_list, budget, objective, pinned_list, weights), strict=True):
            keep[r, : len(mask)] = mask
        return keep
