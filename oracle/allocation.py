"""Oracle of the budget allocation and the controller's keep mask -- TEST INFRASTRUCTURE ONLY.

``shares``, ``allocate``, ``uniform`` and ``greedy`` restate observe/allocation.py:46-118
(``Request.shares``, ``allocate``, ``_uniform``, ``_greedy``) with their exact tie rules: ``uniform``
ranks each request by its own shares, equal shares going to the older block (:89), with quotas by
largest remainder, equal remainders to the earlier request (:83-86); ``sum`` keeps the globally
largest weighted shares, equal ones going to the newer block and then the earlier request (:107-113).
``controller_keep`` restates the parts of Controller._allocate (observe/controller.py:398-451) that
define the keep mask: which rows are measured, their pins and the budget formula.
"""

from __future__ import annotations

import math

import numpy as np


def shares(scores: np.ndarray) -> np.ndarray:
    """Scores clamped at 0 and scaled to sum to 1 in float64; equal shares without evidence (:46-52)."""
    s = np.maximum(np.asarray(scores, dtype=np.float64), 0.0)
    total = s.sum()
    if total <= 0.0:
        return np.full(len(s), 1.0 / max(len(s), 1))
    return s / total


def default_pins(n: int) -> np.ndarray:
    """The first and the last block (:39-44)."""
    mask = np.zeros(n, dtype=bool)
    if n:
        mask[0] = mask[-1] = True
    return mask


def uniform(score_list, pinned_list, free: int) -> list[np.ndarray]:
    open_idx = [np.flatnonzero(~p) for p in pinned_list]
    total = sum(len(o) for o in open_idx)
    # Python int arithmetic, one correctly rounded true division, as allocation.py:83
    exact = [free * len(o) / total if total else 0.0 for o in open_idx]
    quota = [int(x) for x in exact]
    extra = free - sum(quota)
    ranked = sorted(range(len(open_idx)), key=lambda i: (quota[i] - exact[i], i))
    for i in ranked[:extra]:  # extra >= 0: each quota is a floor of a correctly rounded ratio
        quota[i] += 1
    kept = []
    for scores, pinned, o, q in zip(score_list, pinned_list, open_idx, quota, strict=True):
        mask = pinned.copy()
        s = shares(scores)[o]
        # descending share, equal shares in ascending position: lexsort sorts by the last key first
        order = o[np.lexsort((o, -s))]
        mask[order[:q]] = True
        kept.append(mask)
    return kept


def greedy(score_list, pinned_list, weights, free: int) -> list[np.ndarray]:
    kept = [p.copy() for p in pinned_list]
    if free <= 0 or not score_list:
        return kept
    cells = []  # (gain, block, request)
    for r, (scores, pinned, w) in enumerate(zip(score_list, pinned_list, weights, strict=True)):
        s = shares(scores)
        for b in np.flatnonzero(~pinned):
            cells.append((w * s[b], int(b), r))
    cells.sort(key=lambda c: (-c[0], -c[1], c[2]))
    for _gain, b, r in cells[:free]:
        kept[r][b] = True
    return kept


def water_level(score_list, pinned_list, free: int) -> list[np.ndarray]:
    """maxmin (allocation.py:121-166): the highest level of retained share every request can reach within
    ``free`` blocks (60 bisection steps over searchsorted running sums), then one block at a time to the
    request with the lowest retained share, ties to the earlier request."""
    import heapq

    shares_list = [shares(s) for s in score_list]
    order = [np.flatnonzero(~p)[np.argsort(-sh[~p], kind="stable")] for sh, p in zip(shares_list, pinned_list,
                                                                                       strict=True)]
    base = [float(sh[p].sum()) for sh, p in zip(shares_list, pinned_list, strict=True)]
    prefix = [np.cumsum(sh[o]) for sh, o in zip(shares_list, order, strict=True)]
    stacked = np.concatenate([pr + 2.0 * r for r, pr in enumerate(prefix)]) if prefix else np.zeros(0)
    sizes = np.array([len(o) for o in order])
    starts = np.concatenate(([0], np.cumsum(sizes)[:-1]))
    offsets = 2.0 * np.arange(len(score_list))
    base_a = np.array(base)

    def extra(level: float) -> np.ndarray:
        need = level - base_a
        position = np.searchsorted(stacked, need - 1e-12 + offsets) - starts
        return np.where(need <= 1e-12, 0, np.minimum(position + 1, sizes))

    low, high = 0.0, 1.0
    for _ in range(60):
        mid = (low + high) / 2
        if int(extra(mid).sum()) <= free:
            low = mid
        else:
            high = mid
    counts = [int(c) for c in extra(low)]
    kept = [p.copy() for p in pinned_list]
    for r, k in enumerate(counts):
        kept[r][order[r][:k]] = True
    leftover = free - sum(counts)
    retained = [base[r] + (float(prefix[r][counts[r] - 1]) if counts[r] else 0.0) for r in range(len(score_list))]
    heap = [(retained[r], r) for r in range(len(score_list)) if counts[r] < len(order[r])]
    heapq.heapify(heap)
    while leftover > 0 and heap:
        level, r = heapq.heappop(heap)
        block = order[r][counts[r]]
        kept[r][block] = True
        counts[r] += 1
        leftover -= 1
        if counts[r] < len(order[r]):
            heapq.heappush(heap, (level + float(shares_list[r][block]), r))
    return kept


def allocate(score_list, budget: int, objective: str = "sum", pinned_list=None, weights=None) -> list[np.ndarray]:
    """Masks of kept blocks per request, at most ``budget`` in all (allocation.py:55-76)."""
    sizes = [len(s) for s in score_list]
    pinned_list = [default_pins(n) for n in sizes] if pinned_list is None else [np.asarray(p, bool) for p in pinned_list]
    weights = [1.0] * len(sizes) if weights is None else list(weights)
    if budget < 0:
        raise ValueError("the budget cannot be negative")
    must = sum(int(p.sum()) for p in pinned_list)
    if must > budget and budget < sum(sizes):
        raise ValueError(f"the budget {budget} cannot hold the {must} pinned blocks")
    if budget >= sum(sizes):
        return [np.ones(n, dtype=bool) for n in sizes]
    if objective == "sum":
        return greedy(score_list, pinned_list, weights, budget - must)
    if objective == "uniform":
        return uniform(score_list, pinned_list, budget - must)
    if objective == "maxmin":
        return water_level(score_list, pinned_list, budget - must)
    raise ValueError(f"unknown objective {objective!r}")


def controller_pins(n: int, recent_blocks: int, measured: int | None = None) -> np.ndarray:
    """Block 0, the newest recent_blocks + 1 blocks, and those added since the audit (controller.py:420-424)."""
    pinned = np.zeros(n, dtype=bool)
    if n:
        pinned[0] = True
        pinned[max(0, n - 1 - recent_blocks) :] = True
        if measured is not None:
            pinned[max(measured, 0) :] = True
    return pinned


def controller_keep(
    row_blocks: np.ndarray,
    width: int,
    scores_of,
    budget_fraction: float,
    objective: str,
    recent_blocks: int = 4,
    cap_above_blocks: int = 0,
    measured: np.ndarray | None = None,
    weights: np.ndarray | None = None,
) -> np.ndarray:
    """The keep mask uint8 [rows, width] the controller commits; ``scores_of(row, n)`` gives a row's scores,
    ``weights[row]`` its request weight (None: 1.0)."""
    rows = len(row_blocks)
    keep = np.ones((rows, width), dtype=np.uint8)
    chosen = [r for r in range(rows) if int(row_blocks[r]) > cap_above_blocks and int(row_blocks[r]) > 0]
    if not chosen:
        return keep
    score_list, pinned_list = [], []
    for r in chosen:
        n = min(int(row_blocks[r]), width)
        score_list.append(np.asarray(scores_of(r, n), dtype=np.float64))
        pinned_list.append(controller_pins(n, recent_blocks, None if measured is None else int(measured[r])))
    total = sum(len(s) for s in score_list)
    floor = sum(int(p.sum()) for p in pinned_list)
    budget = max(floor, int(math.ceil(budget_fraction * total)))
    w = None if weights is None else [float(weights[r]) for r in chosen]
    for r, mask in zip(chosen, allocate(score_list, budget, objective, pinned_list, w), strict=True):
        keep[r, : len(mask)] = mask
    return keep


def per_row_keep(
    row_blocks: np.ndarray,
    width: int,
    scores: np.ndarray,
    row_fraction: np.ndarray,
    objective: str,
    recent_blocks: int = 0,
) -> np.ndarray:
    """Every row its own allocate() call with budget max(pins, ceil(fraction * n)) (the view stress case)."""
    rows = len(row_blocks)
    keep = np.ones((rows, width), dtype=np.uint8)
    for r in range(rows):
        n = min(int(row_blocks[r]), width)
        if n <= 0:
            continue
        pinned = controller_pins(n, recent_blocks)
        budget = max(int(pinned.sum()), int(math.ceil(float(row_fraction[r]) * n)))
        (mask,) = allocate([scores[r, :n]], budget, objective, [pinned])
        keep[r, :n] = mask
    return keep
