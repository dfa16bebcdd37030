"""Allocate a read budget across requests by the attention each block carries, on the device.

Drop-in for observe/allocation.py of the reference: ``Objective``, ``Request`` and ``allocate``
keep their names, signature, pins, validation and tie rules. ``uniform`` gives every request the
same fraction of its unpinned blocks by largest remainder (equal remainders to the earlier request)
and keeps each request's best blocks by its own shares, equal shares to the older block
(allocation.py:79-91). ``sum`` keeps the unpinned blocks with the largest weighted share over all
requests, equal gains to the newer block, then to the earlier request (:94-118). ``maxmin`` raises
the smallest retained share as far as the budget allows (:121-166). The quotas run in the sm_100a
kernels ``ekv_allocate_quotas`` (uniform), ``ekv_allocate_sum`` (sum: a global radix select over the
float64 gains, with each request's total summed as NumPy sums it) and ``ekv_allocate_maxmin`` (the
water level), the per-request top-k selection in ``ekv_view_build``.

``allocate`` ranks the float64 values the reference ranks: the share max(score, 0) / total, or the
gain weight * share for ``sum``, each rounded as NumPy rounds it, with the total summed as NumPy's
pairwise sum (``ekv_allocate_sum_f64``, ``ekv_allocate_maxmin_f64``, ``ekv_view_build_f64``); distinct
scores whose shares round to one value tie, as they do in the reference. ``sum_quotas``,
``maxmin_quotas`` and the view also run on float32 scores, whose order is then the order of the shares.
Negative request weights raise ``RuntimeError``; NaN scores count as 0, as the controller passes them
(controller.py:337).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Literal

import numpy as np
import torch

from .. import _lib

Objective = Literal["sum", "maxmin", "uniform"]
# the view's ranking per objective: maxmin keeps each request's blocks by share, equal shares to the older block
_POLICIES = {"sum": _lib.POLICY_SUM, "uniform": _lib.POLICY_UNIFORM, "newest": _lib.POLICY_NEWEST,
             "maxmin": _lib.POLICY_UNIFORM}


@dataclass(frozen=True)
class Request:
    """One request: the score of each of its blocks, and how much its retained share counts."""

    scores: np.ndarray
    weight: float = 1.0
    pinned: np.ndarray | None = None

    def pinned_mask(self) -> np.ndarray:
        if self.pinned is not None:
            return np.asarray(self.pinned, dtype=bool)
        mask = np.zeros(len(self.scores), dtype=bool)
        mask[[0, -1]] = len(self.scores) > 0
        return mask

    def shares(self) -> np.ndarray:
        """Scores normalised to sum to 1 (float64). A request with no evidence gets equal shares."""
        scores = np.maximum(np.asarray(self.scores, dtype=np.float64), 0.0)
        total = scores.sum()
        if total <= 0.0:
            return np.full(len(scores), 1.0 / max(len(scores), 1))
        return scores / total


def _pin_start(pinned: np.ndarray) -> int | None:
    """``ps`` with pinned == {0} | [ps, n) (the controller's pins), or None for any other pin set."""
    n = len(pinned)
    if n == 0:
        return 0
    tail = n
    while tail > 0 and pinned[tail - 1]:
        tail -= 1
    expected = np.zeros(n, dtype=bool)
    expected[0] = True
    expected[tail:] = True
    return tail if np.array_equal(pinned, expected) else None


def _score_layout(scores: torch.Tensor, row_blocks: torch.Tensor, score_rows: torch.Tensor | None) -> tuple[int, int]:
    """(rows, width) of a quota call: one row per ``row_blocks`` entry; ``score_rows`` maps them to score rows."""
    if scores.dtype not in (torch.float32, torch.float64) or scores.ndim != 2 or scores.stride(1) != 1:
        raise ValueError("scores must be float32 or float64 [rows, width] with contiguous rows")
    if score_rows is not None and scores.dtype != torch.float64:
        raise ValueError("score_rows needs float64 scores")
    rows = int(row_blocks.shape[0]) if score_rows is not None else int(scores.shape[0])
    return rows, int(scores.shape[1])


def sum_quotas(
    scores: torch.Tensor,
    row_blocks: torch.Tensor,
    quota: torch.Tensor,
    *,
    measured: torch.Tensor | None,
    recent_blocks: int,
    cap_above_blocks: int,
    budget: int = -1,
    budget_fraction: float = 0.0,
    weights: torch.Tensor | None = None,
    score_rows: torch.Tensor | None = None,
    mask_out: torch.Tensor | None = None,
) -> torch.Tensor:
    """The per-row quotas of the ``sum`` objective with one shared budget (``ekv_allocate_sum``).

    ``scores`` float32 or float64 [., width] on the device, ``row_blocks`` int32 [rows], ``quota`` int32
    [rows] (out), ``weights`` float64 [rows] or None; ``score_rows`` (int32 [rows], float64 scores only)
    reads row r's scores from row ``score_rows[r]``; ``mask_out`` (uint8 [rows, width], float64 scores
    only) receives the committed keep mask straight from the threshold. ``budget`` >= 0 as given, else
    from ``budget_fraction`` as the controller computes it. No host synchronisation.
    """
    rows, width = _score_layout(scores, row_blocks, score_rows)
    lib = _lib.load()
    size = int(lib.ekv_allocate_sum_workspace_bytes(rows, width))
    workspace = torch.empty(size + 256, dtype=torch.uint8, device=scores.device)
    base = (workspace.data_ptr() + 255) // 256 * 256
    common = (
        None if weights is None else weights.data_ptr(), row_blocks.data_ptr(),
        None if measured is None else measured.data_ptr(), int(recent_blocks), int(cap_above_blocks),
        float(budget_fraction), int(budget), rows, width, quota.data_ptr(), base, size, _lib.current_stream(),
    )
    if scores.dtype == torch.float64:
        rows_ptr = None if score_rows is None else score_rows.data_ptr()
        mask = (None, 0) if mask_out is None else (mask_out.data_ptr(), mask_out.stride(0))
        rc = lib.ekv_allocate_sum_f64(scores.data_ptr(), scores.stride(0), rows_ptr, *common[:10], *mask, *common[10:])
        _lib.check(rc, "ekv_allocate_sum_f64")
    else:
        if mask_out is not None:
            raise ValueError("the mask straight from the threshold is written for float64 scores")
        rc = lib.ekv_allocate_sum(scores.data_ptr(), scores.stride(0), *common)
        _lib.check(rc, "ekv_allocate_sum")
    return quota


def maxmin_quotas(
    scores: torch.Tensor,
    row_blocks: torch.Tensor,
    quota: torch.Tensor,
    *,
    measured: torch.Tensor | None,
    recent_blocks: int,
    cap_above_blocks: int,
    budget: int = -1,
    budget_fraction: float = 0.0,
    score_rows: torch.Tensor | None = None,
) -> torch.Tensor:
    """The per-row quotas of the ``maxmin`` objective with one shared budget (``ekv_allocate_maxmin``), for a
    view built with the ``uniform`` ranking. Arguments as ``sum_quotas``; no weights."""
    rows, width = _score_layout(scores, row_blocks, score_rows)
    lib = _lib.load()
    size = int(lib.ekv_allocate_maxmin_workspace_bytes(rows, width))
    workspace = torch.empty(size + 256, dtype=torch.uint8, device=scores.device)
    base = (workspace.data_ptr() + 255) // 256 * 256
    common = (
        row_blocks.data_ptr(), None if measured is None else measured.data_ptr(), int(recent_blocks),
        int(cap_above_blocks), float(budget_fraction), int(budget), rows, width, quota.data_ptr(), base, size,
        _lib.current_stream(),
    )
    if scores.dtype == torch.float64:
        rows_ptr = None if score_rows is None else score_rows.data_ptr()
        rc = lib.ekv_allocate_maxmin_f64(scores.data_ptr(), scores.stride(0), rows_ptr, *common)
        _lib.check(rc, "ekv_allocate_maxmin_f64")
    else:
        rc = lib.ekv_allocate_maxmin(scores.data_ptr(), scores.stride(0), *common)
        _lib.check(rc, "ekv_allocate_maxmin")
    return quota


def allocate(requests: Sequence[Request], budget: int, objective: Objective = "sum") -> list[np.ndarray]:
    """Return, for each request, a bool mask of the blocks to keep. At most ``budget`` blocks are kept."""
    sizes = [len(r.scores) for r in requests]
    pinned = [r.pinned_mask() for r in requests]
    if any(len(p) != n for p, n in zip(pinned, sizes, strict=True)):
        raise ValueError("a pinned mask must have one entry per block")
    if budget < 0:
        raise ValueError("the budget cannot be negative")
    must = sum(int(p.sum()) for p in pinned)
    if must > budget and budget < sum(sizes):
        raise ValueError(f"the budget {budget} cannot hold the {must} pinned blocks")
    if budget >= sum(sizes):
        return [np.ones(n, dtype=bool) for n in sizes]
    if objective not in ("sum", "maxmin", "uniform"):
        raise ValueError(f"unknown objective {objective!r}")
    if objective in ("maxmin", "uniform") and any(r.weight != 1.0 for r in requests):
        raise ValueError(f"the {objective} objective does not use request weights")
    width = max(sizes) if sizes else 0
    rows = len(requests)
    if rows == 0 or width == 0:
        return [p.copy() for p in pinned]
    if objective == "sum" and any(not r.weight >= 0.0 or not np.isfinite(r.weight) for r in requests):
        raise RuntimeError("negative or non-finite request weights are not supported on the device")
    scores = np.zeros((rows, width), dtype=np.float64)
    for r, req in enumerate(requests):
        s = np.asarray(req.scores, dtype=np.float64)
        scores[r, : sizes[r]] = np.where(np.isnan(s), 0.0, s)
    device = torch.device("cuda", torch.cuda.current_device())
    lib = _lib.load()
    stream = _lib.current_stream()
    row_blocks = torch.tensor(sizes, dtype=torch.int32).to(device)
    starts = [_pin_start(p) for p in pinned]
    if any(start is None for start in starts):
        return _allocate_pinned(scores, pinned, sizes, requests, budget, objective, row_blocks)
    # pins {0} | [pin_start, n): passed as the "measured" start, with no recent pins of their own
    measured = torch.tensor(starts, dtype=torch.int32).to(device)
    quota = torch.empty(rows, dtype=torch.int32, device=device)
    scores_t = torch.from_numpy(scores).to(device)
    if objective == "uniform":
        rc = lib.ekv_allocate_quotas(row_blocks.data_ptr(), measured.data_ptr(), -1, -1, 0.0, int(budget), None,
                                     _lib.POLICY_UNIFORM, rows, width, quota.data_ptr(), stream)
        _lib.check(rc, "ekv_allocate_quotas")
    elif objective == "maxmin":
        maxmin_quotas(scores_t, row_blocks, quota, measured=measured, recent_blocks=-1, cap_above_blocks=-1,
                      budget=int(budget))
    mask = torch.empty(rows, width, dtype=torch.uint8, device=device)
    if objective == "sum":  # the mask straight from the global threshold
        weights = torch.tensor([float(r.weight) for r in requests], dtype=torch.float64).to(device)
        sum_quotas(scores_t, row_blocks, quota, measured=measured, recent_blocks=-1, cap_above_blocks=-1,
                   budget=int(budget), weights=weights, mask_out=mask)
    else:
        rc = lib.ekv_view_build_f64(
            None, 0, None, row_blocks.data_ptr(), quota.data_ptr(), measured.data_ptr(), -1, scores_t.data_ptr(),
            width, None, None, _POLICIES[objective], None, None, 0, rows, width, 16, None, 0, None,
            mask.data_ptr(), width, stream,
        )
        _lib.check(rc, "ekv_view_build_f64")
    out = mask.cpu().numpy().astype(bool)
    return [out[r, : sizes[r]].copy() for r in range(rows)]


def _allocate_pinned(scores: np.ndarray, pinned: list[np.ndarray], sizes: list[int], requests: Sequence[Request],
                     budget: int, objective: Objective, row_blocks: torch.Tensor) -> list[np.ndarray]:
    """``allocate`` for pins other than block 0 and a newest suffix (``ekv_allocate_pinned_f64``): the shares
    are computed and ranked on the device with the pinned blocks brought to the kernels' pin shape."""
    rows, width = scores.shape
    lib = _lib.load()
    size = int(lib.ekv_allocate_pinned_workspace_bytes(rows, width))
    if size == 0:
        raise RuntimeError(f"requests of {width} blocks with arbitrary pins exceed the device allocation's 16383")
    device = row_blocks.device
    pin = np.zeros((rows, width), dtype=np.uint8)
    for r, p in enumerate(pinned):
        pin[r, : sizes[r]] = p
    scores_t = torch.from_numpy(scores).to(device)
    pin_t = torch.from_numpy(pin).to(device)
    weights = None
    if objective == "sum":
        weights = torch.tensor([float(r.weight) for r in requests], dtype=torch.float64).to(device)
    code = {"sum": _lib.POLICY_SUM, "uniform": _lib.POLICY_UNIFORM, "maxmin": _lib.POLICY_MAXMIN}[objective]
    workspace = torch.empty(size + 256, dtype=torch.uint8, device=device)
    base = (workspace.data_ptr() + 255) // 256 * 256
    mask = torch.empty(rows, width, dtype=torch.uint8, device=device)
    rc = lib.ekv_allocate_pinned_f64(
        scores_t.data_ptr(), width, pin_t.data_ptr(), width, _lib.ptr(weights), row_blocks.data_ptr(), code,
        int(budget), rows, width, mask.data_ptr(), width, base, size, _lib.current_stream(),
    )
    _lib.check(rc, "ekv_allocate_pinned_f64")
    out = mask.cpu().numpy().astype(bool)
    return [out[r, : sizes[r]].copy() for r in range(rows)]
