"""A per-request view of the block table for decode attention, built on the device.

Drop-in for runtime/block_view.py of the reference. A paged attention kernel reads a request's KV
cache through its row of the block table and its length; a shorter row with a shorter length is a
read budget the kernel enforces unchanged. ``compact_block_table`` and ``DecodeView.build`` keep the
reference's semantics exactly (kept blocks first in order, then the rest in order; block 0 and the
last block always kept; lease, audit, prefill and released-block rules) and run as one sm_100a
kernel per call (``ekv_view_build``). ``plan_view`` fuses the controller's decision into it: pins,
budget quotas and per-row top-k from the device shares, then the compaction, with no host round trip.
"""

from __future__ import annotations

import os
import time
from collections.abc import Callable
from typing import Protocol

import numpy as np
import torch

from .. import _lib
from .audit import AuditPlane

# the view's ranking per objective: maxmin keeps each request's blocks by share, equal shares to the older block
_POLICIES = {"sum": _lib.POLICY_SUM, "uniform": _lib.POLICY_UNIFORM, "newest": _lib.POLICY_NEWEST,
             "maxmin": _lib.POLICY_UNIFORM}


class StatisticSwitch(Protocol):
    """What the view needs to turn the statistic on for a step and off after it."""

    def set(self, on: bool) -> None: ...

    def select(self, audited: np.ndarray, token_start: np.ndarray) -> None: ...


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _view_build(
    table: torch.Tensor,
    seq_lens: torch.Tensor,
    block_size: int,
    *,
    keep: torch.Tensor | None = None,
    full_rows: torch.Tensor | None = None,
    released: torch.Tensor | None = None,
    row_blocks: torch.Tensor | None = None,
    quota: torch.Tensor | None = None,
    measured: torch.Tensor | None = None,
    recent_blocks: int = 0,
    scores: torch.Tensor | None = None,
    policy: str = "uniform",
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
    mask_out: torch.Tensor | None = None,
    weights: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    rows, width = int(table.shape[0]), int(table.shape[1])
    if table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise ValueError("the block table and the lengths must be int32")
    if table.stride(1) != 1:
        raise ValueError("the block table's rows must be contiguous")
    view, view_lens = out if out is not None else (
        torch.empty(rows, width, dtype=torch.int32, device=table.device),
        torch.empty(rows, dtype=torch.int32, device=table.device),
    )
    if rows == 0:
        return view, view_lens

    def u8(t):
        if t is None:
            return None
        t = t.to(torch.uint8) if t.dtype != torch.uint8 else t
        return t if t.stride(-1) == 1 else t.contiguous()

    keep, full_rows, released = u8(keep), u8(full_rows), u8(released)
    if scores is not None and scores.dtype == torch.float64 and keep is None:
        # float64 scores: ranked by the float64 share (or weighted gain) itself
        rc = _lib.load().ekv_view_build_f64(
            table.data_ptr(), table.stride(0), seq_lens.data_ptr(), _ptr(row_blocks), _ptr(quota), _ptr(measured),
            int(recent_blocks), scores.data_ptr(), scores.stride(0), None,
            _ptr(weights) if policy == "sum" else None, _POLICIES[policy],
            _ptr(full_rows), _ptr(released), released.stride(0) if released is not None else 0, rows, width,
            int(block_size), view.data_ptr(), view.stride(0), view_lens.data_ptr(), _ptr(mask_out),
            mask_out.stride(0) if mask_out is not None else 0, _lib.current_stream(),
        )
        _lib.check(rc, "ekv_view_build_f64")
        return view, view_lens
    rc = _lib.load().ekv_view_build(
        table.data_ptr(), table.stride(0), seq_lens.data_ptr(), _ptr(row_blocks), _ptr(quota), _ptr(measured),
        int(recent_blocks), _ptr(scores), scores.stride(0) if scores is not None else 0, _POLICIES[policy],
        _ptr(keep), keep.stride(0) if keep is not None else 0, _ptr(full_rows), _ptr(released),
        released.stride(0) if released is not None else 0, rows, width, int(block_size),
        view.data_ptr(), view.stride(0), view_lens.data_ptr(), _ptr(mask_out),
        mask_out.stride(0) if mask_out is not None else 0, _lib.current_stream(),
    )
    _lib.check(rc, "ekv_view_build")
    return view, view_lens


def _sum_budget_fits(table: torch.Tensor, seq_lens: torch.Tensor, scores: torch.Tensor) -> bool:
    """Whether a shared `sum` budget and its view can be one ekv_view_build_sum_budget call: int32 table rows
    of at most 16384 blocks and float32 or float64 scores of the table's width."""
    return (table.dtype == torch.int32 and seq_lens.dtype == torch.int32 and table.stride(1) == 1
            and 0 < int(table.shape[1]) <= 16384 and scores.dtype in (torch.float32, torch.float64)
            and scores.dim() == 2 and int(scores.shape[1]) == int(table.shape[1]) and scores.stride(1) == 1
            and int(scores.shape[0]) >= int(table.shape[0]))


def _sum_budget_view(table, seq_lens, block_size, row_blocks, scores, budget_fraction, recent_blocks,
                     cap_above_blocks, measured, weights, released, full_rows, mask_out, out):
    """The shared `sum` budget's decision and the view in one call: the select finds the threshold gain and
    the view keeps every request's blocks above it (ekv_view_build_sum_budget), no per-row ranking."""
    rows, width = int(table.shape[0]), int(table.shape[1])
    view, view_lens = out if out is not None else (
        torch.empty(rows, width, dtype=torch.int32, device=table.device),
        torch.empty(rows, dtype=torch.int32, device=table.device),
    )
    if rows == 0:
        return view, view_lens
    u8 = [None if t is None else (t.to(torch.uint8) if t.dtype != torch.uint8 else t).contiguous()
          for t in (released, full_rows)]
    released, full_rows = u8
    lib = _lib.load()
    size = int(lib.ekv_allocate_sum_workspace_bytes(rows, width))
    workspace = torch.empty(size + 256, dtype=torch.uint8, device=table.device)
    base = (workspace.data_ptr() + 255) // 256 * 256
    rc = lib.ekv_view_build_sum_budget(
        scores.data_ptr(), scores.element_size(), scores.stride(0), None, _ptr(weights), row_blocks.data_ptr(),
        _ptr(measured), int(recent_blocks), int(cap_above_blocks), budget_fraction, -1, table.data_ptr(),
        table.stride(0), seq_lens.data_ptr(), _ptr(full_rows), _ptr(released),
        released.stride(0) if released is not None else 0, rows, width, int(block_size), view.data_ptr(),
        view.stride(0), view_lens.data_ptr(), _ptr(mask_out), mask_out.stride(0) if mask_out is not None else 0,
        base, size, _lib.current_stream(),
    )
    _lib.check(rc, "ekv_view_build_sum_budget")
    return view, view_lens


def compact_block_table(
    table: torch.Tensor, seq_lens: torch.Tensor, keep: torch.Tensor, block_size: int
) -> tuple[torch.Tensor, torch.Tensor]:
    """The view of each row that keeps the blocks marked in ``keep`` (reference block_view.py:36-56).

    ``table`` int32 [rows, width], ``seq_lens`` int32 [rows], ``keep`` bool [rows, width], all CUDA.
    Block 0 and the last block of each request are always kept; kept blocks stay in order and come
    first, the other positions follow in order; the view length is the kept blocks times
    ``block_size`` less the unfilled part of the last block (0 for a row with no tokens).
    """
    if keep.shape != table.shape:
        raise ValueError(f"keep shape {tuple(keep.shape)} != table shape {tuple(table.shape)}")
    return _view_build(table, seq_lens, block_size, keep=keep)


def plan_view(
    table: torch.Tensor,
    seq_lens: torch.Tensor,
    block_size: int,
    row_blocks: torch.Tensor,
    *,
    scores: torch.Tensor | None,
    policy: str = "uniform",
    budget_fraction: float | None = None,
    row_fraction: torch.Tensor | None = None,
    recent_blocks: int = 4,
    cap_above_blocks: int = 0,
    measured: torch.Tensor | None = None,
    released: torch.Tensor | None = None,
    full_rows: torch.Tensor | None = None,
    mask_out: torch.Tensor | None = None,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
    weights: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Decide and compact: the controller's quotas, then pins + top-k + compaction.

    ``row_blocks`` int32 [rows]: each request's length in blocks at the decision (0 = no request).
    Rows at or below ``cap_above_blocks`` read in full. With ``budget_fraction`` the measured rows
    share the budget max(pins, ceil(fraction * blocks)) (controller.py:398-451), split by uniform
    quotas, or under ``sum`` by the global greedy over the weighted shares (``weights`` float64
    [rows], None for 1.0; with float32 scores a row of weight 0 must pass zero scores); with
    ``row_fraction`` (float64 [rows]) each row is its own allocate() call. ``policy`` "uniform"/"sum"
    ranks by ``scores`` (float32 [rows, width], the device shares, or float64: the smoothed shares),
    "newest" keeps the newest blocks (the daemon's recency rule). ``mask_out`` receives the mask the
    controller commits.
    """
    if (budget_fraction is None) == (row_fraction is None):
        raise ValueError("give a shared budget fraction or per-row fractions, not both and not neither")
    rows = int(table.shape[0])
    if row_fraction is not None and (scores is None or scores.dtype == torch.float32) and policy in ("sum", "uniform", "newest"):
        # per-row budgets: the quotas and the view in one kernel
        if table.dtype != torch.int32 or seq_lens.dtype != torch.int32 or table.stride(1) != 1:
            raise ValueError("the block table (rows contiguous) and the lengths must be int32")
        if policy != "newest" and scores is None:
            raise ValueError(f"the {policy} objective ranks by scores")
        width = int(table.shape[1])
        view, view_lens = out if out is not None else (
            torch.empty(rows, width, dtype=torch.int32, device=table.device),
            torch.empty(rows, dtype=torch.int32, device=table.device),
        )
        if rows == 0:
            return view, view_lens
        rc = _lib.load().ekv_view_build_fractions(
            table.data_ptr(), table.stride(0), seq_lens.data_ptr(), row_blocks.data_ptr(), row_fraction.data_ptr(),
            _ptr(measured), int(recent_blocks), int(cap_above_blocks), _ptr(scores),
            scores.stride(0) if scores is not None else 0, _POLICIES[policy], _ptr(full_rows), _ptr(released),
            released.stride(0) if released is not None else 0, rows, width, int(block_size), view.data_ptr(),
            view.stride(0), view_lens.data_ptr(), _ptr(mask_out), mask_out.stride(0) if mask_out is not None else 0,
            _lib.current_stream(),
        )
        _lib.check(rc, "ekv_view_build_fractions")
        return view, view_lens
    quota = torch.empty(rows, dtype=torch.int32, device=table.device)
    objective = _POLICIES[policy]
    if policy == "sum" and budget_fraction is not None:
        # one budget over every measured row: the global greedy of the controller's default objective
        if scores is None:
            raise ValueError("the sum objective ranks by scores")
        if _sum_budget_fits(table, seq_lens, scores):
            return _sum_budget_view(table, seq_lens, block_size, row_blocks, scores, float(budget_fraction),
                                    recent_blocks, cap_above_blocks, measured, weights, released, full_rows,
                                    mask_out, out)
        from ..observe.allocation import sum_quotas

        sum_quotas(scores, row_blocks, quota, measured=measured, recent_blocks=recent_blocks,
                   cap_above_blocks=cap_above_blocks, budget_fraction=float(budget_fraction), weights=weights)
    elif policy == "maxmin" and budget_fraction is not None:
        # one budget: raise the lowest retained share first (allocation.py:121-166)
        if scores is None:
            raise ValueError("the maxmin objective ranks by scores")
        from ..observe.allocation import maxmin_quotas

        maxmin_quotas(scores, row_blocks, quota, measured=measured, recent_blocks=recent_blocks,
                      cap_above_blocks=cap_above_blocks, budget_fraction=float(budget_fraction))
    else:
        rc = _lib.load().ekv_allocate_quotas(
            row_blocks.data_ptr(), _ptr(measured), int(recent_blocks), int(cap_above_blocks),
            float(budget_fraction or 0.0), -1, _ptr(row_fraction), objective, rows, int(table.shape[1]),
            quota.data_ptr(), _lib.current_stream(),
        )
        _lib.check(rc, "ekv_allocate_quotas")
    return _view_build(
        table, seq_lens, block_size, row_blocks=row_blocks, quota=quota, measured=measured,
        recent_blocks=recent_blocks, scores=scores, policy=policy, released=released, full_rows=full_rows,
        mask_out=mask_out, out=out, weights=weights,
    )


# One host record per scheduler row: the fields the scheduler-facing decisions read and the controller's
# writes change (audit: the row's next decode step is an audit; audited: its request has had a completed
# audit; blocks: the request's length in blocks at that audit).
_ROW = np.dtype([("audit", "?"), ("audited", "?"), ("blocks", "<i8")])


class DecodeView:
    """The committed read policy of one serving process, and the view it gives each decode batch.

    The reference's contract (runtime/block_view.py:59-401): the controller's generations arrive through
    the ``write_*`` methods; an expired or never-committed lease gives the identity view; a row asked to
    audit reads in full for one decode step, which consumes the request; prefill rows read in full;
    released blocks are never read.

    State lives where it is used. The committed mask and the released blocks are device tensors (one
    ``[2, rows + 2, width]`` uint8 tensor: plane 0 the policy, plane 1 the released blocks, and two spare
    rows holding a fresh row's values): a commit is one asynchronous copy, a reassignment of rows one
    gather on the device, and ``build`` reads them in place in one ``ekv_decode_view`` launch into
    fixed-address view buffers (CUDA-graph safe). The per-row flags the host decides with (audit
    requests, completed audits and their lengths) are one host record array whose fields are the public
    ``audit_rows``, ``row_audited`` and ``audited_blocks``. ``keep`` and ``released`` read the device state
    back as host arrays (and assigning them writes it). The device is the current CUDA device, or
    ``device``; without one the writes still work and ``build`` raises.
    """

    def __init__(
        self,
        rows: int,
        width: int,
        block_size: int,
        audit: StatisticSwitch | None = None,
        prefill_audit: bool = False,
        *,
        device: torch.device | None = None,
    ) -> None:
        if min(rows, width, block_size) <= 0:
            raise ValueError("view dimensions must be positive")
        if prefill_audit and audit is None:
            raise ValueError("an audit in the last prefill step needs an audit plane")
        self.rows, self.width, self.block_size = rows, width, block_size
        self.audit = audit
        self.prefill_audit = prefill_audit
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        self.device = device
        self._records = np.zeros(rows + 2, dtype=_ROW)  # the two spares: a new request's row, an empty row
        self.audit_rows = self._records["audit"][:rows]
        self.row_audited = self._records["audited"][:rows]
        self.audited_blocks = self._records["blocks"][:rows]
        self.final_prefill = np.zeros(rows, dtype=bool)  # rows computing their prompt's last tokens next step
        self.last_audit_rows = np.zeros(rows, dtype=bool)  # rows read in full at the last completed audit
        self._masks = torch.zeros(2, rows + 2, width, dtype=torch.uint8, device=device)
        self._masks[0] = 1  # no commit yet: every block
        self._any_released = False
        self.version = 0
        self.released_version = 0
        self.deadline_ns = 0
        self.audit_step = False
        self.audits_started = 0
        self.audits_completed = 0
        # hooks of the serving integration: before a build, when an audit starts, whether one may start, and
        # when an audit step serves a prefilling row (the plane's check)
        self.before_build: Callable[[], None] | None = None
        self.on_audit_start: Callable[[], None] | None = None
        self.audit_gate: Callable[[], bool] | None = None
        self.on_prefill_audit: Callable[[], None] | None = None
        # the audit step in flight: its rows, and the lengths in blocks it read them at (device or host)
        self._audit_pending = False
        self._pending_rows = np.zeros(rows, dtype=bool)
        self._pending_blocks: torch.Tensor | np.ndarray | None = None
        self._counts = torch.zeros(5, dtype=torch.int64, device=device)
        self._table: torch.Tensor | None = None
        self._lens: torch.Tensor | None = None
        self._flag_ring: list[torch.Tensor] | None = None
        self._flag_slot = 0

    # -- the device state, read back and written as host arrays ------------------------------------

    @property
    def keep(self) -> np.ndarray:
        """The committed mask, bool [rows, width] (a copy read from the device)."""
        return self._masks[0, : self.rows].cpu().numpy().astype(bool)

    @keep.setter
    def keep(self, mask: np.ndarray) -> None:
        self._upload(0, np.asarray(mask) != 0)

    @property
    def released(self) -> np.ndarray:
        """The released blocks, bool [rows, width] (a copy read from the device)."""
        return self._masks[1, : self.rows].cpu().numpy().astype(bool)

    @released.setter
    def released(self, mask: np.ndarray) -> None:
        mask = np.asarray(mask) != 0
        self._upload(1, mask)
        self._any_released = bool(mask.any())
        self.released_version += 1

    def _upload(self, plane: int, mask: np.ndarray) -> None:
        if mask.shape != (self.rows, self.width):
            raise ValueError(f"mask shape {mask.shape} != view shape {(self.rows, self.width)}")
        host = torch.from_numpy(mask.astype(np.uint8))
        if self.device.type == "cuda":
            host = host.pin_memory()
        self._masks[plane, : self.rows].copy_(host, non_blocking=True)

    # -- the controller-facing writes ------------------------------------------------------------

    def write_row_controls(self, mask: np.ndarray, log_weight: np.ndarray | None = None) -> int:
        """Commit one generation: ``mask[row, block]`` nonzero means read that block."""
        if log_weight is not None:
            raise ValueError("a block-table view enforces hard keep decisions only")
        self.keep = mask
        self.version += 1
        return 1

    def write_lease_deadline(self, deadline_ns: int) -> int:
        self.deadline_ns = int(deadline_ns)
        return 1

    def write_audit_rows(self, requested: np.ndarray) -> int:
        """Ask for an audit of the marked rows; each request is consumed by one decode step."""
        requested = np.asarray(requested, dtype=bool)
        if requested.shape != (self.rows,):
            raise ValueError(f"audit shape {requested.shape} != {(self.rows,)}")
        if self.audit is None and requested.any():
            raise ValueError("an audit was requested but the view has no audit plane to switch the statistic on")
        np.logical_or(self.audit_rows, requested, out=self.audit_rows)
        return 1

    def write_final_prefill(self, rows: np.ndarray) -> None:
        """Mark the rows that compute the last tokens of their prompt in the next step (that step only)."""
        rows = np.asarray(rows, dtype=bool)
        if len(rows) > self.rows:
            raise ValueError(f"{len(rows)} rows exceed the view's {self.rows}")
        self.final_prefill.fill(False)
        self.final_prefill[: len(rows)] = rows

    def write_release(self, mask: np.ndarray) -> list[tuple[int, int]]:
        """Release the marked blocks a completed audit of the row's request covered, except block 0 and the
        request's last block at that audit; returns the (row, block) pairs released now."""
        mask = np.asarray(mask) != 0
        if mask.shape != (self.rows, self.width):
            raise ValueError(f"release shape {mask.shape} != view shape {(self.rows, self.width)}")
        # the covered blocks of a row: [1, blocks - 1) once its request has had an audit
        covered_end = np.where(self.row_audited, np.maximum(self.audited_blocks - 1, 0), 0)
        if not covered_end.any() or not mask.any():
            return []
        dev = self.device
        pos = torch.arange(self.width, device=dev)
        covered = (pos[None, :] >= 1) & (pos[None, :] < torch.from_numpy(covered_end).to(dev)[:, None])
        freed = self._masks[1, : self.rows]
        fresh = torch.from_numpy(mask).to(dev) & covered & (freed == 0)
        pairs = fresh.nonzero().cpu().tolist()
        if pairs:
            freed |= fresh.to(torch.uint8)
            self._any_released = True
            self.released_version += 1
        return [(int(r), int(b)) for r, b in pairs]

    def reassign_rows(self, moved: dict[int, int], new: list[int], empty: list[int]) -> None:
        """The scheduler changed which request each row holds (reference :166-199): a moved request takes its
        row's state along, a new one starts with full reads (and, with an audit plane, an audit at its first
        decode step), an empty row holds nothing. One gather of the host records and one of the device
        masks, from a source row per row (the two spares give the fresh rows)."""
        spare_new, spare_empty = self.rows, self.rows + 1
        source = np.arange(self.rows)
        if moved:
            source[np.fromiter(moved.keys(), dtype=np.int64)] = np.fromiter(moved.values(), dtype=np.int64)
        source[np.asarray(new, dtype=np.int64)] = spare_new
        source[np.asarray(empty, dtype=np.int64)] = spare_empty
        self._records[spare_new] = (self.audit is not None, False, 0)
        self._records[spare_empty] = (False, False, 0)
        self._records[: self.rows] = self._records[source]
        # the spare device rows hold a fresh row: every block kept, none released
        self._masks[0, self.rows :] = 1
        self._masks[1, self.rows :] = 0
        self._masks[:, : self.rows] = self._masks[:, torch.from_numpy(source).to(self.device)]
        if self._any_released:
            self.released_version += 1
        self.version += 1

    # -- the engine-facing view -----------------------------------------------------------------

    def active(self) -> bool:
        return self.deadline_ns > time.monotonic_ns()

    def _begin_step(self, servable: np.ndarray, decode: np.ndarray | None) -> np.ndarray:
        """The rows this step audits, out of the first ``len(servable)``: requested and servable, when the gate
        allows an audit now. Their requests are consumed, the step is marked and published as started."""
        n = len(servable)
        audited = np.zeros(self.rows, dtype=bool)
        np.logical_and(self.audit_rows[:n], servable, out=audited[:n])
        if audited.any() and not self.may_audit():
            audited.fill(False)  # the requests wait for a step after the controller has read the last audit
        if decode is not None and self.on_prefill_audit is not None and (audited[:n] & ~decode).any():
            self.on_prefill_audit()
        self.audit_rows[audited] = False
        self.audit_step = bool(audited.any())
        self._audit_pending = self.audit_step
        self._pending_rows = audited
        if self.audit_step:
            self.start_audit()
        return audited

    def build(
        self, table: torch.Tensor, seq_lens: torch.Tensor, query_lens: torch.Tensor
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """The view buffers (table, lengths) for a batch of ``len(query_lens)`` rows (reference :225-295).

        ``query_lens`` (host) is the tokens each row computes: one token decodes and gets the view; more is a
        prefill, which reads in full. The lease is read once, first; the keep algebra, the compaction and
        the read counters then run in one kernel with no host synchronisation."""
        if self.before_build is not None:
            self.before_build()
        live = self.active()
        self.finish_audit()
        n = len(query_lens)
        if table.shape[1] != self.width or n > self.rows:
            raise ValueError(f"batch ({n} rows, {table.shape[1]} blocks) exceeds view ({self.rows}, {self.width})")
        if table.device != self.device or self.device.type != "cuda":
            raise RuntimeError(f"the view builds on its CUDA device {self.device}; the batch is on {table.device}")
        t = table[:n]
        if t.dtype != torch.int32 or seq_lens.dtype != torch.int32 or t.stride(1) != 1:
            raise ValueError("the block table (rows contiguous) and the lengths must be int32")
        if self._table is None:
            self._table = torch.zeros(self.rows, self.width, dtype=torch.int32, device=self.device)
            self._lens = torch.zeros(self.rows, dtype=torch.int32, device=self.device)
        decode = query_lens.numpy() == 1
        servable = decode | (self.final_prefill[:n] & self.prefill_audit)
        self.final_prefill.fill(False)
        audited = self._begin_step(servable, decode)
        if self.audit_step:  # each audited request's length in blocks, kept on the device until the step ends
            self._pending_blocks = (seq_lens[:n].long() + self.block_size - 1) // self.block_size
        # one flag byte per row for the kernel: reads every block (no live lease, audited, prefilling), decodes,
        # audited
        full = ~decode | audited[:n] if live else np.ones(n, dtype=bool)
        flags = full.astype(np.uint8) | (decode.astype(np.uint8) << 1) | (audited[:n].astype(np.uint8) << 2)
        row_flags = self._flags_on(flags)
        if self.audit is not None:
            starts = np.zeros(n, dtype=np.int64)
            np.cumsum(query_lens.numpy()[:-1], out=starts[1:])
            self.audit.select(audited[:n], starts)
            self.audit.set(self.audit_step)
        keep, freed = self._masks[0, :n], self._masks[1, :n]
        rc = _lib.load().ekv_decode_view(
            t.data_ptr(), t.stride(0), seq_lens.data_ptr(), keep.data_ptr(), keep.stride(0), row_flags.data_ptr(),
            freed.data_ptr() if self._any_released else None, freed.stride(0), int(not live), n, self.width,
            self.block_size, self._table.data_ptr(), self._table.stride(0), self._lens.data_ptr(),
            self._counts.data_ptr(), _lib.current_stream(),
        )
        _lib.check(rc, "ekv_decode_view")
        return self._table[:n], self._lens[:n]

    def _flags_on(self, flags: np.ndarray) -> torch.Tensor:
        """The row flags on the device, through a ring of pinned buffers: no copy waits for the device."""
        if self._flag_ring is None:
            self._flag_ring = [torch.empty(self.rows, dtype=torch.uint8).pin_memory() for _ in range(4)]
            self._flag_done: list[torch.cuda.Event | None] = [None] * 4
            self._flags_dev = torch.zeros(self.rows, dtype=torch.uint8, device=self.device)
        slot = self._flag_slot = (self._flag_slot + 1) % len(self._flag_ring)
        if self._flag_done[slot] is not None:
            self._flag_done[slot].synchronize()  # its copy four steps ago has long finished
        self._flag_ring[slot].numpy()[: len(flags)] = flags
        self._flags_dev[: len(flags)].copy_(self._flag_ring[slot][: len(flags)], non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self._flag_done[slot] = done
        return self._flags_dev

    @property
    def buffers(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self._table is None or self._lens is None:
            raise RuntimeError("the view has built no batch yet")
        return self._table, self._lens

    def reads(self) -> tuple[int, int]:
        read, full = self._counts[:2].tolist()
        return int(read), int(full)

    def read_breakdown(self) -> dict[str, int]:
        names = ("read", "full", "audit", "untrimmed", "expired")
        return {name: int(x) for name, x in zip(names, self._counts.tolist(), strict=True)}

    def skip(self, seq_lens: torch.Tensor, query_lens: torch.Tensor) -> None:
        """A shared-prefix batch reads the engine's own table and records nothing; its decode rows count as
        full reads read with a live policy and no evidence."""
        self.finish_audit()
        self.audit_step = False
        if self.audit is not None:
            self.audit.set(False)
        n = len(query_lens)
        decoding = torch.from_numpy(query_lens.numpy() == 1).to(seq_lens.device)
        blocks = ((seq_lens[:n].long() + self.block_size - 1) // self.block_size * decoding).sum()
        zero = torch.zeros((), dtype=torch.int64, device=blocks.device)
        self._counts += torch.stack([blocks, blocks, zero, blocks, zero]).to(self._counts.device)

    def may_audit(self) -> bool:
        return self.audit_gate is None or self.audit_gate()

    def start_audit(self) -> None:
        self.audits_started += 1
        if self.on_audit_start is not None:
            self.on_audit_start()

    def finish_audit(self) -> None:
        """Count the step before as a completed audit, once the work queued for it on this stream has run: its
        statistic is then complete (an audit step's only wait). Runs before rows are reassigned."""
        if not self._audit_pending:
            return
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        blocks = self._pending_blocks
        if isinstance(blocks, torch.Tensor):
            blocks = blocks.cpu().numpy()  # already computed: the wait above covers it
        rows = self._pending_rows
        self.last_audit_rows = rows
        self.row_audited[rows] = True
        k = len(blocks)  # the audited rows are rows of that batch
        self.audited_blocks[:k][rows[:k]] = np.asarray(blocks)[rows[:k]]
        self.audits_completed += 1
        self._audit_pending = False


# -- vLLM integration: the reference's patch targets (runtime/block_view.py:404-626) -------------------------
#
# The process's view and audit plane are made by its first attention batch (the engine's own row count,
# table width and block size), so the CUDA graphs vLLM captures then read the view's fixed buffers.

_view: DecodeView | None = None
_plane: AuditPlane | None = None
_layers: tuple[str, ...] = ()  # the attention layers of the one KV-cache group the view serves


def _enabled(name: str) -> bool:
    return os.environ.get(name, "") not in ("", "0", "false")


def _refusals(builder):
    """Why the view cannot trim this cache group exactly, first reason first (nothing for plain full causal
    decoder attention over one cache group): the cache spec, then each layer."""
    from vllm.v1.attention.backend import AttentionType
    from vllm.v1.kv_cache_interface import FullAttentionSpec

    spec = builder.kv_cache_spec
    if type(spec) is not FullAttentionSpec:
        yield f"the view supports full causal attention only; this cache group is {type(spec).__name__}"
    elif spec.sliding_window is not None or spec.attention_chunk_size is not None:
        yield "the view does not support a sliding window or chunked attention in a cache group"
    context = builder.vllm_config.compilation_config.static_forward_context
    for name in builder.layer_names:
        layer = context[name]
        if layer.sliding_window is not None:
            yield f"layer {name} has a sliding window: the view cannot trim its blocks exactly"
        elif getattr(layer.impl, "alibi_slopes", None) is not None:
            yield f"layer {name} has a position bias (ALiBi): the view cannot trim its blocks"
        elif layer.attn_type != AttentionType.DECODER:
            yield f"layer {name} is {layer.attn_type.value} attention: the view supports decoder attention"


def require_supported_attention(builder) -> None:
    """Raise RuntimeError with the first reason the view cannot serve this cache group (reference :436-469):
    a cache spec other than plain full attention, or a layer with a sliding window, a position bias or
    attention other than decoder self-attention."""
    reason = next(_refusals(builder), None)
    if reason is not None:
        raise RuntimeError(reason)


def _audit_plane(builder, batch) -> AuditPlane | None:
    """The plane that records the statistic: the audit kernel's (EKV_AUDIT_KERNEL), or none. The reference's
    other recorder, its Triton compiler pass (EKV_ATTN_SHARE), has no counterpart here: asking for it is an
    error."""
    if _enabled("EKV_ATTN_SHARE"):
        raise RuntimeError("EKV_ATTN_SHARE needs the Triton compiler pass; this build records with EKV_AUDIT_KERNEL")
    if not _enabled("EKV_AUDIT_KERNEL"):
        return None
    from .audit_kernel import RecordingPlane

    config = builder.vllm_config
    model, parallel = config.model_config, config.parallel_config
    return RecordingPlane(
        layers=model.get_num_layers_by_block_type(parallel, "attention"),
        rows=config.scheduler_config.max_num_seqs,
        width=batch.block_table_tensor.shape[1],
        group_rows=model.get_num_attention_heads(parallel) // model.get_num_kv_heads(parallel),
        block_size=builder.kv_cache_spec.block_size,
    )


def _view_for(builder, batch) -> DecodeView:
    """The process's view, made by the first batch; a second KV-cache group is refused."""
    global _view, _plane, _layers
    names = tuple(builder.layer_names)
    if _view is None:
        require_supported_attention(builder)
        if _enabled("EKV_PREFILL_AUDIT"):
            raise RuntimeError("EKV_PREFILL_AUDIT needs the compiler pass's statistic (EKV_ATTN_SHARE)")
        plane = _audit_plane(builder, batch)
        _view = DecodeView(
            rows=builder.vllm_config.scheduler_config.max_num_seqs,
            width=batch.block_table_tensor.shape[1],
            block_size=builder.kv_cache_spec.block_size,
            audit=plane,
        )
        _plane, _layers = plane, names
    elif names != _layers:
        raise RuntimeError("a block-table view supports one KV-cache group; this model has several")
    return _view


def _query_lens(batch) -> torch.Tensor:
    """Tokens each row computes this step, from the host copy of the batch's query offsets."""
    return torch.diff(batch.query_start_loc_cpu[: batch.num_reqs + 1])


def _patch(cls, name: str, marker: str, wrap: Callable) -> bool:
    """Replace ``cls.name`` by ``wrap(original)`` once, tagging the replacement with ``marker``."""
    original = getattr(cls, name)
    if getattr(original, marker, False):
        return False
    replacement = wrap(original)
    setattr(replacement, marker, True)
    setattr(cls, name, replacement)
    return True


def _viewed_triton_build(original):
    """Triton's builder takes the batch as it is; its metadata's table and lengths are then the view's."""

    def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        metadata = original(self, common_prefix_len, common_attn_metadata, fast_build)
        batch = common_attn_metadata
        view = _view_for(self, batch)
        if common_prefix_len > 0:  # a shared-prefix cascade reads the engine's own table
            view.skip(batch.seq_lens, _query_lens(batch))
        else:
            metadata.block_table, metadata.seq_lens = view.build(batch.block_table_tensor, batch.seq_lens,
                                                                 _query_lens(batch))
        return metadata

    return build


def _viewed_flashinfer_build(original):
    """FlashInfer's builder plans its launch on the host from the lengths, so it is given the view's table
    and lengths as the batch."""

    def build(self, common_prefix_len, common_attn_metadata, fast_build=False):
        batch = common_attn_metadata
        view = _view_for(self, batch)
        if common_prefix_len > 0:
            view.skip(batch.seq_lens, _query_lens(batch))
            return original(self, common_prefix_len, batch, fast_build)
        table, lens = view.build(batch.block_table_tensor, batch.seq_lens, _query_lens(batch))
        viewed = batch.replace(block_table_tensor=table, seq_lens=lens, max_seq_len=int(lens.max()), _seq_lens_cpu=None)
        return original(self, common_prefix_len, viewed, fast_build)

    return build


def install_decode_view() -> int:
    """Give every attention batch of vLLM's Triton and FlashInfer backends its view, before the engine is
    created (reference :504-560). Returns the builders patched now."""
    from vllm.v1.attention.backends.flashinfer import FlashInferMetadataBuilder
    from vllm.v1.attention.backends.triton_attn import TritonAttentionMetadataBuilder

    targets = ((TritonAttentionMetadataBuilder, _viewed_triton_build),
               (FlashInferMetadataBuilder, _viewed_flashinfer_build))
    return sum(_patch(cls, "build", "_ekv_decode_view", wrap) for cls, wrap in targets)


def _recording_forward(original):
    """After the layer's attention, the audit kernel records it from the view's buffers (a profiling run,
    which has no batch, records nothing). The launch is the same every step: graphs capture it."""
    from .audit_kernel import RecordingPlane

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs):
        output = original(self, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs)
        if attn_metadata is not None:
            view = current_view()
            if not isinstance(view.audit, RecordingPlane):
                raise RuntimeError("the audit kernel is installed but the view has no recording plane")
            table, lens = view.buffers
            view.audit.record(layer.layer_name, table, lens, query, kv_cache, self.scale)
        return output

    return forward


def install_audit_kernel() -> int:
    """Record the statistic after each attention layer of vLLM's Triton and FlashInfer backends (reference
    :563-596), with EKV_AUDIT_KERNEL set, before the engine is created. Returns the implementations patched."""
    from vllm.v1.attention.backends.flashinfer import FlashInferImpl
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl

    return sum(_patch(impl, "forward", "_ekv_audit_kernel", _recording_forward)
               for impl in (TritonAttentionImpl, FlashInferImpl))


def current_view() -> DecodeView:
    if _view is None:
        raise RuntimeError("no attention batch has been built: install the decode view before the engine starts")
    return _view


def attach_audit_plane(runner) -> DecodeView:
    """The view, once the audit plane holds each layer's KV-cache address (reference :599-626): the audit
    kernel numbers layers by name, so its table follows its layer names; another plane takes the runner's
    caches in order."""
    from .audit_kernel import RecordingPlane

    view = current_view()
    if isinstance(_plane, RecordingPlane):
        context = runner.compilation_config.static_forward_context
        _plane.attach([context[name].kv_cache.data_ptr() for name in _plane.layer_names])
    elif _plane is not None:
        _plane.attach([cache.data_ptr() for cache in runner.kv_caches if cache is not None])
    return view
