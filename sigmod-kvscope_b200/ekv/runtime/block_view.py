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


class DecodeView:
    """The committed read policy of one serving process, and the view it gives each decode batch.

    Same contract as the reference's DecodeView (block_view.py:59-401): the controller's
    generations arrive through the ``write_*`` methods; an expired or never-committed lease gives
    the identity view; a row asked to audit reads in full for one decode step, which consumes the
    request; prefill rows read in full; released blocks are never read. The keep algebra and the
    compaction run in one device kernel per step into fixed-address buffers (CUDA-graph safe).
    """

    def __init__(
        self,
        rows: int,
        width: int,
        block_size: int,
        audit: StatisticSwitch | None = None,
        prefill_audit: bool = False,
    ) -> None:
        if min(rows, width, block_size) <= 0:
            raise ValueError("view dimensions must be positive")
        if prefill_audit and audit is None:
            raise ValueError("an audit in the last prefill step needs an audit plane")
        self.rows, self.width, self.block_size = rows, width, block_size
        self.audit = audit
        self.prefill_audit = prefill_audit
        self.final_prefill = np.zeros(rows, dtype=bool)
        self.on_prefill_audit: Callable[[], None] | None = None
        self.keep = np.ones((rows, width), dtype=bool)
        self.released = np.zeros((rows, width), dtype=bool)
        self.released_version = 0
        self.row_audited = np.zeros(rows, dtype=bool)
        self.audited_blocks = np.zeros(rows, dtype=np.int64)
        self._pending_blocks = np.zeros(rows, dtype=np.int64)
        self.audit_rows = np.zeros(rows, dtype=bool)
        self.last_audit_rows = np.zeros(rows, dtype=bool)
        self.deadline_ns = 0
        self.version = 0
        self.audit_step = False
        self.audits_completed = 0
        self.audits_started = 0
        self.on_audit_start: Callable[[], None] | None = None
        self.audit_gate: Callable[[], bool] | None = None
        self.before_build: Callable[[], None] | None = None
        self._audit_pending = False
        self._pending_rows = np.zeros(rows, dtype=bool)
        self._counts: torch.Tensor | None = None
        self._flag_ring: list[torch.Tensor] | None = None
        self._flag_slot = 0
        self._device: torch.device | None = None
        self._device_keep: torch.Tensor | None = None
        self._device_version = -1
        self._device_released: torch.Tensor | None = None
        self._released_device_version = -1
        self._table: torch.Tensor | None = None
        self._lens: torch.Tensor | None = None

    # -- the controller-facing writes ------------------------------------------------------------

    def write_row_controls(self, mask: np.ndarray, log_weight: np.ndarray | None = None) -> int:
        """Commit one generation: ``mask[row, block]`` nonzero means read that block."""
        if log_weight is not None:
            raise ValueError("a block-table view enforces hard keep decisions only")
        mask = np.asarray(mask)
        if mask.shape != self.keep.shape:
            raise ValueError(f"mask shape {mask.shape} != view shape {self.keep.shape}")
        self.keep = mask != 0
        self.version += 1
        return 1

    def write_lease_deadline(self, deadline_ns: int) -> int:
        self.deadline_ns = int(deadline_ns)
        return 1

    def write_audit_rows(self, requested: np.ndarray) -> int:
        """Ask for an audit of the marked rows; each request is consumed by one decode step."""
        requested = np.asarray(requested, dtype=bool)
        if requested.shape != self.audit_rows.shape:
            raise ValueError(f"audit shape {requested.shape} != {self.audit_rows.shape}")
        if requested.any() and self.audit is None:
            raise ValueError("an audit was requested but the view has no audit plane to switch the statistic on")
        self.audit_rows |= requested
        return 1

    def write_final_prefill(self, rows: np.ndarray) -> None:
        rows = np.asarray(rows, dtype=bool)
        if rows.shape[0] > self.rows:
            raise ValueError(f"{rows.shape[0]} rows exceed the view's {self.rows}")
        self.final_prefill[:] = False
        self.final_prefill[: rows.shape[0]] = rows

    def write_release(self, mask: np.ndarray) -> list[tuple[int, int]]:
        """Mark blocks released; only blocks an audit of the row's request covered, never block 0 or
        the last block at that audit. Returns the new (row, block) pairs."""
        mask = np.asarray(mask) != 0
        if mask.shape != self.released.shape:
            raise ValueError(f"release shape {mask.shape} != view shape {self.released.shape}")
        eligible = np.zeros_like(mask)
        for row in np.flatnonzero(self.row_audited):
            eligible[row, : max(int(self.audited_blocks[row]) - 1, 0)] = True
        eligible[:, 0] = False
        new = mask & eligible & ~self.released
        rows, blocks = np.nonzero(new)
        if rows.size:
            self.released |= new
            self.released_version += 1
        return list(zip(rows.tolist(), blocks.tolist(), strict=True))

    def reassign_rows(self, moved: dict[int, int], new: list[int], empty: list[int]) -> None:
        """The scheduler changed which request each row holds (reference :166-199)."""
        keep, audit = self.keep.copy(), self.audit_rows.copy()
        released, audited, blocks = self.released.copy(), self.row_audited.copy(), self.audited_blocks.copy()
        for row, old in moved.items():
            keep[row], audit[row] = self.keep[old], self.audit_rows[old]
            released[row], audited[row], blocks[row] = self.released[old], self.row_audited[old], self.audited_blocks[old]
        for row in new:
            keep[row], audit[row] = True, self.audit is not None
            released[row], audited[row], blocks[row] = False, False, 0
        for row in empty:
            keep[row], audit[row] = True, False
            released[row], audited[row], blocks[row] = False, False, 0
        self.keep, self.audit_rows = keep, audit
        if (released != self.released).any():
            self.released_version += 1
        self.released, self.row_audited, self.audited_blocks = released, audited, blocks
        self.version += 1

    # -- the engine-facing view -----------------------------------------------------------------

    def active(self) -> bool:
        return self.deadline_ns > time.monotonic_ns()

    def build(
        self, table: torch.Tensor, seq_lens: torch.Tensor, query_lens: torch.Tensor
    ) -> tuple[torch.Tensor, torch.Tensor]:
        """The view buffers (table, lengths) for a batch of ``len(query_lens)`` rows (reference :225-295)."""
        if self.before_build is not None:
            self.before_build()
        live = self.active()
        self.finish_audit()
        self._device = table.device
        num_reqs = len(query_lens)
        width = table.shape[1]
        if width != self.width or num_reqs > self.rows:
            raise ValueError(f"batch ({num_reqs} rows, {width} blocks) exceeds view ({self.rows}, {self.width})")
        if self._table is None:
            self._table = torch.zeros(self.rows, width, dtype=torch.int32, device=table.device)
            self._lens = torch.zeros(self.rows, dtype=torch.int32, device=table.device)
        assert self._lens is not None
        decode = query_lens.numpy() == 1
        servable = decode | (self.final_prefill[:num_reqs] & self.prefill_audit)
        self.final_prefill[:] = False
        audited = np.zeros(self.rows, dtype=bool)
        audited[:num_reqs] = self.audit_rows[:num_reqs] & servable
        if audited.any() and not self.may_audit():
            audited[:] = False
        if (audited[:num_reqs] & ~decode).any() and self.on_prefill_audit is not None:
            self.on_prefill_audit()
        self.audit_rows[audited] = False
        self.audit_step = bool(audited.any())
        self._audit_pending = self.audit_step
        self._pending_rows = audited
        if self.audit_step:
            self.start_audit()
            size = self.block_size
            self._pending_blocks[:num_reqs] = ((seq_lens[:num_reqs] + size - 1) // size).cpu().numpy()
        # one flag byte per row: it reads every block (an expired lease, an audited row, a prefill row),
        # it decodes, it is audited; the view kernel applies them and counts the reads (:272-329)
        full = np.ones(num_reqs, dtype=bool) if not live else (audited[:num_reqs] | ~decode)
        flags = full.astype(np.uint8) | (decode.astype(np.uint8) << 1) | (audited[:num_reqs].astype(np.uint8) << 2)
        row_flags = self._flags_on(flags, table.device)
        keep = self._keep_on(table.device)[:num_reqs]
        released = self._released_on(table.device)[:num_reqs] if self.released.any() else None
        if self.audit is not None:
            starts = np.concatenate(([0], np.cumsum(query_lens.numpy())[:-1]))
            self.audit.select(audited[:num_reqs], starts)
            self.audit.set(self.audit_step)
        if self._counts is None:
            self._counts = torch.zeros(5, dtype=torch.int64, device=table.device)
        t = table[:num_reqs]
        if t.dtype != torch.int32 or seq_lens.dtype != torch.int32 or t.stride(1) != 1:
            raise ValueError("the block table (rows contiguous) and the lengths must be int32")
        rc = _lib.load().ekv_decode_view(
            t.data_ptr(), t.stride(0), seq_lens.data_ptr(), keep.data_ptr(), keep.stride(0), row_flags.data_ptr(),
            _ptr(released), 0 if released is None else released.stride(0), int(not live), num_reqs, width,
            self.block_size, self._table.data_ptr(), self._table.stride(0), self._lens.data_ptr(),
            self._counts.data_ptr(), _lib.current_stream(),
        )
        _lib.check(rc, "ekv_decode_view")
        return self._table[:num_reqs], self._lens[:num_reqs]

    def _flags_on(self, flags: np.ndarray, device: torch.device) -> torch.Tensor:
        """The row flags on the device, through a ring of pinned buffers: no copy waits for the device."""
        if self._flag_ring is None:
            self._flag_ring = [torch.empty(self.rows, dtype=torch.uint8).pin_memory() for _ in range(4)]
            self._flag_done: list[torch.cuda.Event | None] = [None] * 4
            self._flags_dev = torch.zeros(self.rows, dtype=torch.uint8, device=device)
        slot = self._flag_slot = (self._flag_slot + 1) % len(self._flag_ring)
        if self._flag_done[slot] is not None:
            self._flag_done[slot].synchronize()  # its copy four steps ago has long finished
        self._flag_ring[slot].numpy()[: len(flags)] = flags
        self._flags_dev[: len(flags)].copy_(self._flag_ring[slot][: len(flags)], non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self._flag_done[slot] = done
        return self._flags_dev

    def _count(self, read_lens, full_lens, decoding, audited=None, expired: bool = False) -> None:
        """Read counters of decode rows: read, full, audited, untrimmed-live, expired (reference :297-329)."""
        if self._counts is None:
            self._counts = torch.zeros(5, dtype=torch.int64, device=read_lens.device)
        size = self.block_size
        read = (read_lens.long() + size - 1) // size
        full = (full_lens.long() + size - 1) // size
        whole = read_lens == full_lens
        if decoding is not None:
            read, full = read * decoding, full * decoding
        in_audit = torch.zeros_like(whole) if audited is None else audited
        live_whole = whole & ~in_audit & (not expired)
        zero = torch.zeros((), dtype=torch.int64, device=read.device)
        self._counts += torch.stack(
            [read.sum(), full.sum(), (read * in_audit).sum(), (read * live_whole).sum(), read.sum() if expired else zero]
        )

    @property
    def buffers(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self._table is None or self._lens is None:
            raise RuntimeError("the view has built no batch yet")
        return self._table, self._lens

    def reads(self) -> tuple[int, int]:
        if self._counts is None:
            return 0, 0
        read, full = (int(x) for x in self._counts.tolist()[:2])
        return read, full

    def read_breakdown(self) -> dict[str, int]:
        names = ("read", "full", "audit", "untrimmed", "expired")
        if self._counts is None:
            return dict.fromkeys(names, 0)
        return dict(zip(names, (int(x) for x in self._counts.tolist()), strict=True))

    def skip(self, seq_lens: torch.Tensor, query_lens: torch.Tensor) -> None:
        """A shared-prefix batch reads the engine's own table; its decode rows count as full reads."""
        self.finish_audit()
        self.audit_step = False
        if self.audit is not None:
            self.audit.set(False)
        decoding = torch.from_numpy(query_lens.numpy() == 1).to(seq_lens.device)
        self._count(seq_lens[: len(query_lens)], seq_lens[: len(query_lens)], decoding)

    def may_audit(self) -> bool:
        return self.audit_gate is None or self.audit_gate()

    def start_audit(self) -> None:
        self.audits_started += 1
        if self.on_audit_start is not None:
            self.on_audit_start()

    def finish_audit(self) -> None:
        """Count the previous step as a completed audit once the device has finished it (one sync)."""
        if not self._audit_pending:
            return
        if self._device is not None and self._device.type == "cuda":
            torch.cuda.synchronize(self._device)
        self.last_audit_rows = self._pending_rows
        self.row_audited |= self._pending_rows
        self.audited_blocks[self._pending_rows] = self._pending_blocks[self._pending_rows]
        self.audits_completed += 1
        self._audit_pending = False

    def _keep_on(self, device: torch.device) -> torch.Tensor:
        if self._device_keep is None or self._device_version != self.version:
            self._device_keep = torch.from_numpy(self.keep.astype(np.uint8)).to(device, non_blocking=True)
            self._device_version = self.version
        return self._device_keep

    def _released_on(self, device: torch.device) -> torch.Tensor:
        if self._device_released is None or self._released_device_version != self.released_version:
            self._device_released = torch.from_numpy(self.released.astype(np.uint8)).to(device, non_blocking=True)
            self._released_device_version = self.released_version
        return self._device_released


# -- vLLM integration (the patch targets of the reference, block_view.py:404-626) ---------------------

_view: DecodeView | None = None
_plane: AuditPlane | None = None
_layers: tuple[str, ...] = ()


def _enabled(name: str) -> bool:
    return os.environ.get(name, "") not in ("", "0", "false")


def _audit_plane(builder, cam) -> AuditPlane | None:
    """The plane that records the statistic: the audit kernel's (EKV_AUDIT_KERNEL) or none.

    The reference's compiler pass (EKV_ATTN_SHARE) instruments Triton kernels; this build has no
    Triton path, so asking for it is an error."""
    if _enabled("EKV_ATTN_SHARE"):
        raise RuntimeError("EKV_ATTN_SHARE needs the Triton compiler pass; this build records with EKV_AUDIT_KERNEL")
    if _enabled("EKV_AUDIT_KERNEL"):
        from .audit_kernel import RecordingPlane

        model, parallel = builder.vllm_config.model_config, builder.vllm_config.parallel_config
        return RecordingPlane(
            layers=model.get_num_layers_by_block_type(parallel, "attention"),
            rows=builder.vllm_config.scheduler_config.max_num_seqs,
            width=cam.block_table_tensor.shape[1],
            group_rows=model.get_num_attention_heads(parallel) // model.get_num_kv_heads(parallel),
            block_size=builder.kv_cache_spec.block_size,
        )
    return None


def require_supported_attention(builder) -> None:
    """Refuse a cache group the view cannot trim exactly: anything but plain full causal attention
    over one cache group (reference :436-469)."""
    from vllm.v1.attention.backend import AttentionType
    from vllm.v1.kv_cache_interface import FullAttentionSpec

    spec = builder.kv_cache_spec
    if type(spec) is not FullAttentionSpec:
        raise RuntimeError(f"the view supports full causal attention only; this cache group is {type(spec).__name__}")
    if spec.sliding_window is not None or spec.attention_chunk_size is not None:
        raise RuntimeError("the view does not support a sliding window or chunked attention in a cache group")
    layers = builder.vllm_config.compilation_config.static_forward_context
    for name in builder.layer_names:
        layer = layers[name]
        if layer.sliding_window is not None:
            raise RuntimeError(f"layer {name} has a sliding window: the view cannot trim its blocks exactly")
        if getattr(layer.impl, "alibi_slopes", None) is not None:
            raise RuntimeError(f"layer {name} has a position bias (ALiBi): the view cannot trim its blocks")
        if layer.attn_type != AttentionType.DECODER:
            raise RuntimeError(f"layer {name} is {layer.attn_type.value} attention: the view supports decoder attention")


def _view_for(builder, cam) -> DecodeView:
    global _view, _plane, _layers
    layers = tuple(builder.layer_names)
    if _view is None:
        require_supported_attention(builder)
        _plane = _audit_plane(builder, cam)
        if _enabled("EKV_PREFILL_AUDIT"):
            raise RuntimeError("EKV_PREFILL_AUDIT needs the compiler pass's statistic (EKV_ATTN_SHARE)")
        _view = DecodeView(
            rows=builder.vllm_config.scheduler_config.max_num_seqs,
            width=cam.block_table_tensor.shape[1],
            block_size=builder.kv_cache_spec.block_size,
            audit=_plane,
        )
        _layers = layers
    if layers != _layers:
        raise RuntimeError("a block-table view supports one KV-cache group; this model has several")
    return _view


def _query_lens(cam) -> torch.Tensor:
    starts = cam.query_start_loc_cpu[: cam.num_reqs + 1]
    return starts[1:] - starts[:-1]


def install_decode_view() -> int:
    """Give every attention batch of the Triton and FlashInfer backends its view (reference :504-560)."""
    from vllm.v1.attention.backends.flashinfer import FlashInferMetadataBuilder
    from vllm.v1.attention.backends.triton_attn import TritonAttentionMetadataBuilder

    patched = 0
    triton_build = TritonAttentionMetadataBuilder.build
    if not getattr(triton_build, "_ekv_decode_view", False):

        def build_triton(self, common_prefix_len, common_attn_metadata, fast_build=False):
            metadata = triton_build(self, common_prefix_len, common_attn_metadata, fast_build)
            cam = common_attn_metadata
            view = _view_for(self, cam)
            if common_prefix_len > 0:
                view.skip(cam.seq_lens, _query_lens(cam))
                return metadata
            metadata.block_table, metadata.seq_lens = view.build(cam.block_table_tensor, cam.seq_lens, _query_lens(cam))
            return metadata

        build_triton._ekv_decode_view = True
        TritonAttentionMetadataBuilder.build = build_triton
        patched += 1
    flashinfer_build = FlashInferMetadataBuilder.build
    if not getattr(flashinfer_build, "_ekv_decode_view", False):

        def build_flashinfer(self, common_prefix_len, common_attn_metadata, fast_build=False):
            cam = common_attn_metadata
            view = _view_for(self, cam)
            if common_prefix_len > 0:
                view.skip(cam.seq_lens, _query_lens(cam))
                return flashinfer_build(self, common_prefix_len, cam, fast_build)
            table, lens = view.build(cam.block_table_tensor, cam.seq_lens, _query_lens(cam))
            seen = cam.replace(block_table_tensor=table, seq_lens=lens, max_seq_len=int(lens.max()), _seq_lens_cpu=None)
            return flashinfer_build(self, common_prefix_len, seen, fast_build)

        build_flashinfer._ekv_decode_view = True
        FlashInferMetadataBuilder.build = build_flashinfer
        patched += 1
    return patched


def install_audit_kernel() -> int:
    """After each attention layer of the Triton and FlashInfer backends, record the statistic
    (reference :563-596). The launch is the same every step, so CUDA graphs capture it."""
    from vllm.v1.attention.backends.flashinfer import FlashInferImpl
    from vllm.v1.attention.backends.triton_attn import TritonAttentionImpl

    from .audit_kernel import RecordingPlane

    patched = 0
    for impl in (TritonAttentionImpl, FlashInferImpl):
        original = impl.forward
        if getattr(original, "_ekv_audit_kernel", False):
            continue

        def forward(self, layer, query, key, value, kv_cache, attn_metadata, *args, _original=original, **kwargs):
            output = _original(self, layer, query, key, value, kv_cache, attn_metadata, *args, **kwargs)
            if attn_metadata is not None:
                view = current_view()
                if not isinstance(view.audit, RecordingPlane):
                    raise RuntimeError("the audit kernel is installed but the view has no recording plane")
                table, lens = view.buffers
                view.audit.record(layer.layer_name, table, lens, query, kv_cache, self.scale)
            return output

        forward._ekv_audit_kernel = True
        impl.forward = forward
        patched += 1
    return patched


def current_view() -> DecodeView:
    if _view is None:
        raise RuntimeError("no attention batch has been built: install the decode view before the engine starts")
    return _view


def attach_audit_plane(runner) -> DecodeView:
    """The view, with the audit plane given the engine's per-layer KV-cache addresses (reference :599-626)."""
    from .audit_kernel import RecordingPlane

    view = current_view()
    if isinstance(_plane, RecordingPlane):
        layers = runner.compilation_config.static_forward_context
        _plane.attach([layers[name].kv_cache.data_ptr() for name in _plane.layer_names])
    elif _plane is not None:
        _plane.attach([cache.data_ptr() for cache in runner.kv_caches if cache is not None])
    return view
