"""The controller's decide stage on the device: ingest of the statistic, smoothing, and the keep mask.

The reference controller (observe/controller.py) copies the statistic of the audited rows out of the
serving process over IPC, one cudaMemcpy per (plane, layer, run of rows) (TileShareSource.read,
:111-136, with read_tile_rows, observe/tile_shares.py:129-173), normalises it with NumPy, folds it
into a float64 share vector per request key (Controller._absorb_audit, :332-345) and builds the keep
mask of every row with ``allocate`` (Controller._allocate, :398-451). Here the data stay on the GPU:

* ``DeviceShareSource`` opens the serving process's statistic table through the IPC handle its
  descriptor line publishes (the format RecordingPlane writes, runtime/audit_kernel.py:162-180) and
  returns the shares [live_rows, width] (float32, on the device) in one kernel (ekv_normalize_tile_lse).
* ``ShareLedger`` holds one float64 row per request (the reference's ``shares`` dict) and folds a new
  audit into it with ``ekv_ledger_absorb``: same evidence rule, same NaN handling, same rounding.
* ``ShareLedger.keep_mask`` computes the mask Controller._allocate commits, from the ledger in place
  (``ekv_allocate_sum_f64`` with the mask straight from its threshold, or ``ekv_allocate_quotas`` /
  ``ekv_allocate_maxmin_f64`` and ``ekv_view_build_f64``), bit-exact with the reference for the same
  shares; ``fixed_keep_mask`` does the same for a controller with a fixed scoring rule.

Only the request-key bookkeeping (which ledger row holds which request, which blocks the last audit
measured) stays on the host, as small dicts; the one host synchronisation per absorbed audit reads one
evidence byte per row. The mailbox, leases, audit requests, step-time target and block release are
the controller's control plane and are not rebuilt: ``keep_mask`` covers a controller with
``release_after`` = 0 and measured shares (no fixed scoring rule).
"""

from __future__ import annotations

import ctypes
import os
from collections.abc import Callable, Mapping, Sequence

import numpy as np
import torch

from .. import _lib
from ..runtime.audit import _cudart
from .allocation import Objective, maxmin_quotas, sum_quotas
from .tile_shares import _AGGREGATES, Aggregate, _check_aggregate

_TORCH_DTYPES = {np.dtype(np.int32): torch.int32, np.dtype(np.uint8): torch.uint8, np.dtype(np.float64): torch.float64}
_CUDA_IPC_LAZY_ENABLE_PEER_ACCESS = 1
_CUDA_MEMCPY_DEVICE_TO_HOST = 2


class _IpcMemHandle(ctypes.Structure):
    """cudaIpcMemHandle_t: 64 opaque bytes, passed by value to cudaIpcOpenMemHandle."""

    _fields_ = [("reserved", ctypes.c_ubyte * 64)]


def audit_row_blocks(audit_keys: np.ndarray, keys: np.ndarray, lengths: np.ndarray,
                     cap_above_blocks: int) -> tuple[int, np.ndarray]:
    """(live, row_blocks) of a completed audit (observe/controller.py:319-323): the rows up to the last
    audited one, each with its request's current length in blocks looked up by key (the batch may have
    been reordered since the audit), 0 for a request that has finished or is at or below the cap."""
    audit_keys = np.asarray(audit_keys, dtype=np.uint64)
    audited = np.flatnonzero(audit_keys)
    live = int(audited[-1]) + 1 if audited.size else 0
    current = {int(k): int(n) for k, n in zip(np.asarray(keys, dtype=np.uint64).tolist(), lengths) if int(k)}
    row_blocks = np.array([current.get(int(audit_keys[row]), 0) for row in range(live)], dtype=np.int64)
    row_blocks[row_blocks <= cap_above_blocks] = 0
    return live, row_blocks


class DeviceShareSource:
    """The attention share of the live rows, read on the device from a serving process's table.

    The device counterpart of TileShareSource (observe/controller.py:92-136): the same descriptor entry
    (``share_descriptor(pid)``) and the same ``read(live_rows, row_blocks)``, but the result is a float32
    tensor [live_rows, width] on this process's current device, NaN for rows without evidence (rows of 0
    blocks are not read). For the serving process itself the device addresses are used directly; another
    process opens the IPC handles once."""

    def __init__(self, entry: dict[str, int | str], pid: int, aggregate: Aggregate = "mean") -> None:
        _check_aggregate(aggregate)
        self.aggregate = aggregate
        self.rows = int(entry["max_rows"])
        self.width = int(entry["ncap"])
        self.group_rows = int(entry["tile_lse_group_rows"])
        self.max_layers = int(entry["tile_lse_layers"])
        self.tile_blocks = int(entry["attn_share_tile_blocks"])
        self._cuda = _cudart()
        self._opened: list[int] = []
        if pid == os.getpid():
            self.base = int(entry["tile_lse_dev"])
            self.table = int(entry["layer_table_dev"])
        else:
            self.base = self._open(str(entry["tile_lse_ipc"]))
            self.table = self._open(str(entry["layer_table_ipc"]))
        self.device = torch.device("cuda", torch.cuda.current_device())

    def _open(self, handle_hex: str) -> int:
        handle = _IpcMemHandle.from_buffer_copy(bytes.fromhex(handle_hex))
        pointer = ctypes.c_void_p()
        rc = self._cuda.cudaIpcOpenMemHandle(ctypes.byref(pointer), handle, ctypes.c_uint(_CUDA_IPC_LAZY_ENABLE_PEER_ACCESS))
        if rc != 0 or pointer.value is None:
            raise RuntimeError(f"cudaIpcOpenMemHandle failed with code {rc}")
        self._opened.append(pointer.value)
        return pointer.value

    def close(self) -> None:
        for address in self._opened:
            self._cuda.cudaIpcCloseMemHandle(ctypes.c_void_p(address))
        self._opened.clear()

    def layers(self) -> int:
        """The layers the serving process has filled in its layer table (reference :122-125)."""
        raw = (ctypes.c_uint64 * self.max_layers)()
        rc = self._cuda.cudaMemcpy(raw, ctypes.c_void_p(self.table), ctypes.c_size_t(self.max_layers * 8),
                                   _CUDA_MEMCPY_DEVICE_TO_HOST)
        if rc != 0:
            raise RuntimeError(f"cudaMemcpy of the layer table failed with code {rc}")
        return int(np.count_nonzero(np.frombuffer(raw, dtype=np.uint64)))

    def read(self, live_rows: int, row_blocks: np.ndarray) -> torch.Tensor:
        layers = self.layers()
        if layers == 0:
            raise RuntimeError("the layer table is empty: the serving process has not filled it")
        live = int(live_rows)
        out = torch.full((max(live, 0), self.width), float("nan"), dtype=torch.float32, device=self.device)
        if live <= 0:
            return out
        blocks = np.asarray(row_blocks)[:live].astype(np.int64)
        if not (blocks > 0).any():
            return out
        # rows of 0 blocks have no evidence: a row id outside the table makes the kernel write NaN
        ids = np.where(blocks > 0, np.arange(live), -1).astype(np.int32)
        ids_t = torch.from_numpy(ids).to(self.device)
        rb_t = torch.from_numpy(np.clip(blocks, -1, 2**31 - 1).astype(np.int32)).to(self.device)
        rc = _lib.load().ekv_normalize_tile_lse(
            self.base, self.max_layers, layers, self.rows, self.width, self.group_rows, ids_t.data_ptr(),
            rb_t.data_ptr(), live, self.tile_blocks, _AGGREGATES[self.aggregate], out.data_ptr(), None,
            _lib.current_stream(),
        )
        _lib.check(rc, "ekv_normalize_tile_lse")
        return out


def _to_device(device: torch.device, *arrays: np.ndarray) -> list[torch.Tensor]:
    """The arrays on the device through one pinned buffer and one asynchronous copy (8-byte aligned)."""
    offsets, total = [], 0
    for a in arrays:
        offsets.append(total)
        total += (a.nbytes + 7) // 8 * 8
    host = torch.empty(max(total, 8), dtype=torch.uint8, pin_memory=True)
    view = host.numpy()
    for a, o in zip(arrays, offsets, strict=True):
        view[o : o + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
    dev = host.to(device, non_blocking=True)
    return [dev[o : o + a.nbytes].view(_TORCH_DTYPES[a.dtype]) for a, o in zip(arrays, offsets, strict=True)]


def _check_weights(objective: str, weights: np.ndarray) -> None:
    if objective not in ("sum", "maxmin", "uniform"):
        raise ValueError(f"unknown objective {objective!r}")
    if objective != "sum" and np.any(weights != 1.0):
        raise ValueError(f"the {objective} objective does not use request weights")
    if objective == "sum" and (np.any(weights < 0.0) or not np.all(np.isfinite(weights))):
        raise RuntimeError("negative or non-finite request weights are not supported on the device")


def _committed_mask(scores: torch.Tensor, score_rows: torch.Tensor | None, row_blocks: torch.Tensor,
                    measured: torch.Tensor | None, weights: torch.Tensor, objective: str, budget_fraction: float,
                    recent_blocks: int, cap_above_blocks: int) -> torch.Tensor:
    """The keep mask uint8 [rows, width] of one budget over the rows' float64 scores (Controller._allocate)."""
    rows, width = int(row_blocks.shape[0]), int(scores.shape[1])
    dev = scores.device
    quota = torch.empty(rows, dtype=torch.int32, device=dev)
    mask = torch.empty(rows, width, dtype=torch.uint8, device=dev)
    if objective == "sum":  # the mask comes straight from the global threshold: no ranking per row
        sum_quotas(scores, row_blocks, quota, measured=measured, recent_blocks=recent_blocks,
                   cap_above_blocks=cap_above_blocks, budget_fraction=budget_fraction, weights=weights,
                   score_rows=score_rows, mask_out=mask)
        return mask
    lib = _lib.load()
    stream = _lib.current_stream()
    if objective == "maxmin":
        maxmin_quotas(scores, row_blocks, quota, measured=measured, recent_blocks=recent_blocks,
                      cap_above_blocks=cap_above_blocks, budget_fraction=budget_fraction, score_rows=score_rows)
    else:
        rc = lib.ekv_allocate_quotas(row_blocks.data_ptr(), None if measured is None else measured.data_ptr(),
                                     int(recent_blocks), int(cap_above_blocks), float(budget_fraction), -1, None,
                                     _lib.POLICY_UNIFORM, rows, width, quota.data_ptr(), stream)
        _lib.check(rc, "ekv_allocate_quotas")
    rc = lib.ekv_view_build_f64(
        None, 0, None, row_blocks.data_ptr(), quota.data_ptr(), None if measured is None else measured.data_ptr(),
        int(recent_blocks), scores.data_ptr(), scores.stride(0), None if score_rows is None else score_rows.data_ptr(),
        None, _lib.POLICY_UNIFORM, None, None, 0, rows, width, 16, None, 0, None, mask.data_ptr(), width, stream,
    )
    _lib.check(rc, "ekv_view_build_f64")
    return mask


def fixed_keep_mask(
    keys: np.ndarray,
    lengths: np.ndarray,
    scores_of: Callable[[int], np.ndarray],
    *,
    width: int,
    budget_fraction: float,
    objective: Objective = "sum",
    recent_blocks: int = 4,
    cap_above_blocks: int = 0,
    weight: Callable[[int], float] | None = None,
    device=None,
) -> torch.Tensor:
    """The keep mask uint8 [rows, width] of a controller with a fixed scoring rule instead of measured
    shares (observe/controller.py:148-160, :411-417): every row longer than ``cap_above_blocks`` with a
    request is one request of ``scores_of(n)`` scores (n = min(length, width)), pinned at block 0 and its
    newest ``recent_blocks`` + 1 blocks, under one budget max(pins, ceil(budget_fraction * blocks))."""
    if not 0.0 < budget_fraction <= 1.0:
        raise ValueError("the budget fraction must be in (0, 1]")
    keys = np.asarray(keys, dtype=np.uint64)
    lengths = np.asarray(lengths).astype(np.int64)
    rows = len(keys)
    chosen = (lengths > cap_above_blocks) & (keys != 0)
    scores = np.zeros((rows, width), dtype=np.float64)
    weights = np.ones(rows, dtype=np.float64)
    for r in np.flatnonzero(chosen).tolist():
        n = int(min(lengths[r], width))
        x = np.asarray(scores_of(n), dtype=np.float64)
        if x.shape != (n,):
            raise ValueError(f"the scoring rule gave {x.shape} scores for {n} blocks")
        scores[r, :n] = np.where(np.isnan(x), 0.0, x)
        if weight is not None:
            weights[r] = float(weight(int(keys[r])))
    _check_weights(objective, weights)
    row_blocks = np.where(chosen, np.minimum(lengths, 2**31 - 1), 0).astype(np.int32)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    sc_t, rb_t, w_t = _to_device(dev, scores, row_blocks, weights)
    return _committed_mask(sc_t.view(rows, width), None, rb_t, None, w_t, objective, budget_fraction,
                           recent_blocks, cap_above_blocks)


class _MeasuredView(Mapping):
    """request key -> blocks its latest audit covered (the reference's ``measured`` dict), read-only."""

    def __init__(self, ledger: "ShareLedger") -> None:
        self._ledger = ledger

    def __getitem__(self, key: int) -> int:
        return int(self._ledger._measured[self._ledger.slots[int(key)]])

    def __iter__(self):
        return iter(self._ledger.slots)

    def __len__(self) -> int:
        return len(self._ledger.slots)


class ShareLedger:
    """The smoothed float64 share of every block of every measured request, one device row per request.

    ``absorb`` is the fold of Controller._absorb_audit (observe/controller.py:332-345); ``slots`` and
    ``measured`` are the reference's ``shares`` keys (as ledger rows) and ``measured`` dict; ``forget``
    is the shares part of _forget_departed (:347-359); ``keep_mask`` is Controller._allocate's keep mask
    (:398-451) with no released blocks. The per-row bookkeeping is vectorised (a sorted key index, one
    pinned host-to-device copy per call), so a tick over a thousand requests costs launches, not Python."""

    def __init__(self, width: int, capacity: int = 256, *, share_decay: float = 0.5, device=None) -> None:
        if width <= 0 or capacity <= 0:
            raise ValueError("the ledger needs a positive width and capacity")
        if not 0.0 <= share_decay < 1.0:
            raise ValueError("invalid controller settings")
        self.width = int(width)
        self.decay = float(share_decay)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.table = torch.zeros(int(capacity), self.width, dtype=torch.float64, device=self.device)
        self.slots: dict[int, int] = {}  # request key -> ledger row
        self._measured = np.zeros(int(capacity), dtype=np.int64)  # ledger row -> blocks its audit covered
        self.measured = _MeasuredView(self)
        self._free = list(range(int(capacity) - 1, -1, -1))
        self._index: tuple[np.ndarray, np.ndarray] | None = None  # sorted keys and their rows
        self.evidence_version = 0

    # -- bookkeeping ---------------------------------------------------------------------------------

    def _take_slots(self, count: int) -> np.ndarray:
        while len(self._free) < count:  # grow: the rows keep their slots
            old = self.table.shape[0]
            grown = torch.zeros(2 * old, self.width, dtype=torch.float64, device=self.device)
            grown[:old].copy_(self.table)
            self.table = grown
            self._measured = np.concatenate([self._measured, np.zeros(old, dtype=np.int64)])
            self._free = list(range(2 * old - 1, old - 1, -1)) + self._free
        taken = self._free[len(self._free) - count:][::-1]
        del self._free[len(self._free) - count:]
        return np.asarray(taken, dtype=np.int32)

    def _slot_of(self, keys: np.ndarray) -> np.ndarray:
        """The ledger row of each key, -1 for key 0 and for keys without shares."""
        if self._index is None:
            k = np.fromiter(self.slots.keys(), dtype=np.uint64, count=len(self.slots))
            v = np.fromiter(self.slots.values(), dtype=np.int32, count=len(self.slots))
            order = np.argsort(k)
            self._index = (k[order], v[order])
        sorted_keys, rows = self._index
        if sorted_keys.size == 0:
            return np.full(len(keys), -1, dtype=np.int32)
        at = np.minimum(np.searchsorted(sorted_keys, keys), sorted_keys.size - 1)
        return np.where((sorted_keys[at] == keys) & (keys != 0), rows[at], -1).astype(np.int32)

    def __contains__(self, key: int) -> bool:
        return int(key) in self.slots

    def shares(self, key: int) -> np.ndarray:
        """The request's smoothed shares (float64 [width]), copied to the host."""
        return self.table[self.slots[int(key)]].cpu().numpy()

    def forget(self, present_keys: Sequence[int] | np.ndarray) -> None:
        """Drop the requests that are no longer in the batch (observe/controller.py:347-359)."""
        if not self.slots:
            return
        held = np.fromiter(self.slots.keys(), dtype=np.uint64, count=len(self.slots))
        gone = held[~np.isin(held, np.asarray(present_keys, dtype=np.uint64))]
        for key in gone.tolist():
            self._free.append(self.slots.pop(key))
        if gone.size:
            self._index = None

    # -- the fold of one audit -----------------------------------------------------------------------

    def absorb(self, fresh: torch.Tensor, audit_keys: np.ndarray, row_blocks: np.ndarray) -> list[int]:
        """Fold one audit's shares ``fresh`` [live, width] (float32 or float64, on the device; NaN without
        evidence) into the requests ``audit_keys[row]`` (0: no request). ``row_blocks[row]`` is the
        request's length in blocks, which becomes its ``measured`` count. Returns the keys that received
        evidence, in row order."""
        if fresh.ndim != 2 or fresh.shape[1] != self.width or not fresh.is_cuda:
            raise ValueError(f"fresh shares must be a device tensor [rows, {self.width}]")
        if fresh.dtype not in (torch.float32, torch.float64) or fresh.stride(1) != 1:
            raise ValueError("fresh shares must be float32 or float64 with contiguous rows")
        live = int(fresh.shape[0])
        keys = np.asarray(audit_keys, dtype=np.uint64)[:live]
        blocks = np.asarray(row_blocks)[:live].astype(np.int64)
        present = np.flatnonzero(keys)
        if present.size == 0:
            return []
        # a key met twice folds twice, in row order: rows are folded in rounds of first occurrences,
        # second occurrences, ...
        order = np.argsort(keys[present], kind="stable")
        sorted_keys = keys[present][order]
        first = np.ones(present.size, dtype=bool)
        first[1:] = sorted_keys[1:] != sorted_keys[:-1]
        group_start = np.maximum.accumulate(np.where(first, np.arange(present.size), 0))
        occurrence = np.empty(present.size, dtype=np.int64)
        occurrence[order] = np.arange(present.size) - group_start
        updated: list[np.ndarray] = []
        for k in range(int(occurrence.max()) + 1):
            rows = present[occurrence == k]
            updated.append(self._fold(fresh, live, keys, blocks, rows))
        got = np.sort(np.concatenate(updated))
        return keys[got].tolist()

    def _fold(self, fresh: torch.Tensor, live: int, keys: np.ndarray, blocks: np.ndarray, rows: np.ndarray) -> np.ndarray:
        """One kernel over the rows ``rows`` (distinct keys); returns the rows that had evidence."""
        slot = np.full(live, -1, dtype=np.int32)
        slot[rows] = self._slot_of(keys[rows])
        blend = (slot >= 0).astype(np.uint8)
        new = rows[slot[rows] < 0]
        if new.size:
            slot[new] = self._take_slots(new.size)
        slot_t, blend_t = _to_device(self.device, slot, blend)
        evidence = torch.empty(live, dtype=torch.uint8, device=self.device)
        rc = _lib.load().ekv_ledger_absorb(
            fresh.data_ptr(), int(fresh.dtype == torch.float64), fresh.stride(0), slot_t.data_ptr(),
            blend_t.data_ptr(), self.decay, live, self.width, self.table.data_ptr(), self.table.stride(0),
            self.table.shape[0], evidence.data_ptr(), _lib.current_stream(),
        )
        _lib.check(rc, "ekv_ledger_absorb")
        has = evidence.cpu().numpy().astype(bool)
        got = rows[has[rows]]
        if new.size:
            kept_new = new[has[new]]
            self._free.extend(slot[new[~has[new]]].tolist())
            for row in kept_new.tolist():
                self.slots[int(keys[row])] = int(slot[row])
            if kept_new.size:
                self._index = None
        self._measured[slot[got]] = blocks[got]
        self.evidence_version += int(got.size)
        return got

    # -- the committed keep mask ---------------------------------------------------------------------

    def keep_mask(
        self,
        keys: np.ndarray,
        lengths: np.ndarray,
        *,
        budget_fraction: float,
        objective: Objective = "sum",
        recent_blocks: int = 4,
        cap_above_blocks: int = 0,
        weight: Callable[[int], float] | None = None,
    ) -> torch.Tensor:
        """The keep mask uint8 [rows, width] (on the device) of Controller._allocate for the rows' request
        ``keys`` and ``lengths`` (blocks): measured rows (longer than ``cap_above_blocks``, with shares)
        keep their pins and their share of one budget, max(pins, ceil(budget_fraction * blocks)); every
        other row, and every position past a request's length, keeps all."""
        if objective not in ("sum", "maxmin", "uniform"):
            raise ValueError(f"unknown objective {objective!r}")
        if not 0.0 < budget_fraction <= 1.0:
            raise ValueError("the budget fraction must be in (0, 1]")
        keys = np.asarray(keys, dtype=np.uint64)
        lengths = np.asarray(lengths).astype(np.int64)
        rows = len(keys)
        slot = self._slot_of(keys)
        chosen = (lengths > cap_above_blocks) & (keys != 0) & (slot >= 0)
        big = 2**31 - 1
        row_blocks = np.where(chosen, np.minimum(lengths, big), 0).astype(np.int32)
        measured = np.where(chosen, np.minimum(self._measured[np.maximum(slot, 0)], big), 0).astype(np.int32)
        score_rows = np.where(chosen, slot, 0).astype(np.int32)
        weights = np.ones(rows, dtype=np.float64)
        if weight is not None:
            picked = np.flatnonzero(chosen)
            weights[picked] = [float(weight(k)) for k in keys[picked].tolist()]
        _check_weights(objective, weights)
        rb_t, ms_t, sr_t, w_t = _to_device(self.device, row_blocks, measured, score_rows, weights)
        return _committed_mask(self.table, sr_t, rb_t, ms_t, w_t, objective, budget_fraction, recent_blocks,
                               cap_above_blocks)
