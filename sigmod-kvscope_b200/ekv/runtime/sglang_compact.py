"""The compaction of SGLang's key-value index list on the device, with no host synchronisation.

Interface of runtime/sglang_compact.py of the reference: ``COUNTS`` and ``SlotCompactor`` with its
``counts``, ``new_indptr``, ``lens`` and ``table`` buffers and its ``compact`` signature and meaning.
SGLang's decode kernel reads request ``r`` from ``slots[indptr[r]:indptr[r+1]]``, one token slot per
entry; the view groups ``block_tokens`` consecutive entries into a block and keeps some blocks (the
first and last always; all of them when the policy is not live, when the row is audited, and for the
rows a CUDA graph adds from ``n_real`` on). The work runs in the sm_100a kernels of
``ekv_slot_compact``: a warp per row, a scan of the new lengths, a gather of every new entry, and the
copy back into the engine's buffers.

The compactor's buffers are views of two arenas on the device, one of int32 (the new indptr, the new
lengths and the kept-block table) and one of slot entries (the gathered list); an arena is replaced by
one twice as large when a batch needs more, so a steady batch size allocates nothing.
"""

from __future__ import annotations

import torch

from .. import _lib

COUNTS = 5  # blocks read, blocks a full read would read, read in audits, read untrimmed, read without a live policy


class SlotCompactor:
    """The compaction of one serving process, with its buffers kept from batch to batch."""

    def __init__(self, width: int, block_tokens: int, device: torch.device) -> None:
        if width <= 0 or block_tokens <= 0:
            raise ValueError("width and block_tokens must be positive")
        self.width, self.block_tokens, self.device = width, block_tokens, device
        self.counts = torch.zeros(COUNTS, dtype=torch.int64, device=device)
        self._rows = 0  # rows the int32 arena holds
        self._ints = torch.empty(0, dtype=torch.int32, device=device)
        self._out = torch.empty(0, dtype=torch.int64, device=device)
        self._carve()

    def _carve(self) -> None:
        """new_indptr [rows + 1], lens [rows], table [rows, width] as views of the int32 arena."""
        rows = self._rows
        self.new_indptr = self._ints[: rows + 1] if rows else self._ints[:0]
        self.lens = self._ints[rows + 1 : 2 * rows + 1]
        self.table = self._ints[2 * rows + 1 :].view(rows, self.width)

    def _fit(self, rows: int, entries: int, dtype: torch.dtype) -> None:
        if rows > self._rows:
            self._rows = max(rows, 2 * self._rows)
            self._ints = torch.empty(2 * self._rows + 1 + self._rows * self.width, dtype=torch.int32,
                                     device=self.device)
            self._carve()
        if dtype != self._out.dtype or entries > self._out.numel():
            size = max(entries, 2 * self._out.numel() if dtype == self._out.dtype else 0, 1)
            self._out = torch.empty(size, dtype=dtype, device=self.device)

    def compact(
        self,
        indptr: torch.Tensor,
        slots: torch.Tensor,
        keep: torch.Tensor,
        audit: torch.Tensor | None,
        active: bool,
        n_real: int,
        n_rows: int,
        entries: int,
    ) -> torch.Tensor:
        """Rewrite ``indptr[:n_rows + 1]`` and ``slots[:entries]`` in place to the view; the new lengths.

        ``keep`` is the view's policy (bool or uint8 [rows, >= width]), ``audit`` the uint8 rows audited in this
        step or None, ``entries`` the length of the engine's list (``indptr[n_rows]``, known on the host)."""
        if indptr.dtype != torch.int32:
            raise ValueError("indptr must be int32")
        if slots.dtype not in (torch.int32, torch.int64):
            raise ValueError("slots must be int32 or int64")
        if keep.dtype not in (torch.bool, torch.uint8) or keep.stride(1) != 1 or keep.shape[1] < self.width:
            raise ValueError(f"keep must be a bool or uint8 [rows, >= {self.width}] tensor with contiguous rows")
        if not (indptr.is_cuda and slots.is_cuda and keep.is_cuda):
            raise ValueError("the compaction runs on the device: indptr, slots and keep must be CUDA tensors")
        self._fit(n_rows, entries, slots.dtype)
        audit_rows = None if audit is None else (audit if audit.dtype == torch.uint8 else audit.to(torch.uint8))
        rc = _lib.load().ekv_slot_compact(
            indptr.data_ptr(), slots.data_ptr(), slots.element_size(), keep.data_ptr(), keep.stride(0),
            _lib.ptr(audit_rows), int(bool(active)), int(n_real), int(n_rows), int(entries), self.block_tokens,
            self.width, self.new_indptr.data_ptr(), self.lens.data_ptr(), self.table.data_ptr(),
            self.table.stride(0), self.counts.data_ptr(), self._out.data_ptr(), _lib.current_stream(),
        )
        _lib.check(rc, "ekv_slot_compact")
        return self.lens[:n_rows]
