"""The compaction of SGLang's key-value index list on the device, with no host synchronisation.

Drop-in for runtime/sglang_compact.py of the reference: ``COUNTS`` and ``SlotCompactor`` keep their
names, buffers (``counts``, ``new_indptr``, ``lens``, ``table``) and ``compact`` signature and
meaning. SGLang's decode kernel reads request ``r`` from ``slots[indptr[r]:indptr[r+1]]``, one token
slot per entry; the view groups ``block_tokens`` consecutive entries into a block and keeps some
blocks (the first and last always; all of them when the policy is not live, when the row is audited,
and for the rows a CUDA graph adds from ``n_real`` on). The work runs in the sm_100a kernels of
``ekv_slot_compact``: a warp per row (the reference walks the rows in one Triton program), a scan of
the new lengths, a gather of every new entry, and the copy back into the engine's buffers.
"""

from __future__ import annotations

import torch

from .. import _lib

COUNTS = 5  # blocks read, blocks a full read would read, read in audits, read untrimmed, read without a live policy


class SlotCompactor:
    """The buffers of the compaction, kept from step to step. They grow when a batch needs more and never shrink."""

    GATHER_BLOCK = 1024

    def __init__(self, width: int, block_tokens: int, device: torch.device) -> None:
        if width <= 0 or block_tokens <= 0:
            raise ValueError("width and block_tokens must be positive")
        self.width, self.block_tokens, self.device = width, block_tokens, device
        self.counts = torch.zeros(COUNTS, dtype=torch.int64, device=device)
        self.no_audit = torch.zeros(1, dtype=torch.uint8, device=device)
        self._rows = 0
        self.new_indptr = self.lens = self.table = torch.empty(0, dtype=torch.int32, device=device)
        self._out: torch.Tensor = torch.empty(0, dtype=torch.int64, device=device)

    def _reserve(self, rows: int, entries: int, dtype: torch.dtype) -> None:
        if rows > self._rows:
            self._rows = rows
            self.new_indptr = torch.empty(rows + 1, dtype=torch.int32, device=self.device)
            self.lens = torch.empty(rows, dtype=torch.int32, device=self.device)
            self.table = torch.empty(rows, self.width, dtype=torch.int32, device=self.device)
        if entries > self._out.shape[0] or dtype != self._out.dtype:
            self._out = torch.empty(max(entries, self._out.shape[0], 1), dtype=dtype, device=self.device)

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
        """Rewrite ``indptr[:n_rows + 1]`` and ``slots[:entries]`` in place to the view, and return the new lengths.

        ``keep`` is the bool ``[rows, width]`` policy of the view, ``audit`` the uint8 rows audited in this step (or
        ``None``), and ``entries`` the length of the engine's list, ``indptr[n_rows]``, which the host knows."""
        if indptr.dtype != torch.int32:
            raise ValueError("indptr must be int32")
        if slots.dtype not in (torch.int32, torch.int64):
            raise ValueError("slots must be int32 or int64")
        if keep.dtype not in (torch.bool, torch.uint8) or keep.stride(1) != 1 or keep.shape[1] < self.width:
            raise ValueError(f"keep must be a bool or uint8 [rows, >= {self.width}] tensor with contiguous rows")
        if not (indptr.is_cuda and slots.is_cuda and keep.is_cuda):
            raise ValueError("the compaction runs on the device: indptr, slots and keep must be CUDA tensors")
        self._reserve(n_rows, entries, slots.dtype)
        audit_ptr = None if audit is None else audit.to(torch.uint8).data_ptr()
        rc = _lib.load().ekv_slot_compact(
            indptr.data_ptr(), slots.data_ptr(), slots.element_size(), keep.data_ptr(), keep.stride(0), audit_ptr,
            int(bool(active)), int(n_real), int(n_rows), int(entries), self.block_tokens, self.width,
            self.new_indptr.data_ptr(), self.lens.data_ptr(), self.table.data_ptr(), self.table.stride(0),
            self.counts.data_ptr(), self._out.data_ptr(), _lib.current_stream(),
        )
        _lib.check(rc, "ekv_slot_compact")
        return self.lens[:n_rows]
