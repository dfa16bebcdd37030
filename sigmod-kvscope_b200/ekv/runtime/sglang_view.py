"""The block-table view for SGLang's Triton attention backend (runtime/sglang_view.py:46-97 of the reference).

SGLang's decode kernel reads a request's cache through a CSR list of token slots: ``kv_indptr`` marks where each
request's slots start in ``kv_indices``. Its page size is one token, so the view defines a block of
``BLOCK_TOKENS`` consecutive tokens and keeps or drops whole blocks of a request. ``SlotView`` is the
reference's class: the policy, audits and read counters of ``DecodeView``, and ``rewrite``, which compacts a
decode batch's list in place on the device (``ekv.runtime.sglang_compact``) from lengths the host already knows.

The engine hooks of the reference module (its scheduler safe point and attention-backend patches) belong to the
serving integration and the controller's mailbox, which this package does not carry; an integration calls
``SlotView.rewrite`` from the same places.
"""

from __future__ import annotations

import numpy as np
import torch

from .block_view import DecodeView, StatisticSwitch
from .sglang_compact import SlotCompactor

BLOCK_TOKENS = 16


def kv_pointers(pool) -> list[int]:
    """The address of each layer's key cache in layer order, which is the order the plane looks a layer up in."""
    return [pool.get_key_buffer(layer).data_ptr() for layer in range(pool.layer_num)]


class SlotView(DecodeView):
    """The view of SGLang. It keeps the policy and the audits of ``DecodeView`` and compacts the key-value list of a
    decode batch on the device. It reads fewer blocks and does not give their memory back to the engine."""

    def __init__(
        self, rows: int, width: int, block_size: int, audit: StatisticSwitch | None, device: torch.device
    ) -> None:
        super().__init__(rows, width, block_size, audit=audit)
        self.compactor = SlotCompactor(width, block_size, device)
        self._counts = self.compactor.counts  # reads() and read_breakdown() read the counters the kernel adds to

    def write_release(self, mask: np.ndarray) -> list[tuple[int, int]]:
        if np.asarray(mask).any():
            raise RuntimeError("the SGLang view does not release blocks: the controller asked for a release")
        return []

    def rewrite(
        self, indptr: torch.Tensor, slots: torch.Tensor, lengths: np.ndarray, n_rows: int, entries: int
    ) -> torch.Tensor:
        """Rewrite a decode batch's list in place to the view, and return the new length of each of its rows.

        ``lengths`` holds the tokens of each request, from the host, so an audit needs no device read. The batch has
        ``n_rows`` rows, more than the requests when a CUDA graph fills its batch, and ``entries`` list entries. The
        bookkeeping is that of ``DecodeView.build`` for a batch in which every row decodes."""
        self.finish_audit()
        lengths = np.asarray(lengths)
        requests = len(lengths)
        if requests > self.rows:
            raise ValueError(f"batch of {requests} requests exceeds the view's {self.rows} rows")
        self._device = indptr.device
        audited = np.zeros(self.rows, dtype=bool)
        audited[:requests] = self.audit_rows[:requests]
        if audited.any() and not self.may_audit():
            audited[:] = False  # the requests wait for a step after the controller has read the last audit
        self.audit_rows[audited] = False  # an audit request is consumed by the step that serves it
        self.audit_step = bool(audited.any())
        self._audit_pending = self.audit_step
        self._pending_rows = audited
        audit = None
        if self.audit_step:
            self.start_audit()
            self._pending_blocks[:requests] = -(-lengths // self.block_size)
            audit = torch.from_numpy(audited.astype(np.uint8)).to(indptr.device)
            if self.audit is not None:
                self.audit.select(audited[:requests], np.arange(requests))
        if self.audit is not None:
            self.audit.set(self.audit_step)
        keep = self._keep_on(indptr.device)
        return self.compactor.compact(indptr, slots, keep, audit, self.active(), requests, n_rows, entries)
