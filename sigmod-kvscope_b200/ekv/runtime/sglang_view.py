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
    """The view of SGLang: ``DecodeView``'s policy, audits and counters over SGLang's key-value list. It
    reads fewer blocks and gives none of their memory back to the engine, so it releases nothing."""

    def __init__(
        self, rows: int, width: int, block_size: int, audit: StatisticSwitch | None, device: torch.device
    ) -> None:
        super().__init__(rows, width, block_size, audit=audit, device=device)
        self.compactor = SlotCompactor(width, block_size, device)
        self._counts = self.compactor.counts  # the compaction kernel adds the read counters here

    def write_release(self, mask: np.ndarray) -> list[tuple[int, int]]:
        if np.asarray(mask).any():
            raise RuntimeError("the SGLang view does not release blocks: the controller asked for a release")
        return []

    def rewrite(
        self, indptr: torch.Tensor, slots: torch.Tensor, lengths: np.ndarray, n_rows: int, entries: int
    ) -> torch.Tensor:
        """Rewrite a decode batch's list in place to the view; the new length of each of its ``n_rows`` rows.

        ``lengths`` holds each request's tokens (host), so an audit reads nothing back; a CUDA graph's batch
        has more rows than requests, and the list ``entries`` entries. Every row decodes: the bookkeeping is
        ``DecodeView.build``'s for such a batch (``_begin_step``)."""
        self.finish_audit()
        lengths = np.asarray(lengths)
        requests = len(lengths)
        if requests > self.rows:
            raise ValueError(f"batch of {requests} requests exceeds the view's {self.rows} rows")
        audited = self._begin_step(np.ones(requests, dtype=bool), None)
        audit_rows = None
        if self.audit_step:
            self._pending_blocks = -(-lengths // self.block_size)
            audit_rows = torch.from_numpy(audited.astype(np.uint8)).to(indptr.device)
            if self.audit is not None:
                self.audit.select(audited[:requests], np.arange(requests))
        if self.audit is not None:
            self.audit.set(self.audit_step)
        return self.compactor.compact(indptr, slots, self._masks[0], audit_rows, self.active(), requests, n_rows,
                                      entries)
