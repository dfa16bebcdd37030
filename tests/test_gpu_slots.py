"""Parity of the SGLang CSR compaction (SlotCompactor / ekv_slot_compact) with the reference's own kernels
(tests/golden/slot_cases.npz, made by running runtime/sglang_compact.py in the Triton interpreter) and with the
oracle on large batches: the new indptr, every entry of the new list, the new lengths and the read counters,
bit-exact; nothing past the list is written."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import load_golden

from oracle import view as ov

pytestmark = pytest.mark.gpu


def compact(indptr, slots, keep, audit, active, n_real, dtype=torch.int64, compactor=None, tail=7):
    from ekv.runtime.sglang_compact import SlotCompactor

    dev = torch.device("cuda")
    width = keep.shape[1]
    compactor = compactor or SlotCompactor(width, 16, dev)
    d_indptr = torch.from_numpy(np.asarray(indptr, dtype=np.int32)).to(dev)
    d_slots = torch.from_numpy(np.concatenate([np.asarray(slots), np.full(tail, -1)]).astype(np.int64)).to(dtype).to(dev)
    d_keep = torch.from_numpy(np.asarray(keep, dtype=bool)).to(dev)
    d_audit = None if audit is None else torch.from_numpy(np.asarray(audit, dtype=np.uint8)).to(dev)
    n_rows = len(indptr) - 1
    lens = compactor.compact(d_indptr, d_slots, d_keep, d_audit, active, n_real, n_rows, int(indptr[-1]))
    torch.cuda.synchronize()
    return d_indptr.cpu().numpy(), d_slots.cpu().numpy(), lens.cpu().numpy(), compactor.counts.cpu().numpy()


def test_compaction_matches_the_reference_kernels():
    g = load_golden("slot_cases")
    for i in range(60):
        indptr, slots = g[f"indptr{i}"], g[f"slots{i}"]
        audit = g[f"audit{i}"] if len(g[f"audit{i}"]) else None
        new_indptr, new_slots, lens, counts = compact(indptr, slots, g[f"keep{i}"], audit, bool(g[f"active{i}"]),
                                                      int(g[f"n_real{i}"]))
        total = int(new_indptr[-1])
        np.testing.assert_array_equal(new_indptr, g[f"new_indptr{i}"], err_msg=f"case {i}")
        np.testing.assert_array_equal(new_slots[:total], g[f"new_slots{i}"], err_msg=f"case {i}")
        np.testing.assert_array_equal(lens, g[f"lens{i}"], err_msg=f"case {i}")
        np.testing.assert_array_equal(counts, g[f"counts{i}"], err_msg=f"case {i}")
        assert (new_slots[int(indptr[-1]):] == -1).all(), f"case {i}: an entry past the list was written"


@pytest.mark.parametrize("dtype", [torch.int64, torch.int32])
def test_large_batches_against_the_oracle(dtype):
    rng = np.random.default_rng(53)
    width = 300
    for trial in range(4):
        n_real = int(rng.integers(50, 400))
        padding = int(rng.integers(0, 8))
        lens = rng.integers(1, 16 * width + 1, n_real).tolist() + [1] * padding
        indptr = np.array([0, *np.cumsum(lens).tolist()], dtype=np.int64)
        slots = rng.integers(0, 1 << 30, int(indptr[-1]))
        keep = rng.random((n_real + padding, width)) < rng.random()
        audit = (rng.random(n_real + padding) < 0.1).astype(np.uint8) if trial % 2 else None
        active = trial != 3
        want_indptr, want_slots, want_lens, want_counts = ov.slot_compact(indptr, slots, keep, audit, active, n_real,
                                                                          n_real + padding, 16)
        new_indptr, new_slots, got_lens, counts = compact(indptr.astype(np.int32), slots, keep, audit, active, n_real,
                                                          dtype=dtype)
        np.testing.assert_array_equal(new_indptr, want_indptr)
        np.testing.assert_array_equal(new_slots[: int(want_indptr[-1])], want_slots.astype(new_slots.dtype))
        np.testing.assert_array_equal(got_lens, want_lens)
        np.testing.assert_array_equal(counts, want_counts)


def test_counters_accumulate_over_steps():
    from ekv.runtime.sglang_compact import SlotCompactor

    g = load_golden("slot_cases")
    compactor = SlotCompactor(20, 16, torch.device("cuda"))
    total = np.zeros(5, dtype=np.int64)
    for i in range(8):
        audit = g[f"audit{i}"] if len(g[f"audit{i}"]) else None
        compact(g[f"indptr{i}"], g[f"slots{i}"], g[f"keep{i}"], audit, bool(g[f"active{i}"]), int(g[f"n_real{i}"]),
                compactor=compactor)
        total += g[f"counts{i}"]
    np.testing.assert_array_equal(compactor.counts.cpu().numpy(), total)


def test_slot_view_rewrites_a_batch_and_consumes_its_audits():
    from ekv.runtime.sglang_view import SlotView

    class Switch:  # the audit plane's switch: records what the view asks of it
        def __init__(self):
            self.on, self.selected = [], None

        def set(self, on):
            self.on.append(bool(on))

        def select(self, audited, token_start):
            self.selected = np.asarray(audited).copy()

    rng = np.random.default_rng(61)
    rows, width = 8, 40
    switch = Switch()
    view = SlotView(rows, width, 16, switch, torch.device("cuda"))
    mask = rng.random((rows, width)) < 0.4
    view.write_row_controls(mask.astype(np.uint8))
    view.write_lease_deadline(2**62)
    requested = np.zeros(rows, dtype=bool)
    requested[2] = True
    view.write_audit_rows(requested)
    lengths = rng.integers(1, 16 * width, 6)
    indptr = np.array([0, *np.cumsum(list(lengths) + [1, 1]).tolist()], dtype=np.int64)
    slots = rng.permutation(200_000)[: int(indptr[-1])]
    dev = torch.device("cuda")
    d_indptr = torch.from_numpy(indptr.astype(np.int32)).to(dev)
    d_slots = torch.from_numpy(slots.astype(np.int64)).to(dev)
    lens = view.rewrite(d_indptr, d_slots, lengths, 8, int(indptr[-1]))
    audit = np.zeros(8, dtype=np.uint8)
    audit[2] = 1
    want_indptr, want_slots, want_lens, want_counts = ov.slot_compact(indptr, slots, view.keep, audit, view.active(), 6,
                                                                      8, 16)
    np.testing.assert_array_equal(lens.cpu().numpy(), want_lens)
    np.testing.assert_array_equal(d_indptr.cpu().numpy(), want_indptr)
    np.testing.assert_array_equal(d_slots.cpu().numpy()[: int(want_indptr[-1])], want_slots)
    assert view.audit_step and not view.audit_rows[2]  # the audit request was consumed by this step
    assert switch.on == [True] and switch.selected.tolist() == [False, False, True, False, False, False]
    assert view.reads() == (int(want_counts[0]), int(want_counts[1]))
    with pytest.raises(RuntimeError):
        view.write_release(np.ones((rows, width), dtype=bool))
