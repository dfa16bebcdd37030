"""The oracle pinned against the reference: golden vectors made by running the reference's own code
(tests/golden/make_golden.py), and the known answers of the reference's own unit tests. CPU only."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import load_golden

from oracle import allocation as oa
from oracle import audit as oaud
from oracle import shares as osh
from oracle import view as ov


def unpack(x: np.ndarray, dtype: str) -> np.ndarray:
    """fp16 arrays as stored; bf16 stored as the upper 16 bits of float32."""
    if dtype == "fp16":
        return x.astype(np.float32)
    return (x.astype(np.uint32) << 16).view(np.float32)


def run_oracle_audit(g: dict) -> np.ndarray:
    dtype = str(g["dtype"])
    q, k = unpack(g["query"], dtype), unpack(g["keys"], dtype)
    layers = q.shape[0]
    rows, width = g["table"].shape
    lse = oaud.new_table(layers, rows, width, int(g["group_rows"]))
    for layer in range(layers):
        oaud.tile_lse(q[layer], k[layer], g["table"], g["lens"], g["qrow"], g["select"], int(g["flags"][layer]),
                      lse, float(g["scale"]), layer, layer % int(g["kv_heads"]), int(g["block_size"]),
                      int(g["tile_blocks"]))
    return lse


AUDIT_CASES = ["audit_cfg1_fp16", "audit_layers_fp16", "audit_g8_bf16"]


@pytest.mark.parametrize("name", AUDIT_CASES)
def test_oracle_tile_lse_matches_the_reference_kernel(name):
    g = load_golden(name)
    lse = run_oracle_audit(g)
    ref = g["lse"]
    assert np.array_equal(np.isnan(lse), np.isnan(ref)), "the same cells are written"
    written = ~np.isnan(ref)
    assert written.any()
    np.testing.assert_allclose(lse[written], ref[written], rtol=2e-5, atol=2e-5)


def test_unselected_rows_and_layers_with_the_flag_off_stay_nan():
    g = load_golden("audit_layers_fp16")
    ref = g["lse"]
    assert np.isnan(ref[:, 1]).all(), "layer 1 ran with the flag off"
    assert np.isnan(ref[:, :, 2]).all(), "row 2 was not selected"


@pytest.mark.parametrize("name", AUDIT_CASES)
@pytest.mark.parametrize("aggregate", ["mean", "max"])
def test_oracle_shares_match_the_reference_normalisation(name, aggregate):
    g = load_golden(name)
    live = g["live"]
    u = osh.log_weights(g["lse"], g["lse"].shape[1], live, int(g["tile_blocks"]))
    np.testing.assert_array_equal(u, g["u"])  # the same float32 arithmetic as read_tile_rows
    share = np.full_like(g[f"share_{aggregate}"], np.nan)
    share[live] = osh.normalize(u, g["row_blocks"][live], int(g["tile_blocks"]), aggregate)
    np.testing.assert_allclose(share, g[f"share_{aggregate}"], rtol=1e-12, atol=1e-15, equal_nan=True)


@pytest.mark.parametrize("name", AUDIT_CASES)
def test_oracle_controller_view_matches_the_reference(name):
    g = load_golden(name)
    rows, width = g["table"].shape
    share = g["share_mean"]
    keep = oa.controller_keep(g["row_blocks"], width, lambda r, n: np.nan_to_num(share[r, :n], nan=0.0), 0.5, "uniform",
                              recent_blocks=4)
    np.testing.assert_array_equal(keep, g["keep"])
    view, view_lens = ov.compact_block_table(g["table"], g["lens"], keep, int(g["block_size"]))
    np.testing.assert_array_equal(view, g["view"])
    np.testing.assert_array_equal(view_lens, g["view_lens"])


def test_oracle_normalize_matches_reference_cases():
    g = load_golden("shares_cases")
    for i in range(12):
        for aggregate in ("mean", "max"):
            got = osh.normalize(g[f"u{i}"], g[f"rb{i}"], int(g[f"tb{i}"]), aggregate)
            np.testing.assert_allclose(got, g[f"{aggregate}{i}"], rtol=1e-12, atol=1e-15, equal_nan=True)


def test_vectorised_normalize_matches_reference_cases_and_the_loop_form():
    """normalize_rows, the per-row vectorised form used at full model sizes, against the reference's
    outputs and against normalize on random cells with NaN holes, partial tails and empty rows."""
    g = load_golden("shares_cases")
    for i in range(12):
        for aggregate in ("mean", "max"):
            got = osh.normalize_rows(g[f"u{i}"], g[f"rb{i}"], int(g[f"tb{i}"]), aggregate)
            np.testing.assert_allclose(got, g[f"{aggregate}{i}"], rtol=1e-12, atol=1e-15, equal_nan=True)
    rng = np.random.default_rng(4)
    for trial in range(6):
        layers, rows, width, q = 3, 5, 23, 1 + trial % 4
        u = rng.normal(0, 3, (layers, rows, width, q)).astype(np.float32)
        u[rng.random(u.shape) < 0.1] = np.nan
        row_blocks = rng.integers(0, width + 1, rows)
        for aggregate in ("mean", "max"):
            a = osh.normalize(u, row_blocks, 1 + trial % 3, aggregate)
            b = osh.normalize_rows(u, row_blocks, 1 + trial % 3, aggregate)
            np.testing.assert_allclose(b, a, rtol=1e-12, atol=1e-15, equal_nan=True)


def test_oracle_log_weights_match_read_tile_rows():
    g = load_golden("shares_cases")
    table_layers, layers, rows, width, group, tile_blocks = 4, 3, 5, 6, 2, 2
    lse = g["read_table"].reshape(2, table_layers, rows, width, group)
    u = osh.log_weights(lse, layers, g["read_rows"], tile_blocks)
    np.testing.assert_array_equal(u, g["read_u"])
    assert u[0, 0, 3, 1] == -np.inf  # cell 7 holds l = 0: no weight


def test_oracle_allocation_matches_the_reference_bit_exactly():
    g = load_golden("allocation_cases")
    for i in range(60):
        sizes = g[f"sizes{i}"]
        flat = g[f"scores{i}"]
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        scores = [flat[bounds[j] : bounds[j + 1]] for j in range(len(sizes))]
        recent = int(g[f"recent{i}"])
        pinned = [oa.controller_pins(int(n), recent) for n in sizes]
        masks = oa.allocate(scores, int(g[f"budget{i}"]), str(g[f"objective{i}"]), pinned)
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")


def test_oracle_view_matches_300_reference_batches():
    g = load_golden("view_cases")
    for i in range(300):
        view, lens = ov.compact_block_table(g[f"table{i}"], g[f"lens{i}"], g[f"keep{i}"], 16)
        np.testing.assert_array_equal(view, g[f"view{i}"], err_msg=f"batch {i}")
        np.testing.assert_array_equal(lens, g[f"view_lens{i}"], err_msg=f"batch {i}")


# ---- known answers of the reference's own unit tests ---------------------------------------------


def test_known_answer_unwritten_cells_and_empty_blocks_carry_no_mass():
    u = np.full((1, 2, 4, 2), np.nan, dtype=np.float32)
    u[0, 0, :, 0] = [0.0, np.log(3.0), -np.inf, np.nan]
    got = osh.normalize(u, np.array([4, 4]), 1)
    np.testing.assert_allclose(got[0], [0.25, 0.75, 0.0, 0.0])
    assert np.isnan(got[1]).all()


def test_known_answer_a_query_row_without_data_does_not_dilute_the_mean():
    u = np.full((1, 1, 3, 2), np.nan, dtype=np.float32)
    u[0, 0, :, 0] = np.log([1.0, 1.0, 2.0])
    np.testing.assert_allclose(osh.normalize(u, np.array([3]), 1)[0], [0.25, 0.25, 0.5])


def test_known_answer_a_partial_last_tile_gets_its_whole_mass():
    cells = np.repeat(np.log(np.array([1.0, 2.0, 5.0]) / 2), 2).astype(np.float32).reshape(1, 1, 6, 1)
    got = osh.normalize(cells, np.array([5]), 2)
    np.testing.assert_allclose(got[0], np.array([0.5, 0.5, 1.0, 1.0, 5.0, 0.0]) / 8.0, rtol=1e-6)


def test_known_answer_a_complete_last_tile_is_left_alone():
    cells = np.repeat(np.log(np.array([3.0, 1.0]) / 2), 2).astype(np.float32).reshape(1, 1, 4, 1)
    np.testing.assert_allclose(osh.normalize(cells, np.array([4]), 2)[0], [0.375, 0.375, 0.125, 0.125], rtol=1e-6)


def test_known_answer_max_keeps_a_block_that_one_head_needs():
    u = np.log(np.array([[9.0, 1.0, 1.0], [1.0, 9.0, 1.0]])).T.astype(np.float32).reshape(1, 1, 3, 2)
    np.testing.assert_allclose(osh.normalize(u, np.array([3]), 1)[0], np.array([10.0, 10.0, 2.0]) / 22.0, atol=1e-6)
    np.testing.assert_allclose(osh.normalize(u, np.array([3]), 1, "max")[0], np.array([9.0, 9.0, 1.0]) / 19.0, atol=1e-6)


def test_known_answer_views():
    def view_of(table, lens, keep):
        v, n = ov.compact_block_table(np.array(table), np.array(lens), np.array(keep), 16)
        return v, n

    v, n = view_of([[7, 8, 9, 10]], [64], [[True] * 4])
    assert v.tolist() == [[7, 8, 9, 10]] and n.tolist() == [64]
    v, n = view_of([[7, 8, 9, 10]], [40], [[False] * 4])
    assert v[0, :2].tolist() == [7, 9] and n.tolist() == [24]
    v, n = view_of([[7, 8, 9, 10]], [64], [[False, True, False, False]])
    assert v[0, :3].tolist() == [7, 8, 10] and n.tolist() == [48]
    v, n = view_of([[1, 2, 3, 4, 5, 6]], [96], [[True, False, True, False, True, False]])
    assert v[0, :4].tolist() == [1, 3, 5, 6] and n.tolist() == [64]
    _, n = view_of([[1, 2], [3, 4]], [0, 20], [[True, True], [False, False]])
    assert n.tolist() == [0, 20]
    v, n = view_of([[5]], [3], [[False]])
    assert v[0, 0] == 5 and n.tolist() == [3]


def test_known_answer_keep_newest():
    """The fixed rule scores = arange(n) at budget 0.5 with no recent pins keeps [0, 6, 7, 8, 9]."""
    keep = oa.controller_keep(np.array([10]), 12, lambda r, n: np.arange(n, dtype=float), 0.5, "uniform", recent_blocks=0)
    assert np.flatnonzero(keep[0, :10]).tolist() == [0, 6, 7, 8, 9]
    g = load_golden("allocation_cases")
    assert np.flatnonzero(g["newest_mask"]).tolist() == [0, 6, 7, 8, 9]


def test_oracle_rejects_a_budget_below_the_pins():
    with pytest.raises(ValueError):
        oa.allocate([np.ones(5)], 1, "sum")


def test_oracle_slot_compaction_matches_the_reference_kernels():
    """oracle.view.slot_compact against SlotCompactor.compact run by make_golden.py in the interpreter."""
    from oracle import view as ov

    g = load_golden("slot_cases")
    for i in range(60):
        indptr, slots, keep = g[f"indptr{i}"], g[f"slots{i}"], g[f"keep{i}"]
        audit = g[f"audit{i}"] if len(g[f"audit{i}"]) else None
        n_rows = len(indptr) - 1
        new_indptr, new_slots, lens, counts = ov.slot_compact(indptr, slots, keep, audit, bool(g[f"active{i}"]),
                                                              int(g[f"n_real{i}"]), n_rows, 16)
        np.testing.assert_array_equal(new_indptr, g[f"new_indptr{i}"], err_msg=f"case {i}")
        np.testing.assert_array_equal(new_slots, g[f"new_slots{i}"], err_msg=f"case {i}")
        np.testing.assert_array_equal(lens, g[f"lens{i}"], err_msg=f"case {i}")
        np.testing.assert_array_equal(counts, g[f"counts{i}"], err_msg=f"case {i}")


def test_oracle_maxmin_matches_the_reference_allocate():
    """oracle.allocation.water_level against allocate(..., "maxmin") run by make_golden.py."""
    g = load_golden("maxmin_cases")
    for i in range(50):
        sizes = g[f"sizes{i}"]
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        scores = [g[f"scores{i}"][bounds[j] : bounds[j + 1]] for j in range(len(sizes))]
        pinned = [oa.controller_pins(int(n), int(g[f"recent{i}"])) for n in sizes]
        masks = oa.allocate(scores, int(g[f"budget{i}"]), "maxmin", pinned)
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")


def pinned_case(g, i):
    sizes = g[f"sizes{i}"]
    bounds = np.concatenate([[0], np.cumsum(sizes)])
    cut = [slice(bounds[j], bounds[j + 1]) for j in range(len(sizes))]
    return ([g[f"scores{i}"][c] for c in cut], [g[f"pinned{i}"][c] for c in cut], list(g[f"weights{i}"]),
            int(g[f"budget{i}"]), str(g[f"objective{i}"]))


def test_oracle_allocation_with_pins_anywhere_matches_the_reference():
    """Request.pinned marking any blocks (none, every one, middle ones): allocate() run by make_golden.py."""
    g = load_golden("pinned_cases")
    for i in range(120):
        scores, pinned, weights, budget, objective = pinned_case(g, i)
        masks = oa.allocate(scores, budget, objective, pinned, weights)
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")


def test_oracle_float64_allocation_matches_the_reference():
    """Every objective on float64 scores whose shares (and weighted gains) round together."""
    g = load_golden("float64_cases")
    for i in range(90):
        sizes = g[f"sizes{i}"]
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        scores = [g[f"scores{i}"][bounds[j] : bounds[j + 1]] for j in range(len(sizes))]
        pinned = [oa.controller_pins(int(n), int(g[f"recent{i}"])) for n in sizes]
        masks = oa.allocate(scores, int(g[f"budget{i}"]), str(g[f"objective{i}"]), pinned, list(g[f"weights{i}"]))
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")


def controller_setups(g):
    out = []
    for text in g["setups"]:
        objective, fraction, recent, decay, cap = str(text).split(",")
        out.append((objective, float(fraction), int(recent), float(decay), int(cap)))
    return out


def controller_weight(key):
    """The request weights make_golden.py gives the reference controller (sum objective only)."""
    return 1.0 + 0.25 * (int(key) % 4) - (0.5 if int(key) % 7 == 0 else 0.0)


def test_oracle_controller_matches_the_reference_sequence():
    """oracle.controller.Ledger against the reference Controller over a sequence of audits: the smoothed
    shares, the measured lengths and the committed keep mask after every audit, bit for bit."""
    from oracle import controller as oc

    g = load_golden("controller_cases")
    width = int(g["width"])
    for c, (objective, fraction, recent, decay, cap) in enumerate(controller_setups(g)):
        ledger = oc.Ledger(width, decay)
        for step in range(int(g["steps"])):
            keys, lengths, audit_keys = g[f"keys{step}"], g[f"lengths{step}"], g[f"audit_keys{step}"]
            live, row_blocks = oc.audit_row_blocks(audit_keys, keys, lengths, cap)
            fresh = g[f"fresh{step}"][:live].copy()
            fresh[row_blocks <= 0] = np.nan
            ledger.absorb(fresh, audit_keys, row_blocks)
            ledger.forget(keys)
            keep = ledger.keep(keys, lengths, width, fraction, objective, recent, cap,
                               controller_weight if objective == "sum" else None)
            ks = sorted(ledger.shares)
            np.testing.assert_array_equal(np.array(ks, dtype=np.uint64), g[f"share_keys{c}_{step}"])
            got = np.array([ledger.shares[k] for k in ks]).reshape(len(ks), width)
            np.testing.assert_array_equal(got, g[f"shares{c}_{step}"], err_msg=f"setup {c} step {step}")
            np.testing.assert_array_equal([ledger.measured[k] for k in ks], g[f"measured{c}_{step}"])
            np.testing.assert_array_equal(keep, g[f"keep{c}_{step}"], err_msg=f"setup {c} step {step}")


def test_oracle_fixed_scoring_controller_matches_the_reference():
    """A controller with a fixed scoring rule (no measured shares): every row longer than the cap is a
    request of fixed(n) scores with the recent pins, weighted, under one budget."""
    g = load_golden("controller_cases")
    width = int(g["width"])
    for step in range(int(g["steps"])):
        keys, lengths = g[f"keys{step}"], g[f"lengths{step}"]
        row_blocks = np.where(keys != 0, lengths, 0)
        weights = np.array([controller_weight(k) for k in keys])
        keep = oa.controller_keep(row_blocks, width, lambda r, n: np.sin(np.arange(n) * 0.37) + 1.0, 0.35, "sum",
                                  recent_blocks=2, cap_above_blocks=4, weights=weights)
        np.testing.assert_array_equal(keep, g[f"fixed_keep{step}"], err_msg=f"step {step}")
