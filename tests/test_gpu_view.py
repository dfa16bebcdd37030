"""Parity of the device view builder with the reference: compaction, allocation and the controller's
keep mask, bit-exact (ids, order and lengths), on the golden vectors, the oracle, and the full-size
view stress shape through size-independent properties."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from conftest import load_golden

from oracle import allocation as oa
from oracle import view as ov

pytestmark = pytest.mark.gpu


def test_compact_block_table_matches_300_reference_batches():
    from ekv.runtime.block_view import compact_block_table

    g = load_golden("view_cases")
    for i in range(300):
        table = torch.from_numpy(g[f"table{i}"]).cuda()
        lens = torch.from_numpy(g[f"lens{i}"]).cuda()
        keep = torch.from_numpy(g[f"keep{i}"]).cuda()
        view, view_lens = compact_block_table(table, lens, keep, 16)
        np.testing.assert_array_equal(view.cpu().numpy(), g[f"view{i}"], err_msg=f"batch {i}")
        np.testing.assert_array_equal(view_lens.cpu().numpy(), g[f"view_lens{i}"], err_msg=f"batch {i}")


def test_known_answer_views_on_the_device():
    from ekv.runtime.block_view import compact_block_table

    def view_of(table, lens, keep):
        t = torch.tensor(table, dtype=torch.int32).cuda()
        return compact_block_table(t, torch.tensor(lens, dtype=torch.int32).cuda(), torch.tensor(keep).cuda(), 16)

    v, n = view_of([[7, 8, 9, 10]], [40], [[False] * 4])
    assert v[0, :2].tolist() == [7, 9] and n.tolist() == [24]
    v, n = view_of([[1, 2, 3, 4, 5, 6]], [96], [[True, False, True, False, True, False]])
    assert v[0, :4].tolist() == [1, 3, 5, 6] and n.tolist() == [64]
    _, n = view_of([[1, 2], [3, 4]], [0, 20], [[True, True], [False, False]])
    assert n.tolist() == [0, 20]
    v, n = view_of([[5]], [3], [[False]])
    assert v[0, 0].item() == 5 and n.tolist() == [3]


def golden_requests(g, i):
    sizes = g[f"sizes{i}"]
    flat = g[f"scores{i}"]
    bounds = np.concatenate([[0], np.cumsum(sizes)])
    scores = [flat[bounds[j] : bounds[j + 1]] for j in range(len(sizes))]
    recent = int(g[f"recent{i}"])
    pinned = [oa.controller_pins(int(n), recent) for n in sizes]
    return scores, pinned


def test_allocate_matches_the_reference_bit_exactly_including_ties():
    from ekv.observe.allocation import Request, allocate

    g = load_golden("allocation_cases")
    several_sum = 0
    for i in range(60):
        scores, pinned = golden_requests(g, i)
        objective = str(g[f"objective{i}"])
        requests = [Request(scores=s, pinned=p) for s, p in zip(scores, pinned, strict=True)]
        masks = allocate(requests, int(g[f"budget{i}"]), objective)
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")
        several_sum += objective == "sum" and len(requests) > 1
    assert several_sum >= 10  # the global greedy over several requests is among the pinned cases


def test_allocate_against_the_oracle_with_many_ties():
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(5)
    for trial in range(80):
        n_req = 1 if trial % 2 else int(rng.integers(1, 9))
        objective = "sum" if (trial % 2 and trial % 4 == 1) else "uniform"
        scores = [rng.integers(0, 3, int(rng.integers(1, 300))).astype(np.float64) for _ in range(n_req)]
        if trial % 5 == 0:
            scores = [rng.random(len(s)).astype(np.float32).astype(np.float64) for s in scores]
        recent = int(rng.integers(0, 6))
        pinned = [oa.controller_pins(len(s), recent) for s in scores]
        must = sum(int(p.sum()) for p in pinned)
        total = sum(len(s) for s in scores)
        budget = int(rng.integers(must, total + 1))
        got = allocate([Request(scores=s, pinned=p) for s, p in zip(scores, pinned, strict=True)], budget, objective)
        want = oa.allocate(scores, budget, objective, pinned)
        for a, b in zip(got, want, strict=True):
            np.testing.assert_array_equal(a, b, err_msg=f"trial {trial}")


def test_uniform_quotas_over_thousands_of_requests():
    """Largest remainders over ~2000 requests of a few sizes: many equal remainders, which go to the
    earlier request (allocation.py:85)."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(29)
    for trial in range(4):
        n_req = int(rng.integers(1500, 2500))
        sizes = rng.choice([3, 7, 12, 40], n_req)
        scores = [rng.integers(0, 3, n).astype(np.float64) for n in sizes]
        pinned = [oa.controller_pins(int(n), 1) for n in sizes]
        must = sum(int(p.sum()) for p in pinned)
        budget = int(rng.integers(must + 1, int(sizes.sum())))
        got = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)], budget, "uniform")
        want = oa.allocate(scores, budget, "uniform", pinned)
        for r, (a, b) in enumerate(zip(got, want, strict=True)):
            np.testing.assert_array_equal(a, b, err_msg=f"trial {trial}, request {r}")


def test_maxmin_matches_the_reference_and_the_oracle():
    """The water level: the reference's own allocate(..., "maxmin") on 50 cases, then larger requests with
    ties and requests without evidence against the oracle."""
    from ekv.observe.allocation import Request, allocate

    g = load_golden("maxmin_cases")
    for i in range(50):
        sizes = g[f"sizes{i}"]
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        scores = [g[f"scores{i}"][bounds[j] : bounds[j + 1]] for j in range(len(sizes))]
        pinned = [oa.controller_pins(int(n), int(g[f"recent{i}"])) for n in sizes]
        masks = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)],
                         int(g[f"budget{i}"]), "maxmin")
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")
    rng = np.random.default_rng(59)
    for trial in range(12):
        n_req = int(rng.integers(2, 120))
        sizes = rng.integers(1, 700, n_req)
        if trial % 2:
            scores = [rng.integers(0, 3, n).astype(np.float64) for n in sizes]
        else:
            scores = [(rng.random(n) ** 2).astype(np.float32).astype(np.float64) for n in sizes]
        scores[0][:] = 0.0 if trial % 3 == 0 else scores[0]
        pinned = [oa.controller_pins(int(n), int(rng.integers(0, 5))) for n in sizes]
        must = sum(int(p.sum()) for p in pinned)
        budget = int(rng.integers(must, int(sizes.sum())))
        got = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)], budget, "maxmin")
        want = oa.allocate(scores, budget, "maxmin", pinned)
        for r, (a, b) in enumerate(zip(got, want, strict=True)):
            np.testing.assert_array_equal(a, b, err_msg=f"trial {trial}, request {r}")


def water_leftover(scores, pinned, budget):
    """Blocks the water level leaves over for the heap (allocation.py:121-160), as the oracle computes it."""
    shares = [oa.shares(s) for s in scores]
    order = [np.flatnonzero(~p)[np.argsort(-shares[r][~p], kind="stable")] for r, p in enumerate(pinned)]
    base = np.array([float(shares[r][p].sum()) for r, p in enumerate(pinned)])
    prefix = [np.cumsum(shares[r][order[r]]) for r in range(len(scores))]
    stacked = np.concatenate([p + 2.0 * r for r, p in enumerate(prefix)])
    sizes = np.array([len(o) for o in order])
    starts = np.concatenate(([0], np.cumsum(sizes)[:-1]))
    offsets = 2.0 * np.arange(len(scores))
    free = budget - sum(int(p.sum()) for p in pinned)

    def extra(level):
        need = level - base
        position = np.searchsorted(stacked, need - 1e-12 + offsets) - starts
        return np.where(need <= 1e-12, 0, np.minimum(position + 1, sizes))

    low, high = 0.0, 1.0
    for _ in range(60):
        mid = (low + high) / 2
        if int(extra(mid).sum()) <= free:
            low = mid
        else:
            high = mid
    return free - int(extra(low).sum())


def test_maxmin_leftover_blocks_by_argmin_and_by_heap():
    """Requests that reach the water level together leave blocks over: a few go out one block-wide argmin
    at a time, many through the heap; both give the reference's order (lowest retained share, then the
    earlier request)."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(71)
    one = rng.random(50)
    scores = [one.copy() for _ in range(240)]
    pinned = [oa.controller_pins(len(x), 2) for x in scores]
    must = sum(int(p.sum()) for p in pinned)
    seen = set()
    for budget in range(must + 2400, must + 2640, 9):
        left = water_leftover(scores, pinned, budget)
        seen.add("none" if left == 0 else ("few" if left <= 64 else "many"))
        got = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)], budget, "maxmin")
        want = oa.allocate(scores, budget, "maxmin", pinned)
        for r, (a, b) in enumerate(zip(got, want, strict=True)):
            np.testing.assert_array_equal(a, b, err_msg=f"budget {budget} ({left} left over), request {r}")
    assert {"few", "many"} <= seen, seen


def test_plan_view_maxmin_at_the_view_stress_size_matches_the_controller():
    """1024 requests of up to 8192 blocks (the bench's shape): every bisection stage, searches over
    whole rows and the full sort, against the oracle's controller pipeline."""
    from ekv.runtime.block_view import plan_view

    rng = np.random.default_rng(73)
    rows, width = 1024, 8192
    row_blocks = rng.integers(1, width + 1, rows).astype(np.int32)
    lens = (row_blocks * 16 - rng.integers(0, 16, rows)).astype(np.int32)
    table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
    scores = rng.dirichlet(np.full(width, 0.3), rows).astype(np.float32)
    scores[3, :] = 0.0  # a request without evidence: equal shares
    for fraction in (0.2, 0.5):
        keep = oa.controller_keep(row_blocks, width, lambda r, n: scores[r, :n].astype(np.float64), fraction,
                                  "maxmin", recent_blocks=4)
        mask = torch.empty(rows, width, dtype=torch.uint8).cuda()
        view, view_lens = plan_view(
            torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), 16, torch.from_numpy(row_blocks).cuda(),
            scores=torch.from_numpy(scores).cuda(), policy="maxmin", budget_fraction=fraction, recent_blocks=4,
            mask_out=mask)
        got = mask.cpu().numpy().astype(bool)
        inside = np.arange(width)[None, :] < row_blocks[:, None]
        np.testing.assert_array_equal(got & inside, keep.astype(bool) & inside, err_msg=f"fraction {fraction}")
        ref_view, ref_lens = ov.compact_block_table(table, lens, keep.astype(bool), 16)
        np.testing.assert_array_equal(view.cpu().numpy(), ref_view, err_msg=f"fraction {fraction}")
        np.testing.assert_array_equal(view_lens.cpu().numpy(), ref_lens, err_msg=f"fraction {fraction}")


def test_plan_view_maxmin_with_a_shared_budget_matches_the_controller():
    from ekv.runtime.block_view import plan_view

    rng = np.random.default_rng(67)
    for trial in range(6):
        rows, width = int(rng.integers(1, 80)), int(rng.integers(8, 600))
        row_blocks = rng.integers(0, width + 1, rows).astype(np.int32)
        lens = (row_blocks * 16 - rng.integers(0, 16, rows)).clip(0).astype(np.int32)
        table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
        scores = rng.dirichlet(np.full(width, 0.3), rows).astype(np.float32)
        fraction = float(rng.choice([0.2, 0.5, 0.8]))
        keep = oa.controller_keep(row_blocks, width, lambda r, n: scores[r, :n].astype(np.float64), fraction, "maxmin",
                                  recent_blocks=4)
        mask = torch.empty(rows, width, dtype=torch.uint8).cuda()
        view, view_lens = plan_view(
            torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), 16, torch.from_numpy(row_blocks).cuda(),
            scores=torch.from_numpy(scores).cuda(), policy="maxmin", budget_fraction=fraction, recent_blocks=4,
            mask_out=mask)
        got_mask = mask.cpu().numpy()
        for r in range(rows):
            n = min(int(row_blocks[r]), width)
            np.testing.assert_array_equal(got_mask[r, :n], keep[r, :n], err_msg=f"trial {trial} row {r}")
        ref_view, ref_lens = ov.compact_block_table(table, lens, keep.astype(bool), 16)
        np.testing.assert_array_equal(view.cpu().numpy(), ref_view, err_msg=f"trial {trial}")
        np.testing.assert_array_equal(view_lens.cpu().numpy(), ref_lens, err_msg=f"trial {trial}")


def test_sum_over_many_requests_against_the_oracle():
    """The global greedy: ties across requests (newer block, then earlier request), weights, requests
    without evidence, and budgets from just above the pins to just below every block."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(17)
    for trial in range(60):
        n_req = int(rng.integers(2, 40))
        sizes = rng.integers(1, 400, n_req)
        kind = trial % 3
        scores = []
        for n in sizes:
            if kind == 0:
                scores.append(rng.integers(0, 3, n).astype(np.float64))  # many ties
            else:
                scores.append((rng.random(n) ** 3).astype(np.float32).astype(np.float64))
        if trial % 4 == 0:
            scores[int(rng.integers(0, n_req))][:] = 0.0  # no evidence: equal shares 1/n
        weights = [1.0] * n_req if trial % 2 else [float(rng.choice([0.0, 0.5, 1.0, 2.0, 3.0])) for _ in range(n_req)]
        recent = int(rng.integers(0, 6))
        pinned = [oa.controller_pins(len(x), recent) for x in scores]
        must = sum(int(p.sum()) for p in pinned)
        total = int(sizes.sum())
        budget = int(rng.choice([must, must + 1, (must + total) // 2, total - 1, int(rng.integers(must, total + 1))]))
        budget = max(budget, must)
        requests = [Request(scores=x, weight=w, pinned=p) for x, w, p in zip(scores, weights, pinned, strict=True)]
        got = allocate(requests, budget, "sum")
        want = oa.allocate(scores, budget, "sum", pinned, weights)
        for r, (a, b) in enumerate(zip(got, want, strict=True)):
            np.testing.assert_array_equal(a, b, err_msg=f"trial {trial}, request {r}")
        assert sum(int(m.sum()) for m in got) == min(budget, total)


def test_sum_totals_follow_numpys_pairwise_summation():
    """A request and a permutation of it hold the same scores but their float64 totals differ in the
    last bits with the summation order, which then decides the ranking of equal scores across the two;
    long rows exercise the pairwise tree above 128 values."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(23)
    order_sensitive = 0
    for trial in range(20):
        n = int(rng.integers(129, 6000))
        base = np.exp(rng.normal(0.0, 4.0, n)).astype(np.float32).astype(np.float64)  # a wide range of magnitudes
        scores = [base, rng.permutation(base), rng.permutation(base)]
        order_sensitive += len({float(np.sum(x)) for x in scores}) > 1
        pinned = [oa.controller_pins(n, 4) for _ in scores]
        must = sum(int(p.sum()) for p in pinned)
        budget = int(rng.integers(must + 1, 3 * n - 1))
        got = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)], budget, "sum")
        want = oa.allocate(scores, budget, "sum", pinned)
        for a, b in zip(got, want, strict=True):
            np.testing.assert_array_equal(a, b, err_msg=f"trial {trial}")
    assert order_sensitive >= 10  # the totals of permuted copies differ: the summation order matters


def test_pairwise_totals_of_rows_longer_than_8192_values():
    """Rows of 8193 to 32768 values, whose pairwise recursion is 8 or 9 levels deep: three permutations of one
    row hold the same scores, so which of their equal gains are kept follows the last bits of their float64
    totals. Float64 rows through allocate() (up to 16384 values), float32 rows through ekv_allocate_sum (up to
    32768), against the oracle."""
    import ekv._lib as L
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(29)
    order_sensitive = 0
    for n in (8193, 12001, 16384):
        base = np.exp(rng.normal(0.0, 4.0, n)).astype(np.float32).astype(np.float64)
        scores = [base, rng.permutation(base), rng.permutation(base)]
        order_sensitive += len({float(np.sum(x)) for x in scores}) > 1
        pinned = [oa.controller_pins(n, 4) for _ in scores]
        budget = int(rng.integers(sum(int(p.sum()) for p in pinned) + 1, 3 * n - 1))
        got = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)], budget, "sum")
        want = oa.allocate(scores, budget, "sum", pinned)
        for a, b in zip(got, want, strict=True):
            np.testing.assert_array_equal(a, b, err_msg=f"float64, {n} values")
    lib = L.load()
    for n in (16385, 24007, 32768):
        base = np.exp(rng.normal(0.0, 4.0, n)).astype(np.float32)
        rows = np.stack([base, rng.permutation(base), rng.permutation(base)])
        order_sensitive += len({float(np.sum(x.astype(np.float64))) for x in rows}) > 1
        pinned = [oa.controller_pins(n, 4) for _ in rows]
        must = sum(int(p.sum()) for p in pinned)
        budget = int(rng.integers(must + 1, 3 * n - 1))
        scores = torch.from_numpy(rows).cuda()
        row_blocks = torch.full((3,), n, dtype=torch.int32).cuda()
        quota = torch.empty(3, dtype=torch.int32).cuda()
        ws_bytes = int(lib.ekv_allocate_sum_workspace_bytes(3, n))
        ws = torch.empty(ws_bytes + 256, dtype=torch.uint8).cuda()
        rc = lib.ekv_allocate_sum(scores.data_ptr(), scores.stride(0), None, row_blocks.data_ptr(), None, 4, -1, 0.0,
                                  budget, 3, n, quota.data_ptr(), (ws.data_ptr() + 255) // 256 * 256, ws_bytes,
                                  L.current_stream())
        L.check(rc, "ekv_allocate_sum")
        want = oa.allocate([x.astype(np.float64) for x in rows], budget, "sum", pinned)
        want_quota = [int(m.sum()) - int(p.sum()) for m, p in zip(want, pinned, strict=True)]
        assert quota.cpu().tolist() == want_quota, f"float32, {n} values"
    assert order_sensitive >= 4  # the totals of permuted copies differ: the summation order matters


def test_plan_view_sum_with_a_shared_budget_matches_the_controller():
    """The controller's default objective: one budget over every measured row (cap, recent pins and
    unmeasured suffixes), then the view, against the oracle's controller and compaction."""
    from ekv.runtime.block_view import plan_view

    rng = np.random.default_rng(31)
    for trial in range(12):
        rows, width = int(rng.integers(1, 96)), int(rng.integers(8, 700))
        row_blocks = rng.integers(0, width + 1, rows).astype(np.int32)
        lens = (row_blocks * 16 - rng.integers(0, 16, rows)).clip(0).astype(np.int32)
        table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
        if trial % 2:
            scores = rng.integers(0, 4, (rows, width)).astype(np.float32)
        else:
            scores = rng.dirichlet(np.full(width, 0.3), rows).astype(np.float32)
        measured = rng.integers(0, width + 1, rows).astype(np.int32) if trial % 3 == 0 else None
        cap = int(rng.choice([0, 0, 5]))
        fraction = float(rng.choice([0.1, 0.25, 0.5, 0.9]))
        keep = oa.controller_keep(row_blocks, width, lambda r, n: scores[r, :n].astype(np.float64), fraction, "sum",
                                  recent_blocks=4, cap_above_blocks=cap, measured=measured)
        mask = torch.empty(rows, width, dtype=torch.uint8).cuda()
        view, view_lens = plan_view(
            torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), 16, torch.from_numpy(row_blocks).cuda(),
            scores=torch.from_numpy(scores).cuda(), policy="sum", budget_fraction=fraction, recent_blocks=4,
            cap_above_blocks=cap, measured=None if measured is None else torch.from_numpy(measured).cuda(),
            mask_out=mask)
        got_mask = mask.cpu().numpy()
        for r in range(rows):
            n = min(int(row_blocks[r]), width)
            np.testing.assert_array_equal(got_mask[r, :n], keep[r, :n], err_msg=f"trial {trial} row {r}")
        ref_view, ref_lens = ov.compact_block_table(table, lens, keep.astype(bool), 16)
        np.testing.assert_array_equal(view.cpu().numpy(), ref_view, err_msg=f"trial {trial}")
        np.testing.assert_array_equal(view_lens.cpu().numpy(), ref_lens, err_msg=f"trial {trial}")


def _greedy_masks(scores, pinned, free):
    """allocation.py:_greedy restated with NumPy for a large case (the oracle's per-cell sort is slow)."""
    open_blocks = [np.flatnonzero(~p) for p in pinned]
    index = np.concatenate(open_blocks)
    gain = np.concatenate([oa.shares(s)[b] for s, b in zip(scores, open_blocks, strict=True)])
    worst = -gain
    threshold = np.partition(worst, free - 1)[free - 1]
    selected = worst < threshold
    ties = np.flatnonzero(worst == threshold)
    selected[ties[np.argsort(-index[ties], kind="stable")][: free - int(selected.sum())]] = True
    kept, start = [p.copy() for p in pinned], 0
    for r, b in enumerate(open_blocks):
        kept[r][b[selected[start : start + len(b)]]] = True
        start += len(b)
    return kept


def test_sum_at_the_view_stress_size():
    """1024 requests of up to 8192 blocks under one budget (4.2 M gains), against NumPy."""
    from ekv.observe.allocation import sum_quotas
    from ekv.runtime.block_view import _view_build

    rng = np.random.default_rng(41)
    rows, width = 1024, 8192
    n = rng.integers(1, width + 1, rows)
    scores = np.zeros((rows, width), dtype=np.float32)
    for r in range(rows):
        scores[r, : n[r]] = rng.dirichlet(np.full(n[r], 0.3)).astype(np.float32)
    pinned = [oa.controller_pins(int(k), 4) for k in n]
    must = sum(int(p.sum()) for p in pinned)
    budget = max(must, int(math.ceil(0.3 * int(n.sum()))))
    want = _greedy_masks([scores[r, : n[r]].astype(np.float64) for r in range(rows)], pinned, budget - must)
    dev = torch.device("cuda")
    s_t = torch.from_numpy(scores).to(dev)
    nb = torch.from_numpy(n.astype(np.int32)).to(dev)
    quota = torch.empty(rows, dtype=torch.int32, device=dev)
    sum_quotas(s_t, nb, quota, measured=None, recent_blocks=4, cap_above_blocks=0, budget=budget)
    table = torch.zeros(rows, width, dtype=torch.int32, device=dev)
    mask = torch.empty(rows, width, dtype=torch.uint8, device=dev)
    _view_build(table, (nb * 16).contiguous(), 16, row_blocks=nb, quota=quota, measured=None, recent_blocks=4,
                scores=s_t, policy="sum", mask_out=mask)
    got = mask.cpu().numpy()
    for r in range(rows):
        np.testing.assert_array_equal(got[r, : n[r]].astype(bool), want[r], err_msg=f"row {r}")
    assert int(sum(int(got[r, : n[r]].sum()) for r in range(rows))) == budget


@pytest.mark.parametrize("name", ["audit_cfg1_fp16", "audit_layers_fp16", "audit_g8_bf16"])
def test_plan_view_matches_the_reference_controller_and_view(name):
    """The controller's uniform keep mask at budget 0.5 (recent_blocks 4) and the view, as the golden
    fixture's reference pipeline computed them from the reference shares."""
    from ekv.runtime.block_view import plan_view

    g = load_golden(name)
    rows, width = g["table"].shape
    table = torch.from_numpy(g["table"]).cuda()
    lens = torch.from_numpy(g["lens"]).cuda()
    scores = torch.from_numpy(np.nan_to_num(g["share_mean"], nan=0.0).astype(np.float32)).cuda()
    # the reference ranked the float64 shares; the float32 copies rank identically unless two shares
    # collapse to one float32 value, which the fixture does not contain
    f32 = np.nan_to_num(g["share_mean"], nan=0.0).astype(np.float32)
    keep_f32 = oa.controller_keep(g["row_blocks"], width, lambda r, n: f32[r, :n].astype(np.float64), 0.5, "uniform",
                                  recent_blocks=4)
    np.testing.assert_array_equal(keep_f32, g["keep"])
    mask = torch.empty(rows, width, dtype=torch.uint8).cuda()
    view, view_lens = plan_view(table, lens, 16, torch.from_numpy(g["row_blocks"].astype(np.int32)).cuda(),
                                scores=scores, policy="uniform", budget_fraction=0.5, recent_blocks=4, mask_out=mask)
    np.testing.assert_array_equal(mask.cpu().numpy(), g["keep"])
    np.testing.assert_array_equal(view.cpu().numpy(), g["view"])
    np.testing.assert_array_equal(view_lens.cpu().numpy(), g["view_lens"])


def test_keep_newest_gives_the_reference_answer():
    from ekv.runtime.block_view import plan_view

    table = torch.arange(12, dtype=torch.int32).reshape(1, 12).cuda() + 100
    lens = torch.tensor([160], dtype=torch.int32).cuda()
    mask = torch.empty(1, 12, dtype=torch.uint8).cuda()
    view, view_lens = plan_view(table, lens, 16, torch.tensor([10], dtype=torch.int32).cuda(), scores=None,
                                policy="newest", budget_fraction=0.5, recent_blocks=0, mask_out=mask)
    assert np.flatnonzero(mask.cpu().numpy()[0, :10]).tolist() == [0, 6, 7, 8, 9]
    assert view[0, :5].tolist() == [100, 106, 107, 108, 109] and view_lens.tolist() == [80]


def view_stress_inputs(rows, width, seed=0):
    """The view stress shape: 1..width blocks per row, ids from a 2^20 pool, Dirichlet(0.3) shares,
    per-row budget fractions in [0.2, 1.0]."""
    gen = torch.Generator().manual_seed(seed)
    n = torch.randint(1, width + 1, (rows,), generator=gen).to(torch.int32)
    table = torch.randint(0, 2**20, (rows, width), generator=gen, dtype=torch.int32)
    conc = torch.full((width,), 0.3, dtype=torch.float64)
    scores = torch.distributions.Dirichlet(conc).sample((rows,)).to(torch.float32)
    scores = torch.where(torch.arange(width)[None, :] < n[:, None].long(), scores, torch.zeros_like(scores))
    fraction = 0.2 + 0.8 * torch.rand(rows, generator=gen, dtype=torch.float64)
    lens = n * 16 - torch.randint(0, 16, (rows,), generator=gen, dtype=torch.int32)
    return table, n, lens, scores, fraction


@pytest.mark.parametrize("policy", ["sum", "uniform"])
def test_view_stress_rows_match_the_oracle(policy):
    """Per-row budgets (each row its own allocate call): 256 rows of width 8192 against the oracle."""
    from ekv.runtime.block_view import plan_view

    rows, width = 256, 8192
    table, n, lens, scores, fraction = view_stress_inputs(rows, width, seed=1 if policy == "sum" else 2)
    mask = torch.empty(rows, width, dtype=torch.uint8).cuda()
    view, view_lens = plan_view(table.cuda(), lens.cuda(), 16, n.cuda(), scores=scores.cuda(), policy=policy,
                                row_fraction=fraction.cuda(), recent_blocks=0, mask_out=mask)
    keep = oa.per_row_keep(n.numpy(), width, scores.numpy().astype(np.float64), fraction.numpy(), policy)
    np.testing.assert_array_equal(mask.cpu().numpy(), keep)
    ref_view, ref_lens = ov.compact_block_table(table.numpy(), lens.numpy(), keep, 16)
    np.testing.assert_array_equal(view.cpu().numpy(), ref_view)
    np.testing.assert_array_equal(view_lens.cpu().numpy(), ref_lens)


@pytest.mark.parametrize("policy", ["sum", "uniform"])
@pytest.mark.parametrize("with_mask", [False, True])
def test_wide_rows_of_equal_scores_match_the_oracle(policy, with_mask):
    """Rows of up to 8192 blocks whose scores take four values, so the threshold always falls among equal keys
    that span every warp's run of positions: which of them are kept (newer first under `sum`, older first
    under `uniform`) follows the oracle, with and without the committed mask written."""
    from ekv.runtime.block_view import plan_view

    rng = np.random.default_rng(11 if policy == "sum" else 12)
    rows, width = 96, 8192
    n = rng.integers(2000, width + 1, rows).astype(np.int32)
    n[:4] = [width, width - 1, 2049, 2048]
    table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
    scores = rng.integers(0, 4, (rows, width)).astype(np.float32)
    fraction = rng.uniform(0.05, 0.95, rows)
    lens = (n * 16 - rng.integers(0, 16, rows)).astype(np.int32)
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    mask = torch.empty(rows, width, dtype=torch.uint8).cuda() if with_mask else None
    view, view_lens = plan_view(dev(table), dev(lens), 16, dev(n), scores=dev(scores), policy=policy,
                                row_fraction=dev(fraction), recent_blocks=0, mask_out=mask)
    keep = oa.per_row_keep(n, width, scores.astype(np.float64), fraction, policy)
    if with_mask:
        np.testing.assert_array_equal(mask.cpu().numpy(), keep)
    ref_view, ref_lens = ov.compact_block_table(table, lens, keep, 16)
    np.testing.assert_array_equal(view.cpu().numpy(), ref_view)
    np.testing.assert_array_equal(view_lens.cpu().numpy(), ref_lens)


def test_wide_float64_requests_of_equal_scores_match_the_oracle():
    """The float64 ranking (allocate over one wide request, its gains ranked as float64 keys) with the
    threshold among equal gains spread over the whole row."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(13)
    for trial in range(6):
        objective = "sum" if trial % 2 else "uniform"
        n = int(rng.integers(3000, 8193))
        scores = rng.integers(0, 4, n).astype(np.float64)
        pinned = oa.controller_pins(n, int(rng.integers(0, 6)))
        budget = int(rng.integers(int(pinned.sum()) + 1, n))
        (got,) = allocate([Request(scores=scores, pinned=pinned)], budget, objective)
        (want,) = oa.allocate([scores], budget, objective, [pinned])
        np.testing.assert_array_equal(got, want, err_msg=f"trial {trial}")


@pytest.mark.parametrize("policy", ["sum", "uniform", "newest"])
def test_per_row_budgets_in_one_kernel_match_the_two_launch_path(policy):
    """ekv_view_build_fractions (quotas computed in the view kernel) against ekv_allocate_quotas followed by
    ekv_view_build: length caps, measured suffixes, recent pins, rows longer than the table, empty rows,
    full rows and released blocks, bit for bit."""
    import ekv._lib as L
    from ekv.runtime.block_view import _view_build, plan_view

    rng = np.random.default_rng({"sum": 3, "uniform": 4, "newest": 5}[policy])
    rows, width, cap, recent = 300, 1000, 16, 3
    row_blocks = rng.integers(0, 1100, rows).astype(np.int32)
    row_blocks[::13] = 0
    measured = (row_blocks - rng.integers(0, 40, rows)).clip(0).astype(np.int32)
    lens = (np.minimum(row_blocks, width) * 16 - rng.integers(0, 16, rows)).clip(0).astype(np.int32)
    table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
    scores = np.round(rng.dirichlet(np.full(width, 0.3), rows), 4).astype(np.float32)
    fraction = rng.uniform(0.1, 1.0, rows)
    full = (rng.random(rows) < 0.1).astype(np.uint8)
    released = (rng.random((rows, width)) < 0.05).astype(np.uint8)
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    args = dict(scores=dev(scores) if policy != "newest" else None, measured=dev(measured), recent_blocks=recent,
                full_rows=dev(full), released=dev(released))
    mask1 = torch.empty(rows, width, dtype=torch.uint8).cuda()
    view1, lens1 = plan_view(dev(table), dev(lens), 16, dev(row_blocks), policy=policy, row_fraction=dev(fraction),
                             cap_above_blocks=cap, mask_out=mask1, **args)
    quota = torch.empty(rows, dtype=torch.int32).cuda()
    rb, fr = dev(row_blocks), dev(fraction)  # held: the launches read them after this line
    rc = L.load().ekv_allocate_quotas(rb.data_ptr(), args["measured"].data_ptr(), recent, cap, 0.0, -1, fr.data_ptr(),
                                      L.POLICY_SUM, rows, width, quota.data_ptr(), L.current_stream())
    L.check(rc, "ekv_allocate_quotas")
    mask2 = torch.empty(rows, width, dtype=torch.uint8).cuda()
    view2, lens2 = _view_build(dev(table), dev(lens), 16, row_blocks=rb, quota=quota, policy=policy, mask_out=mask2,
                               **args)
    np.testing.assert_array_equal(mask1.cpu().numpy(), mask2.cpu().numpy())
    np.testing.assert_array_equal(view1.cpu().numpy(), view2.cpu().numpy())
    np.testing.assert_array_equal(lens1.cpu().numpy(), lens2.cpu().numpy())


@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_shared_sum_view_from_the_threshold_matches_quotas_and_ranking(dtype):
    """ekv_view_build_sum_budget (the select's threshold applied in the view kernel, no per-row ranking)
    against ekv_allocate_sum's quotas followed by the ranking view: length caps, measured suffixes, recent
    pins, weights, empty rows, full rows, released blocks and many equal scores, bit for bit."""
    from ekv.observe.allocation import sum_quotas
    from ekv.runtime.block_view import _view_build, plan_view

    rng = np.random.default_rng({"float32": 7, "float64": 8}[dtype])
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    for trial in range(6):
        rows, width = int(rng.integers(1, 300)), int(rng.integers(8, 1200))
        row_blocks = rng.integers(0, width + 100, rows).astype(np.int32)
        row_blocks[:: 11] = 0
        measured = (row_blocks - rng.integers(0, 40, rows)).clip(0).astype(np.int32) if trial % 2 else None
        lens = (np.minimum(row_blocks, width) * 16 - rng.integers(0, 16, rows)).clip(0).astype(np.int32)
        table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
        scores = rng.dirichlet(np.full(width, 0.3), rows)
        if trial % 3 == 0:
            scores = np.round(scores, 3)  # many equal gains: the threshold falls among ties
        scores = scores.astype(np.float32 if dtype == "float32" else np.float64)
        weights = rng.uniform(0.5, 2.0, rows) if trial % 2 == 0 else None
        full = (rng.random(rows) < 0.1).astype(np.uint8)
        released = (rng.random((rows, width)) < 0.05).astype(np.uint8)
        cap = int(rng.choice([0, 4]))
        fraction = float(rng.choice([0.1, 0.3, 0.6, 0.95]))
        args = dict(measured=None if measured is None else dev(measured), recent_blocks=3, full_rows=dev(full),
                    released=dev(released))
        w = None if weights is None else dev(weights)
        rb, sc = dev(row_blocks), dev(scores)
        mask1 = torch.empty(rows, width, dtype=torch.uint8).cuda()
        view1, lens1 = plan_view(dev(table), dev(lens), 16, rb, scores=sc, policy="sum", budget_fraction=fraction,
                                 cap_above_blocks=cap, weights=w, mask_out=mask1, **args)
        quota = torch.empty(rows, dtype=torch.int32).cuda()
        sum_quotas(sc, rb, quota, measured=args["measured"], recent_blocks=3, cap_above_blocks=cap,
                   budget_fraction=fraction, weights=w)
        mask2 = torch.empty(rows, width, dtype=torch.uint8).cuda()
        view2, lens2 = _view_build(dev(table), dev(lens), 16, row_blocks=rb, quota=quota, scores=sc, policy="sum",
                                   mask_out=mask2, weights=w, **args)
        np.testing.assert_array_equal(mask1.cpu().numpy(), mask2.cpu().numpy(), err_msg=f"trial {trial}")
        np.testing.assert_array_equal(view1.cpu().numpy(), view2.cpu().numpy(), err_msg=f"trial {trial}")
        np.testing.assert_array_equal(lens1.cpu().numpy(), lens2.cpu().numpy(), err_msg=f"trial {trial}")


def test_full_size_view_stress_properties():
    """1024 rows x 8192: the view is a permutation of the row, kept ids come first in their original
    order, the kept count is pins + quota, and the length formula holds."""
    from ekv.runtime.block_view import plan_view

    rows, width = 1024, 8192
    table, n, lens, scores, fraction = view_stress_inputs(rows, width)
    mask = torch.empty(rows, width, dtype=torch.uint8).cuda()
    view, view_lens = plan_view(table.cuda(), lens.cuda(), 16, n.cuda(), scores=scores.cuda(), policy="sum",
                                row_fraction=fraction.cuda(), recent_blocks=0, mask_out=mask)
    v, m, t = view.cpu().numpy(), mask.cpu().numpy().astype(bool), table.numpy()
    nn, fr = n.numpy(), fraction.numpy()
    for r in range(0, rows, 7):
        k = m[r] & (np.arange(width) < nn[r])
        k[0] = True
        k[nn[r] - 1] = True
        kept = int(k.sum())
        pins = 1 if nn[r] == 1 else 2
        budget = max(pins, math.ceil(fr[r] * nn[r]))
        assert kept == min(budget, nn[r]), r
        np.testing.assert_array_equal(v[r, :kept], t[r, k])
        np.testing.assert_array_equal(np.sort(v[r]), np.sort(t[r]))
        assert view_lens[r].item() == (kept - 1) * 16 + int(lens[r]) - (nn[r] - 1) * 16


def test_decode_view_policy_lease_audit_and_release():
    """The DecodeView contract: identity before a commit, the committed view while the lease lives,
    identity after expiry, a full read for an audited row, never a released block."""
    import time

    from ekv.runtime.block_view import DecodeView

    class Plane:
        def __init__(self):
            self.flags, self.selected = [], []

        def set(self, on):
            self.flags.append(on)

        def select(self, audited, token_start):
            self.selected.append(audited.copy())

    table = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8]], dtype=torch.int32).cuda()
    lens = torch.tensor([64, 48], dtype=torch.int32).cuda()
    decode = torch.ones(2, dtype=torch.int32)
    mask = np.array([[1, 0, 0, 1], [1, 1, 0, 0]], dtype=np.uint32)
    hour = 3600 * 10**9

    view = DecodeView(rows=2, width=4, block_size=16)
    t, n = view.build(table, lens, decode)
    assert t.tolist() == table.tolist() and n.tolist() == [64, 48]
    view.write_row_controls(mask)
    view.write_lease_deadline(time.monotonic_ns() + hour)
    t, n = view.build(table, lens, decode)
    assert t[0, :2].tolist() == [1, 4] and n.tolist() == [32, 48]
    assert t[1, :3].tolist() == [5, 6, 7]
    view.write_lease_deadline(time.monotonic_ns() - 1)
    t, n = view.build(table, lens, decode)
    assert n.tolist() == [64, 48]
    # the build before any commit and the one after expiry both read without a live policy: 7 + 7
    assert view.read_breakdown()["expired"] == 14

    plane = Plane()
    view = DecodeView(rows=2, width=4, block_size=16, audit=plane)
    view.write_row_controls(mask)
    view.write_lease_deadline(time.monotonic_ns() + hour)
    view.write_audit_rows(np.array([True, False]))
    t, n = view.build(table, lens, decode)
    assert n.tolist() == [64, 48] and plane.flags[-1] is True and plane.selected[-1].tolist() == [True, False]
    t, n = view.build(table, lens, decode)  # the audit request was consumed
    assert n.tolist() == [32, 48] and plane.flags[-1] is False
    assert view.audits_completed == 1 and view.audited_blocks[0] == 4
    new = view.write_release(np.array([[0, 1, 1, 1], [0, 1, 0, 0]]))
    assert new == [(0, 1), (0, 2)]  # block 0 and the last block at the audit are never released
    view.write_lease_deadline(time.monotonic_ns() - 1)
    t, n = view.build(table, lens, decode)
    assert t[0, :2].tolist() == [1, 4] and n.tolist() == [32, 48]  # expired, yet released blocks stay out
    prefill = torch.tensor([1, 5], dtype=torch.int32)
    view.write_lease_deadline(time.monotonic_ns() + hour)
    t, n = view.build(table, lens, prefill)
    assert n.tolist() == [32, 48]  # row 1 prefills: it reads in full


def test_decode_view_counters_follow_the_reference_count():
    """Thirty builds with new masks, live and expired leases, audits, prefill rows and released blocks: the
    view against the oracle's keep algebra and compaction, and the five read counters against
    DecodeView._count's formulas (runtime/block_view.py:297-329)."""
    import time

    from ekv.runtime.block_view import DecodeView

    class Plane:
        def set(self, on):
            pass

        def select(self, audited, token_start):
            pass

    rng = np.random.default_rng(71)
    rows, width, bs = 48, 64, 16
    view = DecodeView(rows=rows, width=width, block_size=bs, audit=Plane())
    expected = np.zeros(5, dtype=np.int64)
    hour = 3600 * 10**9
    for step in range(30):
        n = int(rng.integers(1, rows + 1))
        lens = rng.integers(0, width * bs + 1, n).astype(np.int32)
        table = rng.integers(0, 1 << 20, (n, width)).astype(np.int32)
        query = np.where(rng.random(n) < 0.2, rng.integers(2, 9, n), 1).astype(np.int32)
        if step % 4 == 0:
            view.write_row_controls((rng.random((rows, width)) < 0.5).astype(np.uint8))
        live = step % 5 != 3
        view.write_lease_deadline(time.monotonic_ns() + (hour if live else -hour))
        if step % 3 == 0:
            view.write_audit_rows(rng.random(rows) < 0.2)
        if step == 10:
            freed = rng.random((rows, width)) < 0.1
            freed[:, 0] = False
            view.released = freed  # written to the device state
        t, vl = view.build(torch.from_numpy(table).cuda(), torch.from_numpy(lens).cuda(), torch.from_numpy(query))
        audited = view._pending_rows[:n]
        decoding = query == 1
        full = np.ones(n, dtype=bool) if not live else (audited | ~decoding)
        keep = ov.decode_keep(view.keep[:n], full, view.released[:n] if view.released.any() else None)
        ref_view, ref_lens = ov.compact_block_table(table, lens, keep, bs)
        np.testing.assert_array_equal(t.cpu().numpy(), ref_view, err_msg=f"step {step}")
        np.testing.assert_array_equal(vl.cpu().numpy(), ref_lens, err_msg=f"step {step}")
        read = -(-ref_lens.astype(np.int64) // bs) * decoding
        blocks = -(-lens.astype(np.int64) // bs) * decoding
        whole = ref_lens == lens
        expected += [read.sum(), blocks.sum(), (read * audited).sum(), (read * (whole & ~audited & live)).sum(),
                     0 if live else read.sum()]
        got = np.array(list(view.read_breakdown().values()), dtype=np.int64)
        np.testing.assert_array_equal(got, expected, err_msg=f"step {step}")
