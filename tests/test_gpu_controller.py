"""Parity of the controller's decide stage on the device with the reference: allocate() on float64 scores,
the per-request share ledger (the fold of each audit, its smoothing and the committed keep mask) over
a sequence of audits run through the reference Controller, and the read of another process's
statistic table over IPC. Bit-exact throughout."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch
from conftest import ROOT, load_golden
from test_oracle_golden import controller_setups, controller_weight

from oracle import allocation as oa
from oracle import controller as oc
from oracle import view as ov

pytestmark = pytest.mark.gpu


def test_allocate_on_float64_scores_matches_the_reference():
    """Shares that round together tie, weighted gains that round together tie: every objective."""
    from ekv.observe.allocation import Request, allocate

    g = load_golden("float64_cases")
    for i in range(90):
        sizes = g[f"sizes{i}"]
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        requests = [
            Request(scores=g[f"scores{i}"][bounds[j] : bounds[j + 1]], weight=float(g[f"weights{i}"][j]),
                    pinned=oa.controller_pins(int(n), int(g[f"recent{i}"])))
            for j, n in enumerate(sizes)
        ]
        masks = allocate(requests, int(g[f"budget{i}"]), str(g[f"objective{i}"]))
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")


def test_allocate_with_pins_anywhere_matches_the_reference():
    """allocate() with Request.pinned marking any blocks (observe/allocation.py:37-75): the reference's own
    outputs over 120 cases of every objective, bit for bit (ekv_allocate_pinned_f64)."""
    from ekv.observe.allocation import Request, allocate

    g = load_golden("pinned_cases")
    paths = set()
    for i in range(120):
        sizes = g[f"sizes{i}"]
        bounds = np.concatenate([[0], np.cumsum(sizes)])
        requests = [
            Request(scores=g[f"scores{i}"][bounds[j] : bounds[j + 1]], weight=float(g[f"weights{i}"][j]),
                    pinned=g[f"pinned{i}"][bounds[j] : bounds[j + 1]])
            for j in range(len(sizes))
        ]
        masks = allocate(requests, int(g[f"budget{i}"]), str(g[f"objective{i}"]))
        np.testing.assert_array_equal(np.concatenate(masks), g[f"mask{i}"], err_msg=f"case {i}")
        paths.add(str(g[f"objective{i}"]))
    assert paths == {"sum", "uniform", "maxmin"}


@pytest.mark.parametrize("objective", ["sum", "uniform", "maxmin"])
def test_allocate_with_random_pins_at_larger_sizes_matches_the_oracle(objective):
    """Beyond the fixture's sizes: 40 requests of up to 3000 blocks, pins anywhere, near-tied scores."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(5 + len(objective))
    sizes = rng.integers(1, 3001, 40)
    scores = [np.round(rng.random(n), 3) for n in sizes]  # three decimals: many exact ties
    pinned = [rng.random(n) < rng.choice([0.0, 0.05, 0.5]) for n in sizes]
    weights = rng.choice([1.0, 0.5, 2.0], len(sizes)) if objective == "sum" else np.ones(len(sizes))
    must = sum(int(p.sum()) for p in pinned)
    for budget in (must, (must + int(sizes.sum())) // 2, int(sizes.sum()) - 1):
        want = oa.allocate(scores, budget, objective, pinned, list(weights))
        got = allocate([Request(scores=s, weight=float(w), pinned=p) for s, w, p in zip(scores, weights, pinned,
                                                                                           strict=True)],
                       budget, objective)
        np.testing.assert_array_equal(np.concatenate(got), np.concatenate(want), err_msg=f"budget {budget}")


def run_ledger(g, c, fresh_dtype=torch.float64):
    from ekv.observe.controller import ShareLedger, audit_row_blocks

    objective, fraction, recent, decay, cap = controller_setups(g)[c]
    width = int(g["width"])
    ledger = ShareLedger(width, capacity=4, share_decay=decay)  # small: the ledger grows as requests arrive
    for step in range(int(g["steps"])):
        keys, lengths, audit_keys = g[f"keys{step}"], g[f"lengths{step}"], g[f"audit_keys{step}"]
        live, row_blocks = audit_row_blocks(audit_keys, keys, lengths, cap)
        fresh = g[f"fresh{step}"][:live].copy()
        fresh[row_blocks <= 0] = np.nan  # rows the source does not read
        ledger.absorb(torch.from_numpy(fresh).to(fresh_dtype).cuda(), audit_keys, row_blocks)
        ledger.forget(keys)
        keep = ledger.keep_mask(keys, lengths, budget_fraction=fraction, objective=objective, recent_blocks=recent,
                                cap_above_blocks=cap, weight=controller_weight if objective == "sum" else None)
        yield step, ledger, keep.cpu().numpy()


@pytest.mark.parametrize("c", range(4))
def test_share_ledger_follows_the_reference_controller(c):
    """Audit after audit: the smoothed shares, the measured lengths and the committed keep mask."""
    g = load_golden("controller_cases")
    width = int(g["width"])
    for step, ledger, keep in run_ledger(g, c):
        ks = sorted(ledger.slots)
        np.testing.assert_array_equal(np.array(ks, dtype=np.uint64), g[f"share_keys{c}_{step}"])
        got = np.array([ledger.shares(k) for k in ks]).reshape(len(ks), width)
        np.testing.assert_array_equal(got, g[f"shares{c}_{step}"], err_msg=f"setup {c} step {step}")
        np.testing.assert_array_equal([ledger.measured[k] for k in ks], g[f"measured{c}_{step}"])
        np.testing.assert_array_equal(keep, g[f"keep{c}_{step}"], err_msg=f"setup {c} step {step}")


def test_share_ledger_folds_float32_shares_and_a_key_met_twice():
    """The device's own float32 shares are folded exactly as their float64 values; a key on two rows of
    one audit folds twice, in row order, as the reference's loop does."""
    from ekv.observe.controller import ShareLedger

    rng = np.random.default_rng(5)
    width, rows = 300, 12
    keys = rng.integers(1, 2**63, 8, dtype=np.uint64)
    ledger = ShareLedger(width, capacity=2, share_decay=0.375)
    ref = oc.Ledger(width, 0.375)
    for step in range(6):
        audit_keys = keys[rng.integers(0, len(keys), rows)]
        audit_keys[rng.random(rows) < 0.2] = 0
        audit_keys[3] = audit_keys[7] = keys[step % len(keys)]  # the same request on two rows
        fresh = rng.dirichlet(np.full(width, 0.5), rows).astype(np.float32)
        fresh[rng.random((rows, width)) < 0.1] = np.nan
        fresh[rng.random(rows) < 0.2] = np.nan  # rows without evidence
        fresh[1, 5] = np.inf
        row_blocks = rng.integers(1, width, rows)
        updated = ledger.absorb(torch.from_numpy(fresh).cuda(), audit_keys, row_blocks)
        ref.absorb(fresh.astype(np.float64), audit_keys, row_blocks)
        assert set(updated) <= set(ref.shares)
        assert sorted(ledger.slots) == sorted(ref.shares)
        for k in ref.shares:
            np.testing.assert_array_equal(ledger.shares(k), ref.shares[k], err_msg=f"step {step}")
            assert ledger.measured[k] == ref.measured[k]


@pytest.mark.parametrize("objective", ["sum", "maxmin", "uniform"])
def test_float64_views_at_scale_match_the_oracle(objective):
    """plan_view on float64 scores with one shared budget: 192 requests of up to 2048 blocks whose shares
    round together, weights that merge gains, the controller's pins and length cap."""
    from ekv.runtime.block_view import plan_view

    rng = np.random.default_rng({"sum": 1, "maxmin": 2, "uniform": 3}[objective])
    rows, width = 192, 2048
    blocks = rng.integers(1, width + 1, rows).astype(np.int32)
    blocks[::17] = 0
    scores = np.zeros((rows, width))
    for r in range(rows):
        base = np.repeat(rng.random(width // 4) ** 3, 4)  # runs of adjacent doubles
        scores[r] = base
        for k in range(1, 4):
            scores[r, k::4] = np.nextafter(scores[r, k - 1 :: 4], np.inf)
        scores[r, rng.random(width) < 0.05] = scores[r, 0]
    weights = rng.choice([1.0, 0.3, 1.7, 1.0 / 3.0], rows) if objective == "sum" else np.ones(rows)
    measured = (blocks - rng.integers(0, 8, rows)).clip(0).astype(np.int32)
    table = rng.integers(0, 1 << 20, (rows, width)).astype(np.int32)
    seq = (blocks.astype(np.int64) * 16 - rng.integers(0, 16, rows)).clip(0).astype(np.int32)
    fraction, recent, cap = 0.3, 4, 32
    mask = torch.empty(rows, width, dtype=torch.uint8, device="cuda")
    view, view_lens = plan_view(
        torch.from_numpy(table).cuda(), torch.from_numpy(seq).cuda(), 16, torch.from_numpy(blocks).cuda(),
        scores=torch.from_numpy(scores).cuda(), policy=objective, budget_fraction=fraction, recent_blocks=recent,
        cap_above_blocks=cap, measured=torch.from_numpy(measured).cuda(),
        weights=torch.from_numpy(weights).cuda() if objective == "sum" else None, mask_out=mask,
    )
    chosen = [r for r in range(rows) if blocks[r] > cap]
    pinned = [oa.controller_pins(int(blocks[r]), recent, int(measured[r])) for r in chosen]
    total = sum(int(blocks[r]) for r in chosen)
    budget = max(sum(int(p.sum()) for p in pinned), int(np.ceil(fraction * total)))
    masks = oa.allocate([scores[r, : blocks[r]] for r in chosen], budget, objective, pinned,
                        [weights[r] for r in chosen])
    keep = np.ones((rows, width), dtype=np.uint8)
    for r, m in zip(chosen, masks, strict=True):
        keep[r, : len(m)] = m
    np.testing.assert_array_equal(mask.cpu().numpy(), keep)
    if objective == "sum":  # the same mask straight from the global threshold, with no view launch
        from ekv.observe.allocation import sum_quotas

        direct = torch.empty(rows, width, dtype=torch.uint8, device="cuda")
        quota = torch.empty(rows, dtype=torch.int32, device="cuda")
        sc, rb, ms, wt = (torch.from_numpy(x).cuda() for x in (scores, blocks, measured, weights))
        sum_quotas(sc, rb, quota, measured=ms, recent_blocks=recent, cap_above_blocks=cap, budget_fraction=fraction,
                   weights=wt, mask_out=direct)
        np.testing.assert_array_equal(direct.cpu().numpy(), keep)
    ref_view, ref_lens = ov.compact_block_table(table, seq, keep.astype(bool), 16)
    np.testing.assert_array_equal(view.cpu().numpy(), ref_view)
    np.testing.assert_array_equal(view_lens.cpu().numpy(), ref_lens)


def test_device_share_source_reads_another_process_over_ipc(tmp_path, monkeypatch):
    """A controller process opens the serving process's table through its descriptor's IPC handles and
    computes, on its own device context, the same shares as the serving process's in-place read."""
    from ekv.observe.controller import DeviceShareSource
    from ekv.observe.tile_shares import share_descriptor, table_shares
    from ekv.runtime.audit_kernel import RecordingPlane

    monkeypatch.setenv("EKV_RUNTIME_DIR", str(tmp_path))
    rng = np.random.default_rng(9)
    layers, rows, width, kv_heads, q_heads = 2, 6, 24, 2, 8
    plane = RecordingPlane(layers, rows, width, q_heads // kv_heads, 16, deferred=False)
    caches = [torch.randn(200, 2, 16, kv_heads, 128, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    plane.attach([c.data_ptr() for c in caches])
    table = torch.from_numpy(rng.permutation(200)[: rows * width].reshape(rows, width).astype(np.int32)).cuda()
    lens = torch.from_numpy(rng.integers(1, width * 16, rows).astype(np.int32)).cuda()
    plane.select(np.ones(rows, dtype=bool), np.arange(rows))
    plane.set(True)
    for layer in range(layers):
        q = torch.randn(rows, q_heads, 128, device="cuda").to(torch.bfloat16)
        plane.record(f"layer.{layer}", table, lens, q, caches[layer], 0.088)
    torch.cuda.synchronize()
    row_blocks = ((lens.cpu().numpy() + 15) // 16).astype(np.int64)
    row_blocks[2] = 0  # a row the controller does not read
    own = DeviceShareSource(share_descriptor(plane.pid), plane.pid).read(rows, row_blocks).cpu().numpy()
    ids = np.where(row_blocks > 0, np.arange(rows), -1)
    expect = table_shares(plane.table(), layers, ids, row_blocks, 2).cpu().numpy()
    np.testing.assert_array_equal(own, expect)
    assert np.isnan(own[2]).all() and not np.isnan(own[0]).all()
    out = tmp_path / "shares.npy"
    child = textwrap.dedent(f"""
        import sys, numpy as np, torch
        sys.path[:0] = [{ROOT!r}, {os.path.join(ROOT, "sigmod-kvscope_b200")!r}]
        from ekv.observe.controller import DeviceShareSource
        from ekv.observe.tile_shares import share_descriptor
        source = DeviceShareSource(share_descriptor({plane.pid}), {plane.pid})
        shares = source.read({rows}, np.array({row_blocks.tolist()}))
        np.save({str(out)!r}, shares.cpu().numpy())
        print(source.layers(), flush=True)
        source.close()
    """)
    result = subprocess.run([sys.executable, "-c", child], capture_output=True, text=True, timeout=300,
                            env={**os.environ, "EKV_RUNTIME_DIR": str(tmp_path)})
    assert result.returncode == 0, result.stderr[-2000:]
    np.testing.assert_array_equal(np.load(out), expect)
    assert json.loads(result.stdout.strip().splitlines()[-1]) == layers


@pytest.mark.parametrize("objective,width", [("sum", 16384), ("uniform", 16384), ("maxmin", 8192)])
def test_float64_allocation_at_the_widest_rows(objective, width):
    """The float64 paths at their width limits (a row of scores staged whole in shared memory: 16384
    blocks for the view and `sum`, 8192 for `maxmin`), against the oracle."""
    from ekv.observe.allocation import Request, allocate

    rng = np.random.default_rng(width + len(objective))
    sizes = [width, width - 3, 1, 2, width // 3, 700]
    scores = []
    for n in sizes:
        x = np.repeat(rng.random((n + 3) // 4) ** 2, 4)[:n]
        x[1::4] = np.nextafter(x[1::4], np.inf)  # adjacent doubles: shares that round together
        scores.append(x)
    weights = [1.0, 0.3, 2.0, 1.0, 1.0 / 3.0, 1.7] if objective == "sum" else [1.0] * len(sizes)
    pinned = [oa.controller_pins(n, 4, n - 20) for n in sizes]
    must = sum(int(p.sum()) for p in pinned)
    for budget in (must, must + 5000, sum(sizes) - 7):
        got = allocate([Request(scores=x, weight=w, pinned=p) for x, w, p in zip(scores, weights, pinned, strict=True)],
                       budget, objective)
        want = oa.allocate(scores, budget, objective, pinned, weights)
        for r, (a, b) in enumerate(zip(got, want, strict=True)):
            np.testing.assert_array_equal(a, b, err_msg=f"budget {budget}, request {r}")


def test_fixed_scoring_rule_follows_the_reference_controller():
    """A controller with a fixed scoring rule (float64 scores no float32 holds, weights, recent pins, a
    length cap), step after step, against the reference Controller; and the other objectives against the
    oracle."""
    from ekv.observe.controller import fixed_keep_mask

    g = load_golden("controller_cases")
    width = int(g["width"])

    def rule(n):
        return np.sin(np.arange(n) * 0.37) + 1.0

    for step in range(int(g["steps"])):
        keys, lengths = g[f"keys{step}"], g[f"lengths{step}"]
        keep = fixed_keep_mask(keys, lengths, rule, width=width, budget_fraction=0.35, objective="sum",
                               recent_blocks=2, cap_above_blocks=4, weight=controller_weight)
        np.testing.assert_array_equal(keep.cpu().numpy(), g[f"fixed_keep{step}"], err_msg=f"step {step}")
        row_blocks = np.where(keys != 0, lengths, 0)
        for objective in ("maxmin", "uniform"):
            keep = fixed_keep_mask(keys, lengths, rule, width=width, budget_fraction=0.35, objective=objective,
                                   recent_blocks=2, cap_above_blocks=4)
            want = oa.controller_keep(row_blocks, width, lambda r, n: rule(n), 0.35, objective, recent_blocks=2,
                                      cap_above_blocks=4)
            np.testing.assert_array_equal(keep.cpu().numpy(), want, err_msg=f"step {step} {objective}")
