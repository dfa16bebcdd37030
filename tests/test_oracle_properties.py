"""Size-independent properties of the oracle's `allocate` at sizes beyond the golden fixtures (CPU).

observe/allocation.py:55-166 defines what every objective keeps: all pinned blocks, exactly the budget
when it lies between the pins and the total, and, per objective, the unpinned blocks in a fixed order --
`sum` the globally largest weighted shares (equal gains: the newer block, then the earlier request,
:107-113), `uniform` and `maxmin` a prefix of each request's blocks by decreasing share (equal shares:
the older block first, :89, :129). These hold at any size, so they check the oracle where no golden
vector reaches.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import allocation as oa


def _case(rng, n_req, max_len, ties):
    sizes = rng.integers(1, max_len, n_req)
    if ties:
        scores = [rng.integers(0, 4, n).astype(np.float64) for n in sizes]
    else:
        scores = [(rng.random(n) ** 3).astype(np.float32).astype(np.float64) for n in sizes]
    scores[0][:] = 0.0  # a request without evidence: equal shares
    pinned = [oa.controller_pins(int(n), int(rng.integers(0, 5))) for n in sizes]
    must = sum(int(p.sum()) for p in pinned)
    budget = int(rng.integers(must, int(sizes.sum())))
    return scores, pinned, budget


def _prefix_by_share(score, pin, kept):
    """The kept unpinned blocks are the first ones by decreasing share, the older block first on ties."""
    s = oa.shares(score)
    free = np.flatnonzero(~pin)
    order = free[np.lexsort((free, -s[free]))]
    k = int(kept[free].sum())
    return bool(kept[order[:k]].all()) and not kept[order[k:]].any()


@pytest.mark.parametrize("objective", ["sum", "uniform", "maxmin"])
@pytest.mark.parametrize("ties", [False, True])
def test_oracle_allocation_keeps_the_pins_spends_the_budget_and_keeps_the_order(objective, ties):
    rng = np.random.default_rng(101 + 7 * ties + len(objective))
    for trial in range(4):
        scores, pinned, budget = _case(rng, int(rng.integers(50, 300)), 2000, ties)
        weights = rng.random(len(scores)) + 0.5 if objective == "sum" and trial % 2 else None
        kept = oa.allocate(scores, budget, objective, pinned, weights)
        assert sum(int(k.sum()) for k in kept) == budget, (objective, trial)
        for k, p in zip(kept, pinned, strict=True):
            assert k[p].all()
        if objective in ("uniform", "maxmin"):
            for r, (s, p, k) in enumerate(zip(scores, pinned, kept, strict=True)):
                assert _prefix_by_share(s, p, k), (objective, trial, r)
            continue
        # sum: every kept unpinned block comes before every dropped one in the order
        # (-gain, -block, request)
        w = np.ones(len(scores)) if weights is None else weights
        rows = []
        for r, (s, p, k) in enumerate(zip(scores, pinned, kept, strict=True)):
            free = np.flatnonzero(~p)
            g = w[r] * oa.shares(s)[free]
            rows.append(np.stack([-g, -free.astype(np.float64), np.full(free.size, r, np.float64),
                                  k[free].astype(np.float64)], axis=1))
        table = np.concatenate(rows)
        order = np.lexsort((table[:, 2], table[:, 1], table[:, 0]))
        flags = table[order, 3].astype(bool)
        n_kept = int(flags.sum())
        assert flags[:n_kept].all() and not flags[n_kept:].any(), (trial, weights is not None)


@pytest.mark.parametrize("objective", ["sum", "uniform", "maxmin"])
def test_oracle_controller_keep_spends_the_controller_budget(objective):
    """controller.py:420-437: measured rows (longer than the cap) share max(pins, ceil(f * blocks));
    every other row, and every position past a row's length, is kept."""
    rng = np.random.default_rng(211 + len(objective))
    rows, width = 256, 4096
    row_blocks = rng.integers(0, width + 1, rows).astype(np.int32)
    scores = rng.dirichlet(np.full(width, 0.3), rows).astype(np.float32)
    for fraction, cap in ((0.2, 0), (0.5, 64), (0.9, 0)):
        keep = oa.controller_keep(row_blocks, width, lambda r, n: scores[r, :n].astype(np.float64), fraction,
                                  objective, recent_blocks=4, cap_above_blocks=cap)
        chosen = (row_blocks > cap) & (row_blocks > 0)
        inside = np.arange(width)[None, :] < row_blocks[:, None]
        assert keep[~chosen].all() and keep[~inside].all()
        total = int(row_blocks[chosen].sum())
        pins = sum(int(oa.controller_pins(int(n), 4).sum()) for n in row_blocks[chosen])
        want = min(total, max(pins, int(np.ceil(fraction * total))))
        assert int(keep[inside & chosen[:, None]].sum()) == want, (fraction, cap)
