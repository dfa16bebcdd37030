"""Parity of the device normalisation (ekv_normalize_log_weights / ekv_normalize_tile_lse) with the
reference's normalize_tile_lse (golden vectors) and the oracle. Shares within 1e-3 relative (the
north-star bar; atol 1e-9 for shares that underflow differently); NaN rows bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch
from conftest import load_golden

from oracle import shares as osh

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-3, atol=1e-9)


def test_normalize_tile_lse_matches_the_reference_cases():
    from ekv.observe.tile_shares import normalize_tile_lse

    g = load_golden("shares_cases")
    for i in range(12):
        for aggregate in ("mean", "max"):
            got = normalize_tile_lse(g[f"u{i}"], g[f"rb{i}"], int(g[f"tb{i}"]), aggregate)
            ref = g[f"{aggregate}{i}"]
            assert got.dtype == np.float64 and got.shape == ref.shape
            assert np.array_equal(np.isnan(got), np.isnan(ref)), f"case {i} {aggregate}"
            np.testing.assert_allclose(got, ref, equal_nan=True, err_msg=f"case {i} {aggregate}", **TOL)


def test_device_tensors_stay_on_the_device():
    from ekv.observe.tile_shares import normalize_tile_lse

    g = load_golden("shares_cases")
    u = torch.from_numpy(g["u3"]).cuda()
    got = normalize_tile_lse(u, torch.from_numpy(g["rb3"]), int(g["tb3"]))
    assert got.is_cuda and got.dtype == torch.float32
    np.testing.assert_allclose(got.cpu().numpy(), g["mean3"], equal_nan=True, **TOL)


def test_known_answers_on_the_device():
    from ekv.observe.tile_shares import normalize_tile_lse

    u = np.full((1, 2, 4, 2), np.nan, dtype=np.float32)
    u[0, 0, :, 0] = [0.0, np.log(3.0), -np.inf, np.nan]
    got = normalize_tile_lse(u, np.array([4, 4]), 1)
    np.testing.assert_allclose(got[0], [0.25, 0.75, 0.0, 0.0], rtol=1e-6)
    assert np.isnan(got[1]).all()
    cells = np.repeat(np.log(np.array([1.0, 2.0, 5.0]) / 2), 2).astype(np.float32).reshape(1, 1, 6, 1)
    np.testing.assert_allclose(normalize_tile_lse(cells, np.array([5]), 2)[0], np.array([0.5, 0.5, 1, 1, 5, 0]) / 8,
                               rtol=1e-6)
    lse = np.log(np.array([[9.0, 1.0, 1.0], [1.0, 9.0, 1.0]])).T.astype(np.float32).reshape(1, 1, 3, 2)
    np.testing.assert_allclose(normalize_tile_lse(lse, np.array([3]), 1, "max")[0], np.array([9, 9, 1]) / 19, atol=1e-6)


def test_validation_raises_the_reference_exceptions():
    from ekv.observe.tile_shares import normalize_tile_lse

    with pytest.raises(ValueError):
        normalize_tile_lse(np.zeros((1, 1, 2, 1), np.float32), np.array([2]), 1, "median")
    with pytest.raises(ValueError):
        normalize_tile_lse(np.zeros((2, 3, 4), np.float32), np.array([1, 1, 1]), 1)
    with pytest.raises(ValueError):
        normalize_tile_lse(np.zeros((1, 3, 4, 1), np.float32), np.array([4, 4]), 1)


@pytest.mark.parametrize("aggregate", ["mean", "max"])
@pytest.mark.parametrize("tile_blocks", [1, 2, 4])
def test_table_shares_match_read_tile_rows_then_normalize(aggregate, tile_blocks):
    """The on-device read of a statistic table equals the reference read path on the same table."""
    from ekv.observe.tile_shares import table_shares

    rng = np.random.default_rng(tile_blocks)
    table_layers, layers, rows, width, cell = 5, 4, 9, 37, 8
    m = rng.normal(0, 3, (table_layers, rows, width, cell)).astype(np.float32)
    total = rng.uniform(1, 30, (table_layers, rows, width, cell)).astype(np.float32)
    m[rng.random(m.shape) < 0.05] = np.nan
    total[rng.random(total.shape) < 0.02] = 0.0
    m[:, 3] = np.nan  # a row never written
    lse = np.stack([m, total])
    row_ids = np.array([0, 2, 3, 4, 7, 8])
    row_blocks = np.array([37, 11, 20, 0, 45, 1])
    share, count = table_shares(torch.from_numpy(lse).cuda(), layers, row_ids, row_blocks, tile_blocks, aggregate,
                                contributors=True)
    u = osh.log_weights(lse, layers, row_ids, tile_blocks)
    ref = osh.normalize(u, row_blocks, tile_blocks, aggregate)
    got = share.cpu().numpy().astype(np.float64)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got, ref, equal_nan=True, **TOL)
    np.testing.assert_array_equal(count.cpu().numpy(), osh.contributors(u, row_blocks, tile_blocks))


def test_share_finalize_matches_the_fused_finalisation():
    import ekv._lib as L

    rng = np.random.default_rng(4)
    rows, width = 6, 50
    acc = torch.from_numpy(rng.uniform(0, 3, (rows, width)).astype(np.float32)).cuda()
    contrib = torch.tensor([4, 0, 4, 8, 4, 4], dtype=torch.int32).cuda()
    select = torch.tensor([1, 1, 1, 1, 0, 1], dtype=torch.uint8).cuda()
    for aggregate, code in (("mean", L.AGG_MEAN), ("max", L.AGG_MAX)):
        out = torch.empty(rows, width).cuda()
        rc = L.load().ekv_share_finalize(acc.data_ptr(), contrib.data_ptr(), select.data_ptr(), rows, width, code,
                                         out.data_ptr(), L.current_stream())
        L.check(rc, "ekv_share_finalize")
        got = out.cpu().numpy()
        a, c = acc.cpu().numpy().astype(np.float64), contrib.cpu().numpy()
        for r in range(rows):
            if c[r] == 0 or r == 4:
                assert np.isnan(got[r]).all()
            elif aggregate == "mean":
                np.testing.assert_allclose(got[r], a[r] / c[r], rtol=1e-6)
            else:
                np.testing.assert_allclose(got[r], a[r] / a[r].sum(), rtol=1e-5)
