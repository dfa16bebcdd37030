"""The C restatement of the audit (the timed CPU baseline) against the numpy oracle and the golden
vectors of the reference kernel. CPU only."""

from __future__ import annotations

import numpy as np
import pytest
from conftest import load_golden

from oracle import audit as oaud
from oracle import cpu


@pytest.fixture(scope="module", autouse=True)
def built():
    cpu.build()


@pytest.mark.parametrize("name", ["audit_cfg1_fp16", "audit_layers_fp16", "audit_g8_bf16"])
def test_c_restatement_matches_the_reference_kernel(name):
    g = load_golden(name)
    dtype = str(g["dtype"])
    q = g["query"].view(np.uint16) if dtype == "fp16" else g["query"]
    k = g["keys"].view(np.uint16) if dtype == "fp16" else g["keys"]
    layers = q.shape[0]
    rows, width = g["table"].shape
    lse = oaud.new_table(layers, rows, width, int(g["group_rows"]))
    for layer in range(layers):
        cpu.tile_lse(q[layer], k[layer], dtype, g["table"], g["lens"], g["qrow"], g["select"], int(g["flags"][layer]),
                     lse, float(g["scale"]), layer, layer % int(g["kv_heads"]), int(g["block_size"]),
                     int(g["tile_blocks"]))
    ref = g["lse"]
    assert np.array_equal(np.isnan(lse), np.isnan(ref))
    w = ~np.isnan(ref)
    np.testing.assert_allclose(lse[w], ref[w], rtol=2e-5, atol=2e-5)


def test_c_restatement_matches_the_numpy_oracle_on_a_strided_cache():
    rng = np.random.default_rng(3)
    rows, width, kv_heads, g_rows, pool = 5, 30, 4, 4, 200
    lens = rng.integers(0, width * 16, rows).astype(np.int32)
    table = rng.permutation(pool)[: rows * width].reshape(rows, width).astype(np.int32)
    kv = rng.standard_normal((pool, 2, 16, kv_heads, 128)).astype(np.float16)
    q = rng.standard_normal((rows + 2, kv_heads * g_rows, 128)).astype(np.float16)
    qrow = rng.permutation(rows + 2)[:rows].astype(np.int32)
    select = np.array([1, 1, 0, 1, 1], dtype=np.uint8)
    a = oaud.new_table(1, rows, width, g_rows)
    b = oaud.new_table(1, rows, width, g_rows)
    oaud.tile_lse(q, kv[:, 0], table, lens, qrow, select, 1, a, 0.088, 0, 3, 16, 2)
    cpu.tile_lse(q.view(np.uint16), kv.view(np.uint16)[:, 0], "fp16", table, lens, qrow, select, 1, b, 0.088, 0, 3, 16, 2)
    assert np.array_equal(np.isnan(a), np.isnan(b))
    w = ~np.isnan(a)
    np.testing.assert_allclose(a[w], b[w], rtol=2e-5, atol=2e-5)
