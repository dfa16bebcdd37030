"""Every cell and share of full-size audit steps against the C restatement of the reference kernel.

The benchmark's steps are checked whole, not sampled:

* the Llama-3.1-8B step (64 rows of U[1024, 8192] tokens, 32 layers, G = 4, layer l auditing KV head
  l % 8 as the reference samples), recorded both ways the plane offers: ``RecordingPlane.record`` per
  layer (deferred: a query stash per layer, every layer in one launch after the last) and
  ``record_step`` from resident queries;
* a Llama-3-70B-shaped all-heads step (G = 8, the 8 KV heads side by side: 64 query rows per cell,
  80 layers, lognormal lengths of median 2048 clipped to [64, 32768]) over as many rows as the host
  oracle finishes in a few seconds;
* the long-context configuration end to end: its shares, then the controller's uniform keep mask at
  budget 0.2 for rows above 256 blocks (4 recent blocks pinned) and the compacted view, bit for bit
  against the oracle's controller and compact_block_table fed the same shares.

Tolerances as in the other audit tests: cells rtol/atol 1e-4 with the same unwritten (NaN) cells,
shares rtol 1e-3 (atol 1e-9), masks, views and lengths exact. Pools hold just the blocks the rows
use, so each test needs a few GB of device memory; the value cache is never read, so each layer's
cache tensor lays the key pool at both K and V positions instead of holding a value pool.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import allocation as oa
from oracle import audit as oaud
from oracle import cpu as ocpu
from oracle import shares as osh
from oracle import view as oview

pytestmark = pytest.mark.gpu

LSE_TOL = dict(rtol=1e-4, atol=1e-4)
SHARE_TOL = dict(rtol=1e-3, atol=1e-9)
BLOCK, TILE_BLOCKS, DIM = 16, 2, 128
SCALE = 1 / math.sqrt(DIM)


@pytest.fixture(scope="module", autouse=True)
def built():
    ocpu.build()


@pytest.fixture
def runtime_dir(tmp_path, monkeypatch):
    monkeypatch.setenv("EKV_RUNTIME_DIR", str(tmp_path))
    return tmp_path


class Step:
    """Seeded inputs of one audit step on the device: key pools, block table, lengths, per-layer queries."""

    def __init__(self, lens: np.ndarray, q_heads: int, kv_heads: int, layers: int, pools: int, seed: int,
                 width: int | None = None) -> None:
        rng = np.random.default_rng(seed)
        self.rows, self.layers, self.kv_heads = len(lens), layers, kv_heads
        self.group_rows = q_heads // kv_heads
        self.lens = lens.astype(np.int32)
        blocks = -(-self.lens // BLOCK)
        self.width = int(width or blocks.max())
        self.pool = int(blocks.sum()) + 3
        ids = rng.permutation(self.pool)[: int(blocks.sum())].astype(np.int32)
        self.table_host = np.zeros((self.rows, self.width), dtype=np.int32)
        start = 0
        for r, n in enumerate(blocks):
            self.table_host[r, :n] = ids[start : start + n]
            start += n
        gen = torch.Generator(device="cuda").manual_seed(seed)
        self.keys = [torch.randn(self.pool, BLOCK, kv_heads, DIM, device="cuda", generator=gen).to(torch.bfloat16)
                     for _ in range(pools)]
        # [blocks, 2, block, heads, dim] with the value position laid over the keys (never read)
        self.caches = [k.as_strided((self.pool, 2, BLOCK, kv_heads, DIM), (k.stride(0), 0, *k.stride()[1:]))
                       for k in self.keys]
        self.tokens = self.rows + 3
        self.queries = [torch.randn(self.tokens, q_heads, DIM, device="cuda", generator=gen).to(torch.bfloat16)
                        for _ in range(layers)]
        self.qrow = rng.permutation(self.tokens)[: self.rows].astype(np.int32)
        self.table = torch.from_numpy(self.table_host).cuda()
        self.lens_t = torch.from_numpy(self.lens).cuda()

    def cache(self, layer: int) -> torch.Tensor:
        return self.caches[self.pool_of(layer)]

    def pool_of(self, layer: int) -> int:
        raise NotImplementedError


class RotatingStep(Step):
    """The reference's sampling: layer l audits KV head l % kv_heads of pool l // kv_heads, so every
    layer reads keys of its own (as the benchmark lays them out)."""

    def pool_of(self, layer: int) -> int:
        return (layer // self.kv_heads) % len(self.caches)


class CycledStep(Step):
    """All-heads mode: layer l reads every head of pool l % pools."""

    def pool_of(self, layer: int) -> int:
        return layer % len(self.caches)


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def oracle_rotating(s: Step) -> np.ndarray:
    """The C restatement over every layer: one KV head per layer, head layer % kv_heads. The layers that
    read one (pool, head) are run together, so each head's keys cross to the host once."""
    lse = oaud.new_table(s.layers, s.rows, s.width, s.group_rows)
    select = np.ones(s.rows, dtype=np.uint8)
    groups: dict[tuple[int, int], list[int]] = {}
    for layer in range(s.layers):
        groups.setdefault((s.pool_of(layer), layer % s.kv_heads), []).append(layer)
    for (pool, h), layers in groups.items():
        keys = u16(s.keys[pool][:, :, h : h + 1])
        for layer in layers:
            q = u16(s.queries[layer][:, h * s.group_rows : (h + 1) * s.group_rows])
            ocpu.tile_lse(q, keys, "bf16", s.table_host, s.lens, s.qrow, select, 1, lse, SCALE, layer, 0, BLOCK,
                          TILE_BLOCKS)
    return lse


def oracle_all_heads(s: Step) -> np.ndarray:
    """The C restatement per (layer, KV head), each head's G query rows at its place in the cell."""
    g = s.group_rows
    lse = oaud.new_table(s.layers, s.rows, s.width, s.kv_heads * g)
    one = oaud.new_table(1, s.rows, s.width, g)
    select = np.ones(s.rows, dtype=np.uint8)
    for p in range(len(s.keys)):
        keys = u16(s.keys[p])
        for layer in range(p, s.layers, len(s.keys)):
            q = u16(s.queries[layer])
            for h in range(s.kv_heads):
                one.fill(np.nan)
                ocpu.tile_lse(q, keys, "bf16", s.table_host, s.lens, s.qrow, select, 1, one, SCALE, 0, h, BLOCK,
                              TILE_BLOCKS)
                lse[:, layer, :, :, h * g : (h + 1) * g] = one[:, 0]
    return lse


def check_cells(table: torch.Tensor, ref: np.ndarray) -> None:
    """The device table [2, layers, rows, width, cell] against the oracle's, a few layers at a time."""
    for first in range(0, ref.shape[1], 8):
        got, want = table[:, first : first + 8].cpu().numpy(), ref[:, first : first + 8]
        assert np.array_equal(np.isnan(got), np.isnan(want)), f"layers {first}+: the written cells differ"
        w = ~np.isnan(want)
        np.testing.assert_allclose(got[w], want[w], err_msg=f"layers {first}+", **LSE_TOL)


def oracle_shares(ref: np.ndarray, lens: np.ndarray) -> np.ndarray:
    rows = ref.shape[2]
    u = osh.log_weights(ref, ref.shape[1], np.arange(rows), TILE_BLOCKS)
    return osh.normalize_rows(u, -(-lens // BLOCK), TILE_BLOCKS)


def check_shares(got: torch.Tensor, want: np.ndarray) -> None:
    share = got.cpu().numpy().astype(np.float64)
    assert np.array_equal(np.isnan(share), np.isnan(want))
    np.testing.assert_allclose(share, want, equal_nan=True, **SHARE_TOL)


def llama8b_lens(rows: int = 64, seed: int = 0) -> np.ndarray:
    return np.random.default_rng(seed).integers(1024, 8193, rows)


@pytest.mark.parametrize("path", ["record_per_layer_deferred", "record_step"])
def test_full_llama8b_step_matches_the_c_oracle(path, runtime_dir):
    from ekv.runtime.audit_kernel import RecordingPlane

    s = RotatingStep(llama8b_lens(), q_heads=32, kv_heads=8, layers=32, pools=4, seed=1)
    plane = RecordingPlane(s.layers, s.rows, s.width, s.group_rows, BLOCK, deferred=path != "record_step")
    plane.attach([s.cache(layer)[:, 0].data_ptr() for layer in range(s.layers)])
    plane.select(np.ones(s.rows, dtype=bool), s.qrow)
    plane.set(True)
    if path == "record_step":
        plane.record_step(s.table, s.lens_t, s.queries, [s.cache(layer) for layer in range(s.layers)], SCALE)
    else:
        for layer in range(s.layers):
            plane.record(f"model.layers.{layer}.attn", s.table, s.lens_t, s.queries[layer], s.cache(layer), SCALE)
    torch.cuda.synchronize()
    assert plane.status() == 0
    ref = oracle_rotating(s)
    check_cells(plane.table(), ref)
    check_shares(plane.shares(), oracle_shares(ref, s.lens))


def test_llama70b_all_heads_step_matches_the_c_oracle(runtime_dir):
    from ekv.runtime.audit_kernel import RecordingPlane

    rng = np.random.default_rng(7)
    rows = 32
    lens = np.clip(np.round(rng.lognormal(math.log(2048), 1.0, rows)), 64, 32768).astype(np.int64)
    lens[0] = 64  # the clipped range's lower end
    s = CycledStep(lens, q_heads=64, kv_heads=8, layers=80, pools=4, seed=2)
    plane = RecordingPlane(s.layers, s.rows, s.width, s.group_rows, BLOCK, heads=s.kv_heads)
    plane.select(np.ones(s.rows, dtype=bool), s.qrow)
    plane.attach([s.cache(layer)[:, 0].data_ptr() for layer in range(s.layers)])
    plane.set(True)
    plane.record_step(s.table, s.lens_t, s.queries, [s.cache(layer) for layer in range(s.layers)], SCALE)
    torch.cuda.synchronize()
    assert plane.status() == 0
    ref = oracle_all_heads(s)
    check_cells(plane.table(), ref)
    check_shares(plane.shares(), oracle_shares(ref, s.lens))


@pytest.mark.parametrize("short_rows", [0, 2])
def test_long_context_view_end_to_end(short_rows, runtime_dir):
    """Config 3: 8 rows of 32k-128k tokens, shares, then the uniform view at budget 0.2 over the rows above
    256 blocks (keep-newest pins: block 0 and the 5 newest). ``short_rows`` adds rows at or below the cap,
    which the controller leaves unmeasured (read in full)."""
    from ekv.runtime.audit_kernel import RecordingPlane
    from ekv.runtime.block_view import plan_view

    rng = np.random.default_rng(11)
    lens = rng.integers(32768, 131073, 8)
    if short_rows:
        lens = np.concatenate([lens[:4], [256 * BLOCK, 100 * BLOCK - 5][:short_rows], lens[4:]])
    s = RotatingStep(lens, q_heads=32, kv_heads=8, layers=32, pools=1, seed=3, width=8192)
    plane = RecordingPlane(s.layers, s.rows, s.width, s.group_rows, BLOCK, deferred=False)
    plane.select(np.ones(s.rows, dtype=bool), s.qrow)
    plane.attach([s.cache(layer)[:, 0].data_ptr() for layer in range(s.layers)])
    plane.set(True)
    plane.record_step(s.table, s.lens_t, s.queries, [s.cache(layer) for layer in range(s.layers)], SCALE)
    torch.cuda.synchronize()
    assert plane.status() == 0
    ref = oracle_rotating(s)
    check_cells(plane.table(), ref)
    shares = plane.shares()
    check_shares(shares, oracle_shares(ref, s.lens))
    # the view, from the device's own shares (the view is a function of the scores it ranks)
    row_blocks = -(-s.lens // BLOCK)
    scores = torch.nan_to_num(shares, nan=0.0)
    mask = torch.empty(s.rows, s.width, dtype=torch.uint8, device="cuda")
    view, view_lens = plan_view(s.table, s.lens_t, BLOCK, torch.from_numpy(row_blocks.astype(np.int32)).cuda(),
                                scores=scores, policy="uniform", budget_fraction=0.2, recent_blocks=4,
                                cap_above_blocks=256, mask_out=mask)
    f32 = scores.cpu().numpy()
    keep = oa.controller_keep(row_blocks, s.width, lambda r, n: f32[r, :n].astype(np.float64), 0.2, "uniform",
                              recent_blocks=4, cap_above_blocks=256)
    np.testing.assert_array_equal(mask.cpu().numpy(), keep)
    want_view, want_lens = oview.compact_block_table(s.table_host, s.lens, keep.astype(bool), BLOCK)
    np.testing.assert_array_equal(view.cpu().numpy(), want_view)
    np.testing.assert_array_equal(view_lens.cpu().numpy(), want_lens)
    # the budget is spent exactly: the measured rows keep max(pins, ceil(0.2 * their blocks)) blocks
    measured = row_blocks > 256
    assert (keep[~measured] == 1).all()
    kept = sum(int(keep[r, : row_blocks[r]].sum()) for r in np.flatnonzero(measured))
    assert kept == max(6 * int(measured.sum()), math.ceil(0.2 * int(row_blocks[measured].sum())))
