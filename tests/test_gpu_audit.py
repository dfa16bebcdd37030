"""Parity of the sm_100a audit kernel (tile LSE + fused shares) with the reference and the oracle.

Tolerances: the tile values m and l are float32 reductions of float32 dot products whose summation
order differs from the reference kernel's, so they agree to rtol 1e-4 / atol 1e-4; shares agree with
the reference normalisation to 1e-3 relative, with atol 1e-9 for shares that
underflow differently. Cells the reference leaves unwritten must be NaN here too (bit-exact pattern).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from conftest import load_golden

from oracle import audit as oaud
from oracle import shares as osh

pytestmark = pytest.mark.gpu

LSE_TOL = dict(rtol=1e-4, atol=1e-4)
SHARE_TOL = dict(rtol=1e-3, atol=1e-9)


def unpack(x: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "fp16":
        return torch.from_numpy(x.astype(np.float16))
    return torch.from_numpy((x.astype(np.uint32) << 16).view(np.float32)).to(torch.bfloat16)


@pytest.fixture
def runtime_dir(tmp_path, monkeypatch):
    monkeypatch.setenv("EKV_RUNTIME_DIR", str(tmp_path))
    return tmp_path


def run_plane_on_golden(g: dict, aggregate: str = "mean", deferred: bool = False):
    """The golden case through RecordingPlane: per layer (eager) or all layers after the last (deferred)."""
    from ekv.runtime.audit_kernel import RecordingPlane

    dtype = str(g["dtype"])
    q_all, k_all = unpack(g["query"], dtype), unpack(g["keys"], dtype)
    layers = q_all.shape[0]
    rows, width = g["table"].shape
    caches = []
    for layer in range(layers):
        k = k_all[layer].cuda()
        caches.append(torch.stack([k, torch.zeros_like(k)], dim=1))
    plane = RecordingPlane(layers, rows, width, int(g["group_rows"]), int(g["block_size"]), aggregate=aggregate,
                           deferred=deferred)
    plane.attach([c.data_ptr() for c in caches])
    plane.select(g["select"].astype(bool), g["qrow"])
    table = torch.from_numpy(g["table"]).cuda()
    lens = torch.from_numpy(g["lens"]).cuda()
    for layer in range(layers):
        if not deferred:
            plane.set(bool(g["flags"][layer]))
        elif layer == 0:
            plane.set(True)
        plane.record(f"layer.{layer}", table, lens, q_all[layer].cuda(), caches[layer], float(g["scale"]))
    torch.cuda.synchronize()
    return plane


@pytest.mark.parametrize("name", ["audit_cfg1_fp16", "audit_layers_fp16", "audit_g8_bf16"])
def test_recording_plane_matches_the_reference_kernel(name, runtime_dir):
    g = load_golden(name)
    plane = run_plane_on_golden(g)
    lse = plane.table().cpu().numpy()
    ref = g["lse"]
    assert np.array_equal(np.isnan(lse), np.isnan(ref)), "the written cells differ from the reference's"
    written = ~np.isnan(ref)
    np.testing.assert_allclose(lse[written], ref[written], **LSE_TOL)
    assert plane.status() == 0
    assert plane.layer_names == [f"layer.{i}" for i in range(ref.shape[1])]


@pytest.mark.parametrize("name", ["audit_cfg1_fp16", "audit_layers_fp16", "audit_g8_bf16"])
@pytest.mark.parametrize("aggregate", ["mean", "max"])
def test_fused_shares_match_the_reference_normalisation(name, aggregate, runtime_dir):
    g = load_golden(name)
    plane = run_plane_on_golden(g, aggregate)
    share = plane.shares().cpu().numpy().astype(np.float64)
    ref = g[f"share_{aggregate}"]
    assert np.array_equal(np.isnan(share), np.isnan(ref))
    np.testing.assert_allclose(share, ref, equal_nan=True, **SHARE_TOL)
    live = ~np.isnan(ref).all(axis=1)
    np.testing.assert_allclose(share[live].sum(axis=1), 1.0, rtol=1e-5)


@pytest.mark.parametrize("name", ["audit_cfg1_fp16", "audit_g8_bf16"])
@pytest.mark.parametrize("aggregate", ["mean", "max"])
def test_deferred_recording_matches_the_reference(name, aggregate, runtime_dir):
    """All layers in one launch after the last layer: the same cells and shares as the reference."""
    g = load_golden(name)
    plane = run_plane_on_golden(g, aggregate, deferred=True)
    lse = plane.table().cpu().numpy()
    ref = g["lse"]
    assert np.array_equal(np.isnan(lse), np.isnan(ref))
    w = ~np.isnan(ref)
    np.testing.assert_allclose(lse[w], ref[w], **LSE_TOL)
    share = plane.shares().cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(share, g[f"share_{aggregate}"], equal_nan=True, **SHARE_TOL)
    assert plane.status() == 0


def test_deferred_and_per_layer_recording_agree_bit_for_bit(runtime_dir):
    g = load_golden("audit_g8_bf16")
    eager = run_plane_on_golden(g, deferred=False)
    deferred = run_plane_on_golden(g, deferred=True)
    assert torch.equal(torch.nan_to_num(eager.table(), 3.0), torch.nan_to_num(deferred.table(), 3.0))
    assert torch.equal(torch.nan_to_num(eager.shares(), 3.0), torch.nan_to_num(deferred.shares(), 3.0))


def test_the_descriptor_is_published_in_the_reference_format(runtime_dir):
    from ekv.observe.tile_shares import share_descriptor
    from ekv.runtime.audit_kernel import RecordingPlane

    plane = RecordingPlane(2, 4, 8, 4, 16)
    d = share_descriptor(plane.pid)
    assert d["tile_lse_dev"] == plane._lse and d["ncap"] == 8 and d["max_rows"] == 4
    assert d["tile_lse_layers"] == 2 and d["tile_lse_group_rows"] == 4 and d["attn_share_tile_blocks"] == 2
    assert len(d["tile_lse_ipc"]) == 128 and len(d["layer_table_ipc"]) == 128
    assert np.isnan(plane.table().cpu().numpy()).all(), "a new table is all NaN"


def test_plane_validation_raises_the_reference_exceptions(runtime_dir):
    from ekv.runtime.audit_kernel import RecordingPlane

    with pytest.raises(ValueError):
        RecordingPlane(1, 2, 4, 17, 16)
    with pytest.raises(ValueError):
        RecordingPlane(1, 2, 4, 4, 12)
    plane = RecordingPlane(1, 2, 4, 4, 16, deferred=False)
    with pytest.raises(RuntimeError):
        plane.set(True)  # before the layer table is filled
    plane.attach([0x1000])
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(16, 2, 16, 2, 128, dtype=torch.bfloat16, device="cuda")
    table = torch.zeros(2, 4, dtype=torch.int32, device="cuda")
    lens = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        plane.record("a", table, lens, q, kv[:, :, :8], 0.1)  # block size differs
    with pytest.raises(ValueError):
        plane.record("a", table, lens, q[:, :6], kv, 0.1)  # group size differs
    plane.record("a", table, lens, q, kv, 0.1)
    with pytest.raises(RuntimeError):
        plane.record("b", table, lens, q, kv, 0.1)  # more layers than the plane holds


# ---- random cases through the C ABI against the oracle ------------------------------------------------


def random_case(seed, rows, width, q_heads, kv_heads, lens, dtype=torch.bfloat16, block_size=16, pool=None):
    gen = torch.Generator().manual_seed(seed)
    pool = pool or rows * width + 7
    tokens = rows + 5
    q = torch.randn(tokens, q_heads, 128, generator=gen).to(dtype)
    k = torch.randn(pool, block_size, kv_heads, 128, generator=gen).to(dtype)
    table = torch.randperm(pool, generator=gen)[: rows * width].reshape(rows, width).to(torch.int32)
    qrow = torch.randperm(tokens, generator=gen)[:rows].to(torch.int32)
    return q, k, table, torch.tensor(lens, dtype=torch.int32), qrow


class Run:
    """The device buffers of one audit step through the C ABI: table, workspace, shares, status."""

    def __init__(self, layers, rows, width, cell):
        import ekv._lib as L

        dev = torch.device("cuda")
        self.lse = torch.full((2, layers, rows, width, cell), float("nan"), device=dev)
        self.ws_bytes = L.load().ekv_audit_workspace_bytes(layers, rows, width)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.share = torch.full((rows, width), float("nan"), device=dev)
        self.contrib = torch.zeros(rows, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)


def launch(q, k, table, lens, qrow, select, flag_on, layers, layer, group_rows, heads=1, group=None,
           tile_blocks=2, aggregate="mean", finalize=None, run=None):
    """One ekv_audit_launch; returns (lse, (share, contributors), status) and keeps `run` for the step."""
    import ekv._lib as L

    lib = L.load()
    rows, width = table.shape
    block_size, kv_heads = k.shape[1], k.shape[2]
    dev = torch.device("cuda")
    run = run or Run(layers, rows, width, heads * group_rows)
    flag = torch.tensor([1 if flag_on else 0], dtype=torch.int32, device=dev)
    sel = torch.as_tensor(np.asarray(select, dtype=np.uint8)).to(dev)
    qd, kd, td, ld, rd = (x.to(dev) for x in (q, k, table, lens, qrow))
    if finalize is None:
        finalize = layer == layers - 1
    rc = lib.ekv_audit_launch(
        qd.data_ptr(), kd.data_ptr(), td.data_ptr(), ld.data_ptr(), rd.data_ptr(), sel.data_ptr(), flag.data_ptr(),
        run.lse.data_ptr(), 1 / math.sqrt(128), layer, layer % kv_heads if group is None else group,
        qd.stride(0), qd.stride(1), kd.stride(0), kd.stride(1), kd.stride(2), td.stride(0),
        layers, rows, width, group_rows, block_size, tile_blocks, 128,
        L.DTYPE_BF16 if q.dtype == torch.bfloat16 else L.DTYPE_F16, heads, kv_heads, kd.shape[0], qd.shape[0],
        run.share.data_ptr(), run.contrib.data_ptr(), L.AGG_MEAN if aggregate == "mean" else L.AGG_MAX,
        L.SHARE_FINALIZE if finalize else 0, run.ws.data_ptr(), run.ws_bytes, run.status.data_ptr(),
        L.current_stream(),
    )
    L.check(rc, "ekv_audit_launch")
    torch.cuda.synchronize()
    return run


def oracle_case(table, lens, qrow, select, layers_q, layers_k, group_rows, block_size, tile_blocks, heads=1,
                groups=None):
    rows, width = table.shape
    layers = len(layers_q)
    lse = oaud.new_table(layers, rows, width, heads * group_rows)
    for layer in range(layers):
        group = (layer % layers_k[layer].shape[2]) if groups is None else groups[layer]
        oaud.tile_lse(layers_q[layer].float().numpy(), layers_k[layer].float().numpy(), table.numpy(), lens.numpy(),
                      qrow.numpy(), np.asarray(select), 1, lse, 1 / math.sqrt(128), layer, group, block_size,
                      tile_blocks, heads)
    return lse


def compare_shares(lse_ref, lens, select, block_size, tile_blocks, got_share, aggregate="mean"):
    rows = len(lens)
    row_blocks = np.where(np.asarray(select) != 0, -(-np.asarray(lens) // block_size), 0)
    live = np.flatnonzero(row_blocks > 0)
    ref = np.full(got_share.shape, np.nan)
    if live.size:
        u = osh.log_weights(lse_ref, lse_ref.shape[1], live, tile_blocks)
        ref[live] = osh.normalize(u, row_blocks[live], tile_blocks, aggregate)
    got = got_share.astype(np.float64)
    assert np.array_equal(np.isnan(got), np.isnan(ref)), (np.isnan(got).sum(), np.isnan(ref).sum(), rows)
    np.testing.assert_allclose(got, ref, equal_nan=True, **SHARE_TOL)


@pytest.mark.parametrize(
    "q_heads, kv_heads, tile_blocks, dtype",
    [(32, 8, 2, torch.bfloat16), (64, 8, 2, torch.bfloat16), (8, 8, 2, torch.float16), (48, 4, 2, torch.bfloat16),
     (24, 8, 2, torch.float16), (32, 8, 1, torch.bfloat16), (32, 8, 4, torch.bfloat16)],
)
def test_random_rows_match_the_oracle(q_heads, kv_heads, tile_blocks, dtype):
    """G = 4, 8, 1, 12 (two n-tiles), 3 (odd); tiles of 32, 16 and 64 tokens; edge lengths."""
    rows, width, block_size, layers = 9, 40, 16, 3
    lens = [640, 1, 0, 31, 32, 33, 100, 17, 639]
    select = [1, 1, 1, 1, 0, 1, 1, 1, 1]
    group_rows = q_heads // kv_heads
    gen_layers = [random_case(11 + layer, rows, width, q_heads, kv_heads, lens, dtype) for layer in range(layers)]
    _, _, table, lens_t, qrow = gen_layers[0]
    run = None
    for layer in range(layers):
        q, k = gen_layers[layer][0], gen_layers[layer][1]
        run = launch(q, k, table, lens_t, qrow, select, True, layers, layer, group_rows, tile_blocks=tile_blocks,
                     run=run)
        assert int(run.status.item()) == 0
    ref = oracle_case(table, lens_t, qrow, select, [g[0] for g in gen_layers], [g[1] for g in gen_layers],
                      group_rows, block_size, tile_blocks)
    got = run.lse.cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    w = ~np.isnan(ref)
    np.testing.assert_allclose(got[w], ref[w], **LSE_TOL)
    compare_shares(ref, lens, select, block_size, tile_blocks, run.share.cpu().numpy())


@pytest.mark.parametrize(
    "q_heads, heads, width, lens",
    [
        (32, 8, 24, [377, 16, 200, 384]),  # 32 values a cell: eight warps of four
        (128, 8, 24, [377, 16, 200, 384]),  # 128 values: two units a warp, log totals kept
        (72, 5, 24, [377, 16, 200, 384]),  # G = 9, 45 values: single loads, log totals merged again per batch
        (32, 8, 600, [9600, 16, 4100, 9599]),  # rows of 300 tiles: the cells read again, in two batches
        (72, 5, 600, [9600, 16, 4100, 9599]),
    ],
)
def test_all_heads_mode_matches_the_oracle(q_heads, heads, width, lens):
    """Every shape of the share pass: cells of 32, 45 and 128 values, rows of more tiles than a warp holds."""
    rows, layers, kv_heads = 4, 2, 8
    select = [1, 1, 1, 1]
    gen_layers = [random_case(40 + layer, rows, width, q_heads, kv_heads, lens) for layer in range(layers)]
    _, _, table, lens_t, qrow = gen_layers[0]
    run = None
    for layer in range(layers):
        run = launch(gen_layers[layer][0], gen_layers[layer][1], table, lens_t, qrow, select, True, layers, layer,
                     q_heads // kv_heads, heads=heads, group=0, run=run)
    ref = oracle_case(table, lens_t, qrow, select, [g[0] for g in gen_layers], [g[1] for g in gen_layers],
                      q_heads // kv_heads, 16, 2, heads=heads, groups=[0] * layers)
    got = run.lse.cpu().numpy()
    w = ~np.isnan(ref)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got[w], ref[w], **LSE_TOL)
    compare_shares(ref, lens, select, 16, 2, run.share.cpu().numpy())


def test_the_flag_off_writes_nothing():
    q, k, table, lens, qrow = random_case(3, 4, 16, 32, 8, [100, 200, 50, 256])
    run = launch(q, k, table, lens, qrow, [1, 1, 1, 1], False, 1, 0, 4)
    assert torch.isnan(run.lse).all()
    assert torch.isnan(run.share).all()  # the share output is untouched too


def test_out_of_range_block_ids_are_skipped_and_reported():
    import ekv._lib as L

    q, k, table, lens, qrow = random_case(5, 3, 16, 32, 8, [100, 200, 250], pool=64)
    table = table % 64
    table[1, 2] = 64  # one past the pool
    table[2, 0] = -5
    run = launch(q, k, table, lens, qrow, [1, 1, 1], True, 1, 0, 4)
    assert int(run.status.item()) & L.STATUS_BAD_BLOCK_ID


def test_a_length_past_the_table_is_clamped_and_reported():
    import ekv._lib as L

    q, k, table, lens, qrow = random_case(6, 2, 8, 32, 8, [128, 129])
    run = launch(q, k, table, lens, qrow, [1, 1], True, 1, 0, 4)
    assert int(run.status.item()) & L.STATUS_LEN_OVER_WIDTH
    assert not torch.isnan(run.lse[0, 0, 1]).any()


def test_a_bad_query_row_is_skipped_and_reported():
    import ekv._lib as L

    q, k, table, lens, qrow = random_case(7, 2, 8, 32, 8, [100, 100])
    qrow[1] = q.shape[0] + 3
    run = launch(q, k, table, lens, qrow, [1, 1], True, 1, 0, 4)
    assert int(run.status.item()) & L.STATUS_BAD_QROW
    assert torch.isnan(run.lse[:, :, 1]).all() and torch.isnan(run.share[1]).all()
    assert not torch.isnan(run.lse[0, 0, 0, :7]).any()


def test_repeated_launches_are_deterministic():
    q, k, table, lens, qrow = random_case(8, 16, 64, 32, 8, list(np.random.default_rng(0).integers(1, 1024, 16)))
    a = launch(q, k, table, lens, qrow, [1] * 16, True, 1, 0, 4)
    b = launch(q, k, table, lens, qrow, [1] * 16, True, 1, 0, 4)
    assert torch.equal(torch.nan_to_num(a.lse, 7.0), torch.nan_to_num(b.lse, 7.0))
    assert torch.equal(torch.nan_to_num(a.share, 7.0), torch.nan_to_num(b.share, 7.0))


def test_full_size_llama8b_rows_sum_to_one():
    """Size-independent properties at the Llama-3.1-8B shape (64 rows, lengths up to 8192, a pool of
    32868 blocks): every audited row's shares are finite, non-negative and sum to 1, the unaudited row
    is NaN, and four rows match the oracle cell for cell and share for share."""
    rows, width, q_heads, kv_heads, pool = 64, 512, 32, 8, 64 * 512 + 100
    rng = np.random.default_rng(1)
    lens = rng.integers(1024, 8193, rows)
    select = np.ones(rows, dtype=np.uint8)
    select[5] = 0
    gen = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(rows + 5, q_heads, 128, device="cuda", generator=gen).to(torch.bfloat16)
    k = torch.randn(pool, 16, kv_heads, 128, device="cuda", generator=gen).to(torch.bfloat16)
    table = torch.from_numpy(rng.permutation(pool)[: rows * width].reshape(rows, width).astype(np.int32))
    qrow = torch.from_numpy(rng.permutation(rows + 5)[:rows].astype(np.int32))
    lens_t = torch.from_numpy(lens.astype(np.int32))
    run = launch(q, k, table, lens_t, qrow, select, True, 1, 0, 4)
    assert int(run.status.item()) == 0
    share = run.share.cpu().numpy().astype(np.float64)
    assert np.isnan(share[5]).all()
    live = np.flatnonzero(select)
    assert np.isfinite(share[live]).all() and (share[live] >= 0).all()
    np.testing.assert_allclose(share[live].sum(axis=1), 1.0, rtol=1e-4)
    # the oracle on four rows, over a compacted copy of just their blocks
    pick = np.array([0, 17, 40, 63])
    ids = np.unique(np.concatenate([table[r, : -(-int(lens[r]) // 16)].numpy() for r in pick]))
    remap = np.full(pool, 0, dtype=np.int32)
    remap[ids] = np.arange(len(ids), dtype=np.int32)
    small_table = remap[table.numpy()[pick]]
    k_small = k[torch.from_numpy(ids).cuda()].float().cpu().numpy()
    ref = oaud.new_table(1, len(pick), width, 4)
    oaud.tile_lse(q.float().cpu().numpy(), k_small, small_table, lens[pick], qrow.numpy()[pick],
                  np.ones(len(pick), dtype=np.uint8), 1, ref, 1 / math.sqrt(128), 0, 0, 16, 2)
    got = run.lse.cpu().numpy()[:, :, pick]
    w = ~np.isnan(ref)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got[w], ref[w], **LSE_TOL)
    u = osh.log_weights(ref, 1, np.arange(len(pick)), 2)
    np.testing.assert_allclose(share[pick], osh.normalize(u, -(-lens[pick] // 16), 2), **SHARE_TOL)


def test_one_step_launch_equals_per_layer_launches():
    """ekv_audit_step over every layer gives bit-identical cells and shares to per-layer launches."""
    import ekv._lib as L

    rows, width, q_heads, kv_heads, layers = 7, 48, 32, 8, 5
    lens = [700, 16, 0, 500, 768, 33, 1]
    select = [1, 1, 1, 0, 1, 1, 1]
    gen_layers = [random_case(60 + layer, rows, width, q_heads, kv_heads, lens) for layer in range(layers)]
    _, _, table, lens_t, qrow = gen_layers[0]
    run = None
    for layer in range(layers):
        run = launch(gen_layers[layer][0], gen_layers[layer][1], table, lens_t, qrow, select, True, layers, layer, 4,
                     run=run)
    dev = torch.device("cuda")
    qs = [g[0].to(dev) for g in gen_layers]
    ks = [g[1].to(dev) for g in gen_layers]
    q_addr = torch.tensor([q.data_ptr() for q in qs], dtype=torch.uint64, device=dev)
    k_addr = torch.tensor([k.data_ptr() for k in ks], dtype=torch.uint64, device=dev)
    step = Run(layers, rows, width, 4)
    flag = torch.ones(1, dtype=torch.int32, device=dev)
    sel = torch.tensor(select, dtype=torch.uint8, device=dev)
    td, ld, rd = table.to(dev), lens_t.to(dev), qrow.to(dev)
    rc = L.load().ekv_audit_step(
        q_addr.data_ptr(), k_addr.data_ptr(), td.data_ptr(), ld.data_ptr(), rd.data_ptr(), sel.data_ptr(),
        flag.data_ptr(), step.lse.data_ptr(), 1 / math.sqrt(128), 0, layers, 0, 1, 0, qs[0].stride(0), qs[0].stride(1),
        ks[0].stride(0), ks[0].stride(1), ks[0].stride(2), td.stride(0), layers, rows, width, 4, 16, 2, 128,
        L.DTYPE_BF16, 1, kv_heads, ks[0].shape[0], qs[0].shape[0], step.share.data_ptr(), step.contrib.data_ptr(),
        L.AGG_MEAN, step.ws.data_ptr(), step.ws_bytes, step.status.data_ptr(), L.current_stream(),
    )
    L.check(rc, "ekv_audit_step")
    torch.cuda.synchronize()
    assert int(step.status.item()) == 0
    assert torch.equal(torch.nan_to_num(run.lse, 3.0), torch.nan_to_num(step.lse, 3.0))
    assert torch.equal(torch.nan_to_num(run.share, 3.0), torch.nan_to_num(step.share, 3.0))
    assert torch.equal(run.contrib, step.contrib)
    assert torch.isnan(step.share[2]).all() and torch.isnan(step.share[3]).all()
    assert step.contrib.tolist() == [20, 20, 0, 0, 20, 20, 20]
    # nothing of a step carries over into the next (the work counter and tensor maps are rewritten): a second
    # step gives the same result
    rc = L.load().ekv_audit_step(
        q_addr.data_ptr(), k_addr.data_ptr(), td.data_ptr(), ld.data_ptr(), rd.data_ptr(), sel.data_ptr(),
        flag.data_ptr(), step.lse.data_ptr(), 1 / math.sqrt(128), 0, layers, 0, 1, 0, qs[0].stride(0), qs[0].stride(1),
        ks[0].stride(0), ks[0].stride(1), ks[0].stride(2), td.stride(0), layers, rows, width, 4, 16, 2, 128,
        L.DTYPE_BF16, 1, kv_heads, ks[0].shape[0], qs[0].shape[0], step.share.data_ptr(), step.contrib.data_ptr(),
        L.AGG_MEAN, step.ws.data_ptr(), step.ws_bytes, step.status.data_ptr(), L.current_stream(),
    )
    L.check(rc, "ekv_audit_step")
    torch.cuda.synchronize()
    assert torch.equal(torch.nan_to_num(run.share, 3.0), torch.nan_to_num(step.share, 3.0))


def test_long_context_rows_match_the_c_oracle():
    """Rows of 32k to 128k tokens in an 8192-block table (the long-context shape): every cell against the C
    restatement of the reference kernel, the shares against the oracle's normalisation."""
    from oracle import cpu as ocpu

    rows, q_heads, kv_heads, width = 6, 32, 8, 8192
    rng = np.random.default_rng(13)
    lens = rng.integers(32768, 131073, rows)
    lens[0], lens[1] = 131072, 32769  # the widest row, and a tail block of one token
    blocks = -(-lens // 16)
    pool = int(blocks.sum()) + 7
    ids = rng.permutation(pool)[: int(blocks.sum())].astype(np.int32)
    table = np.zeros((rows, width), dtype=np.int32)
    start = 0
    for r in range(rows):
        table[r, : blocks[r]] = ids[start : start + blocks[r]]
        start += blocks[r]
    gen = torch.Generator(device="cuda").manual_seed(21)
    q = torch.randn(rows + 3, q_heads, 128, device="cuda", generator=gen).to(torch.bfloat16)
    k = torch.randn(pool, 16, kv_heads, 128, device="cuda", generator=gen).to(torch.bfloat16)
    qrow = rng.permutation(rows + 3)[:rows].astype(np.int32)
    run = launch(q, k, torch.from_numpy(table), torch.from_numpy(lens.astype(np.int32)), torch.from_numpy(qrow),
                 [1] * rows, True, 1, 0, 4)
    assert int(run.status.item()) == 0
    ref = oaud.new_table(1, rows, width, 4)
    q16 = q.cpu().view(torch.int16).numpy().view(np.uint16)
    k16 = k.cpu().view(torch.int16).numpy().view(np.uint16)
    ocpu.tile_lse(q16, k16, "bf16", table, lens.astype(np.int32), qrow, np.ones(rows, dtype=np.uint8), 1, ref,
                  1 / math.sqrt(128), 0, 0, 16, 2)
    got = run.lse.cpu().numpy()
    w = ~np.isnan(ref)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got[w], ref[w], **LSE_TOL)
    u = osh.log_weights(ref, 1, np.arange(rows), 2)
    share = run.share.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(share, osh.normalize(u, blocks, 2), **SHARE_TOL)


def test_select_is_one_ordered_copy_per_call(runtime_dir):
    """select() stages both arrays in pinned memory and copies them on the current stream: calls in a
    row land in order, a shorter selection leaves the later rows as they were, and shapes torch's
    copy would refuse raise RuntimeError, as the reference's select does."""
    from ekv.runtime.audit_kernel import RecordingPlane

    rows = 6
    plane = RecordingPlane(2, rows, 4, 4, 16)
    for i in range(5):  # more calls than staging buffers, without a synchronisation between them
        plane.select(np.arange(rows) % 2 == i % 2, np.arange(rows) + 10 * i)
    plane.select(np.array([True, True]), np.array([7, 8]))
    torch.cuda.synchronize()
    assert plane._token.cpu().tolist() == [7, 8, 42, 43, 44, 45]
    assert plane._select.cpu().tolist() == [1, 1, 1, 0, 1, 0]
    with pytest.raises(RuntimeError):
        plane.select(np.ones(rows + 1, dtype=bool), np.arange(rows + 1))
    with pytest.raises(RuntimeError):
        plane.select(np.ones(3, dtype=bool), np.arange(2))
