"""The allocation-free audit step, ekv_audit_step_static, against the workspace one, ekv_audit_step.

Some callers cannot allocate device memory at the moment they record: a binding with no CUDA allocator
of its own (a cgo or ctypes caller holding only the engine's tensors), or engine code after memory
profiling has sized the KV-cache pool, where one more cudaMalloc can fail or fragment the pool.
ekv_audit_step_static runs the same kernels on a static device workspace. Called twice in a row, it
must give what ekv_audit_step gives on the same inputs, within the audit tests' tolerances (cells
rtol/atol 1e-4, shares rtol 1e-3), with the same unwritten (NaN) cells and rows.

This file is named to be collected last, so a run that stops at the first failure has run every
other test first; it passes on its own in a fresh process as well.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import audit as oaud
from oracle import shares as osh

pytestmark = pytest.mark.gpu

LSE_TOL = dict(rtol=1e-4, atol=1e-4)
SHARE_TOL = dict(rtol=1e-3, atol=1e-9)


def make_inputs(seed: int = 3):
    rows, width, q_heads, kv_heads, layers = 6, 40, 32, 8, 4
    gen = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    pool = rows * width + 5
    lens = torch.tensor([640, 17, 0, 300, 512, 33], dtype=torch.int32)
    select = torch.tensor([1, 1, 1, 0, 1, 1], dtype=torch.uint8)
    table = torch.randperm(pool, generator=gen)[: rows * width].reshape(rows, width).to(torch.int32)
    qs = [torch.randn(rows, q_heads, 128, generator=gen).to(torch.bfloat16).to(dev) for _ in range(layers)]
    ks = [torch.randn(pool, 16, kv_heads, 128, generator=gen).to(torch.bfloat16).to(dev) for _ in range(layers)]
    return dict(
        rows=rows, width=width, kv_heads=kv_heads, layers=layers, qs=qs, ks=ks,
        table=table.to(dev), lens=lens.to(dev), select=select.to(dev),
        qrow=torch.arange(rows, dtype=torch.int32, device=dev),
        flag=torch.ones(1, dtype=torch.int32, device=dev),
        q_addr=torch.tensor([q.data_ptr() for q in qs], dtype=torch.uint64, device=dev),
        k_addr=torch.tensor([k.data_ptr() for k in ks], dtype=torch.uint64, device=dev),
    )


def outputs(x):
    dev = torch.device("cuda")
    return (torch.full((2, x["layers"], x["rows"], x["width"], 4), float("nan"), device=dev),
            torch.full((x["rows"], x["width"]), -1.0, device=dev),
            torch.full((x["rows"],), -1, dtype=torch.int32, device=dev),
            torch.zeros(1, dtype=torch.int32, device=dev))


def common_args(x, lse):
    q, k = x["qs"][0], x["ks"][0]
    return [x["q_addr"].data_ptr(), x["k_addr"].data_ptr(), x["table"].data_ptr(), x["lens"].data_ptr(),
            x["qrow"].data_ptr(), x["select"].data_ptr(), x["flag"].data_ptr(), lse.data_ptr(), 1 / math.sqrt(128),
            0, x["layers"], 0, 1, 0, q.stride(0), q.stride(1), k.stride(0), k.stride(1), k.stride(2),
            x["table"].stride(0), x["layers"], x["rows"], x["width"], 4, 16, 2, 128, 1, 1, x["kv_heads"],
            k.shape[0], q.shape[0]]


def test_the_static_workspace_step_equals_the_workspace_step_on_two_calls():
    import ekv._lib as L

    lib = L.load()
    x = make_inputs()
    lse_a, share_a, contrib_a, status_a = outputs(x)
    ws_bytes = lib.ekv_audit_workspace_bytes(x["layers"], x["rows"], x["width"])
    workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    rc = lib.ekv_audit_step(*common_args(x, lse_a), share_a.data_ptr(), contrib_a.data_ptr(), L.AGG_MEAN,
                            workspace.data_ptr(), ws_bytes, status_a.data_ptr(), L.current_stream())
    L.check(rc, "ekv_audit_step")
    for call in range(2):
        lse_b, share_b, contrib_b, status_b = outputs(x)
        rc = lib.ekv_audit_step_static(*common_args(x, lse_b), share_b.data_ptr(), contrib_b.data_ptr(),
                                       L.AGG_MEAN, status_b.data_ptr(), L.current_stream())
        L.check(rc, "ekv_audit_step_static")
        torch.cuda.synchronize()
        assert int(status_b.item()) == 0 == int(status_a.item())
        a, b = lse_a.cpu().numpy(), lse_b.cpu().numpy()
        assert np.array_equal(np.isnan(a), np.isnan(b)), f"call {call}: the written cells differ"
        np.testing.assert_allclose(b[~np.isnan(a)], a[~np.isnan(a)], err_msg=f"call {call}", **LSE_TOL)
        sa, sb = share_a.cpu().numpy().astype(np.float64), share_b.cpu().numpy().astype(np.float64)
        assert np.array_equal(np.isnan(sa), np.isnan(sb)), f"call {call}: the NaN rows differ"
        np.testing.assert_allclose(sb, sa, equal_nan=True, err_msg=f"call {call}", **SHARE_TOL)
        assert torch.equal(contrib_a, contrib_b)
        assert np.isnan(sb[2]).all() and np.isnan(sb[3]).all()  # an empty row and an unselected row
    # the last static call against the oracle as well: the restatement of the reference kernel, one KV
    # head per layer (head layer % kv_heads), then the reference normalisation of the cells
    ref = oracle_table(x)
    got = lse_b.cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got[~np.isnan(ref)], ref[~np.isnan(ref)], **LSE_TOL)
    lens, select = x["lens"].cpu().numpy(), x["select"].cpu().numpy()
    row_blocks = np.where(select != 0, -(-lens // 16), 0)
    live = np.flatnonzero(row_blocks > 0)
    expect = np.full((x["rows"], x["width"]), np.nan)
    expect[live] = osh.normalize(osh.log_weights(ref, x["layers"], live, 2), row_blocks[live], 2)
    np.testing.assert_allclose(share_b.cpu().numpy().astype(np.float64), expect, equal_nan=True, **SHARE_TOL)


def oracle_table(x) -> np.ndarray:
    lse = oaud.new_table(x["layers"], x["rows"], x["width"], 4)
    for layer in range(x["layers"]):
        oaud.tile_lse(x["qs"][layer].float().cpu().numpy(), x["ks"][layer].float().cpu().numpy(),
                      x["table"].cpu().numpy(), x["lens"].cpu().numpy(), x["qrow"].cpu().numpy(),
                      x["select"].cpu().numpy(), 1, lse, 1 / math.sqrt(128), layer, layer % x["kv_heads"], 16, 2)
    return lse


def test_a_refused_call_launches_nothing():
    """Arguments the step refuses (a group size past 16) return EINVAL before any work is queued: the
    outputs keep their contents, and the next valid call still gives the workspace step's result."""
    import ekv._lib as L

    lib = L.load()
    x = make_inputs(seed=5)
    lse, share, contrib, status = outputs(x)
    args = common_args(x, lse)
    args[23] = 17  # query rows per KV head
    rc = lib.ekv_audit_step_static(*args, share.data_ptr(), contrib.data_ptr(), L.AGG_MEAN, status.data_ptr(),
                                   L.current_stream())
    assert rc == L.EINVAL
    torch.cuda.synchronize()
    assert torch.isnan(lse).all() and bool((share == -1.0).all()) and bool((contrib == -1).all())
    rc = lib.ekv_audit_step_static(*common_args(x, lse), share.data_ptr(), contrib.data_ptr(), L.AGG_MEAN,
                                   status.data_ptr(), L.current_stream())
    L.check(rc, "ekv_audit_step_static")
    torch.cuda.synchronize()
    ref = oracle_table(x)
    got = lse.cpu().numpy()
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    np.testing.assert_allclose(got[~np.isnan(ref)], ref[~np.isnan(ref)], **LSE_TOL)


def test_a_step_beyond_the_static_workspace_is_rejected():
    import ekv._lib as L

    lib = L.load()
    x = make_inputs()
    lse, share, contrib, status = outputs(x)
    args = common_args(x, lse)
    # a table of 2048 layers: its workspace is beyond the static one, so the call is refused before
    # anything is launched (checked first, as the buffers here are not that large)
    assert lib.ekv_audit_workspace_bytes(2048, x["rows"], x["width"]) > lib.ekv_audit_static_scratch_bytes()
    args[20] = 2048
    rc = lib.ekv_audit_step_static(*args, share.data_ptr(), contrib.data_ptr(), L.AGG_MEAN, status.data_ptr(),
                                   L.current_stream())
    assert rc == L.ERANGE
    assert b"static" in lib.ekv_last_error_string()
