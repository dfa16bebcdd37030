"""The C ABI: the library loads, exports every function include/ekv_b200.h declares, and rejects
bad arguments with the documented codes before it touches a device. CPU only."""

from __future__ import annotations

import ctypes
import os
import re

import pytest
from conftest import ROOT

import ekv._lib as L

HEADER = os.path.join(ROOT, "include", "ekv_b200.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ekv_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import ekv.build

    ekv.build.build()
    return L.load()


def test_every_declared_function_is_exported_and_bound(lib):
    names = declared_functions()
    assert "ekv_audit_launch" in names and "ekv_view_build" in names
    for name in names:
        assert hasattr(lib, name), f"{name} is declared but not exported"
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"


def test_constants_agree_with_the_header():
    text = open(HEADER).read()
    defines = dict(re.findall(r"#define\s+(EKV_[A-Z0-9_]+)\s+\(?(-?\d+)u?\)?", text))
    assert int(defines["EKV_EINVAL"]) == L.EINVAL and int(defines["EKV_ENOTSUP"]) == L.ENOTSUP
    assert int(defines["EKV_SHARE_FINALIZE"]) == L.SHARE_FINALIZE
    assert int(defines["EKV_POLICY_SUM"]) == L.POLICY_SUM and int(defines["EKV_POLICY_NEWEST"]) == L.POLICY_NEWEST
    assert int(defines["EKV_POLICY_MAXMIN"]) == L.POLICY_MAXMIN
    assert int(defines["EKV_AUDIT_CHUNK_TILES"]) == L.AUDIT_CHUNK_TILES
    assert int(defines["EKV_DTYPE_BF16"]) == L.DTYPE_BF16


def test_workspace_size(lib):
    # the step's item counter + a 128-byte key-cache descriptor per layer; rows and width do not change it
    layers, rows, width = 32, 64, 512

    def up(x):
        return -(-x // 256) * 256

    want = 256 + up(layers * 128)
    assert lib.ekv_audit_workspace_bytes(layers, rows, width) == want
    assert lib.ekv_audit_workspace_bytes(layers, 2 * rows, 4 * width) == want
    # the static workspace holds the widest step this build accepts (1024 layers) and no more
    assert lib.ekv_audit_static_scratch_bytes() == lib.ekv_audit_workspace_bytes(1024, rows, width)
    assert lib.ekv_audit_workspace_bytes(0, rows, width) == 0


def audit_args(**over):
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first
    args = dict(
        q=fake, k=ctypes.c_void_p(0x2000), table=fake, lens=fake, qrow=fake, select=fake, flag=fake, lse=fake,
        scale=0.1, layer=0, group=0, qs0=1024, qs1=128, ks0=4096, ks1=256, ks2=128, ts=8,
        layers=1, rows=4, width=8, G=4, bs=16, tb=2, D=128, dtype=L.DTYPE_BF16, heads=1, kv_heads=2,
        pool=256, q_tokens=8, out=None, contrib=None, agg=L.AGG_MEAN, flags=0, ws=None, ws_bytes=0,
        status=None, stream=None,
    )
    args.update(over)
    return list(args.values())


@pytest.mark.parametrize(
    "over, code",
    [
        (dict(q=None), L.EINVAL),
        (dict(layer=1), L.ERANGE),
        (dict(G=17), L.EINVAL),
        (dict(group=2), L.EINVAL),
        (dict(bs=12), L.EINVAL),  # a tile of 24 tokens is not a power of two
        (dict(D=64), L.ENOTSUP),
        (dict(dtype=7), L.EINVAL),
        (dict(ks1=100), L.EINVAL),  # key rows not in whole 16-byte units
        (dict(ts=4), L.EINVAL),
        (dict(agg=5), L.EINVAL),
        (dict(out=ctypes.c_void_p(0x3000)), L.EINVAL),  # no contributors
        # rows of more tiles than the share pass holds (32768)
        (dict(out=ctypes.c_void_p(0x3000), contrib=ctypes.c_void_p(0x4000), width=65538, ts=65538), L.ENOTSUP),
        (dict(rows=4096), L.ENOTSUP),
    ],
)
def test_audit_launch_rejects_bad_arguments(lib, over, code):
    rc = lib.ekv_audit_launch(*audit_args(**over))
    assert rc == code
    assert lib.ekv_last_error_string()


def test_error_codes_map_to_the_reference_exceptions(lib):
    rc = lib.ekv_audit_launch(*audit_args(G=17))
    with pytest.raises(ValueError, match="16"):
        L.check(rc, "ekv_audit_launch")
    rc = lib.ekv_audit_launch(*audit_args(layer=3))
    with pytest.raises(RuntimeError, match="layer"):
        L.check(rc, "ekv_audit_launch")


def test_other_entry_points_validate_before_launching(lib):
    fake = ctypes.c_void_p(0x1000)
    assert lib.ekv_normalize_tile_lse(fake, 1, 1, 1, 1, 1, fake, fake, 1, 2, 9, fake, None, None) == L.EINVAL
    assert lib.ekv_normalize_tile_lse(fake, 1, 2, 1, 1, 1, fake, fake, 1, 2, 0, fake, None, None) == L.ERANGE
    assert lib.ekv_normalize_tile_lse(fake, 1, 1, 1, 1, 1, fake, fake, 0, 2, 0, fake, None, None) == L.OK  # no rows
    assert lib.ekv_normalize_log_weights(fake, 1, 1, 1, 1, fake, 0, 0, fake, None, None) == L.EINVAL
    assert lib.ekv_share_finalize(None, fake, None, 1, 1, 0, fake, None) == L.EINVAL
    assert lib.ekv_allocate_quotas(fake, None, 4, 0, 0.5, -1, None, L.POLICY_SUM, 4, 0, fake, None) == L.ENOTSUP
    assert lib.ekv_allocate_quotas(fake, None, 4, 0, 1.5, -1, None, L.POLICY_UNIFORM, 4, 0, fake, None) == L.EINVAL
    assert lib.ekv_allocate_quotas(fake, None, 4, 0, 0.5, -1, None, L.POLICY_UNIFORM, 9000, 0, fake, None) == L.ENOTSUP
    view_args = [fake, 8, fake, fake, fake, None, 0, None, 8, L.POLICY_SUM, None, 0, None, None, 0, 2, 8, 16,
                 fake, 8, fake, None, 0, None]
    assert lib.ekv_view_build(*view_args) == L.EINVAL  # ranking by shares without scores
    view_args[16] = 20000
    assert lib.ekv_view_build(*view_args) == L.ENOTSUP  # wider than 16384
    assert lib.ekv_compact_block_table(fake, 8, fake, None, 8, 2, 8, 16, fake, 8, fake, None) == L.EINVAL
    # the sum quotas: workspace, width, stride and budget are checked before anything is launched
    assert lib.ekv_allocate_sum_workspace_bytes(0, 8) == 0
    ws = lib.ekv_allocate_sum_workspace_bytes(2, 8)
    assert ws >= 256 + 2048 * 4 + 2 * 8 * 2
    sum_args = [fake, 8, None, fake, None, 4, 0, 0.5, -1, 2, 8, fake, None, 0, None]
    assert lib.ekv_allocate_sum(*sum_args) == L.ERANGE  # no workspace
    sum_args[12], sum_args[13] = ctypes.c_void_p(0x1000), ws
    sum_args[1] = 4
    assert lib.ekv_allocate_sum(*sum_args) == L.EINVAL  # score stride below the width
    sum_args[1], sum_args[7] = 8, 1.5
    assert lib.ekv_allocate_sum(*sum_args) == L.EINVAL  # a fraction above 1 with no explicit budget
    sum_args[7], sum_args[10] = 0.5, 40000
    assert lib.ekv_allocate_sum(*sum_args) == L.ENOTSUP  # wider than 32768
    # the maxmin quotas: workspace and width are checked before anything is launched
    mm_args = [fake, 8, fake, None, 4, 0, 0.5, -1, 2, 8, fake, None, 0, None]
    assert lib.ekv_allocate_maxmin(*mm_args) == L.ERANGE  # no workspace
    mm_args[11], mm_args[12], mm_args[9] = ctypes.c_void_p(0x1000), 1 << 30, 9000
    assert lib.ekv_allocate_maxmin(*mm_args) == L.ENOTSUP  # wider than 8192
    # the float64 entry points
    sum64 = [fake, 8, None, None, fake, None, 4, 0, 0.5, -1, 2, 8, fake, None, 0, ctypes.c_void_p(0x1000), ws, None]
    sum64[11] = 20000
    assert lib.ekv_allocate_sum_f64(*sum64) == L.ENOTSUP  # a float64 row is staged whole: wider than 16384
    sum64[11], sum64[13], sum64[14] = 8, fake, 4
    assert lib.ekv_allocate_sum_f64(*sum64) == L.EINVAL  # mask stride below the width
    sum64[13], sum64[14], sum64[15] = None, 0, None
    assert lib.ekv_allocate_sum_f64(*sum64) == L.ERANGE  # no workspace
    mm64 = [fake, 4, None, fake, None, 4, 0, 0.5, -1, 2, 8, fake, ctypes.c_void_p(0x1000), 1 << 30, None]
    assert lib.ekv_allocate_maxmin_f64(*mm64) == L.EINVAL  # score stride below the width
    v64 = [None, 0, None, fake, fake, None, 0, fake, 8, None, None, L.POLICY_SUM, None, None, 0, 2, 8, 16,
           None, 0, None, None, 0, None]
    assert lib.ekv_view_build_f64(*v64) == L.EINVAL  # neither a view nor a mask
    v64[21], v64[22] = fake, 8
    v64[8] = 4
    assert lib.ekv_view_build_f64(*v64) == L.EINVAL  # score stride below the width
    v64[8], v64[11] = 8, 7
    assert lib.ekv_view_build_f64(*v64) == L.EINVAL  # unknown policy
    ledger = [fake, 1, 8, fake, fake, 0.5, 2, 8, fake, 8, 4, fake, None]
    ledger[5] = 1.0
    assert lib.ekv_ledger_absorb(*ledger) == L.EINVAL  # a decay of 1 keeps nothing new
    ledger[5], ledger[9] = 0.5, 4
    assert lib.ekv_ledger_absorb(*ledger) == L.EINVAL  # ledger stride below the width
    frac = [fake, 8, fake, fake, fake, None, 0, 0, fake, 8, L.POLICY_SUM, None, None, 0, 2, 8, 16, fake, 8, fake,
            None, 0, None]
    frac[4] = None
    assert lib.ekv_view_build_fractions(*frac) == L.EINVAL  # no fractions
    frac[4], frac[7] = fake, -2
    assert lib.ekv_view_build_fractions(*frac) == L.EINVAL  # a cap below -1
    frac[7], frac[15] = 0, 20000
    assert lib.ekv_view_build_fractions(*frac) == L.ENOTSUP  # wider than 16384
    # the SGLang compaction: entry size, pointers and strides
    slot_args = [fake, fake, 8, fake, 20, None, 1, 2, 2, 40, 16, 20, fake, fake, fake, 20, fake, fake, None]
    slot_args[2] = 3
    assert lib.ekv_slot_compact(*slot_args) == L.EINVAL  # 3-byte entries
    slot_args[2], slot_args[4] = 8, 10
    assert lib.ekv_slot_compact(*slot_args) == L.EINVAL  # keep stride below the width
    slot_args[4], slot_args[16] = 20, None
    assert lib.ekv_slot_compact(*slot_args) == L.EINVAL  # no counters


def test_step_and_stash_validate_before_launching(lib):
    fake = ctypes.c_void_p(0x1000)
    step = [fake, fake, fake, fake, fake, fake, fake, fake, 0.1, 0, 4, 0, 1, 0, 1024, 128, 4096, 256, 128, 8,
            4, 4, 8, 4, 16, 2, 128, L.DTYPE_BF16, 1, 2, 256, 8, fake, fake, L.AGG_MEAN, None, 0, None, None]
    assert lib.ekv_audit_step(*step) == L.ERANGE  # share_out without a workspace
    step[35], step[36] = fake, 1 << 30
    step[10] = 5
    assert lib.ekv_audit_step(*step) == L.ERANGE  # layers [0, 5) of a table of 4
    step[0] = None
    assert lib.ekv_audit_step(*step) == L.EINVAL
    assert lib.ekv_audit_stash(None, 8, 128, fake, 4, 8, 0, 1, 4, 128, fake, None, None) == L.EINVAL
    assert lib.ekv_audit_stash(fake, 8, 128, fake, 4, 8, 0, 1, 4, 64, fake, None, None) == L.ENOTSUP
    assert lib.ekv_audit_stash(ctypes.c_void_p(0x1008), 8, 128, fake, 4, 8, 0, 1, 4, 128, fake, None, None) == L.EINVAL


def test_abi_version(lib):
    assert lib.ekv_abi_version() == 7
