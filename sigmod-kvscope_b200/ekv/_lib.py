"""The ctypes binding of libekv_b200.so, the sm_100a kernels behind every device call of this package.

There is no other implementation: if the library is missing or a CUDA device is absent, the calls
that need it raise. ``load()`` finds the library next to this file (built in-tree by ``ekv.build``).
Return codes map to the exceptions the reference raises for the same conditions: ``EKV_EINVAL`` to
``ValueError`` (shapes, groups, tile sizes), everything else to ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os

LIB_NAME = "libekv_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

OK, EINVAL, ERANGE, ENOTSUP, ECUDA = 0, -1, -2, -3, -4
DTYPE_F16, DTYPE_BF16 = 0, 1
AGG_MEAN, AGG_MAX = 0, 1
SHARE_FINALIZE = 2
STATUS_BAD_BLOCK_ID, STATUS_LEN_OVER_WIDTH, STATUS_BAD_QROW, STATUS_WAIT_TIMEOUT = 1, 2, 4, 8
POLICY_SUM, POLICY_UNIFORM, POLICY_NEWEST, POLICY_MAXMIN = 0, 1, 2, 3
AUDIT_CHUNK_TILES = 8

_c = ctypes
_p = _c.c_void_p
_i32 = _c.c_int
_i64 = _c.c_int64
_f32 = _c.c_float
_f64 = _c.c_double
_sz = _c.c_size_t

# name -> (restype, argtypes); the order follows include/ekv_b200.h
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ekv_last_error_string": (_c.c_char_p, []),
    "ekv_abi_version": (_i32, []),
    "ekv_audit_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "ekv_audit_launch": (
        _i32,
        [_p, _p, _p, _p, _p, _p, _p, _p,  # q k table lens qrow select flag lse
         _f32, _i32, _i32,  # scale layer group
         _i64, _i64, _i64, _i64, _i64, _i64,  # q strides, k strides, table stride
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,  # layers rows width G bs tb D dtype
         _i32, _i32, _i64, _i64,  # heads kv_heads pool_blocks q_tokens
         _p, _p, _i32, _i32,  # share_out contributors aggregate flags
         _p, _sz, _p, _p],  # workspace bytes status stream
    ),
    "ekv_audit_stash": (_i32, [_p, _i64, _i64, _p, _i32, _i64, _i32, _i32, _i32, _i32, _p, _p, _p]),
    "ekv_audit_step": (
        _i32,
        [_p, _p, _p, _p, _p, _p, _p, _p,  # q_layers k_layers table lens qrow select flag lse
         _f32, _i32, _i32, _i32, _i32, _i32,  # scale layer0 n_layers group rotate q_layout
         _i64, _i64, _i64, _i64, _i64, _i64,  # q strides, k strides, table stride
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,  # layers rows width G bs tb D dtype
         _i32, _i32, _i64, _i64,  # heads kv_heads pool_blocks q_tokens
         _p, _p, _i32,  # share_out contributors aggregate
         _p, _sz, _p, _p],  # workspace bytes status stream
    ),
    "ekv_audit_static_scratch_bytes": (_sz, []),
    "ekv_audit_step_static": (
        _i32,
        [_p, _p, _p, _p, _p, _p, _p, _p,  # q_layers k_layers table lens qrow select flag lse
         _f32, _i32, _i32, _i32, _i32, _i32,  # scale layer0 n_layers group rotate q_layout
         _i64, _i64, _i64, _i64, _i64, _i64,  # q strides, k strides, table stride
         _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,  # layers rows width G bs tb D dtype
         _i32, _i32, _i64, _i64,  # heads kv_heads pool_blocks q_tokens
         _p, _p, _i32,  # share_out contributors aggregate
         _p, _p],  # status stream
    ),
    "ekv_normalize_tile_lse": (
        _i32, [_p, _i32, _i32, _i32, _i32, _i32, _p, _p, _i32, _i32, _i32, _p, _p, _p]
    ),
    "ekv_normalize_log_weights": (
        _i32, [_p, _i32, _i32, _i32, _i32, _p, _i32, _i32, _p, _p, _p]
    ),
    "ekv_share_finalize": (_i32, [_p, _p, _p, _i32, _i32, _i32, _p, _p]),
    "ekv_allocate_quotas": (_i32, [_p, _p, _i32, _i32, _f64, _i64, _p, _i32, _i32, _i32, _p, _p]),
    "ekv_allocate_sum_workspace_bytes": (ctypes.c_size_t, [_i32, _i32]),
    "ekv_allocate_maxmin_workspace_bytes": (ctypes.c_size_t, [_i32, _i32]),
    "ekv_allocate_maxmin": (_i32, [_p, _i64, _p, _p, _i32, _i32, _f64, _i64, _i32, _i32, _p, _p, ctypes.c_size_t, _p]),
    "ekv_decode_view": (_i32, [_p, _i64, _p, _p, _i64, _p, _p, _i64, _i32, _i32, _i32, _i32, _p, _i64, _p, _p, _p]),
    "ekv_slot_compact": (_i32, [_p, _p, _i32, _p, _i64, _p, _i32, _i32, _i32, _i64, _i32, _i32, _p, _p, _p, _i64,
                                _p, _p, _p]),
    "ekv_allocate_sum": (_i32, [_p, _i64, _p, _p, _p, _i32, _i32, _f64, _i64, _i32, _i32, _p, _p, ctypes.c_size_t, _p]),
    "ekv_allocate_sum_f64": (
        _i32, [_p, _i64, _p, _p, _p, _p, _i32, _i32, _f64, _i64, _i32, _i32, _p, _p, _i64, _p, ctypes.c_size_t, _p],
    ),
    "ekv_view_build_sum_budget": (
        _i32,
        [_p, _i32, _i64, _p, _p, _p, _p, _i32, _i32, _f64, _i64,  # scores .. budget
         _p, _i64, _p, _p, _p, _i64, _i32, _i32, _i32,  # table .. block_size
         _p, _i64, _p, _p, _i64, _p, ctypes.c_size_t, _p],  # view .. stream
    ),
    "ekv_allocate_maxmin_f64": (
        _i32, [_p, _i64, _p, _p, _p, _i32, _i32, _f64, _i64, _i32, _i32, _p, _p, ctypes.c_size_t, _p],
    ),
    "ekv_allocate_pinned_workspace_bytes": (ctypes.c_size_t, [_i32, _i32]),
    "ekv_allocate_pinned_f64": (
        _i32, [_p, _i64, _p, _i64, _p, _p, _i32, _i64, _i32, _i32, _p, _i64, _p, ctypes.c_size_t, _p],
    ),
    "ekv_view_build_f64": (
        _i32,
        [_p, _i64, _p, _p, _p, _p, _i32, _p, _i64, _p, _p, _i32, _p, _p, _i64,
         _i32, _i32, _i32, _p, _i64, _p, _p, _i64, _p],
    ),
    "ekv_ledger_absorb": (_i32, [_p, _i32, _i64, _p, _p, _f64, _i32, _i32, _p, _i64, _i32, _p, _p]),
    "ekv_view_build": (
        _i32,
        [_p, _i64, _p, _p, _p, _p, _i32, _p, _i64, _i32, _p, _i64, _p, _p, _i64,
         _i32, _i32, _i32, _p, _i64, _p, _p, _i64, _p],
    ),
    "ekv_view_build_fractions": (
        _i32,
        [_p, _i64, _p, _p, _p, _p, _i32, _i32, _p, _i64, _i32, _p, _p, _i64,
         _i32, _i32, _i32, _p, _i64, _p, _p, _i64, _p],
    ),
    "ekv_compact_block_table": (_i32, [_p, _i64, _p, _p, _i64, _i32, _i32, _i32, _p, _i64, _p, _p]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library, with every signature declared. Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -c 'import ekv.build; ekv.build.build()'`"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    """Raise the reference's exception type for a failed call."""
    if rc == OK:
        return
    message = load().ekv_last_error_string().decode(errors="replace") or what
    if rc == EINVAL:
        raise ValueError(message)
    raise RuntimeError(f"{what}: {message}")


def ptr(tensor) -> int | None:  # a torch tensor or None
    """The device address of a tensor, or None (NULL)."""
    return None if tensor is None else tensor.data_ptr()


def current_stream() -> int:
    """torch's current CUDA stream as a handle for the ABI."""
    import torch

    return torch.cuda.current_stream().cuda_stream
