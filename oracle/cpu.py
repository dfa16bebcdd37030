"""Build and bind oracle/audit_cpu.c -- TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``build()`` compiles the C restatement with gcc (-O3, OpenMP) into oracle/_build/; ``tile_lse``
runs it on numpy arrays with the same meaning as ``oracle.audit.tile_lse`` (one KV head).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCE = os.path.join(HERE, "audit_cpu.c")
OUTPUT = os.path.join(HERE, "_build", "libekv_oracle.so")

_lib = None


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUTPUT) and os.path.getmtime(OUTPUT) >= os.path.getmtime(SOURCE):
        return OUTPUT
    os.makedirs(os.path.dirname(OUTPUT), exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-o", OUTPUT, SOURCE, "-lm"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"gcc failed: {result.stderr[-2000:]}")
    return OUTPUT


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(OUTPUT):
            build()
        lib = ctypes.CDLL(OUTPUT)
        p, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        lib.ekv_oracle_tile_lse.restype = None
        lib.ekv_oracle_tile_lse.argtypes = [p, p, i32, p, p, p, p, i32, p, f32, i32, i32,
                                            i64, i64, i64, i64, i64, i64, i32, i32, i32, i32, i32, i32, i32, i32]
        lib.ekv_oracle_threads.restype = i32
        _lib = lib
    return _lib


def threads() -> int:
    return int(load().ekv_oracle_threads())


def tile_lse(query, keys, dtype: str, table, lens, qrow, select, flag, lse, scale, layer, group, block_size,
             tile_blocks, n_threads: int = 0) -> None:
    """In place on lse [2, layers, rows, width, G]; query/keys are uint16 views of fp16/bf16 arrays."""
    lib = load()
    q = np.ascontiguousarray(query)
    k = keys  # may be a strided view of a [blocks, 2, ...] cache: strides passed as they are
    assert q.dtype == np.uint16 and k.dtype == np.uint16 and lse.dtype == np.float32 and lse.flags.c_contiguous
    table = np.ascontiguousarray(table, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    qrow = np.ascontiguousarray(qrow, dtype=np.int32)
    select = np.ascontiguousarray(select, dtype=np.uint8)
    layers, rows, width, group_rows = lse.shape[1:]
    es = 2  # bytes per element
    lib.ekv_oracle_tile_lse(
        q.ctypes.data, k.ctypes.data, 1 if dtype == "bf16" else 0, table.ctypes.data, lens.ctypes.data,
        qrow.ctypes.data, select.ctypes.data, int(flag), lse.ctypes.data, float(scale), layer, group,
        q.strides[0] // es, q.strides[1] // es, k.strides[0] // es, k.strides[1] // es, k.strides[2] // es,
        table.strides[0] // 4, layers, rows, width, group_rows, block_size, tile_blocks, q.shape[2], n_threads,
    )
