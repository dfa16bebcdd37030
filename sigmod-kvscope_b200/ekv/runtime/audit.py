"""The serving-process side of the attention-share statistic: the device flag and the layer table.

Mirrors runtime/audit.py of the reference (AuditPlane, :26-113) with the same names, descriptor
files and exceptions. The flag (uint32) switches recording on for audit steps; the layer table
(uint64 per layer) holds the base address of each layer's KV cache. Both live in device memory
described by the descriptor line ``$EKV_RUNTIME_DIR/ekv_pass_<pid>.json``.
"""

from __future__ import annotations

import ctypes
import json
import os

import numpy as np


def _cudart() -> ctypes.CDLL:
    """The CUDA runtime the process already uses (torch loads it first), found by soname."""
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            return ctypes.CDLL(name)
        except OSError:
            continue
    raise RuntimeError("libcudart not found")


def runtime_dir() -> str:
    return os.environ.get("EKV_RUNTIME_DIR") or "/tmp"


class AuditPlane:
    """Sets the audit flag and fills the layer table of one serving process (reference audit.py:26)."""

    def __init__(self, pid: int | None = None) -> None:
        self.pid = os.getpid() if pid is None else pid
        self._cuda = _cudart()
        self._flag_dev = 0
        self._table_dev = 0
        self._layers = 0
        self._table_filled = False
        self._flag_on: bool | None = None
        self._newest_rows_checked = False

    def _discover(self) -> bool:
        """Find the statistic block's flag and layer table in the descriptor file; False if none yet."""
        path = f"{runtime_dir()}/ekv_pass_{self.pid}.json"
        try:
            with open(path) as f:
                entries = [json.loads(line) for line in f if line.strip()]
        except FileNotFoundError:
            return False
        for entry in entries:
            if int(entry.get("stat_flag_dev", 0)):
                self._flag_dev = int(entry["stat_flag_dev"])
                self._table_dev = int(entry["layer_table_dev"])
                self._layers = int(entry["tile_lse_layers"])
                return True
        return False

    def _copy_to_device(self, device: int, data: np.ndarray) -> None:
        data = np.ascontiguousarray(data)
        rc = self._cuda.cudaMemcpy(
            ctypes.c_void_p(device), data.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(data.nbytes), 1
        )
        if rc != 0:
            raise RuntimeError(f"cudaMemcpy host to device failed with code {rc}")

    def require_newest_rows(self) -> None:
        """Refuse a prefill audit unless every recording kernel records only from the program holding a
        request's newest query tokens (reference audit.py:62-81). Checked once."""
        if self._newest_rows_checked:
            return
        path = f"{runtime_dir()}/ekv_coverage_{self.pid}.json"
        with open(path) as f:
            recording = [e for e in (json.loads(line) for line in f if line.strip()) if int(e.get("attn_share_sites", 0))]
        if not recording:
            raise RuntimeError("a prefill audit was requested before any kernel that records the statistic compiled")
        unsafe = [e["kernel"] for e in recording if not int(e.get("attn_share_newest_rows", 0))]
        if unsafe:
            raise RuntimeError(
                f"kernels {unsafe} record the statistic from every program of a request: a prefill step cannot "
                "be an audit step with them"
            )
        self._newest_rows_checked = True

    def select(self, audited: np.ndarray, token_start: np.ndarray) -> None:
        """Choose the rows to record next; a plane that records every row it is given needs none."""

    def attach(self, cache_addresses: list[int]) -> bool:
        """Fill the layer table with each layer's KV-cache base address. True once it is filled."""
        if self._table_filled:
            return True
        if not self._flag_dev and not self._discover():
            return False
        if len(cache_addresses) > self._layers:
            raise ValueError(
                f"the statistic block was sized for {self._layers} layers, the engine has {len(cache_addresses)}"
            )
        table = np.zeros(self._layers, dtype=np.uint64)
        table[: len(cache_addresses)] = cache_addresses
        self._copy_to_device(self._table_dev, table)
        self._table_filled = True
        return True

    def set(self, on: bool) -> None:
        """Turn recording on or off for the launches that follow (an H2D copy only when it changes)."""
        if on == self._flag_on:
            return
        if not self._flag_dev and not self._discover():
            if on:
                raise RuntimeError("an audit step was requested but no statistic buffers were published")
            return
        if on and not self._table_filled:
            raise RuntimeError("an audit step was requested before the layer table was filled")
        self._copy_to_device(self._flag_dev, np.array([1 if on else 0], dtype=np.uint32))
        self._flag_on = on
