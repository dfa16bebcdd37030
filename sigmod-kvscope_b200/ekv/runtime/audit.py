"""The serving-process side of the attention-share statistic: the device flag and the layer table.

Interface of runtime/audit.py of the reference (AuditPlane, :26-113): the same class, methods,
private attribute names, descriptor files and exceptions. The statistic block a recording kernel
uses is described by a JSON line in ``$EKV_RUNTIME_DIR/ekv_pass_<pid>.json``: a uint32 flag that turns
recording on for an audit step, and a uint64 table with each layer's KV-cache base address.

Every write to those device words is an asynchronous copy from page-locked memory on torch's current
stream, ordered with the launches the engine queues after it, with no wait on the host (the reference
writes them with a blocking cudaMemcpy); a write that would not change the device value is skipped.
"""

from __future__ import annotations

import ctypes
import json
import os
from collections.abc import Iterator
from typing import NamedTuple

import numpy as np


def _cudart() -> ctypes.CDLL:
    """The CUDA runtime already in the process (torch loads it), opened by its soname."""
    errors = []
    for soname in ("libcudart.so.12", "libcudart.so"):
        try:
            return ctypes.CDLL(soname)
        except OSError as e:
            errors.append(str(e))
    raise RuntimeError(f"libcudart not found ({'; '.join(errors)})")


def runtime_dir() -> str:
    return os.environ.get("EKV_RUNTIME_DIR") or "/tmp"


def _json_lines(path: str) -> Iterator[dict]:
    """The JSON objects of a descriptor file, one per non-empty line; nothing if the file is absent."""
    try:
        with open(path) as f:
            lines = f.read().splitlines()
    except FileNotFoundError:
        return
    for line in lines:
        if line.strip():
            yield json.loads(line)


def device_bytes(address: int, nbytes: int):
    """A uint8 torch tensor over ``nbytes`` of device memory at ``address`` on the current device (no
    ownership: the memory belongs to whoever allocated it)."""
    import torch

    class _Bytes:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (address, False), "version": 3,
                                    "strides": None}

    return torch.as_tensor(_Bytes(), device=torch.device("cuda", torch.cuda.current_device()))


class StatBlock(NamedTuple):
    """Where the statistic block's control words live on the device."""

    flag: int  # uint32: nonzero while recording
    layer_table: int  # uint64 [layers]: each layer's KV-cache base address
    layers: int


def published_block(pid: int) -> StatBlock | None:
    """The first statistic block the process ``pid`` published, or None while it has published none."""
    for entry in _json_lines(f"{runtime_dir()}/ekv_pass_{pid}.json"):
        flag = int(entry.get("stat_flag_dev", 0))
        if flag:
            return StatBlock(flag, int(entry["layer_table_dev"]), int(entry["tile_lse_layers"]))
    return None


class AuditPlane:
    """Sets the audit flag and fills the layer table of one serving process (reference audit.py:26)."""

    def __init__(self, pid: int | None = None) -> None:
        self.pid = os.getpid() if pid is None else pid
        self._cuda = _cudart()
        self._block: StatBlock | None = None
        self._table_filled = False
        self._flag_on: bool | None = None  # what the flag holds on the device, once written
        self._newest_rows_checked = False

    # the device addresses under the reference's attribute names (read by its live checks)
    @property
    def _flag_dev(self) -> int:
        return self._block.flag if self._block else 0

    @property
    def _table_dev(self) -> int:
        return self._block.layer_table if self._block else 0

    @property
    def _layers(self) -> int:
        return self._block.layers if self._block else 0

    def _discover(self) -> bool:
        """Look for the published block if it is not known yet; True once it is."""
        if self._block is None:
            self._block = published_block(self.pid)
        return self._block is not None

    def _copy_to_device(self, device: int, data: np.ndarray) -> None:
        """Write ``data`` to the device address ``device``: one asynchronous copy on torch's current stream
        from page-locked memory (torch's pinned-memory cache keeps that buffer until the copy has run)."""
        import torch

        raw = np.ascontiguousarray(data).reshape(-1).view(np.uint8)
        staged = torch.from_numpy(raw.copy()).pin_memory()
        device_bytes(device, raw.size).copy_(staged, non_blocking=True)

    def require_newest_rows(self) -> None:
        """Refuse a prefill audit unless every kernel that records the statistic records it only from the
        program holding a request's newest query tokens (reference audit.py:62-81). Checked once."""
        if self._newest_rows_checked:
            return
        coverage = [e for e in _json_lines(f"{runtime_dir()}/ekv_coverage_{self.pid}.json")
                    if int(e.get("attn_share_sites", 0))]
        if not coverage:
            raise RuntimeError("a prefill audit was requested before any kernel that records the statistic compiled")
        every_program = [e["kernel"] for e in coverage if not int(e.get("attn_share_newest_rows", 0))]
        if every_program:
            raise RuntimeError(
                f"kernels {every_program} record the statistic from every program of a request, so a prefill "
                "step cannot be an audit step with them"
            )
        self._newest_rows_checked = True

    def select(self, audited: np.ndarray, token_start: np.ndarray) -> None:
        """Choose the rows to record next; a plane that records every row it is given needs none."""

    def attach(self, cache_addresses: list[int]) -> bool:
        """Fill the layer table with each layer's KV-cache base address; True once it is filled (the
        table is written once, the first time the block is known)."""
        if self._table_filled:
            return True
        if not self._discover():
            return False
        if len(cache_addresses) > self._layers:
            raise ValueError(
                f"{len(cache_addresses)} KV caches for a statistic block of {self._layers} layers"
            )
        table = np.zeros(self._layers, dtype=np.uint64)
        table[: len(cache_addresses)] = np.asarray(cache_addresses, dtype=np.uint64)
        self._copy_to_device(self._table_dev, table)
        self._table_filled = True
        return True

    def set(self, on: bool) -> None:
        """Turn recording on or off for the launches that follow (a device write only on a change)."""
        on = bool(on)
        if self._flag_on is on:
            return
        if not self._discover():
            if not on:
                return  # nothing records yet, so nothing to switch off
            raise RuntimeError("an audit step was requested but no statistic block has been published")
        if on and not self._table_filled:
            raise RuntimeError("an audit step was requested before the layer table was filled")
        self._copy_to_device(self._flag_dev, np.array([1 if on else 0], dtype=np.uint32))
        self._flag_on = on
