"""The attention-share statistic recorded by the sm_100a audit kernel, for any attention backend.

Drop-in for runtime/audit_kernel.py of the reference: ``TILE_BLOCKS`` and ``RecordingPlane`` keep
their names, constructor, methods, table layout, NaN initialisation, descriptor files and
exceptions. For one KV group per layer (group ``layer % kv_heads``, as the reference samples) and
only for the rows of an audit step, the kernel records

  m[layer][row][block][query row] = the largest score over the keys of the block's tile
  l[layer][row][block][query row] = the sum of exp(score - m) over those keys

and, in the same launch, folds the layer into the exact per-block attention share of each row
(``shares()``), which the reference computed later on the host (observe/tile_shares.py). The launch
is the same on every step (the flag is read on the device), so a CUDA graph can capture it.
"""

from __future__ import annotations

import ctypes
import json
import os

import numpy as np
import torch

from .. import _lib
from .audit import AuditPlane, StatBlock, runtime_dir

TILE_BLOCKS = 2  # blocks per tile: one value per tile, as the reference kernel records

_DTYPES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}
_AGGREGATES = {"mean": _lib.AGG_MEAN, "max": _lib.AGG_MAX}


def pub_path(pid: int) -> str:
    return f"{runtime_dir()}/ekv_pass_{pid}.json"


class RecordingPlane(AuditPlane):
    """An audit plane whose statistic block is allocated here and recorded by the audit kernel.

    ``heads`` > 1 records that many KV heads per layer side by side in a cell (all-heads mode,
    ``group_rows`` then counts the query rows of one KV head); 1 is the reference's sampling.
    ``aggregate`` chooses how the fused shares combine layers and query rows ("mean" or "max").
    ``deferred`` keeps each layer's audited queries (a small copy per layer) and records every layer
    in one launch after the last layer: the cells and shares are the same, written at the end of the
    step instead of after each layer. It needs the layer table (``attach``) to hold the caches the
    layers are recorded from. ``None`` (the default) defers every step that starts with the layer
    table filled and records the others layer by layer.
    """

    _SIDE_STREAMS = 8  # deferred recording: the layers' stash copies run on this many parallel branches

    def __init__(
        self,
        layers: int,
        rows: int,
        width: int,
        group_rows: int,
        block_size: int,
        *,
        heads: int = 1,
        aggregate: str = "mean",
        deferred: bool | None = None,
    ) -> None:
        super().__init__()
        if group_rows > 16:
            raise ValueError(f"{group_rows} query heads per KV head: the kernel handles at most 16")
        if (block_size * TILE_BLOCKS) & (block_size * TILE_BLOCKS - 1):
            raise ValueError("a tile of the audit kernel must hold a power of two of tokens")
        if aggregate not in _AGGREGATES:
            raise ValueError(f"unknown aggregate {aggregate!r}")
        if heads < 1:
            raise ValueError("heads must be positive")
        self.rows, self.width, self.group_rows, self.block_size = rows, width, group_rows, block_size
        self.heads = heads
        self.cell = heads * group_rows  # values per (layer, row, block)
        self.aggregate = aggregate
        self.deferred = deferred
        self._step_deferred = False  # the mode of the step in progress, chosen at its layer 0
        self._layer_of: dict[str, int] = {}  # layer name -> number, in the order the layers first run
        self._addresses: list[int] = []
        self._lib = _lib.load()
        lse_bytes = 2 * layers * rows * width * self.cell * 4
        self._lse = self._allocate(lse_bytes)
        self._cuda.cudaMemset(ctypes.c_void_p(self._lse), 0xFF, ctypes.c_size_t(lse_bytes))  # NaN: unwritten
        # the block's control words: its own, so there is nothing to discover
        self._block = StatBlock(self._allocate(4), self._allocate(layers * 8), layers)
        self._cuda.cudaMemset(ctypes.c_void_p(self._flag_dev), 0, ctypes.c_size_t(4))
        self._cuda.cudaMemset(ctypes.c_void_p(self._table_dev), 0, ctypes.c_size_t(layers * 8))
        device = torch.device("cuda", torch.cuda.current_device())
        self._device = device
        # the selection: query token rows then audited flags, one device buffer that one copy fills
        self._inputs = torch.zeros(5 * rows, dtype=torch.uint8, device=device)
        self._token = self._inputs[: 4 * rows].view(torch.int32)
        self._select = self._inputs[4 * rows :]
        self._inputs_host = np.zeros(5 * rows, dtype=np.uint8)  # what the device buffer holds
        # two pinned staging buffers, each reused once the copy from it has run
        self._staging = [torch.zeros(5 * rows, dtype=torch.uint8).pin_memory() for _ in range(2)]
        self._staged = [torch.cuda.Event(), torch.cuda.Event()]
        self._stage = 0
        # the fused share: final shares and contributors, and the kernel's workspace
        self._contributors = torch.zeros(rows, dtype=torch.int32, device=device)
        self._share = torch.full((rows, width), float("nan"), dtype=torch.float32, device=device)
        self._workspace_bytes = int(self._lib.ekv_audit_workspace_bytes(layers, rows, width))
        self._workspace = torch.zeros(self._workspace_bytes + 256, dtype=torch.uint8, device=device)
        self._status = torch.zeros(1, dtype=torch.int32, device=device)
        # deferred recording: per-layer query stash, its addresses, and stash row indices
        self._stash: torch.Tensor | None = None
        self._stash_addresses: torch.Tensor | None = None
        self._rows_index = torch.arange(rows, dtype=torch.int32, device=device)
        self._key_shape: tuple | None = None
        self._step_addresses: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}
        self._side: list[torch.cuda.Stream] | None = None  # the stash copies' streams (deferred recording)
        torch.cuda.synchronize()
        self._publish()

    def attach(self, cache_addresses: list[int]) -> bool:
        """Fill the layer table with each layer's KV-cache base address (also kept on the host)."""
        filled = super().attach(cache_addresses)
        if filled and not self._addresses:
            self._addresses = [int(a) for a in cache_addresses]
        return filled

    # -- device memory of the statistic block (cudaMalloc, so that it can be exported by IPC) -------

    def _allocate(self, size: int) -> int:
        pointer = ctypes.c_void_p()
        rc = self._cuda.cudaMalloc(ctypes.byref(pointer), ctypes.c_size_t(size))
        if rc != 0 or pointer.value is None:
            raise RuntimeError(f"cudaMalloc of {size} bytes failed with code {rc}")
        return pointer.value

    def _ipc(self, address: int) -> str:
        handle = (ctypes.c_ubyte * 64)()
        rc = self._cuda.cudaIpcGetMemHandle(ctypes.byref(handle), ctypes.c_void_p(address))
        if rc != 0:
            raise RuntimeError(f"cudaIpcGetMemHandle failed with code {rc}")
        return bytes(handle).hex()

    def _publish(self) -> None:
        """Descriptor lines in the reference's format, so a controller reads this block unchanged."""
        entry = {
            "host_va": self._lse,
            "ncap": self.width,
            "max_rows": self.rows,
            "tile_lse_dev": self._lse,
            "tile_lse_ipc": self._ipc(self._lse),
            "tile_lse_layers": self._layers,
            "tile_lse_group_rows": self.cell,
            "stat_flag_dev": self._flag_dev,
            "layer_table_dev": self._table_dev,
            "layer_table_ipc": self._ipc(self._table_dev),
        }
        path = pub_path(self.pid)
        with open(path, "a") as f:
            f.write(json.dumps(entry) + "\n")
        os.chmod(path, 0o600)
        coverage = {"host_va": self._lse, "attn_share_tile_blocks": TILE_BLOCKS}
        with open(path.replace("ekv_pass_", "ekv_coverage_"), "a") as f:
            f.write(json.dumps(coverage) + "\n")

    def close(self) -> None:
        """Free the cudaMalloc blocks (the tensors go with the object)."""
        for address in (self._lse, self._flag_dev, self._table_dev):
            if address:
                self._cuda.cudaFree(ctypes.c_void_p(address))
        self._lse = 0
        self._block = None

    # -- the engine-facing calls -------------------------------------------------------------------

    @property
    def layer_names(self) -> list[str]:
        """The attention layers in the order they first ran, which is their layer number."""
        return sorted(self._layer_of, key=lambda name: self._layer_of[name])

    def select(self, audited: np.ndarray, token_start: np.ndarray) -> None:
        """Choose the rows to record in the next step, and the token index of each row's query
        (runtime/audit_kernel.py:190-194: the first ``len(audited)`` rows change, the rest keep their
        values; shapes that torch's copy would refuse raise RuntimeError).

        Unlike the reference's two pageable copies, which block the host, both arrays go to the device
        in one asynchronous copy on the current stream from a pinned staging buffer: work launched on
        that stream afterwards sees them; a caller that records on another stream orders it after this
        one first (``other.wait_stream(torch.cuda.current_stream())``). Two staging buffers alternate; a
        call waits only for the copy made from its buffer two calls earlier."""
        audited = np.asarray(audited)
        rows = len(audited)
        try:  # the shapes torch's copy into the first `rows` rows accepts
            if rows > self.rows:
                raise ValueError
            token_start = np.broadcast_to(np.asarray(token_start), (rows,))
        except ValueError:
            raise RuntimeError(
                f"{rows} audited flags and {np.shape(token_start)} token rows for a plane of {self.rows} rows"
            ) from None
        host = self._inputs_host
        host[: 4 * self.rows].view(np.int32)[:rows] = token_start.astype(np.int32)
        host[4 * self.rows : 4 * self.rows + rows] = audited.astype(np.uint8)
        # one asynchronous copy on the current stream from a pinned buffer whose last copy has run
        i = self._stage
        self._staged[i].synchronize()
        self._staging[i].numpy()[:] = host
        self._inputs.copy_(self._staging[i], non_blocking=True)
        self._staged[i].record()
        self._stage = 1 - i

    def record(
        self,
        layer_name: str,
        table: torch.Tensor,
        lens: torch.Tensor,
        query: torch.Tensor,
        kv_cache: torch.Tensor,
        scale: float,
    ) -> None:
        """Launch the kernel for one attention layer, after the layer has attended.

        A layer is numbered by its name in the order the layers first run (cache addresses are not
        stable while the engine profiles memory; names are). ``kv_cache`` is [blocks, 2, block, heads, dim].
        """
        if kv_cache.ndim != 5 or kv_cache.shape[1] != 2:
            raise ValueError(f"expected a KV cache [blocks, 2, block, heads, dim], got {tuple(kv_cache.shape)}")
        if kv_cache.shape[2] != self.block_size:
            raise ValueError("the KV cache's block size differs from the view's")
        layer = self._layer_of.setdefault(layer_name, len(self._layer_of))
        self.launch(layer, table, lens, query, kv_cache[:, 0], scale)

    def launch(
        self,
        layer: int,
        table: torch.Tensor,
        lens: torch.Tensor,
        query: torch.Tensor,
        keys: torch.Tensor,
        scale: float,
        stream: int | None = None,
    ) -> None:
        """Launch the kernel for ``layer``; ``keys`` is the layer's key cache [blocks, block, heads, dim].

        The plane's last layer finalises the step's shares (and, deferred, records every layer).
        """
        if layer >= self._layers:
            raise RuntimeError(f"more attention layers ran than the {self._layers} the plane was sized for")
        kv_heads, dim = keys.shape[2], keys.shape[3]
        if kv_heads * self.group_rows != query.shape[1] or dim != query.shape[2]:
            raise ValueError("the query and KV cache shapes do not match the plane's group size")
        if query.dtype not in _DTYPES or keys.dtype != query.dtype:
            raise ValueError(f"query and keys must both be float16 or bfloat16, got {query.dtype}, {keys.dtype}")
        if query.stride(2) != 1 or keys.stride(3) != 1:
            raise ValueError("the head dimension of the query and the keys must be contiguous")
        if table.dtype != torch.int32 or lens.dtype != torch.int32:
            raise ValueError("the block table and the lengths must be int32")
        if table.shape[1] != self.width or table.shape[0] < self.rows or lens.shape[0] < self.rows:
            raise ValueError("the block table does not match the plane's rows and width")
        if self.heads == 1:
            group = layer % kv_heads
        else:
            if self.heads != kv_heads:
                raise ValueError(f"an all-heads plane of {self.heads} heads got a cache of {kv_heads}")
            group = 0
        stream = _lib.current_stream() if stream is None else stream
        dtype = _DTYPES[query.dtype]
        workspace = (self._workspace.data_ptr() + 255) // 256 * 256
        if layer == 0:
            self._step_deferred = bool(self._addresses) if self.deferred is None else self.deferred
        if self._step_deferred:
            self._record_deferred(layer, group, table, lens, query, keys, scale, dtype, workspace, stream)
            return
        flags = _lib.SHARE_FINALIZE if layer == self._layers - 1 else 0
        rc = self._lib.ekv_audit_launch(
            query.data_ptr(), keys.data_ptr(), table.data_ptr(), lens.data_ptr(), self._token.data_ptr(),
            self._select.data_ptr(), self._flag_dev, self._lse, float(scale), layer, group,
            query.stride(0), query.stride(1), keys.stride(0), keys.stride(1), keys.stride(2), table.stride(0),
            self._layers, self.rows, self.width, self.group_rows, self.block_size, TILE_BLOCKS, dim,
            dtype, self.heads, kv_heads, keys.shape[0], query.shape[0],
            self._share.data_ptr(), self._contributors.data_ptr(), _AGGREGATES[self.aggregate], flags,
            workspace, self._workspace_bytes, self._status.data_ptr(), stream,
        )
        _lib.check(rc, "ekv_audit_launch")

    def _record_deferred(self, layer, group, table, lens, query, keys, scale, dtype, workspace, stream) -> None:
        """Keep the layer's audited queries; after the last layer record every layer in one launch."""
        if len(self._addresses) <= layer:
            raise RuntimeError("deferred recording needs the layer table filled with every layer's cache")
        if keys.data_ptr() != self._addresses[layer]:
            raise ValueError(f"layer {layer}'s key cache is not the one in the layer table")
        shape = (tuple(keys.shape), tuple(keys.stride()), query.dtype)
        if self._key_shape is None:
            self._key_shape = shape
        elif shape != self._key_shape:
            raise ValueError("every layer's key cache must have the same shape and strides")
        if self._stash is None:
            self._stash = torch.empty(self._layers, self.rows, self.cell, query.shape[2], dtype=query.dtype,
                                      device=self._device)
            step = self._stash[0].numel() * self._stash.element_size()
            addresses = [self._stash.data_ptr() + i * step for i in range(self._layers)]
            self._stash_addresses = torch.tensor(addresses, dtype=torch.uint64, device=self._device)
        if self._stash.dtype != query.dtype:
            raise ValueError("every layer's query must have the same dtype")
        # The layer's stash copy runs on a side stream forked from the caller's stream here (after the
        # layer's attention, which made the query), so it overlaps whatever the caller queues next instead
        # of lengthening its stream; the side streams join the caller's before the step's launch. Under
        # capture the forks and the join become branches of the graph.
        main = torch.cuda.ExternalStream(stream, device=self._device)
        if self._side is None:
            self._side = [torch.cuda.Stream(device=self._device) for _ in range(self._SIDE_STREAMS)]
        side = self._side[layer % len(self._side)]
        side.wait_stream(main)
        rc = self._lib.ekv_audit_stash(
            query.data_ptr(), query.stride(0), query.stride(1), self._token.data_ptr(), self.rows, query.shape[0],
            group, self.heads, self.group_rows, query.shape[2], self._stash[layer].data_ptr(), self._status.data_ptr(),
            side.cuda_stream,
        )
        _lib.check(rc, "ekv_audit_stash")
        if layer != self._layers - 1:
            return
        for branch in self._side[: min(len(self._side), self._layers)]:
            main.wait_stream(branch)
        stash = self._stash[0]
        rc = self._lib.ekv_audit_step(
            self._stash_addresses.data_ptr(), self._table_dev, table.data_ptr(), lens.data_ptr(),
            self._rows_index.data_ptr(), self._select.data_ptr(), self._flag_dev, self._lse, float(scale),
            0, self._layers, 0 if self.heads > 1 else 0, 1 if self.heads == 1 else 0, 1,
            stash.stride(0), stash.stride(1), keys.stride(0), keys.stride(1), keys.stride(2), table.stride(0),
            self._layers, self.rows, self.width, self.group_rows, self.block_size, TILE_BLOCKS, keys.shape[3],
            dtype, self.heads, keys.shape[2], keys.shape[0], self.rows,
            self._share.data_ptr(), self._contributors.data_ptr(), _AGGREGATES[self.aggregate],
            workspace, self._workspace_bytes, self._status.data_ptr(), stream,
        )
        _lib.check(rc, "ekv_audit_step")

    def record_step(
        self,
        table: torch.Tensor,
        lens: torch.Tensor,
        queries: list[torch.Tensor],
        kv_caches: list[torch.Tensor],
        scale: float,
        stream: int | None = None,
        shares: bool = True,
    ) -> None:
        """Record every layer of a step in one launch, from each layer's query and KV cache.

        For a caller that holds every layer's query [tokens, q_heads, dim] (an offline audit, or an
        engine that keeps them): the cells and shares equal those of ``record`` called layer by layer.
        The layers are numbered 0 .. len(queries) - 1; the address arrays are cached per set of
        tensors, so a CUDA graph can capture the call. ``shares=False`` records the cells only.
        """
        if len(queries) != self._layers or len(kv_caches) != self._layers:
            raise ValueError(f"a step records all {self._layers} layers")
        keys = [kv[:, 0] for kv in kv_caches]
        q0, k0 = queries[0], keys[0]
        for q, k in zip(queries, keys, strict=True):
            if q.shape != q0.shape or q.stride() != q0.stride() or q.dtype != q0.dtype:
                raise ValueError("every layer's query must have the same shape, strides and dtype")
            if k.shape != k0.shape or k.stride() != k0.stride() or k.dtype != q0.dtype:
                raise ValueError("every layer's key cache must have the same shape, strides and dtype as the query")
        kv_heads, dim = k0.shape[2], k0.shape[3]
        if kv_heads * self.group_rows != q0.shape[1] or dim != q0.shape[2] or q0.dtype not in _DTYPES:
            raise ValueError("the query and KV cache shapes do not match the plane's group size")
        if self.heads != 1 and self.heads != kv_heads:
            raise ValueError(f"an all-heads plane of {self.heads} heads got a cache of {kv_heads}")
        if table.dtype != torch.int32 or lens.dtype != torch.int32 or table.shape[1] != self.width:
            raise ValueError("the block table and the lengths must be int32 and match the plane's width")
        key = tuple(q.data_ptr() for q in queries) + tuple(k.data_ptr() for k in keys)
        addresses = self._step_addresses.get(key)
        if addresses is None:
            q_addr = torch.tensor([q.data_ptr() for q in queries], dtype=torch.uint64, device=self._device)
            k_addr = torch.tensor([k.data_ptr() for k in keys], dtype=torch.uint64, device=self._device)
            addresses = self._step_addresses[key] = (q_addr, k_addr)
        q_addr, k_addr = addresses
        workspace = (self._workspace.data_ptr() + 255) // 256 * 256
        rc = self._lib.ekv_audit_step(
            q_addr.data_ptr(), k_addr.data_ptr(), table.data_ptr(), lens.data_ptr(), self._token.data_ptr(),
            self._select.data_ptr(), self._flag_dev, self._lse, float(scale), 0, self._layers, 0,
            1 if self.heads == 1 else 0, 0, q0.stride(0), q0.stride(1), k0.stride(0), k0.stride(1), k0.stride(2),
            table.stride(0), self._layers, self.rows, self.width, self.group_rows, self.block_size, TILE_BLOCKS, dim,
            _DTYPES[q0.dtype], self.heads, kv_heads, k0.shape[0], q0.shape[0],
            self._share.data_ptr() if shares else None, self._contributors.data_ptr() if shares else None,
            _AGGREGATES[self.aggregate], workspace, self._workspace_bytes,
            self._status.data_ptr(), _lib.current_stream() if stream is None else stream,
        )
        _lib.check(rc, "ekv_audit_step")

    # -- what the fused launch leaves behind --------------------------------------------------------

    def shares(self) -> torch.Tensor:
        """The attention share per (row, block) of the last completed audit step, float32 on the device.

        A row not audited in that step, or with no data, is NaN; every other row sums to 1. It equals
        normalize_tile_lse over the step's cells with row_blocks = ceil(lens / block_size).
        """
        return self._share

    def direct_shares(self, out: torch.Tensor) -> None:
        """Write the shares of the launches that follow into ``out`` (float32 [rows, width] on the plane's
        device) instead of the plane's own buffer; ``shares()`` then returns ``out``. Launches already
        captured in a CUDA graph keep the buffer they were captured with, so two buffers captured in two
        graphs let one step's shares be combined across ranks while the next step writes the other."""
        if out.dtype != torch.float32 or tuple(out.shape) != (self.rows, self.width) or not out.is_contiguous():
            raise ValueError(f"the share buffer must be a contiguous float32 [{self.rows}, {self.width}] tensor")
        if out.device != self._device:
            raise ValueError("the share buffer must be on the plane's device")
        self._share = out

    def status(self) -> int:
        """The EKV_STATUS_* bits the kernel raised since the last ``clear_status`` (synchronises)."""
        return int(self._status.item())

    def clear_status(self) -> None:
        self._status.zero_()

    def table(self) -> torch.Tensor:
        """A view of the statistic table [2, layers, rows, width, cell] as a float32 tensor (no copy)."""
        return _wrap(self._lse, (2, self._layers, self.rows, self.width, self.cell))


def _wrap(address: int, shape: tuple[int, ...]) -> torch.Tensor:
    """A float32 tensor over device memory this process allocated with cudaMalloc (no ownership)."""

    class _Array:
        __cuda_array_interface__ = {
            "shape": shape,
            "typestr": "<f4",
            "data": (address, False),
            "version": 3,
            "strides": None,
        }

    return torch.as_tensor(_Array(), device=torch.device("cuda", torch.cuda.current_device()))
