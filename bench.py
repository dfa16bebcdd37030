#!/usr/bin/env python
"""Benchmark of the attention-share audit path on B200: audited KV tokens/s and % of HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config llama8b|llama70b|long]
                    [--mode reference|all-heads] [--impl ours|reference]

One step is one audit step of the configured model over synthetic seeded inputs: the audit kernel
for every layer (captured in one CUDA graph, as the engine captures its decode step), which also
leaves the exact per-block shares on the device; with N > 1 ranks (one per GPU, KV heads split over
the ranks) one NCCL all-reduce averages the ranks' shares, captured in the step's graph and run while
the next step records (two share buffers alternate; the last step's all-reduce runs inside the timed
region too). ``value`` is whole-job audited KV tokens/s (one token = one (row, position, layer,
audited KV head) key vector) with inputs resident in HBM; ``e2e`` is the same through the public API
with the step's host inputs copied in from pinned memory and its shares copied out every step.
``view`` times the block-view build of the view stress shape (1024 rows x 8192 blocks, per-row `sum`
budgets), row-sharded over the ranks. ``strong_70b`` times the Llama-3-70B-shaped step in all-heads
mode (every KV head of every layer, split over the ranks: a fixed total, strong scaling). ``parity``
checks sampled rows of the final (rank-combined) shares against the oracle run on each rank's own
inputs, after the timed regions.

``--impl reference`` times the reference algorithm on the host cores instead (the C restatement of
the reference kernel in oracle/, every host thread), on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "sigmod-kvscope_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

HEAD_DIM = 128
BLOCK = 16
TILE_BLOCKS = 2

CONFIGS = {
    # Llama-3.1-8B decode audit on one B200 (the metric's headline configuration)
    "llama8b": dict(rows=64, q_heads=32, kv_heads=8, layers=32, pool=40_000, lens=("uniform", 1024, 8192), pools=8),
    # Llama-3-70B head-sharded audit (the scaling configuration)
    "llama70b": dict(rows=256, q_heads=64, kv_heads=8, layers=80, pool=60_000, lens=("lognormal", 2048, 1.0, 64, 32768),
                     pools=4),
    # long context: 8 rows of 32k-128k tokens
    "long": dict(rows=8, q_heads=32, kv_heads=8, layers=32, pool=66_000, lens=("uniform", 32768, 131072), pools=4),
}

# dram__bytes_read.sum + dram__bytes_write.sum of one record-kernel launch (an audit step of all 32
# layers) of the llama8b workload: an ncu capture of the same launch over 8 layers (`--layers 8
# --pools 1`: one 2.6 GB pool, every layer a head of its own) scaled by 4, the traffic growing with the
# layers (every layer reads its own keys once).
NCU_TRAFFIC_PER_LAUNCH: dict[str, float | None] = {"llama8b": 4 * (614.871e6 + 5.805e6)}
NCU_TRAFFIC_SOURCE = ("ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum of the record kernel, "
                      "bench.py --layers 8 --pools 1 (8 of the 32 layers), scaled by 4; profiles/record_kernel_llama8b.md")


def lengths(spec, rows: int, rng: np.random.Generator) -> np.ndarray:
    if spec[0] == "uniform":
        return rng.integers(spec[1], spec[2] + 1, rows)
    _, median, sigma, lo, hi = spec
    return np.clip(np.round(rng.lognormal(math.log(median), sigma, rows)), lo, hi).astype(np.int64)


def bytes_per_unit(group_rows: int) -> float:
    """Algorithmic DRAM bytes per audited key vector: its K row, its table entry (per block), the
    m and l cells (per block, G values each), and the share accumulator write (per block)."""
    return 2 * HEAD_DIM + 4 / BLOCK + 8 * group_rows / BLOCK + 4 / BLOCK


def measured_peak() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def host_threads() -> int:
    """Every host core this process may run on (not OMP_NUM_THREADS, which torchrun sets to 1)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class ClockSampler:
    """nvidia-smi clock and throttle samples every 100 ms while the sampler is open."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        deadline = time.time() + 5.0  # let the sampler print its first line before timing starts
        while time.time() < deadline and os.path.getsize(self.path) == 0:
            time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        if self.path and os.path.exists(self.path):
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 9:
                    rows.append(parts)
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows), "span": "warm-up through the last timed section"}


# ---- the workload -------------------------------------------------------------------------------------


def plan(cfg: dict, mode: str, world: int) -> dict:
    """What a rank's workload holds, computed on the host alone (both arms report the same config)."""
    if cfg["kv_heads"] % world:
        raise SystemExit(f"{cfg['kv_heads']} KV heads do not split over {world} GPUs")
    lens = lengths(cfg["lens"], cfg["rows"], np.random.default_rng(0)).astype(np.int32)
    kv_local = cfg["kv_heads"] // world
    heads = kv_local if mode == "all-heads" else 1
    # reference mode: a layer audits one KV head, head layer % kv_heads (the reference's rule), so
    # ceil(layers / kv_heads) pools give every layer keys of its own, as a model's layers have; all-heads
    # mode reads every head of a layer's pool and cycles over the configured pools
    pools = cfg["pools"] if mode == "all-heads" or cfg.get("pools_fixed") else -(-cfg["layers"] // kv_local)
    return dict(lens=lens, kv_local=kv_local, heads=heads, pools=pools, width=int(math.ceil(lens.max() / BLOCK)),
                units_rank=int(lens.astype(np.int64).sum()) * cfg["layers"] * heads)


def line_config(name: str, cfg: dict, mode: str, record: str, world: int) -> dict:
    p = plan(cfg, mode, world)
    return {"workload": name, "mode": mode, "record": record, "rows": cfg["rows"], "layers": cfg["layers"],
            "q_heads": cfg["q_heads"], "kv_heads": cfg["kv_heads"], "kv_heads_per_gpu": p["kv_local"],
            "audited_heads_per_layer_per_gpu": p["heads"], "block_size": BLOCK, "tile_blocks": TILE_BLOCKS,
            "mean_len": float(p["lens"].mean()), "width": p["width"], "pools": p["pools"],
            "l2": f"inputs larger than L2: {p['units_rank'] / cfg['layers'] * 256 / 1e6:.0f} MB of keys per launch",
            "parallelism": f"tp{world} (KV heads)"}


class Workload:
    """Seeded synthetic inputs of one rank: KV pools, block tables, lengths and queries on the device."""

    def __init__(self, cfg: dict, rank: int, world: int, mode: str, seed: int = 0) -> None:
        self.cfg = cfg
        self.rows, self.layers = cfg["rows"], cfg["layers"]
        self.group_rows = cfg["q_heads"] // cfg["kv_heads"]
        p = plan(cfg, mode, world)
        self.kv_local, self.heads = p["kv_local"], p["heads"]
        rng = np.random.default_rng(seed)  # identical on every rank: one batch, heads split
        self.lens = lengths(cfg["lens"], self.rows, rng).astype(np.int32)
        assert np.array_equal(self.lens, p["lens"])
        self.width = p["width"]
        blocks = -(-self.lens // BLOCK)
        pool = max(cfg["pool"], int(blocks.sum()) + 1)
        self.pool = pool
        # distinct random blocks for the positions each row holds; the rest of a row is never read
        ids = rng.permutation(pool)[: int(blocks.sum())].astype(np.int32)
        table = np.zeros((self.rows, self.width), dtype=np.int32)
        start = 0
        for r, n in enumerate(blocks):
            table[r, :n] = ids[start : start + n]
            start += n
        self.table_host = table
        dev = torch.device("cuda", torch.cuda.current_device())
        gen = torch.Generator(device=dev).manual_seed(1000 + rank)
        self.caches = [
            torch.randn(pool, 2, BLOCK, self.kv_local, HEAD_DIM, device=dev, generator=gen, dtype=torch.bfloat16)
            for _ in range(p["pools"])
        ]
        tokens = self.rows
        self.queries = [  # every layer's query of the step, resident in HBM
            torch.randn(tokens, self.kv_local * self.group_rows, HEAD_DIM, device=dev, generator=gen,
                        dtype=torch.bfloat16) for _ in range(self.layers)
        ]
        # the engine's step inputs, block table then lengths, in one buffer that one copy fills
        self.inputs_host = np.concatenate([table.ravel(), self.lens])
        self.inputs = torch.from_numpy(self.inputs_host).to(dev)
        self.table = self.inputs[: table.size].view(self.rows, self.width)
        self.lens_t = self.inputs[table.size :]
        self.qrow = np.arange(self.rows, dtype=np.int32)
        self.select = np.ones(self.rows, dtype=bool)
        self.scale = 1.0 / math.sqrt(HEAD_DIM)

    def units_per_step(self) -> int:
        return int(self.lens.astype(np.int64).sum()) * self.layers * self.heads

    def pool_index(self, layer: int) -> int:
        """In reference mode layer l reads head l % kv_heads of pool l // kv_heads: no two layers read the
        same keys, so no read is served from L2 by another layer's."""
        if self.heads > 1 or self.cfg.get("pools_fixed"):
            return layer % len(self.caches)
        return (layer // self.kv_local) % len(self.caches)

    def cache(self, layer: int) -> torch.Tensor:
        return self.caches[self.pool_index(layer)]

    def keys(self, layer: int) -> torch.Tensor:
        return self.cache(layer)[:, 0]

    def query(self, layer: int) -> torch.Tensor:
        return self.queries[layer]


def make_plane(w: Workload, deferred: bool):
    from ekv.runtime.audit_kernel import RecordingPlane

    os.environ.setdefault("EKV_RUNTIME_DIR", tempfile.mkdtemp(prefix="ekv_bench_"))
    plane = RecordingPlane(w.layers, w.rows, w.width, w.group_rows, BLOCK, heads=w.heads, deferred=deferred)
    plane.attach([w.cache(layer).data_ptr() for layer in range(w.layers)])
    plane.select(w.select, w.qrow)
    plane.set(True)
    return plane


def audit_step(plane, w: Workload) -> None:
    """One audit step through RecordingPlane.record's path: a call per layer (deferred: a query stash
    per layer and one launch of every layer after the last; per-layer: a launch per layer)."""
    for layer in range(w.layers):
        plane.launch(layer, w.table, w.lens_t, w.query(layer), w.keys(layer), w.scale)


def audit_step_resident(plane, w: Workload, shares: bool = True) -> None:
    """One audit step from queries resident per layer: one launch of every layer (record_step)."""
    plane.record_step(w.table, w.lens_t, [w.query(layer) for layer in range(w.layers)],
                      [w.cache(layer) for layer in range(w.layers)], w.scale, shares=shares)


def capture(fn) -> torch.cuda.CUDAGraph:
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        fn()  # warm: one-time kernel attributes are set outside the capture
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize()
    return graph


def timed(fn, steps: int, warmup: int, dist_on: bool, finish=None) -> float:
    """Seconds for `steps` calls of fn (then `finish`, inside the timed region), max over ranks; CUDA
    events on the current stream."""
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    if finish is not None:
        finish()
    torch.cuda.synchronize()
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    if finish is not None:
        finish()
    end.record()
    torch.cuda.synchronize()
    seconds = start.elapsed_time(end) / 1e3
    if dist_on:
        t = torch.tensor([seconds], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        seconds = float(t.item())
    return seconds


class Stepper:
    """One audit step as the timed loop calls it: a CUDA graph on one rank; with ranks, the graphs of a
    StepCombiner (this step recorded, the previous step's shares combined) and a final flush."""

    def __init__(self, plane, record, dist_on: bool) -> None:
        self.plane = plane
        self.combiner = None
        if dist_on:
            from ekv.observe.ranks import StepCombiner

            self.combiner = StepCombiner(plane, record)
            self.step, self.finish = self.combiner.step, self.combiner.flush
        else:
            self.graph = capture(record)
            self.step, self.finish = self.graph.replay, None

    def shares(self) -> torch.Tensor:
        """The last step's (combined) shares, once `finish` has run."""
        return self.combiner.last() if self.combiner is not None else self.plane.shares()

    def release(self) -> None:
        if self.combiner is not None:
            self.combiner.release()
        self.graph = self.step = self.finish = None


# ---- parity of the combined shares (a checker, after the timed regions) --------------------------------


def oracle_row_shares(w: Workload, sample: np.ndarray) -> np.ndarray:
    """This rank's shares of the sampled rows from the oracle (the C restatement of the reference kernel on
    this rank's own keys and queries, then the reference normalisation): float64 [len(sample), width]."""
    from oracle import audit as oaud
    from oracle import cpu as ocpu
    from oracle import shares as osh

    ocpu.build()
    g = w.group_rows
    lens = w.lens[sample]
    blocks = -(-lens // BLOCK)
    ids = np.unique(np.concatenate([w.table_host[r, :n] for r, n in zip(sample, blocks, strict=True)]))
    remap = np.zeros(w.pool, dtype=np.int32)
    remap[ids] = np.arange(len(ids), dtype=np.int32)
    table = np.where(np.arange(w.width)[None, :] < blocks[:, None], remap[w.table_host[sample]], 0).astype(np.int32)
    ids_dev = torch.from_numpy(ids.astype(np.int64)).to(w.caches[0].device)
    lse = oaud.new_table(w.layers, len(sample), w.width, w.heads * g)
    one = oaud.new_table(1, len(sample), w.width, g)
    qrow = w.qrow[sample]
    select = np.ones(len(sample), dtype=np.uint8)
    # the layers that read one (pool, KV head), so each head's keys cross to the host once
    groups: dict[tuple[int, int], list[tuple[int, int]]] = {}
    for layer in range(w.layers):
        heads = [layer % w.kv_local] if w.heads == 1 else list(range(w.kv_local))
        for slot, h in enumerate(heads):
            groups.setdefault((w.pool_index(layer), h), []).append((layer, slot))
    for (pool, h), uses in groups.items():
        keys = w.caches[pool][ids_dev, 0, :, h : h + 1].contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
        for layer, slot in uses:
            q = w.query(layer)[:, h * g : (h + 1) * g].contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
            one.fill(np.nan)
            ocpu.tile_lse(q, keys, "bf16", table, lens, qrow, select, 1, one, w.scale, 0, 0, BLOCK, TILE_BLOCKS)
            lse[:, layer, :, :, slot * g : (slot + 1) * g] = one[:, 0]
    u = osh.log_weights(lse, w.layers, np.arange(len(sample)), TILE_BLOCKS)
    return osh.normalize_rows(u, blocks, TILE_BLOCKS)


def parity_check(w: Workload, combined: torch.Tensor, rank: int, world: int, dist_on: bool, rows: int) -> dict | None:
    """Sampled rows of the final shares against the mean over ranks of every rank's oracle shares
    (RankedShareSource.read, observe/ranks.py:117-119), gathered to rank 0. Every rank takes part."""
    import torch.distributed as dist

    from oracle import shares as osh

    sample = np.unique(np.linspace(0, w.rows - 1, rows).round().astype(np.int64))
    mine = torch.from_numpy(oracle_row_shares(w, sample)).to(combined.device)
    if dist_on:
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
    else:
        gathered = [mine]
    if rank != 0:
        return None
    want = osh.mean_over_ranks([t.cpu().numpy() for t in gathered])
    got = combined[torch.from_numpy(sample).to(combined.device)].cpu().numpy().astype(np.float64)
    same_nan = bool(np.array_equal(np.isnan(got), np.isnan(want)))
    f = np.isfinite(want) & np.isfinite(got)
    rel = np.abs(got[f] - want[f]) / np.maximum(np.abs(want[f]), 1e-9)
    close = bool(np.allclose(got, want, rtol=1e-3, atol=1e-9, equal_nan=True))
    return {"rows": int(len(sample)), "ranks": world, "max_rel": float(rel.max()) if rel.size else 0.0,
            "ok": same_nan and close, "tolerance": "rtol 1e-3, atol 1e-9, same NaN rows",
            "against": "mean over ranks of each rank's oracle shares"}


# ---- sections of our arm ---------------------------------------------------------------------------------


def view_bench(rank: int, world: int, steps: int, warmup: int, dist_on: bool) -> dict:
    """The view stress shape: 1024 rows x 8192, per-row `sum` budgets, rows split over the ranks."""
    from ekv.runtime.block_view import plan_view

    rows_total, width = 1024, 8192
    gen = torch.Generator().manual_seed(0)
    n = torch.randint(1, width + 1, (rows_total,), generator=gen).to(torch.int32)
    table = torch.randint(0, 2**20, (rows_total, width), generator=gen, dtype=torch.int32)
    scores = torch.distributions.Dirichlet(torch.full((width,), 0.3, dtype=torch.float64)).sample((rows_total,))
    scores = torch.where(torch.arange(width)[None, :] < n[:, None].long(), scores, torch.zeros_like(scores)).float()
    fraction = 0.2 + 0.8 * torch.rand(rows_total, generator=gen, dtype=torch.float64)
    lens = n * BLOCK
    mine = slice(rank * rows_total // world, (rank + 1) * rows_total // world)
    dev = torch.device("cuda", torch.cuda.current_device())
    t, nn, ln, sc, fr = (x[mine].contiguous().to(dev) for x in (table, n, lens, scores, fraction))
    out = (torch.empty_like(t), torch.empty(len(nn), dtype=torch.int32, device=dev))

    def build():
        plan_view(t, ln, BLOCK, nn, scores=sc, policy="sum", row_fraction=fr, recent_blocks=0, out=out)

    def build_shared():  # the controller's default: `sum` with one budget over every row
        plan_view(t, ln, BLOCK, nn, scores=sc, policy="sum", budget_fraction=0.5, recent_blocks=4, out=out)

    def build_maxmin():  # one budget: raise the lowest retained share first
        plan_view(t, ln, BLOCK, nn, scores=sc, policy="maxmin", budget_fraction=0.5, recent_blocks=4, out=out)

    newest = torch.arange(width, dtype=torch.float32, device=dev).expand(len(nn), width).contiguous()
    # float64 scores, as the controller smooths them: 0.5 * older shares + 0.5 * the latest audit's
    older = torch.distributions.Dirichlet(torch.full((width,), 0.3, dtype=torch.float64)).sample((rows_total,))
    sc64 = (0.5 * older[mine].to(dev) + 0.5 * sc.double()).contiguous()

    def build_shared64():  # the controller's default over float64 shares, ranked by the float64 gains
        plan_view(t, ln, BLOCK, nn, scores=sc64, policy="sum", budget_fraction=0.5, recent_blocks=4, out=out)

    # the controller's decide stage on the device: fold an audit of every row into the per-request ledger,
    # then the committed keep mask of every row (one host synchronisation: the evidence bytes)
    from ekv.observe.controller import ShareLedger

    ledger = ShareLedger(width, capacity=len(nn))
    req_keys = np.arange(1, len(nn) + 1, dtype=np.uint64) + np.uint64(rank * rows_total)
    req_lens = nn.cpu().numpy().astype(np.int64)
    ledger.absorb(sc, req_keys, req_lens)

    def controller_tick():
        ledger.absorb(sc, req_keys, req_lens)
        ledger.keep_mask(req_keys, req_lens, budget_fraction=0.5, objective="sum", recent_blocks=4)

    def build_newest():  # keep-newest: scores = arange(n) under `uniform`, budget 0.5
        plan_view(t, ln, BLOCK, nn, scores=newest, policy="uniform", budget_fraction=0.5, recent_blocks=0, out=out)

    # SGLang's CSR list: 256 decode rows of U[1, 8192] tokens (int64 slots), half the blocks kept
    from ekv.runtime.sglang_compact import SlotCompactor

    slot_rows, slot_width = 256, 512
    sl_lens = torch.randint(1, slot_width * BLOCK + 1, (slot_rows,), generator=gen)
    sl_indptr = torch.cat([torch.zeros(1, dtype=torch.int64), sl_lens.cumsum(0)]).to(torch.int32).to(dev)
    entries = int(sl_lens.sum())
    sl_slots = torch.randint(0, 1 << 30, (entries,), generator=gen, dtype=torch.int64).to(dev)
    sl_keep = (torch.rand(slot_rows, slot_width, generator=gen) < 0.5).to(dev)
    work_indptr, work_slots = sl_indptr.clone(), sl_slots.clone()
    compactor = SlotCompactor(slot_width, BLOCK, dev)

    def restore():  # the compaction rewrites its input in place
        work_indptr.copy_(sl_indptr)
        work_slots.copy_(sl_slots)

    def slot_step():
        restore()
        compactor.compact(work_indptr, work_slots, sl_keep, None, True, slot_rows, slot_rows, entries)

    ids = int(n.long().sum())
    result = {"rows": rows_total, "width": width, "ids": ids, "policy": "sum per row", "rows_per_gpu": len(nn)}
    for key, fn in (("sglang_restore_us", restore), ("sglang_us", slot_step)):
        graph = capture(fn)
        result[key] = round(timed(graph.replay, steps, warmup, dist_on) / steps * 1e6, 2)
        del graph
    result["sglang_us"] = round(result["sglang_us"] - result.pop("sglang_restore_us"), 2)
    result["sglang_entries"] = entries
    result["sglang_launches"] = 4
    for key, fn, launches in (("us", build, 1), ("sum_shared_us", build_shared, 10), ("maxmin_shared_us", build_maxmin, 6),
                              ("newest_us", build_newest, 2), ("sum_shared_f64_us", build_shared64, 10)):
        graph = capture(fn)
        result[key] = round(timed(graph.replay, steps, warmup, dist_on) / steps * 1e6, 2)
        result[key.replace("us", "launches")] = launches
        del graph
    # not capturable (the fold reads its evidence bytes back): timed as called, host work included
    result["controller_tick_us"] = round(timed(controller_tick, steps, warmup, dist_on) / steps * 1e6, 2)
    result["controller_tick_launches"] = 11
    return result


def record_roofline(plane, w: Workload, steps: int, warmup: int, dist_on: bool) -> dict:
    """The record kernel alone (one launch per audit step of every layer), timed over its own launches."""
    graph = capture(lambda: audit_step_resident(plane, w, shares=False))
    launch_seconds = timed(graph.replay, steps, warmup, dist_on) / steps
    del graph
    units = w.units_per_step()
    b_unit = bytes_per_unit(w.heads * w.group_rows)
    achieved = units * b_unit / launch_seconds / 1e9
    peak, peak_kind = measured_peak()
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_kind": peak_kind, "kernel": "record_kernel", "bytes_per_unit": b_unit, "units_per_launch": units,
            "launch_us": launch_seconds * 1e6}


def strong_70b(args, rank: int, world: int, dist_on: bool) -> dict:
    """The Llama-3-70B-shaped step in all-heads mode: every KV head of every layer, split over the ranks."""
    cfg = CONFIGS["llama70b"]
    w = Workload(cfg, rank, world, "all-heads")
    plane = make_plane(w, deferred=True)
    stepper = Stepper(plane, lambda: audit_step_resident(plane, w), dist_on)
    steps = max(10, min(args.steps, 40))
    seconds = timed(stepper.step, steps, args.warmup, dist_on, stepper.finish)
    if plane.status():
        raise SystemExit(f"the audit kernel reported status {plane.status()} (70B all-heads step)")
    parity = parity_check(w, stepper.shares(), rank, world, dist_on, rows=3)
    stepper.release()
    roofline = record_roofline(plane, w, steps, args.warmup, dist_on)
    units_all = w.units_per_step() * world
    result = {"value": units_all * steps / seconds, "unit": "audited KV tokens/s", "steps": steps,
              "warmup": args.warmup, "ms_per_step": seconds / steps * 1e3, "units_per_step": units_all,
              "scaling": "strong", "config": line_config("llama70b", cfg, "all-heads", "deferred", world),
              "roofline": roofline, "parity": parity,
              "note": "every KV head of every layer (cells of kv_heads_per_gpu x 8 query rows), the total split "
                      "over the ranks; shares averaged over the ranks in the step's graph"}
    plane.close()
    del plane, w
    torch.cuda.empty_cache()
    return result


# ---- the CPU arms ----------------------------------------------------------------------------------------


class CpuSample:
    """The C restatement of the reference kernel (oracle/audit_cpu.c) on every host thread, over a
    sample of the workload: all its rows and lengths, one KV head's keys (the audited head of a
    layer), repeated for as many layers as the time target allows; then the rest of the reference's
    CPU path on that sample: the normalisation, the controller's `sum` allocation at budget 0.5 and
    the compaction."""

    def __init__(self, cfg: dict) -> None:
        from oracle import audit as oaud
        from oracle import cpu as ocpu

        ocpu.build()
        self.ocpu, self.oaud = ocpu, oaud
        rng = np.random.default_rng(0)
        self.lens = lengths(cfg["lens"], cfg["rows"], rng).astype(np.int32)
        self.g_rows = cfg["q_heads"] // cfg["kv_heads"]
        self.rows = cfg["rows"]
        self.cfg_layers = cfg["layers"]
        self.width = int(math.ceil(self.lens.max() / BLOCK))
        blocks = -(-self.lens // BLOCK)
        pool = int(blocks.sum()) + 1
        gen = np.random.default_rng(1)
        k = gen.standard_normal((pool, BLOCK, 1, HEAD_DIM), dtype=np.float32)
        self.k16 = (k.view(np.uint32) >> 16).astype(np.uint16)  # bf16 bit patterns
        q = gen.standard_normal((self.rows, self.g_rows, HEAD_DIM), dtype=np.float32)
        self.q16 = (q.view(np.uint32) >> 16).astype(np.uint16)
        ids = gen.permutation(pool)[: int(blocks.sum())].astype(np.int32)
        self.table = np.zeros((self.rows, self.width), dtype=np.int32)
        start = 0
        for r, n in enumerate(blocks):
            self.table[r, :n] = ids[start : start + n]
            start += n
        self.threads = host_threads()
        self.layers = 1
        self.lse = None

    def run(self, layers: int) -> tuple[float, int]:
        lse = self.oaud.new_table(layers, self.rows, self.width, self.g_rows)
        qrow = np.arange(self.rows, dtype=np.int32)
        select = np.ones(self.rows, dtype=np.uint8)
        t0 = time.perf_counter()
        for layer in range(layers):
            self.ocpu.tile_lse(self.q16, self.k16, "bf16", self.table, self.lens, qrow, select, 1, lse,
                               1 / math.sqrt(HEAD_DIM), layer, 0, BLOCK, TILE_BLOCKS, self.threads)
        seconds = time.perf_counter() - t0
        self.lse = lse
        return seconds, int(self.lens.astype(np.int64).sum()) * layers

    def calibrate(self, seconds_target: float) -> None:
        sec, units = self.run(1)
        self.layers = max(1, int(seconds_target / max(sec, 1e-6)))

    def later_stages(self) -> dict:
        """Seconds of the normalisation (scaled to every layer of a step), the allocation and the
        compaction over the last run's table."""
        from oracle import allocation as oa
        from oracle import shares as osh
        from oracle import view as oview

        layers = self.lse.shape[1]
        row_blocks = -(-self.lens // BLOCK)
        t0 = time.perf_counter()
        u = osh.log_weights(self.lse, layers, np.arange(self.rows), TILE_BLOCKS)
        share = osh.normalize_rows(u, row_blocks, TILE_BLOCKS)
        t1 = time.perf_counter()
        scores = np.nan_to_num(share, nan=0.0)
        keep = oa.controller_keep(row_blocks, self.width, lambda r, n: scores[r, :n], 0.5, "sum", recent_blocks=4)
        t2 = time.perf_counter()
        oview.compact_block_table(self.table, self.lens, keep, BLOCK)
        t3 = time.perf_counter()
        return {"normalize": (t1 - t0) * self.cfg_layers / layers, "allocate_sum": t2 - t1, "compact": t3 - t2}

    def describe(self, units: int) -> str:
        return (f"{self.rows} rows x {self.layers} layers of the workload ({units} key vectors, one KV head's keys "
                f"per layer), C restatement of tile_lse_kernel on {self.threads} OpenMP threads; then the numpy "
                f"normalisation, the controller's sum allocation (budget 0.5, 4 recent blocks) and the compaction")


def cpu_sample(cfg: dict, seconds_target: float, heads_all: int) -> dict:
    """Audited tokens/s of the reference algorithm on the host cores, over a bounded sample, and the
    reference's whole CPU path per step at that rate."""
    sample = CpuSample(cfg)
    sample.calibrate(seconds_target)
    sec, units = sample.run(sample.layers)
    rate = units / sec
    stages = sample.later_stages()
    step_units = int(sample.lens.astype(np.int64).sum()) * cfg["layers"] * heads_all
    stages_ms = {"tile_lse": step_units / rate * 1e3} | {k: v * 1e3 for k, v in stages.items()}
    path_ms = sum(stages_ms.values())
    return {"value": rate, "unit": "audited KV tokens/s", "cores": sample.threads, "kind": "port",
            "sample": sample.describe(units), "seconds": round(sec, 2),
            "stages_ms_per_step": {k: round(v, 3) for k, v in stages_ms.items()},
            "path_ms_per_step": round(path_ms, 3), "path_value": step_units / path_ms * 1e3}


def reference_arm(args, cfg: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sample = CpuSample(cfg)
    sample.calibrate(seconds_target=2.0)
    rates, units = [], 0
    for step in range(args.warmup + args.steps):
        sec, units = sample.run(sample.layers)
        if step >= args.warmup:
            rates.append(units / sec)
    value = statistics.median(rates)
    # one whole-job step of the workload (every rank's heads of every layer) at that rate
    heads_all = args.gpus if args.mode == "reference" else cfg["kv_heads"]
    step_units = int(sample.lens.astype(np.int64).sum()) * cfg["layers"] * heads_all
    line = {
        "impl": "reference", "metric": "audited KV tokens/s", "value": value, "unit": "audited KV tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_units / value * 1e3, "higher_is_better": True,
        "scaling": "weak" if args.mode == "reference" else "strong", "dtype": "bf16", "data": "synthetic",
        "config": line_config(args.config, cfg, args.mode, args.record, args.gpus),
        "cpu_baseline": {"kind": "port", "cores": sample.threads, "sample": sample.describe(units), "value": value,
                         "unit": "audited KV tokens/s"},
        "e2e": {"value": value, "unit": "audited KV tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


# ---- our arm ---------------------------------------------------------------------------------------------


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", choices=sorted(CONFIGS), default="llama8b")
    ap.add_argument("--mode", choices=["reference", "all-heads"], default="reference")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the timed CPU sample")
    ap.add_argument("--no-view", action="store_true", help="skip the block-view build timing")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end timing")
    ap.add_argument("--no-strong", action="store_true", help="skip the 70B all-heads strong-scaling step")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the final shares")
    ap.add_argument("--pools", type=int, default=None,
                    help="a fixed number of KV pools cycled over the layers (default: reference mode gives every "
                         "layer keys of its own)")
    ap.add_argument("--layers", type=int, default=None, help="audit this many layers instead of the model's")
    ap.add_argument("--record", choices=["deferred", "per-layer"], default="deferred",
                    help="RecordingPlane mode: every layer in one launch after the last, or a launch per layer")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    cfg = dict(CONFIGS[args.config])
    if args.layers:  # fewer layers (profiling: with one pool, every layer still reads a head of its own)
        cfg["layers"] = args.layers
    if args.pools:  # a fixed number of pools, cycled over the layers (profiling: a few GB on the device)
        cfg["pools"] = args.pools
        cfg["pools_fixed"] = True
    if args.impl == "reference":
        reference_arm(args, cfg)
        return

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist_on = world > 1
    if dist_on:
        from datetime import timedelta

        # the communicator's set-up may print a version banner on the process's stdout, where the one JSON
        # line goes: send file descriptor 1 to stderr until the first collective has run
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    import ekv.build

    ekv.build.build()

    w = Workload(cfg, rank, world, args.mode)
    plane = make_plane(w, deferred=args.record == "deferred")
    record = (lambda: audit_step_resident(plane, w)) if args.record == "deferred" else (lambda: audit_step(plane, w))
    stepper = Stepper(plane, record, dist_on)

    with ClockSampler(local) as clocks:
        seconds = timed(stepper.step, args.steps, args.warmup, dist_on, stepper.finish)
        status = plane.status()
        if status:
            raise SystemExit(f"the audit kernel reported status {status}")
        # the roofline of the dominant kernel: the record kernel alone, one launch per audit step (deferred),
        # timed over its own launches right after the step, on the same plane and inputs
        roofline = record_roofline(plane, w, args.steps, args.warmup, dist_on) if args.record == "deferred" else None
        parity = None
        if not args.no_parity:
            parity = parity_check(w, stepper.shares(), rank, world, dist_on, rows=4)
        stepper.release()
        per_layer = None
        if args.record == "deferred" and not args.no_e2e:
            # the same step recorded layer by layer (a launch per layer), for comparison
            plane_pl = make_plane(w, deferred=False)
            graph_pl = capture(lambda: audit_step(plane_pl, w))
            pl_seconds = timed(graph_pl.replay, args.steps, args.warmup, dist_on)
            per_layer = {"value": w.units_per_step() * world * args.steps / pl_seconds, "unit": "audited KV tokens/s",
                         "ms_per_step": pl_seconds / args.steps * 1e3}
            del graph_pl
            plane_pl.close()
        units_rank = w.units_per_step()
        units_all = units_rank * world
        value = units_all * args.steps / seconds
        # per-layer: the record kernel is the step, a launch per layer
        if roofline is None:
            peak, peak_kind = measured_peak()
            launch_seconds = seconds / args.steps / w.layers
            b_unit = bytes_per_unit(w.heads * w.group_rows)
            achieved = units_rank / w.layers * b_unit / launch_seconds / 1e9
            roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                        "peak_kind": peak_kind, "kernel": "record_kernel", "bytes_per_unit": b_unit,
                        "units_per_launch": units_rank / w.layers, "launch_us": launch_seconds * 1e6}
        roofline["note"] = ("record kernel alone, one launch per audit step of every layer (per-layer: one per "
                            "layer); CUDA events over its own timed launches")

        # e2e: the step's host inputs in from pinned memory, the shares out, every step (the engine's block
        # table and lengths: one copy; the selection: RecordingPlane.select, one copy). The steps alternate
        # two share buffers (a StepCombiner's two graphs; with ranks, a step's shares are combined while
        # the next step records): each step's shares are copied out on a copy stream once they are complete,
        # the next step writing the other buffer meanwhile, and the host waits for them one step later.
        from ekv.observe.ranks import StepCombiner

        pinned_inputs = torch.from_numpy(w.inputs_host).pin_memory()
        share0 = plane.shares()
        out_host = [torch.empty(share0.shape, dtype=share0.dtype).pin_memory() for _ in range(2)]
        copied = [torch.cuda.Event(), torch.cuda.Event()]
        copy_stream = torch.cuda.Stream()
        api = StepCombiner(plane, lambda: audit_step(plane, w))
        e2e = {"copied": -1, "pending": [False, False]}  # the last step copied out; copies not yet waited for

        def copy_out(step: int) -> None:
            b = step % 2
            copy_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(copy_stream):
                out_host[b].copy_(api.buffers[b], non_blocking=True)
                copied[b].record(copy_stream)
            e2e["copied"], e2e["pending"][b] = step, True

        def e2e_step():
            w.inputs.copy_(pinned_inputs, non_blocking=True)
            plane.select(w.select, w.qrow)
            b = api.steps % 2  # the buffer this step records into: its last copy out must have run
            if e2e["pending"][b]:
                torch.cuda.current_stream().wait_event(copied[b])
            api.step()
            done = api.steps - 1 if not dist_on else api.steps - 2  # the last step whose shares are complete
            if done > e2e["copied"]:
                copy_out(done)
                prev = 1 - done % 2
                if e2e["pending"][prev]:
                    copied[prev].synchronize()  # the host holds the step before's shares
                    e2e["pending"][prev] = False

        def e2e_finish():
            if dist_on and api.steps - 1 > e2e["copied"]:
                api.flush()  # the last step's combine
                copy_out(api.steps - 1)
            torch.cuda.current_stream().wait_stream(copy_stream)  # every copy out inside the timed region

        e2e_seconds = timed(e2e_step, args.steps, args.warmup, dist_on, e2e_finish) if not args.no_e2e else float("nan")
        api.release()
        h2d = pinned_inputs.nbytes + 5 * w.rows  # select(): a token row (int32) and a flag per row
        d2h = out_host[0].nbytes
        view = None if args.no_view else view_bench(rank, world, args.steps, args.warmup, dist_on)
        strong = None
        if not args.no_strong and args.config == "llama8b" and not args.layers and not args.pools:
            plane.close()
            del plane, stepper, api
            w.caches, w.queries = [], []  # the 70B step's pools take their place
            torch.cuda.empty_cache()
            strong = strong_70b(args, rank, world, dist_on)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_sample(cfg, seconds_target=10.0, heads_all=w.heads * world)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    traffic_applies = (args.mode == "reference" and args.record == "deferred" and not args.layers and not args.pools
                       and world == 1)
    roofline["traffic"] = NCU_TRAFFIC_PER_LAUNCH.get(args.config) if traffic_applies else None
    roofline["traffic_source"] = NCU_TRAFFIC_SOURCE if roofline["traffic"] is not None else None
    line = {
        "metric": "audited KV tokens/s", "value": value, "unit": "audited KV tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": seconds / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak" if args.mode == "reference" else "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": line_config(args.config, cfg, args.mode, args.record, world),
        "roofline": roofline,
        "e2e": {"value": units_all * args.steps / e2e_seconds, "unit": "audited KV tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "RecordingPlane.select (one copy from pinned staging), then RecordingPlane.record per "
                        "layer (a query stash per layer on parallel side streams, one launch of every layer "
                        "after the last) in CUDA graphs alternating two share buffers; the block table and "
                        "lengths in by one copy from pinned host memory, each step's shares out to pinned "
                        "memory on a copy stream, the host waiting for them one step later; KV cache resident"},
        # per step: the descriptor, record and share kernels (deferred), or a record kernel per layer plus
        # the share kernel (per-layer)
        "gpu_launches": args.steps * (3 if args.record == "deferred" else w.layers + 1),
        "clocks": clocks.summary(),
        "parity": parity,
        "combine": ("one NCCL all-reduce (average) per step in the step's CUDA graph, overlapping the next "
                    "step's audit; the last step's inside the timed region") if dist_on else None,
        "per_layer_launches": per_layer,
        "view": view,
        "strong_70b": strong,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
