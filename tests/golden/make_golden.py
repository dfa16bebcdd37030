"""Generate the golden fixtures of tests/golden/ by running the reference's own code.

Run in a container that has the reference checkout, named by $EKV_REFERENCE (its root directory, the
one that holds ``runtime/`` and ``observe/``):

    EKV_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports the reference read-only and runs, on CPU:
  * its Triton audit kernel ``tile_lse_kernel`` (runtime/audit_kernel.py:34-109) under
    ``TRITON_INTERPRET=1``, launched as RecordingPlane.launch does (:239-265). bf16 cases are run on
    the exact float32 upcast, because the interpreter's ``tl.dot`` on bf16 is wrong;
  * ``read_tile_rows`` and ``normalize_tile_lse`` (observe/tile_shares.py) through a fake D2H reader;
  * ``allocate`` (observe/allocation.py) with the pins and budget of Controller._allocate;
  * ``compact_block_table`` (runtime/block_view.py:36-56);
  * ``SlotCompactor.compact`` (runtime/sglang_compact.py), the SGLang CSR compaction, both Triton
    kernels under the interpreter;
  * ``allocate`` on float64 scores whose shares round together (``float64_cases``);
  * ``allocate`` with pinned blocks anywhere in a request (``pinned_cases``);
  * ``Controller._absorb_audit`` and ``Controller._allocate`` (observe/controller.py) over a sequence
    of audits, with stand-ins for the mailbox writer and the share source (``controller_cases``).
Inputs are seeded; the fixtures hold inputs and outputs, so the tests never need the reference.
"""

from __future__ import annotations

import math
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
REFERENCE = os.environ.get("EKV_REFERENCE")
if not REFERENCE or not os.path.isdir(os.path.join(REFERENCE, "runtime")):
    raise SystemExit("set EKV_REFERENCE to the reference checkout (the directory holding runtime/ and observe/)")
sys.path.insert(0, REFERENCE)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402
from observe.allocation import Request, allocate  # noqa: E402
from observe.tile_shares import normalize_tile_lse, read_tile_rows  # noqa: E402
from runtime.audit_kernel import TILE_BLOCKS, tile_lse_kernel  # noqa: E402
from runtime.block_view import compact_block_table  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_launch(lse, layers, rows, width, group_rows, block_size, layer, table, lens, query, keys,
                     scale, token, select, flag):
    """tile_lse_kernel launched with the arguments RecordingPlane.launch gives it, on CPU tensors."""
    kv_heads = keys.shape[2]
    tile_lse_kernel[(rows, triton.cdiv(width, TILE_BLOCKS))](
        query, keys, table, lens, token, select, flag, lse, scale, layer, layer % kv_heads,
        query.stride(0), query.stride(1), keys.stride(0), keys.stride(1), keys.stride(2), table.stride(0),
        rows * width * group_rows, width * group_rows, layers * rows * width * group_rows,
        BLOCK_SIZE=block_size, TILE_BLOCKS=TILE_BLOCKS, GROUP_ROWS=group_rows, ROWS_PAD=16,
        HEAD_DIM=keys.shape[3],
    )


class FakeCuda:
    """Serves the D2H reads of read_tile_rows from a host copy of the table."""

    def __init__(self, blob: bytes) -> None:
        self.blob = blob

    def d2h_many(self, requests):
        return [self.blob[a : a + n] for a, n in requests]


def audit_case(name, seed, rows, q_heads, kv_heads, layers, len_lo, len_hi, pool, dtype, select=None,
               flags=None, width=None, block_size=16):
    rng = np.random.default_rng(seed)
    head_dim = 128
    group_rows = q_heads // kv_heads
    lens = rng.integers(len_lo, len_hi + 1, rows).astype(np.int32)
    width = width or int(math.ceil(lens.max() / block_size)) + 2
    perm = rng.permutation(pool).astype(np.int32)
    table = perm[(np.arange(rows)[:, None] * width + np.arange(width)[None, :]) % pool].astype(np.int32)
    tokens = rows + 3
    qrow = rng.permutation(tokens)[:rows].astype(np.int32)
    select = np.ones(rows, dtype=np.uint8) if select is None else np.asarray(select, dtype=np.uint8)
    flags = [1] * layers if flags is None else flags
    scale = 1.0 / math.sqrt(head_dim)
    np_dtype = np.float16 if dtype == "fp16" else np.float32
    queries, pools = [], []
    for _layer in range(layers):
        q = rng.standard_normal((tokens, q_heads, head_dim)).astype(np.float32)
        k = np.zeros((pool, block_size, kv_heads, head_dim), dtype=np.float32)  # unused blocks stay 0
        used = np.unique(np.concatenate([table[r, : -(-int(lens[r]) // block_size)] for r in range(rows)]))
        k[used] = rng.standard_normal((len(used), block_size, kv_heads, head_dim)).astype(np.float32)
        if dtype == "bf16":  # values exactly representable in bf16
            q = torch.from_numpy(q).to(torch.bfloat16).float().numpy()
            k = torch.from_numpy(k).to(torch.bfloat16).float().numpy()
        queries.append(q.astype(np_dtype))
        pools.append(k.astype(np_dtype))
    lse = torch.full((2 * layers * rows * width * group_rows,), float("nan"), dtype=torch.float32)
    t_table, t_lens = torch.from_numpy(table), torch.from_numpy(lens)
    t_token, t_select = torch.from_numpy(qrow), torch.from_numpy(select)
    for layer in range(layers):
        flag = torch.tensor([flags[layer]], dtype=torch.int32)
        q = torch.from_numpy(queries[layer].astype(np.float16 if dtype == "fp16" else np.float32))
        k = torch.from_numpy(pools[layer].astype(np.float16 if dtype == "fp16" else np.float32))
        kv = torch.stack([k, torch.zeros_like(k)], dim=1)  # [blocks, 2, block, heads, dim], as vLLM's cache
        reference_launch(lse, layers, rows, width, group_rows, block_size, layer, t_table, t_lens, q,
                         kv[:, 0], scale, t_token, t_select, flag)
    lse_np = lse.numpy().reshape(2, layers, rows, width, group_rows)
    row_blocks = np.where(select != 0, -(-lens // block_size), 0).astype(np.int64)
    live = np.flatnonzero(row_blocks > 0)
    u = read_tile_rows(FakeCuda(lse.numpy().tobytes()), 0, layers, layers, rows, width, group_rows, live, TILE_BLOCKS)
    out = {}
    for aggregate in ("mean", "max"):
        share = np.full((rows, width), np.nan)
        if live.size:
            share[live] = normalize_tile_lse(u, row_blocks[live], TILE_BLOCKS, aggregate)
        out[f"share_{aggregate}"] = share
    # the controller's uniform keep mask at budget 0.5 with its default pins, and the view
    recent = 4
    requests, chosen = [], []
    for r in range(rows):
        n = int(row_blocks[r])
        if n <= 0:
            continue
        pinned = np.zeros(n, dtype=bool)
        pinned[0] = True
        pinned[max(0, n - 1 - recent):] = True
        requests.append(Request(scores=np.nan_to_num(out["share_mean"][r, :n], nan=0.0), pinned=pinned))
        chosen.append(r)
    keep = np.ones((rows, width), dtype=np.uint8)
    if requests:
        total = sum(len(q.scores) for q in requests)
        floor = sum(int(q.pinned_mask().sum()) for q in requests)
        budget = max(floor, int(np.ceil(0.5 * total)))
        for r, mask in zip(chosen, allocate(requests, budget, "uniform"), strict=True):
            keep[r, : len(mask)] = mask
    view, view_lens = compact_block_table(t_table, t_lens, torch.from_numpy(keep.astype(bool)), block_size)
    def packed(x):  # fp16 as is; bf16-exact float32 as its upper 16 bits
        x = np.stack(x)
        return x if dtype == "fp16" else (x.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)

    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        query=packed(queries), keys=packed(pools), table=table, lens=lens,
        qrow=qrow, select=select, flags=np.asarray(flags, dtype=np.int32), scale=np.float32(scale),
        block_size=block_size, tile_blocks=TILE_BLOCKS, kv_heads=kv_heads, group_rows=group_rows,
        dtype=dtype, lse=lse_np, u=u, live=live, row_blocks=row_blocks, keep=keep,
        view=view.numpy(), view_lens=view_lens.numpy(), **out,
    )
    print(name, "rows", rows, "width", width, "layers", layers, "written")


def shares_cases():
    """normalize_tile_lse on random u tables with NaN, -inf, partial tails and empty rows."""
    rng = np.random.default_rng(11)
    cases = {}
    for i in range(12):
        layers, rows, width, q = int(rng.integers(1, 5)), int(rng.integers(1, 7)), int(rng.integers(1, 30)), int(rng.integers(1, 9))
        tile_blocks = int(rng.choice([1, 2, 4]))
        u = rng.normal(0, 4, (layers, rows, width, q)).astype(np.float32)
        u[rng.random(u.shape) < 0.1] = np.nan
        u[rng.random(u.shape) < 0.05] = -np.inf
        row_blocks = rng.integers(0, width + 3, rows)
        if i % 4 == 0:
            u[:, 0] = np.nan  # a row with no evidence
        cases[f"u{i}"] = u
        cases[f"rb{i}"] = row_blocks
        cases[f"tb{i}"] = np.int64(tile_blocks)
        for aggregate in ("mean", "max"):
            cases[f"{aggregate}{i}"] = normalize_tile_lse(u, row_blocks, tile_blocks, aggregate)
    # read_tile_rows over a table with a tile of no keys (l = 0)
    table_layers, layers, rows, width, group, tile_blocks = 4, 3, 5, 6, 2, 2
    cells = table_layers * rows * width * group
    m = rng.normal(0, 3, cells).astype(np.float32)
    total = rng.uniform(0.5, 9, cells).astype(np.float32)
    total[7] = 0.0
    blob = np.concatenate([m, total])
    cases["read_table"] = blob
    cases["read_rows"] = np.array([0, 2, 3])
    cases["read_u"] = read_tile_rows(FakeCuda(blob.tobytes()), 0, table_layers, layers, rows, width, group,
                                     cases["read_rows"], tile_blocks)
    np.savez_compressed(os.path.join(HERE, "shares_cases.npz"), **cases)
    print("shares_cases written")


def allocation_cases():
    """allocate() with many ties: uniform over several requests, sum over one and over several."""
    rng = np.random.default_rng(21)
    cases = {}
    for i in range(60):
        n_req = int(rng.integers(1, 6))
        sizes = rng.integers(1, 40, n_req)
        ties = i % 2 == 0
        scores = [
            (rng.integers(0, 4, n).astype(np.float32) if ties else rng.random(n).astype(np.float32)).astype(np.float64)
            for n in sizes
        ]
        if i % 7 == 3:
            scores[0][:] = 0.0  # no evidence: equal shares
        recent = int(rng.integers(0, 5))
        pinned = []
        for n in sizes:
            p = np.zeros(n, dtype=bool)
            p[0] = True
            p[max(0, n - 1 - recent):] = True
            pinned.append(p)
        must = sum(int(p.sum()) for p in pinned)
        total = int(sizes.sum())
        budget = int(rng.integers(must, total + 2))
        objective = "uniform" if i % 3 else "sum"
        requests = [Request(scores=s, pinned=p) for s, p in zip(scores, pinned, strict=True)]
        masks = allocate(requests, budget, objective)
        cases[f"sizes{i}"] = sizes
        cases[f"scores{i}"] = np.concatenate(scores)
        cases[f"recent{i}"] = np.int64(recent)
        cases[f"budget{i}"] = np.int64(budget)
        cases[f"objective{i}"] = objective
        cases[f"mask{i}"] = np.concatenate(masks)
    # keep-newest: the fixed rule scores = arange(n), budget 0.5, no recent pins, 10 blocks
    req = Request(scores=np.arange(10, dtype=float), pinned=np.eye(1, 10, 0, dtype=bool)[0] | np.eye(1, 10, 9, dtype=bool)[0])
    cases["newest_mask"] = allocate([req], max(2, int(np.ceil(0.5 * 10))), "uniform")[0]
    np.savez_compressed(os.path.join(HERE, "allocation_cases.npz"), **cases)
    print("allocation_cases written")


def view_cases():
    """compact_block_table on 300 random batches, as the reference's own randomized check draws them."""
    rng = np.random.default_rng(31)
    cases = {}
    for i in range(300):
        rows, width = int(rng.integers(1, 7)), int(rng.integers(1, 41))
        table = rng.integers(1, 10_000, (rows, width)).astype(np.int32)
        lens = rng.integers(0, width * 16 + 1, rows).astype(np.int32)
        keep = rng.random((rows, width)) < 0.5
        view, view_lens = compact_block_table(torch.from_numpy(table), torch.from_numpy(lens), torch.from_numpy(keep), 16)
        cases[f"table{i}"], cases[f"lens{i}"], cases[f"keep{i}"] = table, lens, keep
        cases[f"view{i}"], cases[f"view_lens{i}"] = view.numpy(), view_lens.numpy()
    np.savez_compressed(os.path.join(HERE, "view_cases.npz"), **cases)
    print("view_cases written")


def maxmin_cases():
    """allocate(..., "maxmin") (observe/allocation.py:121-166): requests with ties, without evidence, of one
    block, and budgets from just above the pins to just below every block."""
    rng = np.random.default_rng(47)
    cases = {}
    for i in range(50):
        n_req = int(rng.integers(1, 12))
        sizes = rng.integers(1, 60, n_req)
        ties = i % 2 == 0
        scores = [
            (rng.integers(0, 4, n).astype(np.float32) if ties else rng.random(n).astype(np.float32)).astype(np.float64)
            for n in sizes
        ]
        if i % 5 == 2:
            scores[0][:] = 0.0  # no evidence: equal shares
        recent = int(rng.integers(0, 4))
        pinned = []
        for n in sizes:
            p = np.zeros(n, dtype=bool)
            p[0] = True
            p[max(0, n - 1 - recent):] = True
            pinned.append(p)
        must = sum(int(p.sum()) for p in pinned)
        total = int(sizes.sum())
        budget = int(rng.integers(must, total + 1))
        masks = allocate([Request(scores=x, pinned=p) for x, p in zip(scores, pinned, strict=True)], budget, "maxmin")
        cases[f"sizes{i}"], cases[f"scores{i}"] = sizes, np.concatenate(scores)
        cases[f"recent{i}"], cases[f"budget{i}"] = np.int64(recent), np.int64(budget)
        cases[f"mask{i}"] = np.concatenate(masks)
    np.savez_compressed(os.path.join(HERE, "maxmin_cases.npz"), **cases)
    print("maxmin_cases written")


def slot_cases():
    """SlotCompactor.compact (runtime/sglang_compact.py:111-167) on SGLang-style CSR batches: the hand
    cases of the reference's own test (tests/test_sglang_view.py:80-104) and seeded random batches with
    audits, padding rows of a CUDA graph and a policy that is not live. Each case starts from fresh read
    counters."""
    from runtime.sglang_compact import SlotCompactor

    block, width = 16, 20
    rng = np.random.default_rng(43)
    hand = [
        ([5, 16, 17, 100, 33], np.ones((5, width), dtype=bool), 0, None, True),
        ([200, 64, 150, 17, 1], (np.arange(width)[None, :] % 2 == 0).repeat(5, axis=0), 0, None, True),
        ([200, 150, 90], np.zeros((3, width), dtype=bool), 0, np.array([False, True, False]), True),
        ([200, 150, 90], np.zeros((3, width), dtype=bool), 0, None, False),
        ([35], np.zeros((1, width), dtype=bool), 0, None, True),
    ]
    cases = {}
    for i in range(60):
        if i < len(hand):
            lens, keep, padding, audited, active = hand[i]
        else:
            rows = int(rng.integers(1, 12))
            keep = rng.random((rows, width)) < rng.random()
            audited = rng.random(rows) < 0.3 if i % 2 else None
            lens = rng.integers(1, block * width, rows).tolist()
            padding = int(rng.integers(0, 4))
            active = bool(i % 7)
        full = list(lens) + [1] * padding
        indptr = np.array([0, *np.cumsum(full).tolist()], dtype=np.int32)
        slots = rng.permutation(100_000)[: indptr[-1]].astype(np.int64)
        d_indptr = torch.from_numpy(indptr.copy())
        d_slots = torch.from_numpy(np.concatenate([slots, np.full(7, -1, dtype=np.int64)]))
        compactor = SlotCompactor(width, block, torch.device("cpu"))
        audit = None if audited is None else torch.from_numpy(np.asarray(audited).astype(np.uint8))
        new_lens = compactor.compact(d_indptr, d_slots, torch.from_numpy(keep), audit, active, len(lens), len(full),
                                     int(indptr[-1]))
        cases[f"indptr{i}"], cases[f"slots{i}"], cases[f"keep{i}"] = indptr, slots, keep
        cases[f"audit{i}"] = np.zeros(0, dtype=np.uint8) if audited is None else np.asarray(audited).astype(np.uint8)
        cases[f"active{i}"], cases[f"n_real{i}"] = np.int64(active), np.int64(len(lens))
        cases[f"new_indptr{i}"] = d_indptr.numpy().copy()
        total = int(d_indptr[len(full)])
        cases[f"new_slots{i}"] = d_slots.numpy()[:total].copy()
        cases[f"lens{i}"] = new_lens.numpy().copy()
        cases[f"counts{i}"] = compactor.counts.numpy().copy()
    np.savez_compressed(os.path.join(HERE, "slot_cases.npz"), **cases)
    print("slot_cases written")


def _near_ties(rng, n):
    """float64 scores with runs of adjacent doubles, whose shares often round to one value."""
    base = rng.random(n) * 10.0 ** rng.integers(-3, 2)
    runs = rng.integers(1, 5, n)
    out = []
    for x, k in zip(base.tolist(), runs.tolist(), strict=True):
        for _ in range(k):
            out.append(x)
            x = float(np.nextafter(x, np.inf))
    return np.array(out[:n])


def float64_cases():
    """allocate() on float64 scores: adjacent doubles (distinct scores with equal shares), weights that
    merge gains, negative scores, exact float32 values and requests without evidence."""
    rng = np.random.default_rng(53)
    cases = {}
    for i in range(90):
        n_req = int(rng.integers(1, 9))
        sizes = rng.integers(1, 120, n_req)
        kind = i % 3
        scores = []
        for n in sizes:
            if kind == 0:
                x = _near_ties(rng, n)
            elif kind == 1:
                x = rng.dirichlet(np.full(n, 0.3)) if n > 1 else rng.random(1)
            else:
                x = np.where(rng.random(n) < 0.5, _near_ties(rng, n), rng.integers(-1, 3, n).astype(np.float64))
            scores.append(x)
        if i % 11 == 4:
            scores[0][:] = 0.0  # no evidence: equal shares
        objective = ("sum", "uniform", "maxmin")[(i // 3) % 3]
        weights = np.ones(n_req)
        if objective == "sum":
            weights = rng.choice([1.0, 0.3, 1.7, 2.0, 0.0, 1.0 / 3.0], n_req)
        recent = int(rng.integers(0, 5))
        pinned = []
        for n in sizes:
            p = np.zeros(n, dtype=bool)
            p[0] = True
            p[max(0, n - 1 - recent):] = True
            pinned.append(p)
        must = sum(int(p.sum()) for p in pinned)
        total = int(sizes.sum())
        budget = int(rng.integers(must, total + 1))
        requests = [Request(scores=x, weight=float(w), pinned=p) for x, w, p in zip(scores, weights, pinned, strict=True)]
        masks = allocate(requests, budget, objective)
        cases[f"sizes{i}"], cases[f"scores{i}"], cases[f"weights{i}"] = sizes, np.concatenate(scores), weights
        cases[f"recent{i}"], cases[f"budget{i}"] = np.int64(recent), np.int64(budget)
        cases[f"objective{i}"] = objective
        cases[f"mask{i}"] = np.concatenate(masks)
    np.savez_compressed(os.path.join(HERE, "float64_cases.npz"), **cases)
    print("float64_cases written")


class _Box:
    def __init__(self, rows, width):
        self.max_rows, self.row_width = rows, width
        self.record = (0, 0, np.zeros(rows, dtype=np.uint64))

    def audit_record(self):
        return self.record


class _Writer:
    def __init__(self, rows, width):
        self.box = _Box(rows, width)

    def ack_audit(self, done):
        pass


class _Source:
    """Serves a prepared share matrix, NaN for the rows of 0 blocks as TileShareSource.read leaves them."""

    def __init__(self):
        self.fresh = None

    def read(self, live_rows, row_blocks):
        out = self.fresh[:live_rows].copy()
        out[np.asarray(row_blocks)[:live_rows] <= 0] = np.nan
        return out


def controller_cases():
    """Controller._absorb_audit then _forget_departed then _allocate (observe/controller.py:311-451), as a
    tick runs them, over a sequence of audits: requests that come, grow, are audited again (their shares
    blended), have no evidence, are at or below the length cap, and leave. One controller per objective."""
    from observe.controller import Controller, Settings

    rows, width = 20, 64
    rng = np.random.default_rng(61)
    pool = rng.integers(1, 2**63, 40, dtype=np.uint64)
    cases = {"rows": np.int64(rows), "width": np.int64(width)}
    setups = [("sum", 0.4, 4, 0.5, 0), ("uniform", 0.3, 2, 0.25, 8), ("maxmin", 0.5, 3, 0.5, 4), ("sum", 0.25, 0, 0.0, 16)]

    def weight(key):
        return 1.0 + 0.25 * (int(key) % 4) - (0.5 if int(key) % 7 == 0 else 0.0)

    steps = 10
    cases["steps"] = np.int64(steps)
    cases["setups"] = np.array([f"{o},{f},{r},{d},{c}" for o, f, r, d, c in setups])
    controllers = []
    for objective, fraction, recent, decay, cap in setups:
        settings = Settings(budget_fraction=fraction, objective=objective, recent_blocks=recent, share_decay=decay,
                            cap_above_blocks=cap)
        writer, source = _Writer(rows, width), _Source()
        controllers.append((Controller(writer, source, settings, weight=weight if objective == "sum" else None),
                            writer, source))
    present = list(pool[:14])
    length = {int(k): int(rng.integers(1, 60)) for k in pool}
    for step in range(steps):
        # the batch: some requests leave, some arrive, every request grows
        if step:
            for _ in range(int(rng.integers(0, 3))):
                if present:
                    present.pop(int(rng.integers(0, len(present))))
            for k in pool[rng.permutation(len(pool))[: int(rng.integers(0, 4))]]:
                if k not in present and len(present) < rows:
                    present.append(k)
        for k in present:
            length[int(k)] = min(width + 20, length[int(k)] + int(rng.integers(0, 6)))
        keys = np.zeros(rows, dtype=np.uint64)
        lengths = np.zeros(rows, dtype=np.int64)
        slots = rng.permutation(rows)[: len(present)]
        for k, r in zip(present, slots, strict=True):
            keys[r], lengths[r] = k, length[int(k)]
        # the audit: a subset of the rows (by key), in an order of its own
        audit_keys = np.zeros(rows, dtype=np.uint64)
        audited = [k for k in present if rng.random() < 0.7]
        for k, r in zip(audited, rng.permutation(rows)[: len(audited)], strict=True):
            audit_keys[r] = k
        fresh = np.full((rows, width), np.nan)
        for r in range(rows):
            if rng.random() < 0.15:
                continue  # no evidence for this row
            x = rng.dirichlet(np.full(width, 0.4))
            if rng.random() < 0.3:
                x[rng.random(width) < 0.2] = np.nan  # cells without data
            fresh[r] = x
        cases[f"keys{step}"], cases[f"lengths{step}"] = keys, lengths
        cases[f"audit_keys{step}"], cases[f"fresh{step}"] = audit_keys, fresh
        for c, (controller, writer, source) in enumerate(controllers):
            writer.box.record = (step + 1, step + 1, audit_keys)
            source.fresh = fresh
            controller._absorb_audit(keys, lengths)
            controller._forget_departed(keys)
            keep, _release = controller._allocate(keys, lengths)
            cases[f"keep{c}_{step}"] = keep
            ks = sorted(controller.shares)
            cases[f"share_keys{c}_{step}"] = np.array(ks, dtype=np.uint64)
            cases[f"shares{c}_{step}"] = np.array([controller.shares[k] for k in ks]).reshape(len(ks), width)
            cases[f"measured{c}_{step}"] = np.array([controller.measured[k] for k in ks], dtype=np.int64)
    # a controller with a fixed scoring rule instead of measured shares (observe/controller.py:148-160,
    # :411-417): float64 scores no float32 holds, weights, recent pins and a length cap
    def fixed(n):
        return np.sin(np.arange(n) * 0.37) + 1.0

    settings = Settings(budget_fraction=0.35, objective="sum", recent_blocks=2, cap_above_blocks=4)
    fixed_ctl = Controller(_Writer(rows, width), None, settings, weight=weight, scores=fixed)
    for step in range(steps):
        keep, _release = fixed_ctl._allocate(cases[f"keys{step}"], cases[f"lengths{step}"])
        cases[f"fixed_keep{step}"] = keep
    np.savez_compressed(os.path.join(HERE, "controller_cases.npz"), **cases)
    print("controller_cases written")


def pinned_cases():
    """allocate() with Request.pinned marking any blocks (observe/allocation.py:37-44): middle blocks,
    none at all, every block, the first or last left open; all three objectives, weights under `sum`,
    ties across requests and requests without evidence."""
    rng = np.random.default_rng(67)
    cases = {}
    for i in range(120):
        n_req = int(rng.integers(1, 8))
        sizes = rng.integers(1, 90, n_req)
        kind = i % 4
        scores, pinned = [], []
        for n in sizes:
            if kind == 0:
                x = rng.integers(0, 4, n).astype(np.float64)  # many ties, within and across requests
            elif kind == 1:
                x = rng.dirichlet(np.full(n, 0.3)) if n > 1 else rng.random(1)
            elif kind == 2:
                x = _near_ties(rng, n)
            else:
                x = np.where(rng.random(n) < 0.3, 0.0, rng.random(n))
            scores.append(x)
            style = int(rng.integers(0, 5))
            if style == 0:
                p = np.zeros(n, dtype=bool)  # no pins
            elif style == 1:
                p = rng.random(n) < 0.3  # anywhere
            elif style == 2:
                p = rng.random(n) < 0.8  # most
            elif style == 3:
                p = np.ones(n, dtype=bool)  # every block
            else:
                p = np.zeros(n, dtype=bool)
                p[n // 2] = True  # one middle block
            pinned.append(p)
        if i % 13 == 5:
            scores[0][:] = 0.0  # no evidence: equal shares
        objective = ("sum", "uniform", "maxmin")[i % 3]
        weights = np.ones(n_req)
        if objective == "sum" and i % 2:
            weights = rng.choice([1.0, 0.5, 2.0, 0.0, 1.0 / 3.0], n_req)
        must = sum(int(p.sum()) for p in pinned)
        total = int(sizes.sum())
        budget = int(rng.integers(must, total + 1))
        requests = [Request(scores=x, weight=float(w), pinned=p) for x, w, p in zip(scores, weights, pinned, strict=True)]
        masks = allocate(requests, budget, objective)
        cases[f"sizes{i}"], cases[f"scores{i}"], cases[f"weights{i}"] = sizes, np.concatenate(scores), weights
        cases[f"pinned{i}"], cases[f"budget{i}"] = np.concatenate(pinned), np.int64(budget)
        cases[f"objective{i}"] = objective
        cases[f"mask{i}"] = np.concatenate(masks)
    np.savez_compressed(os.path.join(HERE, "pinned_cases.npz"), **cases)
    print("pinned_cases written")


def all_cases():
    audit_case("audit_cfg1_fp16", 0, rows=4, q_heads=8, kv_heads=2, layers=1, len_lo=100, len_hi=600, pool=256, dtype="fp16")
    audit_case("audit_layers_fp16", 1, rows=6, q_heads=8, kv_heads=2, layers=3, len_lo=1, len_hi=300, pool=256,
               dtype="fp16", select=[1, 1, 0, 1, 1, 1], flags=[1, 0, 1])
    audit_case("audit_g8_bf16", 2, rows=5, q_heads=16, kv_heads=2, layers=2, len_lo=5, len_hi=200, pool=128, dtype="bf16")
    shares_cases()
    allocation_cases()
    view_cases()
    slot_cases()
    maxmin_cases()
    float64_cases()
    controller_cases()
    pinned_cases()


if __name__ == "__main__":
    # `python make_golden.py` writes every fixture; `python make_golden.py slot_cases ...` only those named
    chosen = sys.argv[1:]
    if not chosen:
        all_cases()
    for name in chosen:
        globals()[name]()
