// The audit step on the device: a streaming kernel that records every (layer, row, tile) cell, and a
// share kernel that turns the cells into the exact per-block attention share.
//
// Streaming. An item is one (layer, KV head, row, chunk of EKV_AUDIT_CHUNK_TILES tiles); the items of
// a launch are numbered layer-major and every warp of a persistent grid (SMs x resident CTAs) works
// through items worker, worker + workers, ... on its own, with a ring of STAGES shared-memory stages
// of one tile each kept in flight across item boundaries. The key cache of a layer is a 4-D tensor
// map (head dim, KV head, token of the block, block); for each block of a tile two lanes ask the TMA
// engine for the block's 16 key rows of the audited head, one 64-dim half each (a 128-byte-swizzled
// box, L2 evict-first), and lane 0 arms the stage's mbarrier with the byte count. Two copies per
// block instead of one per key row keep the TMA issue cost off each warp's critical path; the swizzle
// lets ldmatrix read the rows without bank conflicts. Nothing on a tile's critical path reads global
// memory: the rows' lengths and query tokens sit in shared memory, the block ids of the next item and
// the query fragments of the next item are prefetched into registers one item ahead.
//
// Scores. One m16n8k16 mma per (16 tokens, 16 dims): A = 16 key rows by ldmatrix, B = the G query
// rows of the KV head (registers, padded to 8 or 16 columns), fp32 accumulation. Tokens sit on the
// C fragment's rows and query rows on its columns, so the tile max and sum are three xor-shuffles
// per column: tile_lse_kernel's computation (runtime/audit_kernel.py:70-96), stored as at :97-109.
//
// Shares. After the record kernel, one share kernel reads the cells back from L2, a CTA per (row, group
// of layers): u = m + log(l) - log(tile_blocks) per tile (observe/tile_shares.py:172-173), each query
// row's log total, and every tile's share from the same cells still in registers; the CTA that finishes
// a row last adds the groups and gives the partial tail tile's weight back to its blocks (:82-103).
// Every sum has a fixed order, so the output is deterministic.
#include <cooperative_groups.h>
#include <type_traits>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "ekv_common.cuh"

namespace ekv {

namespace cg = cooperative_groups;

// Warps per CTA of the record kernel and ring stages per warp (tiles of 32 tokens; tiles of 16 hold
// twice as many, tiles of 64 half as many). Overridable at build time for tuning sweeps.
#ifndef EKV_AUDIT_WARPS
#define EKV_AUDIT_WARPS 4
#endif
#ifndef EKV_AUDIT_STAGES32
#define EKV_AUDIT_STAGES32 2
#endif
constexpr int kWarps = EKV_AUDIT_WARPS;
constexpr int kMaxQ = 128;
constexpr int kMaxRows = 2048;
constexpr int kMaxLayers = 1024;
constexpr int kChunkTiles = EKV_AUDIT_CHUNK_TILES;
constexpr int kMinCtas = 12 / kWarps > 0 ? 12 / kWarps : 1;  // registers for 12 warps per SM
constexpr int kItemQueue = 16;  // items a warp has taken but not yet consumed (at most STAGES + 2)

struct AuditParams {
  // the key cache of a single-layer launch as a tensor map (encoded on the host), or one map per
  // layer in the workspace (written by kmap_kernel from k_layers)
  CUtensorMap kmap0;
  const CUtensorMap* kmaps;
  // per-layer sources: device arrays of addresses, or one address for a single layer
  const uint64_t* q_layers;
  const uint64_t* k_layers;
  const void* q;
  const void* k;
  int layer0, n_layers;
  int group, rotate;  // KV head of layer L: rotate ? (group + L) % kv_heads : group
  int q_stash;        // queries hold only the audited heads: query head = head * G + g
  const int32_t* table;
  const int32_t* lens;
  const int32_t* qrow;
  const uint8_t* select;
  const uint32_t* flag;
  float* lse;
  float scale;
  int64_t q_s0, q_s1, k_s0, k_s1, k_s2, table_s0;
  int layers, rows, width;
  int G, heads, Q;
  int block_size, tile_blocks;
  int kv_heads;
  int64_t pool_blocks, q_tokens;
  // the share
  float* share_out;
  int32_t* contrib_out;
  int aggregate;
  uint32_t* item_counter;   // items handed out beyond each warp's first (zeroed by kmap_kernel); NULL: static order
  // the share pass (set on the host): query rows per load (4 or 1), units per layer (Q / V), layers per group,
  // groups, tiles of the width each CTA of a row's cluster writes, log2 of tile_blocks
  int share_V, share_QG, share_Lg, share_groups, share_slice, tb_shift;
  uint32_t* status;
};

// A stage holds a tile of TT key rows as two [TT][128 B] halves (dims 0-63, 64-127) in the TMA
// engine's 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8). Every box (one
// block's rows of one half) starts on a 1024-byte boundary, so block_size must be a multiple of 8.
template <int D>
struct Layout {
  static_assert(D == 128, "two 128-byte halves per key row");
  static constexpr int kHalfRow = 128;
};

template <int TT>
struct Ring {
  static constexpr int kStages = TT <= 16 ? 2 * EKV_AUDIT_STAGES32 : (TT <= 32 ? EKV_AUDIT_STAGES32 : (EKV_AUDIT_STAGES32 + 1) / 2 > 2 ? (EKV_AUDIT_STAGES32 + 1) / 2 : 2);
};

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Makes a tensor map written in global memory by an earlier kernel visible to this thread's copies.
__device__ __forceinline__ void tensormap_acquire(const CUtensorMap* map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(__cvta_generic_to_global(map))
               : "memory");
}

// One tiled tensor copy global -> shared (4-D coordinates, innermost first), completing on `bar`.
__device__ __forceinline__ void tensor_copy_g2s(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                int c3, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Row r of the step: its length (tokens, clamped to the table), blocks, tiles and chunks; no chunks
// when it records nothing (not selected, empty, or a query token outside the batch).
struct RowInfo {
  int n_blocks, n_tiles, n_chunks, len;
};

__device__ __forceinline__ RowInfo row_info(const AuditParams& p, int r, bool report) {
  RowInfo ri{0, 0, 0, 0};
  if (!p.select[r]) return ri;
  int len = p.lens[r];
  if (len <= 0) return ri;
  int n = (len + p.block_size - 1) / p.block_size;
  if (n > p.width) {
    if (report) set_status(p.status, EKV_STATUS_LEN_OVER_WIDTH);
    n = p.width;
    len = p.width * p.block_size;
  }
  const int token = p.qrow[r];
  if (token < 0 || (int64_t)token >= p.q_tokens) {
    if (report) set_status(p.status, EKV_STATUS_BAD_QROW);
    return ri;
  }
  ri.len = len;
  ri.n_blocks = n;
  ri.n_tiles = (n + p.tile_blocks - 1) / p.tile_blocks;
  ri.n_chunks = (ri.n_tiles + kChunkTiles - 1) / kChunkTiles;
  return ri;
}

__device__ __forceinline__ int kv_head_of(const AuditParams& p, int layer, int h) {
  return (p.rotate ? (p.group + layer) % p.kv_heads : p.group) + h;
}

// A warp's position in its sequence of tiles: the item and the tile inside it.
struct Cursor {
  long long item;  // index into the launch's items; >= the total when done
  int layer, head, row, t0, t, t_end;
};

template <int TT, int NT, int D, typename T>
__global__ void __launch_bounds__(kWarps * 32, kMinCtas) record_kernel(const __grid_constant__ AuditParams p) {
  using Lay = Layout<D>;
  constexpr int STAGES = Ring<TT>::kStages;
  constexpr int HALF = TT * Lay::kHalfRow;  // one half of a stage
  constexpr int STAGE = 2 * HALF;
  constexpr int MT = TT / 16;
  constexpr int KS = D / 16;
  // hold a whole tile's A fragments in registers (MT * KS * 4 of them) when that keeps 3 CTAs per SM
  constexpr bool kEarlyRelease = MT * NT <= 2;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // swizzled boxes: 1024-aligned
  uint8_t* rings = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * STAGES * STAGE);
  uint32_t* vmasks = reinterpret_cast<uint32_t*>(bars + kWarps * STAGES);  // [warp][stage]: copied blocks
  int* prefix = reinterpret_cast<int*>(vmasks + kWarps * STAGES);          // [rows + 1]
  int* s_blocks = prefix + p.rows + 1;                                     // [rows]
  int* s_len = s_blocks + p.rows;                                          // [rows]
  int* s_tok = s_len + p.rows;                                             // [rows]
  __shared__ int s_scan[kWarps + 1];
  __shared__ long long s_queue[kWarps][kItemQueue];  // each warp's items in the order it took them

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The share kernel may take the SMs this grid leaves as it ends (it waits for the cells itself). The
  // flag and the rows' lengths, selection and query rows are the step's inputs, written before its chain
  // of launches, so the rows are set up while the launches before this one end.
  chain_release();
  if (*p.flag == 0) return;  // the statistic is off: nothing is recorded (:64)

  // ---- the rows of the step and the items: chunks per row, prefix-summed in shared memory --------
  {
    int carry = 0;
    for (int base = 0; base < p.rows; base += kWarps * 32) {
      const int r = base + threadIdx.x;
      RowInfo ri{0, 0, 0, 0};
      if (r < p.rows) {
        ri = row_info(p, r, blockIdx.x == 0);
        s_blocks[r] = ri.n_blocks;
        s_len[r] = ri.len;
        s_tok[r] = ri.n_chunks ? p.qrow[r] : 0;
      }
      int total = 0;
      const int before = block_exclusive_scan<kWarps * 32>(ri.n_chunks, s_scan, &total);
      if (r < p.rows) prefix[r] = carry + before;
      carry += total;
    }
    if (threadIdx.x == 0) prefix[p.rows] = carry;
    __syncthreads();
  }
  chain_wait();  // the query stash, the tensor maps and the item counter come from the launches before
  const int chunks_per_lh = prefix[p.rows];
  const long long total_items = (long long)chunks_per_lh * p.heads * p.n_layers;
  const long long workers = (long long)gridDim.x * kWarps;
  const long long worker = (long long)blockIdx.x * kWarps + warp;
  uint32_t* const ctr = p.item_counter;
  if (worker >= total_items) return;

  // Items: a warp's first is its own index; after that it takes the next free one from the counter
  // (SMs do not stream at the same rate: with a static share the fast ones sit idle for the last
  // third of a step), or with no counter every workers-th. The issue side takes them; the consume
  // side follows the same sequence through s_queue.
  long long n_taken = 0;
  bool drained = false;
  auto take = [&]() -> long long {
    long long item = total_items;
    if (!drained) {
      if (n_taken == 0) {
        item = worker;
      } else if (ctr != nullptr) {
        uint32_t v = 0;
        if (lane == 0) v = atomicAdd(ctr, 1u);
        item = workers + (long long)__shfl_sync(kFullMask, v, 0);
      } else {
        item = worker + n_taken * workers;
      }
      if (item >= total_items) {
        item = total_items;
        drained = true;
      }
    }
    if (lane == 0) s_queue[warp][n_taken % kItemQueue] = item;
    ++n_taken;
    return item;
  };

  auto decode = [&](long long item, Cursor& c) {
    c.item = item;
    if (item >= total_items) return;
    const long long lh = item / chunks_per_lh;
    const int idx = (int)(item - lh * chunks_per_lh);
    int lo = 0, hi = p.rows;  // the last row with prefix[row] <= idx
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix[mid] <= idx) lo = mid; else hi = mid;
    }
    c.row = lo;
    c.layer = p.layer0 + (int)(lh / p.heads);
    c.head = (int)(lh % p.heads);
    const int n_tiles = (s_blocks[lo] + p.tile_blocks - 1) / p.tile_blocks;
    c.t0 = c.t = (idx - prefix[lo]) * kChunkTiles;
    c.t_end = min(c.t + kChunkTiles, n_tiles);
  };

  // the block ids of an item: lane i holds blocks t0 * tile_blocks + i and + 32 + i
  auto load_ids = [&](const Cursor& c, int32_t& lo_id, int32_t& hi_id) {
    lo_id = hi_id = -1;
    if (c.item >= total_items) return;
    const int32_t* trow = p.table + (int64_t)c.row * p.table_s0;
    const int b0 = c.t0 * p.tile_blocks;
    const int nb = min(s_blocks[c.row], c.t_end * p.tile_blocks) - b0;
    if (lane < nb) lo_id = __ldg(trow + b0 + lane);
    if (lane + 32 < nb) hi_id = __ldg(trow + b0 + lane + 32);
  };

  // the query rows of an item's (layer, row, head), as mma B fragments (k16 x n8, column = query row)
  auto load_q = [&](const Cursor& c, uint32_t (&bq)[NT][KS][2]) {
    if (c.item >= total_items) return;
    const void* qsrc = p.q_layers ? reinterpret_cast<const void*>(p.q_layers[c.layer]) : p.q;
    const bool q_ok = (reinterpret_cast<uintptr_t>(qsrc) & 3) == 0;
    const T* qtok = static_cast<const T*>(qsrc) + (int64_t)s_tok[c.row] * p.q_s0;
    const int qhead = p.q_stash ? c.head : kv_head_of(p, c.layer, c.head);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int g = nt * 8 + (lane >> 2);
      const bool ok = q_ok && g < p.G;
      const T* qh = qtok + (int64_t)(qhead * p.G + (ok ? g : 0)) * p.q_s1;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const int d = k * 16 + 2 * (lane & 3);
        bq[nt][k][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qh + d)) : 0u;
        bq[nt][k][1] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qh + d + 8)) : 0u;
      }
    }
  };

  uint8_t* my_ring = rings + warp * STAGES * STAGE;
  uint64_t* my_bars = bars + warp * STAGES;
  uint32_t* my_masks = vmasks + warp * STAGES;
  const int bs_shift = __ffs(p.block_size) - 1;  // block_size is a power of two
  int fenced_layer = -1;                         // the layer whose tensor map this warp has acquired
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&my_bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const uint64_t policy = l2_evict_first_policy();

  // the issue side: cursor `in`, the ids of its item and of the item after it. The next item is
  // taken when `in` reaches its last tile: late enough that no warp holds an item it will not start
  // soon (the end of a launch stays even), early enough for its block ids to land.
  Cursor in{}, in_next{};
  int32_t ids_lo, ids_hi, nids_lo = -1, nids_hi = -1;
  bool next_taken = false;
  auto take_next_if_due = [&]() {
    if (!next_taken && in.item < total_items && in.t >= in.t_end - 1) {
      decode(take(), in_next);
      load_ids(in_next, nids_lo, nids_hi);
      next_taken = true;
    }
  };
  decode(take(), in);
  load_ids(in, ids_lo, ids_hi);
  take_next_if_due();

  // Issue the tensor copies of the tile at `in` into stage s, then step `in` forward: lanes 2j and
  // 2j + 1 copy the two halves of block j of the tile.
  auto issue_and_advance = [&](int s) {
    const CUtensorMap* map = &p.kmap0;
    bool aligned = true;
    if (p.kmaps != nullptr) {
      map = p.kmaps + in.layer;
      aligned = (p.k_layers[in.layer] & 15) == 0;
      if (in.layer != fenced_layer) {
        tensormap_acquire(map);
        fenced_layer = in.layer;
      }
    }
    const int TB = p.tile_blocks;
    const int n_blocks = s_blocks[in.row];
    const int tl = in.t - in.t0;
    const int jb = (lane >> 1) < TB ? (lane >> 1) : 0;  // this lane's block of the tile
    const int bi = tl * TB + jb;                        // ... of the item
    const int32_t lo_id = __shfl_sync(kFullMask, ids_lo, bi & 31);
    const int32_t hi_id = __shfl_sync(kFullMask, ids_hi, bi & 31);
    const int32_t id = bi < 32 ? lo_id : hi_id;
    bool ok = false;
    if (lane < 2 * TB && in.t * TB + jb < n_blocks) {
      ok = aligned && id >= 0 && (int64_t)id < p.pool_blocks;
      if (!ok && (lane & 1) == 0) set_status(p.status, EKV_STATUS_BAD_BLOCK_ID);
    }
    const uint32_t pairs = __ballot_sync(kFullMask, ok);
    uint32_t bmask = 0;  // bit j: block j of the tile is copied
#pragma unroll
    for (int j = 0; j < TT / 8; ++j) bmask |= ((pairs >> (2 * j)) & 1u) << j;
    if (lane == 0) {
      my_masks[s] = bmask;
      if (bmask) {
        mbar_arrive_expect_tx(&my_bars[s], (uint32_t)__popc(bmask) * (uint32_t)p.block_size * 2u * Lay::kHalfRow);
      } else {
        mbar_arrive(&my_bars[s]);
      }
    }
    __syncwarp();
    if (ok) {
      const int half = lane & 1;
      uint8_t* dst = my_ring + s * STAGE + half * HALF + (jb << bs_shift) * Lay::kHalfRow;
      tensor_copy_g2s(dst, map, 64 * half, kv_head_of(p, in.layer, in.head), 0, id, &my_bars[s], policy);
    }
    ++in.t;
    take_next_if_due();
    if (in.t >= in.t_end) {  // the next item: its ids were prefetched
      in = in_next;
      ids_lo = nids_lo;
      ids_hi = nids_hi;
      next_taken = false;
      take_next_if_due();
    }
  };

  long long issued = 0;
  for (int s = 0; s < STAGES && in.item < total_items; ++s) {
    issue_and_advance(s);
    ++issued;
  }

  // the consume side: cursor `out`, the query fragments of its item and of the next one
  Cursor out{};
  long long n_used = 0;  // the consume side's position in s_queue
  __syncwarp();
  decode(s_queue[warp][0], out);
  uint32_t bq[NT][KS][2], bqn[NT][KS][2];
  load_q(out, bqn);
  const size_t plane = (size_t)p.layers * p.rows * p.width * p.Q;
  bool timed_out = false;
  long long consumed = 0, unwaited = 0;  // copies from tile `unwaited` on were never waited for

  while (out.item < total_items) {
    const int s = (int)(consumed % STAGES);
    const uint32_t parity = (uint32_t)((consumed / STAGES) & 1);
    if (out.t == out.t0) {  // an item starts: its fragments were prefetched
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int k = 0; k < KS; ++k) bq[nt][k][0] = bqn[nt][k][0], bq[nt][k][1] = bqn[nt][k][1];
    }
    if (out.t == out.t_end - 1) {  // its last tile: the issue side has taken the next item; prefetch
      Cursor nxt{};
      __syncwarp();
      decode(s_queue[warp][(n_used + 1) % kItemQueue], nxt);
      load_q(nxt, bqn);
    }
    if (!timed_out && !mbar_wait_bounded(&my_bars[s], parity, p.status)) {
      timed_out = true;
      unwaited = consumed;
    }
    bool released = false;
    if (!timed_out) {
      const uint8_t* stage = my_ring + s * STAGE;
      float c[MT][NT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) c[mt][nt][e] = 0.f;
      // lane l reads row (l % 8) + 8 * ((l / 8) % 2) of the m-tile, 16-byte chunk 2k + l / 16 of the
      // row: in the swizzled half k / 4 that chunk sits at ((2k) % 8) ^ (l / 16) ^ (l % 8)
      const uint32_t a_base = smem_u32(stage) + ((lane & 7) + ((lane >> 3) & 1) * 8) * Lay::kHalfRow;
      const uint32_t swz = (uint32_t)((lane >> 4) ^ (lane & 7));
      const uint32_t vm = my_masks[s];
      if constexpr (kEarlyRelease) {
        // the whole tile into registers, the stage back to the TMA engine, then the math: both of the
        // warp's stages stay in flight while it computes
        uint32_t a[MT][KS][4];
#pragma unroll
        for (int k = 0; k < KS; ++k)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            ldmatrix_x4(a[mt][k], a_base + (k >> 2) * HALF + mt * 16 * Lay::kHalfRow + ((((2 * k) & 7) ^ swz) << 4));
        __syncwarp();
        fence_proxy_async();
        ++consumed;
        if (in.item < total_items) {
          issue_and_advance((int)(issued % STAGES));
          ++issued;
        }
        released = true;
#pragma unroll
        for (int k = 0; k < KS; ++k)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Mma<T>::run(c[mt][nt], a[mt][k], bq[nt][k]);
      } else {
#pragma unroll
        for (int k = 0; k < KS; ++k) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            uint32_t a[4];
            ldmatrix_x4(a, a_base + (k >> 2) * HALF + mt * 16 * Lay::kHalfRow + ((((2 * k) & 7) ^ swz) << 4));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Mma<T>::run(c[mt][nt], a, bq[nt][k]);
          }
        }
      }
      const int first = out.t * TT;
      const int len = s_len[out.row];
      float mx[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mx[nt][0] = mx[nt][1] = -INFINITY;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int tok = mt * 16 + (lane >> 2) + 8 * h;
          const bool ok = first + tok < len && ((vm >> (tok >> bs_shift)) & 1u);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float sc = ok ? c[mt][nt][2 * h + e] * p.scale : -INFINITY;
              c[mt][nt][2 * h + e] = sc;
              mx[nt][e] = fmaxf(mx[nt][e], sc);
            }
        }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
          for (int off = 4; off < 32; off <<= 1)
            mx[nt][e] = fmaxf(mx[nt][e], __shfl_xor_sync(kFullMask, mx[nt][e], off));
      float sm[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sm[nt][0] = sm[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) sm[nt][e] += __expf(c[mt][nt][2 * h + e] - mx[nt][e]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) sm[nt][e] += __shfl_xor_sync(kFullMask, sm[nt][e], off);
      // every block cell of the tile inside the row gets the tile's (m, l); lane / 4 picks the block
      const int bi = lane >> 2;
      const int b = out.t * p.tile_blocks + bi;
      if (bi < p.tile_blocks && b < s_blocks[out.row]) {
        float* cm = p.lse + (((size_t)out.layer * p.rows + out.row) * p.width + b) * p.Q + out.head * p.G;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int g = nt * 8 + 2 * (lane & 3) + e;
            if (g < p.G) {
              cm[g] = mx[nt][e];
              cm[g + plane] = sm[nt][e];
            }
          }
      }
    }
    if (!released) {  // the stage is consumed: refill it with the tile STAGES ahead
      __syncwarp();
      fence_proxy_async();
      ++consumed;
      if (in.item < total_items && !timed_out) {
        issue_and_advance((int)(issued % STAGES));
        ++issued;
      }
    }
    if (++out.t >= out.t_end) {
      ++n_used;
      __syncwarp();
      decode(s_queue[warp][n_used % kItemQueue], out);
    }
  }
  if (timed_out) {
    // let copies still in flight land before the shared memory is released
    for (long long i = unwaited; i < issued; ++i)
      mbar_wait_bounded(&my_bars[i % STAGES], (uint32_t)((i / STAGES) & 1), p.status);
  }
}

// ---- the share pass: a cluster of CTAs per row, each CTA some groups of layers ---------------------------
//
// A unit is (layer, V query rows): V = 4 when the cells allow 16-byte loads, else 1. A group is Lg layers of
// one row, Lg * Q / V units, about four, spread over the CTA's warps; the row's C CTAs (a cluster) take groups
// rank, rank + C, ... For a unit a warp reads the tiles' cells (lane l: tiles l, l + 32, ...), takes each query
// row's largest m among its cells with data (l > 0, m > -inf), each cell's weight w = l exp(m - M), their sum
// S (xor-shuffles: the same order on every launch), and gives every tile its share over the unit's query rows
// with data, w / S = exp(u_b) / sum_b' exp(u_b') with u = m + log(l) - log(tile_blocks) (summed, or maxed for
// the max aggregate). A row of at most kShareBatch tiles keeps a unit's cells in registers throughout and a
// warp adds all its units' shares before the CTA adds its warps; a longer row is read twice per unit, a batch
// of tiles at a time (a running maximum and a rescaled sum first, then the shares). The C CTAs of the row then read each other's per-tile sums (distributed shared
// memory, in rank order) and each writes a slice of the row: each block of tile t gets the tile's sum / n_t
// (n_t the tile's blocks in the row: a partial last tile's blocks share its whole weight, the reference's
// regain) divided by the contributors, the (layer, query row) pairs with data (mean), or the row divided by its
// total (max). A row that records nothing, or has no contributor, is NaN; blocks past the row are 0.
constexpr int kShareMaxWarps = 16;
constexpr int kShareRegTiles = 8;  // tiles a lane holds at once
constexpr int kShareBatch = 32 * kShareRegTiles;
constexpr int kShareMaxCluster = 8;   // the portable cluster size
constexpr int kShareMaxTiles = 32768;  // a row's partials in shared memory (128 KB)

struct ShareShape {
  int V, QG, Lg, groups, warps, cluster;  // query rows per load, units per layer, layers per group, groups,
                                          // warps per CTA, CTAs per row
};

// lse_aligned: the cell table starts on a 16-byte boundary.
inline ShareShape share_shape(int Q, int n_layers, bool lse_aligned) {
  ShareShape s{};
  s.V = (Q & 3) == 0 && lse_aligned ? 4 : 1;
  s.QG = Q / s.V;
  s.Lg = s.QG >= 4 ? 1 : 4 / s.QG;  // about four units a group, one per warp, or more warps for wide cells
  if (s.Lg > n_layers) s.Lg = n_layers;
  s.groups = (n_layers + s.Lg - 1) / s.Lg;
  const int units = s.Lg * s.QG;
  s.warps = units < kShareMaxWarps ? units : kShareMaxWarps;
  s.cluster = s.groups < kShareMaxCluster ? s.groups : kShareMaxCluster;
  return s;
}

// The cells of the warp's tiles t0 + lane + 32 i, i < SL, V query rows each. A cell without data (l = 0,
// m = -inf or NaN) is marked m = -inf, l = 0; so is a tile past the row.
template <int V, int SL>
__device__ __forceinline__ void load_unit_tiles(const float* cm, const float* cl, int tile_stride, int t0, int n_tiles,
                                                int lane, float (&m)[SL][V], float (&l)[SL][V]) {
#pragma unroll
  for (int i = 0; i < SL; ++i) {
    const int t = t0 + lane + 32 * i;
    const bool ok = t < n_tiles;
    const size_t at = (size_t)(ok ? t : 0) * tile_stride;
    if constexpr (V == 4) {
      const float4 a = ok ? __ldcg(reinterpret_cast<const float4*>(cm + at)) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float4 b = ok ? __ldcg(reinterpret_cast<const float4*>(cl + at)) : make_float4(0.f, 0.f, 0.f, 0.f);
      m[i][0] = a.x, m[i][1] = a.y, m[i][2] = a.z, m[i][3] = a.w;
      l[i][0] = b.x, l[i][1] = b.y, l[i][2] = b.z, l[i][3] = b.w;
    } else {
      m[i][0] = ok ? __ldcg(cm + at) : -INFINITY;
      l[i][0] = ok ? __ldcg(cl + at) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const bool data = l[i][k] > 0.f && m[i][k] > -INFINITY;
      m[i][k] = data ? m[i][k] : -INFINITY;
      l[i][k] = data ? l[i][k] : 0.f;
    }
  }
}

// The largest m over the lane's tiles.
template <int V, int SL>
__device__ __forceinline__ void unit_max(float (&M)[V], const float (&m)[SL][V]) {
#pragma unroll
  for (int i = 0; i < SL; ++i)
#pragma unroll
    for (int k = 0; k < V; ++k) M[k] = fmaxf(M[k], m[i][k]);
}

// Each cell's weight w = l exp(m - M) (0 without data), written over l, and its sum into S.
template <int V, int SL>
__device__ __forceinline__ void unit_weights(float (&S)[V], const float (&M)[V], const float (&m)[SL][V],
                                             float (&l)[SL][V]) {
#pragma unroll
  for (int i = 0; i < SL; ++i)
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float w = m[i][k] > -INFINITY ? l[i][k] * __expf(m[i][k] - M[k]) : 0.f;
      l[i][k] = w;
      S[k] += w;
    }
}

template <int V>
__device__ __forceinline__ void lanes_max(float (&x)[V]) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1)
#pragma unroll
    for (int k = 0; k < V; ++k) x[k] = fmaxf(x[k], __shfl_xor_sync(kFullMask, x[k], off));
}

template <int V>
__device__ __forceinline__ void lanes_sum(float (&x)[V]) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1)
#pragma unroll
    for (int k = 0; k < V; ++k) x[k] += __shfl_xor_sync(kFullMask, x[k], off);
}

// acc[i] gets tile i's share over the query rows, w * inv (summed, or maxed).
template <int V, int SL>
__device__ __forceinline__ void add_unit_shares(float (&acc)[kShareRegTiles], const float (&w)[SL][V],
                                                const float (&inv)[V], bool agg_max) {
#pragma unroll
  for (int i = 0; i < SL; ++i)
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float sh = w[i][k] * inv[k];
      acc[i] = agg_max ? fmaxf(acc[i], sh) : acc[i] + sh;
    }
}

// The reciprocal of each query row's total weight (0 without data); the query rows with data.
template <int V>
__device__ __forceinline__ int unit_inverse(float (&inv)[V], const float (&S)[V]) {
  int cnt = 0;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    inv[k] = S[k] > 0.f ? __frcp_rn(S[k]) : 0.f;
    cnt += S[k] > 0.f;
  }
  return cnt;
}

// A unit of a row of at most 32 * SL tiles, every cell in registers: the maximum, the weights and their sum,
// the shares added into acc; the query rows with data.
template <int V, int SL>
__device__ __forceinline__ int unit_in_registers(float (&acc)[kShareRegTiles], const float* cm, const float* cl,
                                                 int tile_stride, int n_tiles, int lane, bool agg_max) {
  float m[SL][V], l[SL][V], M[V], S[V], inv[V];
  load_unit_tiles<V, SL>(cm, cl, tile_stride, 0, n_tiles, lane, m, l);
#pragma unroll
  for (int k = 0; k < V; ++k) M[k] = -INFINITY, S[k] = 0.f;
  unit_max<V, SL>(M, m);
  lanes_max<V>(M);
  unit_weights<V, SL>(S, M, m, l);
  lanes_sum<V>(S);
  const int cnt = unit_inverse<V>(inv, S);
  add_unit_shares<V, SL>(acc, l, inv, agg_max);
  return cnt;
}

template <int V>
__global__ void __launch_bounds__(kShareMaxWarps * 32) share_kernel(const AuditParams p) {
  extern __shared__ float s_part[];  // [tiles of the width]: this CTA's groups' partial per tile
  __shared__ float s_acc[kShareMaxWarps][kShareBatch];
  __shared__ float2 s_norm[kShareMaxWarps][8];  // (M, 1 / S) of a warp's units' query rows (the long-row path)
  __shared__ int s_cnt[kShareMaxWarps];
  __shared__ float s_red[kShareMaxWarps];
  __shared__ int s_count;    // this CTA's (layer, query row) pairs with data
  __shared__ float s_total;  // (max) the total of this CTA's slice of the row
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank(), C = (int)cluster.num_blocks();
  const int r = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
  chain_release();
  // the row's length and selection are the step's inputs, not the record kernel's: read while it ends
  const RowInfo ri = row_info(p, r, false);
  chain_wait();  // the record kernel's cells
  if (*p.flag == 0) return;  // nothing was recorded this step (the same for every CTA)
  float* out = p.share_out + (size_t)r * p.width;
  if (ri.n_chunks == 0) {  // the row records nothing: NaN (the same for the whole cluster)
    for (int b = rank * blockDim.x + tid; b < p.width; b += C * blockDim.x) out[b] = NAN;
    if (rank == 0 && tid == 0) p.contrib_out[r] = 0;
    return;
  }
  const int Q = p.Q, QG = p.share_QG, TB = p.tile_blocks;
  const int n = ri.n_blocks, n_tiles = ri.n_tiles;
  const int groups = p.share_groups;
  const size_t plane = (size_t)p.layers * p.rows * p.width * Q;
  const int tile_stride = TB * Q;  // floats from one tile's cell (its first block's) to the next tile's
  const bool agg_max = p.aggregate == EKV_AGG_MAX;
  int cnt = 0;  // this warp's (layer, query row) pairs with data
  // Unit u of a group is its layer u / QG and query rows (u % QG) * V ...; a warp's units are u = warp,
  // warp + warps, ..., walked as (layer, query-row unit) pairs without a division.
  struct Unit {
    int l, q;
  };
  const Unit u0{warp / QG, warp % QG}, du{warps / QG, warps % QG};
  auto step = [&](Unit u) {
    u.l += du.l, u.q += du.q;
    if (u.q >= QG) u.q -= QG, ++u.l;
    return u;
  };
  auto group_layers = [&](int g) { return min(p.share_Lg, p.n_layers - g * p.share_Lg); };
  auto unit_cells = [&](int g, Unit u, const float*& cm, const float*& cl) {
    const size_t lr = (size_t)(p.layer0 + g * p.share_Lg + u.l) * p.rows + r;
    cm = p.lse + lr * p.width * Q + u.q * V;
    cl = cm + plane;
  };
  float acc[kShareRegTiles];
  if (n_tiles <= kShareBatch) {
    // Every tile of a unit in registers: its maximum, the weights and their sum, the shares. A warp takes its
    // units of every group of the CTA in turn (groups rank, rank + C, ...; in each, units warp, warp + warps,
    // ...) with no barrier between them, adding into one set of per-tile sums; the CTA adds its warps once.
    // With at most two slots a lane the next unit's cells are loaded while the current one is computed.
#pragma unroll
    for (int i = 0; i < kShareRegTiles; ++i) acc[i] = 0.f;
    struct Cursor {
      int g;
      Unit u;
    };
    auto settle = [&](Cursor c) {  // the first unit at or after c
      while (c.g < groups && c.u.l >= group_layers(c.g)) c.g += C, c.u = u0;
      return c;
    };
    auto walk = [&](auto slots_tag) {
      constexpr int SL = decltype(slots_tag)::value;
      auto load = [&](Cursor c, float (&m)[SL][V], float (&l)[SL][V]) {
        const float *cm, *cl;
        unit_cells(c.g, c.u, cm, cl);
        load_unit_tiles<V, SL>(cm, cl, tile_stride, 0, n_tiles, lane, m, l);
      };
      auto compute = [&](float (&m)[SL][V], float (&l)[SL][V]) {
        float M[V], S[V], inv[V];
#pragma unroll
        for (int k = 0; k < V; ++k) M[k] = -INFINITY, S[k] = 0.f;
        unit_max<V, SL>(M, m);
        lanes_max<V>(M);
        unit_weights<V, SL>(S, M, m, l);
        lanes_sum<V>(S);
        cnt += unit_inverse<V>(inv, S);
        add_unit_shares<V, SL>(acc, l, inv, agg_max);
      };
      Cursor c = settle(Cursor{rank, u0});
      if (c.g >= groups) return;
      float ma[SL][V], la[SL][V];
      load(c, ma, la);
      if constexpr (SL > 2) {
        while (true) {
          compute(ma, la);
          c = settle(Cursor{c.g, step(c.u)});
          if (c.g >= groups) break;
          load(c, ma, la);
        }
      } else {
        float mb[SL][V], lb[SL][V];
        while (true) {
          Cursor n = settle(Cursor{c.g, step(c.u)});
          if (n.g < groups) load(n, mb, lb);
          compute(ma, la);
          if (n.g >= groups) break;
          c = settle(Cursor{n.g, step(n.u)});
          if (c.g < groups) load(c, ma, la);
          compute(mb, lb);
          if (c.g >= groups) break;
        }
      }
    };
    // the slots in use (the same for the whole CTA), rounded up to a compiled count
    const int slots = (n_tiles + 31) >> 5;
    if (slots <= 1) walk(std::integral_constant<int, 1>{});
    else if (slots <= 2) walk(std::integral_constant<int, 2>{});
    else if (slots <= 4) walk(std::integral_constant<int, 4>{});
    else walk(std::integral_constant<int, kShareRegTiles>{});
#pragma unroll
    for (int i = 0; i < kShareRegTiles; ++i) s_acc[warp][lane + 32 * i] = acc[i];
    __syncthreads();
    for (int t = tid; t < n_tiles; t += blockDim.x) {
      float v = 0.f;
      for (int w = 0; w < warps; ++w) v = agg_max ? fmaxf(v, s_acc[w][t]) : v + s_acc[w][t];
      s_part[t] = v;
    }
  } else {
    // Long rows, a group at a time: each unit's maximum and total weight in one pass over every batch of tiles
    // (a running maximum and a sum rescaled when it grows: one exponential a cell), kept in s_norm (at most
    // eight query rows a warp in a group: see share_shape), then the shares a batch at a time (a second read),
    // the warps added per batch into s_part.
    for (int g = rank; g < groups; g += C) {
      const bool first = g == rank;
      const int layers_g = group_layers(g);
      int j = 0;
      for (Unit u = u0; u.l < layers_g; u = step(u), ++j) {
        const float *cm, *cl;
        unit_cells(g, u, cm, cl);
        float M[V], S[V], inv[V];
#pragma unroll
        for (int k = 0; k < V; ++k) M[k] = -INFINITY, S[k] = 0.f;
        for (int t0 = 0; t0 < n_tiles; t0 += kShareBatch) {
          float m[kShareRegTiles][V], l[kShareRegTiles][V];
          load_unit_tiles<V, kShareRegTiles>(cm, cl, tile_stride, t0, n_tiles, lane, m, l);
#pragma unroll
          for (int i = 0; i < kShareRegTiles; ++i)
#pragma unroll
            for (int k = 0; k < V; ++k) {
              const bool data = m[i][k] > -INFINITY;
              const float d = m[i][k] - M[k];  // +inf while M is -inf
              const float e = __expf(-fabsf(d));
              const bool up = d > 0.f;
              S[k] = data ? (up ? fmaf(S[k], e, l[i][k]) : fmaf(l[i][k], e, S[k])) : S[k];
              M[k] = data && up ? m[i][k] : M[k];
            }
        }
#pragma unroll
        for (int off = 1; off < 32; off <<= 1)
#pragma unroll
          for (int k = 0; k < V; ++k) {
            const float m2 = __shfl_xor_sync(kFullMask, M[k], off), s2 = __shfl_xor_sync(kFullMask, S[k], off);
            lse_merge(M[k], S[k], m2, s2);
          }
        cnt += unit_inverse<V>(inv, S);
        if (lane == 0)
#pragma unroll
          for (int k = 0; k < V; ++k) s_norm[warp][j * V + k] = make_float2(M[k], inv[k]);
      }
      __syncwarp();
      for (int t0 = 0; t0 < n_tiles; t0 += kShareBatch) {
#pragma unroll
        for (int i = 0; i < kShareRegTiles; ++i) acc[i] = 0.f;
        int j = 0;
        for (Unit u = u0; u.l < layers_g; u = step(u), ++j) {
          const float *cm, *cl;
          unit_cells(g, u, cm, cl);
          float m[kShareRegTiles][V], l[kShareRegTiles][V], M[V], inv[V], S[V];
#pragma unroll
          for (int k = 0; k < V; ++k) {
            const float2 z = s_norm[warp][j * V + k];
            M[k] = z.x, inv[k] = z.y, S[k] = 0.f;
          }
          load_unit_tiles<V, kShareRegTiles>(cm, cl, tile_stride, t0, n_tiles, lane, m, l);
          unit_weights<V, kShareRegTiles>(S, M, m, l);
          add_unit_shares<V, kShareRegTiles>(acc, l, inv, agg_max);
        }
#pragma unroll
        for (int i = 0; i < kShareRegTiles; ++i) s_acc[warp][lane + 32 * i] = acc[i];
        __syncthreads();
        for (int t = tid; t < kShareBatch && t0 + t < n_tiles; t += blockDim.x) {
          float v = 0.f;
          for (int w = 0; w < warps; ++w) v = agg_max ? fmaxf(v, s_acc[w][t]) : v + s_acc[w][t];
          const float prev = s_part[t0 + t];
          s_part[t0 + t] = first ? v : (agg_max ? fmaxf(prev, v) : prev + v);
        }
        __syncthreads();
      }
      __syncwarp();  // s_norm is written again by the next group
    }
  }
  if (lane == 0) s_cnt[warp] = cnt;
  __syncthreads();
  if (tid == 0) {
    int c = 0;
    for (int w = 0; w < warps; ++w) c += s_cnt[w];
    s_count = c;
  }
  cluster.sync();  // every CTA's partials and count are complete and visible to the cluster
  int contributors = 0;
  for (int j = 0; j < C; ++j) contributors += *cluster.map_shared_rank(&s_count, j);
  if (rank == 0 && tid == 0) p.contrib_out[r] = contributors;
  // this CTA's slice of the row: tiles [t_lo, t_hi)
  const int width_tiles = (p.width + TB - 1) >> p.tb_shift, per = p.share_slice;
  const int t_lo = min(rank * per, width_tiles), t_hi = min(t_lo + per, width_tiles);
  if (contributors == 0) {
    for (int b = t_lo * TB + tid; b < min(t_hi * TB, p.width); b += blockDim.x) out[b] = NAN;
  } else {
    float row_total = 0.f;  // (max) this thread's blocks' sum
    for (int t = t_lo + tid; t < t_hi; t += blockDim.x) {
      float v = 0.f;
      if (t < n_tiles)
        for (int j = 0; j < C; ++j) {
          const float x = cluster.map_shared_rank(s_part, j)[t];
          v = agg_max ? fmaxf(v, x) : v + x;
        }
      const int bt0 = t * TB;
      const int in_row = t < n_tiles ? min(TB, n - bt0) : 0;
      const float each = in_row > 0 ? v * __frcp_rn(agg_max ? (float)in_row : (float)(in_row * contributors)) : 0.f;
      for (int b = bt0; b < bt0 + TB && b < p.width; ++b) {
        out[b] = b < n ? each : 0.f;
        if (b < n) row_total += each;
      }
    }
    if (agg_max) {
      // the row's total in a fixed order (xor-shuffles, the warps in order, the CTAs in rank order), then
      // each CTA divides its slice by it
      for (int off = 16; off > 0; off >>= 1) row_total += __shfl_xor_sync(kFullMask, row_total, off);
      if (lane == 0) s_red[warp] = row_total;
      __syncthreads();
      if (tid == 0) {
        float part = 0.f;
        for (int w = 0; w < warps; ++w) part += s_red[w];
        s_total = part;
      }
      cluster.sync();
      float total = 0.f;
      for (int j = 0; j < C; ++j) total += *cluster.map_shared_rank(&s_total, j);
      const float inv_total = total > 0.f ? __frcp_rn(total) : 0.f;
      for (int t = t_lo + tid; t < t_hi && t < n_tiles; t += blockDim.x)
        for (int b = t * TB; b < t * TB + TB && b < n; ++b) out[b] *= inv_total;
    }
  }
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

// The share kernel's shared-memory limit, set once per device to the most any launch asks for (one setting
// for every caller: the kernel is the same whatever the record kernel's template arguments).
inline int configure_share_kernel(int device) {
  static bool configured[kMaxDevices] = {};
  if (!configured[device]) {
    if (cudaFuncSetAttribute(share_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kShareMaxTiles * (int)sizeof(float)) != cudaSuccess ||
        cudaFuncSetAttribute(share_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kShareMaxTiles * (int)sizeof(float)) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(share_kernel)");
    configured[device] = true;
  }
  return EKV_OK;
}

// One tensor map per layer of a step: the host-encoded template with the layer's key-cache address
// (a misaligned address is left out; the record kernel skips that layer's copies and reports them).
__global__ void __launch_bounds__(128) kmap_kernel(const __grid_constant__ CUtensorMap tmpl, const uint64_t* k_layers,
                                                   int layer0, int n_layers, CUtensorMap* maps, uint32_t* item_counter) {
  chain_release();  // the record kernel may set up its rows meanwhile
  chain_wait();
  if (threadIdx.x == 0) *item_counter = 0u;  // the record kernel's dynamic items start again
  for (int i = threadIdx.x; i < n_layers; i += blockDim.x) {
    CUtensorMap* map = maps + layer0 + i;
    const uint64_t* src = reinterpret_cast<const uint64_t*>(&tmpl);
    uint64_t* dst = reinterpret_cast<uint64_t*>(map);
#pragma unroll
    for (int w = 0; w < 16; ++w) dst[w] = src[w];
    const uint64_t k = k_layers[layer0 + i];
    if ((k & 15) == 0)
      asm volatile("tensormap.replace.tile.global_address.global.b1024.b64 [%0], %1;" ::"l"(
                       __cvta_generic_to_global(map)), "l"(k)
                   : "memory");
  }
  asm volatile("fence.proxy.tensormap::generic.release.gpu;" ::: "memory");
}

// The record kernel over p.layer0 .. p.layer0 + p.n_layers, then (finalize) the share kernel over the
// layers [share0, share0 + share_layers): every layer of the step, so the table's current cells decide.
template <int TT, int NT, int D, typename T>
int launch_audit(const AuditParams& p, bool finalize, int share0, int share_layers, cudaStream_t stream) {
  using Lay = Layout<D>;
  constexpr int STAGES = Ring<TT>::kStages;
  constexpr size_t fixed = 1024 + (size_t)kWarps * STAGES * TT * 2 * Lay::kHalfRow + kWarps * STAGES * (8 + 4);
  const size_t smem = fixed + (size_t)(4 * p.rows + 1) * 4;
  static int grid_of[kMaxDevices] = {};
  static size_t smem_of[kMaxDevices] = {};
  int device = 0;
  {
    const int dev_rc = current_device(&device);
    if (dev_rc != EKV_OK) return dev_rc;
  }
  auto kernel = record_kernel<TT, NT, D, T>;
  if (grid_of[device] == 0 || smem_of[device] != smem) {
    int sms = 0, per_sm = 0, optin = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess)
      return check_launch("cudaDeviceGetAttribute");
    if (smem > (size_t)optin)
      return fail(EKV_ENOTSUP, "the record kernel needs %zu bytes of shared memory for %d rows; the device has %d",
                  smem, p.rows, optin);
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(record_kernel)");
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kWarps * 32, smem) != cudaSuccess)
      return check_launch("cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    grid_of[device] = sms * (per_sm > 0 ? per_sm : 1);
    smem_of[device] = smem;
  }
  if (p.kmaps != nullptr) {
    launch_chained(kmap_kernel, dim3(1), dim3(128), 0, stream, p.kmap0, p.k_layers, p.layer0, p.n_layers,
                   const_cast<CUtensorMap*>(p.kmaps), p.item_counter);
    const int rc = check_launch("kmap_kernel");
    if (rc != EKV_OK) return rc;
  }
  launch_chained(kernel, dim3(grid_of[device]), dim3(kWarps * 32), smem, stream, p);
  int rc = check_launch("record_kernel");
  if (rc != EKV_OK || !finalize || p.share_out == nullptr) return rc;
  AuditParams ps = p;
  ps.layer0 = share0;
  ps.n_layers = share_layers;
  const ShareShape sh = share_shape(p.Q, share_layers, (reinterpret_cast<uintptr_t>(p.lse) & 15) == 0);
  ps.share_V = sh.V;
  ps.share_QG = sh.QG;
  ps.share_Lg = sh.Lg;
  ps.share_groups = sh.groups;
  ps.share_slice = cdiv(cdiv(p.width, p.tile_blocks), sh.cluster);
  ps.tb_shift = __builtin_ctz((unsigned)p.tile_blocks);
  const size_t share_smem = (size_t)cdiv(p.width, p.tile_blocks) * sizeof(float);
  rc = configure_share_kernel(device);
  if (rc != EKV_OK) return rc;
  launch_chained_cluster(sh.V == 4 ? share_kernel<4> : share_kernel<1>, dim3(sh.cluster, p.rows), dim3(sh.warps * 32),
                         share_smem, stream, (unsigned)sh.cluster, ps);
  return check_launch("share_kernel");
}

template <typename T>
int dispatch(const AuditParams& p, int tt, bool finalize, int share0, int share_layers, cudaStream_t stream) {
  const int nt = p.G <= 8 ? 1 : 2;
  switch (tt * 4 + nt) {
    case 16 * 4 + 1: return launch_audit<16, 1, 128, T>(p, finalize, share0, share_layers, stream);
    case 16 * 4 + 2: return launch_audit<16, 2, 128, T>(p, finalize, share0, share_layers, stream);
    case 32 * 4 + 1: return launch_audit<32, 1, 128, T>(p, finalize, share0, share_layers, stream);
    case 32 * 4 + 2: return launch_audit<32, 2, 128, T>(p, finalize, share0, share_layers, stream);
    case 64 * 4 + 1: return launch_audit<64, 1, 128, T>(p, finalize, share0, share_layers, stream);
    case 64 * 4 + 2: return launch_audit<64, 2, 128, T>(p, finalize, share0, share_layers, stream);
    default: break;
  }
  return fail(EKV_ENOTSUP, "no audit kernel for a tile of %d tokens", tt);
}

// The workspace: the step's work counter (zeroed by kmap_kernel) and the per-layer tensor maps.
struct WorkspaceLayout {
  size_t counters, kmaps, total;
};

WorkspaceLayout workspace_layout(int layers, int rows, int width) {
  (void)rows;
  (void)width;  // the share pass keeps its partials in shared memory
  WorkspaceLayout w{};
  w.counters = 0;
  w.kmaps = 256;
  w.total = w.kmaps + round_up((size_t)layers * sizeof(CUtensorMap), 256);
  return w;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// The key cache at `k` as a 4-D tensor (head dim, KV head, token of the block, block) with boxes of
// 64 dims x 1 head x one block's tokens in the 128-byte swizzle.
int encode_key_map(CUtensorMap* map, const void* k, const AuditParams& p, int dtype) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return fail(EKV_ECUDA, "the driver does not provide cuTensorMapEncodeTiled");
  const cuuint64_t dims[4] = {128, (cuuint64_t)p.kv_heads, (cuuint64_t)p.block_size, (cuuint64_t)p.pool_blocks};
  const cuuint64_t strides[3] = {(cuuint64_t)p.k_s2 * 2, (cuuint64_t)p.k_s1 * 2, (cuuint64_t)p.k_s0 * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)p.block_size, 1};
  const cuuint32_t unit[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, dtype == EKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            4, const_cast<void*>(k), dims, strides, box, unit, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(EKV_ENOTSUP, "the key cache (strides %lld, %lld, %lld elements) has no tensor map (CUresult %d)",
                (long long)p.k_s0, (long long)p.k_s1, (long long)p.k_s2, (int)r);
  return EKV_OK;
}

// Checks shared by both entry points; fills the common fields of p.
int prepare(AuditParams& p, const int32_t* table, const int32_t* lens, const int32_t* qrow,
            const uint8_t* select, const uint32_t* flag, float* lse, float scale, int64_t q_s0,
            int64_t q_s1, int64_t k_s0, int64_t k_s1, int64_t k_s2, int64_t table_s0, int layers,
            int rows, int width, int group_rows, int block_size, int tile_blocks, int head_dim,
            int dtype, int heads, int kv_heads, int64_t pool_blocks, int64_t q_tokens,
            float* share_out, int32_t* contributors, int aggregate, void* workspace,
            size_t workspace_bytes, uint32_t* status, bool need_workspace) {
  if (!table || !lens || !qrow || !select || !flag || !lse)
    return fail(EKV_EINVAL, "a required device pointer is NULL");
  if (rows <= 0 || width <= 0 || layers <= 0) return fail(EKV_EINVAL, "rows, width and layers must be positive");
  if (rows > kMaxRows) return fail(EKV_ENOTSUP, "%d rows: this build handles up to %d", rows, kMaxRows);
  if (layers > kMaxLayers) return fail(EKV_ENOTSUP, "%d layers: this build handles up to %d", layers, kMaxLayers);
  if (group_rows < 1 || group_rows > 16)
    return fail(EKV_EINVAL, "%d query heads per KV head: the kernel handles 1 to 16", group_rows);
  if (heads < 1 || heads > kv_heads) return fail(EKV_EINVAL, "%d heads per layer of a cache with %d", heads, kv_heads);
  if (heads * group_rows > kMaxQ) return fail(EKV_ENOTSUP, "%d values per cell exceed %d", heads * group_rows, kMaxQ);
  if (block_size <= 0 || tile_blocks <= 0) return fail(EKV_EINVAL, "block_size and tile_blocks must be positive");
  const int tt = block_size * tile_blocks;
  if (tt & (tt - 1)) return fail(EKV_EINVAL, "a tile of the audit kernel must hold a power of two of tokens");
  if (tile_blocks > 8) return fail(EKV_ENOTSUP, "tile_blocks %d: this build handles up to 8", tile_blocks);
  if (block_size & 7)
    return fail(EKV_ENOTSUP, "block_size %d: the kernel copies whole blocks of a multiple of 8 tokens", block_size);
  if (pool_blocks > 0x7fffffffll) return fail(EKV_ENOTSUP, "%lld blocks in the pool exceed 2^31 - 1", (long long)pool_blocks);
  if ((long long)rows * cdiv(width, tile_blocks * EKV_AUDIT_CHUNK_TILES) * heads * layers > 0x7fffffffll)
    return fail(EKV_ENOTSUP, "a launch of more than 2^31 - 1 work items (rows x chunks x heads x layers)");
  if (head_dim != 128) return fail(EKV_ENOTSUP, "head_dim %d: this build has kernels for 128", head_dim);
  if (dtype != EKV_DTYPE_F16 && dtype != EKV_DTYPE_BF16) return fail(EKV_EINVAL, "unknown dtype %d", dtype);
  if (pool_blocks <= 0 || q_tokens <= 0) return fail(EKV_EINVAL, "pool_blocks and q_tokens must be positive");
  if ((k_s0 & 7) || (k_s1 & 7) || (k_s2 & 7))
    return fail(EKV_EINVAL, "the key cache's strides must be whole 16-byte units");
  if ((q_s0 & 1) || (q_s1 & 1)) return fail(EKV_EINVAL, "the query's strides must be even");
  if (table_s0 < width) return fail(EKV_EINVAL, "table_stride %lld < width %d", (long long)table_s0, width);
  if (aggregate != EKV_AGG_MEAN && aggregate != EKV_AGG_MAX) return fail(EKV_EINVAL, "unknown aggregate %d", aggregate);
  p.table = table; p.lens = lens; p.qrow = qrow; p.select = select; p.flag = flag; p.lse = lse;
  p.scale = scale; p.q_s0 = q_s0; p.q_s1 = q_s1; p.k_s0 = k_s0; p.k_s1 = k_s1; p.k_s2 = k_s2;
  p.table_s0 = table_s0; p.layers = layers; p.rows = rows; p.width = width; p.G = group_rows;
  p.heads = heads; p.Q = heads * group_rows; p.block_size = block_size; p.tile_blocks = tile_blocks;
  p.kv_heads = kv_heads; p.pool_blocks = pool_blocks; p.q_tokens = q_tokens; p.status = status;
  p.share_out = share_out; p.contrib_out = contributors; p.aggregate = aggregate;
  if (share_out && !contributors) return fail(EKV_EINVAL, "share_out needs contributors");
  if (share_out && cdiv(width, tile_blocks) > kShareMaxTiles)
    return fail(EKV_ENOTSUP, "width %d: the share pass holds up to %d tiles of a row", width, kShareMaxTiles);
  if (need_workspace) {
    const WorkspaceLayout w = workspace_layout(layers, rows, width);
    if (!workspace || workspace_bytes < w.total)
      return fail(EKV_ERANGE, "the audit workspace holds %zu bytes, the launch needs %zu", workspace_bytes, w.total);
    if ((uintptr_t)workspace & 255) return fail(EKV_EINVAL, "the audit workspace must be 256-byte aligned");
    uint8_t* base = static_cast<uint8_t*>(workspace);
    p.item_counter = reinterpret_cast<uint32_t*>(base + w.counters);
    p.kmaps = reinterpret_cast<const CUtensorMap*>(base + w.kmaps);
  }
  return EKV_OK;
}

// Copies the query rows of the audited heads of every row, q[qrow[r], (group + h) * G + g, :], into
// stash[r][h * G + g][:] (16 bytes per thread), so a later multi-layer launch can read them.
template <int D>
__global__ void __launch_bounds__(256) stash_kernel(const uint8_t* q, int64_t q_s0, int64_t q_s1,
                                                    const int32_t* qrow, int rows, int64_t q_tokens,
                                                    int first_head, int heads_x_g, uint8_t* stash,
                                                    uint32_t* status) {
  chain_release();
  chain_wait();  // the query may come from the launch before this one
  constexpr int kChunks = 2 * D / 16;  // 16-byte pieces of one query row
  const long long total = (long long)rows * heads_x_g * kChunks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int piece = (int)(i % kChunks);
    const long long rj = i / kChunks;
    const int j = (int)(rj % heads_x_g);
    const int r = (int)(rj / heads_x_g);
    const int token = qrow[r];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (token >= 0 && (int64_t)token < q_tokens) {
      v = *reinterpret_cast<const uint4*>(q + 2 * ((int64_t)token * q_s0 + (int64_t)(first_head + j) * q_s1) + 16 * piece);
    } else if (piece == 0 && j == 0) {
      set_status(status, EKV_STATUS_BAD_QROW);
    }
    *reinterpret_cast<uint4*>(stash + ((long long)r * heads_x_g + j) * 2 * D + 16 * piece) = v;
  }
}

}  // namespace ekv

using namespace ekv;

extern "C" int ekv_audit_stash(const void* q, int64_t q_stride_token, int64_t q_stride_head,
                               const int32_t* qrow, int rows, int64_t q_tokens, int group, int heads,
                               int group_rows, int head_dim, void* stash, uint32_t* status, void* stream) {
  clear_error();
  if (!q || !qrow || !stash) return fail(EKV_EINVAL, "a required device pointer is NULL");
  if (rows <= 0 || heads <= 0 || group_rows <= 0 || group < 0 || q_tokens <= 0)
    return fail(EKV_EINVAL, "rows, heads, group_rows and q_tokens must be positive");
  if (head_dim != 128) return fail(EKV_ENOTSUP, "head_dim %d: this build has kernels for 128", head_dim);
  if (((uintptr_t)q & 15) || (q_stride_token & 7) || (q_stride_head & 7) || ((uintptr_t)stash & 15))
    return fail(EKV_EINVAL, "the query and the stash must be 16-byte aligned with strides of whole 16-byte units");
  const long long pieces = (long long)rows * heads * group_rows * (2 * 128 / 16);
  const int blocks = (int)((pieces + 255) / 256 < 1024 ? (pieces + 255) / 256 : 1024);
  launch_chained(stash_kernel<128>, dim3(blocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                 static_cast<const uint8_t*>(q), q_stride_token, q_stride_head, qrow, rows, q_tokens,
                 group * group_rows, heads * group_rows, static_cast<uint8_t*>(stash), status);
  return check_launch("stash_kernel");
}

extern "C" size_t ekv_audit_workspace_bytes(int layers, int rows, int width) {
  if (layers <= 0 || rows <= 0 || width <= 0) return 0;
  return workspace_layout(layers, rows, width).total;
}

extern "C" int ekv_audit_launch(
    const void* q, const void* k, const int32_t* table, const int32_t* lens, const int32_t* qrow,
    const uint8_t* select, const uint32_t* flag, float* lse, float scale, int layer, int group,
    int64_t q_stride_token, int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos,
    int64_t k_stride_head, int64_t table_stride, int layers, int rows, int width, int group_rows,
    int block_size, int tile_blocks, int head_dim, int dtype, int heads, int kv_heads,
    int64_t pool_blocks, int64_t q_tokens, float* share_out, int32_t* contributors, int aggregate,
    int share_flags, void* workspace, size_t workspace_bytes, uint32_t* status, void* stream) {
  clear_error();
  if (!q || !k) return fail(EKV_EINVAL, "a required device pointer is NULL");
  AuditParams p{};
  const int rc = prepare(p, table, lens, qrow, select, flag, lse, scale, q_stride_token, q_stride_head,
                         k_stride_block, k_stride_pos, k_stride_head, table_stride, layers, rows, width,
                         group_rows, block_size, tile_blocks, head_dim, dtype, heads, kv_heads,
                         pool_blocks, q_tokens, share_out, contributors, aggregate, workspace,
                         workspace_bytes, status, false);
  if (rc != EKV_OK) return rc;
  if (layer < 0 || layer >= layers)
    return fail(EKV_ERANGE, "layer %d is outside the %d layers the table was sized for", layer, layers);
  if (group < 0 || group + heads > kv_heads)
    return fail(EKV_EINVAL, "KV heads [%d, %d) are outside the cache's %d heads", group, group + heads, kv_heads);
  if (((uintptr_t)k & 15) || ((uintptr_t)q & 3))
    return fail(EKV_EINVAL, "the key cache must be 16-byte aligned and the query 4-byte aligned");
  p.q = q; p.k = k; p.layer0 = layer; p.n_layers = 1; p.group = group; p.rotate = 0;
  const int enc = encode_key_map(&p.kmap0, k, p, dtype);
  if (enc != EKV_OK) return enc;
  const bool finalize = (share_flags & EKV_SHARE_FINALIZE) != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tt = block_size * tile_blocks;
  return dtype == EKV_DTYPE_BF16 ? dispatch<__nv_bfloat16>(p, tt, finalize, 0, layers, s)
                                 : dispatch<__half>(p, tt, finalize, 0, layers, s);
}

namespace {

// The audit step of ekv_audit_step and ekv_audit_step_static.
int audit_step(const uint64_t* q_layers, const uint64_t* k_layers, const int32_t* table, const int32_t* lens,
               const int32_t* qrow, const uint8_t* select, const uint32_t* flag, float* lse, float scale,
               int layer0, int n_layers, int group, int rotate, int q_layout, int64_t q_stride_token,
               int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos, int64_t k_stride_head,
               int64_t table_stride, int layers, int rows, int width, int group_rows, int block_size,
               int tile_blocks, int head_dim, int dtype, int heads, int kv_heads, int64_t pool_blocks,
               int64_t q_tokens, float* share_out, int32_t* contributors, int aggregate, void* workspace,
               size_t workspace_bytes, uint32_t* status, void* stream) {
  if (!q_layers || !k_layers) return fail(EKV_EINVAL, "the per-layer address arrays must not be NULL");
  AuditParams p{};
  const int rc = prepare(p, table, lens, qrow, select, flag, lse, scale, q_stride_token, q_stride_head,
                         k_stride_block, k_stride_pos, k_stride_head, table_stride, layers, rows, width,
                         group_rows, block_size, tile_blocks, head_dim, dtype, heads, kv_heads,
                         pool_blocks, q_tokens, share_out, contributors, aggregate, workspace,
                         workspace_bytes, status, true);
  if (rc != EKV_OK) return rc;
  if (n_layers <= 0 || layer0 < 0 || layer0 + n_layers > layers)
    return fail(EKV_ERANGE, "layers [%d, %d) are outside the %d the table was sized for", layer0,
                layer0 + n_layers, layers);
  if (group < 0 || (rotate ? (heads != 1 || group >= kv_heads) : group + heads > kv_heads))
    return fail(EKV_EINVAL, "KV head %d (rotate %d, %d heads) does not fit a cache of %d heads", group,
                rotate, heads, kv_heads);
  p.q_layers = q_layers; p.k_layers = k_layers; p.layer0 = layer0; p.n_layers = n_layers;
  p.group = group; p.rotate = rotate != 0; p.q_stash = q_layout != 0;
  // the template of the per-layer maps: any aligned device address stands in for the layers' caches
  const int enc = encode_key_map(&p.kmap0, workspace, p, dtype);
  if (enc != EKV_OK) return enc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tt = block_size * tile_blocks;
  return dtype == EKV_DTYPE_BF16 ? dispatch<__nv_bfloat16>(p, tt, true, layer0, n_layers, s)
                                 : dispatch<__half>(p, tt, true, layer0, n_layers, s);
}

}  // namespace

extern "C" int ekv_audit_step(
    const uint64_t* q_layers, const uint64_t* k_layers, const int32_t* table, const int32_t* lens,
    const int32_t* qrow, const uint8_t* select, const uint32_t* flag, float* lse, float scale,
    int layer0, int n_layers, int group, int rotate, int q_layout, int64_t q_stride_token, int64_t q_stride_head,
    int64_t k_stride_block, int64_t k_stride_pos, int64_t k_stride_head, int64_t table_stride,
    int layers, int rows, int width, int group_rows, int block_size, int tile_blocks, int head_dim,
    int dtype, int heads, int kv_heads, int64_t pool_blocks, int64_t q_tokens, float* share_out,
    int32_t* contributors, int aggregate, void* workspace, size_t workspace_bytes,
    uint32_t* status, void* stream) {
  clear_error();
  return audit_step(q_layers, k_layers, table, lens, qrow, select, flag, lse, scale, layer0, n_layers, group,
                    rotate, q_layout, q_stride_token, q_stride_head, k_stride_block, k_stride_pos, k_stride_head,
                    table_stride, layers, rows, width, group_rows, block_size, tile_blocks, head_dim, dtype, heads,
                    kv_heads, pool_blocks, q_tokens, share_out, contributors, aggregate, workspace,
                    workspace_bytes, status, stream);
}

// ---- the audit step without a caller-provided workspace ---------------------------------------------
//
// Some callers cannot allocate device memory when they record: a binding that has no CUDA allocator of
// its own (a cgo or ctypes caller that only holds the engine's tensors), or engine code after memory
// profiling has sized the KV-cache pool, where one more cudaMalloc can fail or fragment the pool. For
// them the step's workspace lives in this file-scope array, which every GPU that loads the library
// holds until the process exits. Every call shares it: calls whose launches overlap on the GPU race.

// The workspace of the widest step this build accepts: the work counter and kMaxLayers tensor maps.
#define EKV_AUDIT_STATIC_SCRATCH_BYTES (256u + 1024u * 128u)
static_assert(EKV_AUDIT_STATIC_SCRATCH_BYTES >= 256 + kMaxLayers * sizeof(CUtensorMap), "the static workspace holds every step");

static __device__ __align__(256) uint8_t g_audit_scratch[EKV_AUDIT_STATIC_SCRATCH_BYTES];

#include <mutex>

extern "C" size_t ekv_audit_static_scratch_bytes(void) { return EKV_AUDIT_STATIC_SCRATCH_BYTES; }

namespace {

// The device address of g_audit_scratch in the current context, looked up with cudaGetSymbolAddress
// the first time a context calls (the lookup loads the module on that device, so that first call
// belongs before any stream capture) and kept per device together with the context's ID: a new
// context on the same ordinal (after cudaDeviceReset, or another process-level context) has its own
// copy of the module and looks the address up again.
int static_scratch(void** out) {
  *out = nullptr;
  int device = 0;
  const int rc = current_device(&device);
  if (rc != EKV_OK) return rc;
  static const auto get_current = []() -> PFN_cuCtxGetCurrent_v4000 {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  }();
  static const auto get_id = []() -> PFN_cuCtxGetId_v12000 {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuCtxGetId_v12000>(f);
  }();
  if (get_current == nullptr || get_id == nullptr)
    return fail(EKV_ENOTSUP, "the driver does not export cuCtxGetCurrent and cuCtxGetId");
  // A thread that has not used the runtime yet has no current context: the symbol lookup makes the
  // device's primary context current, and its ID is read after it.
  auto context_id = [&](unsigned long long* id) {
    CUcontext ctx = nullptr;
    return get_current(&ctx) == CUDA_SUCCESS && ctx != nullptr && get_id(ctx, id) == CUDA_SUCCESS;
  };
  unsigned long long ctx_id = 0;
  const bool known = context_id(&ctx_id);
  struct Entry {
    unsigned long long ctx_id;
    void* ptr;
  };
  static Entry entries[kMaxDevices] = {};
  static std::mutex setup;
  std::lock_guard<std::mutex> lock(setup);
  Entry& e = entries[device];
  if (!known || e.ptr == nullptr || e.ctx_id != ctx_id) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_audit_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return fail(EKV_ECUDA, "cudaGetSymbolAddress(static audit workspace): %s", cudaGetErrorString(err));
    if (!known && !context_id(&ctx_id)) return fail(EKV_ECUDA, "device %d has no current context", device);
    e.ctx_id = ctx_id;
    e.ptr = ptr;
  }
  *out = e.ptr;
  return EKV_OK;
}

}  // namespace

extern "C" int ekv_audit_step_static(
    const uint64_t* q_layers, const uint64_t* k_layers, const int32_t* table, const int32_t* lens,
    const int32_t* qrow, const uint8_t* select, const uint32_t* flag, float* lse, float scale,
    int layer0, int n_layers, int group, int rotate, int q_layout, int64_t q_stride_token,
    int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos, int64_t k_stride_head,
    int64_t table_stride, int layers, int rows, int width, int group_rows, int block_size,
    int tile_blocks, int head_dim, int dtype, int heads, int kv_heads, int64_t pool_blocks,
    int64_t q_tokens, float* share_out, int32_t* contributors, int aggregate, uint32_t* status,
    void* stream) {
  clear_error();
  if (!share_out || !contributors) return fail(EKV_EINVAL, "share_out and contributors are required");
  if (layers <= 0 || rows <= 0 || width <= 0) return fail(EKV_EINVAL, "rows, width and layers must be positive");
  const size_t need = ekv_audit_workspace_bytes(layers, rows, width);
  if (need > EKV_AUDIT_STATIC_SCRATCH_BYTES)
    return fail(EKV_ERANGE,
                "a step of %d layers x %d rows x %d blocks needs %zu bytes of workspace; the static one holds %u: "
                "pass a workspace to ekv_audit_step instead",
                layers, rows, width, need, (unsigned)EKV_AUDIT_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  const int rc = static_scratch(&scratch);
  if (rc != EKV_OK) return rc;
  // Nothing in the array needs clearing: every step's kmap_kernel rewrites the tensor maps and zeroes the work
  // counter before the record kernel reads them.
  return audit_step(q_layers, k_layers, table, lens, qrow, select, flag, lse, scale, layer0, n_layers, group,
                    rotate, q_layout, q_stride_token, q_stride_head, k_stride_block, k_stride_pos, k_stride_head,
                    table_stride, layers, rows, width, group_rows, block_size, tile_blocks, head_dim, dtype, heads,
                    kv_heads, pool_blocks, q_tokens, share_out, contributors, aggregate, scratch,
                    EKV_AUDIT_STATIC_SCRATCH_BYTES, status, stream);
}
