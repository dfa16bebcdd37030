// The `maxmin` objective on the device: raise the smallest retained share of any request as far as one
// shared budget allows, then spend what is left (observe/allocation.py:121-166, _water_level).
//
// The reference, per request r: shares s = max(score, 0) / total (float64, total by NumPy's pairwise
// sum; equal shares without evidence), the unpinned blocks in order of decreasing share (equal shares:
// the older block first), base_r = the pairwise sum of the pinned shares, prefix_r = the running sum
// (np.cumsum) of the ordered shares. extra_r(level) = 0 when level - base_r <= 1e-12, else
// min(searchsorted(prefix + 2 r', level - base_r - 1e-12 + 2 r') + 1, open_r), with r' the request's
// index; 60 bisection steps on [0, 1] find the highest level whose extras fit the free budget, and
// the rest of the budget goes one block at a time to the request with the lowest retained share
// (ties: the earlier request). Here:
//   mm_prep_kernel, one CTA per row: the total, the shares of the pinned blocks summed as NumPy sums
//     them, the unpinned blocks ordered by a stable radix sort of their share keys (equal keys keep the
//     older block first), their shares in that order; the CTA that finishes last sets the budget and
//     each request's index.
//   mm_cumsum_kernel, a thread per row: the running sums, one addition after another as np.cumsum.
//   mm_wide_kernel, a thread per (request, level), in stages of six steps: the first bisection steps'
//     levels evaluated over every SM (their searches span most of a row: one SM's loads would be the
//     bottleneck).
//   mm_level_kernel, one CTA: the rest of the bisection (a binary search per request and a reduction
//     per step) and the leftover blocks through a binary heap in shared memory. The row quotas it
//     writes make ekv_view_build (EKV_POLICY_UNIFORM: equal shares to the older block) keep exactly
//     the reference's blocks.
#include <type_traits>

#include "ekv_common.cuh"
#include "pairwise.cuh"
#include "pins.cuh"

namespace ekv {

constexpr int kMmThreads = 1024;
constexpr int kMmMaxWidth = 8192;
constexpr int kMmMaxRows = 4096;
constexpr int kMmBisection = 60;

enum MmMode : int { kMmSelect = 0, kMmNone = 1, kMmAll = 2 };

constexpr int kMmWideSteps = 6;                            // bisection steps of one mm_wide_kernel stage
constexpr int kMmWideNodes = (1 << kMmWideSteps) - 1;      // the levels they can probe
constexpr int kMmWideStages = 2;                           // stages before the single CTA's rounds

struct MmState {
  long long must, blocks, total_open, free_;
  int mode;
  unsigned int ticket;
  long long wide[kMmWideStages * kMmWideNodes];  // blocks the requests take at each wide level
};

struct MmParams {
  const void* scores;          // float or double [.][score_s0] (mm_prep_kernel<float> / <double>)
  int64_t score_s0;
  const int32_t* score_rows;   // may be NULL: row r's scores are scores row score_rows[r]
  const int32_t* row_blocks;
  const int32_t* measured;
  int recent, cap;
  double fraction;
  long long budget;
  int rows, width;
  int32_t* quota;
  // workspace
  MmState* state;
  double* base;     // [rows] pinned share
  int* row_m;       // [rows] unpinned blocks; -1 for a row that is not a request
  int* req;         // [rows] index of the request among the requests
  double* sorted;   // [width][rows] unpinned shares in decreasing order (block-major: a warp's rows adjacent)
  double* prefix;   // [width][rows] their running sums
  uint16_t* wide_lbs;  // [kMmWideStages * kMmWideNodes][rows] each request's search result at the wide levels
  // float64 rows that already hold each request's shares (the pinned allocation): no total is taken
  bool presummed;
  const long long* budget_add;  // may be NULL: blocks added on the device to a budget given as a count
};

struct MmLayout {
  size_t state, base, row_m, req, wide_lbs, sorted, prefix, bytes;
};

MmLayout mm_layout(int rows, int width) {
  MmLayout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += round_up(bytes, 256);
    return at;
  };
  l.state = take(sizeof(MmState));
  l.base = take((size_t)rows * 8);
  l.row_m = take((size_t)rows * 4);
  l.req = take((size_t)rows * 4);
  l.wide_lbs = take((size_t)rows * kMmWideStages * kMmWideNodes * 2);
  l.sorted = take((size_t)rows * width * 8);
  l.prefix = take((size_t)rows * width * 8);
  l.bytes = o;
  return l;
}

__device__ __forceinline__ double mm_clamped(float s) { return s > 0.f ? (double)s : 0.0; }
__device__ __forceinline__ double mm_clamped(double s) { return s > 0.0 ? s : 0.0; }

constexpr int kMmSortItems = kMmMaxWidth / kMmThreads;  // keys a thread holds in a sort pass
constexpr int kMmDigits = 256;                            // 8-bit digits
// A warp's digit counts (uint16) take kMmCountStride entries: rows two entries longer than the digits
// put the 8 warps x 4 digit pairs that a warp of the count scan reads in 32 different banks.
constexpr int kMmCountStride = kMmDigits + 2;
constexpr int kMmWarps = kMmThreads / 32;
constexpr int kMmScanWarps = 8;                                   // counts of one digit a thread scans
constexpr int kMmDigitThreads = kMmWarps / kMmScanWarps;          // threads per digit in the scan
static_assert(kMmDigitThreads * kMmDigits == kMmThreads, "the count scan gives every thread 8 warps of a digit");
static_assert(kMmWarps <= 32, "a warp scans the warp totals");

// Keys of a row's sort: a multiple of kMmThreads covering the width.
__host__ __device__ __forceinline__ int mm_sort_n(int width) {
  return (width + kMmThreads - 1) / kMmThreads * kMmThreads;
}

// Shared memory of mm_prep_kernel<S>: the row's scores, then the sort keys (uint32 for float32 scores,
// uint64 for float64, [mm_sort_n(width)]), the block of each key (uint16) and the digit counts of
// every warp (uint16 [warps][kMmCountStride]); the pairwise sums' scratch, used before the sort, lies over these.
template <typename S>
__host__ __device__ __forceinline__ size_t mm_prep_smem(int width) {
  const size_t scores = ((size_t)width * sizeof(S) + 15) / 16 * 16;
  const size_t keys = (size_t)mm_sort_n(width) * sizeof(S);
  const size_t blocks = ((size_t)mm_sort_n(width) * 2 + 15) / 16 * 16;
  const size_t sort = keys + blocks + (size_t)kMmWarps * kMmCountStride * 2;
  const size_t tree = pairwise_bytes(pairwise_slots(width));
  return scores + (sort > tree ? sort : tree);
}

// Stable ascending sort of the keys s_key[0, kMmThreads * items) with their blocks s_blk, in shared memory:
// least significant digit first, 8 bits a pass. Warp w holds elements [w * 32 * items, (w + 1) * 32 *
// items), item k of lane l being element w * 32 * items + 32 k + l; a warp ranks its items in element
// order (items in order, lanes with the same digit by eight ballots), the counts of every (digit, warp)
// are scanned digit-major, warp-minor, and every key goes to its digit's start + the count of
// earlier equal digits: a stable pass.
template <typename K>
__device__ void mm_radix_sort(K* s_key, uint16_t* s_blk, uint16_t* s_cnt, int* s_scan, int items) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int span = 32 * items;
  uint16_t* wcnt = s_cnt + warp * kMmCountStride;  // this warp's counts
  for (int shift = 0; shift < 8 * (int)sizeof(K); shift += 8) {
    K key[kMmSortItems];
    uint32_t item[kMmSortItems];  // the key's block (low half), then its rank in the warp's digit (high)
#pragma unroll
    for (int k = 0; k < kMmSortItems; ++k) {
      if (k < items) {
        const int e = warp * span + 32 * k + lane;
        key[k] = s_key[e];
        item[k] = s_blk[e];
      }
    }
    for (int i = tid; i < kMmWarps * kMmCountStride; i += kMmThreads) s_cnt[i] = 0;
    __syncthreads();  // every key read, every count zero
#pragma unroll
    for (int k = 0; k < kMmSortItems; ++k) {
      if (k < items) {
        const unsigned d = (unsigned)(key[k] >> shift) & (kMmDigits - 1);
        uint32_t peers = kFullMask;  // the lanes with this digit: eight ballots (faster than match.any)
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          const uint32_t bal = __ballot_sync(kFullMask, (d >> b) & 1u);
          peers &= ((d >> b) & 1u) ? bal : ~bal;
        }
        const int below = __popc(peers & lanes_below());
        const int seen = wcnt[d];
        item[k] |= (uint32_t)(seen + below) << 16;
        __syncwarp();
        if (below == 0) wcnt[d] = (uint16_t)(seen + __popc(peers));
        __syncwarp();
      }
    }
    __syncthreads();
    // thread t: the counts of 8 warps of one digit, in the digit-major order of the scan
    const int d = tid / kMmDigitThreads, w0 = (tid % kMmDigitThreads) * kMmScanWarps;
    int c[kMmScanWarps], sum = 0;
#pragma unroll
    for (int i = 0; i < kMmScanWarps; ++i) c[i] = s_cnt[(w0 + i) * kMmCountStride + d], sum += c[i];
    // the exclusive prefix of `sum` over the threads: a warp scan, then every warp scans the warp totals
    int inc = sum;
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(kFullMask, inc, off);
      if (lane >= off) inc += v;
    }
    if (lane == 31) s_scan[warp] = inc;
    __syncthreads();
    int before = lane < warp ? s_scan[lane] : 0;  // the totals of the warps before this one
    for (int off = 16; off > 0; off >>= 1) before += __shfl_xor_sync(kFullMask, before, off);
    int at = before + inc - sum;
#pragma unroll
    for (int i = 0; i < kMmScanWarps; ++i) s_cnt[(w0 + i) * kMmCountStride + d] = (uint16_t)at, at += c[i];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kMmSortItems; ++k) {
      if (k < items) {
        const unsigned dk = (unsigned)(key[k] >> shift) & (kMmDigits - 1);
        const int pos = wcnt[dk] + (int)(item[k] >> 16);
        s_key[pos] = key[k];
        s_blk[pos] = (uint16_t)item[k];
      }
    }
    __syncthreads();
  }
}

// max(score, 0) as an order-preserving uint32 (NaN as 0)
__device__ __forceinline__ uint32_t mm_score_key(float s) { return s > 0.f ? __float_as_uint(s) : 0u; }

// One CTA per row. Float32 scores sort one uint64 per block, (~score bits, block): for scores that
// float32 holds, the order of the scores is the order of the shares. Float64 scores sort pairs
// (~share bits, block), the share being the very float64 value the reference orders
// (allocation.py:129): distinct scores can give equal shares.
template <typename S>
__global__ void __launch_bounds__(kMmThreads) mm_prep_kernel(const MmParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  extern __shared__ __align__(16) unsigned char mm_smem[];
  __shared__ bool s_last;
  constexpr bool kWide = sizeof(S) == 8;
  const int r = blockIdx.x, tid = threadIdx.x;
  int n = p.row_blocks[r];
  const bool request = n > p.cap && n > 0;
  if (n > p.width) n = p.width;
  using Key = typename std::conditional<sizeof(S) == 8, unsigned long long, uint32_t>::type;
  const int N = mm_sort_n(p.width);
  S* s_x = reinterpret_cast<S*>(mm_smem);
  Key* s_key = reinterpret_cast<Key*>(mm_smem + ((size_t)p.width * sizeof(S) + 15) / 16 * 16);
  uint16_t* s_blk = reinterpret_cast<uint16_t*>(s_key + N);
  uint16_t* s_cnt = reinterpret_cast<uint16_t*>(reinterpret_cast<unsigned char*>(s_blk) + ((size_t)N * 2 + 15) / 16 * 16);
  __shared__ int s_scan[kMmThreads / 32 + 1];
  const PairwiseScratch s_tree = pairwise_scratch(s_key, pairwise_slots(p.width));  // until the keys are written
  const int ps = request ? pin_start(n, p.recent, p.measured, r) : 0;
  const int m = ps > 1 ? ps - 1 : 0;  // unpinned blocks [1, ps)
  if (request) {
    const S* xg = static_cast<const S*>(p.scores) +
                  (p.score_rows != nullptr ? (int64_t)p.score_rows[r] : (int64_t)r) * p.score_s0;
    stage_row<kMmThreads>(s_x, xg, n);
    const double total =
        p.presummed ? 1.0 : block_pairwise_sum<kMmThreads>(s_tree, n, [&](int i) { return mm_clamped(s_x[i]); });
    const double equal = __ddiv_rn(1.0, (double)(n > 1 ? n : 1));
    auto share = [&](int i) { return total > 0.0 ? __ddiv_rn(mm_clamped(s_x[i]), total) : equal; };
    // the pinned blocks in index order: block 0 and [ps, n) (every block when ps == 0)
    const int npin = ps >= 1 ? 1 + (n - ps) : n;
    const double base = block_pairwise_sum<kMmThreads>(
        s_tree, npin, [&](int j) { return share(ps >= 1 ? (j == 0 ? 0 : ps + j - 1) : j); });
    __syncthreads();  // every thread has the sums: the keys may overwrite the scratch
    // the unpinned blocks by decreasing share, equal shares by increasing block: ascending keys in
    // block order through a stable sort; the padding (all ones) sorts last
    const int items = (m + kMmThreads - 1) / kMmThreads;
    for (int j = tid; j < items * kMmThreads; j += kMmThreads) {
      if constexpr (kWide) {
        s_key[j] = j < m ? ~(unsigned long long)__double_as_longlong(share(1 + j)) : ~0ull;
      } else {
        s_key[j] = j < m ? ~mm_score_key(s_x[1 + j]) : ~0u;
      }
      s_blk[j] = (uint16_t)(j < m ? 1 + j : 0);
    }
    __syncthreads();
    if (items > 0) mm_radix_sort<Key>(s_key, s_blk, s_cnt, s_scan, items);
    for (int j = tid; j < m; j += kMmThreads) p.sorted[(int64_t)j * p.rows + r] = share((int)s_blk[j]);
    if (tid == 0) {
      p.base[r] = base;
      atomicAdd((unsigned long long*)&p.state->must, (unsigned long long)pin_count(n, ps));
      atomicAdd((unsigned long long*)&p.state->blocks, (unsigned long long)n);
      atomicAdd((unsigned long long*)&p.state->total_open, (unsigned long long)m);
    }
  }
  if (tid == 0) p.row_m[r] = request ? m : -1;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&p.state->ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // the budget (controller.py:435-437), what to do with it (allocation.py:64-67) and each request's index
  MmState* st = p.state;
  if (tid == 0) {
    const long long must = *(volatile long long*)&st->must, blocks = *(volatile long long*)&st->blocks;
    long long budget = p.budget;
    if (budget < 0) {
      budget = (long long)ceil(p.fraction * (double)blocks);
      if (budget < must) budget = must;
    } else if (p.budget_add != nullptr) {
      budget += *p.budget_add;
    }
    const long long free_ = budget - must;
    st->free_ = free_;
    st->mode = budget >= blocks ? kMmAll : (free_ <= 0 ? kMmNone : kMmSelect);
    st->ticket = 0;
  }
  int carry = 0;
  for (int b0 = 0; b0 < p.rows; b0 += kMmThreads) {
    const int row = b0 + tid;
    const int is_req = row < p.rows && __ldcg(p.row_m + row) >= 0;
    int total = 0;
    const int before = block_exclusive_scan<kMmThreads>(is_req, s_scan, &total);
    if (row < p.rows) p.req[row] = carry + before;
    carry += total;
  }
}

// A thread per row: prefix[j] = prefix[j - 1] + sorted[j], one addition after another (block-major
// arrays: a warp's loads and stores are contiguous). The additions of a row are a dependent chain, so
// the loads run far ahead of it: each lane copies its own row's next shares into a ring of shared-memory
// stages with cp.async (8 bytes per copy, 256 bytes per warp instruction) and reads back only what it
// copied itself, so no barrier is needed.
constexpr int kCsChunk = 32;   // shares of a row per stage
constexpr int kCsStages = 8;   // stages in the ring: 7 in flight while one is added up
constexpr size_t kCsSmem = (size_t)kCsStages * kCsChunk * 32 * sizeof(double);

__global__ void __launch_bounds__(32) mm_cumsum_kernel(const MmParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  extern __shared__ __align__(16) double cs_ring[];  // [kCsStages][kCsChunk][32]
  const int lane = threadIdx.x;
  const int r = blockIdx.x * 32 + lane;
  const int m = r < p.rows ? p.row_m[r] : 0;
  const int64_t R = p.rows;
  int most = m;
  for (int off = 16; off > 0; off >>= 1) most = max(most, __shfl_xor_sync(kFullMask, most, off));
  const int chunks = most > 0 ? (most + kCsChunk - 1) / kCsChunk : 0;
  const double* src = p.sorted + (r < p.rows ? r : 0);
  double* dst = p.prefix + (r < p.rows ? r : 0);
  double* ring = cs_ring + lane;
  // chunk c: this lane's shares c * kCsChunk + u, u < kCsChunk, into stage c % kCsStages
  auto issue = [&](int c) {
    if (c < chunks) {
      const int left = m - c * kCsChunk;
      const double* g = src + (int64_t)c * kCsChunk * R;
      double* sh = ring + (c % kCsStages) * kCsChunk * 32;
      if (left >= kCsChunk) {
#pragma unroll
        for (int u = 0; u < kCsChunk; ++u) cp_async8(sh + u * 32, g + u * R);
      } else {
        for (int u = 0; u < left; ++u) cp_async8(sh + u * 32, g + u * R);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // an empty group keeps the count in step
  };
  for (int c = 0; c < kCsStages - 1; ++c) issue(c);
  // np.cumsum: out[0] = a[0], out[j] = out[j - 1] + a[j]; the shares are +0 or positive, so starting
  // from +0 gives out[0] bit for bit
  double acc = 0.0;
  for (int c = 0; c < chunks; ++c) {
    issue(c + kCsStages - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(kCsStages - 1) : "memory");  // chunk c has landed
    const double* sh = ring + (c % kCsStages) * kCsChunk * 32;
    double* g = dst + (int64_t)c * kCsChunk * R;
    const int left = m - c * kCsChunk;
    if (left >= kCsChunk) {
#pragma unroll
      for (int u = 0; u < kCsChunk; ++u) {
        acc = __dadd_rn(acc, sh[u * 32]);
        g[u * R] = acc;
      }
    } else {
      for (int u = 0; u < left; ++u) {
        acc = __dadd_rn(acc, sh[u * 32]);
        g[u * R] = acc;
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// The water level by bisection, several steps per round: the 2^S - 1 levels the next S steps can
// probe (a binary tree: a step that fits the budget raises `low`, else it lowers `high`) are evaluated
// together, then the path through them is taken. Each evaluation is, per request, the searchsorted of
// allocation.py:146-150 -- the first j with prefix[j] + offset >= x -- confined to the request's
// results at the round's two ends (the result grows with the level). mm_wide_kernel takes the first
// kMmWideStages * kMmWideSteps steps over the whole GPU; mm_level_kernel, one CTA, the rest, its
// threads running the 2^S - 1 searches of two requests each side by side so their loads overlap.
constexpr int kMmSpec = 3;
constexpr int kMmNodes = (1 << kMmSpec) - 1;
static_assert((kMmBisection - kMmWideStages * kMmWideSteps) % kMmSpec == 0, "whole rounds after the wide steps");
constexpr int kMmLevelThreads = 512;
constexpr int kMmAhead = 2;  // next shares per request staged in shared memory for the leftover blocks
constexpr int kMmFewLeftovers = 64;  // up to this many leftover blocks: argmin per block, no heap

// Shared memory of mm_level_kernel, per request: counts and blocks (kept throughout), then either the
// bisection's state or the leftover heap.
struct MmLevelSmem {
  size_t counts, m, u, base, off, lo, hi, lbs, level, ahead, row, start, bytes;
};

__host__ __device__ inline MmLevelSmem mm_level_smem(int rows) {
  MmLevelSmem l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 15) / 16 * 16;
    return at;
  };
  l.counts = take((size_t)rows * 4);
  l.m = take((size_t)rows * 4);
  l.u = o;  // the union
  l.base = take((size_t)rows * 8);
  l.off = take((size_t)rows * 8);
  l.lo = take((size_t)rows * 4);
  l.hi = take((size_t)rows * 4);
  l.lbs = take((size_t)rows * kMmNodes * 2);
  const size_t bisection_end = o;
  o = l.u;
  l.level = take((size_t)rows * 8);
  l.ahead = take((size_t)rows * 8 * kMmAhead);
  l.row = take((size_t)rows * 4);
  l.start = take((size_t)rows * 4);
  l.bytes = o > bisection_end ? o : bisection_end;
  return l;
}

// Level of node n of a stage's tree whose first step splits [lo, hi] (node n's children: 2n + 1 when
// its level does not fit the budget, so `high` falls to it, and 2n + 2 when it fits and `low` rises to
// it): the midpoints the sequential bisection computes on that path.
__device__ __forceinline__ double mm_tree_level(int n, double lo, double hi) {
  const int depth = 31 - __clz(n + 1);
  for (int d = 0; d < depth; ++d) {
    const double mid = (lo + hi) / 2;
    if (((n + 1) >> (depth - d - 1)) & 1) lo = mid; else hi = mid;  // an even child: the level fit
  }
  return (lo + hi) / 2;
}

// The bisection through the wide stages [0, stages): low and high after their steps, and the wide
// levels (indices into the stages' nodes) of the last step that fit and the last that did not (-1:
// none).
struct MmWalk {
  double low, high;
  int lo_node, hi_node;
};

__device__ __forceinline__ MmWalk mm_wide_walk(const MmState* st, int stages) {
  MmWalk w{0.0, 1.0, -1, -1};
  const long long free_ = __ldcg(&st->free_);
  for (int g = 0; g < stages; ++g) {
    for (int d = 0, n = 0; d < kMmWideSteps; ++d) {
      const double level = (w.low + w.high) / 2;
      if (__ldcg(&st->wide[g * kMmWideNodes + n]) <= free_) {
        w.low = level, w.lo_node = g * kMmWideNodes + n, n = 2 * n + 2;
      } else {
        w.high = level, w.hi_node = g * kMmWideNodes + n, n = 2 * n + 1;
      }
    }
  }
  return w;
}

constexpr int kMmWideThreads = 256;

// Stage g, grid (requests / kMmWideThreads, kMmWideNodes): thread (r, n) walks the earlier stages'
// decisions, runs request r's search at node n's level between its results at the walk's two ends,
// keeps the result for the later stages and mm_level_kernel and adds the request's blocks to the
// node's total.
__global__ void __launch_bounds__(kMmWideThreads) mm_wide_kernel(const MmParams p, int g) {
  chain_release();
  chain_wait();  // the running sums, the earlier stages' totals
  __shared__ long long s_part[kMmWideThreads / 32];
  if (p.state->mode != kMmSelect) return;
  const int n = blockIdx.y, r = blockIdx.x * kMmWideThreads + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const MmWalk w = mm_wide_walk(p.state, g);
  const double level = mm_tree_level(n, w.low, w.high);
  long long take = 0;
  const int m = r < p.rows ? p.row_m[r] : -1;
  if (m >= 0) {
    const double base = p.base[r], off = 2.0 * (double)p.req[r];
    const double x = (level - base) - 1e-12 + off;
    int lo = w.lo_node >= 0 ? p.wide_lbs[(size_t)w.lo_node * p.rows + r] : 0;
    int hi = w.hi_node >= 0 ? p.wide_lbs[(size_t)w.hi_node * p.rows + r] : m;
    while (lo < hi) {  // the first j with prefix[j] + off >= x
      const int md = (lo + hi) >> 1;
      if (p.prefix[(int64_t)md * p.rows + r] + off < x) lo = md + 1; else hi = md;
    }
    p.wide_lbs[(size_t)(g * kMmWideNodes + n) * p.rows + r] = (uint16_t)lo;
    take = level - base <= 1e-12 ? 0 : (lo + 1 < m ? lo + 1 : m);
  }
  for (int o = 16; o > 0; o >>= 1) take += __shfl_xor_sync(kFullMask, take, o);
  if (lane == 0) s_part[warp] = take;
  __syncthreads();
  if (threadIdx.x == 0) {
    long long t = 0;
    for (int k = 0; k < kMmWideThreads / 32; ++k) t += s_part[k];
    atomicAdd(reinterpret_cast<unsigned long long*>(&p.state->wide[g * kMmWideNodes + n]), (unsigned long long)t);
  }
}

// One CTA: the water level, the leftover blocks and the quotas.
__global__ void __launch_bounds__(kMmLevelThreads) mm_level_kernel(const MmParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  extern __shared__ __align__(16) unsigned char lv_smem[];
  const MmLevelSmem L = mm_level_smem(p.rows);
  int* counts = reinterpret_cast<int*>(lv_smem + L.counts);
  int* s_m = reinterpret_cast<int*>(lv_smem + L.m);
  double* s_base = reinterpret_cast<double*>(lv_smem + L.base);
  double* s_off = reinterpret_cast<double*>(lv_smem + L.off);
  int* s_lo = reinterpret_cast<int*>(lv_smem + L.lo);
  int* s_hi = reinterpret_cast<int*>(lv_smem + L.hi);
  uint16_t* s_lbs = reinterpret_cast<uint16_t*>(lv_smem + L.lbs);
  double* h_level = reinterpret_cast<double*>(lv_smem + L.level);
  double* ahead = reinterpret_cast<double*>(lv_smem + L.ahead);  // [rows][kMmAhead]
  int* h_row = reinterpret_cast<int*>(lv_smem + L.row);
  int* start = reinterpret_cast<int*>(lv_smem + L.start);
  __shared__ long long s_red[kMmLevelThreads / 32][kMmNodes];
  __shared__ long long s_tot[kMmNodes];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const MmState* st = p.state;
  const int mode = st->mode;
  if (mode != kMmSelect) {
    for (int r = tid; r < p.rows; r += kMmLevelThreads) {
      const int m = p.row_m[r];
      p.quota[r] = m < 0 ? -1 : (mode == kMmAll ? m : 0);
    }
    return;
  }
  const long long free_ = st->free_;
  const int64_t R = p.rows;
  for (int r = tid; r < p.rows; r += kMmLevelThreads) {
    const int m = p.row_m[r];
    s_m[r] = m;
    s_base[r] = p.base[r];
    s_off[r] = 2.0 * (double)p.req[r];
  }
  // the wide stages' steps: the path through their levels, and each request's search results at the
  // path's two ends
  const MmWalk walk = mm_wide_walk(st, kMmWideStages);
  double low = walk.low, high = walk.high;
  for (int r = tid; r < p.rows; r += kMmLevelThreads) {
    const int m = s_m[r];
    s_lo[r] = m >= 0 && walk.lo_node >= 0 ? p.wide_lbs[(size_t)walk.lo_node * p.rows + r] : 0;
    s_hi[r] = m >= 0 && walk.hi_node >= 0 ? p.wide_lbs[(size_t)walk.hi_node * p.rows + r] : (m > 0 ? m : 0);
  }
  __syncthreads();
  for (int round = 0; round < (kMmBisection - kMmWideStages * kMmWideSteps) / kMmSpec; ++round) {
    // the levels of the tree: node n's children are 2n + 1 (its level did not fit: high = mid) and
    // 2n + 2 (it fit: low = mid); every thread builds the same tree
    double lo_v[kMmNodes], hi_v[kMmNodes], mid[kMmNodes];
    lo_v[0] = low, hi_v[0] = high;
#pragma unroll
    for (int n = 0; n < kMmNodes; ++n) {
      mid[n] = (lo_v[n] + hi_v[n]) / 2;
      if (2 * n + 2 < kMmNodes) {
        lo_v[2 * n + 1] = lo_v[n], hi_v[2 * n + 1] = mid[n];
        lo_v[2 * n + 2] = mid[n], hi_v[2 * n + 2] = hi_v[n];
      }
    }
    int sum[kMmNodes];  // at most 4096 requests x 8192 blocks
#pragma unroll
    for (int n = 0; n < kMmNodes; ++n) sum[n] = 0;
    // two requests a thread, r0 and r0 + kMmLevelThreads, their 2 x kMmNodes searches side by side
    for (int r0 = tid; r0 < p.rows; r0 += 2 * kMmLevelThreads) {
      int rq[2], mq[2];
      double base[2], off[2];
      uint32_t lh[2][kMmNodes];  // the search's bounds: lo | hi << 16 (both at most 8192)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int r = r0 + q * kMmLevelThreads;
        rq[q] = r < p.rows ? r : r0;
        mq[q] = r < p.rows ? s_m[r] : -1;
        base[q] = s_base[rq[q]], off[q] = s_off[rq[q]];
        const uint32_t b = mq[q] >= 0 ? (uint32_t)s_lo[rq[q]] | ((uint32_t)s_hi[rq[q]] << 16) : 0u;
#pragma unroll
        for (int n = 0; n < kMmNodes; ++n) lh[q][n] = b;
      }
      for (;;) {  // one load per open search per step
        // (the search targets are recomputed each step rather than held: 14 more doubles would spill)
        asm volatile("" : "+d"(base[0]), "+d"(base[1]), "+d"(off[0]), "+d"(off[1]));
        double v[2][kMmNodes];
        bool active = false;
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int n = 0; n < kMmNodes; ++n) {
            const int lo = (int)(lh[q][n] & 0xffffu), hi = (int)(lh[q][n] >> 16);
            if (lo < hi) v[q][n] = p.prefix[(int64_t)((lo + hi) >> 1) * R + rq[q]], active = true;
          }
        if (!active) break;
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int n = 0; n < kMmNodes; ++n) {
            const int lo = (int)(lh[q][n] & 0xffffu), hi = (int)(lh[q][n] >> 16);
            if (lo < hi) {  // searchsorted's test, prefix + 2 r' < level - base - 1e-12 + 2 r'
              const int md = (lo + hi) >> 1;
              const double x = (mid[n] - base[q]) - 1e-12 + off[q];
              lh[q][n] = v[q][n] + off[q] < x ? (uint32_t)(md + 1) | ((uint32_t)hi << 16)
                                              : (uint32_t)lo | ((uint32_t)md << 16);
            }
          }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (mq[q] < 0) continue;
        const int r = rq[q], m = mq[q];
#pragma unroll
        for (int n = 0; n < kMmNodes; ++n) {
          const int lo = (int)(lh[q][n] & 0xffffu);
          s_lbs[(size_t)r * kMmNodes + n] = (uint16_t)lo;
          const double need = mid[n] - base[q];
          sum[n] += need <= 1e-12 ? 0 : (lo + 1 < m ? lo + 1 : m);
        }
      }
    }
#pragma unroll
    for (int n = 0; n < kMmNodes; ++n)
      for (int off = 16; off > 0; off >>= 1) sum[n] += __shfl_xor_sync(kFullMask, sum[n], off);
    if (lane == 0)
#pragma unroll
      for (int n = 0; n < kMmNodes; ++n) s_red[warp][n] = sum[n];
    __syncthreads();
    if (tid < kMmNodes) {
      long long t = 0;
      for (int w = 0; w < kMmLevelThreads / 32; ++w) t += s_red[w][tid];
      s_tot[tid] = t;
    }
    __syncthreads();
    int n = 0, lo_node = -1, hi_node = -1;
    for (int d = 0; d < kMmSpec; ++d) {
      double level = mid[0];  // mid[n] without indexing a register array at run time
#pragma unroll
      for (int k = 1; k < kMmNodes; ++k) level = k == n ? mid[k] : level;
      if (s_tot[n] <= free_) {
        low = level, lo_node = n, n = 2 * n + 2;
      } else {
        high = level, hi_node = n, n = 2 * n + 1;
      }
    }
    for (int r = tid; r < p.rows; r += kMmLevelThreads) {
      if (s_m[r] < 0) continue;
      if (lo_node >= 0) s_lo[r] = s_lbs[(size_t)r * kMmNodes + lo_node];
      if (hi_node >= 0) s_hi[r] = s_lbs[(size_t)r * kMmNodes + hi_node];
    }
    // (the next bisection round's first barrier comes after every thread's last read of s_tot and s_lbs here)
  }
  long long used = 0;
  for (int r = tid; r < p.rows; r += kMmLevelThreads) {  // the blocks each request takes at `low`
    const int m = s_m[r];
    int c = 0;
    if (m >= 0) {
      const double need = low - s_base[r];
      c = need <= 1e-12 ? 0 : (s_lo[r] + 1 < m ? s_lo[r] + 1 : m);
    }
    counts[r] = c;
    used += c;
  }
  for (int off = 16; off > 0; off >>= 1) used += __shfl_xor_sync(kFullMask, used, off);
  if (lane == 0) s_red[warp][0] = used;
  __syncthreads();  // the bisection's state is dead from here: the heap takes its place
  // each request's retained share (its heap entry) and the shares of its next blocks, loaded in parallel
  for (int r = tid; r < p.rows; r += kMmLevelThreads) {
    const int m = s_m[r], c = counts[r];
    h_level[r] = m < 0 ? 0.0 : p.base[r] + (c ? p.prefix[(int64_t)(c - 1) * R + r] : 0.0);
    start[r] = c;
#pragma unroll
    for (int a = 0; a < kMmAhead; ++a) ahead[(size_t)r * kMmAhead + a] = c + a < m ? p.sorted[(int64_t)(c + a) * R + r] : 0.0;
  }
  __syncthreads();
  long long leftover = free_;
  for (int w = 0; w < kMmLevelThreads / 32; ++w) leftover -= s_red[w][0];
  if (leftover > 0 && leftover <= kMmFewLeftovers) {
    // a few blocks left over: each goes to the request of lowest (retained share, index) that can take
    // one, found by a block-wide argmin (heappop of allocation.py:160-166, without building the heap)
    __shared__ double s_best_level[kMmLevelThreads / 32];
    __shared__ int s_best_row[kMmLevelThreads / 32];
    for (long long k = 0; k < leftover; ++k) {
      double best = 0.0;
      int best_row = -1;
      for (int r = tid; r < p.rows; r += kMmLevelThreads) {
        const int m = s_m[r];
        if (m < 0 || counts[r] >= m) continue;
        if (best_row < 0 || h_level[r] < best) best = h_level[r], best_row = r;  // rows ascend: ties keep the lower
      }
      for (int off = 16; off > 0; off >>= 1) {
        const double ol = __shfl_xor_sync(kFullMask, best, off);
        const int orow = __shfl_xor_sync(kFullMask, best_row, off);
        if (orow >= 0 && (best_row < 0 || ol < best || (ol == best && orow < best_row))) best = ol, best_row = orow;
      }
      if (lane == 0) s_best_level[warp] = best, s_best_row[warp] = best_row;
      __syncthreads();
      if (tid == 0) {
        for (int w = 1; w < kMmLevelThreads / 32; ++w) {
          const double ol = s_best_level[w];
          const int orow = s_best_row[w];
          if (orow >= 0 && (best_row < 0 || ol < best || (ol == best && orow < best_row))) best = ol, best_row = orow;
        }
        if (best_row >= 0) {
          const int c = counts[best_row]++;
          const int a = c - start[best_row];
          h_level[best_row] = best + (a < kMmAhead ? ahead[(size_t)best_row * kMmAhead + a]
                                                   : p.sorted[(int64_t)c * R + best_row]);
        }
      }
      __syncthreads();
    }
  } else if (leftover > 0 && tid == 0) {
    // the requests that can still take a block, keyed by (retained share, request); a min-heap
    auto less = [&](int a, int b) {
      return h_level[a] < h_level[b] || (h_level[a] == h_level[b] && h_row[a] < h_row[b]);
    };
    auto swap = [&](int a, int b) {
      const double l = h_level[a];
      const int row = h_row[a];
      h_level[a] = h_level[b], h_row[a] = h_row[b], h_level[b] = l, h_row[b] = row;
    };
    auto sift_down = [&](int i, int size) {
      for (;;) {
        const int a = 2 * i + 1, b = a + 1;
        int best = i;
        if (a < size && less(a, best)) best = a;
        if (b < size && less(b, best)) best = b;
        if (best == i) return;
        swap(i, best);
        i = best;
      }
    };
    int size = 0;  // the requests that can take a block, in order (an in-place compaction)
    for (int r = 0; r < p.rows; ++r) {
      const int m = s_m[r];
      if (m < 0 || counts[r] >= m) continue;
      h_level[size] = h_level[r];
      h_row[size] = r;
      ++size;
    }
    for (int i = size / 2 - 1; i >= 0; --i) sift_down(i, size);
    while (leftover > 0 && size > 0) {
      const int r = h_row[0];
      const double level = h_level[0];
      const int c = counts[r]++;
      --leftover;
      if (counts[r] < s_m[r]) {  // back with its next block's share added (heappop then heappush)
        const int a = c - start[r];
        h_level[0] = level + (a < kMmAhead ? ahead[(size_t)r * kMmAhead + a] : p.sorted[(int64_t)c * p.rows + r]);
        sift_down(0, size);
      } else {
        --size;
        if (size > 0) {
          h_level[0] = h_level[size], h_row[0] = h_row[size];
          sift_down(0, size);
        }
      }
    }
  }
  __syncthreads();
  for (int r = tid; r < p.rows; r += kMmLevelThreads) p.quota[r] = s_m[r] < 0 ? -1 : counts[r];
}

}  // namespace ekv

using namespace ekv;

extern "C" size_t ekv_allocate_maxmin_workspace_bytes(int rows, int width) {
  if (rows <= 0 || width <= 0) return 0;
  return mm_layout(rows, width).bytes;
}

template <typename S>
static int allocate_maxmin(const S* scores, int64_t score_stride, const int32_t* score_rows,
                           const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                           int cap_above_blocks, double budget_fraction, int64_t budget, int rows, int width,
                           int32_t* quota, void* workspace, size_t workspace_bytes, void* stream,
                           bool presummed = false, const long long* budget_add = nullptr) {
  clear_error();
  if (!scores || !row_blocks || !quota) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0) return fail(EKV_EINVAL, "rows and width must be positive");
  if (width > kMmMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d", width, kMmMaxWidth);
  if (rows > kMmMaxRows) return fail(EKV_ENOTSUP, "rows %d > %d", rows, kMmMaxRows);
  if (score_stride < width) return fail(EKV_EINVAL, "score_stride %lld < width %d", (long long)score_stride, width);
  if (recent_blocks < -1 || cap_above_blocks < -1) return fail(EKV_EINVAL, "invalid controller settings");
  if (budget < 0 && !(budget_fraction > 0.0 && budget_fraction <= 1.0))
    return fail(EKV_EINVAL, "the budget fraction must be in (0, 1]");
  const MmLayout l = mm_layout(rows, width);
  if (!workspace || workspace_bytes < l.bytes)
    return fail(EKV_ERANGE, "the maxmin workspace holds %zu bytes, the call needs %zu", workspace_bytes, l.bytes);
  if ((uintptr_t)workspace & 255) return fail(EKV_EINVAL, "the maxmin workspace must be 256-byte aligned");
  uint8_t* base = static_cast<uint8_t*>(workspace);
  MmParams p{};
  p.scores = scores; p.score_s0 = score_stride; p.score_rows = score_rows; p.row_blocks = row_blocks;
  p.measured = measured_blocks;
  p.recent = recent_blocks; p.cap = cap_above_blocks; p.fraction = budget_fraction; p.budget = (long long)budget;
  p.rows = rows; p.width = width; p.quota = quota;
  p.presummed = presummed; p.budget_add = budget_add;
  p.state = reinterpret_cast<MmState*>(base + l.state);
  p.base = reinterpret_cast<double*>(base + l.base);
  p.row_m = reinterpret_cast<int*>(base + l.row_m);
  p.req = reinterpret_cast<int*>(base + l.req);
  p.sorted = reinterpret_cast<double*>(base + l.sorted);
  p.wide_lbs = reinterpret_cast<uint16_t*>(base + l.wide_lbs);
  p.prefix = reinterpret_cast<double*>(base + l.prefix);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(base + l.state, 0, sizeof(MmState), s) != cudaSuccess)
    return check_launch("cudaMemsetAsync(maxmin state)");
  const size_t prep_smem = mm_prep_smem<S>(width);
  const size_t level_smem = mm_level_smem(rows).bytes;
  int device = 0;
  {
    const int dev_rc = current_device(&device);
    if (dev_rc != EKV_OK) return dev_rc;
  }
  static size_t prep_set[kMaxDevices] = {}, level_set[kMaxDevices] = {};
  static bool cumsum_set[kMaxDevices] = {};
  if (!cumsum_set[device]) {
    if (cudaFuncSetAttribute(mm_cumsum_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kCsSmem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(mm_cumsum_kernel)");
    cumsum_set[device] = true;
  }
  if (prep_set[device] < prep_smem) {
    if (cudaFuncSetAttribute(mm_prep_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(mm_prep_kernel)");
    prep_set[device] = prep_smem;
  }
  if (level_set[device] < level_smem) {
    if (cudaFuncSetAttribute(mm_level_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)level_smem) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(mm_level_kernel)");
    level_set[device] = level_smem;
  }
  launch_chained(mm_prep_kernel<S>, dim3(rows), dim3(kMmThreads), prep_smem, s, p);
  int rc = check_launch("mm_prep_kernel");
  if (rc != EKV_OK) return rc;
  launch_chained(mm_cumsum_kernel, dim3((rows + 31) / 32), dim3(32), kCsSmem, s, p);
  if ((rc = check_launch("mm_cumsum_kernel")) != EKV_OK) return rc;
  for (int g = 0; g < kMmWideStages; ++g) {
    launch_chained(mm_wide_kernel, dim3((rows + kMmWideThreads - 1) / kMmWideThreads, kMmWideNodes),
                   dim3(kMmWideThreads), 0, s, p, g);
    if ((rc = check_launch("mm_wide_kernel")) != EKV_OK) return rc;
  }
  launch_chained(mm_level_kernel, dim3(1), dim3(kMmLevelThreads), level_smem, s, p);
  return check_launch("mm_level_kernel");
}

namespace ekv {

// The maxmin quotas of presummed float64 rows whose pins are block 0 and [measured[r], n).
int presummed_maxmin(const double* shares, int64_t share_s0, const int32_t* row_blocks, const int32_t* measured,
                     long long budget, const long long* budget_add, int rows, int width, int32_t* quota,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return allocate_maxmin<double>(shares, share_s0, nullptr, row_blocks, measured, -1, -1, 0.0, budget, rows, width,
                                 quota, workspace, workspace_bytes, stream, true, budget_add);
}

}  // namespace ekv

extern "C" int ekv_allocate_maxmin(const float* scores, int64_t score_stride, const int32_t* row_blocks,
                                   const int32_t* measured_blocks, int recent_blocks, int cap_above_blocks,
                                   double budget_fraction, int64_t budget, int rows, int width, int32_t* quota,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  return allocate_maxmin<float>(scores, score_stride, nullptr, row_blocks, measured_blocks, recent_blocks,
                                cap_above_blocks, budget_fraction, budget, rows, width, quota, workspace,
                                workspace_bytes, stream);
}

extern "C" int ekv_allocate_maxmin_f64(const double* scores, int64_t score_stride, const int32_t* score_rows,
                                       const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                                       int cap_above_blocks, double budget_fraction, int64_t budget, int rows,
                                       int width, int32_t* quota, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  return allocate_maxmin<double>(scores, score_stride, score_rows, row_blocks, measured_blocks, recent_blocks,
                                 cap_above_blocks, budget_fraction, budget, rows, width, quota, workspace,
                                 workspace_bytes, stream);
}
