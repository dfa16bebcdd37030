// The decide-and-enforce half of the path on the device: per-row budgets (quota kernel), the
// per-row keep decision by exact top-k selection, and the stable compaction of the block table
// into the view the attention kernel reads.
//
// The view kernel runs one CTA per row. Ranking mode turns max(score, 0) (float32, NaN as 0) into
// an order-preserving uint32 key and finds the quota-th largest key of the row's unpinned blocks by
// an MSB radix select (digits of 11, 11 and 9 bits over a 2048-bin shared-memory histogram; float64
// gain keys take six digits), while the table row is copied in. Keys above the threshold are
// kept; of the keys equal to it, the first (uniform: older blocks first, allocation.py:89) or last
// (sum: newer blocks first, allocation.py:107-113) ones fill the quota, ranked by the equal keys of
// the warps before and a running count within each warp's run of positions. The warps' counts of
// kept blocks place kept blocks first and the others after them, both in their original order: the
// stable partition of compact_block_table (runtime/block_view.py:52).
#include "ekv_common.cuh"
#include "pairwise.cuh"
#include "pins.cuh"
#include "sum_state.cuh"

namespace ekv {

// ---- quotas ------------------------------------------------------------------------------------

struct QuotaParams {
  const int32_t* row_blocks;
  const int32_t* measured;
  int recent, cap;
  double fraction;
  long long budget;  // >= 0: the shared budget as given; < 0: from `fraction`
  const double* row_fraction;
  int rows, width;  // width > 0: a request holds min(row_blocks, width) blocks
  int32_t* quota;
  const long long* budget_add;  // may be NULL: blocks added on the device to a budget given as a count
};

// The blocks of a request of row_blocks blocks: its length, at most the row width (controller.py:414).
__device__ __forceinline__ int request_blocks(int n, int width) { return width > 0 && n > width ? width : n; }

constexpr int kQuotaThreads = 1024;
constexpr int kQuotaMaxRows = 8192;  // rows of one shared budget (shared-memory remainders)

__device__ __forceinline__ long long block_sum_ll(long long v, long long* scratch) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  long long total = 0;
  for (int w = 0; w < kQuotaThreads / 32; ++w) total += scratch[w];
  return total;
}

__global__ void __launch_bounds__(kQuotaThreads) quota_kernel(const QuotaParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  extern __shared__ double s_rem[];  // [rows] remainders of the shared-budget split
  __shared__ long long s_red[kQuotaThreads / 32];
  const int R = p.rows;
  if (p.row_fraction != nullptr) {
    // Every row is its own allocate() call (allocation.py:55-76) with its own budget.
    for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
      int n = p.row_blocks[r];
      if (n <= p.cap || n <= 0) {
        p.quota[r] = -1;
        continue;
      }
      n = request_blocks(n, p.width);
      const int ps = pin_start(n, p.recent, p.measured, r);
      const int pins = pin_count(n, ps);
      const int open = ps > 1 ? ps - 1 : 0;
      long long budget = (long long)ceil(p.row_fraction[r] * (double)n);
      if (budget < pins) budget = pins;
      p.quota[r] = budget >= n ? open : (int)(budget - pins);
    }
    return;
  }
  // One budget for all measured rows (controller.py:398-451), split by _uniform (allocation.py:79-91).
  long long total = 0, floor_ = 0, total_open = 0;
  for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
    int n = p.row_blocks[r];
    if (n <= p.cap || n <= 0) continue;
    n = request_blocks(n, p.width);
    const int ps = pin_start(n, p.recent, p.measured, r);
    total += n;
    floor_ += pin_count(n, ps);
    total_open += ps > 1 ? ps - 1 : 0;
  }
  total = block_sum_ll(total, s_red);
  floor_ = block_sum_ll(floor_, s_red);
  total_open = block_sum_ll(total_open, s_red);
  long long budget = p.budget;
  if (budget < 0) {
    budget = (long long)ceil(p.fraction * (double)total);
    if (budget < floor_) budget = floor_;
  } else if (p.budget_add != nullptr) {
    budget += *p.budget_add;
  }
  const bool keep_all = budget >= total;
  const long long free_ = budget - floor_;
  long long assigned = 0;
  for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
    int n = p.row_blocks[r];
    s_rem[r] = -1.0;  // not a request
    if (n <= p.cap || n <= 0) {
      p.quota[r] = -1;
      continue;
    }
    n = request_blocks(n, p.width);
    const int ps = pin_start(n, p.recent, p.measured, r);
    const int open = ps > 1 ? ps - 1 : 0;
    if (keep_all) {
      p.quota[r] = open;
      continue;
    }
    // exact = free * len(open) / total, as Python's int / int: one correctly rounded division
    const double exact = total_open ? (double)(free_ * open) / (double)total_open : 0.0;
    const int q = (int)exact;
    p.quota[r] = q;
    s_rem[r] = exact - (double)q;
    assigned += q;
  }
  if (keep_all) return;
  assigned = block_sum_ll(assigned, s_red);  // (its __syncthreads also publishes s_rem)
  const long long extra = free_ - assigned;
  if (extra <= 0) return;
  // The `extra` largest remainders get one more block; equal remainders go to the earlier row
  // (allocation.py:85). The remainders are non-negative doubles, so their bits order them: a radix
  // select over 63-bit keys (digits of 11 bits, the last of 8) finds the extra-th largest.
  __shared__ int s_hist[2048];
  __shared__ int s_pick[3];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long prefix = 0, mask = 0;
  long long k = extra;
  for (int pass = 0; pass < 6; ++pass) {
    const int shift = pass < 5 ? 52 - 11 * pass : 0;
    const unsigned long long dmask = pass < 5 ? 2047ull : 255ull;
    for (int i = threadIdx.x; i < 2048; i += kQuotaThreads) s_hist[i] = 0;
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
      if (s_rem[r] < 0.0) continue;  // not a request
      const unsigned long long key = (unsigned long long)__double_as_longlong(s_rem[r]);
      if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & dmask], 1);
    }
    __syncthreads();
    // thread t owns bins 2t and 2t + 1; the count of keys in the bins above it, from the top
    const int h0 = s_hist[2 * threadIdx.x], h1 = s_hist[2 * threadIdx.x + 1];
    const long long sum = (long long)h0 + h1;
    long long above = sum;
    for (int off = 1; off < 32; off <<= 1) {
      const long long v = __shfl_down_sync(kFullMask, above, off);
      if (lane + off < 32) above += v;
    }
    __syncthreads();
    if (lane == 0) s_red[warp] = above;
    __syncthreads();
    long long gt = above - sum;
    for (int w2 = warp + 1; w2 < kQuotaThreads / 32; ++w2) gt += s_red[w2];
    if (gt < k && gt + h1 >= k) s_pick[0] = 2 * threadIdx.x + 1, s_pick[1] = (int)gt, s_pick[2] = h1;
    gt += h1;
    if (gt < k && gt + h0 >= k) s_pick[0] = 2 * threadIdx.x, s_pick[1] = (int)gt, s_pick[2] = h0;
    __syncthreads();
    k -= s_pick[1];
    prefix |= (unsigned long long)s_pick[0] << shift;
    mask |= dmask << shift;
    const bool done = s_pick[2] == k;  // every key with the prefix is taken
    __syncthreads();
    if (done) break;
  }
  // keys above the threshold get one more; of the keys equal to it, the first k in row order
  int carry = 0;
  for (int base = 0; base < R; base += kQuotaThreads) {
    const int r = base + threadIdx.x;
    bool tie = false, up = false;
    if (r < R && s_rem[r] >= 0.0) {
      const unsigned long long key = (unsigned long long)__double_as_longlong(s_rem[r]) & mask;
      up = key > prefix;
      tie = key == prefix;
    }
    long long tie_rank = 0;
    {
      int total = 0;
      tie_rank = carry + block_exclusive_scan<kQuotaThreads>(tie ? 1 : 0, reinterpret_cast<int*>(s_red), &total);
      carry += total;
    }
    if (up || (tie && tie_rank < k)) p.quota[r] += 1;
  }
}

// ---- view ----------------------------------------------------------------------------------------

struct ViewParams {
  const int32_t* table;
  int64_t table_s0;
  const int32_t* seq_lens;
  const int32_t* row_blocks;
  const int32_t* quota;
  const int32_t* measured;
  int recent;
  const void* scores;          // float [rows][score_s0] (view_kernel<uint32_t>) or double (<unsigned long long>)
  int64_t score_s0;
  const int32_t* score_rows;   // may be NULL: row r ranks scores row score_rows[r] instead of r
  const double* weights;       // may be NULL (1.0): the request weights of the float64 gain keys
  int policy;
  const uint8_t* keep;
  int64_t keep_s0;
  const uint8_t* full_rows;
  const uint8_t* released;
  int64_t released_s0;
  int rows, width, block_size;
  int32_t* view;
  int64_t view_s0;
  int32_t* view_lens;
  uint8_t* mask_out;
  int64_t mask_s0;
  // the read counters of a decode view (ekv_decode_view): full_rows then carries packed row flags
  long long* counts;
  int expired;
  // per-row budgets computed in the kernel (ekv_view_build_fractions) instead of read from quota
  const double* row_fraction;
  int cap;
  // float64 rows that already hold each request's shares (the pinned allocation): ranked as they are
  bool presummed;
  // threshold mode (launch_sum_view): the keep decision of a shared `sum` budget's select, from its state, gain
  // keys [rows][width] and per-row blocks, pin starts and taken ties; no ranking
  const SumState* sum_state;
  const unsigned long long* sum_keys;
  const int32_t* sum_row_n;
  const int32_t* sum_row_ps;
  const int32_t* sum_row_at;
};

// Row flags of ekv_decode_view (full_rows): the row reads every block / decodes / is audited.
constexpr uint8_t kRowFull = 1, kRowDecoding = 2, kRowAudited = 4;

constexpr int kViewThreads = 512;
constexpr int kViewWarps = kViewThreads / 32;
constexpr int kViewMaxWidth = 16384;               // rows staged in shared memory: 8 bytes per position
constexpr int kViewSeg = 128;                      // positions of a segment: four ballots of 32 positions
constexpr int kViewMaxSegs = kViewMaxWidth / kViewSeg;  // (each segment's ballots kept in shared memory)
constexpr int kViewBins = 2048;                    // radix-select digits of 11, 11 and 9 bits
static_assert(kViewBins == 4 * kViewThreads, "each thread owns four histogram bins");

__device__ __forceinline__ uint32_t share_key(float x) {
  // max(x, 0) with NaN as 0; for x >= 0 the IEEE bit pattern is monotone in x and bit 31 is clear
  return x > 0.f ? __float_as_uint(x) : 0u;
}

// n 32-bit words from global to shared memory (16-byte aligned) without blocking the thread.
__device__ __forceinline__ void stage_words(uint32_t* dst, const uint32_t* src, int n) {
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    done = n & ~3;
    for (int i = 4 * threadIdx.x; i < done; i += 4 * kViewThreads) cp_async16(dst + i, src + i);
  }
  for (int i = done + threadIdx.x; i < n; i += kViewThreads) cp_async4(dst + i, src + i);
}

// dst[i] = src[i] for i in [lo, hi), 16 bytes at a time where both rows allow it.
__device__ __forceinline__ void copy_words(int32_t* dst, const int32_t* src, int lo, int hi) {
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0 && (lo & 3) == 0;
  int i = lo;
  if (vec) {
    const int stop = lo + ((hi - lo) & ~3);
    for (int j = lo + 4 * threadIdx.x; j < stop; j += 4 * kViewThreads)
      *reinterpret_cast<int4*>(dst + j) = *reinterpret_cast<const int4*>(src + j);
    i = stop;
  }
  for (int j = i + threadIdx.x; j < hi; j += kViewThreads) dst[j] = src[j];
}


// The per-warp counts c[0..kViewWarps) (written before a barrier): the sum over the warps before this one
// (*before) and over every warp (returned), to every lane.
__device__ __forceinline__ int warp_counts_prefix(const int* c, int* before) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v = lane < kViewWarps ? c[lane] : 0;
  *before = __reduce_add_sync(kFullMask, lane < warp ? v : 0);
  return __reduce_add_sync(kFullMask, v);
}

// The order keys of the ranking. Float32 scores: the bits of max(score, 0), three digits (bits 30-20,
// 19-9, 8-0; bit 31 is always clear). Float64 scores: the bits of the non-negative float64
// weight * share, share = max(score, 0) / total (total: NumPy's pairwise sum of the row's clamped
// scores; 1 / n when it is not positive), the very value the reference ranks (allocation.py:46-52,
// :89, :107), six digits (bits 62-52, 51-41, 40-30, 29-19, 18-8, 7-0).
template <typename K>
struct ViewKey;
template <>
struct ViewKey<uint32_t> {
  static constexpr int kPasses = 3;
  __device__ static void digit(int pass, int& shift, uint32_t& dmask) {
    shift = pass == 0 ? 20 : (pass == 1 ? 9 : 0);
    dmask = pass == 2 ? 511u : 2047u;
  }
  // keys 4g .. 4g + 3 (one 16-byte shared load)
  __device__ static void load4(const uint32_t* keys, int g, uint32_t (&kv)[4]) {
    const uint4 v = reinterpret_cast<const uint4*>(keys)[g];
    kv[0] = v.x, kv[1] = v.y, kv[2] = v.z, kv[3] = v.w;
  }
};
template <>
struct ViewKey<unsigned long long> {
  static constexpr int kPasses = 6;
  __device__ static void digit(int pass, int& shift, unsigned long long& dmask) {
    shift = pass < 5 ? 52 - 11 * pass : 0;
    dmask = pass < 5 ? 2047ull : 255ull;
  }
  __device__ static void load4(const unsigned long long* keys, int g, unsigned long long (&kv)[4]) {
    const ulonglong2 a = reinterpret_cast<const ulonglong2*>(keys)[2 * g];
    const ulonglong2 b = reinterpret_cast<const ulonglong2*>(keys)[2 * g + 1];
    kv[0] = a.x, kv[1] = a.y, kv[2] = b.x, kv[3] = b.y;
  }
};

// The gain key of one block of a float64 row: bits of weight * (max(s, 0) / total) in float64, each
// operation rounded on its own as NumPy rounds it (NaN counts as 0).
__device__ __forceinline__ unsigned long long share_key64(double s, double total, double w, int n) {
  const double c = s > 0.0 ? s : 0.0;
  const double share = total > 0.0 ? __ddiv_rn(c, total) : __ddiv_rn(1.0, (double)(n > 1 ? n : 1));
  const double g = __dmul_rn(w, share);
  return g > 0.0 ? (unsigned long long)__double_as_longlong(g) : 0ull;
}

template <typename K>
__host__ __device__ constexpr size_t view_smem_bytes(int width) {
  // keys (the staged scores, then the keys, then the view row) + the table row (+ the pairwise sum's slots), each
  // padded to whole segments
  return (size_t)((width + kViewSeg - 1) / kViewSeg * kViewSeg) * (sizeof(K) + 4) +
         (sizeof(K) == 8 ? pairwise_bytes(pairwise_slots(width)) : 0);
}

// One CTA per row.
//
// The ranking: the q-th largest key among positions [1, ps) by an MSB radix select over the digits
// of ViewKey<K>. Thread t owns histogram bins [4t, 4t + 4): it reads them for the scan and clears them
// for the next pass in the same step. If the chosen bin holds exactly the keys still wanted, every key
// with that prefix is kept and the select stops early. The equal-key count comes from the last
// histogram, so the scan that ranks equal keys by position runs only when some of them must be dropped.
//
// The layout: only positions [0, min(blocks, width)) can be kept, so those are laid out; the rest of the row,
// never kept, keeps its place (the view there is the table, copied while the row is ranked). The laid-out
// positions form segments of 128 and each warp takes a contiguous run of segments; lane l holds positions
// 128 * s + 32 * k + l (k = 0..3), so a segment's keep flags are four ballots, ballot k covering 32
// consecutive positions. The kept positions before a lane's are the warp's running count plus popcounts of
// the ballots, and one barrier with the warps' counts gives each warp its first place and the row's kept
// total: every store of a ballot's kept ids (and of its dropped ids, placed after all kept ones) is then a
// contiguous run of the view row. With mask_out the flags cover the whole width, as every position's
// committed flag is written; with no view (mask_out only) the kernel ends there.
template <typename K>
__global__ void __launch_bounds__(kViewThreads, sizeof(K) == 4 ? 3 : 2) view_kernel(const ViewParams p) {
  chain_release();
  extern __shared__ __align__(16) unsigned char smem_view[];
  __shared__ __align__(16) int s_hist[kViewBins];
  __shared__ int s_w[kViewWarps + 1];
  __shared__ int s_pick[3];
  __shared__ uint4 s_bits[kViewMaxSegs];  // each segment's four keep ballots
  __shared__ int s_kept[kViewWarps], s_eqw[kViewWarps];  // each warp's kept positions and equal keys
  constexpr bool kWide = sizeof(K) == 8;
  const int r = blockIdx.x;
  const int W = p.width, BS = p.block_size;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w_pad = (W + kViewSeg - 1) / kViewSeg * kViewSeg;
  K* keys = reinterpret_cast<K*>(smem_view);                                       // [w_pad]
  int32_t* trow_s = reinterpret_cast<int32_t*>(smem_view + (size_t)w_pad * sizeof(K));  // [w_pad]: the staged table row

  const bool has_view = p.view != nullptr;
  const int seq = p.seq_lens != nullptr ? p.seq_lens[r] : 0;
  const int blocks = seq > 0 ? (seq + BS - 1) / BS : 0;
  uint8_t* mrow = p.mask_out ? p.mask_out + (int64_t)r * p.mask_s0 : nullptr;
  const int live = mrow != nullptr ? W : (blocks < W ? blocks : W);
  const int n_segs = (live + kViewSeg - 1) / kViewSeg;               // segments flagged
  const int laid = !has_view ? 0 : min((live + 3) & ~3, W);            // positions laid out
  // (address arithmetic only: without a view, laid is 0 and the table is never read)
  const int32_t* trow = reinterpret_cast<const int32_t*>(reinterpret_cast<uintptr_t>(p.table) +
                                                         (uintptr_t)((int64_t)r * p.table_s0 * 4));
  int32_t* vrow = has_view ? p.view + (int64_t)r * p.view_s0 : nullptr;
  const bool sum_mode = p.sum_state != nullptr;
  if (sum_mode) {
    // Threshold mode follows the select's kernels, none of which writes the caller's table or lengths (they
    // were complete before the select's first kernel started): the table row is staged, and past the
    // laid-out positions copied to the view, while those kernels finish.
    stage_words(reinterpret_cast<uint32_t*>(trow_s), reinterpret_cast<const uint32_t*>(trow), laid);
    cp_async_commit();
    if (has_view) copy_words(vrow, trow, laid, W);
  }
  chain_wait();  // what the launch before this one wrote

  // ---- the row's committed mask: pins + selection (ranking mode) or the given mask ---------------
  const bool rank_mode = p.keep == nullptr && !sum_mode;
  int ps = 0, q = 0, open_hi = 1, n_a = 0;  // the selection applies to positions [1, open_hi)
  bool by_threshold = false, newest = false;
  int s_mode = kSumAll, s_istar = 0;
  unsigned long long s_prefix = 0, s_mask = 0;
  bool s_take = false;
  const unsigned long long* s_keys = nullptr;
  if (sum_mode) {
    // a request (n > 0) keeps its unpinned blocks [1, ps) by the threshold; any other row reads in full
    n_a = p.sum_row_n[r];
    ps = p.sum_row_ps[r];
    s_mode = p.sum_state->mode;
    s_prefix = p.sum_state->prefix, s_mask = p.sum_state->mask, s_istar = p.sum_state->istar;
    s_take = p.sum_row_at[r] != 0;
    s_keys = p.sum_keys + (int64_t)r * W;
    if (n_a > 0 && s_mode != kSumAll && ps > 1) open_hi = ps;
  } else if (rank_mode) {
    n_a = p.row_blocks[r];
    const bool request = n_a > p.cap && n_a > 0;
    n_a = n_a < 0 ? 0 : (n_a > W ? W : n_a);
    if (p.row_fraction != nullptr) {
      // the quota of ekv_allocate_quotas for a row that is its own allocate() call, computed here
      q = -1;
      if (request) {
        const int ps0 = pin_start(n_a, p.recent, p.measured, r);
        const int pins = pin_count(n_a, ps0);
        long long budget = (long long)ceil(p.row_fraction[r] * (double)n_a);
        if (budget < pins) budget = pins;
        q = budget >= n_a ? (ps0 > 1 ? ps0 - 1 : 0) : (int)(budget - pins);
      }
    } else {
      q = p.quota[r];
    }
    if (q >= 0 && n_a > 0) {
      ps = pin_start(n_a, p.recent, p.measured, r);
      const int n_open = ps > 1 ? ps - 1 : 0;
      if (q > n_open) q = n_open;
      if (q < n_open) {  // not every open position is selected
        open_hi = ps;
        if (q > 0) {
          if (p.policy == EKV_POLICY_NEWEST) newest = true; else by_threshold = true;
        }
      }
    }
  }
  if (by_threshold) {
    const int64_t srow = p.score_rows != nullptr ? (int64_t)p.score_rows[r] : (int64_t)r;
    if (kWide) {  // every score of the request: the total needs them all
      stage_words(reinterpret_cast<uint32_t*>(keys),
                  reinterpret_cast<const uint32_t*>(static_cast<const double*>(p.scores) + srow * p.score_s0), 2 * n_a);
    } else {
      stage_words(reinterpret_cast<uint32_t*>(keys),
                  reinterpret_cast<const uint32_t*>(static_cast<const float*>(p.scores) + srow * p.score_s0), ps);
    }
    cp_async_commit();
  }
  if (!sum_mode) {
    // the table row lands while the row is ranked; past the laid-out positions nothing is kept, so the view
    // there is the table, copied now
    stage_words(reinterpret_cast<uint32_t*>(trow_s), reinterpret_cast<const uint32_t*>(trow), laid);
    cp_async_commit();
    if (has_view) copy_words(vrow, trow, laid, W);
  }

  K prefix = 0, pmask = 0;
  int k_eq = 0, eq_total = 0;
  if (by_threshold) {
    reinterpret_cast<int4*>(s_hist)[threadIdx.x] = make_int4(0, 0, 0, 0);  // (ordered by the barrier below)
    cp_async_wait<1>();  // the scores have landed (the table row, committed after them, may still be in flight)
    __syncthreads();
    // The keys, and the first digit's histogram as they are written. Positions 0 and from ps on are not
    // keys; they are handled four at a time.
    const int groups = (ps + 3) >> 2;
    int shift0;
    K dmask0;
    ViewKey<K>::digit(0, shift0, dmask0);
    if constexpr (kWide) {
      const double* s_x = reinterpret_cast<const double*>(keys);
      const PairwiseScratch tree = pairwise_scratch(smem_view + (size_t)w_pad * (sizeof(K) + 4), pairwise_slots(W));
      const double total = p.presummed ? 1.0 : block_pairwise_sum<kViewThreads>(tree, n_a, [&](int i) {
        const double s = s_x[i];
        return s > 0.0 ? s : 0.0;
      });
      const double w = p.weights != nullptr ? p.weights[r] : 1.0;
      for (int b = threadIdx.x; b < 4 * groups; b += kViewThreads) {  // in place: each thread its own positions
        const K key = b < ps ? share_key64(s_x[b], total, w, n_a) : 0ull;
        keys[b] = key;
        if (b >= 1 && b < ps) atomicAdd(&s_hist[(int)((key >> shift0) & dmask0)], 1);
      }
    } else {
      uint4* keys4 = reinterpret_cast<uint4*>(keys);
      for (int g = threadIdx.x; g < groups; g += kViewThreads) {
        uint4 v = keys4[g];
        v.x = share_key(__uint_as_float(v.x)), v.y = share_key(__uint_as_float(v.y));
        v.z = share_key(__uint_as_float(v.z)), v.w = share_key(__uint_as_float(v.w));
        keys4[g] = v;
        const uint32_t kv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (4 * g + j >= 1 && 4 * g + j < ps) atomicAdd(&s_hist[(int)((kv[j] >> shift0) & dmask0)], 1);
      }
    }
    int k = q;
#pragma unroll 1
    for (int pass = 0; pass < ViewKey<K>::kPasses; ++pass) {
      int shift;
      K dmask;
      ViewKey<K>::digit(pass, shift, dmask);
      if (pass > 0) {  // (pass 0's histogram was counted as the keys were made)
        for (int g = threadIdx.x; g < groups; g += kViewThreads) {
          K kv[4];
          ViewKey<K>::load4(keys, g, kv);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int b = 4 * g + j;
            const bool in = b >= 1 && b < ps && (kv[j] & pmask) == prefix;
            if (in) atomicAdd(&s_hist[(int)((kv[j] >> shift) & dmask)], 1);
          }
        }
      }
      __syncthreads();
      const int4 h = reinterpret_cast<const int4*>(s_hist)[threadIdx.x];
      reinterpret_cast<int4*>(s_hist)[threadIdx.x] = make_int4(0, 0, 0, 0);
      const int sum = h.x + h.y + h.z + h.w;
      int above = sum;  // keys in bins owned by this lane and the lanes above it in the warp
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_down_sync(kFullMask, above, off);
        if (lane + off < 32) above += v;
      }
      if (lane == 0) s_w[warp] = above;
      __syncthreads();
      // keys in higher bins: the rest of this warp's plus every later warp's (a suffix sum of the warp
      // totals by shuffles: lane j holds the total of warps j .. kViewWarps - 1)
      int later = lane < kViewWarps ? s_w[lane] : 0;
      for (int off = 1; off < kViewWarps; off <<= 1) {
        const int v = __shfl_down_sync(kFullMask, later, off);
        if (lane + off < kViewWarps) later += v;
      }
      later = __shfl_sync(kFullMask, later, (warp + 1) & 31);
      int gt = above - sum + (warp + 1 < kViewWarps ? later : 0);
      const int bin = 4 * threadIdx.x;
      if (gt < k && gt + h.w >= k) s_pick[0] = bin + 3, s_pick[1] = gt, s_pick[2] = h.w;
      gt += h.w;
      if (gt < k && gt + h.z >= k) s_pick[0] = bin + 2, s_pick[1] = gt, s_pick[2] = h.z;
      gt += h.z;
      if (gt < k && gt + h.y >= k) s_pick[0] = bin + 1, s_pick[1] = gt, s_pick[2] = h.y;
      gt += h.y;
      if (gt < k && gt + h.x >= k) s_pick[0] = bin, s_pick[1] = gt, s_pick[2] = h.x;
      __syncthreads();
      k -= s_pick[1];
      prefix |= (K)s_pick[0] << shift;
      pmask |= dmask << shift;
      eq_total = s_pick[2];  // the keys with the chosen prefix
      if (eq_total == k) break;  // all of them are kept: the prefix is the threshold
    }
    k_eq = k;
  }
  const bool ties = eq_total != k_eq;  // only then do keys equal to the threshold need their rank
  const bool older_first = p.policy == EKV_POLICY_UNIFORM;

  // each warp's run of segments
  const int per_warp = (n_segs + kViewWarps - 1) / kViewWarps;
  const int sg_lo = min(warp * per_warp, n_segs), sg_hi = min(sg_lo + per_warp, n_segs);

  // ---- ties: the equal keys of the warps before this one (each equal key's rank, in position order, is
  // that count plus the equal keys before it in this warp's run)
  int eq_run = 0;
  if (ties) {
    int cnt = 0;
    for (int sg = sg_lo; sg < sg_hi; ++sg) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int b = kViewSeg * sg + 32 * k + lane;
        cnt += b >= 1 && b < ps && (keys[b] & pmask) == prefix;
      }
    }
    cnt = __reduce_add_sync(kFullMask, cnt);
    if (lane == 0) s_eqw[warp] = cnt;
    __syncthreads();
    warp_counts_prefix(s_eqw, &eq_run);
  }

  const uint8_t flags = p.full_rows != nullptr ? p.full_rows[r] : 0;
  const bool full = (flags & kRowFull) != 0;
  const uint8_t* krow = rank_mode || sum_mode ? nullptr : p.keep + (int64_t)r * p.keep_s0;
  const uint8_t* rrow = p.released ? p.released + (int64_t)r * p.released_s0 : nullptr;

  // ---- pass 1: the final keep flag of every flagged position, as four ballots per segment -------------
  int kept_mine = 0;
  if (rank_mode && by_threshold && !ties && mrow == nullptr && rrow == nullptr && !full) {
    // the common case: a key at or above the threshold is kept; outside [1, open_hi) every block is. A segment
    // inside [1, min(open_hi, blocks - 1)) needs the key test alone.
    const int inner = min(open_hi, blocks - 1);
    for (int sg = sg_lo; sg < sg_hi; ++sg) {
      const int b0 = kViewSeg * sg + lane;
      uint32_t plane[4];
      if (sg > 0 && kViewSeg * (sg + 1) <= inner) {
#pragma unroll
        for (int k = 0; k < 4; ++k) plane[k] = __ballot_sync(kFullMask, (keys[b0 + 32 * k] & pmask) >= prefix);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int b = b0 + 32 * k;
          const K key = (b >= 1 && b < open_hi) ? keys[b] & pmask : ~(K)0;
          plane[k] = __ballot_sync(kFullMask, (key >= prefix || b == 0 || b == blocks - 1) && b < blocks && b < W);
        }
      }
      if (lane == 0) s_bits[sg] = make_uint4(plane[0], plane[1], plane[2], plane[3]);
      kept_mine += __popc(plane[0]) + __popc(plane[1]) + __popc(plane[2]) + __popc(plane[3]);
    }
  } else if (sum_mode && mrow == nullptr && rrow == nullptr && !full) {
    // the shared `sum` threshold, common case: an unpinned block by its gain key, every other block of the
    // request kept; a segment inside [1, min(open_hi, blocks - 1)) needs the key test alone
    const int inner = min(open_hi, blocks - 1);
    for (int sg = sg_lo; sg < sg_hi; ++sg) {
      const int b0 = kViewSeg * sg + lane;
      uint32_t plane[4];
      if (sg > 0 && kViewSeg * (sg + 1) <= inner) {
        unsigned long long gk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) gk[k] = __ldg(s_keys + b0 + 32 * k);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          plane[k] = __ballot_sync(kFullMask, sum_keeps(s_mode, gk[k] & s_mask, s_prefix, b0 + 32 * k, s_istar, s_take));
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int b = b0 + 32 * k;
          const bool c = b >= 1 && b < open_hi ? sum_keeps(s_mode, __ldg(s_keys + b) & s_mask, s_prefix, b, s_istar, s_take) : true;
          plane[k] = __ballot_sync(kFullMask, (c || b == 0 || b == blocks - 1) && b < blocks && b < W);
        }
      }
      if (lane == 0) s_bits[sg] = make_uint4(plane[0], plane[1], plane[2], plane[3]);
      kept_mine += __popc(plane[0]) + __popc(plane[1]) + __popc(plane[2]) + __popc(plane[3]);
    }
  } else {
    for (int sg = sg_lo; sg < sg_hi; ++sg) {
      const int b0 = kViewSeg * sg + lane;
      uint32_t plane[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int b = b0 + 32 * k;
        const K kv = by_threshold && b < ps ? keys[b] & pmask : (K)0;
        bool c = b < W;  // the committed mask at b
        if (sum_mode) {
          if (b >= 1 && b < open_hi) c = sum_keeps(s_mode, __ldg(s_keys + b) & s_mask, s_prefix, b, s_istar, s_take);
        } else if (!rank_mode) {
          c = b < W && krow[b] != 0;
        } else if (b >= 1 && b < open_hi) {
          if (newest) {
            c = b >= ps - q;
          } else if (by_threshold) {
            c = kv > prefix || (kv == prefix && !ties);  // every equal key is kept unless too many
          } else {
            c = false;  // nothing selected
          }
        }
        if (ties) {
          // an equal key's rank among the equal keys in position order: those before this ballot, then the
          // lanes below
          const bool eq = b >= 1 && b < ps && kv == prefix;
          const uint32_t eq_bits = __ballot_sync(kFullMask, eq);
          const int below = eq_run + __popc(eq_bits & lanes_below());
          if (eq) c = older_first ? below < k_eq : (eq_total - below - 1) < k_eq;
          eq_run += __popc(eq_bits);
        }
        const bool in_row = b < W;
        if (mrow != nullptr && in_row) mrow[b] = c;
        bool keep = c || full;
        if (rrow != nullptr && in_row && rrow[b]) keep = false;  // a released block is never read (block_view.py:280-281)
        keep = (keep || b == 0 || b == blocks - 1) && b < blocks && in_row;
        plane[k] = __ballot_sync(kFullMask, keep);
      }
      if (lane == 0) s_bits[sg] = make_uint4(plane[0], plane[1], plane[2], plane[3]);
      kept_mine += __popc(plane[0]) + __popc(plane[1]) + __popc(plane[2]) + __popc(plane[3]);
    }
  }
  if (lane == 0) s_kept[warp] = kept_mine;
  cp_async_wait<0>();
  __syncthreads();  // the warps' counts are in, the table row has landed and every key read has ended
  int before = 0;  // kept positions before this warp's first
  const int kept_total = warp_counts_prefix(s_kept, &before);

  // ---- pass 2: kept ids first, then the others, both in position order -------------------------------
  for (int sg = sg_lo; sg < sg_hi && kViewSeg * sg < laid; ++sg) {
    const uint4 pl = s_bits[sg];
    const uint32_t plane[4] = {pl.x, pl.y, pl.z, pl.w};
    int32_t ids[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int b = kViewSeg * sg + 32 * k + lane;
      ids[k] = b < laid ? trow_s[b] : 0;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int b = kViewSeg * sg + 32 * k + lane;
      const bool keep = (plane[k] >> lane) & 1u;
      const int kb = before + __popc(plane[k] & lanes_below());  // kept positions before b
      if (b < laid) vrow[keep ? kb : kept_total + (b - kb)] = ids[k];
      before += __popc(plane[k]);
    }
  }
  if (threadIdx.x == 0 && has_view) {
    const int last = seq - (blocks - 1) * BS;
    const int view_len = blocks > 0 ? (kept_total - 1) * BS + last : 0;
    p.view_lens[r] = view_len;
    // DecodeView._count (runtime/block_view.py:297-329) for a decoding row: blocks read and blocks a full
    // read would read; the reads of an audited row, of a row read whole under a live policy without an
    // audit, and of any row while no policy is live
    if (p.counts != nullptr && (flags & kRowDecoding)) {
      const long long read = blocks > 0 ? kept_total : 0;
      const bool audited = (flags & kRowAudited) != 0;
      atomicAdd((unsigned long long*)&p.counts[0], (unsigned long long)read);
      atomicAdd((unsigned long long*)&p.counts[1], (unsigned long long)blocks);
      if (audited) atomicAdd((unsigned long long*)&p.counts[2], (unsigned long long)read);
      if (view_len == seq && !audited && !p.expired) atomicAdd((unsigned long long*)&p.counts[3], (unsigned long long)read);
      if (p.expired) atomicAdd((unsigned long long*)&p.counts[4], (unsigned long long)read);
    }
  }
}

template <typename K>
int launch_view(const ViewParams& p, cudaStream_t stream);

int launch_quota(const QuotaParams& p, size_t smem, cudaStream_t stream) {
  static bool configured[kMaxDevices] = {};
  int device = 0;
  {
    const int dev_rc = current_device(&device);
    if (dev_rc != EKV_OK) return dev_rc;
  }
  if (!configured[device]) {
    if (cudaFuncSetAttribute(quota_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kQuotaMaxRows * (int)sizeof(double)) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(quota_kernel)");
    configured[device] = true;
  }
  launch_chained(quota_kernel, dim3(1), dim3(kQuotaThreads), smem, stream, p);
  return check_launch("quota_kernel");
}

// The uniform quotas of rows whose pins are block 0 and [measured[r], n), with `budget` blocks plus
// *budget_add (on the device) shared by every row.
int presummed_quotas(const int32_t* row_blocks, const int32_t* measured, long long budget,
                     const long long* budget_add, int rows, int width, int32_t* quota, cudaStream_t stream) {
  if (rows > kQuotaMaxRows) return fail(EKV_ENOTSUP, "%d rows share one budget; at most %d", rows, kQuotaMaxRows);
  QuotaParams p{row_blocks, measured, -1, -1, 0.0, budget, nullptr, rows, width, quota, budget_add};
  return launch_quota(p, (size_t)rows * sizeof(double), stream);
}

// The committed mask (no view) of float64 rows that hold shares, ranked by share, equal shares to the
// older block, with the quotas given and pins block 0 and [measured[r], n).
int presummed_mask(const int32_t* row_blocks, const int32_t* quota, const int32_t* measured, const double* shares,
                   int64_t share_s0, int rows, int width, uint8_t* mask_out, int64_t mask_s0, cudaStream_t stream) {
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d (a row is staged in shared memory)", width, kViewMaxWidth);
  ViewParams p{};
  p.row_blocks = row_blocks; p.quota = quota; p.measured = measured; p.recent = -1;
  p.scores = shares; p.score_s0 = share_s0; p.policy = EKV_POLICY_UNIFORM;
  p.rows = rows; p.width = width; p.block_size = 1; p.mask_out = mask_out; p.mask_s0 = mask_s0; p.cap = -1;
  p.presummed = true;
  return launch_view<unsigned long long>(p, stream);
}

int launch_sum_view(const int32_t* table, int64_t table_s0, const int32_t* seq_lens, const uint8_t* full_rows,
                    const uint8_t* released, int64_t released_s0, int rows, int width, int block_size, int32_t* view,
                    int64_t view_s0, int32_t* view_lens, uint8_t* mask_out, int64_t mask_s0, const SumState* state,
                    const unsigned long long* keys, const int32_t* row_n, const int32_t* row_ps, const int32_t* row_at,
                    cudaStream_t stream) {
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d (a view row is staged in shared memory)", width, kViewMaxWidth);
  ViewParams p{};
  p.table = table; p.table_s0 = table_s0; p.seq_lens = seq_lens; p.full_rows = full_rows; p.released = released;
  p.released_s0 = released_s0; p.rows = rows; p.width = width; p.block_size = block_size; p.view = view;
  p.view_s0 = view_s0; p.view_lens = view_lens; p.mask_out = mask_out; p.mask_s0 = mask_s0; p.cap = -1;
  p.sum_state = state; p.sum_keys = keys; p.sum_row_n = row_n; p.sum_row_ps = row_ps; p.sum_row_at = row_at;
  return launch_view<uint32_t>(p, stream);
}

template <typename K>
int launch_view(const ViewParams& p, cudaStream_t stream) {
  const size_t smem = view_smem_bytes<K>(p.width);
  static size_t configured[kMaxDevices] = {};
  int device = 0;
  {
    const int dev_rc = current_device(&device);
    if (dev_rc != EKV_OK) return dev_rc;
  }
  if (configured[device] < smem) {
    if (cudaFuncSetAttribute(view_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(view_kernel)");
    configured[device] = smem;
  }
  launch_chained(view_kernel<K>, dim3(p.rows), dim3(kViewThreads), smem, stream, p);
  return check_launch("view_kernel");
}

}  // namespace ekv

using namespace ekv;

extern "C" int ekv_allocate_quotas(const int32_t* row_blocks, const int32_t* measured_blocks,
                                   int recent_blocks, int cap_above_blocks, double budget_fraction,
                                   int64_t budget, const double* row_fraction, int objective,
                                   int rows, int width, int32_t* quota, void* stream) {
  clear_error();
  if (!row_blocks || !quota) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width < 0) return fail(EKV_EINVAL, "rows must be positive and width not negative");
  if (recent_blocks < -1 || cap_above_blocks < -1) return fail(EKV_EINVAL, "invalid controller settings");
  if (objective != EKV_POLICY_SUM && objective != EKV_POLICY_UNIFORM && objective != EKV_POLICY_NEWEST)
    return fail(EKV_EINVAL, "unknown objective %d", objective);
  size_t smem = 0;
  if (row_fraction == nullptr) {
    if (objective == EKV_POLICY_SUM)
      return fail(EKV_ENOTSUP, "one budget shared by several rows under `sum` needs the global greedy");
    if (budget < 0 && !(budget_fraction > 0.0 && budget_fraction <= 1.0))
      return fail(EKV_EINVAL, "the budget fraction must be in (0, 1]");
    if (rows > kQuotaMaxRows) return fail(EKV_ENOTSUP, "%d rows share one budget; at most %d", rows, kQuotaMaxRows);
    smem = (size_t)rows * sizeof(double);
  } else if (rows > 65536) {
    return fail(EKV_ENOTSUP, "rows <= 65536");
  }
  QuotaParams p{row_blocks, measured_blocks, recent_blocks, cap_above_blocks, budget_fraction,
                (long long)budget, row_fraction, rows, width, quota, nullptr};
  return launch_quota(p, smem, static_cast<cudaStream_t>(stream));
}

extern "C" int ekv_view_build(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                              const int32_t* row_blocks, const int32_t* quota,
                              const int32_t* measured_blocks, int recent_blocks, const float* scores,
                              int64_t score_stride, int policy, const uint8_t* keep,
                              int64_t keep_stride, const uint8_t* full_rows, const uint8_t* released,
                              int64_t released_stride, int rows, int width, int block_size,
                              int32_t* view, int64_t view_stride, int32_t* view_lens,
                              uint8_t* mask_out, int64_t mask_stride, void* stream) {
  clear_error();
  if (!table || !seq_lens || !view || !view_lens) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0 || block_size <= 0)
    return fail(EKV_EINVAL, "rows, width and block_size must be positive");
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d (a view row is staged in shared memory)", width, kViewMaxWidth);
  if (rows > 2147483647) return fail(EKV_ENOTSUP, "too many rows");
  if (table_stride < width || view_stride < width) return fail(EKV_EINVAL, "a row stride is below the width");
  if (keep == nullptr) {
    if (!row_blocks || !quota) return fail(EKV_EINVAL, "ranking mode needs row_blocks and quota");
    if (policy != EKV_POLICY_SUM && policy != EKV_POLICY_UNIFORM && policy != EKV_POLICY_NEWEST)
      return fail(EKV_EINVAL, "unknown policy %d", policy);
    if (policy != EKV_POLICY_NEWEST && (!scores || score_stride < width))
      return fail(EKV_EINVAL, "ranking by shares needs scores with a row stride >= width");
    if (recent_blocks < -1) return fail(EKV_EINVAL, "recent_blocks must be >= -1");
  } else if (keep_stride < width) {
    return fail(EKV_EINVAL, "keep_stride %lld < width %d", (long long)keep_stride, width);
  }
  if (released && released_stride < width) return fail(EKV_EINVAL, "released_stride < width");
  if (mask_out && mask_stride < width) return fail(EKV_EINVAL, "mask_stride < width");
  ViewParams p{table,   table_stride, seq_lens, row_blocks, quota,      measured_blocks,
               recent_blocks, scores, score_stride, nullptr, nullptr, policy, keep,      keep_stride,
               full_rows, released, released_stride, rows, width,     block_size,
               view,    view_stride,  view_lens, mask_out,  mask_stride, nullptr, 0, nullptr, -1};
  return launch_view<uint32_t>(p, static_cast<cudaStream_t>(stream));
}

extern "C" int ekv_compact_block_table(const int32_t* table, int64_t table_stride,
                                       const int32_t* seq_lens, const uint8_t* keep,
                                       int64_t keep_stride, int rows, int width, int block_size,
                                       int32_t* view, int64_t view_stride, int32_t* view_lens,
                                       void* stream) {
  if (!keep) {
    clear_error();
    return fail(EKV_EINVAL, "compact_block_table needs a keep mask");
  }
  return ekv_view_build(table, table_stride, seq_lens, nullptr, nullptr, nullptr, 0, nullptr, 0,
                        EKV_POLICY_UNIFORM, keep, keep_stride, nullptr, nullptr, 0, rows, width,
                        block_size, view, view_stride, view_lens, nullptr, 0, stream);
}

extern "C" int ekv_decode_view(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                               const uint8_t* keep, int64_t keep_stride, const uint8_t* row_flags,
                               const uint8_t* released, int64_t released_stride, int expired, int rows, int width,
                               int block_size, int32_t* view, int64_t view_stride, int32_t* view_lens,
                               int64_t* counts, void* stream) {
  clear_error();
  if (!table || !seq_lens || !keep || !row_flags || !view || !view_lens)
    return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0 || block_size <= 0)
    return fail(EKV_EINVAL, "rows, width and block_size must be positive");
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d (a view row is staged in shared memory)", width, kViewMaxWidth);
  if (table_stride < width || view_stride < width || keep_stride < width)
    return fail(EKV_EINVAL, "a row stride is below the width");
  if (released && released_stride < width) return fail(EKV_EINVAL, "released_stride < width");
  ViewParams p{table, table_stride, seq_lens, nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, nullptr, EKV_POLICY_UNIFORM,
               keep,  keep_stride,  row_flags, released, released_stride, rows, width, block_size,
               view,  view_stride,  view_lens, nullptr, 0, reinterpret_cast<long long*>(counts), expired != 0,
               nullptr, -1};
  return launch_view<uint32_t>(p, static_cast<cudaStream_t>(stream));
}

extern "C" int ekv_view_build_f64(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                                  const int32_t* row_blocks, const int32_t* quota, const int32_t* measured_blocks,
                                  int recent_blocks, const double* scores, int64_t score_stride,
                                  const int32_t* score_rows, const double* weights, int policy,
                                  const uint8_t* full_rows, const uint8_t* released, int64_t released_stride,
                                  int rows, int width, int block_size, int32_t* view, int64_t view_stride,
                                  int32_t* view_lens, uint8_t* mask_out, int64_t mask_stride, void* stream) {
  clear_error();
  if (!row_blocks || !quota) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (view == nullptr ? mask_out == nullptr : (!table || !seq_lens || !view_lens))
    return fail(EKV_EINVAL, "a view needs table, seq_lens, view and view_lens; without one, mask_out is required");
  if (rows <= 0 || width <= 0 || block_size <= 0)
    return fail(EKV_EINVAL, "rows, width and block_size must be positive");
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d (a view row is staged in shared memory)", width, kViewMaxWidth);
  if (view != nullptr && (table_stride < width || view_stride < width)) return fail(EKV_EINVAL, "a row stride is below the width");
  if (policy != EKV_POLICY_SUM && policy != EKV_POLICY_UNIFORM && policy != EKV_POLICY_NEWEST)
    return fail(EKV_EINVAL, "unknown policy %d", policy);
  if (policy != EKV_POLICY_NEWEST && (!scores || score_stride < width))
    return fail(EKV_EINVAL, "ranking by shares needs scores with a row stride >= width");
  if (recent_blocks < -1) return fail(EKV_EINVAL, "recent_blocks must be >= -1");
  if (released && released_stride < width) return fail(EKV_EINVAL, "released_stride < width");
  if (mask_out && mask_stride < width) return fail(EKV_EINVAL, "mask_stride < width");
  ViewParams p{table,   table_stride, seq_lens, row_blocks, quota,      measured_blocks,
               recent_blocks, scores, score_stride, score_rows, weights, policy, nullptr, 0,
               full_rows, released, released_stride, rows, width,     block_size,
               view,    view_stride,  view_lens, mask_out,  mask_stride, nullptr, 0, nullptr, -1};
  return launch_view<unsigned long long>(p, static_cast<cudaStream_t>(stream));
}

extern "C" int ekv_view_build_fractions(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                                        const int32_t* row_blocks, const double* row_fraction,
                                        const int32_t* measured_blocks, int recent_blocks, int cap_above_blocks,
                                        const float* scores, int64_t score_stride, int policy,
                                        const uint8_t* full_rows, const uint8_t* released, int64_t released_stride,
                                        int rows, int width, int block_size, int32_t* view, int64_t view_stride,
                                        int32_t* view_lens, uint8_t* mask_out, int64_t mask_stride, void* stream) {
  clear_error();
  if (!table || !seq_lens || !view || !view_lens || !row_blocks || !row_fraction)
    return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0 || block_size <= 0)
    return fail(EKV_EINVAL, "rows, width and block_size must be positive");
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d (a view row is staged in shared memory)", width, kViewMaxWidth);
  if (table_stride < width || view_stride < width) return fail(EKV_EINVAL, "a row stride is below the width");
  if (policy != EKV_POLICY_SUM && policy != EKV_POLICY_UNIFORM && policy != EKV_POLICY_NEWEST)
    return fail(EKV_EINVAL, "unknown policy %d", policy);
  if (policy != EKV_POLICY_NEWEST && (!scores || score_stride < width))
    return fail(EKV_EINVAL, "ranking by shares needs scores with a row stride >= width");
  if (recent_blocks < -1 || cap_above_blocks < -1) return fail(EKV_EINVAL, "invalid controller settings");
  if (released && released_stride < width) return fail(EKV_EINVAL, "released_stride < width");
  if (mask_out && mask_stride < width) return fail(EKV_EINVAL, "mask_stride < width");
  ViewParams p{table,   table_stride, seq_lens, row_blocks, nullptr,    measured_blocks,
               recent_blocks, scores, score_stride, nullptr, nullptr, policy, nullptr, 0,
               full_rows, released, released_stride, rows, width,     block_size,
               view,    view_stride,  view_lens, mask_out,  mask_stride, nullptr, 0, row_fraction, cap_above_blocks};
  return launch_view<uint32_t>(p, static_cast<cudaStream_t>(stream));
}
