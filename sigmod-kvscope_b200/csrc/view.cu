// The decide-and-enforce half of the path on the device: per-row budgets (quota kernel), the
// per-row keep decision by exact top-k selection, and the stable compaction of the block table
// into the view the attention kernel reads.
//
// The view kernel runs one CTA per row. Ranking mode turns max(score, 0) (float32, NaN as 0) into
// an order-preserving uint32 key and finds the quota-th largest key of the row's unpinned blocks by
// a four-pass MSB radix select (256-bin shared-memory histograms). Keys above the threshold are
// kept; of the keys equal to it, the first (uniform: older blocks first, allocation.py:89) or last
// (sum: newer blocks first, allocation.py:107-113) ones fill the quota, found with a block-wide
// scan. A second block-wide scan over the keep flags places kept blocks first and the others after
// them, both in their original order: the stable partition of compact_block_table
// (runtime/block_view.py:52).
#include "ekv_common.cuh"

namespace ekv {

// The pins of Controller._allocate (observe/controller.py:420-424): block 0 and [pin_start, n).
// The unpinned blocks are then exactly [1, pin_start).
// recent < 0 pins no newest blocks beyond those of `measured`.
__device__ __host__ __forceinline__ int pin_start(int n, int recent, const int32_t* measured, int r) {
  int ps = recent < 0 ? n : n - 1 - recent;
  if (ps < 0) ps = 0;
  if (measured != nullptr) {
    int m = measured[r];
    if (m < 0) m = 0;
    if (m < ps) ps = m;
  }
  return ps;
}

__device__ __forceinline__ int pin_count(int n, int ps) { return n <= 0 ? 0 : (ps > 0 ? 1 : 0) + (n - ps); }

// ---- quotas ------------------------------------------------------------------------------------

struct QuotaParams {
  const int32_t* row_blocks;
  const int32_t* measured;
  int recent, cap;
  double fraction;
  long long budget;  // >= 0: the shared budget as given; < 0: from `fraction`
  const double* row_fraction;
  int rows;
  int32_t* quota;
};

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
  extern __shared__ double s_rem[];  // [rows] remainders of the shared-budget split
  __shared__ long long s_red[kQuotaThreads / 32];
  const int R = p.rows;
  if (p.row_fraction != nullptr) {
    // Every row is its own allocate() call (allocation.py:55-76) with its own budget.
    for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
      const int n = p.row_blocks[r];
      if (n <= p.cap || n <= 0) {
        p.quota[r] = -1;
        continue;
      }
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
    const int n = p.row_blocks[r];
    if (n <= p.cap || n <= 0) continue;
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
  }
  const bool keep_all = budget >= total;
  const long long free_ = budget - floor_;
  long long assigned = 0;
  for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
    const int n = p.row_blocks[r];
    s_rem[r] = -1.0;  // not a request
    if (n <= p.cap || n <= 0) {
      p.quota[r] = -1;
      continue;
    }
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
  // The `extra` largest remainders get one more block; equal remainders go to the earlier row.
  for (int r = threadIdx.x; r < R; r += kQuotaThreads) {
    const double mine = s_rem[r];
    if (mine < 0.0) continue;
    long long rank = 0;
    for (int i = 0; i < R; ++i) {
      const double other = s_rem[i];
      rank += other > mine || (other == mine && other >= 0.0 && i < r);
    }
    if (rank < extra) p.quota[r] += 1;
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
  const float* scores;
  int64_t score_s0;
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
};

constexpr int kViewThreads = 512;
constexpr int kViewMaxWidth = 32768;

__device__ __forceinline__ uint32_t share_key(float x) {
  // max(x, 0) with NaN as 0; for x >= 0 the IEEE bit pattern is monotone in x
  return x > 0.f ? __float_as_uint(x) : 0u;
}

__global__ void __launch_bounds__(kViewThreads) view_kernel(const ViewParams p) {
  extern __shared__ uint32_t s_keys[];  // [width] keys of the unpinned blocks (ranking mode)
  __shared__ int s_hist[256];
  __shared__ int s_scan[kViewThreads / 32 + 1];
  __shared__ int s_pick[2];
  const int r = blockIdx.x;
  const int W = p.width, BS = p.block_size;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- the committed mask: pins + selection (ranking mode) or the given mask ---------------------
  const bool rank_mode = p.keep == nullptr;
  int n_a = 0, ps = 0, q = -1;
  bool select_all = false, select_none = true, by_threshold = false, newest = false;
  uint32_t threshold = 0;
  int k_eq = 0;  // keys equal to the threshold that are kept
  bool ties_need_rank = false;
  if (rank_mode) {
    n_a = p.row_blocks[r];
    n_a = n_a < 0 ? 0 : (n_a > W ? W : n_a);
    q = p.quota[r];
    if (q >= 0 && n_a > 0) {
      ps = pin_start(n_a, p.recent, p.measured, r);
      const int n_open = ps > 1 ? ps - 1 : 0;
      if (q > n_open) q = n_open;
      select_none = q == 0;
      select_all = q == n_open && q > 0;
      if (!select_none && !select_all) {
        if (p.policy == EKV_POLICY_NEWEST) {
          newest = true;
        } else {
          by_threshold = true;
        }
      }
    }
  }
  if (by_threshold) {
    const float* srow = p.scores + (int64_t)r * p.score_s0;
    for (int b = 1 + threadIdx.x; b < ps; b += kViewThreads) s_keys[b] = share_key(srow[b]);
    uint32_t prefix = 0, pmask = 0;
    int k = q;
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      for (int i = threadIdx.x; i < 256; i += kViewThreads) s_hist[i] = 0;
      __syncthreads();
      for (int b = 1 + threadIdx.x; b < ps; b += kViewThreads) {
        const uint32_t key = s_keys[b];
        if ((key & pmask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1);
      }
      __syncthreads();
      if (warp == 0) {
        // lane owns digits [8*lane, 8*lane+8); count the keys above each digit from the top down
        int local[8], sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) local[i] = s_hist[8 * lane + i], sum += local[i];
        int above = sum;  // inclusive suffix sum over lanes >= lane
        for (int off = 1; off < 32; off <<= 1) {
          const int v = __shfl_down_sync(kFullMask, above, off);
          if (lane + off < 32) above += v;
        }
        int gt = above - sum;  // keys in digits owned by higher lanes
#pragma unroll
        for (int i = 7; i >= 0; --i) {
          if (gt < k && gt + local[i] >= k) {
            s_pick[0] = 8 * lane + i;
            s_pick[1] = gt;
          }
          gt += local[i];
        }
      }
      __syncthreads();
      const int d = s_pick[0];
      k -= s_pick[1];
      prefix |= (uint32_t)d << shift;
      pmask |= 255u << shift;
      __syncthreads();  // s_pick is rewritten by the next pass
    }
    threshold = prefix;
    k_eq = k;
    ties_need_rank = true;  // resolved below once the number of equal keys is known
  }

  // ---- per-thread blocked ranges: thread t owns [t*ipt, (t+1)*ipt) ----------------------------------
  const int ipt = (W + kViewThreads - 1) / kViewThreads;
  const int b0 = threadIdx.x * ipt;
  const int b1 = min(b0 + ipt, W);

  // rank of equal keys: how many equal keys precede this thread's range
  int eq_before = 0, eq_total = 0;
  if (by_threshold) {
    int cnt = 0;
    for (int b = max(b0, 1); b < min(b1, ps); ++b) cnt += s_keys[b] == threshold;
    eq_before = block_exclusive_scan<kViewThreads>(cnt, s_scan, &eq_total);
    ties_need_rank = eq_total != k_eq;
  }
  const bool older_first = p.policy == EKV_POLICY_UNIFORM;

  const int seq = p.seq_lens[r];
  const int blocks = seq > 0 ? (seq + BS - 1) / BS : 0;
  const bool full = p.full_rows != nullptr && p.full_rows[r] != 0;
  const int32_t* trow = p.table + (int64_t)r * p.table_s0;
  const uint8_t* krow = rank_mode ? nullptr : p.keep + (int64_t)r * p.keep_s0;
  const uint8_t* rrow = p.released ? p.released + (int64_t)r * p.released_s0 : nullptr;
  uint8_t* mrow = p.mask_out ? p.mask_out + (int64_t)r * p.mask_s0 : nullptr;

  // The committed mask at b (ranking mode: the controller's row).
  auto committed = [&](int b, int& eq_seen) -> bool {
    if (!rank_mode) return krow[b] != 0;
    if (q < 0 || n_a == 0 || b >= n_a || b == 0 || b >= ps) return true;
    if (select_all) return true;
    if (select_none) return false;
    if (newest) return b >= ps - q;
    const uint32_t key = s_keys[b];
    if (key > threshold) return true;
    if (key != threshold) return false;
    const int before = eq_seen++;
    if (!ties_need_rank) return true;
    return older_first ? before < k_eq : (eq_total - before - 1) < k_eq;
  };

  // pass 1: the final keep flags of this thread's range, counted
  int kept_local = 0;
  {
    int eq_seen = eq_before;
    for (int b = b0; b < b1; ++b) {
      bool k = committed(b, eq_seen) || full;
      if (rrow != nullptr && rrow[b]) k = false;  // a released block is never read (block_view.py:280-281)
      k = (k || b == 0 || b == blocks - 1) && b < blocks;
      kept_local += k;
    }
  }
  int kept_total = 0;
  const int kept_before = block_exclusive_scan<kViewThreads>(kept_local, s_scan, &kept_total);

  // pass 2: scatter kept blocks to the front and the rest after them, both in order
  {
    int eq_seen = eq_before;
    int kept = kept_before;
    int32_t* vrow = p.view + (int64_t)r * p.view_s0;
    for (int b = b0; b < b1; ++b) {
      const bool c = committed(b, eq_seen);
      if (mrow != nullptr) mrow[b] = c;
      bool k = c || full;
      if (rrow != nullptr && rrow[b]) k = false;
      k = (k || b == 0 || b == blocks - 1) && b < blocks;
      const int32_t id = trow[b];
      if (k) {
        vrow[kept++] = id;
      } else {
        vrow[kept_total + (b - kept)] = id;
      }
    }
  }
  if (threadIdx.x == 0) {
    const int last = seq - (blocks - 1) * BS;
    p.view_lens[r] = blocks > 0 ? (kept_total - 1) * BS + last : 0;
  }
}

int launch_view(const ViewParams& p, cudaStream_t stream) {
  const size_t smem = p.keep == nullptr ? (size_t)p.width * sizeof(uint32_t) : 0;
  static bool configured[kMaxDevices] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return check_launch("cudaGetDevice");
  if (!configured[device]) {
    if (cudaFuncSetAttribute(view_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kViewMaxWidth * (int)sizeof(uint32_t)) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(view_kernel)");
    configured[device] = true;
  }
  view_kernel<<<p.rows, kViewThreads, smem, stream>>>(p);
  return check_launch("view_kernel");
}

}  // namespace ekv

using namespace ekv;

extern "C" int ekv_allocate_quotas(const int32_t* row_blocks, const int32_t* measured_blocks,
                                   int recent_blocks, int cap_above_blocks, double budget_fraction,
                                   int64_t budget, const double* row_fraction, int objective,
                                   int rows, int32_t* quota, void* stream) {
  clear_error();
  if (!row_blocks || !quota) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0) return fail(EKV_EINVAL, "rows must be positive");
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
  static bool configured[kMaxDevices] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return check_launch("cudaGetDevice");
  if (!configured[device]) {
    if (cudaFuncSetAttribute(quota_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kQuotaMaxRows * (int)sizeof(double)) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(quota_kernel)");
    configured[device] = true;
  }
  QuotaParams p{row_blocks, measured_blocks, recent_blocks, cap_above_blocks, budget_fraction,
                (long long)budget, row_fraction, rows, quota};
  quota_kernel<<<1, kQuotaThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("quota_kernel");
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
  if (width > kViewMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d", width, kViewMaxWidth);
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
               recent_blocks, scores, score_stride, policy, keep,      keep_stride,
               full_rows, released, released_stride, rows, width,     block_size,
               view,    view_stride,  view_lens, mask_out,  mask_stride};
  return launch_view(p, static_cast<cudaStream_t>(stream));
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
