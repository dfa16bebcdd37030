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
//     them, the unpinned blocks ordered by a bitonic sort of (score, block) keys, their shares in that
//     order; the CTA that finishes last sets the budget and each request's index.
//   mm_cumsum_kernel, a thread per row: the running sums, one addition after another as np.cumsum.
//   mm_level_kernel, one CTA: the bisection (a binary search per request and a reduction per step)
//     and the leftover blocks through a binary heap in shared memory. The row quotas it writes make
//     ekv_view_build (EKV_POLICY_UNIFORM: equal shares to the older block) keep exactly the reference's
//     blocks.
#include "ekv_common.cuh"
#include "pairwise.cuh"
#include "pins.cuh"

namespace ekv {

constexpr int kMmThreads = 1024;
constexpr int kMmMaxWidth = 8192;
constexpr int kMmMaxRows = 4096;
constexpr int kMmBisection = 60;

enum MmMode : int { kMmSelect = 0, kMmNone = 1, kMmAll = 2 };

struct MmState {
  long long must, blocks, total_open, free_;
  int mode;
  unsigned int ticket;
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
  int* lb_low;      // [rows] the search result at the bisection's low end
  int* lb_high;     // [rows] ... and at its high end
};

struct MmLayout {
  size_t state, base, row_m, req, lb_low, lb_high, sorted, prefix, bytes;
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
  l.lb_low = take((size_t)rows * 4);
  l.lb_high = take((size_t)rows * 4);
  l.sorted = take((size_t)rows * width * 8);
  l.prefix = take((size_t)rows * width * 8);
  l.bytes = o;
  return l;
}

__device__ __forceinline__ double mm_clamped(float s) { return s > 0.f ? (double)s : 0.0; }
__device__ __forceinline__ double mm_clamped(double s) { return s > 0.0 ? s : 0.0; }

__host__ __device__ __forceinline__ int mm_sort_n(int width) {
  int n = 1;
  while (n < width) n <<= 1;
  return n;
}

// Shared memory of mm_prep_kernel<S>: the row's scores, the sort keys (uint64 [mm_sort_n(width)]) and,
// for float64 scores, the block of each key (uint32 [mm_sort_n(width)]).
template <typename S>
__host__ __device__ __forceinline__ size_t mm_prep_smem(int width) {
  const size_t scores = ((size_t)width * sizeof(S) + 15) / 16 * 16;
  return scores + (size_t)mm_sort_n(width) * (sizeof(S) == 8 ? 12 : 8);
}

// max(score, 0) as an order-preserving uint32 (NaN as 0)
__device__ __forceinline__ uint32_t mm_score_key(float s) { return s > 0.f ? __float_as_uint(s) : 0u; }

// One CTA per row. Float32 scores sort one uint64 per block, (~score bits, block): for scores that
// float32 holds, the order of the scores is the order of the shares. Float64 scores sort pairs
// (~share bits, block), the share being the very float64 value the reference orders
// (allocation.py:129): distinct scores can give equal shares.
template <typename S>
__global__ void __launch_bounds__(kMmThreads) mm_prep_kernel(const MmParams p) {
  extern __shared__ __align__(16) unsigned char mm_smem[];
  __shared__ PairwiseTree s_tree;
  __shared__ bool s_last;
  constexpr bool kWide = sizeof(S) == 8;
  const int r = blockIdx.x, tid = threadIdx.x;
  int n = p.row_blocks[r];
  const bool request = n > p.cap && n > 0;
  if (n > p.width) n = p.width;
  S* s_x = reinterpret_cast<S*>(mm_smem);
  unsigned long long* s_key =
      reinterpret_cast<unsigned long long*>(mm_smem + ((size_t)p.width * sizeof(S) + 15) / 16 * 16);
  uint32_t* s_blk = reinterpret_cast<uint32_t*>(s_key + mm_sort_n(p.width));  // float64 scores only
  const int ps = request ? pin_start(n, p.recent, p.measured, r) : 0;
  const int m = ps > 1 ? ps - 1 : 0;  // unpinned blocks [1, ps)
  if (request) {
    const S* xg = static_cast<const S*>(p.scores) +
                  (p.score_rows != nullptr ? (int64_t)p.score_rows[r] : (int64_t)r) * p.score_s0;
    for (int i = tid; i < n; i += kMmThreads) s_x[i] = xg[i];
    const double total = block_pairwise_sum<kMmThreads>(s_tree, n, [&](int i) { return mm_clamped(s_x[i]); });
    const double equal = __ddiv_rn(1.0, (double)(n > 1 ? n : 1));
    auto share = [&](int i) { return total > 0.0 ? __ddiv_rn(mm_clamped(s_x[i]), total) : equal; };
    // the pinned blocks in index order: block 0 and [ps, n) (every block when ps == 0)
    const int npin = ps >= 1 ? 1 + (n - ps) : n;
    const double base = block_pairwise_sum<kMmThreads>(
        s_tree, npin, [&](int j) { return share(ps >= 1 ? (j == 0 ? 0 : ps + j - 1) : j); });
    // the unpinned blocks by decreasing share, equal shares by increasing block: ascending keys; the
    // padding sorts last
    int P = 1;
    while (P < m) P <<= 1;
    if constexpr (kWide) {
      for (int j = tid; j < P; j += kMmThreads) {
        s_key[j] = j < m ? ~(unsigned long long)__double_as_longlong(share(1 + j)) : ~0ull;
        s_blk[j] = j < m ? (uint32_t)(1 + j) : 0xffffffffu;
      }
    } else {
      for (int j = tid; j < P; j += kMmThreads)
        s_key[j] = j < m ? ((unsigned long long)(~mm_score_key(s_x[1 + j])) << 32) | (unsigned long long)(1 + j)
                         : ~0ull;
    }
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1) {
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < P; i += kMmThreads) {
          const int partner = i ^ j;
          if (partner > i) {
            const unsigned long long a = s_key[i], b = s_key[partner];
            const bool up = (i & k) == 0;
            if constexpr (kWide) {
              const uint32_t ai = s_blk[i], bi = s_blk[partner];
              if ((a > b || (a == b && ai > bi)) == up) s_key[i] = b, s_key[partner] = a, s_blk[i] = bi, s_blk[partner] = ai;
            } else {
              if ((a > b) == up) s_key[i] = b, s_key[partner] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    if constexpr (kWide) {
      for (int j = tid; j < m; j += kMmThreads) p.sorted[(int64_t)j * p.rows + r] = share((int)s_blk[j]);
    } else {
      for (int j = tid; j < m; j += kMmThreads) p.sorted[(int64_t)j * p.rows + r] = share((int)(s_key[j] & 0xffffffffu));
    }
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
    }
    const long long free_ = budget - must;
    st->free_ = free_;
    st->mode = budget >= blocks ? kMmAll : (free_ <= 0 ? kMmNone : kMmSelect);
    st->ticket = 0;
  }
  __shared__ int s_scan[kMmThreads / 32 + 1];
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
// arrays: a warp's loads and stores are contiguous).
__global__ void __launch_bounds__(32) mm_cumsum_kernel(const MmParams p) {
  const int r = blockIdx.x * 32 + threadIdx.x;
  if (r >= p.rows) return;
  const int m = p.row_m[r];
  const int64_t R = p.rows;
  constexpr int C = 16;  // values per chunk; the next chunk is loaded while this one is added
  double acc = 0.0, cur[C], nxt[C];
#pragma unroll
  for (int u = 0; u < C; ++u) cur[u] = u < m ? p.sorted[u * R + r] : 0.0;
  for (int j = 0; j < m; j += C) {
#pragma unroll
    for (int u = 0; u < C; ++u) nxt[u] = j + C + u < m ? p.sorted[(j + C + u) * R + r] : 0.0;
#pragma unroll
    for (int u = 0; u < C; ++u) {
      if (j + u < m) {
        acc = (j + u == 0) ? cur[u] : acc + cur[u];
        p.prefix[(j + u) * R + r] = acc;
      }
    }
#pragma unroll
    for (int u = 0; u < C; ++u) cur[u] = nxt[u];
  }
}

// searchsorted (side left) of x in request r's running sums, each plus the request's offset: the first
// j with prefix[j] + offset >= x, known to lie in [lo, hi] (it grows with x).
__device__ __forceinline__ int mm_search(const MmParams& p, int r, double x, double offset, int lo, int hi) {
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (p.prefix[(int64_t)mid * p.rows + r] + offset < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// The blocks request r needs beyond its pins to retain `level` (allocation.py:146-150), and in *lb the
// search result it comes from.
__device__ __forceinline__ int mm_extra(const MmParams& p, int r, double level, int lo, int hi, int* lb) {
  const int m = p.row_m[r];
  *lb = lo;
  if (m < 0) return 0;
  const double need = level - p.base[r];
  const double offset = 2.0 * (double)p.req[r];
  *lb = mm_search(p, r, need - 1e-12 + offset, offset, lo, hi);
  if (need <= 1e-12) return 0;
  return *lb + 1 < m ? *lb + 1 : m;
}

constexpr int kMmAhead = 2;  // next shares per request staged in shared memory for the leftover blocks
constexpr size_t kMmLevelBytesPerRow = 8 + 8 * kMmAhead + 4 * 3;

// One CTA: the water level, the leftover blocks and the quotas. Dynamic shared memory per request: the
// heap entry (double level, int row), the next kMmAhead shares, the count and the count at the start
// of the leftover blocks.
__global__ void __launch_bounds__(kMmThreads) mm_level_kernel(const MmParams p) {
  extern __shared__ __align__(16) unsigned char lv_smem[];
  double* h_level = reinterpret_cast<double*>(lv_smem);
  double* ahead = h_level + p.rows;  // [rows][kMmAhead]
  int* h_row = reinterpret_cast<int*>(ahead + (size_t)p.rows * kMmAhead);
  int* counts = h_row + p.rows;
  int* start = counts + p.rows;
  __shared__ long long s_red[kMmThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const MmState* st = p.state;
  const int mode = st->mode;
  if (mode != kMmSelect) {
    for (int r = tid; r < p.rows; r += kMmThreads) {
      const int m = p.row_m[r];
      p.quota[r] = m < 0 ? -1 : (mode == kMmAll ? m : 0);
    }
    return;
  }
  const long long free_ = st->free_;
  // each request's search result is monotone in the level: keep it at both ends of the bisection and
  // search only between them
  for (int r = tid; r < p.rows; r += kMmThreads) {
    const int m = p.row_m[r];
    p.lb_low[r] = 0;
    p.lb_high[r] = m > 0 ? m : 0;
  }
  double low = 0.0, high = 1.0;
  for (int it = 0; it < kMmBisection; ++it) {
    const double mid = (low + high) / 2;
    long long sum = 0;
    for (int r = tid; r < p.rows; r += kMmThreads) {
      int lb;
      sum += mm_extra(p, r, mid, p.lb_low[r], p.lb_high[r], &lb);
      counts[r] = lb;  // (scratch: the search result at mid)
    }
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(kFullMask, sum, off);
    __syncthreads();
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    long long t = 0;
    for (int w = 0; w < kMmThreads / 32; ++w) t += s_red[w];
    const bool up = t <= free_;
    for (int r = tid; r < p.rows; r += kMmThreads) (up ? p.lb_low : p.lb_high)[r] = counts[r];
    if (up) low = mid; else high = mid;
  }
  long long used = 0;
  for (int r = tid; r < p.rows; r += kMmThreads) {
    int lb;
    counts[r] = mm_extra(p, r, low, p.lb_low[r], p.lb_low[r], &lb);
    used += counts[r];
  }
  for (int off = 16; off > 0; off >>= 1) used += __shfl_xor_sync(kFullMask, used, off);
  __syncthreads();
  if (lane == 0) s_red[warp] = used;
  // each request's retained share (its heap entry) and the shares of its next blocks, loaded in parallel
  for (int r = tid; r < p.rows; r += kMmThreads) {
    const int m = p.row_m[r], c = counts[r];
    h_level[r] = m < 0 ? 0.0 : p.base[r] + (c ? p.prefix[(int64_t)(c - 1) * p.rows + r] : 0.0);
    start[r] = c;
#pragma unroll
    for (int a = 0; a < kMmAhead; ++a) ahead[(size_t)r * kMmAhead + a] = c + a < m ? p.sorted[(int64_t)(c + a) * p.rows + r] : 0.0;
  }
  __syncthreads();
  if (tid == 0) {
    long long leftover = free_;
    for (int w = 0; w < kMmThreads / 32; ++w) leftover -= s_red[w];
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
      const int m = p.row_m[r];
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
      if (counts[r] < p.row_m[r]) {  // back with its next block's share added (heappop then heappush)
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
  for (int r = tid; r < p.rows; r += kMmThreads) p.quota[r] = p.row_m[r] < 0 ? -1 : counts[r];
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
                           int32_t* quota, void* workspace, size_t workspace_bytes, void* stream) {
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
  p.state = reinterpret_cast<MmState*>(base + l.state);
  p.base = reinterpret_cast<double*>(base + l.base);
  p.row_m = reinterpret_cast<int*>(base + l.row_m);
  p.req = reinterpret_cast<int*>(base + l.req);
  p.sorted = reinterpret_cast<double*>(base + l.sorted);
  p.lb_low = reinterpret_cast<int*>(base + l.lb_low);
  p.lb_high = reinterpret_cast<int*>(base + l.lb_high);
  p.prefix = reinterpret_cast<double*>(base + l.prefix);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(base + l.state, 0, sizeof(MmState), s) != cudaSuccess)
    return check_launch("cudaMemsetAsync(maxmin state)");
  const size_t prep_smem = mm_prep_smem<S>(width);
  const size_t level_smem = (size_t)rows * kMmLevelBytesPerRow;
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return check_launch("cudaGetDevice");
  static size_t prep_set[kMaxDevices] = {}, level_set[kMaxDevices] = {};
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
  mm_prep_kernel<S><<<rows, kMmThreads, prep_smem, s>>>(p);
  int rc = check_launch("mm_prep_kernel");
  if (rc != EKV_OK) return rc;
  mm_cumsum_kernel<<<(rows + 31) / 32, 32, 0, s>>>(p);
  if ((rc = check_launch("mm_cumsum_kernel")) != EKV_OK) return rc;
  mm_level_kernel<<<1, kMmThreads, level_smem, s>>>(p);
  return check_launch("mm_level_kernel");
}

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
