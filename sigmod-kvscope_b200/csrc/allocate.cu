// The `sum` objective over several requests on the device: one budget shared by every measured row,
// spent on the unpinned blocks with the largest weighted share (observe/allocation.py:94-118, the
// controller's default objective, observe/controller.py:30, :398-451).
//
// The reference picks the `free` largest gains weight_r * share_r[b] over all requests, where
// share_r = max(score, 0) / total_r in float64 and total_r is NumPy's pairwise sum of the clamped
// scores; a gain equal to the smallest chosen one goes to the newer block first, then to the earlier
// request. Within one request the gain is strictly increasing in the float32 score (distinct
// float32 values divided by one total and multiplied by one weight stay distinct), so the global
// choice is, per row, "the q_r best blocks by score, newer first on ties" with
//   q_r = (its gains above the threshold) + (its share of the ties at the threshold),
// which ekv_view_build then carries out. This file computes q_r:
//   1. sum_prep_kernel, one CTA per row: total_r exactly as numpy.add.reduce computes it (pairwise
//      over leaves of at most 128 values, eight accumulators per leaf), the pins, and, in the CTA
//      that finishes last, the budget.
//   2. sum_select_kernel, six launches: an MSB radix select of the `free`-th largest gain over the
//      63-bit keys of the non-negative float64 gains (digits of 11 bits, the last of 8). Each CTA
//      histograms its share of the blocks in shared memory and merges it; the CTA that finishes
//      last picks the digit. No CTA waits for another.
//   3. sum_ties_kernel, one CTA per row: gains above the threshold, and a count of the ties at each
//      block index; the CTA that finishes last finds the index i* at which the ties needed run out
//      (ties are taken from the highest index down).
//   4. sum_quota_kernel, one CTA per row: q_r, with the ties at i* going to the earliest rows.
#include "ekv_common.cuh"
#include "pins.cuh"

namespace ekv {

constexpr int kSumThreads = 256;
constexpr int kSumBins = 2048;
constexpr int kSumPasses = 6;
constexpr int kMaxLeaves = 512;  // leaves of a pairwise sum over up to 32768 values (each > 64 values)
constexpr int kSumMaxWidth = 32768;

enum SumMode : int { kSumSelect = 0, kSumNone = 1, kSumAll = 2 };

struct SumState {
  unsigned long long prefix, mask;  // the threshold's known bits
  long long k;                      // gains still to choose at the threshold's prefix
  long long total_open, must, blocks;
  int mode, found;
  int istar;       // the lowest block index whose ties are (partly) taken
  long long m;     // ties taken at istar, from the earliest rows
  unsigned int ticket;
};

struct SumParams {
  const float* scores;
  int64_t score_s0;
  const double* weights;
  const int32_t* row_blocks;
  const int32_t* measured;
  int recent, cap;
  double fraction;
  long long budget;
  int rows, width;
  int32_t* quota;
  // workspace
  SumState* state;
  double* total;       // [rows]
  double* weight;      // [rows]
  int* row_n;          // [rows] blocks of a request, 0 for a row that is not one
  int* row_ps;         // [rows] pin start
  int* row_gt;         // [rows] gains above the threshold
  unsigned int* hist;  // [kSumBins]
  unsigned int* ties;  // [width] ties at each block index
};

struct SumLayout {
  size_t state, total, weight, row_n, row_ps, row_gt, hist, ties, bytes;
};

SumLayout sum_layout(int rows, int width) {
  SumLayout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += round_up(bytes, 256);
    return at;
  };
  l.state = take(sizeof(SumState));
  l.hist = take(kSumBins * 4);
  l.ties = take((size_t)width * 4);
  l.total = take((size_t)rows * 8);
  l.weight = take((size_t)rows * 8);
  l.row_n = take((size_t)rows * 4);
  l.row_ps = take((size_t)rows * 4);
  l.row_gt = take((size_t)rows * 4);
  l.bytes = o;
  return l;
}

// max(score, 0) in float64; NaN counts as 0, as the controller passes it (observe/controller.py:337).
__device__ __forceinline__ double clamped(float s) { return s > 0.f ? (double)s : 0.0; }

// The order-preserving key of request r's gain at a block with score s: the bits of the
// non-negative float64 gain (0 for a gain of +-0).
__device__ __forceinline__ unsigned long long gain_key(float s, double total, double w, int n) {
  const double share = total > 0.0 ? clamped(s) / total : 1.0 / (double)(n > 1 ? n : 1);
  const double g = w * share;
  return g > 0.0 ? (unsigned long long)__double_as_longlong(g) : 0ull;
}

__device__ __forceinline__ void digit_of(int pass, int& shift, unsigned long long& dmask) {
  shift = pass < 5 ? 52 - 11 * pass : 0;
  dmask = pass < 5 ? 2047ull : 255ull;
}

// numpy's pairwise_sum of one leaf (at most 128 values): eight accumulators, combined as
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)), then the rest one by one; below 8 values a plain
// loop from 0.
__device__ double leaf_sum(const float* x, int len) {
  if (len < 8) {
    double res = 0.0;
    for (int i = 0; i < len; ++i) res += clamped(x[i]);
    return res;
  }
  double r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = clamped(x[j]);
  int i = 8;
  for (; i < len - (len % 8); i += 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] += clamped(x[i + j]);
  double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < len; ++i) res += clamped(x[i]);
  return res;
}

// The pairwise tree above the leaves: a segment of more than 128 values splits at n2 = n / 2 rounded
// down to a multiple of 8. Leaves are consumed left to right.
__device__ double tree_sum(int len, const double* leaf, int& next) {
  if (len <= 128) return leaf[next++];
  int n2 = len / 2;
  n2 -= n2 % 8;
  const double a = tree_sum(n2, leaf, next);
  const double b = tree_sum(len - n2, leaf, next);
  return a + b;
}

// One CTA per row.
__global__ void __launch_bounds__(kSumThreads) sum_prep_kernel(const SumParams p) {
  __shared__ int s_lo[kMaxLeaves], s_len[kMaxLeaves];
  __shared__ double s_leaf[kMaxLeaves];
  __shared__ int s_leaves;
  __shared__ bool s_last;
  const int r = blockIdx.x, tid = threadIdx.x;
  int n = p.row_blocks[r];
  const bool request = n > p.cap && n > 0;
  if (n > p.width) n = p.width;
  const float* x = p.scores + (int64_t)r * p.score_s0;
  double total = 0.0;
  if (request) {
    if (tid == 0) {  // the leaves, left to right
      int stack_lo[32], stack_len[32], top = 0, count = 0;
      stack_lo[0] = 0;
      stack_len[0] = n;
      top = 1;
      while (top > 0) {
        --top;
        const int lo = stack_lo[top], len = stack_len[top];
        if (len <= 128) {
          s_lo[count] = lo;
          s_len[count] = len;
          ++count;
        } else {
          int n2 = len / 2;
          n2 -= n2 % 8;
          stack_lo[top] = lo + n2, stack_len[top] = len - n2, ++top;  // right half, popped second
          stack_lo[top] = lo, stack_len[top] = n2, ++top;             // left half, popped first
        }
      }
      s_leaves = count;
    }
    __syncthreads();
    for (int i = tid; i < s_leaves; i += kSumThreads) s_leaf[i] = leaf_sum(x + s_lo[i], s_len[i]);
    __syncthreads();
    if (tid == 0) {
      int next = 0;
      total = tree_sum(n, s_leaf, next);
    }
  }
  if (tid == 0) {
    int ps = 0;
    if (request) {
      ps = pin_start(n, p.recent, p.measured, r);
      atomicAdd((unsigned long long*)&p.state->total_open, (unsigned long long)(ps > 1 ? ps - 1 : 0));
      atomicAdd((unsigned long long*)&p.state->must, (unsigned long long)pin_count(n, ps));
      atomicAdd((unsigned long long*)&p.state->blocks, (unsigned long long)n);
    }
    p.total[r] = total;
    p.weight[r] = p.weights ? p.weights[r] : 1.0;
    p.row_n[r] = request ? n : 0;
    p.row_ps[r] = ps;
    __threadfence();
    s_last = atomicAdd(&p.state->ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || tid != 0) return;
  // the budget (controller.py:435-437) and what to do with it (allocation.py:64-67, :98-104)
  __threadfence();
  SumState* st = p.state;
  const long long must = *(volatile long long*)&st->must, blocks = *(volatile long long*)&st->blocks;
  const long long total_open = *(volatile long long*)&st->total_open;
  long long budget = p.budget;
  if (budget < 0) {
    budget = (long long)ceil(p.fraction * (double)blocks);
    if (budget < must) budget = must;
  }
  const long long free_ = budget - must;
  if (budget >= blocks || free_ >= total_open) {
    st->mode = kSumAll;
  } else if (free_ <= 0) {
    st->mode = kSumNone;
  } else {
    st->mode = kSumSelect;
    st->k = free_;
  }
  st->prefix = 0;
  st->mask = 0;
  st->found = 0;
  st->ticket = 0;
}

// One pass of the radix select; the grid strides over every (row, block).
__global__ void __launch_bounds__(kSumThreads) sum_select_kernel(const SumParams p, int pass) {
  __shared__ unsigned int s_hist[kSumBins];
  __shared__ bool s_last;
  __shared__ int s_pick;
  __shared__ long long s_above;
  __shared__ unsigned int s_count;
  __shared__ long long s_w[kSumThreads / 32];
  const int tid = threadIdx.x;
  SumState* st = p.state;
  if (st->mode != kSumSelect || st->found) return;
  int shift;
  unsigned long long dmask;
  digit_of(pass, shift, dmask);
  const unsigned long long prefix = st->prefix, mask = st->mask;
  for (int i = tid; i < kSumBins; i += kSumThreads) s_hist[i] = 0;
  __syncthreads();
  const long long cells = (long long)p.rows * p.width;
  for (long long e = (long long)blockIdx.x * kSumThreads + tid; e < cells; e += (long long)gridDim.x * kSumThreads) {
    const int r = (int)(e / p.width), b = (int)(e - (long long)r * p.width);
    const int n = p.row_n[r];
    if (n == 0 || b < 1 || b >= p.row_ps[r]) continue;
    const unsigned long long key = gain_key(p.scores[(int64_t)r * p.score_s0 + b], p.total[r], p.weight[r], n);
    if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & dmask], 1u);
  }
  __syncthreads();
  for (int i = tid; i < kSumBins; i += kSumThreads)
    if (s_hist[i]) atomicAdd(&p.hist[i], s_hist[i]);
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&st->ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // the CTA that finished last: the digit of the k-th largest key; thread t owns bins [8t, 8t + 8)
  unsigned int h[8];
  long long sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) h[j] = __ldcg(p.hist + 8 * tid + j), sum += h[j];
  const int warp = tid >> 5, lane = tid & 31;
  long long above = sum;  // this thread's bins and the bins of the lanes above it
  for (int off = 1; off < 32; off <<= 1) {
    const long long v = __shfl_down_sync(kFullMask, above, off);
    if (lane + off < 32) above += v;
  }
  if (lane == 0) s_w[warp] = above;
  __syncthreads();
  long long gt = above - sum;
  for (int w2 = warp + 1; w2 < kSumThreads / 32; ++w2) gt += s_w[w2];
  const long long k = st->k;
#pragma unroll
  for (int j = 7; j >= 0; --j) {
    if (gt < k && gt + h[j] >= k) {
      s_pick = 8 * tid + j;
      s_above = gt;
      s_count = h[j];
    }
    gt += h[j];
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 8; ++j) p.hist[8 * tid + j] = 0;  // ready for the next pass
  if (tid == 0) {
    const long long k2 = k - s_above;
    st->prefix = prefix | ((unsigned long long)s_pick << shift);
    st->mask = mask | (dmask << shift);
    st->k = k2;
    st->found = (long long)s_count == k2 || pass == kSumPasses - 1;  // every key with the prefix is taken
    st->ticket = 0;
  }
}

// One CTA per row: gains above the threshold, ties per block index; the CTA that finishes last finds
// i*, the lowest block index of the ties taken, and m, the ties taken there.
__global__ void __launch_bounds__(kSumThreads) sum_ties_kernel(const SumParams p) {
  __shared__ long long s_w[kSumThreads / 32];
  __shared__ bool s_last;
  const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  SumState* st = p.state;
  if (st->mode != kSumSelect) return;
  const unsigned long long prefix = st->prefix, mask = st->mask;
  const int n = p.row_n[r], ps = p.row_ps[r];
  long long gt = 0;
  if (n > 0) {
    const float* x = p.scores + (int64_t)r * p.score_s0;
    const double total = p.total[r], w = p.weight[r];
    for (int b = 1 + tid; b < ps; b += kSumThreads) {
      const unsigned long long key = gain_key(x[b], total, w, n) & mask;
      if (key > prefix) ++gt;
      else if (key == prefix) atomicAdd(&p.ties[b], 1u);
    }
  }
  for (int off = 16; off > 0; off >>= 1) gt += __shfl_xor_sync(kFullMask, gt, off);
  if (lane == 0) s_w[warp] = gt;
  __syncthreads();
  if (tid == 0) {
    long long t = 0;
    for (int w2 = 0; w2 < kSumThreads / 32; ++w2) t += s_w[w2];
    p.row_gt[r] = (int)t;
    __threadfence();
    s_last = atomicAdd(&st->ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // ties are taken from the highest block index down; thread t owns indices [t * per, t * per + per)
  const int per = (p.width + kSumThreads - 1) / kSumThreads;
  const int lo = tid * per, hi = min(lo + per, p.width);
  long long cnt = 0;
  for (int i = lo; i < hi; ++i) cnt += __ldcg(p.ties + i);
  long long above = cnt;  // this thread's indices and those of the lanes above it
  for (int off = 1; off < 32; off <<= 1) {
    const long long v = __shfl_down_sync(kFullMask, above, off);
    if (lane + off < 32) above += v;
  }
  __syncthreads();
  if (lane == 0) s_w[warp] = above;
  __syncthreads();
  long long taken = above - cnt;  // ties at indices >= hi
  for (int w2 = warp + 1; w2 < kSumThreads / 32; ++w2) taken += s_w[w2];
  const long long k = st->k;
  if (taken < k && taken + cnt >= k) {
    for (int i = hi - 1; i >= lo; --i) {
      const long long c = __ldcg(p.ties + i);
      if (taken + c >= k) {
        st->istar = i;
        st->m = k - taken;
        break;
      }
      taken += c;
    }
  }
  if (tid == 0) st->ticket = 0;
}

// One CTA per row: its quota of unpinned blocks for ekv_view_build (-1: not a request, read in full).
__global__ void __launch_bounds__(kSumThreads) sum_quota_kernel(const SumParams p) {
  __shared__ long long s_w[kSumThreads / 32];
  const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const SumState* st = p.state;
  const int n = p.row_n[r], ps = p.row_ps[r];
  const int open = ps > 1 ? ps - 1 : 0;
  if (n == 0 || st->mode != kSumSelect) {
    if (tid == 0) p.quota[r] = n == 0 ? -1 : (st->mode == kSumAll ? open : 0);
    return;
  }
  const unsigned long long prefix = st->prefix, mask = st->mask;
  const int istar = st->istar;
  const long long m = st->m;
  // this row's ties above i*, and the rows before it that tie at i*
  long long mine = 0, before = 0;
  const float* x = p.scores + (int64_t)r * p.score_s0;
  for (int b = istar + 1 + tid; b < ps; b += kSumThreads)
    mine += (gain_key(x[b], p.total[r], p.weight[r], n) & mask) == prefix;
  for (int q = tid; q < r; q += kSumThreads) {
    const int nq = p.row_n[q];
    if (nq > 0 && istar >= 1 && istar < p.row_ps[q])
      before += (gain_key(p.scores[(int64_t)q * p.score_s0 + istar], p.total[q], p.weight[q], nq) & mask) == prefix;
  }
  for (int off = 16; off > 0; off >>= 1) {
    mine += __shfl_xor_sync(kFullMask, mine, off);
    before += __shfl_xor_sync(kFullMask, before, off);
  }
  if (lane == 0) s_w[warp] = mine;
  __syncthreads();
  long long t_mine = 0;
  for (int w2 = 0; w2 < kSumThreads / 32; ++w2) t_mine += s_w[w2];
  __syncthreads();
  if (lane == 0) s_w[warp] = before;
  __syncthreads();
  if (tid == 0) {
    long long t_before = 0;
    for (int w2 = 0; w2 < kSumThreads / 32; ++w2) t_before += s_w[w2];
    const bool tie_here =
        istar >= 1 && istar < ps && (gain_key(x[istar], p.total[r], p.weight[r], n) & mask) == prefix;
    p.quota[r] = (int)(p.row_gt[r] + t_mine + (tie_here && t_before < m ? 1 : 0));
  }
}

}  // namespace ekv

using namespace ekv;

extern "C" size_t ekv_allocate_sum_workspace_bytes(int rows, int width) {
  if (rows <= 0 || width <= 0) return 0;
  return sum_layout(rows, width).bytes;
}

extern "C" int ekv_allocate_sum(const float* scores, int64_t score_stride, const double* weights,
                                const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                                int cap_above_blocks, double budget_fraction, int64_t budget, int rows, int width,
                                int32_t* quota, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!scores || !row_blocks || !quota) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0) return fail(EKV_EINVAL, "rows and width must be positive");
  if (width > kSumMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d", width, kSumMaxWidth);
  if (score_stride < width) return fail(EKV_EINVAL, "score_stride %lld < width %d", (long long)score_stride, width);
  if (recent_blocks < -1 || cap_above_blocks < -1) return fail(EKV_EINVAL, "invalid controller settings");
  if (budget < 0 && !(budget_fraction > 0.0 && budget_fraction <= 1.0))
    return fail(EKV_EINVAL, "the budget fraction must be in (0, 1]");
  const SumLayout l = sum_layout(rows, width);
  if (!workspace || workspace_bytes < l.bytes)
    return fail(EKV_ERANGE, "the sum workspace holds %zu bytes, the call needs %zu", workspace_bytes, l.bytes);
  if ((uintptr_t)workspace & 255) return fail(EKV_EINVAL, "the sum workspace must be 256-byte aligned");
  uint8_t* base = static_cast<uint8_t*>(workspace);
  SumParams p{};
  p.scores = scores; p.score_s0 = score_stride; p.weights = weights; p.row_blocks = row_blocks;
  p.measured = measured_blocks; p.recent = recent_blocks; p.cap = cap_above_blocks;
  p.fraction = budget_fraction; p.budget = (long long)budget; p.rows = rows; p.width = width; p.quota = quota;
  p.state = reinterpret_cast<SumState*>(base + l.state);
  p.hist = reinterpret_cast<unsigned int*>(base + l.hist);
  p.ties = reinterpret_cast<unsigned int*>(base + l.ties);
  p.total = reinterpret_cast<double*>(base + l.total);
  p.weight = reinterpret_cast<double*>(base + l.weight);
  p.row_n = reinterpret_cast<int*>(base + l.row_n);
  p.row_ps = reinterpret_cast<int*>(base + l.row_ps);
  p.row_gt = reinterpret_cast<int*>(base + l.row_gt);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the state, the histogram and the tie counts start at zero (they precede the per-row arrays)
  if (cudaMemsetAsync(base, 0, l.total, s) != cudaSuccess) return check_launch("cudaMemsetAsync(sum workspace)");
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("cudaDeviceGetAttribute");
  sum_prep_kernel<<<rows, kSumThreads, 0, s>>>(p);
  int rc = check_launch("sum_prep_kernel");
  if (rc != EKV_OK) return rc;
  const long long cells = (long long)rows * width;
  const long long want = (cells + kSumThreads * 8 - 1) / (kSumThreads * 8);
  const int grid = (int)(want < 8LL * sms ? (want > 0 ? want : 1) : 8LL * sms);
  for (int pass = 0; pass < kSumPasses; ++pass) {
    sum_select_kernel<<<grid, kSumThreads, 0, s>>>(p, pass);
    rc = check_launch("sum_select_kernel");
    if (rc != EKV_OK) return rc;
  }
  sum_ties_kernel<<<rows, kSumThreads, 0, s>>>(p);
  rc = check_launch("sum_ties_kernel");
  if (rc != EKV_OK) return rc;
  sum_quota_kernel<<<rows, kSumThreads, 0, s>>>(p);
  return check_launch("sum_quota_kernel");
}
