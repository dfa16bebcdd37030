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
//   1. sum_prep_kernel, one CTA per row (its scores staged in shared memory): total_r exactly as
//      numpy.add.reduce computes it (pairwise over leaves of at most 128 values, eight accumulators
//      per leaf), then the 63-bit key of every unpinned block's gain (the bits of the non-negative
//      float64 gain) and the histogram of their first digits; the CTA that finishes last sets the
//      budget and picks that digit.
//   2. The rest of an MSB radix select of the `free`-th largest key (digits of 11 bits, the last of
//      8): sum_keys_pass_kernel (a CTA per row) reads every key again, counts per row the keys above
//      the first digit and moves the keys of that digit to a candidate list; passes 2-5 read the
//      candidates only. Each CTA histograms in shared memory and merges; the CTA that finishes last picks the
//      digit. No CTA waits for another.
//   3. sum_ties_kernel over the candidates: keys above the threshold per row and ties per block
//      index; the CTA that finishes last finds the index i* at which the ties needed run out (ties
//      are taken from the highest index down) and how many of the ties at i* are taken.
//   4. sum_kept_kernel over the candidates (ties above i*, rows tied at i*) and sum_quota_kernel, one
//      CTA, which hands the ties at i* to the earliest rows and writes q_r.
#include "ekv_common.cuh"
#include "pairwise.cuh"
#include "pins.cuh"
#include "sum_state.cuh"

namespace ekv {

constexpr int kSumThreads = 256;
constexpr int kSumBins = 2048;  // digits of 11 bits (the last of 8)
constexpr int kSumPasses = 6;
constexpr int kSumMaxWidth = 32768;
constexpr int kSumMaxRows = 1 << 17;  // a candidate's place is (row << 15) | block

struct SumParams {
  const void* scores;          // float or double [.][score_s0] (sum_prep_kernel<float> / <double>)
  int64_t score_s0;
  const int32_t* score_rows;   // may be NULL: row r's scores are scores row score_rows[r]
  const double* weights;
  const int32_t* row_blocks;
  const int32_t* measured;
  int recent, cap;
  double fraction;
  long long budget;
  int rows, width;
  int32_t* quota;
  uint8_t* mask_out;  // may be NULL: the committed mask [rows][mask_s0], written straight from the threshold
  int64_t mask_s0;
  // workspace
  SumState* state;
  unsigned int* hist;        // [kSumBins]
  unsigned int* ties;        // [width] ties at each block index
  int* row_above;            // [rows] keys above the threshold
  int* row_kept;             // [rows] ties above i*
  int* row_at;               // [rows] 1: a tie at i*
  double* total;             // [rows]
  double* weight;            // [rows]
  int* row_n;                // [rows] blocks of a request, 0 for a row that is not one
  int* row_ps;               // [rows] pin start
  unsigned long long* keys;  // [rows][width] keys of the unpinned blocks [1, ps)
  unsigned long long* cand_key;  // [rows * width]
  unsigned int* cand_at;         // [rows * width] (row << 15) | block
  // float64 rows that already hold each request's shares, a pinned block marked by +inf (the pinned
  // allocation, ekv_allocate_pinned_f64): no total is taken, and a pinned block outranks every gain
  bool presummed;
  const long long* budget_add;  // may be NULL: blocks added on the device to a budget given as a count
  // the quotas are wanted (their counts need every tie pass); without them, a select that ended exactly on the
  // threshold (every key with the prefix taken) leaves nothing for the tie passes to decide
  bool need_ties;
};

struct SumLayout {
  size_t state, hist, ties, row_above, row_kept, row_at, zeroed, total, weight, row_n, row_ps, keys, cand_key,
      cand_at, bytes;
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
  l.row_above = take((size_t)rows * 4);
  l.row_kept = take((size_t)rows * 4);
  l.row_at = take((size_t)rows * 4);
  l.zeroed = o;  // everything before this starts at zero
  l.total = take((size_t)rows * 8);
  l.weight = take((size_t)rows * 8);
  l.row_n = take((size_t)rows * 4);
  l.row_ps = take((size_t)rows * 4);
  l.keys = take((size_t)rows * width * 8);
  l.cand_key = take((size_t)rows * width * 8);
  l.cand_at = take((size_t)rows * width * 4);
  l.bytes = o;
  return l;
}

// max(score, 0) in float64; NaN counts as 0, as the controller passes it (observe/controller.py:337).
__device__ __forceinline__ double clamped(float s) { return s > 0.f ? (double)s : 0.0; }
__device__ __forceinline__ double clamped(double s) { return s > 0.0 ? s : 0.0; }

// The order-preserving key of request r's gain at a block with score s: the bits of the
// non-negative float64 gain (0 for a gain of +-0), each operation rounded as NumPy rounds it.
// The key of a pinned block in a presummed row: the bits of +inf, above every finite gain.
constexpr unsigned long long kPinnedKey = 0x7ff0000000000000ull;

template <typename S>
__device__ __forceinline__ unsigned long long gain_key(S s, double total, double w, int n) {
  const double share = total > 0.0 ? __ddiv_rn(clamped(s), total) : __ddiv_rn(1.0, (double)(n > 1 ? n : 1));
  const double g = __dmul_rn(w, share);
  return g > 0.0 ? (unsigned long long)__double_as_longlong(g) : 0ull;
}

// The digits of the 63-bit keys, most significant first: bits 52-62 (the exponent), 41-51, 30-40, 19-29,
// 8-18 and 0-7. (A first digit of 13 bits leaves a quarter of the candidates, but the rows' finer
// histograms put four times as many atomics on the global one, and the pass costs more than it saves.)
__device__ __forceinline__ void digit_of(int pass, int& shift, unsigned long long& dmask) {
  shift = pass < 5 ? 52 - 11 * pass : 0;
  dmask = pass < 5 ? 2047ull : 255ull;
}

// Whether this CTA is the last of the grid to get here (after its writes are fenced).
__device__ __forceinline__ bool last_cta(unsigned int* ticket, bool* s_last) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *s_last = atomicAdd(ticket, 1u) == gridDim.x * gridDim.y - 1;
  __syncthreads();
  if (*s_last) __threadfence();
  return *s_last;
}

// In the last CTA: the digit holding the k-th largest of the keys counted in `hist` (thread t owns
// bins [kPer t, kPer t + kPer)); clears `hist` and updates the threshold.
template <int kPer = kSumBins / kSumThreads>
__device__ void pick_digit(SumState* st, unsigned int* hist, int pass) {
  __shared__ long long s_w[kSumThreads / 32];
  __shared__ int s_pick;
  __shared__ long long s_above;
  __shared__ unsigned int s_count;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int shift;
  unsigned long long dmask;
  digit_of(pass, shift, dmask);
  unsigned int h[kPer];
  long long sum = 0;
#pragma unroll
  for (int j = 0; j < kPer; j += 4) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(hist + kPer * tid + j));
    h[j] = v.x, h[j + 1] = v.y, h[j + 2] = v.z, h[j + 3] = v.w;
    sum += (long long)v.x + v.y + v.z + v.w;
  }
  long long above = sum;  // this thread's bins and those of the lanes above it
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
  for (int j = kPer - 1; j >= 0; --j) {
    if (gt < k && gt + h[j] >= k) {
      s_pick = kPer * tid + j;
      s_above = gt;
      s_count = h[j];
    }
    gt += h[j];
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kPer; j += 4) *reinterpret_cast<uint4*>(hist + kPer * tid + j) = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    const long long k2 = k - s_above;
    st->prefix |= (unsigned long long)s_pick << shift;
    st->mask |= dmask << shift;
    st->k = k2;
    st->exact = (long long)s_count == k2;  // every key with the prefix is taken
    st->found = st->exact || pass == kSumPasses - 1;
  }
}

// One CTA per row: the total (numpy's pairwise sum, pairwise.cuh), the keys, the pins; the CTA that
// finishes last sets the budget.
template <typename S>
__global__ void __launch_bounds__(kSumThreads) sum_prep_kernel(const SumParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  extern __shared__ __align__(16) unsigned char sum_smem[];
  S* s_x = reinterpret_cast<S*>(sum_smem);  // [width]: the row's scores, then the pairwise sum's scratch
  const PairwiseScratch s_tree =
      pairwise_scratch(sum_smem + ((size_t)p.width * sizeof(S) + 15) / 16 * 16, pairwise_slots(p.width));
  __shared__ unsigned int s_hist[kSumBins];
  __shared__ double s_total;
  __shared__ bool s_last;
  const int r = blockIdx.x, tid = threadIdx.x;
  int n = p.row_blocks[r];
  const bool request = n > p.cap && n > 0;
  if (n > p.width) n = p.width;
  const S* xg = static_cast<const S*>(p.scores) + (p.score_rows != nullptr ? (int64_t)p.score_rows[r] : (int64_t)r) * p.score_s0;
  const int ps = request ? pin_start(n, p.recent, p.measured, r) : 0;
  const double w = p.weights ? p.weights[r] : 1.0;
  for (int i = tid; i < kSumBins; i += kSumThreads) s_hist[i] = 0;
  if (request) {
    stage_row<kSumThreads>(s_x, xg, n);
    const double sum = p.presummed ? 1.0 : block_pairwise_sum<kSumThreads>(s_tree, n, [&](int i) { return clamped(s_x[i]); });
    if (tid == 0) s_total = sum;
    __syncthreads();
    const double total = s_total;
    unsigned long long* kr = p.keys + (int64_t)r * p.width;
    int shift0;
    unsigned long long dmask0;
    digit_of(0, shift0, dmask0);
    for (int b = 1 + tid; b < ps; b += kSumThreads) {  // the keys and pass 0 of the select
      const unsigned long long key = p.presummed && isinf((double)s_x[b]) ? kPinnedKey : gain_key(s_x[b], total, w, n);
      kr[b] = key;
      atomicAdd(&s_hist[(key >> shift0) & dmask0], 1u);
    }
  }
  __syncthreads();
  for (int i = tid; i < kSumBins; i += kSumThreads)
    if (s_hist[i]) atomicAdd(&p.hist[i], s_hist[i]);
  if (tid == 0) {
    if (request) {
      atomicAdd((unsigned long long*)&p.state->total_open, (unsigned long long)(ps > 1 ? ps - 1 : 0));
      atomicAdd((unsigned long long*)&p.state->must, (unsigned long long)pin_count(n, ps));
      atomicAdd((unsigned long long*)&p.state->blocks, (unsigned long long)n);
    }
    p.total[r] = request ? s_total : 0.0;
    p.weight[r] = w;
    p.row_n[r] = request ? n : 0;
    p.row_ps[r] = ps;
  }
  if (!last_cta(&p.state->ticket, &s_last)) return;
  // the budget (controller.py:435-437) and what to do with it (allocation.py:64-67, :98-104)
  SumState* st = p.state;
  if (tid == 0) {
    const long long must = *(volatile long long*)&st->must, blocks = *(volatile long long*)&st->blocks;
    const long long total_open = *(volatile long long*)&st->total_open;
    long long budget = p.budget;
    if (budget < 0) {
      budget = (long long)ceil(p.fraction * (double)blocks);
      if (budget < must) budget = must;
    } else if (p.budget_add != nullptr) {
      budget += *p.budget_add;
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
    st->ticket = 0;
  }
  __syncthreads();
  if (st->mode == kSumSelect) pick_digit(st, p.hist, 0);  // pass 0 of the select
}

// Pass 1 over every key: a CTA per row. It counts the row's keys above the digit of pass 0 and the next digit
// of the keys of that digit, and appends those keys to the candidates: gathered in shared memory as they are
// met, then copied to the row's place in the list (one atomic); a row with more than kSumStage of them is
// read again (from L2) to write them there.
__global__ void __launch_bounds__(kSumThreads) sum_keys_pass_kernel(const SumParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  constexpr int pass = 1;
  constexpr int kPer = 8;  // keys a thread has in flight
  constexpr int kSumStage = 2048;
  __shared__ unsigned int s_hist[kSumBins];
  __shared__ unsigned long long s_ckey[kSumStage];
  __shared__ unsigned int s_cat[kSumStage];
  __shared__ int s_warp[kSumThreads / 32 + 1];  // each warp's candidates, then the warps' places
  __shared__ int s_above;
  __shared__ unsigned int s_base, s_staged;
  __shared__ bool s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.x;
  SumState* st = p.state;
  if (st->mode != kSumSelect) return;  // (uniform over the grid)
  const bool histogram = !st->found;
  int shift;
  unsigned long long dmask;
  digit_of(pass, shift, dmask);
  int shift0;
  unsigned long long dmask0;
  digit_of(0, shift0, dmask0);
  const unsigned long long top_mask = dmask0 << shift0, top_want = st->prefix & top_mask;
  for (int i = tid; i < kSumBins; i += kSumThreads) s_hist[i] = 0;
  if (tid == 0) s_above = 0, s_staged = 0;
  __syncthreads();
  const int n = p.row_n[r], ps = n > 0 ? p.row_ps[r] : 0;
  const unsigned long long* kr = p.keys + (int64_t)r * p.width;
  int above = 0, mine = 0;  // keys above the digit; this warp's candidates (the same in every lane)
  for (int base = 1; base < ps; base += kPer * kSumThreads) {  // (the same trip count for every thread)
    unsigned long long keys[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int b = base + j * kSumThreads + tid;
      keys[j] = b < ps ? kr[b] : 0ull;
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int b = base + j * kSumThreads + tid;
      const unsigned long long top = keys[j] & top_mask;
      const bool cand = b < ps && top == top_want;
      above += b < ps && top > top_want;
      if (cand && histogram) atomicAdd(&s_hist[(keys[j] >> shift) & dmask], 1u);
      const unsigned int ballot = __ballot_sync(kFullMask, cand);
      if (ballot) {
        unsigned int at = 0;
        if (lane == 0) at = atomicAdd(&s_staged, (unsigned int)__popc(ballot));
        at = __shfl_sync(kFullMask, at, 0) + (unsigned int)__popc(ballot & lanes_below());
        if (cand && at < (unsigned int)kSumStage) {
          s_ckey[at] = keys[j];
          s_cat[at] = ((unsigned int)r << 15) | (unsigned int)b;
        }
      }
      mine += __popc(ballot);
    }
  }
  for (int off = 16; off > 0; off >>= 1) above += __shfl_xor_sync(kFullMask, above, off);
  if (lane == 0) {
    s_warp[warp] = mine;
    if (above) atomicAdd(&s_above, above);
  }
  __syncthreads();
  if (tid == 0) {
    int total = 0;
    for (int w = 0; w < kSumThreads / 32; ++w) {
      const int c = s_warp[w];
      s_warp[w] = total;
      total += c;
    }
    s_base = total ? atomicAdd(&st->n_cand, (unsigned int)total) : 0u;
    if (s_above) atomicAdd(&p.row_above[r], s_above);
  }
  __syncthreads();
  const unsigned int staged = s_staged;
  if (staged <= (unsigned int)kSumStage) {
    for (unsigned int i = tid; i < staged; i += kSumThreads) {
      p.cand_key[s_base + i] = s_ckey[i];
      p.cand_at[s_base + i] = s_cat[i];
    }
  } else if (mine) {  // the second sweep: this warp's candidates at its place, in the order it met them
    unsigned int at = s_base + (unsigned int)s_warp[warp];
    for (int base = 1; base < ps; base += kPer * kSumThreads) {
      unsigned long long keys[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int b = base + j * kSumThreads + tid;
        keys[j] = b < ps ? __ldcg(kr + b) : 0ull;
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int b = base + j * kSumThreads + tid;
        const bool cand = b < ps && (keys[j] & top_mask) == top_want;
        const unsigned int ballot = __ballot_sync(kFullMask, cand);
        if (cand) {
          const unsigned int i = at + (unsigned int)__popc(ballot & lanes_below());
          p.cand_key[i] = keys[j];
          p.cand_at[i] = ((unsigned int)r << 15) | (unsigned int)b;
        }
        at += (unsigned int)__popc(ballot);
      }
    }
  }
  if (histogram)
    for (int i = tid; i < kSumBins; i += kSumThreads)
      if (s_hist[i]) atomicAdd(&p.hist[i], s_hist[i]);
  if (!last_cta(&st->ticket, &s_last)) return;
  if (histogram) pick_digit(st, p.hist, pass);
  if (tid == 0) st->ticket = 0;
}

// Passes 2-5 over the candidates (the keys with pass 0's digit).
__global__ void __launch_bounds__(kSumThreads) sum_cand_pass_kernel(const SumParams p, int pass) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  __shared__ unsigned int s_hist[kSumBins];
  __shared__ bool s_last;
  const int tid = threadIdx.x;
  SumState* st = p.state;
  if (st->mode != kSumSelect || st->found) return;
  int shift;
  unsigned long long dmask;
  digit_of(pass, shift, dmask);
  const unsigned long long prefix = st->prefix, mask = st->mask;
  for (int i = tid; i < kSumBins; i += kSumThreads) s_hist[i] = 0;
  __syncthreads();
  const unsigned int count = st->n_cand;
  for (unsigned int i = blockIdx.x * kSumThreads + tid; i < count; i += gridDim.x * kSumThreads) {
    const unsigned long long key = p.cand_key[i];
    if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & dmask], 1u);
  }
  __syncthreads();
  for (int i = tid; i < kSumBins; i += kSumThreads)
    if (s_hist[i]) atomicAdd(&p.hist[i], s_hist[i]);
  if (!last_cta(&st->ticket, &s_last)) return;
  pick_digit(st, p.hist, pass);
  if (tid == 0) st->ticket = 0;
}

// Over the candidates: keys above the threshold per row, ties per block index; the CTA that
// finishes last finds i*, the lowest block index of the ties taken, and m, the ties taken there.
__global__ void __launch_bounds__(kSumThreads) sum_ties_kernel(const SumParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  __shared__ long long s_w[kSumThreads / 32];
  __shared__ bool s_last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  SumState* st = p.state;
  if (st->mode != kSumSelect || (!p.need_ties && st->exact)) return;  // (uniform over the grid)
  const unsigned long long prefix = st->prefix, mask = st->mask;
  const unsigned int count = st->n_cand;
  for (unsigned int base = blockIdx.x * kSumThreads; base < count; base += gridDim.x * kSumThreads) {
    const unsigned int i = base + tid;  // (warp-uniform trip count)
    const bool in = i < count;
    const unsigned long long key = in ? p.cand_key[i] & mask : 0ull;
    const unsigned int at = in ? p.cand_at[i] : 0u;
    const bool up = in && key > prefix;
    // a CTA of the keys pass moved one row's candidates together: count a row once per warp
    const unsigned int row = up ? at >> 15 : 0xffffffffu;
    const unsigned int same = __match_any_sync(kFullMask, row);
    if (up && lane == __ffs(same) - 1) atomicAdd(&p.row_above[row], __popc(same));
    if (in && key == prefix) atomicAdd(&p.ties[at & 32767u], 1u);
  }
  if (!last_cta(&st->ticket, &s_last)) return;
  // ties are taken from the highest block index down; thread t owns indices [t * per, t * per + per): up to
  // 32 of them held in registers (read as eight 16-byte loads, all in flight), more read eight at a time
  constexpr int kTieRegs = 32, kTieChunk = 8;
  const bool in_regs = p.width <= kSumThreads * kTieRegs;
  const int per = in_regs ? kTieRegs : (p.width + kSumThreads - 1) / kSumThreads;
  const int lo = min(tid * per, p.width), hi = min(lo + per, p.width);
  unsigned int t_reg[kTieRegs];
  long long cnt = 0;
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < kTieRegs; j += 4) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (lo + j + 3 < hi) {
        v = __ldcg(reinterpret_cast<const uint4*>(p.ties + lo + j));
      } else {
        v.x = lo + j < hi ? __ldcg(p.ties + lo + j) : 0u;
        v.y = lo + j + 1 < hi ? __ldcg(p.ties + lo + j + 1) : 0u;
        v.z = lo + j + 2 < hi ? __ldcg(p.ties + lo + j + 2) : 0u;
      }
      t_reg[j] = v.x, t_reg[j + 1] = v.y, t_reg[j + 2] = v.z, t_reg[j + 3] = v.w;
    }
#pragma unroll
    for (int j = 0; j < kTieRegs; ++j) cnt += t_reg[j];
  } else {
    for (int c0 = lo; c0 < hi; c0 += kTieChunk) {
      unsigned int t[kTieChunk];
#pragma unroll
      for (int j = 0; j < kTieChunk; ++j) t[j] = c0 + j < hi ? __ldcg(p.ties + c0 + j) : 0u;
#pragma unroll
      for (int j = 0; j < kTieChunk; ++j) cnt += t[j];
    }
  }
  long long above = cnt;  // this thread's indices and those of the lanes above it
  for (int off = 1; off < 32; off <<= 1) {
    const long long v = __shfl_down_sync(kFullMask, above, off);
    if (lane + off < 32) above += v;
  }
  if (lane == 0) s_w[warp] = above;
  __syncthreads();
  long long taken = above - cnt;  // ties at indices >= hi
  for (int w2 = warp + 1; w2 < kSumThreads / 32; ++w2) taken += s_w[w2];
  const long long k = st->k;
  if (taken < k && taken + cnt >= k) {
    if (in_regs) {
      bool done = false;
#pragma unroll
      for (int j = kTieRegs - 1; j >= 0; --j) {
        if (done || lo + j >= hi) continue;
        const long long c = t_reg[j];
        if (taken + c >= k) {
          st->istar = lo + j;
          st->m = k - taken;
          done = true;
        } else {
          taken += c;
        }
      }
    } else {
      bool done = false;
      for (int c1 = hi; c1 > lo && !done; c1 -= kTieChunk) {  // chunks from the top, eight loads in flight
        const int c0 = max(c1 - kTieChunk, lo);
        unsigned int t[kTieChunk];
#pragma unroll
        for (int j = 0; j < kTieChunk; ++j) t[j] = c0 + j < c1 ? __ldcg(p.ties + c0 + j) : 0u;
#pragma unroll
        for (int j = kTieChunk - 1; j >= 0; --j) {
          if (done || c0 + j >= c1) continue;
          const long long c = t[j];
          if (taken + c >= k) {
            st->istar = c0 + j;
            st->m = k - taken;
            done = true;
          } else {
            taken += c;
          }
        }
      }
    }
  }
  if (tid == 0) st->ticket = 0;
}

// Over the candidates: each row's ties above i* and whether it ties at i*.
__global__ void __launch_bounds__(kSumThreads) sum_kept_kernel(const SumParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  const int tid = threadIdx.x;
  const SumState* st = p.state;
  if (st->mode != kSumSelect || (!p.need_ties && st->exact)) return;
  const unsigned long long prefix = st->prefix, mask = st->mask;
  const unsigned int istar = (unsigned int)st->istar, count = st->n_cand;
  const int lane = tid & 31;
  for (unsigned int base = blockIdx.x * kSumThreads; base < count; base += gridDim.x * kSumThreads) {
    const unsigned int i = base + tid;  // (warp-uniform trip count)
    const bool tie = i < count && (p.cand_key[i] & mask) == prefix;
    const unsigned int at = tie ? p.cand_at[i] : 0u, b = at & 32767u, r = at >> 15;
    const bool above = tie && b > istar;
    const unsigned int same = __match_any_sync(kFullMask, above ? r : 0xffffffffu);
    if (above && lane == __ffs(same) - 1) atomicAdd(&p.row_kept[r], __popc(same));
    if (tie && b == istar) p.row_at[r] = 1;
  }
}

// One CTA: the quotas; the m ties at i* go to the earliest rows that tie there.
__global__ void __launch_bounds__(1024) sum_quota_kernel(const SumParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  __shared__ int s_scan[1024 / 32 + 1];
  const int tid = threadIdx.x;
  const SumState* st = p.state;
  const int mode = st->mode;
  if (!p.need_ties && (mode != kSumSelect || st->exact)) return;  // no quotas wanted, no ties to hand out
  const long long m = st->m;
  int carry = 0;
  for (int base = 0; base < p.rows; base += 1024) {
    const int r = base + tid;
    const bool in = r < p.rows;
    const int n = in ? p.row_n[r] : 0;
    const int at = in && n > 0 && mode == kSumSelect ? p.row_at[r] : 0;
    int total = 0;
    const int before = carry + block_exclusive_scan<1024>(at, s_scan, &total);
    carry += total;
    if (!in) continue;
    if (n == 0) {
      if (p.quota) p.quota[r] = -1;  // not a request: it reads in full
    } else if (mode != kSumSelect) {
      const int ps = p.row_ps[r];
      if (p.quota) p.quota[r] = mode == kSumAll ? (ps > 1 ? ps - 1 : 0) : 0;
    } else {
      const int take = at && before < m ? 1 : 0;
      if (p.quota) p.quota[r] = p.row_above[r] + p.row_kept[r] + take;
      p.row_at[r] = take;  // from here on: the row's tie at i* is taken (sum_mask_kernel, the view)
    }
  }
}

// The committed mask straight from the threshold, without ranking any row: block b of request r is
// kept when it is pinned (block 0 and [ps, n)), past the request, or unpinned with a gain key above the
// threshold, or equal to it at an index above i*, or at i* when the row's tie there is taken. Grid
// (width / kSumMaskSpan, rows); a thread takes kSumMaskGroups groups of four adjacent positions, every
// key loaded before any is used (fewer, fuller CTAs: the pass is a single wave of loads, not several).
constexpr int kSumMaskGroups = 4;
constexpr int kSumMaskSpan = 4 * kSumMaskGroups * kSumThreads;
__global__ void __launch_bounds__(kSumThreads) sum_mask_kernel(const SumParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  const int r = blockIdx.y;
  const SumState* st = p.state;
  const int mode = st->mode;
  const unsigned long long prefix = st->prefix, mask = st->mask;
  const int istar = st->istar;
  const int n = p.row_n[r], ps = p.row_ps[r];
  const bool take = p.row_at[r] != 0;
  const unsigned long long* kr = p.keys + (int64_t)r * p.width;
  uint8_t* out = p.mask_out + (int64_t)r * p.mask_s0;
  const int c0 = blockIdx.x * kSumMaskSpan + 4 * threadIdx.x;  // group g starts at c0 + g * 4 * kSumThreads
  unsigned long long km[kSumMaskGroups][4];  // (predicated loads, no early exit between them)
#pragma unroll
  for (int g = 0; g < kSumMaskGroups; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = c0 + g * 4 * kSumThreads + j;
      const bool ranked = mode == kSumSelect && n > 0 && b >= 1 && b < ps && b < p.width;
      km[g][j] = ranked ? kr[b] & mask : 0ull;
    }
#pragma unroll
  for (int g = 0; g < kSumMaskGroups; ++g) {
    const int b0 = c0 + g * 4 * kSumThreads;
    uint32_t bytes = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = b0 + j;
      bool keep = true;  // not a request, a pin, or past the request
      if (n > 0 && b >= 1 && b < ps) {
        if (mode == kSumAll) {
          keep = true;
        } else if (mode == kSumNone) {
          keep = false;
        } else {
          const unsigned long long k = km[g][j];
          keep = k > prefix || (k == prefix && (b > istar || (b == istar && take)));
        }
      }
      bytes |= (keep ? 1u : 0u) << (8 * j);
    }
    if (b0 + 4 <= p.width && (reinterpret_cast<uintptr_t>(out + b0) & 3) == 0) {
      *reinterpret_cast<uint32_t*>(out + b0) = bytes;
    } else {
      for (int j = 0; j < 4 && b0 + j < p.width; ++j) out[b0 + j] = (uint8_t)(bytes >> (8 * j));
    }
  }
}

}  // namespace ekv

using namespace ekv;

// The view a shared-budget build writes (ekv_view_build_sum_budget).
struct SumViewOut {
  const int32_t* table;
  int64_t table_s0;
  const int32_t* seq_lens;
  const uint8_t* full_rows;
  const uint8_t* released;
  int64_t released_s0;
  int block_size;
  int32_t* view;
  int64_t view_s0;
  int32_t* view_lens;
};

extern "C" size_t ekv_allocate_sum_workspace_bytes(int rows, int width) {
  if (rows <= 0 || width <= 0) return 0;
  return sum_layout(rows, width).bytes;
}

template <typename S>
static int allocate_sum(const S* scores, int64_t score_stride, const int32_t* score_rows, const double* weights,
                        const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                        int cap_above_blocks, double budget_fraction, int64_t budget, int rows, int width,
                        int32_t* quota, uint8_t* mask_out, int64_t mask_stride, void* workspace,
                        size_t workspace_bytes, void* stream, bool presummed = false,
                        const long long* budget_add = nullptr, const SumViewOut* view = nullptr) {
  constexpr int max_width = sizeof(S) == 8 ? kSumMaxWidth / 2 : kSumMaxWidth;  // the prep kernel stages a row
  clear_error();
  if (!scores || !row_blocks || (!quota && !mask_out && !view)) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0) return fail(EKV_EINVAL, "rows and width must be positive");
  if (width > max_width) return fail(EKV_ENOTSUP, "width %d > %d", width, max_width);
  if (rows > kSumMaxRows) return fail(EKV_ENOTSUP, "rows %d > %d", rows, kSumMaxRows);
  if (score_stride < width) return fail(EKV_EINVAL, "score_stride %lld < width %d", (long long)score_stride, width);
  if (mask_out && mask_stride < width) return fail(EKV_EINVAL, "mask_stride %lld < width %d", (long long)mask_stride, width);
  if (recent_blocks < -1 || cap_above_blocks < -1) return fail(EKV_EINVAL, "invalid controller settings");
  if (budget < 0 && !(budget_fraction > 0.0 && budget_fraction <= 1.0))
    return fail(EKV_EINVAL, "the budget fraction must be in (0, 1]");
  const SumLayout l = sum_layout(rows, width);
  if (!workspace || workspace_bytes < l.bytes)
    return fail(EKV_ERANGE, "the sum workspace holds %zu bytes, the call needs %zu", workspace_bytes, l.bytes);
  if ((uintptr_t)workspace & 255) return fail(EKV_EINVAL, "the sum workspace must be 256-byte aligned");
  uint8_t* base = static_cast<uint8_t*>(workspace);
  SumParams p{};
  p.scores = scores; p.score_s0 = score_stride; p.score_rows = score_rows; p.weights = weights; p.row_blocks = row_blocks;
  p.measured = measured_blocks; p.recent = recent_blocks; p.cap = cap_above_blocks;
  p.fraction = budget_fraction; p.budget = (long long)budget; p.rows = rows; p.width = width; p.quota = quota;
  p.mask_out = mask_out; p.mask_s0 = mask_stride;
  p.presummed = presummed; p.budget_add = budget_add; p.need_ties = quota != nullptr;
  p.state = reinterpret_cast<SumState*>(base + l.state);
  p.hist = reinterpret_cast<unsigned int*>(base + l.hist);
  p.ties = reinterpret_cast<unsigned int*>(base + l.ties);
  p.row_above = reinterpret_cast<int*>(base + l.row_above);
  p.row_kept = reinterpret_cast<int*>(base + l.row_kept);
  p.row_at = reinterpret_cast<int*>(base + l.row_at);
  p.total = reinterpret_cast<double*>(base + l.total);
  p.weight = reinterpret_cast<double*>(base + l.weight);
  p.row_n = reinterpret_cast<int*>(base + l.row_n);
  p.row_ps = reinterpret_cast<int*>(base + l.row_ps);
  p.keys = reinterpret_cast<unsigned long long*>(base + l.keys);
  p.cand_key = reinterpret_cast<unsigned long long*>(base + l.cand_key);
  p.cand_at = reinterpret_cast<unsigned int*>(base + l.cand_at);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int device = 0, sms = 0;
  const int dev_rc = current_device(&device);
  if (dev_rc != EKV_OK) return dev_rc;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("cudaDeviceGetAttribute");
  if (cudaMemsetAsync(base, 0, l.zeroed, s) != cudaSuccess) return check_launch("cudaMemsetAsync(sum workspace)");
  const size_t prep_smem = ((size_t)width * sizeof(S) + 15) / 16 * 16 + pairwise_bytes(pairwise_slots(width));
  static size_t configured[kMaxDevices] = {};
  if (configured[device] < prep_smem) {
    if (cudaFuncSetAttribute(sum_prep_kernel<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)prep_smem) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(sum_prep_kernel)");
    configured[device] = prep_smem;
  }
  launch_chained(sum_prep_kernel<S>, dim3(rows), dim3(kSumThreads), prep_smem, s, p);
  int rc = check_launch("sum_prep_kernel");
  if (rc == EKV_OK) {
    launch_chained(sum_keys_pass_kernel, dim3(rows), dim3(kSumThreads), 0, s, p);
    rc = check_launch("sum_keys_pass_kernel");
  }
  const int cand_grid = 2 * sms;
  for (int pass = 2; pass < kSumPasses && rc == EKV_OK; ++pass) {
    launch_chained(sum_cand_pass_kernel, dim3(cand_grid), dim3(kSumThreads), 0, s, p, pass);
    rc = check_launch("sum_cand_pass_kernel");
  }
  if (rc != EKV_OK) return rc;
  launch_chained(sum_ties_kernel, dim3(cand_grid), dim3(kSumThreads), 0, s, p);
  if ((rc = check_launch("sum_ties_kernel")) != EKV_OK) return rc;
  launch_chained(sum_kept_kernel, dim3(cand_grid), dim3(kSumThreads), 0, s, p);
  if ((rc = check_launch("sum_kept_kernel")) != EKV_OK) return rc;
  launch_chained(sum_quota_kernel, dim3(1), dim3(1024), 0, s, p);
  if ((rc = check_launch("sum_quota_kernel")) != EKV_OK) return rc;
  if (view != nullptr)  // the view (and the mask) straight from the threshold
    return launch_sum_view(view->table, view->table_s0, view->seq_lens, view->full_rows, view->released,
                           view->released_s0, rows, width, view->block_size, view->view, view->view_s0,
                           view->view_lens, mask_out, mask_stride, p.state, p.keys, p.row_n, p.row_ps, p.row_at, s);
  if (mask_out == nullptr) return rc;
  launch_chained(sum_mask_kernel, dim3(cdiv(width, kSumMaskSpan), rows), dim3(kSumThreads), 0, s, p);
  return check_launch("sum_mask_kernel");
}

namespace ekv {

// The `sum` objective over presummed float64 rows (see SumParams::presummed), its mask written straight
// from the threshold.
int presummed_sum(const double* shares, int64_t share_s0, const double* weights, const int32_t* row_blocks,
                  const int32_t* measured, long long budget, const long long* budget_add, int rows, int width,
                  int32_t* quota, uint8_t* mask_out, int64_t mask_s0, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream) {
  return allocate_sum<double>(shares, share_s0, nullptr, weights, row_blocks, measured, -1, -1, 0.0, budget, rows,
                              width, quota, mask_out, mask_s0, workspace, workspace_bytes, stream, true, budget_add);
}

}  // namespace ekv

extern "C" int ekv_allocate_sum(const float* scores, int64_t score_stride, const double* weights,
                                const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                                int cap_above_blocks, double budget_fraction, int64_t budget, int rows, int width,
                                int32_t* quota, void* workspace, size_t workspace_bytes, void* stream) {
  return allocate_sum<float>(scores, score_stride, nullptr, weights, row_blocks, measured_blocks, recent_blocks,
                             cap_above_blocks, budget_fraction, budget, rows, width, quota, nullptr, 0, workspace,
                             workspace_bytes, stream);
}

extern "C" int ekv_allocate_sum_f64(const double* scores, int64_t score_stride, const int32_t* score_rows,
                                    const double* weights, const int32_t* row_blocks, const int32_t* measured_blocks,
                                    int recent_blocks, int cap_above_blocks, double budget_fraction, int64_t budget,
                                    int rows, int width, int32_t* quota, uint8_t* mask_out, int64_t mask_stride,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  return allocate_sum<double>(scores, score_stride, score_rows, weights, row_blocks, measured_blocks,
                              recent_blocks, cap_above_blocks, budget_fraction, budget, rows, width, quota,
                              mask_out, mask_stride, workspace, workspace_bytes, stream);
}

extern "C" int ekv_view_build_sum_budget(const void* scores, int score_bytes, int64_t score_stride,
                                         const int32_t* score_rows, const double* weights, const int32_t* row_blocks,
                                         const int32_t* measured_blocks, int recent_blocks, int cap_above_blocks,
                                         double budget_fraction, int64_t budget, const int32_t* table,
                                         int64_t table_stride, const int32_t* seq_lens, const uint8_t* full_rows,
                                         const uint8_t* released, int64_t released_stride, int rows, int width,
                                         int block_size, int32_t* view, int64_t view_stride, int32_t* view_lens,
                                         uint8_t* mask_out, int64_t mask_stride, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  clear_error();
  if (!table || !seq_lens || !view || !view_lens) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (score_bytes != 4 && score_bytes != 8) return fail(EKV_EINVAL, "score_bytes %d: 4 (float32) or 8 (float64)", score_bytes);
  if (score_bytes == 4 && score_rows) return fail(EKV_EINVAL, "score_rows reads float64 scores only");
  if (block_size <= 0) return fail(EKV_EINVAL, "block_size must be positive");
  if (width > 16384) return fail(EKV_ENOTSUP, "width %d > 16384 (a view row is staged in shared memory)", width);
  if (table_stride < width || view_stride < width) return fail(EKV_EINVAL, "a row stride is below the width");
  if (released && released_stride < width) return fail(EKV_EINVAL, "released_stride < width");
  const SumViewOut out{table, table_stride, seq_lens, full_rows, released, released_stride, block_size, view,
                       view_stride, view_lens};
  if (score_bytes == 4)
    return allocate_sum<float>(static_cast<const float*>(scores), score_stride, nullptr, weights, row_blocks,
                               measured_blocks, recent_blocks, cap_above_blocks, budget_fraction, budget, rows, width,
                               nullptr, mask_out, mask_stride, workspace, workspace_bytes, stream, false, nullptr, &out);
  return allocate_sum<double>(static_cast<const double*>(scores), score_stride, score_rows, weights, row_blocks,
                              measured_blocks, recent_blocks, cap_above_blocks, budget_fraction, budget, rows, width,
                              nullptr, mask_out, mask_stride, workspace, workspace_bytes, stream, false, nullptr, &out);
}
