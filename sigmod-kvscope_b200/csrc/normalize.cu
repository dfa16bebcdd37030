// The controller's read of the statistic, on the device: read_tile_rows + normalize_tile_lse
// (observe/tile_shares.py:129-173 and :58-103), for any rows, layers and row lengths.
//
// One CTA per requested row. Per layer it makes two passes over the row's cells (both planes,
// group_rows values per block): the first reduces every query row to an online (max, sum) of
// lse = u + regain over the finite cells below row_blocks, the second adds exp(lse - log total)
// into the row's output, which the CTA owns and uses as its accumulator. A final pass divides by the
// contributors (mean) or by the row total (max). The order of every sum is fixed, so the output is
// deterministic.
#include "ekv_common.cuh"

namespace ekv {

struct NormParams {
  const float* lse;  // m/l table (two planes), or u values (one plane) when log_weights is set
  bool log_weights;
  int table_layers, layers, rows, width, Q;
  const int32_t* row_ids;
  const int32_t* row_blocks;
  int count, tile_blocks, aggregate;
  float* share;
  int32_t* contributors;
};

constexpr int kNormThreads = 256;
constexpr int kNormMaxQ = 256;

__global__ void __launch_bounds__(kNormThreads) normalize_kernel(const NormParams p) {
  __shared__ float s_m[kNormThreads], s_s[kNormThreads];
  __shared__ float s_lse[kNormMaxQ];
  __shared__ int s_has[kNormMaxQ];
  __shared__ float s_red[kNormThreads / 32];
  const int i = blockIdx.x;
  const int row = p.row_ids != nullptr ? p.row_ids[i] : i;
  const int rb = p.row_blocks[i];
  const int W = p.width, Q = p.Q, TB = p.tile_blocks;
  float* out = p.share + (size_t)i * W;
  if (row < 0 || row >= p.rows) {  // not a row of the table: no evidence
    for (int b = threadIdx.x; b < W; b += kNormThreads) out[b] = NAN;
    if (p.contributors != nullptr && threadIdx.x == 0) p.contributors[i] = 0;
    return;
  }
  const int n = rb < 0 ? 0 : (rb < W ? rb : W);  // cells at or past the row length are dropped (:88)
  // the partial last tile: its blocks get back the weight of the blocks it lacks (:82-87)
  const int tail_start = (rb / TB) * TB;
  const bool has_tail = rb % TB != 0;
  const float regain = has_tail ? logf((float)TB / (float)max(rb - tail_start, 1)) : 0.f;
  const float log_tb = logf((float)TB);
  const size_t plane = (size_t)p.table_layers * p.rows * W * Q;
  const bool agg_max = p.aggregate == EKV_AGG_MAX;
  // A thread keeps one query row j = tid % Q across the first pass, so its partial is per j.
  const int lanes_per_j = kNormThreads / Q;  // >= 1 since Q <= kNormThreads
  const int j_of = threadIdx.x % Q;
  const int b_first = threadIdx.x / Q;
  const bool pass1_thread = threadIdx.x < lanes_per_j * Q;

  for (int b = threadIdx.x; b < W; b += kNormThreads) out[b] = 0.f;
  int contrib = 0;
  for (int layer = 0; layer < p.layers; ++layer) {
    const float* cm = p.lse + ((size_t)layer * p.rows + row) * W * Q;
    const float* cl = cm + plane;
    // u = m + log(l) - log(tile_blocks) of a table cell (tile_shares.py:172-173), or the given u
    auto log_weight = [&](size_t c) -> float {
      return p.log_weights ? cm[c] : cm[c] + logf(cl[c]) - log_tb;
    };
    float m = -INFINITY, s = 0.f;
    if (pass1_thread) {
      for (int b = b_first; b < n; b += lanes_per_j) {
        const float u = log_weight((size_t)b * Q + j_of);
        const float v = u + (has_tail && b >= tail_start ? regain : 0.f);
        if (isfinite(v)) lse_merge(m, s, v, 1.f);
      }
    }
    __syncthreads();  // the previous layer's readers of s_lse/s_has are done
    s_m[threadIdx.x] = m;
    s_s[threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.x < Q) {
      float mj = -INFINITY, sj = 0.f;
      for (int k = 0; k < lanes_per_j; ++k)
        lse_merge(mj, sj, s_m[k * Q + threadIdx.x], s_s[k * Q + threadIdx.x]);
      s_has[threadIdx.x] = mj != -INFINITY;
      s_lse[threadIdx.x] = mj != -INFINITY ? mj + logf(sj) : 0.f;
    }
    __syncthreads();
    for (int j = 0; j < Q; ++j) contrib += s_has[j];
    for (int b = threadIdx.x; b < n; b += kNormThreads) {
      const float rg = has_tail && b >= tail_start ? regain : 0.f;
      float a = 0.f;
      for (int j = 0; j < Q; ++j) {
        if (!s_has[j]) continue;
        const float v = log_weight((size_t)b * Q + j) + rg;
        if (isfinite(v)) {
          const float sh = __expf(v - s_lse[j]);
          a = agg_max ? fmaxf(a, sh) : a + sh;
        }
      }
      out[b] = agg_max ? fmaxf(out[b], a) : out[b] + a;
    }
  }
  float total = 1.f;
  if (agg_max) {
    float part = 0.f;
    for (int b = threadIdx.x; b < n; b += kNormThreads) part += out[b];
    total = block_sum_fixed_order<kNormThreads>(part, s_red);
  }
  for (int b = threadIdx.x; b < W; b += kNormThreads) {
    float v;
    if (contrib == 0) {
      v = NAN;  // no evidence about the row (:103)
    } else if (b >= n) {
      v = 0.f;
    } else if (agg_max) {
      v = total > 0.f ? out[b] / total : 0.f;
    } else {
      v = out[b] / (float)contrib;
    }
    out[b] = v;
  }
  if (p.contributors != nullptr && threadIdx.x == 0) p.contributors[i] = contrib;
}

constexpr int kFinalThreads = 256;

__global__ void __launch_bounds__(kFinalThreads)
    finalize_kernel(const float* acc, const int32_t* contrib, const uint8_t* select, int width,
                    int aggregate, float* out) {
  __shared__ float s_red[kFinalThreads / 32];
  const int row = blockIdx.x;
  const float* a = acc + (size_t)row * width;
  float* o = out + (size_t)row * width;
  const int c = contrib[row];
  const bool none = c == 0 || (select != nullptr && select[row] == 0);
  float total = 1.f;
  if (aggregate == EKV_AGG_MAX) {
    float part = 0.f;
    for (int b = threadIdx.x; b < width; b += kFinalThreads) part += a[b];
    total = block_sum_fixed_order<kFinalThreads>(part, s_red);
  }
  for (int b = threadIdx.x; b < width; b += kFinalThreads) {
    float v;
    if (none) {
      v = NAN;
    } else if (aggregate == EKV_AGG_MAX) {
      v = total > 0.f ? a[b] / total : 0.f;
    } else {
      v = a[b] / (float)c;
    }
    o[b] = v;
  }
}

}  // namespace ekv

using namespace ekv;

extern "C" int ekv_normalize_tile_lse(const float* lse, int table_layers, int layers, int rows,
                                      int width, int group_rows, const int32_t* row_ids,
                                      const int32_t* row_blocks, int count, int tile_blocks,
                                      int aggregate, float* share, int32_t* contributors,
                                      void* stream) {
  clear_error();
  if (aggregate != EKV_AGG_MEAN && aggregate != EKV_AGG_MAX)
    return fail(EKV_EINVAL, "unknown aggregate %d", aggregate);
  if (tile_blocks < 1) return fail(EKV_EINVAL, "tile_blocks must be positive");
  if (rows <= 0 || width <= 0 || group_rows <= 0 || table_layers <= 0)
    return fail(EKV_EINVAL, "rows, width, group_rows and table_layers must be positive");
  if (layers < 0 || layers > table_layers)
    return fail(EKV_ERANGE, "%d layers requested from a table of %d", layers, table_layers);
  if (group_rows > kNormMaxQ) return fail(EKV_ENOTSUP, "group_rows %d > %d", group_rows, kNormMaxQ);
  if (count < 0) return fail(EKV_EINVAL, "negative row count");
  if (count == 0) return EKV_OK;
  if (!lse || !row_ids || !row_blocks || !share) return fail(EKV_EINVAL, "a required pointer is NULL");
  NormParams p{lse, false, table_layers, layers, rows, width, group_rows, row_ids, row_blocks,
               count, tile_blocks, aggregate, share, contributors};
  normalize_kernel<<<count, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("normalize_kernel");
}

extern "C" int ekv_normalize_log_weights(const float* u, int layers, int rows, int width,
                                         int group_rows, const int32_t* row_blocks,
                                         int tile_blocks, int aggregate, float* share,
                                         int32_t* contributors, void* stream) {
  clear_error();
  if (aggregate != EKV_AGG_MEAN && aggregate != EKV_AGG_MAX)
    return fail(EKV_EINVAL, "unknown aggregate %d", aggregate);
  if (tile_blocks < 1) return fail(EKV_EINVAL, "tile_blocks must be positive");
  if (layers < 0 || rows < 0 || width < 0 || group_rows < 0)
    return fail(EKV_EINVAL, "negative dimension");
  if (group_rows > kNormMaxQ) return fail(EKV_ENOTSUP, "group_rows %d > %d", group_rows, kNormMaxQ);
  if (rows == 0 || width == 0) return EKV_OK;
  if (!share || !row_blocks || (layers > 0 && group_rows > 0 && !u))
    return fail(EKV_EINVAL, "a required pointer is NULL");
  // An empty layer or query-row axis has no data: every row is NaN, with Q = 1 as a stand-in.
  const bool empty = layers == 0 || group_rows == 0;
  NormParams p{u, true, layers > 0 ? layers : 1, empty ? 0 : layers, rows, width,
               group_rows > 0 ? group_rows : 1, nullptr, row_blocks, rows, tile_blocks,
               aggregate, share, contributors};
  normalize_kernel<<<rows, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("normalize_kernel");
}

extern "C" int ekv_share_finalize(const float* share_acc, const int32_t* contributors,
                                  const uint8_t* select, int rows, int width, int aggregate,
                                  float* share_out, void* stream) {
  clear_error();
  if (aggregate != EKV_AGG_MEAN && aggregate != EKV_AGG_MAX)
    return fail(EKV_EINVAL, "unknown aggregate %d", aggregate);
  if (rows <= 0 || width <= 0) return fail(EKV_EINVAL, "rows and width must be positive");
  if (!share_acc || !contributors || !share_out) return fail(EKV_EINVAL, "a required pointer is NULL");
  finalize_kernel<<<rows, kFinalThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      share_acc, contributors, select, width, aggregate, share_out);
  return check_launch("finalize_kernel");
}
