// allocate() with any pinned blocks (observe/allocation.py:37-75: Request.pinned may mark any blocks).
//
// The allocation kernels take pins of one shape, block 0 and a newest suffix [ps, n), so that the
// unpinned blocks are the range [1, ps). Any other pin set is brought to that shape here, on the
// device, with every share computed once as the reference computes it (Request.shares:
// max(score, 0) / total, total NumPy's pairwise sum over the request in block order; 1 / n when the
// total is not positive), and the objective then ranks those shares as they are ("presummed" rows):
//
//   * uniform and maxmin rank each request by its own shares, ties to the older block, and maxmin sums
//     the pinned shares in block order. A stable partition keeps both: slot 0 holds the first pinned
//     block, slots [1, 1 + u) the u unpinned blocks in block order, the slots after them the other
//     pinned blocks in block order. A request with no pin gets a slot 0 of its own (share 0, which adds
//     nothing to a sum) and one more block of budget.
//   * sum breaks ties between requests by block index (the newer block first), so its rows keep block
//     order: slot 0 is a slot of the request's own (share 0), slot 1 + b is block b, a pinned block
//     holds +inf, which the kernels rank above every gain (kept before any unpinned block), and each
//     request adds one block of budget for its slot 0.
//
// A scatter then writes each request's mask back in block order.

#include "ekv_common.cuh"
#include "pairwise.cuh"

namespace ekv {

int presummed_quotas(const int32_t* row_blocks, const int32_t* measured, long long budget,
                     const long long* budget_add, int rows, int width, int32_t* quota, cudaStream_t stream);
int presummed_mask(const int32_t* row_blocks, const int32_t* quota, const int32_t* measured, const double* shares,
                   int64_t share_s0, int rows, int width, uint8_t* mask_out, int64_t mask_s0, cudaStream_t stream);
int presummed_sum(const double* shares, int64_t share_s0, const double* weights, const int32_t* row_blocks,
                  const int32_t* measured, long long budget, const long long* budget_add, int rows, int width,
                  int32_t* quota, uint8_t* mask_out, int64_t mask_s0, void* workspace, size_t workspace_bytes,
                  cudaStream_t stream);
int presummed_maxmin(const double* shares, int64_t share_s0, const int32_t* row_blocks, const int32_t* measured,
                     long long budget, const long long* budget_add, int rows, int width, int32_t* quota,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream);

namespace {

constexpr int kPinThreads = 512;
constexpr int kPinMaxWidth = 16383;  // the slots of a row, width + 1, are staged by the view kernel (16384)

struct PinLayout {
  size_t added, shares, slot_of, rows_n, rows_ps, quota, mask, objective, bytes;
};

// slot_of[r][j]: the block of slot j (-1: the request's own slot 0)
PinLayout pin_layout(int rows, int width, size_t objective_bytes) {
  PinLayout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += round_up(bytes, 256);
    return at;
  };
  const size_t w1 = (size_t)width + 1;
  l.added = take(sizeof(long long));
  l.shares = take((size_t)rows * w1 * 8);
  l.slot_of = take((size_t)rows * w1 * 4);
  l.rows_n = take((size_t)rows * 4);
  l.rows_ps = take((size_t)rows * 4);
  l.quota = take((size_t)rows * 4);
  l.mask = take((size_t)rows * w1);
  l.objective = take(objective_bytes);
  l.bytes = o;
  return l;
}

struct PinParams {
  const double* scores;
  int64_t score_s0;
  const uint8_t* pinned;
  int64_t pinned_s0;
  const int32_t* row_blocks;
  int rows, width;
  bool keep_order;        // sum: block b at slot 1 + b; otherwise the stable partition
  double* shares;         // [rows][width + 1]
  int32_t* slot_of;       // [rows][width + 1]
  int32_t* rows_n;        // [rows] slots of the request
  int32_t* rows_ps;       // [rows] the first slot of the pinned suffix
  long long* added;       // blocks of budget the requests' own slots take
};

// One CTA per request: the shares (pairwise total), then the slots.
__global__ void __launch_bounds__(kPinThreads) pin_slots_kernel(const PinParams p) {
  chain_release();
  chain_wait();  // what the launch before this one wrote
  extern __shared__ __align__(16) unsigned char pin_smem[];
  const PairwiseScratch s_tree = pairwise_scratch(pin_smem + (size_t)p.width * 8, pairwise_slots(p.width));
  __shared__ int s_scan[kPinThreads / 32 + 1];
  double* s_x = reinterpret_cast<double*>(pin_smem);  // [width]
  const int r = blockIdx.x, tid = threadIdx.x;
  int n = p.row_blocks[r];
  n = n < 0 ? 0 : (n > p.width ? p.width : n);
  const int64_t w1 = (int64_t)p.width + 1;
  double* out = p.shares + (int64_t)r * w1;
  int32_t* slot = p.slot_of + (int64_t)r * w1;
  const uint8_t* pin = p.pinned + (int64_t)r * p.pinned_s0;
  if (n == 0) {
    if (tid == 0) p.rows_n[r] = 0, p.rows_ps[r] = 0;
    return;
  }
  stage_row<kPinThreads>(s_x, p.scores + (int64_t)r * p.score_s0, n);
  const double total = block_pairwise_sum<kPinThreads>(s_tree, n, [&](int i) {
    const double s = s_x[i];
    return s > 0.0 ? s : 0.0;  // NaN counts as 0
  });
  const double equal = __ddiv_rn(1.0, (double)n);
  auto share = [&](int i) {
    const double s = s_x[i];
    return total > 0.0 ? __ddiv_rn(s > 0.0 ? s : 0.0, total) : equal;
  };
  if (p.keep_order) {
    for (int b = tid; b < n; b += kPinThreads) {
      out[1 + b] = pin[b] ? __longlong_as_double(0x7ff0000000000000ll) : share(b);
      slot[1 + b] = b;
    }
    if (tid == 0) {
      out[0] = 0.0, slot[0] = -1;
      p.rows_n[r] = n + 1, p.rows_ps[r] = n + 1;
      atomicAdd(reinterpret_cast<unsigned long long*>(p.added), 1ull);
    }
    return;
  }
  // the stable partition: each thread takes a run of consecutive blocks
  const int per = (n + kPinThreads - 1) / kPinThreads;
  const int lo = tid * per, hi = lo + per < n ? lo + per : n;
  int mine = 0;
  for (int b = lo; b < hi; ++b) mine += pin[b] != 0;
  int pins = 0;
  int pinned_before = block_exclusive_scan<kPinThreads>(mine, s_scan, &pins);
  const int open = n - pins;
  const int own = pins == 0 ? 1 : 0;  // a request with no pin gets a slot 0 of its own
  for (int b = lo; b < hi; ++b) {
    int j;
    if (pin[b]) {
      j = pinned_before == 0 ? 0 : open + pinned_before;
      ++pinned_before;
    } else {
      j = 1 + (b - pinned_before);
    }
    out[j] = share(b);
    slot[j] = b;
  }
  if (tid == 0) {
    if (own) {
      out[0] = 0.0, slot[0] = -1;
      atomicAdd(reinterpret_cast<unsigned long long*>(p.added), 1ull);
    }
    p.rows_n[r] = n + own;
    p.rows_ps[r] = 1 + open;
  }
}

// One CTA per request: mask_out[r][b] for b < width from the mask over its slots.
__global__ void __launch_bounds__(256) pin_scatter_kernel(const uint8_t* slot_mask, const int32_t* slot_of,
                                                          const int32_t* rows_n, const int32_t* row_blocks, int width,
                                                          uint8_t* mask_out, int64_t mask_s0) {
  chain_release();
  chain_wait();  // the objective's mask
  const int r = blockIdx.x;
  const int64_t w1 = (int64_t)width + 1;
  int n = row_blocks[r];
  n = n < 0 ? 0 : (n > width ? width : n);
  const int slots = rows_n[r];
  uint8_t* out = mask_out + (int64_t)r * mask_s0;
  for (int b = n + threadIdx.x; b < width; b += blockDim.x) out[b] = 0;  // past the request
  for (int j = threadIdx.x; j < slots; j += blockDim.x) {
    const int b = slot_of[(int64_t)r * w1 + j];
    if (b >= 0) out[b] = slot_mask[(int64_t)r * w1 + j];
  }
}

}  // namespace
}  // namespace ekv

using namespace ekv;

extern "C" size_t ekv_allocate_pinned_workspace_bytes(int rows, int width) {
  if (rows <= 0 || width <= 0 || width > kPinMaxWidth) return 0;
  const size_t objective = ekv_allocate_sum_workspace_bytes(rows, width + 1) >
                                   ekv_allocate_maxmin_workspace_bytes(rows, width + 1)
                               ? ekv_allocate_sum_workspace_bytes(rows, width + 1)
                               : ekv_allocate_maxmin_workspace_bytes(rows, width + 1);
  return pin_layout(rows, width, objective).bytes;
}

extern "C" int ekv_allocate_pinned_f64(const double* scores, int64_t score_stride, const uint8_t* pinned,
                                       int64_t pinned_stride, const double* weights, const int32_t* row_blocks,
                                       int objective, int64_t budget, int rows, int width, uint8_t* mask_out,
                                       int64_t mask_stride, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  if (!scores || !pinned || !row_blocks || !mask_out) return fail(EKV_EINVAL, "a required pointer is NULL");
  if (rows <= 0 || width <= 0) return fail(EKV_EINVAL, "rows and width must be positive");
  if (width > kPinMaxWidth) return fail(EKV_ENOTSUP, "width %d > %d", width, kPinMaxWidth);
  if (score_stride < width || pinned_stride < width || mask_stride < width)
    return fail(EKV_EINVAL, "a row stride is below the width");
  if (objective != EKV_POLICY_SUM && objective != EKV_POLICY_UNIFORM && objective != EKV_POLICY_MAXMIN)
    return fail(EKV_EINVAL, "unknown objective %d", objective);
  if (objective != EKV_POLICY_SUM && weights != nullptr)
    return fail(EKV_EINVAL, "only the sum objective weighs requests");
  if (objective == EKV_POLICY_MAXMIN && width + 1 > 8192)
    return fail(EKV_ENOTSUP, "maxmin with any pins: width %d > 8191", width);
  if (budget < 0) return fail(EKV_EINVAL, "the budget cannot be negative");
  const size_t need = ekv_allocate_pinned_workspace_bytes(rows, width);
  if (!workspace || workspace_bytes < need)
    return fail(EKV_ERANGE, "the pinned allocation workspace holds %zu bytes, the call needs %zu", workspace_bytes,
                need);
  if ((uintptr_t)workspace & 255) return fail(EKV_EINVAL, "the workspace must be 256-byte aligned");
  const size_t objective_bytes = ekv_allocate_sum_workspace_bytes(rows, width + 1) >
                                         ekv_allocate_maxmin_workspace_bytes(rows, width + 1)
                                     ? ekv_allocate_sum_workspace_bytes(rows, width + 1)
                                     : ekv_allocate_maxmin_workspace_bytes(rows, width + 1);
  const PinLayout l = pin_layout(rows, width, objective_bytes);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PinParams p{};
  p.scores = scores; p.score_s0 = score_stride; p.pinned = pinned; p.pinned_s0 = pinned_stride;
  p.row_blocks = row_blocks; p.rows = rows; p.width = width; p.keep_order = objective == EKV_POLICY_SUM;
  p.shares = reinterpret_cast<double*>(base + l.shares);
  p.slot_of = reinterpret_cast<int32_t*>(base + l.slot_of);
  p.rows_n = reinterpret_cast<int32_t*>(base + l.rows_n);
  p.rows_ps = reinterpret_cast<int32_t*>(base + l.rows_ps);
  p.added = reinterpret_cast<long long*>(base + l.added);
  int32_t* quota = reinterpret_cast<int32_t*>(base + l.quota);
  uint8_t* slot_mask = base + l.mask;
  const int w1 = width + 1;
  int device = 0;
  {
    const int dev_rc = current_device(&device);
    if (dev_rc != EKV_OK) return dev_rc;
  }
  const size_t smem = (size_t)width * 8 + pairwise_bytes(pairwise_slots(width));
  static size_t configured[kMaxDevices] = {};
  if (configured[device] < smem) {
    if (cudaFuncSetAttribute(pin_slots_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(pin_slots_kernel)");
    configured[device] = smem;
  }
  if (cudaMemsetAsync(p.added, 0, sizeof(long long), s) != cudaSuccess)
    return check_launch("cudaMemsetAsync(pinned allocation)");
  launch_chained(pin_slots_kernel, dim3(rows), dim3(kPinThreads), smem, s, p);
  int rc = check_launch("pin_slots_kernel");
  if (rc != EKV_OK) return rc;
  if (objective == EKV_POLICY_SUM) {
    rc = presummed_sum(p.shares, w1, weights, p.rows_n, p.rows_ps, budget, p.added, rows, w1, quota, slot_mask, w1,
                       base + l.objective, objective_bytes, s);
  } else {
    rc = objective == EKV_POLICY_UNIFORM
             ? presummed_quotas(p.rows_n, p.rows_ps, budget, p.added, rows, w1, quota, s)
             : presummed_maxmin(p.shares, w1, p.rows_n, p.rows_ps, budget, p.added, rows, w1, quota,
                                base + l.objective, objective_bytes, s);
    if (rc == EKV_OK) rc = presummed_mask(p.rows_n, quota, p.rows_ps, p.shares, w1, rows, w1, slot_mask, w1, s);
  }
  if (rc != EKV_OK) return rc;
  launch_chained(pin_scatter_kernel, dim3(rows), dim3(256), 0, s, slot_mask, p.slot_of, p.rows_n, row_blocks, width,
                 mask_out, mask_stride);
  return check_launch("pin_scatter_kernel");
}
