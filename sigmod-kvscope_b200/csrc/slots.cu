// The view of SGLang's CSR key-value list on the device (runtime/sglang_compact.py of the reference).
//
// SGLang's decode kernel reads request r from slots[indptr[r] : indptr[r + 1]], one token slot per
// entry. The view groups block_tokens consecutive entries of a request into a block and keeps some
// blocks: the row's first and last always, all of them when the policy is not live, when the row is
// audited, or when it is a row a CUDA graph adds to fill its batch (rows from n_real on).
//   slot_plan_kernel, one CTA: warps take rows in parallel (the reference walks the rows in one
//     program, :22-79). Per row a ballot per 32 blocks gives the kept blocks, their order (written to
//     the table) and the new length; a block scan over the rows gives the new indptr; the read
//     counters are summed in a fixed order and added to the running ones.
//   slot_gather_kernel: every entry of the new list, in parallel, from the entry of the old list it
//     comes from (:82-104); its row by binary search of the new indptr.
//   slot_copy_kernel: the new indptr and list back into the engine's buffers (the gather cannot work
//     in place: an entry can be read by an earlier position of the new list).
#include "ekv_common.cuh"

namespace ekv {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kGatherThreads = 256;

struct SlotParams {
  int32_t* indptr;
  const void* slots;
  void* slots_out;  // the engine's list, written back by slot_copy_kernel
  const uint8_t* keep;
  int64_t keep_s0;
  const uint8_t* audit;
  int active, n_real, n_rows;
  int64_t entries;
  int block_tokens, width;
  int32_t* new_indptr;
  int32_t* lens;
  int32_t* table;
  int64_t table_s0;
  long long* counts;  // [5] running counters
  void* out;          // [entries]
};

__global__ void __launch_bounds__(kPlanThreads) slot_plan_kernel(const SlotParams p) {
  __shared__ int s_scan[kPlanWarps + 1];
  __shared__ long long s_counts[kPlanWarps][4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BT = p.block_tokens;
  long long read = 0, full = 0, audit_read = 0, untrimmed = 0;
  // 1. every row: its kept blocks in order (the table), its new length
  for (int row = warp; row < p.n_rows; row += kPlanWarps) {
    const int length = p.indptr[row + 1] - p.indptr[row];
    const int blocks = length > 0 ? (length + BT - 1) / BT : 0;
    const bool real = row < p.n_real;
    const bool audited = p.audit != nullptr && real && p.audit[row] != 0;
    const bool whole = p.active == 0 || audited || !real;
    const uint8_t* krow = p.keep + (int64_t)row * p.keep_s0;
    int32_t* trow = p.table + (int64_t)row * p.table_s0;
    const int span = blocks < p.width ? blocks : p.width;
    int kept = 0;
    for (int base = 0; base < span; base += 32) {
      const int b = base + lane;
      const bool chosen = b < span && ((real && krow[b] != 0) || whole || b == 0 || b == blocks - 1);
      const uint32_t bits = __ballot_sync(kFullMask, chosen);
      if (chosen) trow[kept + __popc(bits & ((1u << lane) - 1u))] = b;
      kept += __popc(bits);
    }
    const int new_length = blocks > 0 ? (kept - 1) * BT + length - (blocks - 1) * BT : 0;
    if (lane == 0) {
      p.lens[row] = new_length;
      if (real) {
        read += kept;
        full += blocks;
        audit_read += audited ? kept : 0;
        untrimmed += (new_length == length && !audited && p.active != 0) ? kept : 0;
      }
    }
  }
  if (lane == 0) {
    s_counts[warp][0] = read, s_counts[warp][1] = full, s_counts[warp][2] = audit_read, s_counts[warp][3] = untrimmed;
  }
  __syncthreads();  // (also publishes the lengths written above)
  // 2. the new indptr: an exclusive scan of the lengths
  int carry = 0;
  for (int base = 0; base < p.n_rows; base += kPlanThreads) {
    const int row = base + tid;
    const int len = row < p.n_rows ? p.lens[row] : 0;
    int total = 0;
    const int before = block_exclusive_scan<kPlanThreads>(len, s_scan, &total);
    if (row < p.n_rows) p.new_indptr[row + 1] = carry + before + len;
    carry += total;
  }
  if (tid == 0) {
    p.new_indptr[0] = 0;
    long long c[4] = {0, 0, 0, 0};
    for (int w = 0; w < kPlanWarps; ++w)
      for (int j = 0; j < 4; ++j) c[j] += s_counts[w][j];
    p.counts[0] += c[0];
    p.counts[1] += c[1];
    p.counts[2] += c[2];
    p.counts[3] += c[3];
    p.counts[4] += p.active ? 0 : c[0];  // read with no live policy
  }
}

template <typename S>
__global__ void __launch_bounds__(kGatherThreads) slot_gather_kernel(const SlotParams p) {
  const int32_t* ni = p.new_indptr;
  const long long total = ni[p.n_rows];
  const S* slots = static_cast<const S*>(p.slots);
  S* out = static_cast<S*>(p.out);
  for (long long pos = (long long)blockIdx.x * kGatherThreads + threadIdx.x; pos < total;
       pos += (long long)gridDim.x * kGatherThreads) {
    int lo = 0, hi = p.n_rows;  // the last row with new_indptr[row] <= pos
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (ni[mid] <= pos) lo = mid; else hi = mid;
    }
    const int offset = (int)(pos - ni[lo]);
    const int block = p.table[(int64_t)lo * p.table_s0 + offset / p.block_tokens];
    const long long source = (long long)p.indptr[lo] + (long long)block * p.block_tokens + offset % p.block_tokens;
    if (source >= 0 && source < p.entries) out[pos] = slots[source];
  }
}

template <typename S>
__global__ void __launch_bounds__(kGatherThreads) slot_copy_kernel(const SlotParams p) {
  const long long total = p.new_indptr[p.n_rows];
  const long long stride = (long long)gridDim.x * kGatherThreads;
  const long long first = (long long)blockIdx.x * kGatherThreads + threadIdx.x;
  for (long long i = first; i <= p.n_rows; i += stride) p.indptr[i] = p.new_indptr[i];
  const S* out = static_cast<const S*>(p.out);
  S* slots = static_cast<S*>(p.slots_out);
  for (long long i = first; i < total; i += stride) slots[i] = out[i];
}

}  // namespace ekv

using namespace ekv;

extern "C" int ekv_slot_compact(int32_t* indptr, void* slots, int slot_bytes, const uint8_t* keep,
                                int64_t keep_stride, const uint8_t* audit, int active, int n_real, int n_rows,
                                int64_t entries, int block_tokens, int width, int32_t* new_indptr, int32_t* lens,
                                int32_t* table, int64_t table_stride, int64_t* counts, void* out, void* stream) {
  clear_error();
  if (!indptr || !slots || !keep || !new_indptr || !lens || !table || !counts || !out)
    return fail(EKV_EINVAL, "a required pointer is NULL");
  if (slot_bytes != 4 && slot_bytes != 8) return fail(EKV_EINVAL, "slot entries of %d bytes (4 or 8)", slot_bytes);
  if (n_rows < 0 || n_real < 0 || entries < 0) return fail(EKV_EINVAL, "negative rows or entries");
  if (block_tokens <= 0 || width <= 0) return fail(EKV_EINVAL, "block_tokens and width must be positive");
  if (keep_stride < width || table_stride < width) return fail(EKV_EINVAL, "a row stride is below the width");
  if (entries > 0x7fffffffll) return fail(EKV_ENOTSUP, "more than 2^31 - 1 list entries");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SlotParams p{indptr, slots, slots, keep, keep_stride, audit, active != 0, n_real, n_rows, entries, block_tokens,
               width, new_indptr, lens, table, table_stride, reinterpret_cast<long long*>(counts), out};
  slot_plan_kernel<<<1, kPlanThreads, 0, s>>>(p);
  int rc = check_launch("slot_plan_kernel");
  if (rc != EKV_OK) return rc;
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("cudaDeviceGetAttribute");
  const long long want = (entries + kGatherThreads - 1) / kGatherThreads;
  const int grid = (int)(want < 8LL * sms ? (want > 0 ? want : 1) : 8LL * sms);
  if (slot_bytes == 8) {
    slot_gather_kernel<long long><<<grid, kGatherThreads, 0, s>>>(p);
    if ((rc = check_launch("slot_gather_kernel")) != EKV_OK) return rc;
    slot_copy_kernel<long long><<<grid, kGatherThreads, 0, s>>>(p);
  } else {
    slot_gather_kernel<int32_t><<<grid, kGatherThreads, 0, s>>>(p);
    if ((rc = check_launch("slot_gather_kernel")) != EKV_OK) return rc;
    slot_copy_kernel<int32_t><<<grid, kGatherThreads, 0, s>>>(p);
  }
  return check_launch("slot_copy_kernel");
}
