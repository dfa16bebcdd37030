// The view of SGLang's CSR key-value list on the device (runtime/sglang_compact.py of the reference).
//
// SGLang's decode kernel reads request r from slots[indptr[r] : indptr[r + 1]], one token slot per
// entry. The view groups block_tokens consecutive entries of a request into a block and keeps some
// blocks: the row's first and last always, all of them when the policy is not live, when the row is
// audited, or when it is a row a CUDA graph adds to fill its batch (rows from n_real on).
//   slot_rows_kernel, a warp per row (the reference walks the rows in one program, :22-79): each lane
//     takes 16 blocks of the row at a time (one 16-byte load of the keep mask where it is aligned), a
//     warp scan of the lanes' counts places the kept blocks in order (the table) and gives the new
//     length; the read counters are integer sums, added with atomics (their order does not matter).
//   slot_scan_kernel, one CTA: the new indptr, an exclusive scan of the new lengths.
//   slot_gather_kernel: every entry of the new list, in parallel, from the entry of the old list it
//     comes from (:82-104); its row by binary search of the new indptr.
//   slot_copy_kernel: the new indptr and list back into the engine's buffers (the gather cannot work
//     in place: an entry can be read by an earlier position of the new list).
#include "ekv_common.cuh"

namespace ekv {

constexpr int kRowsPerCta = 8;  // one warp per row
constexpr int kScanThreads = 1024;
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

__global__ void __launch_bounds__(kRowsPerCta * 32) slot_rows_kernel(const SlotParams p) {
  chain_release();
  chain_wait();  // the lists and masks written before this launch
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerCta + warp;
  if (row >= p.n_rows) return;
  const int BT = p.block_tokens;
  const int length = p.indptr[row + 1] - p.indptr[row];
  const int blocks = length > 0 ? (length + BT - 1) / BT : 0;
  const bool real = row < p.n_real;
  const bool audited = p.audit != nullptr && real && p.audit[row] != 0;
  const bool whole = p.active == 0 || audited || !real;
  const uint8_t* krow = p.keep + (int64_t)row * p.keep_s0;
  int32_t* trow = p.table + (int64_t)row * p.table_s0;
  const int span = blocks < p.width ? blocks : p.width;
  const bool vec = (reinterpret_cast<uintptr_t>(krow) & 15) == 0;
  int kept = 0;
  for (int base = 0; base < span; base += 32 * 16) {
    const int b0 = base + 16 * lane;  // this lane's blocks [b0, b0 + 16)
    uint32_t mask = 0;               // bit j: block b0 + j is kept
    if (!whole) {
      if (vec && b0 + 16 <= span) {
        const uint4 v = *reinterpret_cast<const uint4*>(krow + b0);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 16; ++j) mask |= (((w[j >> 2] >> (8 * (j & 3))) & 0xffu) != 0u ? 1u : 0u) << j;
      } else {
        for (int j = 0; j < 16 && b0 + j < span; ++j) mask |= (krow[b0 + j] != 0 ? 1u : 0u) << j;
      }
    }
    const int valid = span - b0;  // blocks of this lane inside the row (may be <= 0 or > 16)
    const uint32_t inside = valid <= 0 ? 0u : (valid >= 16 ? 0xffffu : (1u << valid) - 1u);
    if (whole) mask = inside;
    if (b0 == 0 && span > 0) mask |= 1u;                         // the first block
    if (blocks - 1 >= b0 && blocks - 1 < b0 + 16 && blocks - 1 < span) mask |= 1u << (blocks - 1 - b0);  // the last
    mask &= inside;
    const int cnt = __popc(mask);
    int incl = cnt;
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(kFullMask, incl, off);
      if (lane >= off) incl += v;
    }
    int at = kept + incl - cnt;
    while (mask) {
      const int j = __ffs(mask) - 1;
      trow[at++] = b0 + j;
      mask &= mask - 1u;
    }
    kept += __shfl_sync(kFullMask, incl, 31);
  }
  if (lane == 0) {
    const int new_length = blocks > 0 ? (kept - 1) * BT + length - (blocks - 1) * BT : 0;
    p.lens[row] = new_length;
    if (real) {
      unsigned long long* c = reinterpret_cast<unsigned long long*>(p.counts);
      atomicAdd(c + 0, (unsigned long long)kept);
      atomicAdd(c + 1, (unsigned long long)blocks);
      if (audited) atomicAdd(c + 2, (unsigned long long)kept);
      if (new_length == length && !audited && p.active != 0) atomicAdd(c + 3, (unsigned long long)kept);
      if (p.active == 0) atomicAdd(c + 4, (unsigned long long)kept);  // read with no live policy
    }
  }
}

// One CTA: the new indptr, an exclusive scan of the new lengths.
__global__ void __launch_bounds__(kScanThreads) slot_scan_kernel(const SlotParams p) {
  chain_release();
  chain_wait();  // the new lengths
  __shared__ int s_scan[kScanThreads / 32 + 1];
  int carry = 0;
  for (int base = 0; base < p.n_rows; base += kScanThreads) {
    const int row = base + threadIdx.x;
    const int len = row < p.n_rows ? p.lens[row] : 0;
    int total = 0;
    const int before = block_exclusive_scan<kScanThreads>(len, s_scan, &total);
    if (row < p.n_rows) p.new_indptr[row + 1] = carry + before + len;
    carry += total;
  }
  if (threadIdx.x == 0) p.new_indptr[0] = 0;
}

template <typename S>
__global__ void __launch_bounds__(kGatherThreads) slot_gather_kernel(const SlotParams p) {
  chain_release();
  chain_wait();  // the new indptr and the table
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
  chain_release();
  chain_wait();  // every gathered entry
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
  if (n_rows > 0) {
    launch_chained(slot_rows_kernel, dim3((n_rows + kRowsPerCta - 1) / kRowsPerCta), dim3(kRowsPerCta * 32), 0, s, p);
    const int rc = check_launch("slot_rows_kernel");
    if (rc != EKV_OK) return rc;
  }
  launch_chained(slot_scan_kernel, dim3(1), dim3(kScanThreads), 0, s, p);
  int rc = check_launch("slot_scan_kernel");
  if (rc != EKV_OK) return rc;
  int device = 0, sms = 0;
  if (cudaGetDevice(&device) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return check_launch("cudaDeviceGetAttribute");
  const long long want = (entries + kGatherThreads - 1) / kGatherThreads;
  const int grid = (int)(want < 8LL * sms ? (want > 0 ? want : 1) : 8LL * sms);
  if (slot_bytes == 8) {
    launch_chained(slot_gather_kernel<long long>, dim3(grid), dim3(kGatherThreads), 0, s, p);
    if ((rc = check_launch("slot_gather_kernel")) != EKV_OK) return rc;
    launch_chained(slot_copy_kernel<long long>, dim3(grid), dim3(kGatherThreads), 0, s, p);
  } else {
    launch_chained(slot_gather_kernel<int32_t>, dim3(grid), dim3(kGatherThreads), 0, s, p);
    if ((rc = check_launch("slot_gather_kernel")) != EKV_OK) return rc;
    launch_chained(slot_copy_kernel<int32_t>, dim3(grid), dim3(kGatherThreads), 0, s, p);
  }
  return check_launch("slot_copy_kernel");
}
