// Shared device helpers of libekv_b200: PTX wrappers for mbarriers, bulk copies, ldmatrix and
// mma.sync, bounded waits, and the host-side error channel of the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>

#include "ekv_b200.h"

namespace ekv {

// ---- host: error reporting -------------------------------------------------------------------

// Records a printf-style message as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Clears the last error (called on entry to every ABI function).
void clear_error();
// Maps the runtime's launch status to an ABI code (EKV_OK or EKV_ECUDA with the message recorded).
int check_launch(const char* what);

constexpr int kMaxDevices = 64;  // per-device one-time kernel attributes
// The current device's ordinal in *device: EKV_OK, EKV_ECUDA when the runtime cannot say, or EKV_ENOTSUP
// for an ordinal at or past kMaxDevices (the per-device caches of the entry points hold that many).
int current_device(int* device);

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int cdiv(int a, int b) { return (a + b - 1) / b; }

// ---- device: small utilities -------------------------------------------------------------------

constexpr uint32_t kFullMask = 0xffffffffu;

// ---- chained launches (programmatic dependent launch) ----------------------------------------------
// A kernel launched with launch_chained may start while the kernel before it in the stream is still
// finishing; it calls chain_wait() before it reads anything an earlier launch wrote (the wait returns
// once that launch has completed and its writes are visible), and chain_release() once the next
// chained launch may start. Without the launch attribute both are no-ops.
__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void chain_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                  Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}
// launch_chained for a grid of thread-block clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_chained_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                          cudaStream_t stream, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// A bounded wait gives up after this many SM clock cycles (about a second at 1.9 GHz).
constexpr long long kWaitLimitCycles = 2000000000ll;

// The lanes of this warp below this one, as a mask.
__device__ __forceinline__ uint32_t lanes_below() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Asynchronous global -> shared copies (cp.async): 4 and 8 bytes through L1, 16 bytes around it.
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// dst[0, n) = src[0, n) (elements of 4 or 8 bytes) into shared memory by every thread of the CTA, all
// copies in flight at once (16 bytes a copy where both ends are 16-byte aligned); returns after a
// barrier, with the row visible to the whole CTA.
template <int THREADS, typename T>
__device__ __forceinline__ void stage_row(T* dst, const T* src, int n) {
  static_assert(sizeof(T) == 4 || sizeof(T) == 8, "4- or 8-byte elements");
  constexpr int kPer = 16 / sizeof(T);
  int done = 0;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
    done = n / kPer * kPer;
    for (int i = kPer * threadIdx.x; i < done; i += kPer * THREADS) cp_async16(dst + i, src + i);
  }
  for (int i = done + threadIdx.x; i < n; i += THREADS) {
    if constexpr (sizeof(T) == 4) cp_async4(dst + i, src + i); else cp_async8(dst + i, src + i);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
}


__device__ __forceinline__ void set_status(uint32_t* status, uint32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// Merges the log-sum-exp partial (m2, s2) into (m, s): afterwards s * exp(m) is the sum of both.
// -inf marks an empty partial. The result does not depend on which side is which.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    s = s2;
    return;
  }
  const float mn = fmaxf(m, m2);
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

// ---- device: mbarrier + bulk copy (TMA engine) -------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for phase `parity` of `bar` to complete, for at most kWaitLimitCycles. On timeout it sets
// EKV_STATUS_WAIT_TIMEOUT and returns false; the caller then skips its use of the stage.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitLimitCycles) {
      set_status(status, EKV_STATUS_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}

// An L2 policy that evicts the streamed key rows first, so the statistic table stays resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// One bulk copy global -> shared through the TMA engine, completing `bytes` on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---- device: tensor-core fragments -------------------------------------------------------------

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <typename T>
struct Mma;

template <>
struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float (&c)[4], const uint32_t (&a)[4],
                                             const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
};

template <>
struct Mma<__half> {
  __device__ __forceinline__ static void run(float (&c)[4], const uint32_t (&a)[4],
                                             const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
};

// ---- device: block-wide reductions and scans ----------------------------------------------------

template <int THREADS>
__device__ __forceinline__ float block_sum_fixed_order(float v, float* scratch /*THREADS/32*/) {
  // A tree over lanes, then warps in index order: the same inputs give the same bits.
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(kFullMask, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < THREADS / 32; ++w) total += scratch[w];
  return total;
}

// Exclusive prefix sum of one int per thread over the block; *total receives the sum.
// scratch holds THREADS/32 + 1 ints.
template <int THREADS>
__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int inc = v;
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(kFullMask, inc, off);
    if (lane >= off) inc += n;
  }
  __syncthreads();
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    constexpr int W = THREADS / 32;
    int s = lane < W ? scratch[lane] : 0;
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(kFullMask, s, off);
      if (lane >= off) s += n;
    }
    if (lane < W) scratch[lane] = s;  // inclusive scan of warp totals
    if (lane == W - 1) scratch[W] = s;
  }
  __syncthreads();
  const int before = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[THREADS / 32];
  return before + inc - v;
}

}  // namespace ekv
