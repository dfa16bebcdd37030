// The pins of Controller._allocate (observe/controller.py:420-424), shared by the quota, sum and
// view kernels.
#pragma once

#include <stdint.h>

namespace ekv {

// Block 0 and [pin_start, n) are pinned, so the unpinned blocks are exactly [1, pin_start).
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

__device__ __host__ __forceinline__ int pin_count(int n, int ps) { return n <= 0 ? 0 : (ps > 0 ? 1 : 0) + (n - ps); }

}  // namespace ekv
