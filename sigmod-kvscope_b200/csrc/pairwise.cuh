// numpy.add.reduce's pairwise summation of float64 values, reproduced bit for bit by one CTA.
//
// numpy sums a contiguous array of n values as pairwise_sum(a, n): below 8 values a plain loop from
// 0.0; up to 128 values eight accumulators r[j] += a[i + j] over whole groups of 8, combined as
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)), then the rest one by one; above 128 values
// pairwise_sum(a, n2) + pairwise_sum(a + n2, n - n2) with n2 = n / 2 rounded down to a multiple of 8.
// The recursion's shape depends on n alone, and the right half is never the smaller, so its deepest leaves
// lie D levels down the path that always takes the right half. Here every node is named by a slot of D
// bits, the path from the root (a 1 takes the right half), its trailing bits zero below the node's own
// level: the leaves are summed in parallel into their slots, and the levels are combined from the bottom
// up, each inner node adding its right half's slot to its own: the same additions in the same order as
// numpy's recursion.
#pragma once

#include "ekv_common.cuh"

namespace ekv {

// Slots of block_pairwise_sum for up to n values, 2^D: every right half is at most n / 2 + 8 values, so D
// is at most 7 for 8192 values, 8 for 16384 and 9 for 32768.
__host__ __device__ constexpr int pairwise_slots(int n) {
  return n <= 128 ? 1 : (n <= 8192 ? 128 : (n <= 16384 ? 256 : 512));
}

// Bytes of block_pairwise_sum's scratch of `slots` slots (one float64 each).
__host__ __device__ constexpr size_t pairwise_bytes(int slots) { return (size_t)slots * 8; }

// block_pairwise_sum's scratch, carved from pairwise_bytes(slots) of 8-byte aligned shared memory.
struct PairwiseScratch {
  double* val;
};

__device__ __forceinline__ PairwiseScratch pairwise_scratch(void* mem, int slots) {
  (void)slots;
  return PairwiseScratch{static_cast<double*>(mem)};
}

// The sum of value(0 .. n) as numpy computes it, with a scratch of pairwise_slots(n) slots or more; every
// thread of the CTA calls it and gets the sum. THREADS = blockDim.x (a multiple of 32). Each leaf is summed
// by eight lanes: lane j keeps numpy's accumulator r[j] (its additions in numpy's order), the eight are
// combined by shuffles in numpy's order, and lane 0 adds the rest; the lanes of a leaf read eight adjacent
// values. Warp 0 combines the levels.
template <int THREADS, typename V>
__device__ double block_pairwise_sum(const PairwiseScratch& t, int n, const V& value) {
  const int tid = threadIdx.x, lane = tid & 31;
  int D = 0;  // the depth of the deepest leaf
  for (int m = n; m > 128; m -= (m / 2) & ~7) ++D;
  const int slots = 1 << D;
  __syncthreads();  // the scratch may still be read by an earlier call
  // the leaves: slot s follows its bits from the root until a node of at most 128 values; that leaf is the
  // slot's when the bits below the leaf's level are zero
  const int oct = tid >> 3, j = tid & 7;
  for (int s0 = 0; s0 < slots; s0 += THREADS / 8) {  // (the same trip count in every lane)
    const int s = s0 + oct;
    int lo = 0, len = n, depth = 0;
    if (s < slots) {
      for (; depth < D && len > 128; ++depth) {
        const int half = (len / 2) & ~7;
        if ((s >> (D - 1 - depth)) & 1) {
          lo += half;
          len -= half;
        } else {
          len = half;
        }
      }
    }
    const bool leaf = s < slots && (s & ((1 << (D - depth)) - 1)) == 0;
    if (!leaf) len = 0;
    const int whole = len - len % 8;  // values in whole groups of eight (none below 8 values)
    double r = 0.0;
    if (len >= 8) {
      r = value(lo + j);
      for (int k = 8; k < whole; k += 8) r += value(lo + k + j);
    }
    r += __shfl_xor_sync(kFullMask, r, 1);  // r0 + r1, r2 + r3, ...
    r += __shfl_xor_sync(kFullMask, r, 2);  // (r0 + r1) + (r2 + r3), ...
    r += __shfl_xor_sync(kFullMask, r, 4);  // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7))
    if (leaf && j == 0) {
      double res = len >= 8 ? r : 0.0;  // below 8 values a plain loop from 0.0
      for (int k = len >= 8 ? whole : 0; k < len; ++k) res += value(lo + k);
      t.val[s] = res;
    }
  }
  __syncthreads();
  if (tid < 32) {
    // level d, deepest first: node k (its d bits) is the slot k << (D - d); an inner node (every ancestor and
    // itself of more than 128 values) adds its right half, at slot + 2^(D - d - 1)
    for (int d = D - 1; d >= 0; --d) {
      for (int k = lane; k < (1 << d); k += 32) {
        int len = n;
        bool inner = true;
        for (int e = 0; e < d && inner; ++e) {
          if (len <= 128) {
            inner = false;
          } else {
            const int half = (len / 2) & ~7;
            len = ((k >> (d - 1 - e)) & 1) ? len - half : half;
          }
        }
        if (inner && len > 128) {
          const int s = k << (D - d);
          t.val[s] = t.val[s] + t.val[s + (1 << (D - d - 1))];
        }
      }
      __syncwarp();
    }
  }
  __syncthreads();
  return t.val[0];
}

}  // namespace ekv
