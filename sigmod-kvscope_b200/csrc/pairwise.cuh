// numpy.add.reduce's pairwise summation of float64 values, reproduced bit for bit by one CTA.
//
// numpy sums a contiguous array of n values as pairwise_sum(a, n): below 8 values a plain loop from
// 0.0; up to 128 values eight accumulators r[j] += a[i + j] over whole groups of 8, combined as
// ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)), then the rest one by one; above 128 values
// pairwise_sum(a, n2) + pairwise_sum(a + n2, n - n2) with n2 = n / 2 rounded down to a multiple of 8.
// Here the tree is built one level at a time (every node of a level splits and records its children),
// the leaves are summed in parallel, and the levels are combined from the bottom up: the same additions
// in the same order as numpy's recursion.
#pragma once

#include "ekv_common.cuh"

namespace ekv {

constexpr int kPairwiseMaxLevels = 16;

// The most nodes numpy's recursion makes for up to n values: one leaf up to 128 values, and every split of
// more than 128 values gives halves of at least 64, so at most 129 nodes for 8192 values, 257 for 16384
// and 513 for 32768.
__host__ __device__ constexpr int pairwise_nodes(int n) {
  return n <= 128 ? 1 : (n <= 8192 ? 129 : (n <= 16384 ? 257 : 513));
}

// Bytes of block_pairwise_sum's scratch for up to `nodes` nodes: the node values (float64), ranges and
// children, the levels and two counters; a multiple of 8.
__host__ __device__ constexpr size_t pairwise_bytes(int nodes) {
  return (size_t)nodes * 8 + (((size_t)nodes * 3 + kPairwiseMaxLevels + 4) * 4 + 7) / 8 * 8;
}

// block_pairwise_sum's scratch, carved from pairwise_bytes(nodes) of 8-byte aligned shared memory.
struct PairwiseScratch {
  double* val;
  int *lo, *len, *left, *level, *meta;  // meta: the nodes made, the depth
};

__device__ __forceinline__ PairwiseScratch pairwise_scratch(void* mem, int nodes) {
  PairwiseScratch t;
  t.val = static_cast<double*>(mem);
  t.lo = reinterpret_cast<int*>(t.val + nodes);
  t.len = t.lo + nodes;
  t.left = t.len + nodes;
  t.level = t.left + nodes;
  t.meta = t.level + kPairwiseMaxLevels + 2;
  return t;
}

// The sum of value(0 .. n) as numpy computes it, with a scratch of pairwise_nodes(n) nodes or more; every
// thread of the CTA calls it and gets the sum. THREADS = blockDim.x (a multiple of 32). The tree (a few
// hundred nodes at most) is built and combined by warp 0 alone, a level at a time with warp barriers; the
// leaves are summed by the whole CTA, eight lanes a leaf: lane j keeps numpy's accumulator r[j] (its
// additions in numpy's order), the eight are combined by shuffles in numpy's order, and lane 0 adds the rest.
// The lanes of a leaf read eight adjacent values, so leaves that start 128 values apart share a bank only
// between the four leaves of a warp.
template <int THREADS, typename V>
__device__ double block_pairwise_sum(const PairwiseScratch& t, int n, const V& value) {
  const int tid = threadIdx.x, lane = tid & 31;
  __syncthreads();  // the scratch may still be read by an earlier call
  if (tid < 32) {
    // level d holds nodes [level[d], level[d + 1]); a node of more than 128 values splits, its children
    // placed after the level in node order (a ballot gives each splitting node its children's place)
    if (lane == 0) t.lo[0] = 0, t.len[0] = n, t.level[0] = 0, t.level[1] = 1;
    __syncwarp();
    int nodes = 1, depth = 1;
    for (int d = 0; d < kPairwiseMaxLevels; ++d) {
      const int a = t.level[d], b = t.level[d + 1];
      if (a == b) break;
      int next = b;
      for (int i0 = a; i0 < b; i0 += 32) {
        const int i = i0 + lane;
        const int len = i < b ? t.len[i] : 0;
        const bool split = len > 128;
        const unsigned int ballot = __ballot_sync(kFullMask, split);
        if (i < b) {
          if (split) {
            const int c = next + 2 * __popc(ballot & lanes_below());
            int n2 = len / 2;
            n2 -= n2 % 8;
            const int lo = t.lo[i];
            t.lo[c] = lo, t.len[c] = n2, t.lo[c + 1] = lo + n2, t.len[c + 1] = len - n2;
            t.left[i] = c;
          } else {
            t.left[i] = -1;
          }
        }
        next += 2 * __popc(ballot);
      }
      if (lane == 0) t.level[d + 2] = next;
      nodes = next;
      depth = d + 1;
      __syncwarp();
    }
    if (lane == 0) t.meta[0] = nodes, t.meta[1] = depth;
  }
  __syncthreads();
  const int nodes = t.meta[0];
  const int oct = tid >> 3, j = tid & 7;
  for (int i0 = 0; i0 < nodes; i0 += THREADS / 8) {  // (the same trip count in every lane)
    const int i = i0 + oct;
    const bool leaf = i < nodes && t.left[i] < 0;
    const int lo = leaf ? t.lo[i] : 0, len = leaf ? t.len[i] : 0;
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
      t.val[i] = res;
    }
  }
  __syncthreads();
  if (tid < 32) {
    for (int d = t.meta[1] - 1; d >= 0; --d) {  // each inner node: left + right, deepest level first
      for (int i = t.level[d] + lane; i < t.level[d + 1]; i += 32)
        if (t.left[i] >= 0) t.val[i] = t.val[t.left[i]] + t.val[t.left[i] + 1];
      __syncwarp();
    }
  }
  __syncthreads();
  return t.val[0];
}

}  // namespace ekv
