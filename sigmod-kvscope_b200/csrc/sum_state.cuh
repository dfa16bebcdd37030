// The shared-budget `sum` objective's select state (allocate.cu), read by the kernels that apply its
// threshold: the committed mask (sum_mask_kernel) and the view (view_kernel's threshold mode).
#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace ekv {

enum SumMode : int { kSumSelect = 0, kSumNone = 1, kSumAll = 2 };

struct SumState {
  unsigned long long prefix, mask;  // the threshold's known bits
  long long k;                      // keys still to choose at the threshold's prefix
  long long total_open, must, blocks;
  int mode, found;
  int exact;       // every key with the final prefix is taken: no block index decides between equal keys
  int istar;       // the lowest block index whose ties are (partly) taken
  long long m;     // ties taken at istar, from the earliest rows
  unsigned int n_cand;
  unsigned int ticket;
};

// Whether an unpinned block b of a request is kept under the threshold: its masked gain key above the
// prefix, or equal to it at an index above i*, or at i* in a row whose tie there is taken (`take`). With
// istar 0 (its initial value) every equal key is kept, as every unpinned block has b >= 1.
__device__ __forceinline__ bool sum_keeps(int mode, unsigned long long key_masked, unsigned long long prefix, int b,
                                          int istar, bool take) {
  if (mode == kSumAll) return true;
  if (mode == kSumNone) return false;
  return key_masked > prefix || (key_masked == prefix && (b > istar || (b == istar && take)));
}

// The view of every row under the threshold that the shared `sum` select left in `state` (view.cu): the keys
// [rows][width] and the rows' blocks, pin starts and taken ties come from the select's workspace.
int launch_sum_view(const int32_t* table, int64_t table_s0, const int32_t* seq_lens, const uint8_t* full_rows,
                    const uint8_t* released, int64_t released_s0, int rows, int width, int block_size, int32_t* view,
                    int64_t view_s0, int32_t* view_lens, uint8_t* mask_out, int64_t mask_s0, const SumState* state,
                    const unsigned long long* keys, const int32_t* row_n, const int32_t* row_ps, const int32_t* row_at,
                    cudaStream_t stream);

}  // namespace ekv
