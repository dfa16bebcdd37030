// The audit kernel: per-tile log-sum-exp of q.K over a paged key cache, with the exact per-block
// attention share folded in by the last CTA of each row.
//
// Work unit. A CTA owns one (row, chunk of EKV_AUDIT_CHUNK_TILES tiles, KV head). Each of its WARPS
// warps owns TPW tiles of TT tokens. At CTA start every warp asks the TMA engine for all its tiles
// at once: one 2*D-byte bulk copy per token row (lane i copies token i), landing in a shared-memory
// stage whose rows are padded to 2*D+16 bytes so that ldmatrix reads them without bank conflicts.
// The copies carry an L2 evict-first hint: the keys are read once, the statistic table is not.
//
// Scores. One m16n8k16 mma per (16 tokens, 16 dims): A = 16 key rows from shared memory through
// ldmatrix, B = the G query rows of the KV group (held in registers for the whole CTA, padded to 8
// or 16 columns), accumulating in fp32. The C fragment puts tokens on rows and query rows on
// columns, so the tile max and sum are three xor-shuffles per column. This is the computation of
// tile_lse_kernel (runtime/audit_kernel.py:70-96); the cells are stored as at :97-109.
//
// Shares. Each CTA also reduces its tiles into a (max, sum) partial per query row of
// u = m + log(l) - log(tile_blocks) (observe/tile_shares.py:172-173), writes it to the workspace and
// takes a ticket on its row. The CTA that takes the last ticket merges the partials into the row's
// log total per query row, reads the row's cells back (they are in L2), forms the share of every
// block exactly as normalize_tile_lse does (:82-103, with the partial tail tile's weight given back
// to its blocks) and adds it into the row's accumulator. No CTA waits on another.
#include <cstdarg>
#include <cstdio>

#include "ekv_common.cuh"

namespace ekv {

struct AuditParams {
  const void* q;
  const void* k;
  const int32_t* table;
  const int32_t* lens;
  const int32_t* qrow;
  const uint8_t* select;
  const uint32_t* flag;
  float* lse;
  float scale;
  int layer;
  int group;
  int64_t q_s0, q_s1;
  int64_t k_s0, k_s1, k_s2;
  int64_t table_s0;
  int layers, rows, width;
  int G;      // query rows per KV head
  int heads;  // KV heads recorded by this launch
  int Q;      // values per cell: heads * G
  int block_size, tile_blocks;
  int64_t pool_blocks;
  int64_t q_tokens;
  float* share_acc;
  int32_t* contrib;
  float* share_out;
  int aggregate;
  int share_flags;
  uint32_t* tickets;
  float2* partials;
  int max_chunks;
  uint32_t* status;
};

constexpr int kAuditWarps = 4;
constexpr int kAuditTilesPerWarp = EKV_AUDIT_CHUNK_TILES / kAuditWarps;
constexpr int kMaxQ = 128;

template <int D>
struct AuditLayout {
  static constexpr int kRowBytes = 2 * D;
  static constexpr int kRowStride = 2 * D + 16;  // 16-byte pad: conflict-free ldmatrix
};

// Writes the NaN row (FINALIZE) and clears the accumulators (RESET) of a row that no CTA records.
__device__ void audit_row_without_tiles(const AuditParams& p, int row, bool selected) {
  const size_t base = (size_t)row * p.width;
  if ((p.share_flags & EKV_SHARE_RESET) && selected) {
    for (int b = threadIdx.x; b < p.width; b += blockDim.x) p.share_acc[base + b] = 0.f;
    if (threadIdx.x == 0) p.contrib[row] = 0;
  }
  if (p.share_flags & EKV_SHARE_FINALIZE) {
    for (int b = threadIdx.x; b < p.width; b += blockDim.x) p.share_out[base + b] = NAN;
  }
}

// The last CTA of a row: partials -> log totals -> per-block shares -> accumulator (-> final).
template <int THREADS>
__device__ void audit_share_epilogue(const AuditParams& p, int row, int n_blocks, int n_chunks) {
  __shared__ float s_lse[kMaxQ];
  __shared__ int s_has[kMaxQ];
  __shared__ float s_red[THREADS / 32];
  __shared__ int s_contrib;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int Q = p.Q;
  const int TB = p.tile_blocks;
  const float log_tb = logf((float)TB);

  // 1. The log total of each query row: merge the chunk partials, a fixed tree per query row.
  for (int j = warp; j < Q; j += THREADS / 32) {
    float m = -INFINITY, s = 0.f;
    for (int c = lane; c < n_chunks; c += 32) {
      const float2 part = __ldcg(&p.partials[((size_t)row * p.max_chunks + c) * Q + j]);
      lse_merge(m, s, part.x, part.y);
    }
    for (int off = 16; off > 0; off >>= 1) {
      const float m2 = __shfl_xor_sync(kFullMask, m, off);
      const float s2 = __shfl_xor_sync(kFullMask, s, off);
      lse_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      s_has[j] = m != -INFINITY;
      s_lse[j] = m != -INFINITY ? log_tb + m + logf(s) : 0.f;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0;
    for (int j = 0; j < Q; ++j) c += s_has[j];
    const int prev = (p.share_flags & EKV_SHARE_RESET) ? 0 : p.contrib[row];
    s_contrib = prev + c;
    p.contrib[row] = prev + c;
  }

  // 2. The share of each block: exp(u + regain - log total), summed (mean) or maxed over query rows.
  const size_t plane = (size_t)p.layers * p.rows * p.width * Q;
  const float* cell_m = p.lse + ((size_t)p.layer * p.rows + row) * p.width * Q;
  const float* cell_l = cell_m + plane;
  const int tail = n_blocks % TB;
  const int tail_start = n_blocks - tail;
  const float regain = tail ? logf((float)TB / (float)tail) : 0.f;
  const bool reset = (p.share_flags & EKV_SHARE_RESET) != 0;
  const bool agg_max = p.aggregate == EKV_AGG_MAX;
  float* acc = p.share_acc + (size_t)row * p.width;
  const int limit = reset ? p.width : n_blocks;
  for (int b = threadIdx.x; b < limit; b += THREADS) {
    float a = 0.f;
    if (b < n_blocks) {
      const float rg = b >= tail_start ? regain : 0.f;
      for (int j = 0; j < Q; ++j) {
        const float m = __ldcg(cell_m + (size_t)b * Q + j);
        const float l = __ldcg(cell_l + (size_t)b * Q + j);
        const float u = m + logf(l) - log_tb;
        if (s_has[j] && isfinite(u)) {
          const float sh = __expf(u + rg - s_lse[j]);
          a = agg_max ? fmaxf(a, sh) : a + sh;
        }
      }
    }
    const float prev = reset ? 0.f : acc[b];
    acc[b] = agg_max ? fmaxf(prev, a) : prev + a;
  }

  // 3. On the last layer: the normalised share of the row.
  if (p.share_flags & EKV_SHARE_FINALIZE) {
    __syncthreads();
    const int contributors = s_contrib;
    float total = 1.f;
    if (agg_max) {
      float part = 0.f;
      for (int b = threadIdx.x; b < n_blocks; b += THREADS) part += acc[b];
      total = block_sum_fixed_order<THREADS>(part, s_red);
    }
    float* out = p.share_out + (size_t)row * p.width;
    for (int b = threadIdx.x; b < p.width; b += THREADS) {
      float v;
      if (contributors == 0) {
        v = NAN;
      } else if (b >= n_blocks) {
        v = 0.f;
      } else if (agg_max) {
        v = total > 0.f ? acc[b] / total : 0.f;
      } else {
        v = acc[b] / (float)contributors;
      }
      out[b] = v;
    }
  }
}

template <typename T, int D, int TT, int NT>
__global__ void __launch_bounds__(kAuditWarps * 32)
    audit_kernel(const AuditParams p) {
  using L = AuditLayout<D>;
  constexpr int THREADS = kAuditWarps * 32;
  constexpr int TPW = kAuditTilesPerWarp;
  constexpr int CT = EKV_AUDIT_CHUNK_TILES;
  constexpr int STAGE = TT * L::kRowStride;
  constexpr int MT = TT / 16;     // m16 tiles per token tile
  constexpr int KS = D / 16;      // k16 steps over the head dimension
  constexpr int TOK_PER_LANE = (TT + 31) / 32;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + CT * STAGE);
  __shared__ float2 s_merge[kAuditWarps][16];
  __shared__ int s_last;

  const int chunk = blockIdx.x, row = blockIdx.y, head = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (*p.flag == 0) return;  // the statistic is off: this launch records nothing (:64)
  const bool selected = p.select[row] != 0;
  const bool with_share = p.share_acc != nullptr;
  const int BS = p.block_size, TB = p.tile_blocks;

  int len = p.lens[row];
  if (len < 0) len = 0;
  int n_blocks = (len + BS - 1) / BS;
  if (n_blocks > p.width) {
    if (chunk == 0 && head == 0 && threadIdx.x == 0) set_status(p.status, EKV_STATUS_LEN_OVER_WIDTH);
    n_blocks = p.width;
    len = p.width * BS;
  }
  const int token = p.qrow[row];
  const bool bad_qrow = token < 0 || (int64_t)token >= p.q_tokens;
  if (selected && n_blocks > 0 && bad_qrow) {
    if (chunk == 0 && head == 0 && threadIdx.x == 0) set_status(p.status, EKV_STATUS_BAD_QROW);
  }
  const int n_tiles = (n_blocks + TB - 1) / TB;
  const int n_chunks = (n_tiles + CT - 1) / CT;
  if (!selected || n_tiles == 0 || bad_qrow) {
    if (with_share && chunk == 0 && head == 0) audit_row_without_tiles(p, row, selected);
    return;
  }
  if (chunk >= n_chunks) return;

  const int kv_head = p.group + head;
  const T* kbase = static_cast<const T*>(p.k) + (int64_t)kv_head * p.k_s2;
  const int32_t* trow = p.table + (int64_t)row * p.table_s0;

  // ---- issue every bulk copy of this warp's tiles --------------------------------------------
  if (lane == 0) {
    for (int i = 0; i < TPW; ++i) mbar_init(&bars[warp * TPW + i], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const uint64_t policy = l2_evict_first_policy();
  uint32_t vmask[TPW][TOK_PER_LANE];  // ballot of tokens whose block was copied, per tile
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = chunk * CT + i * kAuditWarps + warp;
    uint8_t* stage = smem + (warp * TPW + i) * STAGE;
    uint64_t* bar = &bars[warp * TPW + i];
#pragma unroll
    for (int r = 0; r < TOK_PER_LANE; ++r) vmask[i][r] = 0;
    if (t >= n_tiles) continue;
    int64_t src_off[TOK_PER_LANE];
    uint32_t total = 0;
#pragma unroll
    for (int r = 0; r < TOK_PER_LANE; ++r) {
      const int tok = lane + 32 * r;
      bool ok = false;
      src_off[r] = 0;
      if (tok < TT) {
        const int b = t * TB + tok / BS;
        if (b < n_blocks) {
          const int32_t id = __ldg(trow + b);
          ok = id >= 0 && (int64_t)id < p.pool_blocks;
          if (!ok && tok % BS == 0) set_status(p.status, EKV_STATUS_BAD_BLOCK_ID);
          src_off[r] = (int64_t)id * p.k_s0 + (int64_t)(tok % BS) * p.k_s1;
        }
      }
      vmask[i][r] = __ballot_sync(kFullMask, ok);
      total += __popc(vmask[i][r]);
    }
    if (lane == 0) {
      if (total) {
        mbar_arrive_expect_tx(bar, total * L::kRowBytes);
      } else {
        mbar_arrive(bar);
      }
    }
    __syncwarp();
#pragma unroll
    for (int r = 0; r < TOK_PER_LANE; ++r) {
      if ((vmask[i][r] >> lane) & 1u) {
        const int tok = lane + 32 * r;
        bulk_copy_g2s(stage + tok * L::kRowStride, kbase + src_off[r], L::kRowBytes, bar, policy);
      }
    }
  }

  // ---- the query rows of this KV head, as mma B fragments (k16 x n8, column = query row) ------
  uint32_t bq[NT][KS][2];
  {
    const T* qtok = static_cast<const T*>(p.q) + (int64_t)token * p.q_s0;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int g = nt * 8 + (lane >> 2);
      const bool ok = g < p.G;
      const T* qh = qtok + (int64_t)(kv_head * p.G + (ok ? g : 0)) * p.q_s1;
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int d = s * 16 + 2 * (lane & 3);
        bq[nt][s][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qh + d)) : 0u;
        bq[nt][s][1] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qh + d + 8)) : 0u;
      }
    }
  }

  // ---- consume the tiles in order --------------------------------------------------------------
  const float log_tb = logf((float)TB);
  const size_t plane = (size_t)p.layers * p.rows * p.width * p.Q;
  float* cell_row = p.lse + ((size_t)p.layer * p.rows + row) * p.width * p.Q + head * p.G;
  float run_m[NT][2], run_s[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) run_m[nt][e] = -INFINITY, run_s[nt][e] = 0.f;
  bool timed_out = false;

#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = chunk * CT + i * kAuditWarps + warp;
    if (t >= n_tiles || timed_out) continue;
    uint8_t* stage = smem + (warp * TPW + i) * STAGE;
    if (!mbar_wait_bounded(&bars[warp * TPW + i], 0, p.status)) {
      timed_out = true;
      continue;
    }
    float c[MT][NT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) c[mt][nt][e] = 0.f;
    const uint32_t a_base =
        smem_u32(stage) + ((lane & 7) + ((lane >> 3) & 1) * 8) * L::kRowStride + (lane >> 4) * 16;
#pragma unroll
    for (int s = 0; s < KS; ++s) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t a[4];
        ldmatrix_x4(a, a_base + mt * 16 * L::kRowStride + s * 32);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) Mma<T>::run(c[mt][nt], a, bq[nt][s]);
      }
    }
    // scale, mask tokens at or past the length (or of a skipped block), column max and sum
    const int first = t * TT;
    float mx[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mx[nt][0] = mx[nt][1] = -INFINITY;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int tok = mt * 16 + (lane >> 2) + 8 * h;  // vmask word mt / 2, bit tok % 32
        const bool ok = first + tok < len && ((vmask[i][mt >> 1] >> ((mt & 1) * 16 + (lane >> 2) + 8 * h)) & 1u);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float sc = ok ? c[mt][nt][2 * h + e] * p.scale : -INFINITY;
            c[mt][nt][2 * h + e] = sc;
            mx[nt][e] = fmaxf(mx[nt][e], sc);
          }
      }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1)
          mx[nt][e] = fmaxf(mx[nt][e], __shfl_xor_sync(kFullMask, mx[nt][e], off));
    float sm[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sm[nt][0] = sm[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) sm[nt][e] += __expf(c[mt][nt][2 * h + e] - mx[nt][e]);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1)
          sm[nt][e] += __shfl_xor_sync(kFullMask, sm[nt][e], off);

    // every block cell of the tile inside the row gets the tile's (m, l); lane/4 picks the block
    const int bi = lane >> 2;
    const int b = t * TB + bi;
    if (bi < TB && b < n_blocks) {
      float* cm = cell_row + (size_t)b * p.Q;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int g = nt * 8 + 2 * (lane & 3) + e;
          if (g < p.G) {
            cm[g] = mx[nt][e];
            cm[g + plane] = sm[nt][e];
          }
        }
    }
    if (with_share) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float u = mx[nt][e] + logf(sm[nt][e]) - log_tb;
          if (isfinite(u)) lse_merge(run_m[nt][e], run_s[nt][e], u, 1.f);
        }
    }
  }
  if (timed_out) {
    // Let every copy still in flight land before the CTA's shared memory is released.
#pragma unroll
    for (int i = 0; i < TPW; ++i) {
      const int t = chunk * CT + i * kAuditWarps + warp;
      if (t < n_tiles) mbar_wait_bounded(&bars[warp * TPW + i], 0, p.status);
    }
  }
  if (!with_share) return;

  // ---- this CTA's (max, sum) partial per query row, then the row ticket ------------------------
  if (lane < 4) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) s_merge[warp][nt * 8 + 2 * lane + e] = make_float2(run_m[nt][e], run_s[nt][e]);
  }
  __syncthreads();
  if (threadIdx.x < p.G) {
    float m = -INFINITY, s = 0.f;
    for (int w = 0; w < kAuditWarps; ++w) lse_merge(m, s, s_merge[w][threadIdx.x].x, s_merge[w][threadIdx.x].y);
    p.partials[((size_t)row * p.max_chunks + chunk) * p.Q + head * p.G + threadIdx.x] = make_float2(m, s);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t ticket = atomicAdd(&p.tickets[row], 1u);
    s_last = ticket == (uint32_t)(n_chunks * p.heads - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x == 0) p.tickets[row] = 0;  // ready for the next launch
  audit_share_epilogue<THREADS>(p, row, n_blocks, n_chunks);
}

template <typename T, int D, int TT, int NT>
int launch_audit(const AuditParams& p, cudaStream_t stream) {
  using L = AuditLayout<D>;
  constexpr int smem = EKV_AUDIT_CHUNK_TILES * TT * L::kRowStride + EKV_AUDIT_CHUNK_TILES * 8;
  static bool configured[kMaxDevices] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return check_launch("cudaGetDevice");
  if (!configured[device]) {
    if (cudaFuncSetAttribute(audit_kernel<T, D, TT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(audit_kernel)");
    configured[device] = true;
  }
  const int tiles = cdiv(p.width, p.tile_blocks);
  dim3 grid(cdiv(tiles, EKV_AUDIT_CHUNK_TILES), p.rows, p.heads);
  audit_kernel<T, D, TT, NT><<<grid, kAuditWarps * 32, smem, stream>>>(p);
  return check_launch("audit_kernel");
}

template <typename T>
int dispatch_audit(const AuditParams& p, int tt, cudaStream_t stream) {
  const int nt = p.G <= 8 ? 1 : 2;
  switch (tt * 4 + nt) {
    case 16 * 4 + 1: return launch_audit<T, 128, 16, 1>(p, stream);
    case 16 * 4 + 2: return launch_audit<T, 128, 16, 2>(p, stream);
    case 32 * 4 + 1: return launch_audit<T, 128, 32, 1>(p, stream);
    case 32 * 4 + 2: return launch_audit<T, 128, 32, 2>(p, stream);
    case 64 * 4 + 1: return launch_audit<T, 128, 64, 1>(p, stream);
    case 64 * 4 + 2: return launch_audit<T, 128, 64, 2>(p, stream);
    default: break;
  }
  return fail(EKV_ENOTSUP, "no audit kernel for a tile of %d tokens", tt);
}

size_t audit_ticket_bytes(int rows) { return round_up((size_t)rows * 4, 256); }

}  // namespace ekv

using namespace ekv;

extern "C" size_t ekv_audit_workspace_bytes(int rows, int width, int group_rows, int heads,
                                            int block_size, int tile_blocks) {
  (void)block_size;
  if (rows <= 0 || width <= 0 || group_rows <= 0 || heads <= 0 || tile_blocks <= 0) return 0;
  const int chunks = cdiv(cdiv(width, tile_blocks), EKV_AUDIT_CHUNK_TILES);
  return audit_ticket_bytes(rows) + (size_t)rows * chunks * heads * group_rows * sizeof(float2);
}

extern "C" int ekv_audit_launch(
    const void* q, const void* k, const int32_t* table, const int32_t* lens, const int32_t* qrow,
    const uint8_t* select, const uint32_t* flag, float* lse, float scale, int layer, int group,
    int64_t q_stride_token, int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos,
    int64_t k_stride_head, int64_t table_stride, int layers, int rows, int width, int group_rows,
    int block_size, int tile_blocks, int head_dim, int dtype, int heads, int kv_heads,
    int64_t pool_blocks, int64_t q_tokens, float* share_acc, int32_t* contributors,
    float* share_out, int aggregate, int share_flags, void* workspace, size_t workspace_bytes,
    uint32_t* status, void* stream) {
  clear_error();
  if (!q || !k || !table || !lens || !qrow || !select || !flag || !lse)
    return fail(EKV_EINVAL, "a required device pointer is NULL");
  if (rows <= 0 || width <= 0 || layers <= 0)
    return fail(EKV_EINVAL, "rows, width and layers must be positive");
  if (layer < 0 || layer >= layers)
    return fail(EKV_ERANGE, "layer %d is outside the %d layers the table was sized for", layer, layers);
  if (group_rows < 1 || group_rows > 16)
    return fail(EKV_EINVAL, "%d query heads per KV head: the kernel handles 1 to 16", group_rows);
  if (heads < 1 || group < 0 || group + heads > kv_heads)
    return fail(EKV_EINVAL, "KV heads [%d, %d) are outside the cache's %d heads", group, group + heads, kv_heads);
  if (heads * group_rows > kMaxQ)
    return fail(EKV_ENOTSUP, "%d values per cell exceed %d", heads * group_rows, kMaxQ);
  if (block_size <= 0 || tile_blocks <= 0)
    return fail(EKV_EINVAL, "block_size and tile_blocks must be positive");
  if (tile_blocks > 8) return fail(EKV_ENOTSUP, "tile_blocks %d: this build handles up to 8", tile_blocks);
  if (rows > 65535 || heads > 64) return fail(EKV_ENOTSUP, "rows <= 65535 and heads <= 64");
  const int tt = block_size * tile_blocks;
  if (tt & (tt - 1)) return fail(EKV_EINVAL, "a tile of the audit kernel must hold a power of two of tokens");
  if (head_dim != 128) return fail(EKV_ENOTSUP, "head_dim %d: this build has kernels for 128", head_dim);
  if (dtype != EKV_DTYPE_F16 && dtype != EKV_DTYPE_BF16) return fail(EKV_EINVAL, "unknown dtype %d", dtype);
  if (pool_blocks <= 0 || q_tokens <= 0) return fail(EKV_EINVAL, "pool_blocks and q_tokens must be positive");
  // Bulk copies move whole 256-byte key rows; the query is read as pairs of elements.
  if (((uintptr_t)k & 15) || (k_stride_block & 7) || (k_stride_pos & 7) || (k_stride_head & 7))
    return fail(EKV_EINVAL, "the key cache must be 16-byte aligned with strides of whole 16-byte units");
  if (((uintptr_t)q & 3) || (q_stride_token & 1) || (q_stride_head & 1))
    return fail(EKV_EINVAL, "the query must be 4-byte aligned with even strides");
  if (table_stride < width) return fail(EKV_EINVAL, "table_stride %lld < width %d", (long long)table_stride, width);
  if (aggregate != EKV_AGG_MEAN && aggregate != EKV_AGG_MAX) return fail(EKV_EINVAL, "unknown aggregate %d", aggregate);

  AuditParams p{};
  p.q = q; p.k = k; p.table = table; p.lens = lens; p.qrow = qrow; p.select = select; p.flag = flag;
  p.lse = lse; p.scale = scale; p.layer = layer; p.group = group;
  p.q_s0 = q_stride_token; p.q_s1 = q_stride_head;
  p.k_s0 = k_stride_block; p.k_s1 = k_stride_pos; p.k_s2 = k_stride_head; p.table_s0 = table_stride;
  p.layers = layers; p.rows = rows; p.width = width; p.G = group_rows; p.heads = heads;
  p.Q = heads * group_rows; p.block_size = block_size; p.tile_blocks = tile_blocks;
  p.pool_blocks = pool_blocks; p.q_tokens = q_tokens;
  p.share_acc = share_acc; p.contrib = contributors; p.share_out = share_out;
  p.aggregate = aggregate; p.share_flags = share_flags; p.status = status;
  p.max_chunks = cdiv(cdiv(width, tile_blocks), EKV_AUDIT_CHUNK_TILES);
  if (share_acc) {
    if (!contributors) return fail(EKV_EINVAL, "share_acc needs contributors");
    if ((share_flags & EKV_SHARE_FINALIZE) && !share_out) return fail(EKV_EINVAL, "EKV_SHARE_FINALIZE needs share_out");
    const size_t need = ekv_audit_workspace_bytes(rows, width, group_rows, heads, block_size, tile_blocks);
    if (!workspace || workspace_bytes < need)
      return fail(EKV_ERANGE, "the audit workspace holds %zu bytes, the launch needs %zu", workspace_bytes, need);
    if ((uintptr_t)workspace & 255) return fail(EKV_EINVAL, "the audit workspace must be 256-byte aligned");
    p.tickets = static_cast<uint32_t*>(workspace);
    p.partials = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + audit_ticket_bytes(rows));
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == EKV_DTYPE_BF16 ? dispatch_audit<__nv_bfloat16>(p, tt, s) : dispatch_audit<__half>(p, tt, s);
}
