/*
 * ekv_b200.h -- C ABI of libekv_b200.so, the sm_100a implementation of KVScope's attention-share
 * audit and block-table view path.
 *
 * Every entry point takes plain device pointers, element strides and sizes, and a CUDA stream given
 * as `void*` (a cudaStream_t; NULL is the legacy default stream). None allocates device memory, none
 * synchronises the host, and each launches a grid whose shape depends on its size arguments only, so
 * a sequence of calls can be captured in a CUDA graph. Every function returns EKV_OK (0) or a
 * negative EKV_E* code; ekv_last_error_string() then describes the failure (thread-local).
 *
 * Citations point into the reference project (jc-su/SIGMOD-KVSCOPE) by path:line.
 */
#ifndef EKV_B200_H
#define EKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes ---------------------------------------------------------------------------- */
#define EKV_OK 0
#define EKV_EINVAL (-1)  /* a shape, stride or argument error: the Python layer raises ValueError   */
#define EKV_ERANGE (-2)  /* a count beyond what a buffer was sized for: RuntimeError                 */
#define EKV_ENOTSUP (-3) /* a configuration this build has no kernel for: RuntimeError               */
#define EKV_ECUDA (-4)   /* the CUDA runtime reported an error at launch: RuntimeError               */

/* ---- element types of the query and the key cache --------------------------------------------- */
#define EKV_DTYPE_F16 0
#define EKV_DTYPE_BF16 1

/* ---- how the shares of layers and query rows combine (observe/tile_shares.py:58-103) ------------- */
#define EKV_AGG_MEAN 0
#define EKV_AGG_MAX 1

/* ---- share_flags of ekv_audit_launch --------------------------------------------------------- */
#define EKV_SHARE_FINALIZE 2 /* this launch ends the audit step: combine its layers into share_out   */

/* ---- bits a kernel ORs into the optional device status word ---------------------------------- */
#define EKV_STATUS_BAD_BLOCK_ID 1u  /* a table entry outside [0, pool_blocks): its keys were skipped */
#define EKV_STATUS_LEN_OVER_WIDTH 2u /* a length beyond width*block_size: clamped to the table width */
#define EKV_STATUS_BAD_QROW 4u      /* a query token index outside [0, q_tokens): the row was skipped */
#define EKV_STATUS_WAIT_TIMEOUT 8u  /* a bounded wait on a bulk copy gave up: the output is invalid  */

/* ---- ranking policies of the view builder (observe/allocation.py:79-118, daemon.py:49) --------- */
#define EKV_POLICY_SUM 0     /* highest share first; equal shares: the newer block first           */
#define EKV_POLICY_UNIFORM 1 /* highest share first; equal shares: the older block first           */
#define EKV_POLICY_NEWEST 2  /* the fixed rule scores = arange(n): the newest open blocks           */
#define EKV_POLICY_MAXMIN 3  /* ekv_allocate_pinned_f64's objective: raise the lowest retained share */

/* Tiles of one audit work item (a chunk of a row): the unit a warp of the audit kernel takes. */
#define EKV_AUDIT_CHUNK_TILES 8

/* Human-readable description of the last error on this thread ("" if none). */
const char* ekv_last_error_string(void);

/* ABI version of this library: bumped on any change of a signature or of a documented contract. */
int ekv_abi_version(void);

/* Bytes of workspace ekv_audit_step needs for a table of `layers` layers (rows and width do not change
 * it): the step's work counter and the key cache's TMA descriptor per layer (128 bytes each), both
 * rewritten by every step, so its contents never matter; 256-byte aligned. ekv_audit_launch needs
 * none: its workspace arguments may be NULL and 0 (a workspace given is not used). */
size_t ekv_audit_workspace_bytes(int layers, int rows, int width);

/*
 * ekv_audit_launch -- record the attention-share statistic of one layer.
 *
 * Replaces the Triton launch of tile_lse_kernel at runtime/audit_kernel.py:239-265 (kernel body
 * :34-109); the first 22 arguments keep that kernel's names and meaning:
 *   q        [tokens, q_heads, head_dim] query of the step, element strides q_stride_token/head;
 *   k        [pool_blocks, block_size, kv_heads, head_dim] key cache of the layer (kv_cache[:, 0]);
 *   table    int32 [rows, width] block table (row stride table_stride), lens int32 [rows] tokens;
 *   qrow     int32 [rows] token index of each row's query; select uint8 [rows]; flag uint32 [1];
 *   lse      float32 [2][layers][rows][width][heads*group_rows]: plane 0 the tile max m, plane 1 the
 *            tile sum l, written into every block cell of a tile whose first token is < lens[row].
 * For each row with select != 0 (and only when *flag != 0), KV head `group + h` for h < heads, and
 * each tile of tile_blocks*block_size tokens, it computes m = max_j q.k_j*scale and
 * l = sum_j exp(q.k_j*scale - m) over the tile's tokens below lens[row]. heads = 1 is the
 * reference's sampling (one KV group per layer, group = layer % kv_heads, :250).
 *
 * With share_out != NULL and EKV_SHARE_FINALIZE (the step's last layer) the same call then turns
 * the cells of every layer [0, layers) into the exact per-block attention share: one kernel, a
 * cluster of CTAs per row, reads the cells back from L2 and forms the block shares as
 * normalize_tile_lse computes them (observe/tile_shares.py:58-103 with row_blocks =
 * ceil(lens/block_size)), taking the mean or max over layers and query rows, into share_out
 * [rows][width] and contributors [rows] ((layer, query row) pairs with data); a row that is not
 * selected or has no data is NaN. The share pass handles rows of up to 32768 tiles.
 * status (optional) receives EKV_STATUS_* bits. q_tokens bounds qrow. Supported: head_dim 128,
 * block_size a multiple of 8 (the key cache is read a block at a time through a TMA tensor map),
 * block_size*tile_blocks in {16, 32, 64}, tile_blocks <= 8, heads*group_rows <= 128,
 * group_rows <= 16, rows <= 2048, pool_blocks < 2^31, key-cache strides in whole 16-byte units.
 */
int ekv_audit_launch(const void* q, const void* k, const int32_t* table, const int32_t* lens,
                     const int32_t* qrow, const uint8_t* select, const uint32_t* flag, float* lse,
                     float scale, int layer, int group, int64_t q_stride_token,
                     int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos,
                     int64_t k_stride_head, int64_t table_stride, int layers, int rows, int width,
                     int group_rows, int block_size, int tile_blocks, int head_dim, int dtype,
                     int heads, int kv_heads, int64_t pool_blocks, int64_t q_tokens,
                     float* share_out, int32_t* contributors, int aggregate, int share_flags,
                     void* workspace, size_t workspace_bytes, uint32_t* status, void* stream);

/*
 * ekv_audit_stash -- keep one layer's queries for a later ekv_audit_step.
 *
 * Copies q[qrow[r], (group + h) * group_rows + g, :] to stash[r][h * group_rows + g][:] for every row
 * r < rows, h < heads, g < group_rows (16-byte aligned buffers). The deferred form of
 * RecordingPlane.record: the engine reuses its query buffer across layers, the stash does not.
 */
int ekv_audit_stash(const void* q, int64_t q_stride_token, int64_t q_stride_head, const int32_t* qrow,
                    int rows, int64_t q_tokens, int group, int heads, int group_rows, int head_dim,
                    void* stash, uint32_t* status, void* stream);

/*
 * ekv_audit_step -- every layer of an audit step in one launch.
 *
 * The work of n_layers ekv_audit_launch calls for layers [layer0, layer0 + n_layers), the last one
 * finalising, in one persistent launch. k_layers and q_layers are device arrays of uint64 addresses
 * per table layer: the key cache of layer L (as the plane's layer table holds them,
 * runtime/audit.py:86-100) and its queries, laid out as the engine's query (q_layout 0: query head
 * (KV head) * group_rows + g) or as a stash (q_layout 1: query head h * group_rows + g). The KV head
 * of layer L is (group + L) % kv_heads with rotate != 0 (the reference's sampling), else
 * group + h for h < heads. The workspace is required: it holds each layer's key-cache descriptor
 * (built on the device from k_layers by a small kernel ahead of the record kernel) and the work
 * counter of the record kernel's dynamic items. share_out and
 * contributors are optional: without them only the cells are recorded.
 */
int ekv_audit_step(const uint64_t* q_layers, const uint64_t* k_layers, const int32_t* table,
                   const int32_t* lens, const int32_t* qrow, const uint8_t* select,
                   const uint32_t* flag, float* lse, float scale, int layer0, int n_layers,
                   int group, int rotate, int q_layout, int64_t q_stride_token,
                   int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos,
                   int64_t k_stride_head, int64_t table_stride, int layers, int rows, int width,
                   int group_rows, int block_size, int tile_blocks, int head_dim, int dtype,
                   int heads, int kv_heads, int64_t pool_blocks, int64_t q_tokens,
                   float* share_out, int32_t* contributors, int aggregate, void* workspace,
                   size_t workspace_bytes, uint32_t* status, void* stream);

/*
 * ekv_audit_step_static -- ekv_audit_step for callers that cannot allocate device memory.
 *
 * No counterpart in the reference: an addition of this library. Some callers cannot call cudaMalloc
 * when they record -- a binding with no CUDA allocator of its own (a cgo or ctypes caller that only
 * holds the engine's tensors), or engine code after memory profiling has sized the KV-cache pool,
 * where one more allocation can fail or fragment it. This entry point takes no workspace: it uses a
 * static device array of ekv_audit_static_scratch_bytes() bytes (128.25 KiB: the workspace of a step
 * of 1024 layers, the most this build accepts) that every GPU loading the library holds until exit,
 * and rejects with EKV_ERANGE a step whose ekv_audit_workspace_bytes() exceeds it. The caller still
 * passes every input and output. It allocates nothing: the first call on a device looks the array's
 * device address up (cudaGetSymbolAddress), so make that first call before any stream capture. Every
 * call shares the array (each step rewrites all of it that it reads); calls whose launches overlap on
 * the GPU race.
 */
size_t ekv_audit_static_scratch_bytes(void);
int ekv_audit_step_static(const uint64_t* q_layers, const uint64_t* k_layers, const int32_t* table,
                          const int32_t* lens, const int32_t* qrow, const uint8_t* select,
                          const uint32_t* flag, float* lse, float scale, int layer0, int n_layers,
                          int group, int rotate, int q_layout, int64_t q_stride_token,
                          int64_t q_stride_head, int64_t k_stride_block, int64_t k_stride_pos,
                          int64_t k_stride_head, int64_t table_stride, int layers, int rows,
                          int width, int group_rows, int block_size, int tile_blocks, int head_dim,
                          int dtype, int heads, int kv_heads, int64_t pool_blocks, int64_t q_tokens,
                          float* share_out, int32_t* contributors, int aggregate, uint32_t* status,
                          void* stream);

/*
 * ekv_normalize_tile_lse -- the controller's read of the statistic, on the device.
 *
 * Replaces read_tile_rows (observe/tile_shares.py:129-173) followed by normalize_tile_lse
 * (:58-103), as TileShareSource.read calls them (observe/controller.py:111-136). For the count rows
 * row_ids[i] (int32, any order) of the table lse (layout as above, `table_layers` layers of which the
 * first `layers` are read, group_rows values per cell), it forms u = m + log(l) - log(tile_blocks),
 * gives a partial last tile's weight back to its blocks, drops cells at or beyond row_blocks[i],
 * softmax-normalises each (layer, row, query row) and takes the mean or max over layers and query
 * rows. share [count][width] float32; NaN rows where no (layer, query row) has a finite value.
 * contributors (optional) [count] receives the number of (layer, query row) pairs with data.
 */
int ekv_normalize_tile_lse(const float* lse, int table_layers, int layers, int rows, int width,
                           int group_rows, const int32_t* row_ids, const int32_t* row_blocks,
                           int count, int tile_blocks, int aggregate, float* share,
                           int32_t* contributors, void* stream);

/*
 * ekv_normalize_log_weights -- normalize_tile_lse (observe/tile_shares.py:58-103) on the device for
 * u values already read: u float32 [layers][rows][width][group_rows], row_blocks int32 [rows].
 * share [rows][width] float32 and contributors (optional) [rows] as in ekv_normalize_tile_lse.
 */
int ekv_normalize_log_weights(const float* u, int layers, int rows, int width, int group_rows,
                              const int32_t* row_blocks, int tile_blocks, int aggregate,
                              float* share, int32_t* contributors, void* stream);

/*
 * ekv_share_finalize -- normalise accumulated shares when no launch carried EKV_SHARE_FINALIZE.
 * share_out[r] = share_acc[r] / contributors[r] (mean) or share_acc[r] / sum(share_acc[r]) (max);
 * NaN rows where contributors is 0 or select[r] is 0 (select may be NULL).
 */
int ekv_share_finalize(const float* share_acc, const int32_t* contributors, const uint8_t* select,
                       int rows, int width, int aggregate, float* share_out, void* stream);

/*
 * ekv_allocate_quotas -- how many unpinned blocks each row keeps.
 *
 * The budget arithmetic of Controller._allocate (observe/controller.py:398-451) and the quotas of
 * allocate/_uniform (observe/allocation.py:55-91). Row r holds row_blocks[r] blocks; it is measured
 * when row_blocks[r] > cap_above_blocks (and > 0). Its pins are block 0, the newest
 * recent_blocks + 1 blocks (none for recent_blocks = -1), and the blocks from measured_blocks[r] on
 * (measured_blocks may be NULL). With row_fraction == NULL the measured rows share one budget --
 * `budget` when it is >= 0 (allocate()'s argument), else max(pins, ceil(budget_fraction * blocks))
 * as the controller computes it -- split by `uniform` quotas with largest remainders (objective
 * EKV_POLICY_UNIFORM or EKV_POLICY_NEWEST). With row_fraction != NULL (float64 [rows]) every row is
 * its own allocate() call with budget max(pins, ceil(row_fraction[r] * row_blocks[r])) (any
 * objective). A measured row of more than `width` blocks (width > 0) takes part with width of them,
 * as the controller's n = min(length, row_width) (controller.py:414); width = 0 sets no limit.
 * quota [rows] int32: the unpinned blocks to keep, or -1 for a row that is not measured
 * (it reads in full). One CTA; rows <= 8192 for a shared budget, <= 65536 otherwise.
 */
int ekv_allocate_quotas(const int32_t* row_blocks, const int32_t* measured_blocks,
                        int recent_blocks, int cap_above_blocks, double budget_fraction,
                        int64_t budget, const double* row_fraction, int objective, int rows,
                        int width, int32_t* quota, void* stream);

/*
 * ekv_decode_view -- DecodeView.build on the device: keep algebra, compaction and read counters in one
 * kernel (runtime/block_view.py:272-329).
 *
 * row_flags uint8 [rows]: bit 0 the row reads every block (an expired lease, an audited row, a prefill
 * row), bit 1 it decodes, bit 2 it is audited. keep uint8 [rows][keep_stride] is the committed mask;
 * released (may be NULL) removes blocks last, so nothing brings a released block back. The view and its
 * lengths are those of compact_block_table (:36-56). counts (int64 [5], may be NULL) receives, over the
 * decoding rows, the blocks read, the blocks a full read would read, the blocks read by audited rows, by
 * rows read whole under a live policy without an audit, and (expired != 0) all blocks read while no
 * policy is live. width <= 16384.
 */
int ekv_decode_view(const int32_t* table, int64_t table_stride, const int32_t* seq_lens, const uint8_t* keep,
                    int64_t keep_stride, const uint8_t* row_flags, const uint8_t* released,
                    int64_t released_stride, int expired, int rows, int width, int block_size, int32_t* view,
                    int64_t view_stride, int32_t* view_lens, int64_t* counts, void* stream);

/* Bytes of workspace ekv_allocate_maxmin needs for `rows` rows of `width` blocks (256-byte aligned). */
size_t ekv_allocate_maxmin_workspace_bytes(int rows, int width);

/*
 * ekv_allocate_maxmin -- the quotas of the `maxmin` objective with one budget shared by every measured row.
 *
 * Replaces allocate(requests, budget, "maxmin") (observe/allocation.py:55-76 and _water_level :121-166):
 * the highest retained-share level the budget affords (60 bisection steps over each request's running
 * sums of its unpinned shares in decreasing order, float64 as NumPy computes them), then the blocks left
 * over one at a time to the request with the lowest retained share (ties: the earlier request). Rows,
 * pins, budget and quota as in ekv_allocate_sum (no weights: maxmin does not use them); the quotas are
 * for ekv_view_build with EKV_POLICY_UNIFORM (equal shares to the older block). width <= 8192,
 * rows <= 4096. Three kernels and one memset on `stream`, no host synchronisation.
 */
int ekv_allocate_maxmin(const float* scores, int64_t score_stride, const int32_t* row_blocks,
                        const int32_t* measured_blocks, int recent_blocks, int cap_above_blocks,
                        double budget_fraction, int64_t budget, int rows, int width, int32_t* quota,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * ekv_slot_compact -- the view of SGLang's CSR key-value list, in place (runtime/sglang_compact.py:22-167,
 * SlotCompactor.compact :131-167).
 *
 * Row r of the batch reads slots[indptr[r] : indptr[r + 1]] (int32 indptr [n_rows + 1]; slot entries of
 * slot_bytes = 4 or 8 bytes; entries = indptr[n_rows], the list's length as the host knows it). Blocks
 * are block_tokens consecutive entries. A row keeps its first and last block always, and a block b < width
 * when keep[r][b] != 0 (uint8 or bool, row stride keep_stride), or every block when active == 0, when
 * audit (uint8 [n_rows], may be NULL) marks it, or when r >= n_real (rows a CUDA graph adds). Writes the
 * new lengths lens [n_rows], the kept blocks of each row in order to table [n_rows][table_stride], the new
 * indptr to new_indptr [n_rows + 1] and then to indptr, and the new list to out [entries] and then to
 * slots; adds to counts (int64 [5]: blocks read, blocks a full read reads, read in audits, read untrimmed,
 * read with no live policy) over the rows before n_real. Rows must hold at most width blocks. Three
 * kernels, no host synchronisation.
 */
int ekv_slot_compact(int32_t* indptr, void* slots, int slot_bytes, const uint8_t* keep, int64_t keep_stride,
                     const uint8_t* audit, int active, int n_real, int n_rows, int64_t entries,
                     int block_tokens, int width, int32_t* new_indptr, int32_t* lens, int32_t* table,
                     int64_t table_stride, int64_t* counts, void* out, void* stream);

/* Bytes of workspace ekv_allocate_sum needs for `rows` rows of `width` blocks (256-byte aligned). */
size_t ekv_allocate_sum_workspace_bytes(int rows, int width);

/*
 * ekv_allocate_sum -- the quotas of the `sum` objective with one budget shared by every measured row.
 *
 * Replaces allocate(requests, budget, "sum") over several requests (observe/allocation.py:55-76 and
 * _greedy :94-118), the controller's default objective (observe/controller.py:30, :398-451). Row r
 * is a request when row_blocks[r] > cap_above_blocks (and > 0); its n = min(row_blocks[r], width)
 * scores are scores[r][0..n) (float32, row stride score_stride; NaN counts as 0), its weight
 * weights[r] (float64; NULL: 1.0), its pins those of ekv_allocate_quotas. The budget is `budget` when
 * it is >= 0, else max(pins, ceil(budget_fraction * blocks)). The reference keeps the `free`
 * unpinned blocks of largest weight * max(score, 0) / total (float64, total = NumPy's pairwise sum
 * of the request's clamped scores), equal gains to the newer block, then to the earlier request;
 * this call computes, bit-exactly, how many of them fall in each row: quota [rows] int32 for
 * ekv_view_build with EKV_POLICY_SUM and the same pins, or -1 for a row that is not a request.
 * width <= 32768. Nine kernels and one memset on `stream`, no host synchronisation.
 */
int ekv_allocate_sum(const float* scores, int64_t score_stride, const double* weights,
                     const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                     int cap_above_blocks, double budget_fraction, int64_t budget, int rows, int width,
                     int32_t* quota, void* workspace, size_t workspace_bytes, void* stream);

/*
 * ekv_allocate_sum_f64 -- ekv_allocate_sum over float64 scores, which float32 need not hold
 * (the controller's smoothed shares, observe/controller.py:340-343).
 *
 * Row r's scores are scores[score_rows[r]][0..n) (score_rows may be NULL: row r), so a ledger of shares
 * per request (ekv_ledger_absorb) is read in place. The quotas are for ekv_view_build_f64 with
 * EKV_POLICY_SUM, the same weights and the same pins. mask_out (may be NULL; uint8 [rows][mask_stride])
 * receives the committed mask straight from the threshold -- the pins, the blocks past a request and
 * every row that is not a request kept -- with no view launch: the mask ekv_view_build_f64 would write.
 * width <= 16384. Same workspace as ekv_allocate_sum.
 */
int ekv_allocate_sum_f64(const double* scores, int64_t score_stride, const int32_t* score_rows,
                         const double* weights, const int32_t* row_blocks, const int32_t* measured_blocks,
                         int recent_blocks, int cap_above_blocks, double budget_fraction, int64_t budget,
                         int rows, int width, int32_t* quota, uint8_t* mask_out, int64_t mask_stride,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * ekv_view_build_sum_budget -- the controller's default decision and its view in one call: one `sum`
 * budget over every measured row (Controller._allocate, observe/controller.py:398-451, with
 * allocate(objective="sum"), observe/allocation.py:94-118), then compact_block_table
 * (runtime/block_view.py:36-56) of every row.
 *
 * The select of ekv_allocate_sum / ekv_allocate_sum_f64 (score_bytes 4: float32 scores, 8: float64,
 * score_rows as in ekv_allocate_sum_f64) finds the threshold gain; the view kernel then keeps, in every
 * request, the unpinned blocks whose gain is above it (equal gains as the reference hands them out: newer
 * blocks first, then earlier requests), with no per-row ranking and no quotas. The view, its lengths,
 * full_rows and released as in ekv_view_build; mask_out (may be NULL) receives the committed mask. The
 * result is the view ekv_view_build (_f64) writes with ekv_allocate_sum's (_f64's) quotas and the same
 * pins and weights. width <= 16384. Same workspace as ekv_allocate_sum.
 */
int ekv_view_build_sum_budget(const void* scores, int score_bytes, int64_t score_stride, const int32_t* score_rows,
                              const double* weights, const int32_t* row_blocks, const int32_t* measured_blocks,
                              int recent_blocks, int cap_above_blocks, double budget_fraction, int64_t budget,
                              const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                              const uint8_t* full_rows, const uint8_t* released, int64_t released_stride, int rows,
                              int width, int block_size, int32_t* view, int64_t view_stride, int32_t* view_lens,
                              uint8_t* mask_out, int64_t mask_stride, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * ekv_allocate_maxmin_f64 -- ekv_allocate_maxmin over float64 scores; score_rows as in
 * ekv_allocate_sum_f64. The quotas are for ekv_view_build_f64 with EKV_POLICY_UNIFORM. width <= 8192,
 * rows <= 4096. Same workspace as ekv_allocate_maxmin.
 */
int ekv_allocate_maxmin_f64(const double* scores, int64_t score_stride, const int32_t* score_rows,
                            const int32_t* row_blocks, const int32_t* measured_blocks, int recent_blocks,
                            int cap_above_blocks, double budget_fraction, int64_t budget, int rows, int width,
                            int32_t* quota, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace ekv_allocate_pinned_f64 needs (256-byte aligned); 0 when width > 16383. */
size_t ekv_allocate_pinned_workspace_bytes(int rows, int width);

/*
 * ekv_allocate_pinned_f64 -- allocate(requests, budget, objective) with any pinned blocks.
 *
 * Replaces allocate (observe/allocation.py:55-76 with _uniform :79-91, _greedy :94-118 and
 * _water_level :121-166) for requests whose Request.pinned marks any blocks (:37-44), not only the
 * controller's block 0 and newest suffix. Row r is request r: its n = row_blocks[r] (<= width) float64
 * scores scores[r][0..n) (NaN counts as 0), pinned[r][0..n) (uint8, nonzero: always kept, not counted
 * against the open blocks), weights[r] (float64 [rows], `sum` only; NULL: 1.0). objective is
 * EKV_POLICY_SUM, EKV_POLICY_UNIFORM or EKV_POLICY_MAXMIN. The caller has already checked what the
 * reference checks on the host: budget >= the pinned blocks of every request, and budget < the blocks
 * of every request (else every block is kept). Each request's shares are computed once, as
 * Request.shares computes them (max(score, 0) / total, total NumPy's pairwise sum in block order), and
 * ranked with the reference's tie rules; mask_out[r][0..n) (uint8, row stride mask_stride) receives
 * each request's keep mask, [n, width) zero. width <= 16383 (maxmin: 8191). Seven to fourteen kernels
 * and one memset on `stream`, no host synchronisation.
 */
int ekv_allocate_pinned_f64(const double* scores, int64_t score_stride, const uint8_t* pinned,
                            int64_t pinned_stride, const double* weights, const int32_t* row_blocks, int objective,
                            int64_t budget, int rows, int width, uint8_t* mask_out, int64_t mask_stride,
                            void* workspace, size_t workspace_bytes, void* stream);

/*
 * ekv_view_build_f64 -- ekv_view_build in ranking mode over float64 scores.
 *
 * A request's unpinned blocks are ranked by the float64 value the reference ranks: its gain
 * weight * share (EKV_POLICY_SUM, allocation.py:107) or its share (EKV_POLICY_UNIFORM, :89; weights
 * then must be NULL or 1), share = max(score, 0) / total with total NumPy's pairwise sum of the
 * request's clamped scores (1 / n when it is not positive, :46-52); distinct scores with equal shares
 * tie. scores[score_rows[r]] (score_rows may be NULL: row r), weights [rows] float64 (NULL: 1.0).
 * view == NULL writes mask_out only (the controller's committed mask, controller.py:401, :445): table,
 * seq_lens and view_lens are then not read. width <= 16384.
 */
int ekv_view_build_f64(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                       const int32_t* row_blocks, const int32_t* quota, const int32_t* measured_blocks,
                       int recent_blocks, const double* scores, int64_t score_stride, const int32_t* score_rows,
                       const double* weights, int policy, const uint8_t* full_rows, const uint8_t* released,
                       int64_t released_stride, int rows, int width, int block_size, int32_t* view,
                       int64_t view_stride, int32_t* view_lens, uint8_t* mask_out, int64_t mask_stride,
                       void* stream);

/*
 * ekv_ledger_absorb -- fold one audit's shares into the per-request shares (Controller._absorb_audit,
 * observe/controller.py:332-345).
 *
 * fresh [rows][fresh_stride] (float32, or float64 when fresh_f64 != 0) is the audit's share of each row.
 * Row r belongs to the request whose shares are ledger row slot[r] (float64 [ledger_rows][ledger_stride]);
 * slot[r] < 0 (or >= ledger_rows) skips the row. A row with no value other than NaN carries no evidence:
 * evidence[r] = 0 and the ledger is left alone. Otherwise evidence[r] = 1 and the ledger row becomes
 * nan_to_num(fresh[r]) (blend[r] == 0: a request with no shares yet) or
 * decay * ledger + (1 - decay) * nan_to_num(fresh[r]), rounded as NumPy rounds it. decay in [0, 1).
 * The slots of one call must be distinct. One kernel, no host synchronisation.
 */
int ekv_ledger_absorb(const void* fresh, int fresh_f64, int64_t fresh_stride, const int32_t* slot,
                      const uint8_t* blend, double decay, int rows, int width, double* ledger,
                      int64_t ledger_stride, int ledger_rows, uint8_t* evidence, void* stream);

/*
 * ekv_view_build -- the per-row keep decision and the compacted block-table view, in one kernel.
 *
 * Ranking mode (keep == NULL): row r keeps its pins (as in ekv_allocate_quotas, recent_blocks >= -1)
 * and the quota[r]
 * best unpinned blocks among its first row_blocks[r], ranked by max(scores, 0) (float32, NaN as 0)
 * under `policy` -- the per-request ranking of allocation.py:89 (uniform) and :107-113 (sum, one
 * request) -- or the newest ones (EKV_POLICY_NEWEST); blocks at or beyond row_blocks[r] are kept,
 * and quota[r] < 0 keeps every block. mask_out (optional, uint8 [rows][width]) receives this mask,
 * the row the controller commits (controller.py:401, :445).
 * Mask mode (keep != NULL, uint8): the committed mask is `keep`.
 * Then, as DecodeView.build (runtime/block_view.py:272-292): rows with full_rows[r] != 0 keep every
 * block, released blocks (optional uint8 mask) are dropped, and compact_block_table
 * (runtime/block_view.py:36-56) keeps block 0 and the last block of ceil(seq_lens/block_size),
 * writes the kept blocks in order followed by the others in order into view, and
 * view_lens = (kept - 1) * block_size + tokens of the last block (0 for an empty row).
 * width <= 16384 (a row is staged in shared memory).
 */
int ekv_view_build(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                   const int32_t* row_blocks, const int32_t* quota, const int32_t* measured_blocks,
                   int recent_blocks, const float* scores, int64_t score_stride, int policy,
                   const uint8_t* keep, int64_t keep_stride, const uint8_t* full_rows,
                   const uint8_t* released, int64_t released_stride, int rows, int width,
                   int block_size, int32_t* view, int64_t view_stride, int32_t* view_lens,
                   uint8_t* mask_out, int64_t mask_stride, void* stream);

/*
 * ekv_view_build_fractions -- ekv_allocate_quotas with per-row budgets (row_fraction) followed by
 * ekv_view_build in ranking mode, in one kernel: each measured row (row_blocks[r] > cap_above_blocks
 * and > 0) is its own allocate() call with budget max(pins, ceil(row_fraction[r] * n)), n =
 * min(row_blocks[r], width); other rows read in full. Arguments as in those two calls.
 */
int ekv_view_build_fractions(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                             const int32_t* row_blocks, const double* row_fraction,
                             const int32_t* measured_blocks, int recent_blocks, int cap_above_blocks,
                             const float* scores, int64_t score_stride, int policy, const uint8_t* full_rows,
                             const uint8_t* released, int64_t released_stride, int rows, int width,
                             int block_size, int32_t* view, int64_t view_stride, int32_t* view_lens,
                             uint8_t* mask_out, int64_t mask_stride, void* stream);

/*
 * ekv_compact_block_table -- compact_block_table (runtime/block_view.py:36-56) on the device:
 * ekv_view_build in mask mode with no full rows and no released blocks.
 */
int ekv_compact_block_table(const int32_t* table, int64_t table_stride, const int32_t* seq_lens,
                            const uint8_t* keep, int64_t keep_stride, int rows, int width,
                            int block_size, int32_t* view, int64_t view_stride,
                            int32_t* view_lens, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* EKV_B200_H */
