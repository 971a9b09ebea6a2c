/*
 * hk.h — C ABI of the B200-native continuous-batching decode step.
 *
 * Plain pointers and sizes only: no CUDA, PyTorch or C++ types cross this boundary.
 * Device pointers are raw CUDA device addresses; `stream` is a cudaStream_t passed as
 * void* (NULL = the legacy default stream).  bf16 values travel as uint16_t bit patterns,
 * e4m3 values as uint8_t.
 *
 * Every function returns 0 on success or a negative HK_E* code; hk_last_error() then
 * gives a one-line message (thread-local).  Kernels that find bad input (an index past a
 * buffer, a page id past the pool) skip the access, set a device error word and the next
 * hk_check_errors() on that device reports it.  No entry point ever falls back to a CPU
 * path: without a usable sm_100 device they return HK_ENODEV.
 *
 * Empty problems: a kernel entry point with nothing to process (no tokens, rows or pages)
 * returns 0 without launching anything, and the arrays it would have read or written may
 * then be NULL (as a zero-element tensor's address is).  Arrays that still receive output
 * (hk_permute's offsets, hk_sample_verify's per-lane ids and states) stay required.
 *
 * Reference interfaces replaced (paths inside mr-d-self-driving/Hyperkernel):
 *   - the `Kernel` trait, src/gpu/mod.rs:42-46 (pools / push / drain) and its data types
 *     Share / Command / Event / Sampled, src/gpu/mod.rs:13-40  ->  hk_open ... hk_drain;
 *   - the device half of src/gpu/feed.rs:40-208 and the closed sm_103a megakernel
 *     (kernels/b300/c*, ring message `drafting`) -> the per-kernel entry points below.
 */
#ifndef HK_H
#define HK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HK_OK 0
#define HK_EINVAL -1   /* a bad argument: null pointer, size out of range, misaligned */
#define HK_ENODEV -2   /* no usable sm_100 device */
#define HK_ECUDA -3    /* a CUDA runtime / driver error */
#define HK_EDEVICE -4  /* a kernel set its device error word (bad index, bounded wait ran out) */
#define HK_ESPACE -5   /* a caller buffer or workspace too small */
#define HK_ESTATE -6   /* a call out of order (e.g. push past the granted horizon) */

/* ------------------------------------------------------------------------------------ */
/* Library                                                                               */
/* ------------------------------------------------------------------------------------ */

const char* hk_version(void);
/* Message of the last failed call on this thread ("" if none). */
const char* hk_last_error(void);
/* SM count and compute capability of the current device. */
int hk_device_info(int* sm_count, int* cc_major, int* cc_minor);
/* Number of CUDA kernels this library has launched in this process (all devices). */
uint64_t hk_kernel_launches(void);
/* Reads and clears the device error word of the current device: 0 when clean, else
 * HK_EDEVICE with the first recorded code/site in hk_last_error().  Synchronises. */
int hk_check_errors(void);

/* ------------------------------------------------------------------------------------ */
/* a7  pack: ragged lanes -> one token stream                                            */
/* Replaces the packing the closed megakernel does from the `drafting` ring message      */
/* (per-lane tokens[w*6], pos[w], pages[w*4097], slot[w]); block-table rows are those    */
/* Cache::pages emits, src/engine/cache.rs:195-226.                                      */
/* ------------------------------------------------------------------------------------ */

/* Inputs (device): lane_tokens[num_lanes] new rows this step (0 = idle lane, 1 = decode,
 * 1+d = spec verify, n = prompt chunk); lane_pos[num_lanes] position of the lane's first
 * new row; block_table[num_lanes][bt_stride] page ids (i32, 0 = scratch page).
 * Outputs (device): cu_seqlens[num_lanes+1] exclusive scan of lane_tokens;
 * seq_lens[num_lanes] = lane_pos + lane_tokens (KV rows after the append, 0 if idle);
 * positions[T], slot_mapping[T] = block_table[lane][pos / page_size] * page_size +
 * pos % page_size, token_lane[T]; active[0] = number of non-idle lanes, active[1..] their
 * lane ids in ascending order (entries after them are not written).  T = sum(lane_tokens) must be <= max_tokens, else the
 * rows past max_tokens are not written and the device error word is set.  A row whose
 * page is 0 (the scratch page) or past num_pages is written with slot -1 and flags the
 * error word.  Bit-exact: integer only. */
int hk_pack(const int32_t* lane_tokens, const int32_t* lane_pos, const int32_t* block_table,
            int32_t bt_stride, int32_t num_lanes, int32_t page_size, int32_t num_pages,
            int32_t max_tokens, int32_t* cu_seqlens, int32_t* seq_lens, int32_t* positions,
            int32_t* slot_mapping, int32_t* token_lane, int32_t* active, void* stream);

/* ------------------------------------------------------------------------------------ */
/* a8  KV append into the paged cache                                                    */
/* ------------------------------------------------------------------------------------ */

/* MLA latent rows: kv_new[T][row_elems] bf16 -> the cache row `slot` (row_elems = 576 =
 * 512 latent + 64 rope for the configs).
 * page_rows == 0: row-major cache, element (slot, e) at slot * row_elems + e (row_elems a
 * multiple of 8).
 * page_rows  > 0: the page-blocked latent cache that hk_mla_decode reads: pages of page_rows
 * rows, each page storing its rows in blocks of 64 elements, block-major, so that one block
 * of one page is a contiguous page_rows x 64 tile:
 *   element (slot, e) at (slot / page_rows) * page_rows * row_elems
 *                        + (e / 64) * page_rows * 64 + (slot % page_rows) * 64 + e % 64
 * (row_elems a multiple of 64). */
int hk_kv_append_bf16(const uint16_t* kv_new, const int32_t* slot_mapping, int32_t num_tokens,
                      int32_t row_elems, int32_t page_rows, uint16_t* kv_cache, int64_t num_slots,
                      void* stream);

/* MLA latent rows quantised to e4m3 with one fp32 scale per row:
 * scale = max(amax(row), 1e-12) / 448, q = e4m3_rn_satfinite(x / scale). */
int hk_kv_append_fp8(const uint16_t* kv_new, const int32_t* slot_mapping, int32_t num_tokens,
                     int32_t row_elems, uint8_t* kv_cache, float* kv_scale, int64_t num_slots,
                     void* stream);

/* The FP8 latent cache (row-major [num_slots][row_elems] e4m3 with one scale per row) as the
 * page-blocked bf16 cache hk_mla_decode reads: element (slot, e) = bf16(e4m3(q) * scale[slot])
 * at the blocked position of hk_kv_append_bf16.  num_slots a multiple of page_rows, row_elems a
 * multiple of 64.  `pages` (device, n_pages ids; NULL = every page) restricts the conversion to
 * the listed pages, written at their own positions.  Lets FP8-stored KV use the tcgen05 bf16
 * attention kernel. */
int hk_kv_dequant_fp8(const uint8_t* kv_fp8, const float* kv_scale, int64_t num_slots,
                      int32_t row_elems, int32_t page_rows, const int32_t* pages, int64_t n_pages,
                      uint16_t* kv_bf16, void* stream);
/* The same conversion for the listed cache rows only (device slots[n_rows], e.g. a step's
 * slot_mapping after hk_kv_append_fp8): keeps a bf16 mirror of an FP8 pool current at the
 * cost of the rows appended, instead of converting the pool every step. */
int hk_kv_dequant_fp8_rows(const uint8_t* kv_fp8, const float* kv_scale, int64_t num_slots,
                           int32_t row_elems, int32_t page_rows, const int32_t* slots,
                           int64_t n_rows, uint16_t* kv_bf16, void* stream);

/* GQA rows (config 1): k_new/v_new[T][kv_heads*head_dim] fp32 -> k_cache/v_cache[slot][..]. */
int hk_kv_append_f32(const float* k_new, const float* v_new, const int32_t* slot_mapping,
                     int32_t num_tokens, int32_t row_elems, float* k_cache, float* v_cache,
                     int64_t num_slots, void* stream);

/* ------------------------------------------------------------------------------------ */
/* a9/a10  ragged paged decode attention with split-KV partials and LSE merge           */
/* Query row t of lane b sits at positions[t] and attends KV rows 0..positions[t]       */
/* (causal inside a spec-verify block or a prompt chunk).                                */
/* ------------------------------------------------------------------------------------ */

/* GQA fp32 (config 1): q[T][q_heads][head_dim], caches [num_slots][kv_heads][head_dim].
 * out[T][q_heads][head_dim], lse[T][q_heads] (natural log, of scale*q.k). */
int hk_gqa_decode_f32(const float* q, const float* k_cache, const float* v_cache,
                      const int32_t* block_table, int32_t bt_stride, const int32_t* cu_seqlens,
                      const int32_t* positions, int32_t num_lanes, int32_t num_tokens,
                      int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t page_size,
                      int64_t num_slots, float scale, float* out, float* lse, void* stream);

/* MLA absorbed decode, bf16 (config 2): q[T][heads][576], kv_cache in the page-blocked
 * layout of hk_kv_append_bf16 with page_rows = page_size (576 = latent 512 then rope 64 per
 * row), out[T][heads][512] bf16, lse[T][heads] fp32.  Scores use all 576 dims,
 * values the first 512.  The work is split across SMs by KV range; partials of split
 * lanes go to `workspace` (size from hk_mla_workspace_size) and are merged by LSE.
 * impl: 0 = best available (tcgen05 when heads == 128 and pages hold 64 rows), 1 = portable
 * CUDA-core kernel, 2 = tcgen05 2-SM kernel.  The tcgen05 kernel reads whole pages: rows past
 * a lane's length in its last page, and the scratch page 0, must hold finite values (a
 * zero-filled pool satisfies this); they get zero weight but pass through the tensor core. */
size_t hk_mla_workspace_size(int32_t num_lanes, int32_t num_tokens, int32_t heads,
                             int32_t max_kv_len);
int hk_mla_decode(const uint16_t* q, const uint16_t* kv_cache, const int32_t* block_table,
                  int32_t bt_stride, const int32_t* cu_seqlens, const int32_t* positions,
                  int32_t num_lanes, int32_t num_tokens, int32_t heads, int32_t page_size,
                  int64_t num_slots, int32_t max_kv_len, float scale, uint16_t* out, float* lse,
                  void* workspace, size_t workspace_bytes, int32_t impl, void* stream);

/* MLA decode over an e4m3 latent cache with per-row fp32 scales (config 5). */
int hk_mla_decode_fp8(const uint16_t* q, const uint8_t* kv_cache, const float* kv_scale,
                      const int32_t* block_table, int32_t bt_stride, const int32_t* cu_seqlens,
                      const int32_t* positions, int32_t num_lanes, int32_t num_tokens,
                      int32_t heads, int32_t page_size, int64_t num_slots, int32_t max_kv_len,
                      float scale, uint16_t* out, float* lse, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Partial attention of a KV shard, for context parallelism: the same contract as
 * hk_mla_decode_fp8 restricted to KV rows [kv_begin[b], kv_end[b]) of each lane, writing
 * fp32 o_part[T][heads][512] (normalised within the shard) and lse_part[T][heads] (-inf
 * where the shard holds no row).  max_kv_len bounds kv_end - kv_begin; the workspace size
 * is hk_mla_workspace_size(num_lanes, num_tokens, heads, max_kv_len). */
int hk_mla_partial_fp8(const uint16_t* q, const uint8_t* kv_cache, const float* kv_scale,
                       const int32_t* block_table, int32_t bt_stride, const int32_t* cu_seqlens,
                       const int32_t* positions, const int32_t* kv_begin, const int32_t* kv_end,
                       int32_t num_lanes, int32_t num_tokens, int32_t heads, int32_t page_size,
                       int64_t num_slots, int32_t max_kv_len, float scale, float* o_part,
                       float* lse_part, void* workspace, size_t workspace_bytes, void* stream);

/* The same partial on the tcgen05 kernel, over the page-blocked bf16 cache of hk_mla_decode
 * (128 heads, pages of 64 rows; an FP8 pool goes through hk_kv_dequant_fp8 first, restricted
 * to the shard's pages).  kv_begin need not be page-aligned.  Workspace:
 * hk_mla_workspace_size. */
int hk_mla_partial(const uint16_t* q, const uint16_t* kv_cache, const int32_t* block_table,
                   int32_t bt_stride, const int32_t* cu_seqlens, const int32_t* positions,
                   const int32_t* kv_begin, const int32_t* kv_end, int32_t num_lanes,
                   int32_t num_tokens, int32_t heads, int32_t page_size, int64_t num_slots,
                   int32_t max_kv_len, float scale, float* o_part, float* lse_part,
                   void* workspace, size_t workspace_bytes, void* stream);

/* a10  LSE merge of n_parts partials: o_parts[n][rows][dv] fp32, lse_parts[n][rows]
 * -> out[rows][dv] bf16 and lse_out[rows]:  m = max lse_i,
 * out = sum_i e^(lse_i - m) o_i / sum_i e^(lse_i - m),  lse = m + log(sum e^(lse_i - m)). */
int hk_lse_merge(const float* o_parts, const float* lse_parts, int32_t n_parts, int64_t rows,
                 int32_t dv, uint16_t* out, float* lse_out, void* stream);

/* ------------------------------------------------------------------------------------ */
/* a11  FP8 block-scaled linear                                                          */
/* ------------------------------------------------------------------------------------ */

/* Quantise bf16 activations x[rows][k] to e4m3 in 1x128 blocks:
 * sx[rows][k/128] = max(amax, 1e-12)/448, xq = e4m3_rn_satfinite(x / sx).  k % 128 == 0. */
int hk_quant_fp8(const uint16_t* x, int64_t rows, int32_t k, uint8_t* xq, float* sx,
                 void* stream);

/* y[m][n] bf16 = sum over 128-blocks kb of (xq[m][kb] . wq[n][kb]) * sx[m][kb] * sw[n/128][kb]
 * with wq[n][k] e4m3 and sw[ceil(n/128)][k/128] fp32; fp32 accumulation.
 * k % 128 == 0, n % 16 == 0.  Tensor-core kernels: m >= 256 SM pairs, 128 <= m < 256 one SM,
 * m < 128 swap-AB (the weights on the MMA's M side); a long-K, small-n shape with m < 128 splits
 * K and takes its fp32 partials from a stream-ordered memory pool the library keeps per device. */
int hk_gemm_fp8(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                int64_t m, int32_t n, int32_t k, uint16_t* y, void* stream);

/* ------------------------------------------------------------------------------------ */
/* a12-a15  MoE: router, permutation, grouped FP8 GEMM, combine                          */
/* ------------------------------------------------------------------------------------ */

/* Sigmoid router: s = sigmoid(logits[t][e]); the top_k experts by s + bias[e] (ties: the
 * lower expert id first); weights = s[chosen] / sum s[chosen] * route_scale.
 * ids[t][top_k] i32 in descending order of s + bias, weights[t][top_k] fp32.
 * num_experts <= 256, top_k <= 16. */
int hk_route(const float* logits, const float* bias, int32_t tokens, int32_t num_experts,
             int32_t top_k, float route_scale, int32_t* ids, float* weights, void* stream);

/* Stable permutation of the (token, k) pairs into per-expert groups, ordered by
 * (expert, token, k): offsets[num_experts+1] exclusive scan of the per-expert counts;
 * perm_token[P] source token of permuted row p; perm_weight[P]; inv[t*top_k+k] = the
 * permuted row of pair (t, k).  P = tokens*top_k.  Bit-exact. */
int hk_permute(const int32_t* ids, const float* weights, int32_t tokens, int32_t top_k,
               int32_t num_experts, int32_t* offsets, int32_t* perm_token, float* perm_weight,
               int32_t* inv, void* stream);

/* Grouped expert FFN.  Rows of expert e are permuted rows offsets[e]..offsets[e+1] (at most
 * `rows` in all, offsets[num_experts] <= rows); their inputs are xq[perm_token[p]] (e4m3,
 * 1x128 scales sx, `tokens` rows).  Per expert:
 * h = silu(x Wg^T) * (x Wu^T) (Wg, Wu = halves of w13[e][2*inter][hidden]),
 * y[p] = h Wd^T (w2[e][hidden][inter]), all weights e4m3 with 128x128 fp32 block scales
 * (s13[e][2*inter/128][hidden/128], s2[e][hidden/128][inter/128]); h is re-quantised to
 * e4m3 1x128 blocks before the down projection.  y[P][hidden] bf16.
 * On sm_100 the expert GEMMs run on the tensor cores (weights on the MMA's M side, a tile of
 * an expert's routed rows on N: 16, 32, 64 or 96 rows, picked from the rows per expert on
 * average — below 8, 8-23, 24-55, 56 and up, the last only with `tokens` > 64; a row's result
 * does not depend on the tile width).  A shared expert can run in the same call as one more
 * expert whose rows map to every token.
 * `workspace` (256-byte aligned, hk_moe_workspace_size bytes) holds h, its scales, the tile
 * lists and the routed rows gathered in permuted order. */
size_t hk_moe_workspace_size(int64_t rows, int32_t hidden, int32_t inter);
int hk_moe_grouped(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                   const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden,
                   int32_t inter, const uint8_t* w13, const float* s13, const uint8_t* w2,
                   const float* s2, uint16_t* y, void* workspace, size_t workspace_bytes,
                   void* stream);

/* hk_moe_grouped without a workspace argument, for callers that cannot allocate device memory
 * (an engine reaching this library only through the C ABI with no CUDA allocator of its own, a
 * pool allocator that forbids raw cudaMalloc, a step loop that must not take cudaMalloc's
 * device-wide synchronisation).  No counterpart in the reference.  Its scratch is a fixed
 * 2,167,040-byte device array that every GPU loading this library holds until exit: at most
 * 1024 permuted rows and inter <= 2048, larger problems are refused with HK_EINVAL.  It
 * allocates nothing and runs the CUDA-core expert kernels (the scratch has no room for the
 * gathered rows the tensor-core kernels read).  All calls share the array: calls that overlap on the GPU race and must
 * be serialised.  The first call on a device looks the array up (cudaGetSymbolAddress) and
 * should come before any stream capture.  Out-of-range rows are skipped but not recorded in
 * the device error word; offsets that are not a valid scan (offsets[0] != 0, decreasing, or
 * offsets[num_experts] > rows) leave y entirely unwritten and are not reported either. */
int hk_moe_grouped_noalloc(const uint8_t* xq, const float* sx, int32_t tokens,
                           const int32_t* offsets, const int32_t* perm_token, int64_t rows,
                           int32_t num_experts, int32_t hidden, int32_t inter,
                           const uint8_t* w13, const float* s13, const uint8_t* w2,
                           const float* s2, uint16_t* y, void* stream);

/* Row movement around the expert-parallel all-to-all (dispatch gathers the routed rows of
 * each destination's experts, combine scatters returning rows back into permuted order):
 * gather dst[i] = src[idx[i]] for i < rows (idx < src_rows); scatter dst[idx[i]] = src[i]
 * (idx < dst_rows).  Rows of row_bytes bytes (a multiple of 4, 4-byte aligned buffers).
 * An out-of-range index skips its row and sets the device error word. */
int hk_gather_rows(const void* src, int64_t src_rows, const int32_t* idx, int64_t rows,
                   int32_t row_bytes, void* dst, void* stream);
int hk_scatter_rows(const void* src, int64_t rows, const int32_t* idx, int64_t dst_rows,
                    int32_t row_bytes, void* dst, void* stream);

/* Expert-parallel exchange over NVLink peer memory (no NCCL on the data path).  Rank r of
 * `world` (<= 8) owns experts [r E/world, (r+1) E/world).  Buffer arguments named by rank are
 * host arrays of `world` device addresses, element i = rank i's copy of a symmetric buffer
 * mapped into this process: counts [world][E] int32, flags [3][8] uint32 (zero before the first step),
 * recv_x [rows_cap][hidden] e4m3, recv_s [rows_cap][hidden/128] fp32, back_y [back_cap][hidden]
 * bf16.  `epoch` is a nonzero step counter the caller increments every step; every wait is
 * bounded by timeout_us and a timeout sets the device error word.
 *   hk_ep_counts: exchanges per-expert row counts and computes send_base[E] (where this rank's
 *     rows of expert e start in the owner's receive buffer, expert-major, sources in rank
 *     order), local_off[E/world + 1] (the receive buffer's expert offsets) and
 *     ret_base[world][E/world] (where source s's rows of a local expert sit in s's order).
 *   hk_ep_dispatch: copies routed row p (xq[perm_token[p]] and its scales) straight into its
 *     owner's receive buffer; raises the dispatch flag on every rank when done.
 *   hk_ep_return: copies received row j of y (expert-major, local_off order) back into its
 *     source's back_y at its permuted position; raises the return flag on every rank.  y holds
 *     rows_bound rows: a received total above that (counts a peer wrote for another
 *     configuration) moves no row, sets the device error word and raises no flag.
 *   After a count exchange that timed out, dispatch and return move no row and raise no flag
 *   (the step's plan is marked invalid), so every rank's next wait runs out and reports it.
 *   hk_ep_wait: waits until every rank raised flag set `which` (0 counts, 1 dispatch, 2 return)
 *     in this rank's flags with the epoch.
 * done_ctr: one zeroed device word per launch kind, private to this rank. */
int hk_ep_counts(const int32_t* offsets, int32_t num_experts, int32_t world, int32_t rank,
                 const uint64_t* counts, const uint64_t* flags, uint32_t epoch, int32_t timeout_us,
                 int32_t* send_base, int32_t* local_off, int32_t* ret_base, void* stream);
int hk_ep_dispatch(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* perm_token,
                   const int32_t* offsets, int32_t rows, int32_t num_experts, int32_t world,
                   int32_t rank, int32_t hidden, int32_t rows_cap, const int32_t* send_base,
                   const uint64_t* recv_x, const uint64_t* recv_s, const uint64_t* flags,
                   uint32_t* done_ctr, uint32_t epoch, void* stream);
int hk_ep_return(const uint16_t* y, int32_t num_experts, int32_t world, int32_t rank,
                 int32_t hidden, const int32_t* local_off, const int32_t* counts,
                 const int32_t* ret_base, int32_t back_cap, int32_t rows_bound,
                 const uint64_t* back_y, const uint64_t* flags, uint32_t* done_ctr,
                 uint32_t epoch, void* stream);
int hk_ep_wait(const uint32_t* flags, int32_t which, int32_t world, uint32_t epoch,
               int32_t timeout_us, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Buffers shared across the GPUs of one node, and the context-parallel merge            */
/* The reference maps its ranks' buffers through VMM handles passed over its rank fabric  */
/* (src/gpu/ranks.rs:198-244, fabric_map); here a buffer travels as a CUDA IPC handle.   */
/* ------------------------------------------------------------------------------------ */

/* The bytes of a CUDA IPC memory handle: plain data the host may send to other processes. */
typedef struct {
    uint8_t bytes[64];
} hk_ipc_handle;

/* Allocates `bytes` of zeroed device memory on the current device and its IPC handle. */
int hk_sym_alloc(size_t bytes, void** ptr, hk_ipc_handle* handle);
/* Maps another process's hk_sym_alloc buffer (its handle) into this process on the current
 * device, peer access enabled; *ptr is the address this process's kernels use for it. */
int hk_sym_import(const hk_ipc_handle* handle, void** ptr);
/* Unmaps an imported buffer; frees an hk_sym_alloc buffer (after every importer closed it). */
int hk_sym_close(void* peer_ptr);
int hk_sym_free(void* ptr);

/* Context-parallel exchange fused with the LSE merge: o_parts / lse_parts / flags are host
 * arrays of `world` device addresses (rank i's copy of each symmetric buffer, mapped into this
 * process): o [rows][dv] fp32 and lse [rows] partials of the same query rows (hk_mla_partial
 * writes them), flags [8] uint32 (zero before the first step).  The kernel raises this rank's
 * epoch flag on every rank, waits until every rank's flag carries `epoch` (bounded by timeout_us;
 * a timeout sets the device error word and skips the merge), then reads every rank's partial
 * over NVLink and writes out [rows][dv] bf16 = sum_i e^(lse_i - m) o_i / sum_i e^(lse_i - m),
 * lse_out [rows] = m + log(sum_i e^(lse_i - m)), m = max lse_i.  A rank may write its next
 * partial only into a second set of buffers (alternate sets by epoch parity): a peer may still
 * be reading this epoch's set. */
int hk_cp_merge(const uint64_t* o_parts, const uint64_t* lse_parts, const uint64_t* flags, int32_t world,
                int32_t rank, uint32_t epoch, int32_t timeout_us, int64_t rows, int32_t dv, uint16_t* out,
                float* lse_out, void* stream);

/* out[t][hidden] bf16 = sum_k perm_weight[inv[t,k]] * y[inv[t,k]] (+ shared[t] when not
 * NULL), fp32 accumulation in k order; y has `rows` rows. */
int hk_combine(const uint16_t* y, int64_t rows, const float* perm_weight, const int32_t* inv,
               const uint16_t* shared, int32_t tokens, int32_t top_k, int32_t hidden,
               uint16_t* out, void* stream);

/* Sampling, src/engine/request.rs:31-37 (declared here for hk_sample_verify; the kernel
 * boundary below carries it in hk_command). */
typedef struct {
    float temperature;
    float top_p;
    uint32_t top_k;
    uint32_t logprobs;
    uint64_t seed;
} hk_sampling;

/* Spec-decode verification with on-device sampling (the reply side of the step,
 * src/gpu/feed.rs:163-208).  Lane b's logits rows are cu_rows[b] .. cu_rows[b+1]-1 of
 * logits[num_rows][vocab] (fp32; 1 + drafts rows, at most `block`).  Row j is drawn with
 * sampling[b] (device array) and the lane's generator state[b] (device, advanced once per
 * sampled draw; start it at the request's seed), and the chain continues to row j + 1 only
 * while the token equals drafts[b][j] (drafts [num_lanes][block - 1]).  The draw restates the
 * reference's source sampler (src/evo2/draw.rs:14-58): greedy (first greatest logit) when
 * temperature <= 0 or top_k == 1, else top-k, softmax at the temperature in f64, top-p tail
 * cut, u = splitmix64(state) / 2^53 * kept.  ids [num_lanes][block]: the accepted tokens then
 * -2; a row with a non-finite logit gives -1 and ends the lane.  lp [num_lanes][block]
 * [2 n_logprobs + 1] (may be NULL when n_logprobs = 0): per token, the n_logprobs best
 * (id, logprob) pairs of the row's log-softmax (id -1 past the vocabulary), then the token's
 * own logprob.  vocab <= 4,194,304; 1 <= block <= 32; n_logprobs <= 64; workspace 256-byte
 * aligned, hk_sample_workspace_size bytes. */
size_t hk_sample_workspace_size(int32_t num_rows, int32_t vocab);
int hk_sample_verify(const float* logits, int32_t vocab, const int32_t* cu_rows, int32_t num_lanes,
                     int32_t num_rows, int32_t block, const hk_sampling* sampling, uint64_t* state,
                     const int32_t* drafts, int32_t n_logprobs, int32_t* ids, float* lp,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------ */
/* Kernel boundary: the reference's `Kernel` trait (src/gpu/mod.rs:42-46)                */
/*   pools() -> hk_pools, push(&Share) -> hk_push, drain() -> hk_drain                   */
/* Types mirror Share / Command / Event / Sampled (src/gpu/mod.rs:13-40) as flat arrays.  */
/* ------------------------------------------------------------------------------------ */

typedef struct hk_handle hk_handle;

#define HK_CMD_END 0    /* End { lane } */
#define HK_CMD_PAGES 1  /* Pages { lane, from, upto, row } */
#define HK_CMD_SEAT 2   /* Seat { lane, pos, back, sampling } */
#define HK_CMD_PROMPT 3 /* Prompt { lane, tokens } */
#define HK_CMD_START 4  /* Start { lane } */

/* One Command.  Pages: pos = from, upto, count = row length, arena = offset (in words) of
 * the i32 row in hk_share.arena.  Seat: pos, back, sampling.  Prompt: count tokens (u32 bit
 * patterns) at arena.  Unused fields are ignored. */
typedef struct {
    uint32_t kind;
    uint32_t lane;
    uint32_t pos;
    uint32_t upto;
    uint32_t count;
    uint32_t arena;
    int32_t back[3];
    uint32_t reserved;
    hk_sampling sampling;
} hk_command;

/* Share { at, horizon, commands }: the commands take effect at step `at`; the device may run
 * steps up to `horizon`. */
typedef struct {
    uint32_t at;
    uint32_t horizon;
    const hk_command* commands;
    size_t n_commands;
    const int32_t* arena;
    size_t arena_words;
} hk_share;

#define HK_EV_IDLE 0     /* Idle { step } */
#define HK_EV_STEP 1     /* Step { step, lanes } */
#define HK_EV_PROMPTED 2 /* Prompted { lane, token, clipped } */

/* One Event.  Step: `ids` is the offset in the drain's id array of width * block sampled ids,
 * lane-major; a lane's list ends at its first -2 (lanes that did not decode start with -2).
 * Prompted: `token` (negative = the logits were not finite) and `clipped`.  Each Sampled's
 * logprob list comes from hk_drain_logprobs. */
typedef struct {
    uint32_t kind;
    uint32_t step;
    uint32_t lane;
    int32_t token;
    int32_t clipped;
    uint32_t ids;
} hk_event;

/* The device model behind a handle.  HK_MODEL_FNV is the reference's test model
 * (tests/engine.rs:56-62): the next token of a sequence is an FNV-style fold of its tokens,
 * which the device reads back through the lane's block-table row from the paged token pool,
 * checking that every position was written and that the window pages mirror the pages; a
 * violation fails the next hk_drain.  A decode step emits 1 + ((step + lane) mod block)
 * tokens per lane, the draft acceptance rule of the reference's test device, capped at the
 * lane's reserved rows. */
#define HK_MODEL_FNV 1
/* HK_MODEL_MLA is a DeepSeek-shaped decoder (opened with hk_open_mla): the decode step of the
 * reference's LLM bundles, rebuilt from this library's kernels (see hk_mla_model). */
#define HK_MODEL_MLA 2

typedef struct {
    uint32_t model;          /* HK_MODEL_FNV */
    uint32_t page_rows;      /* Pool.page_rows: token rows per page */
    uint32_t entries;        /* Pool.entries: page entries of a block-table row */
    uint32_t window;         /* Pool.window: window-page entries of a row */
    uint32_t width;          /* lanes (Model.batches.last) */
    uint32_t context;        /* Model.context */
    uint32_t chunk;          /* Model.chunks[0]: most tokens of one Prompt */
    uint32_t block;          /* Model.block: 1 + draft positions */
    uint64_t pages;          /* page pool size, unit 0 = scratch (returned by hk_pools) */
    uint64_t window_pages;   /* window page pool size, unit 0 = scratch */
    int32_t clip;            /* the `clipped` flag the test model returns with prompt replies */
    int32_t device;          /* CUDA device ordinal */
    uint32_t transport;      /* HK_TRANSPORT_LAUNCH or HK_TRANSPORT_RING */
    uint32_t reserved;
} hk_config;

/* How hk_drain drives the device.  LAUNCH: one kernel launch per applied batch and per step,
 * each followed by a synchronous read-back.  RING: a resident executor kernel (one CTA)
 * polls a mailbox in pinned, device-mapped host memory (the reference's device-polled
 * request ring, src/gpu/ring.rs, src/gpu/feed.rs:104-155): the host posts each batch's
 * encoded bytes or a step and waits for the executor's answer, which it writes, with the
 * step's ids and prompt replies, into mapped host memory.  The executor exits after 50 ms
 * without work (every poll is bounded) and is relaunched by the next post; hk_close stops
 * it.  Both transports produce the same events.  An executor that gives no answer within 30 s
 * fails that call with HK_EDEVICE and leaves the handle failed: every later hk_push / hk_drain
 * returns HK_EDEVICE with the same message, and hk_close first waits for the executor to
 * finish the abandoned item and exit (each item and each idle poll is bounded). */
#define HK_TRANSPORT_LAUNCH 0
#define HK_TRANSPORT_RING 1

/* Opens a device kernel: allocates the pools, the block-table rows and the lane state on
 * `device` and returns its handle.  One handle per process and GPU; a handle's calls are
 * not thread-safe.  config->model must be HK_MODEL_FNV (HK_MODEL_MLA opens with hk_open_mla). */
int hk_open(const hk_config* config, hk_handle** handle);

/* The decoder behind HK_MODEL_MLA: `layers` layers of MLA attention (128 heads, a latent of 512
 * plus 64 RoPE dims per token, absorbed projections) and an MoE FFN (`experts` routed experts,
 * top_k sigmoid routing, one shared expert), between a bf16 token embedding and an FP8 vocabulary
 * projection.  Every projection is e4m3 with 128x128 fp32 block scales (hk_gemm_fp8 /
 * hk_moe_grouped); activations are bf16, quantised to e4m3 in 1x128 blocks before each
 * projection.  One decode step of a packed batch (rows of every live lane, or the rows of the
 * prompt chunks being applied):
 *   x = embed[token]
 *   per layer:  a = rmsnorm(x);  q = (rmsnorm(a Wqa)) Wqb;  kv = a Wkva
 *               q.rope and kv.rope rotated by the row's position, kv.latent rmsnorm-ed;
 *               kv appended at the row's slot (hk_kv_append_bf16, page-blocked, pages of 64 rows);
 *               o = MLA attention over the lane's pages (hk_mla_decode);  x += o Wo;
 *               h = rmsnorm(x);  x += combine(top_k experts of sigmoid(h Wr)) + shared(h)
 *   logits = rmsnorm(x) Wvocab for the rows that are sampled; then hk_sample_verify.
 * RMS norms carry no gain (eps 1e-6); RoPE rotates dim i with dim i + 32 of the 64 rope dims by
 * position * rope_theta^(-i/32); attention scale 1/sqrt(576).  Weights are seeded random values
 * (N(0, sigma) quantised, sigma = 1/sqrt(fan-in)); hk_model_tensor gives their device addresses
 * so a loader can overwrite them.
 * Decode steps verify `block` rows per lane: the lane's last token and block - 1 drafts found
 * by prompt lookup (the tokens that followed the latest earlier occurrence of the last token in
 * the lane's last 4096 positions; -1 where there is none).  A share's prompt chunks of
 * distinct lanes are prefilled together, up to max(chunk, min(16 * chunk, 8192)) rows a forward
 * pass (the share's commands for other lanes are applied before the pass, a command for one of
 * its lanes after it), and each is answered, in push order, with a token sampled from the
 * chunk's last row.  Each sampled token carries `logprobs` (id, logprob) pairs then its own
 * logprob. */
typedef struct {
    uint32_t hidden;      /* model width, a multiple of 128 */
    uint32_t q_lora;      /* query low-rank width, a multiple of 128 */
    uint32_t vocab;       /* vocabulary, a multiple of 16, <= 4,194,304 */
    uint32_t experts;     /* routed experts, a multiple of 16, <= 256 */
    uint32_t top_k;       /* experts per token, <= 16 */
    uint32_t inter;       /* expert intermediate width, a multiple of 128 */
    uint32_t layers;      /* decoder layers, >= 1 */
    uint32_t logprobs;    /* (id, logprob) pairs returned with every sampled token, <= 64 */
    uint64_t seed;        /* weight seed */
    float rope_theta;     /* RoPE base (0 = 10000) */
    float route_scale;    /* routed weights' scale (0 = 1) */
} hk_mla_model;

/* Opens a device kernel running HK_MODEL_MLA (config->model == HK_MODEL_MLA, page_rows == 64,
 * transport HK_TRANSPORT_LAUNCH): allocates the pools as hk_open does, plus the weights, a
 * page-blocked bf16 latent cache of config->pages pages per layer and the step's buffers (sized
 * for the larger of a decode step's width * block rows and a prefill pass's rows). */
int hk_open_mla(const hk_config* config, const hk_mla_model* model, hk_handle** handle);

/* Device address and size of one of an HK_MODEL_MLA handle's tensors: `name` is one of "embed"
 * (bf16 [vocab][hidden]), "vocab" / "vocab.scale" (e4m3 [vocab][hidden], fp32 [vocab/128][hidden/
 * 128]), per layer `layer`: "wqa", "wqb", "wkva", "wo", "router" (e4m3 [n][k]) and their ".scale"
 * (fp32 [ceil(n/128)][k/128]), "w13", "w2" (e4m3 [experts + 1][..], the shared expert last) and
 * their ".scale", "kv" (the layer's latent cache, bf16, page-blocked); "tokens" (the token pool,
 * int32 [pages][page_rows], -1 = unwritten).  Shapes: wqa [q_lora][hidden], wqb [128*576][q_lora],
 * wkva [576][hidden], wo [hidden][128*512], router [experts][hidden], w13 [experts+1][2*inter]
 * [hidden], w2 [experts+1][hidden][inter]. */
int hk_model_tensor(hk_handle* handle, uint32_t layer, const char* name, void** ptr, size_t* bytes);
void hk_close(hk_handle* handle);
/* Kernel::pools: (pages, window_pages). */
int hk_pools(const hk_handle* handle, size_t* pages, size_t* window_pages);
/* Pool sizing: how many pages (and window pages) a GPU's free memory holds for a bundle's
 * pools.  Each pool state costs `bytes` per unit of its kind (a page of `page_rows` token rows,
 * or a window page); the window pages are taken whole, the rest of the bytes go to pages, at
 * most the bundle's `pages`, and the result must hold more than one sequence's row of
 * `entries` pages.  Replaces pages_within (src/gpu/load.rs:903-908). */
#define HK_UNIT_PAGE 0
#define HK_UNIT_WINDOW 1

typedef struct {
    uint32_t home;           /* PoolState.home: the device buffer the state lives in */
    uint32_t unit;           /* HK_UNIT_PAGE or HK_UNIT_WINDOW */
    uint64_t bytes;          /* bytes of this state per unit */
} hk_pool_state;

typedef struct {
    uint64_t pages;          /* Pool.pages: the bundle's most pages */
    uint64_t window_pages;   /* Pool.window_pages */
    uint64_t entries;        /* Pool.entries: page entries of one row */
    uint64_t slots;          /* Pool.slots: lane slots (lanes + 1 scratch) */
    const hk_pool_state* states;
    size_t n_states;
} hk_pool_sizing;

/* pages_within: HK_ESPACE (and no outputs) when the bytes do not cover the window pages or
 * hold no more than `entries` pages; HK_EINVAL for a null argument or an overflowing cost. */
int hk_pages_within(const hk_pool_sizing* pool, uint64_t bytes, size_t* pages, size_t* window_pages);

typedef struct {
    uint64_t free;           /* device bytes free; 0 = read cudaMemGetInfo on `device` */
    uint64_t other;          /* the kernel's other device bytes (weights, workspace, staging) */
    uint64_t slack;          /* bytes left unused */
    uint32_t lanes;          /* the widest decode batch */
    uint32_t context;        /* Model.context (for the error message) */
    int32_t device;          /* CUDA device ordinal, read when free == 0 */
    uint32_t reserved;
} hk_pool_budget;

/* The pool part of the loader's plan (src/gpu/load.rs:510-533): pools get free - other -
 * slack bytes, sized by hk_pages_within; the lanes need lanes + 1 <= slots.  Outputs the
 * pages, window pages, slots and the bytes the pools use (sum over states of bytes x units).
 * Errors carry the reference's wording in hk_last_error(): HK_ESPACE for memory, HK_EINVAL
 * for lanes past the slots. */
int hk_plan_pools(const hk_pool_sizing* pool, const hk_pool_budget* budget, size_t* pages,
                  size_t* window_pages, size_t* slots, uint64_t* used);

/* Kernel::push: copies the share (the caller keeps ownership of its arrays).  share->at must
 * be the previous horizon + 1 (HK_ESTATE otherwise) and horizon >= at (HK_EINVAL). */
int hk_push(hk_handle* handle, const hk_share* share);
/* Kernel::drain: applies the commands due, runs the granted steps and returns the events
 * (Prompted replies in push order).  *n / *ids_n receive the counts; when `cap` or `ids_cap`
 * is too small it returns HK_ESPACE with the sizes needed and keeps the events for the next
 * call.  A device-side violation returns HK_EDEVICE with the first one's message. */
int hk_drain(hk_handle* handle, hk_event* events, size_t cap, size_t* n, int32_t* ids,
             size_t ids_cap, size_t* ids_n);

/* One (token id, logprob) pair of a Sampled's logprob list (src/gpu/mod.rs:37-40). */
typedef struct {
    uint32_t id;
    float logprob;
} hk_logprob;

/* The logprob lists of the Sampled values of the events the last successful hk_drain
 * returned, in event order: width * block lists per Step event (one per id slot; slots past
 * a lane's list have none) and one per Prompted event.  List i has counts[i] pairs, stored
 * one list after another in `pairs` (the reply's top pairs, then the token's own, as
 * src/gpu/feed.rs:202-208 reads them).  HK_ESPACE with *n_counts / *n_pairs set when a
 * buffer is short.  The device kernel's test model samples no logprobs: its lists are
 * empty. */
int hk_drain_logprobs(hk_handle* handle, uint32_t* counts, size_t counts_cap, size_t* n_counts,
                      hk_logprob* pairs, size_t pairs_cap, size_t* n_pairs);

/* The request-ring encoding of a share (src/gpu/feed.rs:40-103, src/gpu/ring.rs:59-125):
 * one slot per command (u32 message id at byte 0, the message body at byte 16, slot size
 * 16 + widest body rounded up to 16 bytes) followed by the side blocks the messages' spans
 * point at (Pages rows, Prompt tokens padded to `chunk` words).  Span addresses are byte
 * offsets from the start of `out`.  hk_push sends exactly these bytes to the device.
 * Host-only. */
int hk_encode_share(const hk_config* config, const hk_share* share, uint8_t* out, size_t cap,
                    size_t* bytes);

/* ------------------------------------------------------------------------------------ */
/* Engine: engine::run and its job channel (src/engine/mod.rs:38-359)                     */
/* ------------------------------------------------------------------------------------ */

typedef struct hk_engine hk_engine;

/* A Kernel implementation as callbacks (what hk_engine_run drives).  drain's contract is
 * hk_drain's, HK_ESPACE included; `error` returns the message after a failed call. */
typedef struct {
    void* self;
    int (*pools)(void* self, size_t* pages, size_t* window_pages);
    int (*push)(void* self, const hk_share* share);
    int (*drain)(void* self, hk_event* events, size_t cap, size_t* n, int32_t* ids,
                 size_t ids_cap, size_t* ids_n);
    const char* (*error)(void* self);
    /* Optional (NULL: every Sampled has an empty logprob list): hk_drain_logprobs's contract,
     * called after each successful drain. */
    int (*logprobs)(void* self, uint32_t* counts, size_t counts_cap, size_t* n_counts,
                    hk_logprob* pairs, size_t pairs_cap, size_t* n_pairs);
} hk_kernel_ops;

/* Fills `ops` with the callbacks of a device handle. */
int hk_kernel_ops_of(hk_handle* handle, hk_kernel_ops* ops);

#define HK_UNBOUNDED UINT64_MAX

/* Pool (src/bundle.rs), Model, Plan (src/engine/pacing.rs:1-13) and EngineConfig
 * (src/engine/mod.rs:25-36) fields the engine reads. */
typedef struct {
    uint32_t page_rows, entries, window, window_keep;
    uint32_t context, width, chunk, block;
    int32_t pad;
    uint32_t lead;
    uint64_t budget;   /* Plan.budget, HK_UNBOUNDED = None */
    uint64_t every, headroom;
    uint64_t gap, ahead, max_draft_positions;
} hk_engine_config;

/* Plan::default() and EngineConfig::default() (budget None, every 1, headroom 2048; gap 16,
 * lead 2, ahead 16, max_draft_positions 16); the pool and model fields are zeroed. */
void hk_engine_defaults(hk_engine_config* config);

/* The engine over a kernel.  The job calls below may come from any thread; hk_engine_run
 * from one.  Fails with HK_EINVAL when block - 1 > max_draft_positions (run's check). */
int hk_engine_create(const hk_engine_config* config, const hk_kernel_ops* kernel,
                     hk_engine** engine);
void hk_engine_destroy(hk_engine* engine);

/* Job::Run(Request { prompt, sampling, limit, stop, out }): queues a request; *request
 * names its output channel.  limit = HK_UNBOUNDED for no limit. */
int hk_engine_submit(hk_engine* engine, const uint32_t* prompt, size_t n, const hk_sampling* s,
                     uint64_t limit, const uint32_t* stop, size_t n_stop, uint64_t* request);
/* Job::Reset: queues a prefix-cache reset; hk_engine_reset_answer waits up to timeout_ms
 * (negative = forever) for the number of pages it freed (HK_ESTATE on timeout). */
int hk_engine_reset(hk_engine* engine, uint64_t* ticket);
int hk_engine_reset_answer(hk_engine* engine, uint64_t ticket, int64_t timeout_ms,
                           uint64_t* freed);
/* Drops the job sender: hk_engine_run returns once the engine is idle. */
int hk_engine_close(hk_engine* engine);
/* engine::run: 0 when the jobs closed and every request ended, else the kernel's error code
 * (message in hk_last_error) after every held, waiting and queued request was refused. */
int hk_engine_run(hk_engine* engine);
/* The request's listener went away: its next token send fails and ends it (End::Stop). */
int hk_engine_hangup(hk_engine* engine, uint64_t request);

#define HK_OUT_SEATED 0 /* value = cached tokens */
#define HK_OUT_TOKEN 1  /* value = token id, end = the number of its logprob pairs */
#define HK_OUT_END 2    /* end = HK_END_* */
#define HK_END_STOP 0
#define HK_END_LENGTH 1
#define HK_END_REFUSED 2

typedef struct {
    uint32_t kind;
    uint32_t end;
    int64_t value;
} hk_out;

/* Takes up to `cap` of the request's outputs (Out::Seated / Token / End) in order, waiting
 * up to timeout_ms (negative = forever, 0 = no wait) for the first.  The message of a
 * Refused end is copied into `message` (NUL-terminated, truncated to message_cap). */
int hk_engine_outputs(hk_engine* engine, uint64_t request, int64_t timeout_ms, hk_out* out,
                      size_t cap, size_t* n, char* message, size_t message_cap);
/* hk_engine_outputs with each token's logprobs (Token.logprobs: the token's own pair, then the
 * top Sampling.logprobs pairs, src/engine/lanes.rs:53-73), appended to `pairs` in output order
 * (a token's `end` is its pair count).  It stops before a token whose pairs do not fit;
 * HK_ESPACE with *n_pairs set when not even the first output's pairs fit. */
int hk_engine_outputs_lp(hk_engine* engine, uint64_t request, int64_t timeout_ms, hk_out* out,
                         size_t cap, size_t* n, char* message, size_t message_cap, hk_logprob* pairs,
                         size_t pairs_cap, size_t* n_pairs);

/* StepMetrics (src/engine/metrics.rs:4-19) summed over the run, as Metrics::total. */
typedef struct {
    uint64_t running, waiting, held_pages, pages, spec_tokens, prompt_tokens, cached_tokens,
        prefill_tokens, generation_tokens, preemptions, top_p_clipped, drafts;
} hk_step_metrics;

/* Metrics::total plus accepted_per_pos (its length in *n_pos) and the iteration_tokens
 * histogram (bounds 1, 8, 16, ..., 16384: 14 counts) with its sum. */
int hk_engine_metrics(hk_engine* engine, hk_step_metrics* total, uint64_t* accepted_per_pos,
                      size_t pos_cap, size_t* n_pos, uint64_t* counts, size_t counts_cap,
                      double* sum);

/* ------------------------------------------------------------------------------------ */
/* RoPE table (pinned against the reference's fixtures; src/gpu/load.rs:824-846)         */
/* ------------------------------------------------------------------------------------ */

/* Host function: fills table[rows][dim] fp32 with, per row p, dim/2 cosines then dim/2
 * sines of p * freq_i, freq_i = base^(-2i/dim) with YaRN-style correction when
 * original_seq_len > 0.  No device needed. */
int hk_rope_table(int64_t rows, int32_t dim, float base, int32_t original_seq_len,
                  float factor, float beta_fast, float beta_slow, float* table);

#ifdef __cplusplus
}
#endif

#endif /* HK_H */
