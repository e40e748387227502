/*
 * loraforge_b200 — C ABI of the B200 (sm_100a) multi-LoRA shrink/expand path.
 *
 * Every entry point takes raw device pointers, element counts and strides and a
 * cudaStream_t passed as `void*`; none of them allocates, synchronises or reads
 * device memory on the host. Each returns 0 on success or a negative LF_E_* code;
 * lf_last_error_string() then describes the failure (thread-local).
 *
 * Device metadata (slots, ranks, offsets, segment tables) is trusted the same way
 * the reference trusts it, with one difference: every kernel clamps the device
 * segment count to the host-known table capacity and skips out-of-range slot ids
 * instead of reading out of bounds.
 *
 * Element types: LF_F32 = 0, LF_F16 = 1, LF_BF16 = 2.
 * Reference paths below are relative to the lishenghui/loraforge source tree.
 */
#ifndef LORAFORGE_B200_H
#define LORAFORGE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  LF_OK = 0,
  LF_E_INVALID = -1,  /* structural argument error (shape, stride, alignment) */
  LF_E_CUDA = -2,     /* a CUDA runtime call or kernel launch failed */
  LF_E_UNSUPPORTED = -3,
};

enum { LF_F32 = 0, LF_F16 = 1, LF_BF16 = 2 };

/* Library version (major*10000 + minor*100 + patch). */
int lf_version(void);

/* Description of the last failure on this host thread ("" if none). */
const char* lf_last_error_string(void);

/*
 * Stable grouping of tokens by adapter slot, on device, in one CTA.
 *   token_indices[0:n_active]  = active tokens sorted by slot, ties by token index;
 *   token_indices[n_active:T]  = tokens with slot outside [0, num_slots), in order;
 *   segments: for each slot with tokens (ascending), ceil(count/chunk) segments of
 *   at most `chunk` tokens (chunk <= 0: one segment per slot);
 *   segment_indptr[0..nseg] offsets into token_indices, segment_slots[nseg],
 *   segment_count[0] = nseg.  Buffers must hold T+1 / T / T entries.
 * Replaces SGLang 0.5.22 ChunkedSgmvLoRABackend.prepare_lora_batch's grouping
 * (called at src/loraforge/integrations/_sglang_fleet.py:250-257); the layout of
 * its outputs is the one row_expand consumes (src/loraforge/ops/lora_rows.py:115-131).
 */
int lf_group_tokens(const int32_t* slots, int64_t num_tokens, int32_t num_slots,
                    int32_t chunk, int32_t* segment_indptr, int32_t* segment_slots,
                    int32_t* token_indices, int32_t* segment_count, void* stream);

/*
 * Device grouping of a prefill batch by runs, in one launch: a run is a maximal stretch
 * of consecutive tokens whose slot is in [0, num_slots); each run is cut into segments of
 * at most `chunk` tokens from its own start (chunk <= 0: one segment per run), in token
 * order.  token_indices[0:n_active] = the active tokens in token order, then the others;
 * segment_indptr / segment_slots / segment_count as for lf_group_tokens.  Any
 * segmentation of the same tokens gives the same products; this one makes every prefill
 * segment one run of a request's tokens (2-D tiles in lf_sgmv_prefill) and needs no sort.
 */
int lf_group_token_runs(const int32_t* slots, int64_t num_tokens, int32_t num_slots,
                        int32_t chunk, int32_t* segment_indptr, int32_t* segment_slots,
                        int32_t* token_indices, int32_t* segment_count, void* stream);

/*
 * Re-chunks a grouping (lf_group_tokens' tables) so that no segment spans a gap in token
 * order: inside each slot's range of token_indices, every maximal run of consecutive
 * tokens is cut into pieces of at most `chunk` tokens from its own start (chunk <= 0:
 * one piece per run).  token_indices is unchanged; out_indptr [T+1], out_slots [T] and
 * out_count [1] receive the new segments and must not alias the inputs.  A prefill batch
 * (each request one run of tokens with one adapter) then has only segments whose rows
 * are one run, which the prefill kernels move as 2-D tiles.  Same segment semantics as
 * lf_group_tokens: any segmentation of the grouping gives the same products.
 */
int lf_split_runs(const int32_t* segment_indptr, const int32_t* segment_slots,
                  const int32_t* token_indices, const int32_t* segment_count,
                  int64_t num_tokens, int32_t chunk, int32_t* out_indptr,
                  int32_t* out_slots, int32_t* out_count, void* stream);

/*
 * Inverse of the grouping: routes[t] = the slot of the segment whose token_indices range
 * holds t, -1 for tokens in no segment.  Reads *segment_count on the device (segments
 * beyond it or beyond max_segments, index entries outside [0, num_indices) and
 * positions outside [0, num_tokens) are ignored), so it turns a serving framework's
 * segment table (SGLang's seg_indptr / weight_indices / permutation, consumed by the
 * reference at src/loraforge/integrations/_sglang_fleet.py:390-407) into the
 * per-token slots the row-form shrink takes, inside a captured graph.
 */
int lf_segment_routes(const int32_t* segment_indptr, const int32_t* segment_slots,
                      const int32_t* token_indices, const int32_t* segment_count,
                      int32_t max_segments, int64_t num_indices, int64_t num_tokens,
                      int32_t* routes, void* stream);

/*
 * Retained-rank BF16 shrink: z[t, s*r+k] = bf16(sum_i a[g, s*r+k, i] * x[t, i]) for
 * g = slots[t] >= 0, r = ranks[g] in 1..max_rank, s < num_slices, k < r.  Other z
 * entries are left unchanged.  x row stride `x_stride` (elements), A contiguous
 * [num_slots, num_slices*capacity, width], z contiguous [T, num_slices*capacity].
 * Replaces src/loraforge/ops/csrc/lora_rows.cu:172-186 (`shrink`, bound by
 * src/loraforge/ops/lora_rows.py:106-109) and the fleet form
 * src/loraforge/ops/csrc/rowexpand.cu:87-97 (num_slices up to 4).
 */
int lf_row_shrink(const void* x, int64_t x_stride, const void* a, void* z,
                  const int32_t* slots, const int32_t* ranks, int64_t num_tokens,
                  int64_t width, int32_t num_slots, int32_t num_slices,
                  int32_t capacity, int32_t max_rank, void* stream);

/*
 * Compact-B RowExpand: for each active segment (<= 16 tokens, one slot g with rank
 * r in 1..64) and each output column n of slice s:
 *   acc = sum_{k < bucket} zf[k] * B[b_offsets[g] + n*bucket + k]   (k ascending,
 *         zf[k] = z[t, s*r+k] for k < r else 0),
 *   y[t, n] = bf16(y[t, n] + bf16(acc * scales[g])).
 * Same arithmetic, in the same order, as src/loraforge/ops/csrc/lora_rows.cu:67-162
 * (`expand` at :188-209) and src/loraforge/ops/csrc/rowexpand.cu:33-86.
 * row_tile in {2,4,8,16} splits segments into sub-tiles (work split only).
 * `threads` in {128, 256}; `blocks` is the persistent grid size (0: as many CTAs as the
 * SMs hold at once).  Each item covers 2 * threads output columns.
 */
int lf_row_expand(const void* z, const void* b, const int64_t* b_offsets,
                  const int32_t* b_strides, void* y, int64_t y_stride,
                  const int32_t* segment_indptr, const int32_t* segment_slots,
                  const int32_t* token_indices, const int32_t* ranks,
                  const float* scales, const int32_t* slice_offsets,
                  const int32_t* segment_count, int64_t num_tokens, int32_t out_width,
                  int32_t num_slices, int32_t capacity, int32_t num_slots,
                  int32_t max_segments, int32_t blocks, int32_t threads,
                  int32_t row_tile, void* stream);

/*
 * Padded-A decode shrink (SGLang "compatible" layout): A [num_slots, S*Rmax, width]
 * contiguous, z [T, S*Rmax] contiguous; rank = min(ranks[g], Rmax);
 * z[t, s*rank+k] = dtype(sum_i A[g, s*rank+k, i] * x[t, i]) for k < rank.  Other z
 * entries are not written (the Python layer zero-fills z first).
 * index_bits = 32 or 64 for ranks / token_map.  Replaces the Triton
 * shrink_dot_kernel / shrink_kernel+reduce_kernel launched by
 * src/loraforge/ops/gemv.py:46-127.
 */
int lf_bgmv_shrink(int32_t dtype, const void* x, int64_t x_stride, const void* a,
                   void* z, const void* ranks, const void* token_map,
                   int32_t index_bits, int64_t num_tokens, int64_t width,
                   int32_t num_slots, int32_t num_slices, int32_t rmax, void* stream);

/*
 * Padded-B decode expand: B [num_slots, out_width, Rmax] contiguous, z packed
 * [T, S*Rmax]; for column n in slice s (offsets[s] <= n < offsets[s+1]):
 *   y[t, n] = dtype(y[t, n] + dtype(scale_g * sum_{k<rank} z[t, s*rank+k] B[g,n,k])).
 * Rank-0 tokens are untouched.  scales dtype = scale_dtype (LF_*), offsets and
 * ranks/token_map use offset_bits / index_bits (32 or 64).
 * Replaces the Triton expand_dot_kernel / expand_kernel launched by
 * src/loraforge/ops/gemv.py:130-238.
 */
int lf_bgmv_expand(int32_t dtype, const void* z, const void* b, const void* ranks,
                   const void* scales, int32_t scale_dtype, const void* token_map,
                   int32_t index_bits, const void* offsets, int32_t offset_bits,
                   void* y, int64_t y_stride0, int64_t y_stride1, int64_t num_tokens,
                   int32_t out_width, int32_t num_slots, int32_t num_slices,
                   int32_t rmax, void* stream);

/* Per-slice operand descriptor for the vLLM padded layouts (up to 8 slices). */
typedef struct lf_slice_desc {
  const void* ptr;     /* slice base: A [slots, (1,) rank, width] or B [slots, (1,) n, rank] */
  int64_t slot_stride; /* elements between slots */
  int64_t row_stride;  /* elements between rows (rank rows for A, n rows for B) */
  int64_t rows;        /* rank (A) or n (B) */
} lf_slice_desc;

/*
 * vLLM BGMV shrink: out[s, t, :rank] (fp32, contiguous [S, T, rank]) =
 *   scale * A_s[routes[t]] @ x[t]; routes outside [0, num_slots) leave out untouched
 *   (the Python layer zero-fills out first, so they read as zeros).  Deterministic (no
 * atomics).  Replaces src/loraforge/ops/vllm_gemv.py:49-101 and
 * src/loraforge/ops/_vllm_gemv_kernels.py:12-53.
 */
int lf_vllm_shrink(int32_t dtype, const void* x, int64_t x_stride,
                   const lf_slice_desc* slices, int32_t num_slices, int32_t num_slots,
                   float* out, const int32_t* routes, int64_t num_tokens, int64_t width,
                   int32_t rank, float scale, void* stream);

/*
 * vLLM BGMV expand: y[t, offset + o_s + n] = dtype((add ? y : 0) + B_s[g] @ v[s, t])
 * with FP32 accumulation and one final cast; routes[t] < 0 rows are untouched.
 * Replaces src/loraforge/ops/vllm_gemv.py:107-159 and
 * src/loraforge/ops/_vllm_gemv_kernels.py:57-92.
 */
int lf_vllm_expand(int32_t dtype, const float* v, const lf_slice_desc* slices,
                   int32_t num_slices, int32_t num_slots, void* y, int64_t y_stride,
                   const int32_t* routes, int64_t num_tokens, int32_t rank,
                   int64_t offset, int32_t add, void* stream);

/*
 * Grouped (SGMV) retained-rank shrink -> expand over <= 16-token segments: the
 * operands of lf_row_shrink (x, A [slots, S*capacity, width]) and lf_row_expand
 * (compact B, b_offsets/b_strides, routing tables, scales, slice_offsets) in one
 * call of two chained kernels.  For every active segment (slot g, rank r in 1..64,
 * bucket b) and output column n of slice s:
 *   z[t, j] = sum_i x[t, i] * A[g, j, i]            (j < S*r, FP32)
 *   numerics 0 (fp32):      y[t, n] = bf16(y + scale_g * sum_k z[t, s*r+k] B_g[n, k])
 *   numerics 1 (reference): y[t, n] = bf16(y + bf16(scale_g * sum_k bf16(z) B_g[n, k]))
 * with k < min(r, b).  `workspace` is FP32 scratch of at least
 * lf_fused_workspace_floats(...) floats, 16-byte aligned, holding per-K-chunk
 * partial sums of z (added in chunk order, so results are deterministic; no
 * floating-point atomics), the FP32 z rows and one completion counter per segment.
 * It must be zero-filled before its first use; every call leaves the counters at
 * zero again, so one workspace serves any sequence of calls with the same num_tokens,
 * width, num_slices and capacity on one stream (the counters' offset depends on them:
 * zero the workspace again before calls with other sizes).
 * Requires width and x_stride multiples of 8, 16-byte aligned x/A/B, 8-byte aligned
 * y with y_stride a multiple of 4 and B regions at 8-element offsets.  Fused,
 * grouped form of the reference's two decode kernels (src/loraforge/ops/csrc/
 * lora_rows.cu:35-162, driven from src/loraforge/integrations/_sglang_fleet.py:271-407).
 */
int lf_fused_shrink_expand(const void* x, int64_t x_stride, const void* a, const void* b,
                           const int64_t* b_offsets, const int32_t* b_strides, void* y,
                           int64_t y_stride, const int32_t* segment_indptr,
                           const int32_t* segment_slots, const int32_t* token_indices,
                           const int32_t* ranks, const float* scales,
                           const int32_t* slice_offsets, const int32_t* segment_count,
                           float* workspace, int64_t workspace_floats, int64_t num_tokens,
                           int64_t width, int32_t out_width, int32_t num_slices,
                           int32_t capacity, int32_t num_slots, int32_t max_segments,
                           int32_t numerics, void* stream);

/*
 * Grouped (SGMV) shrink -> expand for prefill batches: the arguments and numerics of
 * lf_fused_shrink_expand, with segments of up to 128 tokens (group_tokens chunk 128;
 * lf_split_runs for segments that are runs of tokens, whose x and y rows move as 2-D TMA
 * tiles).  Every segment runs on the tcgen05 tensor cores with TMEM accumulators (M = 128
 * tokens per tile; shrink N = S*r rounded up to 16, K split in up to 3 parts so that the
 * segments fill the GPU in one wave; the expand adds the parts' FP32 partial z rows in
 * part order, then N = 128 output columns, K = the rank bucket); a short segment only
 * leaves tile rows idle.  `workspace` holds at least lf_sgmv_prefill_workspace_floats(...)
 * floats, 16-byte aligned (no contents carry over between calls).  Replaces the prefill path of the
 * reference: the rank-aware SGMV shrink (src/loraforge/integrations/_sglang_rank_aware.py:
 * 14-171) and the chunked SGMV expand it pairs with (SGLang's
 * chunked_sgmv_lora_expand_forward, called at src/loraforge/integrations/
 * _sglang_fleet.py:310-313 and :375-383).
 */
int lf_sgmv_prefill(const void* x, int64_t x_stride, const void* a, const void* b,
                    const int64_t* b_offsets, const int32_t* b_strides, void* y, int64_t y_stride,
                    const int32_t* segment_indptr, const int32_t* segment_slots,
                    const int32_t* token_indices, const int32_t* ranks, const float* scales,
                    const int32_t* slice_offsets, const int32_t* segment_count, float* workspace,
                    int64_t workspace_floats, int64_t num_tokens, int64_t width, int32_t out_width,
                    int32_t num_slices, int32_t capacity, int32_t num_slots, int32_t max_segments,
                    int32_t numerics, void* stream);

/* Workspace floats lf_sgmv_prefill needs for these sizes (-1 if invalid). */
int64_t lf_sgmv_prefill_workspace_floats(int64_t num_tokens, int64_t width, int32_t num_slices,
                                         int32_t capacity);

/*
 * Base projection with the LoRA delta in the same GEMM: y = x . W^T + scale_g . B_g . (A_g . x)
 * for every routed token, y written once (never read).  Replaces the base-then-delta pair of
 * the reference: lora_expand(..., base=) in src/loraforge/ops/gemv.py:130-238 and the base
 * output the fleet backend threads through (src/loraforge/integrations/_sglang_fleet.py:340-347).
 * W is [out_width, width] BF16 (row stride w_stride); the other operands and the routing are
 * those of lf_sgmv_prefill (segments of up to 128 tokens), FP32 numerics only.  Multi-slice
 * outputs need every slice boundary on a multiple of 256 columns.  Runs the prefill shrink,
 * per-token slots, per-tile slot lists and one persistent tcgen05 GEMM (128 x 256 tiles);
 * `workspace` holds lf_lora_base_gemm_workspace_floats(...) floats.
 */
int lf_lora_base_gemm(const void* x, int64_t x_stride, const void* w, int64_t w_stride, const void* a,
                      const void* b, const int64_t* b_offsets, const int32_t* b_strides, void* y,
                      int64_t y_stride, const int32_t* segment_indptr, const int32_t* segment_slots,
                      const int32_t* token_indices, const int32_t* ranks, const float* scales,
                      const int32_t* slice_offsets, const int32_t* segment_count, float* workspace,
                      int64_t workspace_floats, int64_t num_tokens, int64_t width, int32_t out_width,
                      int32_t num_slices, int32_t capacity, int32_t num_slots, int32_t max_segments,
                      void* stream);

/* Workspace floats lf_lora_base_gemm needs for these sizes (-1 if invalid). */
int64_t lf_lora_base_gemm_workspace_floats(int64_t num_tokens, int64_t width, int32_t num_slices,
                                           int32_t capacity);

/*
 * The two halves of lf_fused_shrink_expand (same arguments, same workspace): the shrink
 * leaves the FP32 z rows in the workspace, the expand reads them.  Between the two a
 * caller may combine z across devices, e.g. sum it over the ranks of a row-parallel
 * projection whose A columns are sharded (one all-reduce of the rows lf_fused_z_rows
 * locates).  Both calls must pass the same num_tokens, width, num_slices and capacity.
 * No counterpart in the reference, which has no tensor parallelism on this path
 * (src/loraforge/integrations/_sglang_fleet.py:177-178 rejects TP != 1).
 */
int lf_sgmv_shrink(const void* x, int64_t x_stride, const void* a, const void* b,
                   const int64_t* b_offsets, const int32_t* b_strides, void* y, int64_t y_stride,
                   const int32_t* segment_indptr, const int32_t* segment_slots,
                   const int32_t* token_indices, const int32_t* ranks, const float* scales,
                   const int32_t* slice_offsets, const int32_t* segment_count, float* workspace,
                   int64_t workspace_floats, int64_t num_tokens, int64_t width, int32_t out_width,
                   int32_t num_slices, int32_t capacity, int32_t num_slots, int32_t max_segments,
                   int32_t numerics, void* stream);
int lf_sgmv_expand(const void* x, int64_t x_stride, const void* a, const void* b,
                   const int64_t* b_offsets, const int32_t* b_strides, void* y, int64_t y_stride,
                   const int32_t* segment_indptr, const int32_t* segment_slots,
                   const int32_t* token_indices, const int32_t* ranks, const float* scales,
                   const int32_t* slice_offsets, const int32_t* segment_count, float* workspace,
                   int64_t workspace_floats, int64_t num_tokens, int64_t width, int32_t out_width,
                   int32_t num_slices, int32_t capacity, int32_t num_slots, int32_t max_segments,
                   int32_t numerics, void* stream);

/*
 * Where lf_sgmv_shrink leaves z in the workspace: `*row_floats` FP32 values per token
 * row, num_tokens rows starting `*offset` floats into the workspace (row = the token's
 * position in token_indices; columns s*r + k hold slice s, rank index k).
 */
int lf_fused_z_rows(int64_t num_tokens, int64_t width, int32_t num_slices, int32_t capacity,
                    int64_t* offset, int64_t* row_floats);

/* Workspace floats lf_fused_shrink_expand needs for these sizes (-1 if invalid). */
int64_t lf_fused_workspace_floats(int64_t num_tokens, int64_t width, int32_t num_slices,
                                  int32_t capacity);

/*
 * lf_fused_shrink_expand without a caller-provided workspace.  No counterpart in the
 * reference.  Some callers cannot allocate device memory: serving engines that hand
 * all free GPU memory to their own KV-cache pool at start-up and forbid later
 * cudaMalloc calls, and foreign-language hosts (cgo, JNI, N-API) that have no access
 * to the framework's caching allocator and must not create untracked allocations.
 * This entry point allocates nothing (no cudaMalloc, cudaFree or allocating library
 * call): its scratch is a 16 MiB array (4 Mi floats) compiled into the library plus a
 * 64 KiB array of per-segment counters at fixed positions, which every GPU that loads
 * the library holds until the process exits.  Sizes whose
 * lf_fused_workspace_floats(...) exceeds 4 Mi floats, or more than 16384 tokens, are
 * rejected with LF_E_INVALID.
 * The first call on a device looks up the buffer's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before any
 * stream capture.  All calls on a device share the buffer and it keeps the last call's
 * contents: the counters start zero-filled and every call leaves them at zero, also when
 * a bounded device wait runs out (the kernel then still counts the work it gave up on;
 * that call's output is invalid and lf_device_wait_timeouts reports it), so calls of any
 * sizes may follow one another; lf_fused_noalloc_reset zeroes them explicitly.  Calls
 * that overlap on the GPU (on other streams) race on the buffers and must be serialised
 * by the caller.  The buffer addresses are looked up again after the device's context
 * is destroyed and re-created (cudaDeviceReset).
 */
int lf_fused_shrink_expand_noalloc(const void* x, int64_t x_stride, const void* a,
                                   const void* b, const int64_t* b_offsets,
                                   const int32_t* b_strides, void* y, int64_t y_stride,
                                   const int32_t* segment_indptr, const int32_t* segment_slots,
                                   const int32_t* token_indices, const int32_t* ranks,
                                   const float* scales, const int32_t* slice_offsets,
                                   const int32_t* segment_count, int64_t num_tokens,
                                   int64_t width, int32_t out_width, int32_t num_slices,
                                   int32_t capacity, int32_t num_slots, int32_t max_segments,
                                   int32_t numerics, void* stream);

/*
 * Zero the per-segment completion counters of the built-in scratch of
 * lf_fused_shrink_expand_noalloc on the current device (cudaMemsetAsync on `stream`;
 * allocates nothing).  No counterpart in the reference.
 */
int lf_fused_noalloc_reset(void* stream);

/*
 * Zero the completion counters of a caller-owned lf_fused_shrink_expand workspace of
 * these sizes (cudaMemsetAsync on `stream`).  Every call leaves them at zero, also after
 * an expired device wait; this restores a workspace whose contents were overwritten.
 * No counterpart in the reference (its operators keep no workspace).
 */
int lf_fused_workspace_reset(float* workspace, int64_t workspace_floats, int64_t num_tokens,
                             int64_t width, int32_t num_slices, int32_t capacity, void* stream);

/*
 * Symmetric buffers and a one-shot sum over NVLink peer memory, for the row-parallel
 * LoRA intermediate (the all-reduce of the FP32 z rows between sgmv_shrink and
 * sgmv_expand; the reference has no tensor-parallel path, src/loraforge/integrations/
 * _sglang_fleet.py:177-178 rejects TP != 1).  Set-up, once per rank and device (these
 * allocate and map; the sum does not):
 *   lf_peer_alloc      cudaMalloc a buffer of lf_peer_buffer_bytes(capacity_floats) bytes,
 *                      zero it, and write its CUDA IPC handle (lf_peer_handle_bytes() bytes);
 *   lf_peer_open       map a peer rank's handle into this process (cudaIpcOpenMemHandle);
 *   lf_peer_close / lf_peer_free  undo them (after every rank's last lf_peer_sum).
 * lf_peer_sum: `bases` is a device array of `world` buffer pointers in rank order (this
 * rank's own buffer at `rank`, the mapped peers elsewhere); every rank calls it with its
 * own z (floats <= capacity_floats FP32 values, 16-byte aligned) in the same order on its
 * stream, and on return every rank's z holds the sum over ranks, added in rank order (the
 * same bits on every rank).  One launch of 16 CTAs; the epoch lives on the device, so the
 * call may be captured in a CUDA graph.  Waits for peers are bounded: at most spin_limit
 * polls of the flag (spin_limit <= 0 or above the default: the default of 2^22 polls, well
 * under 2 s); on expiry z keeps this rank's partial and lf_peer_status reports 1.  A peer
 * that arrives after this rank gave up still computes the full sum, so the ranks' z then
 * differ: callers check lf_peer_status (a synchronising read) at a step boundary and
 * discard the step's outputs when it is 1.
 */
int64_t lf_peer_buffer_bytes(int64_t capacity_floats);
int lf_peer_handle_bytes(void);
int lf_peer_alloc(int64_t capacity_floats, void** buffer, void* ipc_handle);
int lf_peer_open(const void* ipc_handle, void** buffer);
int lf_peer_close(void* buffer);
int lf_peer_free(void* buffer);
int lf_peer_status(void* own_buffer, int32_t* status, int32_t reset);
int lf_peer_sum(const uint64_t* bases, int32_t rank, int32_t world, float* z, int64_t floats,
                int64_t capacity_floats, int64_t spin_limit, void* stream);

/*
 * Number of bounded device-side waits (mbarrier polls in the bulk-copy kernels)
 * that expired since the last reset; a non-zero count means a kernel gave up and
 * skipped work instead of hanging.  Synchronous; reset != 0 clears the counter.
 * No reference counterpart (the reference kernels have no waits).
 */
int lf_device_wait_timeouts(int32_t* count, int32_t reset);

#ifdef __cplusplus
}
#endif

#endif /* LORAFORGE_B200_H */
