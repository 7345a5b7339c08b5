/*
 * agentserve_b200 — C ABI of the B200 (sm_100a) continuous-batching attention step.
 *
 * Plain C: device pointers, sizes and a cudaStream_t.  No torch types.  Every
 * entry point is stream-ordered on the caller's stream, allocates nothing, and
 * returns an int status (AS_OK = 0).  On failure as_last_error() gives a
 * message for the calling host thread.  Kernels never trap: out-of-range block
 * ids / slots / positions and bounded waits that run out set bits in a per-device
 * status word that as_device_status() reads and clears.
 *
 * KV pool layout (one layer, K and V planes given separately) follows the
 * reference's kv_pool[2, L, NB, BS, Kh, D] (agentserve/engine/cache.py:62-66):
 *   k_cache / v_cache = &kv_pool[0|1, layer]  viewed as [NB, BS, Kh, D],
 *   slot s = block_id * BS + offset  addresses row s of [NB*BS, Kh, D].
 * BS (block_size) must be 16 (the reference default, engine.py:86).
 *
 * Reference interfaces replaced (file:line inside krishs0404/agentserve):
 *   as_pack_decode            engine.py:349-357 + llama.py:408-411 (host lists -> tensors)
 *                             + cache.py:152-154 (slot of the decode token)
 *   as_pack_prefill           engine.py:299-307 + cache.py:134-140 (slots of prompt tokens)
 *   as_rope_reshape_and_cache llama.py:80-99 (apply_rope on q,k) + cache.py:125-156
 *                             (write_kv_prefill / write_kv_decode)
 *   as_paged_decode_attention llama.py:419-469 (gather_kv -> pad -> GQA expand -> SDPA)
 *                             and llama.py:303-361 (padded-list decode)
 *   as_rope_paged_decode_attention  llama.py:433-469 (RoPE of the new token, its
 *                             write_kv_decode and the attention) in one launch
 *   as_varlen_prefill_attention llama.py:128-186 (prefill over cached prefix + new tokens)
 *   as_varlen_prefill_attention_ws  the same, split-KV over CTAs with a workspace
 *   as_linear_small_m(_swiglu) nn.Linear of the decode step (llama.py:123-126, 203-211,
 *                             430-431, 471): q/k/v, o_proj, gate/up, down at batch <= 256
 *   as_greedy_argmax          sampling.py:46-58 (greedy branch) + engine.py:379-383
 *   as_block_copy             cache.py:158-189 (gather_kv) and engine.py:274-281,338-345
 *                             (prefix-cache KV clone / seed)
 *   as_rmsnorm / as_add_rmsnorm / as_silu_mul
 *                             llama.py:39-56 (RMSNorm), :234-237 (residuals), :207-211 (SwiGLU)
 */
#ifndef AGENTSERVE_B200_H_
#define AGENTSERVE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AS_API __attribute__((visibility("default")))
#else
#define AS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* as_stream_t; /* == cudaStream_t; NULL = legacy default stream */

/* status codes */
#define AS_OK 0
#define AS_ERR_INVALID_ARG 1
#define AS_ERR_UNSUPPORTED 2
#define AS_ERR_CUDA 3
#define AS_ERR_WORKSPACE 4

/* layouts of the decode attention output [B, H*D] */
#define AS_LAYOUT_HEAD_MAJOR 0 /* out[b, h*D + d] (prefill's flatten, llama.py:184) */
#define AS_LAYOUT_DIM_MAJOR 1  /* out[b, d*H + h] (the reference decode paths' flatten,
                                  SDPA out .transpose(1, 2).reshape(B, H*D), llama.py:362,470) */

/* element types of q / k / v / out / KV pool */
#define AS_DTYPE_F32 0
#define AS_DTYPE_F16 1
#define AS_DTYPE_BF16 2

/* Library version (major*10000 + minor*100 + patch). */
AS_API int as_version(void);

/* Message for the last failing call on this host thread ("" if none). */
AS_API const char* as_last_error(void);

/* Read (and clear when clear != 0) the device status word of the current device.
 * Synchronises `stream`.  Bits: 1 bad block id, 2 bad slot, 4 wait timeout,
 * 8 RoPE position outside the table, 16 sequence longer than its block-table row. */
AS_API int as_device_status(int clear, int* out_bits, as_stream_t stream);

/* Failure detection (no counterpart in the reference, which has no device code).
 * Every mbarrier wait in the attention kernels gives up after a time limit, sets
 * status bit 4, lets the copies it started land (again bounded), frees its tensor
 * memory and returns, so a stuck pipeline costs one failed call, never a hung GPU.
 * as_set_wait_limit_ns sets that limit for kernels launched from now on (0 = the
 * default of 2 s) and returns the previous one.  Launches captured in a CUDA graph
 * keep the limit they were captured with. */
AS_API uint64_t as_set_wait_limit_ns(uint64_t limit_ns);

/* Test hook for that path: the next launch of each kernel named in `kernels`
 * (AS_KERNEL_* bits) issues none of its loads, so its waits run out, and the call
 * must come back with status bit 4 set and the next call must be correct again.
 * Each call replaces the pending set (0 clears it). */
#define AS_KERNEL_DECODE_ATTENTION 1  /* as_paged_decode_attention, bf16/fp16 fast path */
#define AS_KERNEL_PREFILL_ATTENTION 2 /* as_varlen_prefill_attention*, tcgen05 path */
AS_API int as_debug_starve_next_launch(int kernels);

/* ------------------------------------------------------------------------- */
/* (1) Ragged-batch packing                                                  */
/* ------------------------------------------------------------------------- */

/* Decode batch of B sequences.  Inputs:
 *   block_tables [*, bt_stride] int32 — device-resident table rows of the allocator
 *   row_ids      [B] int32            — table row of each sequence (NULL: row b)
 *   seq_lens     [B] int32            — tokens already cached = position of the new token
 *                                       (engine.py:350,356: num_cached + num_out - 1)
 * Outputs (all device):
 *   positions    [B]    int64  = seq_lens
 *   slot_mapping [B]    int64  = bt[row][pos/16]*16 + pos%16    (cache.py:152-154)
 *   seq_lens_k   [B]    int32  = seq_lens + 1 (keys visible to the new token)
 *   cu_seqlens_q [B+1]  int32  = 0,1,...,B
 *   packed_bt    [B, max_blocks] int32 — rows gathered (NULL to skip)
 */
AS_API int as_pack_decode(const int32_t* block_tables, int64_t bt_stride, const int32_t* row_ids,
                   const int32_t* seq_lens, int32_t num_seqs, int32_t max_blocks,
                   int32_t block_size, int64_t* positions, int64_t* slot_mapping,
                   int32_t* seq_lens_k, int32_t* cu_seqlens_q, int32_t* packed_bt,
                   as_stream_t stream);

/* Varlen prefill batch of R sequences with num_cached[r] tokens already in the
 * pool (prefix-cache hit, engine.py:275-276) and num_new[r] new tokens.
 * Outputs: cu_seqlens_q [R+1] (prefix sum of num_new), positions/slot_mapping
 * [total_new] int64 (position num_cached+i, cache.py:136-140), seq_lens_k [R] =
 * num_cached + num_new, packed_bt [R, max_blocks] (NULL to skip).  total_new must
 * equal sum(num_new) (the host knows it; it sizes the outputs). */
AS_API int as_pack_prefill(const int32_t* block_tables, int64_t bt_stride, const int32_t* row_ids,
                    const int32_t* num_cached, const int32_t* num_new, int32_t num_seqs,
                    int32_t total_new, int32_t max_blocks, int32_t block_size,
                    int32_t* cu_seqlens_q, int64_t* positions, int64_t* slot_mapping,
                    int32_t* seq_lens_k, int32_t* packed_bt, as_stream_t stream);

/* ------------------------------------------------------------------------- */
/* (2) Fused RoPE + reshape_and_cache                                        */
/* ------------------------------------------------------------------------- */

/* For T tokens: rotate q [T, H, D] in place (row stride q_stride elements),
 * rotate k [T, Kh, D] and write it to k_cache at slot_mapping[t]; write v
 * unrotated to v_cache.  Rotate-half RoPE in fp32 from the fp32 table
 * cos_sin [table_len, D] (first half cos, second half sin; llama.py:63-77),
 * out = [x1*c - x2*s, x2*c + x1*s] rounded to the element type (llama.py:97-99).
 * A negative slot skips that token's cache write.  k_out (optional, may be NULL)
 * receives the rotated k [T, Kh, D] contiguous.  With cos_sin == NULL nothing is
 * rotated: k and v are copied to their slots as given (write_kv_prefill /
 * write_kv_decode, cache.py:125-156) and q / positions may be NULL. */
AS_API int as_rope_reshape_and_cache(void* q, int64_t q_stride, const void* k, int64_t k_stride,
                              const void* v, int64_t v_stride, const int64_t* positions,
                              const int64_t* slot_mapping, const float* cos_sin,
                              int32_t table_len, void* k_cache, void* v_cache,
                              int64_t num_slots, void* k_out, int32_t num_tokens,
                              int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                              int32_t dtype, as_stream_t stream);

/* ------------------------------------------------------------------------- */
/* (3) Paged GQA split-K decode attention                                    */
/* ------------------------------------------------------------------------- */

/* Bytes of workspace needed by as_paged_decode_attention. */
AS_API size_t as_paged_decode_workspace_size(int32_t num_seqs, int32_t num_heads, int32_t num_kv_heads,
                                      int32_t head_dim, int32_t max_blocks,
                                      int32_t blocks_per_split);

/* One query token per sequence: out[b, h, :] = softmax(scale * q[b,h] . K^T) V over
 * the seq_lens_k[b] keys of sequence b, read in place from the paged pool through
 * block_tables [B, bt_stride] (KV head of query head h is h / (H/Kh)).
 * q: [B, H, D] with row stride q_stride elements between tokens; out: [B, H*D] in
 * out_layout (AS_LAYOUT_HEAD_MAJOR or AS_LAYOUT_DIM_MAJOR).
 * blocks_per_split sets the split-K chunk (0: chosen by the library from B, Kh,
 * max_blocks and the SM count); a sequence of n blocks uses ceil(n / blocks_per_split)
 * CTAs per KV head, combined in-kernel by the last CTA.
 * Workspace (as_paged_decode_workspace_size bytes, 256-byte aligned; needed when a
 * sequence can span more than one split): its first round_up(B*H*4, 256) bytes are
 * per-(sequence, head) arrival counters that must be zero when the call starts, and
 * the call leaves them zero; the bytes after them hold split partials and need no
 * initialisation.  Calls sharing a workspace must be stream-ordered. */
AS_API int as_paged_decode_attention(void* out, const void* q, int64_t q_stride, const void* k_cache,
                              const void* v_cache, const int32_t* block_tables,
                              int64_t bt_stride, const int32_t* seq_lens_k, int32_t num_seqs,
                              int32_t num_heads, int32_t num_kv_heads, int32_t head_dim,
                              int32_t block_size, int32_t num_blocks, int32_t max_blocks,
                              float scale, int32_t blocks_per_split, void* workspace,
                              size_t workspace_bytes, int32_t out_layout, int32_t dtype,
                              as_stream_t stream);

/* The decode step's RoPE + cache write and its attention in one launch: replaces
 * apply_rope on the new token's q and k (llama.py:433-434), write_kv_decode
 * (llama.py:437-439, cache.py:142-156) and the attention (llama.py:441-469).  q, k, v
 * are the new token's UNROTATED projections ([B, H, D] / [B, Kh, D] rows, strides in
 * elements, e.g. column slices of a fused QKV output; none is modified); positions /
 * slot_mapping [B] int64 as for as_rope_reshape_and_cache (a bad position or slot is
 * flagged and skipped the same way).  The CTA that reads a sequence's last block
 * writes the rotated k and v into the pool first; q is rotated as it is loaded.  The
 * pool bytes and the output equal those of as_rope_reshape_and_cache followed by
 * as_paged_decode_attention bit for bit.  Fast path only (bf16 / fp16, head_dim 64 or
 * 128, GQA group <= 8); otherwise AS_ERR_UNSUPPORTED, and the two calls above apply.
 * Other arguments as as_paged_decode_attention (seq_lens_k counts the new token). */
AS_API int as_rope_paged_decode_attention(void* out, const void* q, int64_t q_stride, const void* k,
                              int64_t k_stride, const void* v, int64_t v_stride,
                              const int64_t* positions, const int64_t* slot_mapping,
                              const float* cos_sin, int32_t table_len, void* k_cache,
                              void* v_cache, const int32_t* block_tables, int64_t bt_stride,
                              const int32_t* seq_lens_k, int32_t num_seqs, int32_t num_heads,
                              int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                              int32_t num_blocks, int32_t max_blocks, float scale,
                              int32_t blocks_per_split, void* workspace, size_t workspace_bytes,
                              int32_t out_layout, int32_t dtype, as_stream_t stream);

/* Same computation as as_paged_decode_attention, for callers that cannot allocate
 * device memory (their GPU memory belongs to another allocator, or their serving loop
 * must not reach cudaMalloc's implicit synchronisation) and so have no workspace to
 * pass.  No counterpart in the reference: it has no native code and no workspace.
 * The split-K scratch is a static array of AS_DECODE_NOALLOC_SCRATCH_BYTES inside the
 * library, held by every GPU that loads the library until the process exits.  A call
 * whose scratch need (as_paged_decode_workspace_size) exceeds that is rejected with
 * AS_ERR_WORKSPACE.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) for that device; make that first call before any stream
 * capture.  Each call clears the array's counter region with cudaMemsetAsync on
 * `stream` and allocates nothing.  All calls on a device share the one array: calls
 * whose executions overlap on the GPU (different streams, no ordering) race. */
#define AS_DECODE_NOALLOC_SCRATCH_BYTES (8u << 20)
AS_API int as_paged_decode_attention_noalloc(void* out, const void* q, int64_t q_stride,
                                             const void* k_cache, const void* v_cache,
                                             const int32_t* block_tables, int64_t bt_stride,
                                             const int32_t* seq_lens_k, int32_t num_seqs,
                                             int32_t num_heads, int32_t num_kv_heads,
                                             int32_t head_dim, int32_t block_size,
                                             int32_t num_blocks, int32_t max_blocks, float scale,
                                             int32_t blocks_per_split, int32_t out_layout,
                                             int32_t dtype, as_stream_t stream);

/* ------------------------------------------------------------------------- */
/* (4) Varlen prefill attention over cached prefix blocks + new tokens       */
/* ------------------------------------------------------------------------- */

/* q: [total_q, H, D] (row stride q_stride elements), new tokens of sequence r at
 * rows cu_seqlens_q[r] .. cu_seqlens_q[r+1]-1.  Keys/values: the first
 * seq_lens_k[r] tokens of the sequence in the paged pool (prefix + new tokens,
 * already written by as_rope_reshape_and_cache).  New token i of sequence r sits
 * at position P + i with P = seq_lens_k[r] - num_new[r]; it attends to keys
 * 0..P+i (cached prefix unmasked, new tokens causal: llama.py:171-180).
 * out: [total_q, H*D]. */
AS_API int as_varlen_prefill_attention(void* out, const void* q, int64_t q_stride, const void* k_cache,
                                const void* v_cache, const int32_t* block_tables,
                                int64_t bt_stride, const int32_t* cu_seqlens_q,
                                const int32_t* seq_lens_k, int32_t num_seqs,
                                int32_t max_seqlen_q, int32_t total_q, int32_t num_heads,
                                int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                int32_t num_blocks, int32_t max_blocks, float scale,
                                int32_t dtype, as_stream_t stream);

/* Same computation with split-KV (same reference interface, llama.py:128-186): for
 * head_dim 64 or 128 in bf16/f16 the key range of every query tile pair can be divided over
 * num_splits CTAs, whose partial results (fp32) go to `workspace` and are combined by
 * a second kernel on the same stream.  This fills the GPU when few sequences are
 * prefilled at once (the reference prefills one request per call, engine.py:228-229).
 * num_splits: 0 = chosen from the grid shape and SM count, 1 = no split, k > 1 = k
 * (at most 16).  workspace: as_varlen_prefill_workspace_size() bytes, 256-byte aligned;
 * it needs no initialisation.  With num_splits = 0 and too small (or NULL) a workspace
 * the call runs unsplit; with k > 1 it fails with AS_ERR_WORKSPACE.  Shapes the split
 * does not apply to ignore num_splits and workspace. */
AS_API int as_varlen_prefill_attention_ws(void* out, const void* q, int64_t q_stride,
                                          const void* k_cache, const void* v_cache,
                                          const int32_t* block_tables, int64_t bt_stride,
                                          const int32_t* cu_seqlens_q,
                                          const int32_t* seq_lens_k, int32_t num_seqs,
                                          int32_t max_seqlen_q, int32_t total_q,
                                          int32_t num_heads, int32_t num_kv_heads,
                                          int32_t head_dim, int32_t block_size,
                                          int32_t num_blocks, int32_t max_blocks, float scale,
                                          int32_t dtype, int32_t num_splits, void* workspace,
                                          size_t workspace_bytes, as_stream_t stream);

/* Workspace bytes as_varlen_prefill_attention_ws needs for these sizes and num_splits
 * (0 when no split applies). */
AS_API size_t as_varlen_prefill_workspace_size(int32_t num_seqs, int32_t max_seqlen_q,
                                               int32_t num_heads, int32_t num_kv_heads,
                                               int32_t head_dim, int32_t max_blocks,
                                               int32_t num_splits, int32_t dtype);

/* ------------------------------------------------------------------------- */
/* (6) Decode-step projections at small batch                                */
/* ------------------------------------------------------------------------- */

/* y[m, n] = sum_k x[m, k] * w[n, k] for m < M <= 256 (nn.Linear without bias: the
 * q/k/v, o_proj, gate/up and down projections of the decode step, llama.py:123-126,
 * 203-211, 430-431, 471), bf16/fp16, fp32 accumulation.  Row strides y_stride and
 * x_stride in elements; w is [N, K] row-major (nn.Linear.weight); x, w and their rows
 * 16-byte aligned.  The K range is split over the CTAs of a thread-block cluster when
 * N/128 alone cannot fill the GPU; the fp32 partial sums are added on chip in a fixed
 * order, so results are deterministic and no workspace is needed. */
AS_API int as_linear_small_m(void* y, int64_t y_stride, const void* x, int64_t x_stride,
                             const void* w, int32_t M, int32_t N, int32_t K, int32_t dtype,
                             as_stream_t stream);

/* The gate/up projection with SwiGLU in its epilogue: y[m, j] = to_T(to_T(silu(g)) * u)
 * with g = x w[j]^T and u = x w[inter + j]^T each rounded to the element type first
 * (llama.py:203-211; the same bits as as_linear_small_m on w followed by as_silu_mul).
 * w is the fused [2*inter, K] = [gate; up] weight (the layout as_silu_mul's input
 * comes from), inter a multiple of 64; y is [M, inter] (row stride y_stride).
 * M <= 256, bf16/fp16; each CTA loads 64 gate rows and the matching 64 up rows, K
 * split over a cluster as in as_linear_small_m. */
AS_API int as_linear_small_m_swiglu(void* y, int64_t y_stride, const void* x, int64_t x_stride,
                             const void* w_gate_up, int32_t M, int32_t inter, int32_t K,
                             int32_t dtype, as_stream_t stream);

/* ------------------------------------------------------------------------- */
/* (7) Greedy sampling                                                        */
/* ------------------------------------------------------------------------- */

/* out[r] = index of the first maximum of row r of logits [num_rows, vocab] (row
 * stride in elements) after the reference's sanitising (sampling.py:46-58 at
 * temperature <= 1e-6: fp32, NaN -> 0, +inf -> 1e4, -inf -> -1e4), in one pass over
 * the logits.  workspace: as_greedy_workspace_size(num_rows) bytes, 256-byte aligned,
 * zero on first use; the library leaves it zero (calls sharing it must be ordered on
 * one stream). */
AS_API size_t as_greedy_workspace_size(int32_t num_rows);
AS_API int as_greedy_argmax(int64_t* out, const void* logits, int64_t row_stride,
                            int32_t num_rows, int32_t vocab, int32_t dtype, void* workspace,
                            size_t workspace_bytes, as_stream_t stream);

/* ------------------------------------------------------------------------- */
/* (5) Block gather / copy (prefix-cache seeding, gather_kv)                 */
/* ------------------------------------------------------------------------- */

/* For each plane p < num_planes and i < n:
 *   copy bytes_per_block bytes from src + p*src_plane_stride + src_ids[i]*bytes_per_block
 *                               to dst + p*dst_plane_stride + dst_ids[i]*bytes_per_block
 * (dst_ids NULL means dst block i).  A plane is one (K|V, layer) slice of a pool;
 * with dst_ids NULL and a dense dst this is gather_kv for all layers at once.
 * bytes_per_block and both plane strides must be multiples of 16; src and dst
 * 16-byte aligned.  src_num_blocks / dst_num_blocks bound the ids. */
AS_API int as_block_copy(void* dst, const void* src, const int32_t* src_ids, const int32_t* dst_ids,
                  int32_t n, int64_t bytes_per_block, int32_t num_planes,
                  int64_t src_plane_stride, int64_t dst_plane_stride, int32_t src_num_blocks,
                  int32_t dst_num_blocks, as_stream_t stream);

/* ------------------------------------------------------------------------- */
/* Fused elementwise stages of the decode step (rows x dim, contiguous rows)  */
/* ------------------------------------------------------------------------- */

/* out = to_T(x * rsqrt(mean(x^2) + eps)) * weight, statistics in fp32.
 * Replaces RMSNorm.forward (llama.py:39-56). */
AS_API int as_rmsnorm(void* out, const void* x, const void* weight, int64_t rows, int32_t dim,
                      float eps, int32_t dtype, as_stream_t stream);

/* x = to_T(x + delta) in place (the residual add, llama.py:234-237), then
 * out = rmsnorm(x) as above: the residual add and the next pre-norm in one pass. */
AS_API int as_add_rmsnorm(void* out, void* x, const void* delta, const void* weight,
                          int64_t rows, int32_t dim, float eps, int32_t dtype,
                          as_stream_t stream);

/* gate_up [rows, 2*inter] = [gate | up]; out [rows, inter] = to_T(to_T(silu(gate)) * up).
 * Replaces the SwiGLU activation of LlamaMLP.forward (llama.py:207-211). */
AS_API int as_silu_mul(void* out, const void* gate_up, int64_t rows, int32_t inter,
                       int32_t dtype, as_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* AGENTSERVE_B200_H_ */
