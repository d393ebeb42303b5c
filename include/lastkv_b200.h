/*
 * lastkv_b200 — C ABI of the B200 (sm_100a) kernels for LastKV's shared
 * last-layer-KV attention path.
 *
 * Memory layout shared by every entry point (the reference's merged pool,
 * vllm/src/lastkv/vllm/backends/rmarin_flashinfer/batching.py:1999-2016):
 *   pool_k, pool_v : bf16 [num_pages, page_size=16, num_kv_heads, head_dim]
 *                    pages [0, src_pages) hold the shared final-layer history
 *                    (raw K, raw V); each layer owns ring pages that hold K and
 *                    V / s_l for the previous and current chunk.
 *   block_table    : int32 [batch, >= pages_per_seq] row-strided, one row per
 *                    sequence = [older shared pages | this layer's ring pages]
 *   seq_k          : int32 [batch] number of keys of each sequence
 *   q / out        : bf16 [tokens, num_q_heads, head_dim], head_dim contiguous,
 *                    heads packed, rows strided by q_stride_tok / out_stride_tok
 *
 * All pointers are device pointers unless stated; `stream` is a cudaStream_t
 * (NULL = legacy default stream).  Calls never allocate, never synchronise and
 * are safe to record into a CUDA graph.  Every entry point returns LKV_OK or a
 * nonzero status; nothing is launched when the status is nonzero.
 *
 * Device-side failures (a block-table page outside the pool, an append slot
 * outside the pool, a pipeline wait that gave up) do not fault: the kernel
 * skips the access and records the first failure in the int32[4] error word
 * at the start of the workspace (or the `error_word` argument), readable with
 * lkv_read_error_word().
 */
#ifndef LASTKV_B200_H
#define LASTKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LKV_OK 0
#define LKV_ERR_INVALID_ARGUMENT 1
#define LKV_ERR_UNSUPPORTED 2
#define LKV_ERR_CUDA 3
#define LKV_ERR_ARCH 4
#define LKV_ERR_TENSOR_MAP 5
#define LKV_ERR_WORKSPACE 6

#define LKV_PAGE_SIZE 16

/* Human-readable text of a status code. */
const char* lkv_status_string(int status);

/* ABI version of this library (major * 100 + minor). */
int lkv_abi_version(void);

/* LKV_OK if `device` is an sm_100 (B200-class) GPU this library was built for.
 * When `device` is the current device it also loads the static scratch of
 * lkv_decode_paged_noalloc there (see below), so call it at start-up. */
int lkv_check_device(int device);

/* Copy the int32[4] error word {code, kernel, block, detail} to host memory.
 * Synchronises `stream`.  code 0 means no device-side failure was recorded. */
int lkv_read_error_word(const int32_t* error_word, int32_t host_out[4], void* stream);

/* Zero the error word (asynchronously on `stream`). */
int lkv_clear_error_word(int32_t* error_word, void* stream);

/* ------------------------------------------------------------------ decode
 * One query token per sequence against its paged history (split-KV).
 * Replaces, for uniform decode steps, the merged per-layer attention call
 *   flash_attn_varlen_func(q, pool_k, pool_v, cu_seqlens_q, seqused_k,
 *                          causal=True, block_table=bt_all[l]) + head_scale_
 * (vllm/.../rmarin_flashinfer/fastpath.py:643-650) and, at the HF level, the
 * SDPA call of LastKVAttention.forward (llm/src/lastkv/llm/modeling.py:143-146).
 *   out[b, h, :] = out_scale[h] * softmax(q k^T * softmax_scale) v   (bf16)
 *   lse[b, h]    = natural-log log-sum-exp of the scaled scores (optional)
 * out_scale (fp32 [num_q_heads], optional) folds the per-layer value scale s_l
 * (fused_qkv.py:140-155).  With `partial_o`/`partial_lse` non-NULL the call
 * instead writes fp32 normalised outputs [batch, num_q_heads, head_dim] and
 * natural-log LSE [batch, num_q_heads] for a later lkv_merge_partials (the
 * context-parallel combine); `out`, `lse` and `out_scale` are then ignored.
 * Supported: head_dim 64 or 128; num_q_heads / num_kv_heads in {1, 2, 4, 8}.
 *
 * Programmatic dependent launch (PDL): the kernel may start while the kernels
 * before it in the stream still run; CUDA makes their writes visible to it
 * only at its griddepcontrol.wait.  With flags = 0 it reads nothing (q, seq_k,
 * block table, pages, workspace) before that wait, so any kernel before it may
 * produce any input.  With LKV_DECODE_TABLES_READY it requests its first pages
 * before the wait, overlapping the ring fill with the previous kernel's tail;
 * the caller then guarantees that seq_k, the block table rows and every page
 * of a sequence but its last (where an append kernel just before the call
 * puts this step's key) were written before the most recent operation in the
 * stream that was NOT a PDL kernel launch - a copy, a plain kernel launch
 * (torch's, or this library's lkv_build_layer_block_tables) or the start of a
 * graph - since PDL launches chained back to back may all start before that
 * point, and the first of them before that operation has finished.  Example: a
 * step that copies its tables in, launches any plain kernel, then runs the
 * layers' append + decode pairs; not a step that builds its tables with
 * lkv_build_layer_block_tables right before its first decode.
 */
#define LKV_DECODE_TABLES_READY 1
/* LKV_DECODE_L2_KEEP: this call is one of several over the same history (the
 * layers of a step all read the shared final-layer pages): the first columns of
 * every block-table row - the oldest pages, a quarter of the L2 cache over the
 * batch - load with the L2 evict_last policy and the rest with evict_first, so
 * those pages stay in L2 from one call to the next.  Arithmetic unchanged.
 * It pays at small batches, where a quarter of L2 is a larger share of the
 * history (8B decode step, batch 8: +1.8 %; batch 64: -0.5 %), so the flag
 * takes effect for batches up to 16 only. */
#define LKV_DECODE_L2_KEEP 2

size_t lkv_decode_workspace_bytes(int batch, int num_q_heads, int head_dim, int max_pages_per_seq);

int lkv_decode_paged(const void* q, int64_t q_stride_tok,
                     const void* pool_k, const void* pool_v, int64_t num_pages,
                     const int32_t* block_table, int64_t block_table_stride,
                     const int32_t* seq_k,
                     void* out, int64_t out_stride_tok, float* lse, const float* out_scale,
                     float* partial_o, float* partial_lse,
                     int batch, int num_q_heads, int num_kv_heads, int head_dim,
                     int max_pages_per_seq, float softmax_scale,
                     void* workspace, size_t workspace_bytes, int flags, void* stream);

/* Allocation-free form of lkv_decode_paged.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory - an engine whose
 * KV-cache pool already holds nearly all of HBM (a side cudaMalloc may fail),
 * a C-FFI host that can only pass the inputs and outputs it owns, or a loop
 * that cannot afford cudaMalloc's implicit synchronisation.  Instead of a
 * caller workspace it uses one static device array of
 * LKV_NOALLOC_SCRATCH_BYTES inside the library, held on a GPU from the moment
 * the library's module is loaded there until the process exits.  Module
 * loading is lazy: it happens at lkv_check_device(d) while d is the current
 * device, or else at the first no-alloc call on that device - make one of
 * them before the engine reserves its KV-cache pool.
 *  - Same arguments and result as lkv_decode_paged (final bf16 output only,
 *    flags = 0), without workspace; `error_word` (device int32[4], may be NULL) receives
 *    the call's device error word.
 *  - Rejects, with LKV_ERR_WORKSPACE and nothing launched, shapes where
 *    batch * num_q_heads * (head_dim + 1) * 4 + 512 > LKV_NOALLOC_SCRATCH_BYTES.
 *  - The first of those calls on a device looks up the array's address with
 *    that device current; make it before any stream capture.  The address is
 *    cached for the process: do not reset the device's primary context.
 *  - All calls share the array: calls whose GPU work overlaps race; serialise.
 *  - Allocates nothing (no cudaMalloc / cudaFree). */
#define LKV_NOALLOC_SCRATCH_BYTES (8u << 20)

int lkv_decode_paged_noalloc(const void* q, int64_t q_stride_tok,
                             const void* pool_k, const void* pool_v, int64_t num_pages,
                             const int32_t* block_table, int64_t block_table_stride,
                             const int32_t* seq_k,
                             void* out, int64_t out_stride_tok, float* lse, const float* out_scale,
                             int batch, int num_q_heads, int num_kv_heads, int head_dim,
                             int max_pages_per_seq, float softmax_scale,
                             int32_t* error_word, void* stream);

/* Host query: how many KV splits and kernel launches lkv_decode_paged will use
 * for this shape and workspace on the current device (partial != 0 for the
 * partial-output form).  Needs a device; launches nothing. */
int lkv_decode_plan(int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_pages_per_seq,
                    size_t workspace_bytes, int partial, int* num_splits, int* num_launches);

/* ------------------------------------------------------------------ prefill
 * Varlen (chunked) prefill against the paged history on tcgen05 tensor cores.
 * Replaces the same merged call as lkv_decode_paged for spans of more than one
 * token (fastpath.py:643-650 with cu_seqlens_q / max_seqlen_q, causal,
 * bottom-right aligned) and the masked SDPA of modeling.py:124-146; with
 * causal = 0 it is the non-causal block attention of the Wan path
 * (videogen/src/lastkv/videogen/attention.py:9-32).
 *   q / out      bf16 [total_q, num_q_heads, head_dim] rows (16-byte aligned)
 *   cu_seqlens_q int32 [batch + 1] query offsets; max_q >= every span length
 *   seq_k        int32 [batch] keys per sequence (>= its span when causal);
 *                query i of a span of Lq attends keys [0, seq_k - Lq + i]
 *   out_scale    fp32 [num_q_heads] or NULL (folds s_l)
 *   lse          fp32 [total_q, num_q_heads] natural log, or NULL
 *   error_word   device int32[4] (required) for device-side failures.
 * Pool slots past a sequence's end inside its last page must hold finite
 * values (pools are zero-initialised).  head_dim 64 or 128; GQA group in
 * {1, 2, 4, 8}. */
int lkv_prefill_paged(const void* q, int64_t q_stride_tok,
                      const void* pool_k, const void* pool_v, int64_t num_pages,
                      const int32_t* block_table, int64_t block_table_stride,
                      const int32_t* seq_k, const int32_t* cu_seqlens_q,
                      void* out, int64_t out_stride_tok, float* lse, const float* out_scale,
                      int batch, int total_q, int max_q, int num_q_heads, int num_kv_heads,
                      int head_dim, int max_pages_per_seq, int causal, float softmax_scale,
                      int32_t* error_word, void* stream);

/* Non-causal lkv_prefill_paged with the keys split `kv_splits` ways inside one
 * launch (block attention over a long shared history: Wan's
 * videogen/src/lastkv/videogen/attention.py:9-32, non-causal SDPA over
 * [prefix | shared | blended previous block | block]).  With one CTA per SM a
 * grid of C CTAs takes ceil(C / SMs) waves; S * C CTAs of 1/S the keys fill
 * the last wave better.  Each split writes a normalised fp32 partial and its
 * natural-log LSE, then the call merges them exactly (lkv_merge_partials) into
 * `out` (x out_scale) and `lse`; two launches.  Caller-owned scratch:
 *   partial_o   fp32 [kv_splits][total_q * num_q_heads][head_dim], 16-byte aligned
 *   partial_lse fp32 [kv_splits][total_q * num_q_heads]
 * kv_splits 1..8 (1 = lkv_prefill_paged with causal = 0). */
int lkv_prefill_paged_split(const void* q, int64_t q_stride_tok,
                            const void* pool_k, const void* pool_v, int64_t num_pages,
                            const int32_t* block_table, int64_t block_table_stride,
                            const int32_t* seq_k, const int32_t* cu_seqlens_q,
                            void* out, int64_t out_stride_tok, float* lse, const float* out_scale,
                            int batch, int total_q, int max_q, int num_q_heads, int num_kv_heads,
                            int head_dim, int max_pages_per_seq, float softmax_scale,
                            int kv_splits, float* partial_o, float* partial_lse,
                            int32_t* error_word, void* stream);

/* Key-split count lkv_prefill_paged_split should use for this shape on the
 * current device (1 for causal calls, short key ranges, or grids that already
 * fill their last wave). */
int lkv_prefill_split_plan(int batch, int max_q, int num_q_heads, int num_kv_heads, int head_dim,
                           int max_pages_per_seq, int causal, int* kv_splits);

/* ------------------------------------------------------------------ merge
 * Exact log-sum-exp merge of `num_parts` attention partials over disjoint key
 * sets (flashinfer cascade.merge_state / vLLM merge_attn_states, used at
 * flashinfer_executor.py:185-231 and fastpath.py:719):
 *   o_parts   fp32, part p at o_parts + p * o_part_stride: [rows, head_dim]
 *             (normalised partial outputs)
 *   lse_parts fp32, part p at lse_parts + p * lse_part_stride: [rows]
 *             (natural log, -inf = empty)
 *   out       bf16 [rows, head_dim] = out_scale[row % num_q_heads] * merged
 *   lse_out   fp32 [rows] (optional)
 * rows = tokens * num_q_heads; strides in elements, 0 = packed (rows * head_dim,
 * rows), so one all-gathered buffer of [o | lse] parts can be merged in place.
 * out_scale is optional. */
int lkv_merge_partials(const float* o_parts, const float* lse_parts, int num_parts, int64_t rows,
                       int head_dim, int num_q_heads, int64_t o_part_stride, int64_t lse_part_stride,
                       const float* out_scale, void* out, float* lse_out, void* stream);

/* ------------------------------------------------------------------ append
 * Fused cache-append epilogue of one layer; replaces _fused_qkv_kernel
 * (vllm/.../rmarin_flashinfer/fused_qkv.py:58-126, called at fastpath.py:635-642)
 * and the HF per-layer RoPE + q/k norm + cache append
 * (llm/src/lastkv/llm/modeling.py:103-108).  For every token t:
 *   q_out[t, h]       = RMSNorm(RoPE(q[t, h]))       (norm after RoPE)
 *   ring_k[slot_t, j] = RMSNorm(RoPE(k[t, j]))
 *   ring_v[slot_t, j] = bf16(v[t, j] * inv_scale[j])  (rings hold V / s_l)
 *   and, when src_slot != NULL (the top layer), src_k / src_v at src_slot[t]
 *   receive the normalised k and the raw v (the shared history).
 * q [T, *] row stride q_row, k/v likewise (bf16); positions int64 [T];
 * cos_sin bf16 [max_position, head_dim] = cos | sin halves (NeoX, full head);
 * q_weight / k_weight bf16 [head_dim]; inv_scale fp32 [num_kv_heads] or NULL;
 * cos_sin == NULL skips RoPE (use_nope) and q_weight == k_weight == NULL skips
 * the RMSNorm (use_qk_norm = False), as the reference's config switches allow;
 * ring_k/ring_v/src_k/src_v are flat token views [slots, num_kv_heads, head_dim]
 * of the page pool (slot = page * 16 + row).  Out-of-range positions or slots
 * are skipped and recorded in `error_word` (int32[4], may be NULL). */
#define LKV_ROPE_INTERLEAVED 1 /* rotary pairs (2i, 2i+1) (GPT-J / Wan) instead of (i, i + D/2) */
#define LKV_ROPE_TABLE_FP32 2  /* cos_sin is fp32 (e.g. per-token 3-D tables) instead of bf16 */
/* Every tensor fp32 (q, k, v, q_out, pools, q_weight / k_weight, cos_sin): the
 * reference's fp32 configuration (modeling.py:103-108 in fp32).  RoPE is then
 * q*cos + rotate_half(q)*sin with two rounded products and a rounded sum, and
 * RMSNorm w * (x * (1 / sqrt(mean(x^2) + eps))), as the fp32 torch modules. */
#define LKV_APPEND_FP32 4

int lkv_rope_norm_append(const void* q, int64_t q_row, const void* k, int64_t k_row,
                         const void* v, int64_t v_row, const int64_t* positions,
                         const void* cos_sin, int64_t cos_sin_row, int64_t max_position,
                         const void* q_weight, const void* k_weight, float eps,
                         const float* inv_scale, void* q_out, int64_t q_out_row,
                         const int64_t* ring_slot, void* ring_k, void* ring_v, int64_t ring_slots,
                         const int64_t* src_slot, void* src_k, void* src_v, int64_t src_slots,
                         int num_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                         int flags, int32_t* error_word, void* stream);

/* The append of one layer together with the boundary commit of the chunks
 * that the previous step finished, in one launch (the commit the reference
 * runs lazily when the next step starts, batching.py:1099-1144, with the
 * blend_chunk_ arithmetic of fused_qkv.py:158-201; lkv_blend_chunk below
 * gives its exact form).  The append arguments are lkv_rope_norm_append's
 * (bf16 only); then the commit of lkv_blend_chunk over rows
 * [0, num_commit_rows) of raw_pages / ring_pages [num_commit_rows,
 * pages_per_chunk], or over rows [0, *commit_count) when commit_count (device
 * int32) is not NULL - so one captured launch serves steps with and without
 * a boundary (a count above num_commit_rows or below 0 commits nothing and is
 * recorded in error_word).  commit_blocks = the launch's blocks for the commit,
 * which stride over the (page, row, layer) items; 0 = one block per item when
 * commit_count is NULL, else one wave of 8 per SM.
 * Call it for the first layer of the step after the boundary: every layer's
 * attention over the unblended chunk has run, and the append writes the other
 * half of each 2C ring, so no address is both read and written by the launch.
 * It rewrites pages of every layer's ring as a PDL launch: the decodes of that
 * step must not pass LKV_DECODE_TABLES_READY (their pages would no longer
 * predate the last non-PDL operation). */
int lkv_rope_norm_append_commit(const void* q, int64_t q_row, const void* k, int64_t k_row,
                                const void* v, int64_t v_row, const int64_t* positions,
                                const void* cos_sin, int64_t cos_sin_row, int64_t max_position,
                                const void* q_weight, const void* k_weight, float eps,
                                const float* inv_scale, void* q_out, int64_t q_out_row,
                                const int64_t* ring_slot, void* ring_k, void* ring_v, int64_t ring_slots,
                                const int64_t* src_slot, void* src_k, void* src_v, int64_t src_slots,
                                int num_tokens, int num_q_heads, int num_kv_heads, int head_dim, int flags,
                                void* pool_k, void* pool_v, int64_t num_pages,
                                const int32_t* raw_pages, const int32_t* ring_pages,
                                int64_t ring_layer_stride_pages, const float* alpha, int num_layers,
                                int num_commit_rows, int pages_per_chunk, const int32_t* commit_count,
                                int commit_blocks, int32_t* error_word, void* stream);

/* ------------------------------------------------------------------ fp32 attention
 * The merged attention call for fp32 models (the reference's fp32
 * configuration: LastKVAttention.forward's SDPA over fp32 history,
 * llm/src/lastkv/llm/modeling.py:109-146, with the s_l of _scale folded into
 * out_scale as in lkv_decode_paged).  Decode (one token per sequence) and
 * chunked-prefill spans alike: query i of a span of Lq sees keys
 * [0, seq_k - Lq + i] when causal (bottom-right), all seq_k keys otherwise.
 * All tensors fp32 with the bf16 path's layouts: q / out [total_q, Hq, D] rows,
 * pools [num_pages, 16, Hkv, D] (16-byte aligned), block_table int32 [batch,
 * >= max_pages_per_seq], seq_k int32 [batch], cu_seqlens_q int32 [batch + 1],
 * out_scale fp32 [Hq] or NULL, lse fp32 [total_q, Hq] (natural log) or NULL,
 * error_word (required) device int32[4].  Pages outside the pool are skipped
 * and recorded.  head_dim 64 or 128, any GQA group.  One launch (PDL). */
int lkv_attention_paged_f32(const void* q, int64_t q_stride_tok,
                            const void* pool_k, const void* pool_v, int64_t num_pages,
                            const int32_t* block_table, int64_t block_table_stride,
                            const int32_t* seq_k, const int32_t* cu_seqlens_q,
                            void* out, int64_t out_stride_tok, float* lse, const float* out_scale,
                            int batch, int total_q, int num_q_heads, int num_kv_heads, int head_dim,
                            int max_pages_per_seq, int causal, float softmax_scale,
                            int32_t* error_word, void* stream);

/* ------------------------------------------------------------------ gather / blend
 * Token-level commit for histories whose segments do not start on page
 * boundaries (the Wan block cache: per-layer first-frame prefix, previous
 * block blended with the shared final-layer history,
 * videogen/src/lastkv/videogen/model.py:173-195, 217-272, 716-729).  For every
 * token i (flat pool slots = page * 16 + row), on K and V:
 *   src_b[i] <  0 : dst = a          (copy)
 *   src_a[i] <  0 : dst = b          (copy)
 *   otherwise     : dst = bf16(bf16(x*a) + bf16(bf16(1-x)*b)),  x = alpha[alpha_row[i], head]
 * with a = source (shared final layer) and b = the layer's own K/V.  dst slots
 * must not overlap any source slot of the same call. */
int lkv_gather_blend(void* pool_k, void* pool_v, int64_t num_slots, const int64_t* dst_slot,
                     const int64_t* src_a_slot, const int64_t* src_b_slot, const int32_t* alpha_row,
                     const float* alpha, int num_tokens, int num_kv_heads, int head_dim,
                     int32_t* error_word, void* stream);

/* ------------------------------------------------------------------ blend
 * Chunk-boundary commit; replaces blend_chunk_ / _commit_previous_boundary
 * (fused_qkv.py:158-201, batching.py:1099-1144).  For every layer l, sequence
 * s and page j of the finished chunk:
 *   ring = bf16(bf16(a*raw) + bf16(bf16(1-a)*ring)),  a = alpha[l, head]
 * on K and V (rings hold V / s_l, the shared pages raw V).
 * raw_pages int32 [num_seqs, pages_per_chunk]: shared pages of the chunk;
 * ring_pages int32 [num_seqs, pages_per_chunk]: layer-0 ring pages; layer l
 * uses ring_pages + l * ring_layer_stride_pages.  alpha fp32 [num_layers,
 * num_kv_heads] holding bf16-exact sigmoid values. */
int lkv_blend_chunk(void* pool_k, void* pool_v, int64_t num_pages,
                    const int32_t* raw_pages, const int32_t* ring_pages, int64_t ring_layer_stride_pages,
                    const float* alpha, int num_layers, int num_seqs, int pages_per_chunk,
                    int num_kv_heads, int head_dim, int32_t* error_word, void* stream);
/* The same commit on fp32 pools (the reference's fp32 configuration): ring =
 * a*raw + (1-a)*ring in fp32, a*raw and (1-a)*ring each rounded, then their
 * sum (modeling.py:115-119); alpha fp32 [num_layers, num_kv_heads] holding the
 * fp32 sigmoid of the logits. */
int lkv_blend_chunk_f32(void* pool_k, void* pool_v, int64_t num_pages,
                        const int32_t* raw_pages, const int32_t* ring_pages, int64_t ring_layer_stride_pages,
                        const float* alpha, int num_layers, int num_seqs, int pages_per_chunk,
                        int num_kv_heads, int head_dim, int32_t* error_word, void* stream);

/* ------------------------------------------------------------------ block tables
 * Per-layer block tables of the merged pool (fastpath.py:422-424):
 *   bt_all[l, b, c] = block_table[b, c]                 for c <  nsrc[b]
 *                   = block_table[b, c] + ring_base[l]  for c >= nsrc[b]
 * block_table holds older shared pages then layer-relative ring pages. */
int lkv_build_layer_block_tables(const int32_t* block_table, int64_t block_table_stride,
                                 const int32_t* nsrc, const int32_t* ring_base,
                                 int num_layers, int batch, int width, int32_t* bt_all, void* stream);

/* ------------------------------------------------------------------ dense epilogues
 * The decoder layer's residual-add + RMSNorm and SiLU-and-mul in one launch
 * each, with the eager modules' bf16 rounding points (modeling.py decoder
 * layer; the vLLM model's fused_add_rms_norm / silu_and_mul pair,
 * vllm/src/lastkv/vllm/vllm_model.py:756-789).  All tensors bf16 rows, row
 * strides in elements (multiples of 8), 16-byte aligned.
 *
 * lkv_rmsnorm: if residual != NULL, h = bf16(x + residual) is written to
 * residual_out (may alias residual or x), else h = x; then
 *   out = bf16(weight * bf16(h * rsqrt(mean(h^2) + eps)))   (fp32 accumulation)
 * hidden <= 8192, a multiple of 8.
 *
 * lkv_silu_mul: gate_up rows hold [gate (ffn) | up (ffn)];
 *   out = bf16(bf16(silu(gate)) * up). */
int lkv_rmsnorm(const void* x, int64_t x_row, const void* residual, int64_t residual_row,
                void* residual_out, int64_t residual_out_row, const void* weight,
                void* out, int64_t out_row, int rows, int hidden, float eps, void* stream);
int lkv_silu_mul(const void* gate_up, int64_t gate_up_row, void* out, int64_t out_row,
                 int64_t rows, int ffn, void* stream);

/* Greedy token choice: out[r] = index of the largest bf16 logit of row r, the
 * first such index on ties and NaN counted as largest (torch.argmax order);
 * x 16-byte aligned, row_stride (elements) a multiple of 8; one launch. */
int lkv_argmax_rows(const void* x, int64_t row_stride, int rows, int cols, int64_t* out, void* stream);

/* ------------------------------------------------------------------ decode GEMM
 * y[m, n] = sum_k x[m, k] * w[n, k] for 1 <= m <= 16 activation rows (one decode
 * token per sequence) and a bf16 weight w [n_rows, k] in the nn.Linear layout:
 * the projections around the shared-KV attention at decode batch sizes (the
 * reference's q/k/v, o, gate/up and down projections, modeling.py decoder
 * layer; vLLM's QKVParallelLinear / MergedColumnParallelLinear in its model).
 * tcgen05 with the weight rows as the MMA's M side; fp32 accumulation; split-K
 * partials are reduced inside a thread-block cluster in a fixed order
 * (deterministic).  No workspace; one launch; capturable in CUDA graphs.
 *   LKV_GEMM_PLAIN:     y[m, n] = bf16(acc), n < n_rows.
 *   LKV_GEMM_SILU_MUL:  w = [gate (F rows) | up (F rows)], n_rows = 2F;
 *                       y[m, j] = bf16(bf16(silu(bf16(gate))) * bf16(up)), j < F.
 * x and w: 16-byte aligned, row strides (elements) multiples of 8; y row stride
 * >= the output width.  *splits (optional) receives the split-K factor. */
#define LKV_GEMM_PLAIN 0
#define LKV_GEMM_SILU_MUL 1
/* The launch this device will use: weight tiles, split-K factor, CTAs per SM. */
int lkv_decode_gemm_plan(int64_t n_rows, int64_t k, int mode, int* tiles, int* splits, int* ctas_per_sm);
int lkv_decode_gemm(const void* x, int64_t x_row, const void* w, int64_t w_row, void* y, int64_t y_row,
                    int m, int64_t n_rows, int64_t k, int mode, int32_t* error_word, int* splits,
                    void* stream);

/* ------------------------------------------------------------------ context-parallel combine
 * Exchange + LSE merge of sequence-sharded decode partials over NVLink peer
 * memory, replacing the all-gather of the partials and lkv_merge_partials for
 * the 128K-context path (the two-partial merge_state of
 * flashinfer_executor.py:185-231 applied to `world` ranks; the reference
 * itself enforces CP = 1, runtime_contract.py:124-133).
 * send: this rank's partial packed as o fp32 [rows, head_dim] (normalised) |
 * lse fp32 [rows] (natural log), send_floats floats (lkv_cp_combine_sizes).
 * peer_recv[r] (a HOST array of `world` device addresses valid on this GPU):
 * rank r's receive buffer of recv_words 8-byte words, zero before the first
 * call.  Each value travels as one {value, epoch} word, so no fence or flag is
 * needed.  state: 2 uint32 of device memory per rank (8-byte aligned, zero
 * before the first call): the epoch of the previous call and a done counter;
 * each call uses the next epoch, so a call can be captured in a CUDA graph and
 * replayed.  Every rank must make the same sequence of calls (with its own
 * state, advanced identically).  A rank waits at most
 * ~2 s for its peers (then the error word is set and the rows it could not
 * complete hold garbage).  out: bf16 rows (tok = row / hq, head = row % hq)
 * scaled by out_scale[head] (may be NULL). */
int lkv_cp_combine_sizes(int64_t rows, int head_dim, int world, int64_t* send_floats, int64_t* recv_words);

/* Sequence-sharded decode in one call, the exchange fused into the decode:
 * lkv_decode_paged over this rank's slice of every sequence's keys, whose
 * kernel, as each (sequence, KV head) finishes, merges that unit's splits and
 * pushes the merged rows to every rank's receive buffer (the same {value,
 * epoch} words lkv_cp_combine pushes, so the transfer overlaps the rest of the
 * decode), then the `world` ranks' rows are polled and merged in rank order
 * into `out` (x out_scale).  When no CTA of the decode's persistent grid takes
 * more than 32 work items (every shape of the 128K configuration), that poll
 * and merge runs inside the decode kernel itself: the CTA that pushed a
 * (sequence, KV head) unit, once its own items are done, polls that unit's rows
 * from every rank and writes them - one launch per call.  Otherwise a
 * lkv_cp_combine launch with send = NULL does it - two launches.  No merge
 * launch and no collective call either way; the result equals
 * lkv_decode_paged (partial) + all-gather + lkv_merge_partials bit for bit.  peer_recv / recv sizes as for
 * lkv_cp_combine (rows = batch * num_q_heads); `workspace` as for
 * lkv_decode_paged; state: lkv_decode_cp_state_words uint32 of device memory
 * (8-byte aligned, zero before the first call; every completed call leaves it
 * ready for the next; zero it again after a call reports a device error).
 * flags as for lkv_decode_paged. */
int lkv_decode_cp_state_words(int batch, int num_kv_heads, int64_t* state_words);
int lkv_decode_paged_cp(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v,
                        int64_t num_pages, const int32_t* block_table, int64_t block_table_stride,
                        const int32_t* seq_k, void* out, int64_t out_stride_tok, const float* out_scale,
                        int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_pages_per_seq,
                        float softmax_scale, void* workspace, size_t workspace_bytes,
                        const uint64_t* peer_recv, int rank, int world, uint32_t* state,
                        int32_t* error_word, int flags, void* stream);
/* send may be NULL when this rank's rows were already pushed into every receive
 * buffer (lkv_decode_paged_cp's decode kernel); the call then only polls and merges. */
int lkv_cp_combine(const float* send, const uint64_t* peer_recv, int rank, int world, uint32_t* state,
                   int64_t rows, int head_dim, int hq, const float* out_scale, void* out,
                   int64_t out_stride_tok, int32_t* error_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LASTKV_B200_H */
