// Internal launch interface between the C ABI (capi.cu) and the kernel files.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lkv {

// Bytes reserved at the start of every workspace: the int32[4] error word,
// padded so the partial buffers after it stay 256-byte aligned.
constexpr size_t kWorkspaceHeader = 256;

int make_pool_tensor_map(CUtensorMap* map, const void* pool, int64_t num_pages, int num_kv_heads, int head_dim);
int make_matrix_tensor_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride,
                           int box_rows);
// box_rows: query rows (tokens x group heads) per copy - a 128-row tile, or a
// warp's 32 rows for the output stores.
int make_query_tensor_map(CUtensorMap* map, const void* q, int64_t total_q, int64_t q_stride_tok, int num_q_heads,
                          int head_dim, int group, int box_rows = 128);

struct PrefillArgs {
  const void* q;
  int64_t q_stride_tok;
  const void* pool_k;
  const void* pool_v;
  int64_t num_pages;
  const int32_t* block_table;
  int64_t block_table_stride;
  const int32_t* seq_k;
  const int32_t* cu_q;
  void* out;
  int64_t out_stride_tok;
  float* lse;
  const float* out_scale;
  int batch, total_q, max_q, num_q_heads, num_kv_heads, head_dim, max_pages_per_seq, causal;
  float softmax_scale;
  int32_t* error_word;
  void* stream;
  // key splits (non-causal only): > 1 writes fp32 partials here, then merges into out / lse
  int kv_splits = 1;
  float* part_o = nullptr;    // [kv_splits][total_q * num_q_heads][head_dim]
  float* part_lse = nullptr;  // [kv_splits][total_q * num_q_heads], natural log
};
int prefill_paged(const PrefillArgs& a);
int prefill_split_plan(int batch, int max_q, int num_q_heads, int num_kv_heads, int head_dim, int max_pages,
                       int causal, int* kv_splits);

struct DecodeArgs {
  const void* q;
  int64_t q_stride_tok;
  const void* pool_k;
  const void* pool_v;
  int64_t num_pages;
  const int32_t* block_table;
  int64_t block_table_stride;
  const int32_t* seq_k;
  void* out;
  int64_t out_stride_tok;
  float* lse;
  const float* out_scale;
  float* partial_o;
  float* partial_lse;
  int batch, num_q_heads, num_kv_heads, head_dim, max_pages_per_seq;
  float softmax_scale;
  void* workspace;
  size_t workspace_bytes;
  void* stream;
  int flags = 0;  // LKV_DECODE_TABLES_READY
  // context parallel (decode_paged_cp): every unit's merged partial is pushed to these receive buffers
  const uint64_t* cp_recv = nullptr;  // host array of cp_world device addresses
  int cp_rank = 0, cp_world = 0;
  uint32_t* cp_state = nullptr;       // [0] epoch, [1] combine done counter, [2 + unit] unit arrivals
  int32_t* cp_error = nullptr;
};

size_t decode_split_bytes(int64_t rows, int d);
size_t decode_workspace_bytes(int batch, int hq, int d, int max_pages);
// Loads the allocation-free decode's static scratch on the current device (see
// decode_noalloc.cu); LKV_OK or LKV_ERR_CUDA, with the CUDA error cleared.
int noalloc_scratch_prepare();
int decode_paged(const DecodeArgs& a);
int decode_plan(int batch, int hq, int hkv, int d, int max_pages, size_t workspace_bytes, int partial, int* splits,
                int* launches);
int merge_partials(const float* o_parts, const float* lse_parts, int num_parts, int64_t rows, int head_dim, int hq,
                   int64_t o_part_stride, int64_t lse_part_stride, const float* out_scale, void* out,
                   float* lse_out, cudaStream_t stream, int64_t out_stride_tok = 0);

struct AppendArgs {
  const void* q;
  int64_t q_row;
  const void* k;
  int64_t k_row;
  const void* v;
  int64_t v_row;
  const int64_t* positions;
  const void* cos_sin;
  int64_t cos_sin_row;
  int64_t max_position;
  const void* q_weight;
  const void* k_weight;
  float eps;
  const float* inv_scale;
  void* q_out;
  int64_t q_out_row;
  const int64_t* ring_slot;
  void* ring_k;
  void* ring_v;
  int64_t ring_slots;
  const int64_t* src_slot;
  void* src_k;
  void* src_v;
  int64_t src_slots;
  int num_tokens, num_q_heads, num_kv_heads, head_dim;
  int flags;  // LKV_ROPE_INTERLEAVED | LKV_ROPE_TABLE_FP32
  int32_t* error_word;
  void* stream;
};
int rope_norm_append(const AppendArgs& a);
int rope_norm_append_f32(const AppendArgs& a);  // LKV_APPEND_FP32 (fp32.cu)

struct AttnF32Args {
  const void* q;
  int64_t q_stride_tok;
  const void* pool_k;
  const void* pool_v;
  int64_t num_pages;
  const int32_t* block_table;
  int64_t block_table_stride;
  const int32_t* seq_k;
  const int32_t* cu_seqlens_q;
  void* out;
  int64_t out_stride_tok;
  float* lse;
  const float* out_scale;
  int batch, total_q, num_q_heads, num_kv_heads, head_dim, max_pages_per_seq, causal;
  float softmax_scale;
  int32_t* error_word;
  void* stream;
};
int attention_f32(const AttnF32Args& a);

int gather_blend(void* pool_k, void* pool_v, int64_t num_slots, const int64_t* dst, const int64_t* src_a,
                 const int64_t* src_b, const int32_t* alpha_row, const float* alpha, int num_tokens,
                 int num_kv_heads, int head_dim, int32_t* error_word, cudaStream_t stream);

struct BlendArgs {
  void* pool_k;
  void* pool_v;
  int64_t num_pages;
  const int32_t* raw_pages;
  const int32_t* ring_pages;
  int64_t ring_layer_stride_pages;
  const float* alpha;
  int num_layers, num_seqs, pages_per_chunk, num_kv_heads, head_dim;
  int32_t* error_word;
  void* stream;
};
int blend_chunk(const BlendArgs& a);
// the append and the previous step's boundary commit in one launch (commit_count: device row count or NULL)
int rope_norm_append_commit(const AppendArgs& a, const BlendArgs& b, const int32_t* commit_count, int commit_blocks);
int blend_chunk_f32(const BlendArgs& a);  // fp32 pools (fp32.cu)

int build_layer_block_tables(const int32_t* bt, int64_t bt_stride, const int32_t* nsrc, const int32_t* ring_base,
                             int num_layers, int batch, int width, int32_t* bt_all, cudaStream_t stream);

int rmsnorm(const void* x, int64_t x_row, const void* residual, int64_t residual_row, void* residual_out,
            int64_t residual_out_row, const void* weight, void* out, int64_t out_row, int rows, int hidden, float eps,
            cudaStream_t stream);
int silu_mul(const void* gate_up, int64_t gate_up_row, void* out, int64_t out_row, int64_t rows, int ffn,
             cudaStream_t stream);
int argmax_rows(const void* x, int64_t row_stride, int rows, int cols, int64_t* out, cudaStream_t stream);

constexpr int kCpMaxRanks = 8;
constexpr int kCpRowsPerCta = 4;
// decode + push + combine for sequence-sharded decode (see decode.cu, cp_combine.cu)
int decode_paged_cp(const DecodeArgs& a);
int64_t cp_part_words(int64_t rows, int head_dim);
int cp_combine(const float* send, const uint64_t* peer_recv, int rank, int world, uint32_t* state, int64_t rows,
               int head_dim, int hq, const float* out_scale, void* out, int64_t out_stride_tok, int32_t* error_word,
               cudaStream_t stream);

int decode_gemm_plan(int64_t n_rows, int64_t k, int mode, int* tiles, int* splits, int* ctas_per_sm);
int decode_gemm(const void* x, int64_t x_row, const void* w, int64_t w_row, void* y, int64_t y_row, int m,
                int64_t n_rows, int64_t k, int mode, int32_t* error_word, cudaStream_t stream, int* splits_out);

}  // namespace lkv
