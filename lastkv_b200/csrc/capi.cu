// extern "C" entry points of liblastkv_b200.so (declared in include/lastkv_b200.h)
// and the host-side TMA tensor-map encoder.  The driver entry point is looked
// up through the runtime so the library does not link libcuda directly.

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "kernels.h"
#include "lastkv_b200.h"
#include "launch.cuh"

namespace lkv {

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("LKV_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// 4-D map over the pool [num_pages, 16, Hkv, D] (innermost first: D, Hkv, 16,
// pages), copying one (page, kv head, 64-wide half of D) tile of 16 rows x
// 128 bytes per load, 128-byte swizzled so ldmatrix reads are bank-conflict free.
int make_pool_tensor_map(CUtensorMap* map, const void* pool, int64_t num_pages, int num_kv_heads, int head_dim) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LKV_ERR_TENSOR_MAP;
  if (reinterpret_cast<uintptr_t>(pool) & 15) return LKV_ERR_INVALID_ARGUMENT;
  if (num_pages < 1 || num_pages > (int64_t)0xffffffffLL || num_kv_heads < 1 || num_kv_heads > 256)
    return LKV_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[4] = {(cuuint64_t)head_dim, (cuuint64_t)num_kv_heads, 16, (cuuint64_t)num_pages};
  cuuint64_t strides[3] = {(cuuint64_t)head_dim * 2, (cuuint64_t)num_kv_heads * head_dim * 2,
                           (cuuint64_t)16 * num_kv_heads * head_dim * 2};
  cuuint32_t box[4] = {64, 1, 16, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(pool), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LKV_OK : LKV_ERR_TENSOR_MAP;
}

// 3-D map over q [total_q, Hq, D] (innermost first: D, Hq, tokens), copying a
// (64-wide half of D) x GROUP heads x (128 / GROUP) tokens box: 128 rows of
// 128 bytes, row = token * GROUP + head, 128-byte swizzled (a K-major UMMA tile).
int make_query_tensor_map(CUtensorMap* map, const void* q, int64_t total_q, int64_t q_stride_tok, int num_q_heads,
                          int head_dim, int group, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LKV_ERR_TENSOR_MAP;
  if ((reinterpret_cast<uintptr_t>(q) & 15) || total_q < 1 || total_q > (int64_t)0x7fffffff) return LKV_ERR_INVALID_ARGUMENT;
  if (q_stride_tok < (int64_t)num_q_heads * head_dim) return LKV_ERR_INVALID_ARGUMENT;
  if (group < 1 || box_rows < group || box_rows > 256 || box_rows % group) return LKV_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)num_q_heads, (cuuint64_t)total_q};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)q_stride_tok * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)(box_rows / group)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LKV_OK : LKV_ERR_TENSOR_MAP;
}

// 2-D map over a row-major bf16 matrix [rows, cols] (row stride in elements),
// copying (box_rows x 64 columns) tiles of 128-byte rows, 128-byte swizzled: a
// K-major UMMA operand tile.  Reads past the matrix fill zeros.
int make_matrix_tensor_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t row_stride,
                           int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LKV_ERR_TENSOR_MAP;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || rows < 1 || cols < 1 || rows > (int64_t)0x7fffffff ||
      cols > (int64_t)0x7fffffff || row_stride < cols || (row_stride * 2) % 16 || box_rows < 1 || box_rows > 256)
    return LKV_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LKV_OK : LKV_ERR_TENSOR_MAP;
}

}  // namespace lkv

extern "C" {

const char* lkv_status_string(int status) {
  switch (status) {
    case LKV_OK: return "ok";
    case LKV_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LKV_ERR_UNSUPPORTED: return "unsupported shape or configuration";
    case LKV_ERR_CUDA: return "CUDA runtime error";
    case LKV_ERR_ARCH: return "device is not an sm_100 GPU";
    case LKV_ERR_TENSOR_MAP: return "TMA tensor map could not be encoded";
    case LKV_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    default: return "unknown status";
  }
}

int lkv_abi_version(void) { return 201; }

int lkv_check_device(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) return LKV_ERR_CUDA;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) return LKV_ERR_CUDA;
  if (major != 10 || minor != 0) return LKV_ERR_ARCH;
  // Load the allocation-free decode's static scratch now (lazy module loading
  // would otherwise commit it at the first lkv_decode_paged_noalloc call, which
  // may come after a KV-cache pool has taken the memory).  Best effort: a
  // failure here is retried, and reported, by that call.
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur == device) (void)lkv::noalloc_scratch_prepare();
  (void)cudaGetLastError();
  return LKV_OK;
}

int lkv_read_error_word(const int32_t* error_word, int32_t host_out[4], void* stream) {
  if (!error_word || !host_out) return LKV_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(host_out, error_word, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return LKV_ERR_CUDA;
  return cudaStreamSynchronize(s) == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

int lkv_clear_error_word(int32_t* error_word, void* stream) {
  if (!error_word) return LKV_ERR_INVALID_ARGUMENT;
  return cudaMemsetAsync(error_word, 0, 4 * sizeof(int32_t), static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? LKV_OK
             : LKV_ERR_CUDA;
}

size_t lkv_decode_workspace_bytes(int batch, int num_q_heads, int head_dim, int max_pages_per_seq) {
  return lkv::decode_workspace_bytes(batch, num_q_heads, head_dim, max_pages_per_seq);
}

int lkv_decode_paged(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v, int64_t num_pages,
                     const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_k, void* out,
                     int64_t out_stride_tok, float* lse, const float* out_scale, float* partial_o,
                     float* partial_lse, int batch, int num_q_heads, int num_kv_heads, int head_dim,
                     int max_pages_per_seq, float softmax_scale, void* workspace, size_t workspace_bytes,
                     int flags, void* stream) {
  lkv::DecodeArgs a{};
  a.q = q;
  a.q_stride_tok = q_stride_tok;
  a.pool_k = pool_k;
  a.pool_v = pool_v;
  a.num_pages = num_pages;
  a.block_table = block_table;
  a.block_table_stride = block_table_stride;
  a.seq_k = seq_k;
  a.out = out;
  a.out_stride_tok = out_stride_tok;
  a.lse = lse;
  a.out_scale = out_scale;
  a.partial_o = partial_o;
  a.partial_lse = partial_lse;
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_pages_per_seq = max_pages_per_seq;
  a.softmax_scale = softmax_scale;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.stream = stream;
  a.flags = flags;
  return lkv::decode_paged(a);
}

int lkv_decode_cp_state_words(int batch, int num_kv_heads, int64_t* state_words) {
  if (batch < 1 || num_kv_heads < 1 || !state_words) return LKV_ERR_INVALID_ARGUMENT;
  *state_words = 2 + (int64_t)batch * num_kv_heads;
  return LKV_OK;
}

int lkv_decode_paged_cp(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v, int64_t num_pages,
                        const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_k, void* out,
                        int64_t out_stride_tok, const float* out_scale, int batch, int num_q_heads, int num_kv_heads,
                        int head_dim, int max_pages_per_seq, float softmax_scale, void* workspace,
                        size_t workspace_bytes, const uint64_t* peer_recv, int rank, int world, uint32_t* state,
                        int32_t* error_word, int flags, void* stream) {
  lkv::DecodeArgs a{};
  a.q = q;
  a.q_stride_tok = q_stride_tok;
  a.pool_k = pool_k;
  a.pool_v = pool_v;
  a.num_pages = num_pages;
  a.block_table = block_table;
  a.block_table_stride = block_table_stride;
  a.seq_k = seq_k;
  a.out = out;
  a.out_stride_tok = out_stride_tok;
  a.out_scale = out_scale;
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_pages_per_seq = max_pages_per_seq;
  a.softmax_scale = softmax_scale;
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  a.stream = stream;
  a.cp_recv = peer_recv;
  a.cp_rank = rank;
  a.cp_world = world;
  a.cp_state = state;
  a.cp_error = error_word;
  a.flags = flags;
  return lkv::decode_paged_cp(a);
}

int lkv_decode_plan(int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_pages_per_seq,
                    size_t workspace_bytes, int partial, int* num_splits, int* num_launches) {
  return lkv::decode_plan(batch, num_q_heads, num_kv_heads, head_dim, max_pages_per_seq, workspace_bytes, partial,
                          num_splits, num_launches);
}

int lkv_merge_partials(const float* o_parts, const float* lse_parts, int num_parts, int64_t rows, int head_dim,
                       int num_q_heads, int64_t o_part_stride, int64_t lse_part_stride, const float* out_scale,
                       void* out, float* lse_out, void* stream) {
  return lkv::merge_partials(o_parts, lse_parts, num_parts, rows, head_dim, num_q_heads, o_part_stride,
                             lse_part_stride, out_scale, out, lse_out, static_cast<cudaStream_t>(stream));
}

#define LKV_APPEND_PARAMS                                                                                     \
  const void *q, int64_t q_row, const void *k, int64_t k_row, const void *v, int64_t v_row,                    \
      const int64_t *positions, const void *cos_sin, int64_t cos_sin_row, int64_t max_position,                \
      const void *q_weight, const void *k_weight, float eps, const float *inv_scale, void *q_out,              \
      int64_t q_out_row, const int64_t *ring_slot, void *ring_k, void *ring_v, int64_t ring_slots,             \
      const int64_t *src_slot, void *src_k, void *src_v, int64_t src_slots, int num_tokens, int num_q_heads,   \
      int num_kv_heads, int head_dim, int flags
#define LKV_APPEND_ARGS                                                                                         \
  q, q_row, k, k_row, v, v_row, positions, cos_sin, cos_sin_row, max_position, q_weight, k_weight, eps,        \
      inv_scale, q_out, q_out_row, ring_slot, ring_k, ring_v, ring_slots, src_slot, src_k, src_v, src_slots,   \
      num_tokens, num_q_heads, num_kv_heads, head_dim, flags

static lkv::AppendArgs append_args(LKV_APPEND_PARAMS, int32_t* error_word, void* stream) {
  lkv::AppendArgs a{};
  a.q = q;
  a.q_row = q_row;
  a.k = k;
  a.k_row = k_row;
  a.v = v;
  a.v_row = v_row;
  a.positions = positions;
  a.cos_sin = cos_sin;
  a.cos_sin_row = cos_sin_row;
  a.max_position = max_position;
  a.q_weight = q_weight;
  a.k_weight = k_weight;
  a.eps = eps;
  a.inv_scale = inv_scale;
  a.q_out = q_out;
  a.q_out_row = q_out_row;
  a.ring_slot = ring_slot;
  a.ring_k = ring_k;
  a.ring_v = ring_v;
  a.ring_slots = ring_slots;
  a.src_slot = src_slot;
  a.src_k = src_k;
  a.src_v = src_v;
  a.src_slots = src_slots;
  a.num_tokens = num_tokens;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.flags = flags;
  a.error_word = error_word;
  a.stream = stream;
  return a;
}

static lkv::BlendArgs blend_args(void* pool_k, void* pool_v, int64_t num_pages, const int32_t* raw_pages,
                                 const int32_t* ring_pages, int64_t ring_layer_stride_pages, const float* alpha,
                                 int num_layers, int num_seqs, int pages_per_chunk, int num_kv_heads, int head_dim,
                                 int32_t* error_word, void* stream) {
  lkv::BlendArgs a{};
  a.pool_k = pool_k;
  a.pool_v = pool_v;
  a.num_pages = num_pages;
  a.raw_pages = raw_pages;
  a.ring_pages = ring_pages;
  a.ring_layer_stride_pages = ring_layer_stride_pages;
  a.alpha = alpha;
  a.num_layers = num_layers;
  a.num_seqs = num_seqs;
  a.pages_per_chunk = pages_per_chunk;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.error_word = error_word;
  a.stream = stream;
  return a;
}

int lkv_rope_norm_append(LKV_APPEND_PARAMS, int32_t* error_word, void* stream) {
  return lkv::rope_norm_append(append_args(LKV_APPEND_ARGS, error_word, stream));
}

int lkv_rope_norm_append_commit(LKV_APPEND_PARAMS, void* pool_k, void* pool_v, int64_t num_pages,
                                const int32_t* raw_pages, const int32_t* ring_pages, int64_t ring_layer_stride_pages,
                                const float* alpha, int num_layers, int num_commit_rows, int pages_per_chunk,
                                const int32_t* commit_count, int commit_blocks, int32_t* error_word, void* stream) {
  return lkv::rope_norm_append_commit(
      append_args(LKV_APPEND_ARGS, error_word, stream),
      blend_args(pool_k, pool_v, num_pages, raw_pages, ring_pages, ring_layer_stride_pages, alpha, num_layers,
                 num_commit_rows, pages_per_chunk, num_kv_heads, head_dim, error_word, stream),
      commit_count, commit_blocks);
}

int lkv_gather_blend(void* pool_k, void* pool_v, int64_t num_slots, const int64_t* dst_slot,
                     const int64_t* src_a_slot, const int64_t* src_b_slot, const int32_t* alpha_row,
                     const float* alpha, int num_tokens, int num_kv_heads, int head_dim, int32_t* error_word,
                     void* stream) {
  return lkv::gather_blend(pool_k, pool_v, num_slots, dst_slot, src_a_slot, src_b_slot, alpha_row, alpha,
                           num_tokens, num_kv_heads, head_dim, error_word, static_cast<cudaStream_t>(stream));
}

int lkv_blend_chunk(void* pool_k, void* pool_v, int64_t num_pages, const int32_t* raw_pages,
                    const int32_t* ring_pages, int64_t ring_layer_stride_pages, const float* alpha, int num_layers,
                    int num_seqs, int pages_per_chunk, int num_kv_heads, int head_dim, int32_t* error_word,
                    void* stream) {
  return lkv::blend_chunk(blend_args(pool_k, pool_v, num_pages, raw_pages, ring_pages, ring_layer_stride_pages, alpha,
                                     num_layers, num_seqs, pages_per_chunk, num_kv_heads, head_dim, error_word,
                                     stream));
}

int lkv_blend_chunk_f32(void* pool_k, void* pool_v, int64_t num_pages, const int32_t* raw_pages,
                        const int32_t* ring_pages, int64_t ring_layer_stride_pages, const float* alpha,
                        int num_layers, int num_seqs, int pages_per_chunk, int num_kv_heads, int head_dim,
                        int32_t* error_word, void* stream) {
  return lkv::blend_chunk_f32(blend_args(pool_k, pool_v, num_pages, raw_pages, ring_pages, ring_layer_stride_pages,
                                         alpha, num_layers, num_seqs, pages_per_chunk, num_kv_heads, head_dim,
                                         error_word, stream));
}

int lkv_attention_paged_f32(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v,
                            int64_t num_pages, const int32_t* block_table, int64_t block_table_stride,
                            const int32_t* seq_k, const int32_t* cu_seqlens_q, void* out, int64_t out_stride_tok,
                            float* lse, const float* out_scale, int batch, int total_q, int num_q_heads,
                            int num_kv_heads, int head_dim, int max_pages_per_seq, int causal, float softmax_scale,
                            int32_t* error_word, void* stream) {
  lkv::AttnF32Args a{};
  a.q = q;
  a.q_stride_tok = q_stride_tok;
  a.pool_k = pool_k;
  a.pool_v = pool_v;
  a.num_pages = num_pages;
  a.block_table = block_table;
  a.block_table_stride = block_table_stride;
  a.seq_k = seq_k;
  a.cu_seqlens_q = cu_seqlens_q;
  a.out = out;
  a.out_stride_tok = out_stride_tok;
  a.lse = lse;
  a.out_scale = out_scale;
  a.batch = batch;
  a.total_q = total_q;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_pages_per_seq = max_pages_per_seq;
  a.causal = causal;
  a.softmax_scale = softmax_scale;
  a.error_word = error_word;
  a.stream = stream;
  return lkv::attention_f32(a);
}

int lkv_prefill_paged(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v,
                      int64_t num_pages, const int32_t* block_table, int64_t block_table_stride,
                      const int32_t* seq_k, const int32_t* cu_seqlens_q, void* out, int64_t out_stride_tok,
                      float* lse, const float* out_scale, int batch, int total_q, int max_q, int num_q_heads,
                      int num_kv_heads, int head_dim, int max_pages_per_seq, int causal, float softmax_scale,
                      int32_t* error_word, void* stream) {
  lkv::PrefillArgs a{};
  a.q = q;
  a.q_stride_tok = q_stride_tok;
  a.pool_k = pool_k;
  a.pool_v = pool_v;
  a.num_pages = num_pages;
  a.block_table = block_table;
  a.block_table_stride = block_table_stride;
  a.seq_k = seq_k;
  a.cu_q = cu_seqlens_q;
  a.out = out;
  a.out_stride_tok = out_stride_tok;
  a.lse = lse;
  a.out_scale = out_scale;
  a.batch = batch;
  a.total_q = total_q;
  a.max_q = max_q;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_pages_per_seq = max_pages_per_seq;
  a.causal = causal;
  a.softmax_scale = softmax_scale;
  a.error_word = error_word;
  a.stream = stream;
  return lkv::prefill_paged(a);
}

int lkv_prefill_split_plan(int batch, int max_q, int num_q_heads, int num_kv_heads, int head_dim,
                           int max_pages_per_seq, int causal, int* kv_splits) {
  return lkv::prefill_split_plan(batch, max_q, num_q_heads, num_kv_heads, head_dim, max_pages_per_seq, causal,
                                 kv_splits);
}

int lkv_prefill_paged_split(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v,
                            int64_t num_pages, const int32_t* block_table, int64_t block_table_stride,
                            const int32_t* seq_k, const int32_t* cu_seqlens_q, void* out, int64_t out_stride_tok,
                            float* lse, const float* out_scale, int batch, int total_q, int max_q, int num_q_heads,
                            int num_kv_heads, int head_dim, int max_pages_per_seq, float softmax_scale,
                            int kv_splits, float* partial_o, float* partial_lse, int32_t* error_word,
                            void* stream) {
  lkv::PrefillArgs a{};
  a.q = q;
  a.q_stride_tok = q_stride_tok;
  a.pool_k = pool_k;
  a.pool_v = pool_v;
  a.num_pages = num_pages;
  a.block_table = block_table;
  a.block_table_stride = block_table_stride;
  a.seq_k = seq_k;
  a.cu_q = cu_seqlens_q;
  a.out = out;
  a.out_stride_tok = out_stride_tok;
  a.lse = lse;
  a.out_scale = out_scale;
  a.batch = batch;
  a.total_q = total_q;
  a.max_q = max_q;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_pages_per_seq = max_pages_per_seq;
  a.causal = 0;
  a.softmax_scale = softmax_scale;
  a.error_word = error_word;
  a.stream = stream;
  a.kv_splits = kv_splits;
  a.part_o = partial_o;
  a.part_lse = partial_lse;
  return lkv::prefill_paged(a);
}

int lkv_build_layer_block_tables(const int32_t* block_table, int64_t block_table_stride, const int32_t* nsrc,
                                 const int32_t* ring_base, int num_layers, int batch, int width, int32_t* bt_all,
                                 void* stream) {
  return lkv::build_layer_block_tables(block_table, block_table_stride, nsrc, ring_base, num_layers, batch, width,
                                       bt_all, static_cast<cudaStream_t>(stream));
}

int lkv_rmsnorm(const void* x, int64_t x_row, const void* residual, int64_t residual_row, void* residual_out,
                int64_t residual_out_row, const void* weight, void* out, int64_t out_row, int rows, int hidden,
                float eps, void* stream) {
  return lkv::rmsnorm(x, x_row, residual, residual_row, residual_out, residual_out_row, weight, out, out_row, rows,
                      hidden, eps, static_cast<cudaStream_t>(stream));
}

int lkv_silu_mul(const void* gate_up, int64_t gate_up_row, void* out, int64_t out_row, int64_t rows, int ffn,
                 void* stream) {
  return lkv::silu_mul(gate_up, gate_up_row, out, out_row, rows, ffn, static_cast<cudaStream_t>(stream));
}

int lkv_decode_gemm_plan(int64_t n_rows, int64_t k, int mode, int* tiles, int* splits, int* ctas_per_sm) {
  return lkv::decode_gemm_plan(n_rows, k, mode, tiles, splits, ctas_per_sm);
}

int lkv_decode_gemm(const void* x, int64_t x_row, const void* w, int64_t w_row, void* y, int64_t y_row, int m,
                    int64_t n_rows, int64_t k, int mode, int32_t* error_word, int* splits, void* stream) {
  return lkv::decode_gemm(x, x_row, w, w_row, y, y_row, m, n_rows, k, mode, error_word,
                          static_cast<cudaStream_t>(stream), splits);
}

int lkv_argmax_rows(const void* x, int64_t row_stride, int rows, int cols, int64_t* out, void* stream) {
  return lkv::argmax_rows(x, row_stride, rows, cols, out, static_cast<cudaStream_t>(stream));
}

int lkv_cp_combine_sizes(int64_t rows, int head_dim, int world, int64_t* send_floats, int64_t* recv_words) {
  if (rows < 1 || head_dim < 1 || world < 1 || world > lkv::kCpMaxRanks) return LKV_ERR_INVALID_ARGUMENT;
  if (send_floats) *send_floats = (rows * (head_dim + 1) + 3) / 4 * 4;
  if (recv_words) *recv_words = 2 * (int64_t)world * lkv::cp_part_words(rows, head_dim);
  return LKV_OK;
}

int lkv_cp_combine(const float* send, const uint64_t* peer_recv, int rank, int world, uint32_t* state, int64_t rows,
                   int head_dim, int hq, const float* out_scale, void* out, int64_t out_stride_tok,
                   int32_t* error_word, void* stream) {
  return lkv::cp_combine(send, peer_recv, rank, world, state, rows, head_dim, hq, out_scale, out, out_stride_tok,
                         error_word, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
