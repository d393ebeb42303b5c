// lkv_decode_paged_noalloc: the split-KV decode for callers that cannot
// allocate device memory.
//
// Who needs it: a serving engine that has already handed (almost) all of HBM
// to its KV-cache pool - vLLM reserves gpu_memory_utilization of the device
// up front, so a later cudaMalloc for a side buffer can fail; hosts that reach
// this library through a plain C FFI and can only pass buffers they already
// own (inputs and outputs), with no allocator of their own to call; and hot
// loops where cudaMalloc/cudaFree would add implicit device synchronisation.
// For them the scratch that lkv_decode_paged takes as a caller-provided
// workspace (the split-KV partials and the int32[4] error word) lives in the
// fixed-size array below, inside the library itself.
//
// Rules of use (also stated in include/lastkv_b200.h):
//  * The array costs LKV_NOALLOC_SCRATCH_BYTES of device memory on a GPU once
//    this file's module is loaded there, for the life of the process.  CUDA
//    loads modules lazily, so that happens at lkv_check_device(d) with d the
//    current device, or else at the first no-alloc call on the device: make
//    one of them before the engine reserves its KV-cache pool, or the module's
//    8 MiB may no longer fit.
//  * The first of those calls on each device looks up the array's device
//    address with that device current (cudaGetSymbolAddress); make it before
//    any CUDA-graph stream capture.  The address is cached per device index
//    for the life of the process: it assumes the device's primary context is
//    never reset (no cudaDeviceReset between calls).
//  * Every call shares the one array.  Calls whose GPU work overlaps (other
//    streams, other host threads, concurrent graph replays) race on it and
//    corrupt each other's results; serialise them.
//  * A call needs batch * num_q_heads * (head_dim + 1) * 4 + 256 bytes for one
//    split's partials after a 256-byte header; larger shapes are rejected with
//    LKV_ERR_WORKSPACE before anything is launched.  Smaller shapes get as many
//    KV splits as fit (at most the same number lkv_decode_paged would choose).
//  * The error word at the start of the array is cleared at the start of each
//    call; pass `error_word` (a device int32[4], may be NULL) to receive a copy
//    of it after the call.
//  * Nothing here calls cudaMalloc, cudaFree or any allocating routine.

#include <cuda_runtime.h>

#include <mutex>

#include "kernels.h"
#include "lastkv_b200.h"

namespace {

static __device__ __align__(256) unsigned char g_decode_scratch[LKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of g_decode_scratch on the current device (looked up once per
// device, with that device current).  In host code the symbol itself is only
// a host-side stand-in and must never be passed to a kernel.
int scratch_address(int dev, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();  // leave no pending error for the caller's next CUDA check
      return LKV_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return LKV_OK;
}

}  // namespace

namespace lkv {

// Called by lkv_check_device for the current device: loads the module (and so
// commits the array) at start-up, before a KV-cache pool takes the memory.
int noalloc_scratch_prepare() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    (void)cudaGetLastError();
    return LKV_ERR_CUDA;
  }
  void* p = nullptr;
  return scratch_address(dev, &p);
}

}  // namespace lkv

extern "C" int lkv_decode_paged_noalloc(const void* q, int64_t q_stride_tok, const void* pool_k, const void* pool_v,
                                        int64_t num_pages, const int32_t* block_table, int64_t block_table_stride,
                                        const int32_t* seq_k, void* out, int64_t out_stride_tok, float* lse,
                                        const float* out_scale, int batch, int num_q_heads, int num_kv_heads,
                                        int head_dim, int max_pages_per_seq, float softmax_scale,
                                        int32_t* error_word, void* stream) {
  if (batch < 0 || num_q_heads < 1 || head_dim < 1) return LKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return LKV_OK;
  const size_t need = lkv::kWorkspaceHeader + (size_t)batch * num_q_heads * (size_t)(head_dim + 1) * sizeof(float) +
                      256;
  if (need > (size_t)LKV_NOALLOC_SCRATCH_BYTES) return LKV_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return LKV_ERR_CUDA;
  void* scratch = nullptr;
  const int st = scratch_address(dev, &scratch);
  if (st != LKV_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, 4 * sizeof(int32_t), s) != cudaSuccess) return LKV_ERR_CUDA;

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
  a.batch = batch;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.head_dim = head_dim;
  a.max_pages_per_seq = max_pages_per_seq;
  a.softmax_scale = softmax_scale;
  a.workspace = scratch;
  a.workspace_bytes = LKV_NOALLOC_SCRATCH_BYTES;
  a.stream = stream;
  const int rc = lkv::decode_paged(a);
  if (rc != LKV_OK) return rc;
  if (error_word && cudaMemcpyAsync(error_word, scratch, 4 * sizeof(int32_t), cudaMemcpyDeviceToDevice, s) !=
                        cudaSuccess)
    return LKV_ERR_CUDA;
  return LKV_OK;
}
