// Context-parallel combine over NVLink peer memory (sm_100a): the exchange and
// LSE merge of the per-rank decode partials for sequence-sharded (128K) decode,
// in one kernel instead of an all-gather collective plus a merge launch.
//
// Every rank holds a partial (o fp32 [rows, D] normalised, lse [rows] natural
// log) over its slice of each sequence's keys.  CTA c owns rows
// [c * R, (c + 1) * R) on every rank and, with this call's epoch (a device
// counter advanced once per call, so the launch can live in a CUDA graph),
//   1. pushes those rows of this rank's partial into slot [epoch & 1][rank] of
//      every peer's receive buffer with plain peer stores (NVLink P2P), each
//      fp32 value travelling with the epoch in one 8-byte word {value, epoch}
//      (an aligned 8-byte store arrives whole, so no fence or separate flag
//      is needed: a word is valid once its epoch half matches);
//   2. merges the world partials of its rows in rank order exactly as
//      merge_partials_kernel does (same arithmetic, same order), reading the
//      peers' words from its own receive buffer and polling each until its
//      epoch half matches - bounded by wall time, with the error word set on
//      expiry - then scales by s_l per query head and writes bf16.
// A CTA waits only on CTAs of other GPUs, which push before they wait, so no
// CTA depends on another CTA of its own grid.  Receive slots alternate with the
// epoch parity: a peer can reuse a slot only after it has received this rank's
// next epoch, which this rank pushes after it finished reading that slot.
// No multicast and no NVLS: plain loads and stores to peer-mapped memory.
// With send == null the push already happened inside the decode kernel (its
// context-parallel mode writes every rank's merged rows into the receive slots
// with the same words); the kernel then only polls and merges, reading this
// rank's own rows from its receive buffer like a peer's.

#include <algorithm>

#include "common.cuh"
#include "cp_words.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace lkv {

namespace {

constexpr int kCpThreads = 128;  // 4 warps: one output row each at a time
constexpr int kCpKernelId = 8;

struct CpPeers {
  uint64_t* recv[kCpMaxRanks];
};

struct CpParams {
  const float* send;    // this rank's packed partial: o [rows * D] | lse [rows]; null: already pushed
  int64_t part_words;   // words per partial in a receive slot (>= rows * (D + 1))
  int64_t rows;
  int rows_per_cta;
  int Hq, rank, world;
  uint32_t* state;      // [0] epoch of the previous call, [1] CTAs of this call done
  const float* out_scale;
  __nv_bfloat16* out;
  int64_t out_stride_tok;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(kCpThreads)
    cp_combine_kernel(const __grid_constant__ CpPeers peers, const __grid_constant__ CpParams p) {
  pdl_launch_dependents();
  pdl_wait();  // the partial comes from the decode kernel (and the previous call's epoch update)
  // This call's epoch: one more than the previous call's.  Every CTA reads it
  // before it counts itself done, and only the last CTA to count advances it.
  const uint32_t epoch = __ldcg(p.state) + 1u;
  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)c * p.rows_per_cta;
  const int64_t r1 = r0 + p.rows_per_cta < p.rows ? r0 + p.rows_per_cta : p.rows;
  const int slot = (int)(epoch & 1u);
  const int64_t lse_off = p.rows * D;

  // 1. push this CTA's rows to every peer: pairs of {value, epoch} words
  const int64_t npair = (r1 - r0) * D / 2;
  const float2* src_o = reinterpret_cast<const float2*>(p.send + r0 * D);
  for (int peer = 0; p.send && peer < p.world; ++peer) {
    if (peer == p.rank) continue;
    uint64_t* dst = peers.recv[peer] + ((int64_t)slot * p.world + p.rank) * p.part_words;
    for (int64_t i = threadIdx.x; i < npair; i += kCpThreads) {
      const float2 v = src_o[i];
      st_ll2(dst + r0 * D + 2 * i, ll_word(v.x, epoch), ll_word(v.y, epoch));
    }
    for (int64_t i = r0 + threadIdx.x; i < r1; i += kCpThreads) {
      const uint64_t w = ll_word(p.send[lse_off + i], epoch);
      asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst + lse_off + i), "l"(w) : "memory");
    }
  }

  // 2. merge in rank order (merge_partials_kernel arithmetic); peers' words are polled
  const uint64_t* slot_base = peers.recv[p.rank] + (int64_t)slot * p.world * p.part_words;
  const uint64_t start = global_timer_ns();
  bool fail = false;
  for (int64_t row = r0 + warp; row < r1; row += kCpThreads / 32)
    cp_merge_row<D>(slot_base, p.part_words, p.world, p.rank, p.send, p.rows, row, p.Hq, p.out_scale, p.out,
                    p.out_stride_tok, epoch, start, fail, lane);
  if (fail) report_error(p.err, DEVERR_WAIT_TIMEOUT, kCpKernelId, (int)r0);
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(p.state + 1, 1u) == gridDim.x - 1) {
    p.state[1] = 0u;     // every CTA has read the epoch and counted itself
    p.state[0] = epoch;  // the next call (stream-ordered after this one) uses epoch + 1
  }
}

}  // namespace

int64_t cp_part_words(int64_t rows, int head_dim) { return (rows * (head_dim + 1) + 1) / 2 * 2; }

int cp_combine(const float* send, const uint64_t* peer_recv, int rank, int world, uint32_t* state, int64_t rows,
               int head_dim, int hq, const float* out_scale, void* out, int64_t out_stride_tok, int32_t* error_word,
               cudaStream_t stream) {
  if (world < 1 || world > kCpMaxRanks || rank < 0 || rank >= world || rows < 1 || hq < 1 || rows % hq ||
      (head_dim != 64 && head_dim != 128) || !peer_recv || !out || !state ||
      (reinterpret_cast<uintptr_t>(state) & 7))
    return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(send) & 15) || out_stride_tok < (int64_t)hq * head_dim || (out_stride_tok % 2) ||
      (reinterpret_cast<uintptr_t>(out) & 3))
    return LKV_ERR_INVALID_ARGUMENT;
  CpPeers peers{};
  for (int r = 0; r < world; ++r) {
    if (!peer_recv[r] || (peer_recv[r] & 15)) return LKV_ERR_INVALID_ARGUMENT;
    peers.recv[r] = reinterpret_cast<uint64_t*>(peer_recv[r]);
  }
  CpParams p{};
  p.send = send;
  p.part_words = cp_part_words(rows, head_dim);
  p.rows = rows;
  p.rows_per_cta = kCpRowsPerCta;
  p.Hq = hq;
  p.rank = rank;
  p.world = world;
  p.state = state;
  p.out_scale = out_scale;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride_tok = out_stride_tok;
  p.err = error_word;
  const unsigned grid = (unsigned)((rows + kCpRowsPerCta - 1) / kCpRowsPerCta);
  const cudaError_t e = head_dim == 128
                            ? launch_pdl(cp_combine_kernel<128>, dim3(grid), dim3(kCpThreads), 0, stream, peers, p)
                            : launch_pdl(cp_combine_kernel<64>, dim3(grid), dim3(kCpThreads), 0, stream, peers, p);
  return e == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

}  // namespace lkv
