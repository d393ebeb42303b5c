// Split-KV decode over the shared last-layer paged K/V pool (sm_100a).
//
// Work item = (sequence b, KV head hk, split).  The grid is persistent: as
// many CTAs as fit on the GPU at once, CTA c taking items c, c + grid, ...
// A producer warp streams the pages of all its items back to back with TMA
// (4-D tensor map over [pages, 16, Hkv, D], one 16 x 64 half-tile per copy,
// 128-byte swizzle) into a STAGES-deep ring of shared-memory stages holding NW
// pages of one item each; NW consumer warps each take one page of a stage.  The
// ring therefore fills once per CTA, and each item's epilogue (cross-warp
// merge, output write) overlaps the loads of the next item.  All query heads of the GQA group are folded into one MMA
// tile with the keys as the M dimension:
//     S^T[16 keys, 8 heads] = K[16, D] * Q^T[D, 8]           (mma m16n8k16)
//     O^T[D, 8 heads]      += V^T[D, 16] * P^T[16 keys, 8]    (mma m16n8k16)
// P^T is produced from the S^T accumulators with movmatrix (8x8 transposes),
// so probabilities never leave registers.  The online softmax keeps a running
// max per head (4-lane groups share a head pair) and per-thread partial sums.
// At the end of an item the NW warps merge in a shared-memory area of their
// own (four heads at a time) and the CTA writes either the final bf16 output
// (single split) or a normalised fp32 partial + log2 LSE.
// A second small kernel merges the splits (and serves as the context-parallel
// combine).
//
// Reference semantics: the merged attention call of the vLLM fast path
// (vllm/src/lastkv/vllm/backends/rmarin_flashinfer/fastpath.py:643-650; FA3
// varlen with block_table / seqused_k, causal with bottom-right alignment,
// which for one query token means "all seq_k keys") followed by head_scale_
// (fused_qkv.py:140-155), folded here into the epilogue.

#include <math.h>

#include <algorithm>
#include <climits>

#include "common.cuh"
#include "cp_words.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace lkv {

constexpr int PAGE = 16;

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t q_stride_tok;
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* seq_k;
  __nv_bfloat16* out;
  int64_t out_stride_tok;
  float* lse;              // final natural-log LSE [B, Hq] or null
  const float* out_scale;  // [Hq] or null
  float* part_o;           // [B*Hq, S, D] normalised partials (S > 1 or partial mode)
  float* part_lse;         // [B*Hq, S] log2 units
  int* err;
  int B, Hq, Hkv, W, S;
  int64_t num_pages;
  float scale_log2;  // softmax_scale * log2(e)
  int final_out;     // 1: this kernel writes `out` (S == 1 and not partial mode)
  int early;         // 1: seq_k, the block table and older pages predate the PDL chain (LKV_DECODE_TABLES_READY)
  int keep_pages;    // block-table columns [0, keep_pages) load with L2 evict_last (LKV_DECODE_L2_KEEP), else evict_first
  // Context parallel: the last CTA to finish a (sequence, KV head) unit merges its
  // split partials and pushes the merged rows to every rank's receive buffer.
  uint64_t* cp_recv[kCpMaxRanks];
  uint32_t* cp_state;      // [0] epoch of the previous call, [1] CTAs done, [2 + unit] arrivals (null: no push)
  int64_t cp_part_words;   // words per rank partial in a receive slot
  int cp_rank, cp_world;
  // Fused exchange: after its own items, a CTA counts its units' arrivals once; the
  // last CTA of a unit pushes the unit's merged rows to every rank, then polls the
  // unit's rows from every rank, merges them in rank order and writes `out` (x
  // out_scale); the last CTA to finish advances the epoch.  No combine launch.
  int cp_fused;
  int* cp_err;
};

// Items a CTA may complete after its item loop in the fused context-parallel
// exchange; the host uses that form only when no CTA takes more items than this.
constexpr int kMaxTouched = 32;

// Exact LSE merge of one row's S partials (S <= 32): lane s holds part s's LSE,
// so the accumulation loop has no load-dependent branch and its part loads are
// all in flight at once.  Shared by merge_partials_kernel and the
// context-parallel push, which must produce the same bits.
//   part s of the row: o at o_base + s * o_step (D floats), LSE at lse_base + s * lse_step
//   to2 converts the stored LSE to log2 units.  Returns this lane's D / 32
//   weighted sums in acc (unnormalised), their normaliser in inv (1 / sum of
//   weights, 0 when empty) and the log2 LSE in lse2.
template <int D>
__device__ __forceinline__ void merge_row_parts(const float* o_base, int64_t o_step, const float* lse_base,
                                                int64_t lse_step, int S, float to2, int lane,
                                                float (&acc)[D / 32], float& inv, float& lse2) {
  constexpr int PER = D / 32;
  constexpr int C = 16;  // parts whose o rows are requested together
  float v[C][PER];
  auto load_parts = [&](int s0) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const int s = s0 + c;
      const float* src = o_base + s * o_step + lane * PER;
      if (s >= S) {
#pragma unroll
        for (int e = 0; e < PER; ++e) v[c][e] = 0.f;
      } else if constexpr (PER == 4) {
        const float4 t = __ldcg(reinterpret_cast<const float4*>(src));
        v[c][0] = t.x;
        v[c][1] = t.y;
        v[c][2] = t.z;
        v[c][3] = t.w;
      } else {
#pragma unroll
        for (int e = 0; e < PER; ++e) v[c][e] = __ldcg(src + e);
      }
    }
  };
  load_parts(0);  // in flight together with the LSE loads: no dependency between them
  const float my_ls = lane < S ? __ldcg(lse_base + lane * lse_step) * to2 : -INFINITY;
  float M = my_ls;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
#pragma unroll
  for (int e = 0; e < PER; ++e) acc[e] = 0.f;
  float L = 0.f;
  if (M != -INFINITY) {
    const float my_w = my_ls == -INFINITY ? 0.f : exp2f(my_ls - M);
    for (int s0 = 0; s0 < S; s0 += C) {
      if (s0 > 0) load_parts(s0);
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int s = s0 + c;
        if (s >= S) break;
        const float w = __shfl_sync(0xffffffffu, my_w, s);
        // a part with -inf LSE (w == 0) leaves L and acc untouched, whatever its o holds
        const bool use = w != 0.f;
        const float Ln = L + w;
        L = use ? Ln : L;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const float an = acc[e] + w * v[c][e];
          acc[e] = use ? an : acc[e];
        }
      }
    }
  }
  inv = L > 0.f ? 1.f / L : 0.f;
  lse2 = L > 0.f ? M + log2f(L) : -INFINITY;
}

// Context parallel: merge one row's S split partials (merge_partials_kernel's
// arithmetic) and push it as {value, epoch} words into every rank's receive slot
// [epoch & 1][this rank] - the words cp_combine_kernel's push writes.  One warp.
template <int D>
__device__ __forceinline__ void cp_push_row(const DecodeParams& p, int64_t row, uint32_t epoch, int lane) {
  constexpr int PER = D / 32;
  float acc[PER];
  float inv, lse2;
  merge_row_parts<D>(p.part_o + row * p.S * D, D, p.part_lse + row * p.S, 1, p.S, 1.f, lane, acc, inv, lse2);
#pragma unroll
  for (int e = 0; e < PER; ++e) acc[e] = acc[e] * inv;  // as merge_partials_kernel's fp32 output
  const float lse_e = lse2 * 0.6931471805599453f;
  const int64_t rows = (int64_t)p.B * p.Hq;
  const int slot = (int)(epoch & 1u);
  for (int r = 0; r < p.cp_world; ++r) {
    uint64_t* dst = p.cp_recv[r] + ((int64_t)slot * p.cp_world + p.cp_rank) * p.cp_part_words;
    uint64_t* od = dst + row * D + lane * PER;
#pragma unroll
    for (int e = 0; e < PER; e += 2) st_ll2(od + e, ll_word(acc[e], epoch), ll_word(acc[e + 1], epoch));
    if (lane == 0) {
      const uint64_t wl = ll_word(lse_e, epoch);
      asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst + rows * D + row), "l"(wl) : "memory");
    }
  }
}

template <int D, int NW, int STAGES>
struct DecodeCfg {
  static constexpr int HALVES = D / 64;
  static constexpr int TILE_BYTES = PAGE * 128;               // 16 rows x 64 bf16
  static constexpr int PAGE_BYTES = 2 * HALVES * TILE_BYTES;  // K and V of one page, one head
  static constexpr int STAGE_BYTES = NW * PAGE_BYTES;
  static constexpr int OSTRIDE = D + 4;                       // padded fp32 row of the merge area
  static constexpr int DATA_BYTES = STAGES * STAGE_BYTES;
  // merge area after the ring: o [NW][4 heads][OSTRIDE], then m and l [NW][8]
  static constexpr int MERGE_BYTES = NW * 4 * OSTRIDE * 4 + 2 * NW * 8 * 4;
  // + failure / last flags, the completion count, unit list and last flags
  static constexpr int SMEM_BYTES = 1024 + DATA_BYTES + MERGE_BYTES + 2 * STAGES * 8 + 32 + 2 * kMaxTouched * 4;
};

__device__ __forceinline__ float warp_max_g(float v) {
  // reduce over the 8 lanes sharing (lane & 3)
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  return v;
}

__device__ __forceinline__ float warp_sum_g(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return v;
}

template <int D, int GROUP, int NW, int STAGES>
__global__ void __launch_bounds__((NW + 1) * 32)
    decode_splitkv_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                          const DecodeParams p) {
  using Cfg = DecodeCfg<D, NW, STAGES>;
  constexpr int KT = D / 16;  // 16-wide d tiles
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* mo = reinterpret_cast<float*>(smem + Cfg::DATA_BYTES);  // [NW][4][OSTRIDE]
  float* mm = mo + NW * 4 * Cfg::OSTRIDE;                         // [NW][8]
  float* ml = mm + NW * 8;                                        // [NW][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::DATA_BYTES + Cfg::MERGE_BYTES);
  uint64_t* empty = full + STAGES;
  volatile int* fail_flag = reinterpret_cast<volatile int*>(empty + STAGES);
  volatile int* last_flag = fail_flag + 1;
  // fused exchange: the units of this CTA's items and which of them it completes
  volatile int* n_touched = fail_flag + 4;
  volatile int* touched = n_touched + 4;
  volatile int* last_of = touched + kMaxTouched;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_launch_dependents();
  // Programmatic dependent launch: only after pdl_wait() are the writes of the
  // kernels before this one in the stream guaranteed visible.  Everything is
  // read after it, except with p.early: the caller then guarantees that seq_k,
  // the block table and every page but each sequence's last were written
  // before the most recent launch without the PDL attribute, so the producer
  // may request the first stages of older pages before the wait.

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    *fail_flag = 0;
    *n_touched = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // item i -> (split, hk, b) = (i % S, i / S % Hkv, i / (S * Hkv)); its pages [p0, p1)
  const int n_items = p.S * p.Hkv * p.B;
  struct Item {
    int b, hk, split, n, p0, p1, n_iter;
  };
  auto item_at = [&](int i) {
    Item it;
    it.split = i % p.S;
    it.hk = (i / p.S) % p.Hkv;
    it.b = i / (p.S * p.Hkv);
    it.n = max(0, p.seq_k[it.b]);
    const int npages = min((it.n + PAGE - 1) / PAGE, p.W);
    const int per = (npages + p.S - 1) / p.S;
    it.p0 = min(npages, it.split * per);
    it.p1 = min(npages, it.p0 + per);
    it.n_iter = (it.p1 - it.p0 + NW - 1) / NW;
    return it;
  };

  if (warp == NW) {
    // ------------------------------------------------------------ producer
    // Stages are numbered across items (gs), so the ring never drains between
    // items.  On a failed wait it stops; the consumers' own bounded waits then
    // end their loops.
    if (lane == 0) {
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      const uint64_t pol_first = policy_evict_first(), pol_last = policy_evict_last();
      // Before waiting for the previous kernel: the first item's first stages
      // (fresh slots, so no empty-slot wait), as long as a stage holds neither
      // the sequence's last page - where the previous kernel may just have
      // appended this step's key - nor a page id that would need an error report
      // (a global write, which must follow the wait).  Only with p.early: the
      // sequence lengths and block tables are then inputs of the step that no
      // kernel of the current PDL chain writes.
      int pre = 0;
      if (p.early && (int)blockIdx.x < n_items) {
        const Item w = item_at(blockIdx.x);
        const int32_t* row = p.bt + (int64_t)w.b * p.bt_stride;
        const int last_page = min((w.n + PAGE - 1) / PAGE, p.W) - 1;
        for (; pre < STAGES && pre < w.n_iter; ++pre) {
          const int first = w.p0 + pre * NW;
          const int cnt = min(NW, w.p1 - first);
          if (first + cnt - 1 >= last_page) break;
          int cur[NW];
          bool good = true;
#pragma unroll
          for (int k = 0; k < NW; ++k) {
            cur[k] = k < cnt ? __ldg(row + first + k) : 0;
            good = good && (k >= cnt || (cur[k] >= 0 && (int64_t)cur[k] < p.num_pages));
          }
          if (!good) break;
          mbar_arrive_expect_tx(&full[pre], (uint32_t)(cnt * Cfg::PAGE_BYTES));
          uint8_t* dst = smem + pre * Cfg::STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < NW; ++k) {
            if (k >= cnt) break;
#pragma unroll
            for (int h = 0; h < Cfg::HALVES; ++h) {
              const uint64_t pol = first + k < p.keep_pages ? pol_last : pol_first;
              tma_load_4d_hint(dst + k * Cfg::PAGE_BYTES + h * Cfg::TILE_BYTES, &tmk, &full[pre], h * 64, w.hk, 0,
                               cur[k], pol);
              tma_load_4d_hint(dst + k * Cfg::PAGE_BYTES + (Cfg::HALVES + h) * Cfg::TILE_BYTES, &tmv, &full[pre],
                               h * 64, w.hk, 0, cur[k], pol);
            }
          }
        }
      }
      pdl_wait();
      uint32_t gs = (uint32_t)pre;
      bool ok = true;
      for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
        const Item w = item_at(i);
        const int32_t* row = p.bt + (int64_t)w.b * p.bt_stride;
        const int it0 = i == (int)blockIdx.x ? pre : 0;  // stages already requested above
        // Page ids of a stage are loaded together (one L2 round trip, not one per
        // page), and the next stage's before waiting for a free slot.
        int ids[NW];
#pragma unroll
        for (int k = 0; k < NW; ++k) {
          const int pg = w.p0 + it0 * NW + k;
          ids[k] = pg < w.p1 ? __ldg(row + pg) : 0;
        }
        for (int it = it0; it < w.n_iter; ++it, ++gs) {
          const int first = w.p0 + it * NW;
          const int cnt = min(NW, w.p1 - first);
          int cur[NW];
#pragma unroll
          for (int k = 0; k < NW; ++k) cur[k] = ids[k];
#pragma unroll
          for (int k = 0; k < NW; ++k) ids[k] = (first + NW + k < w.p1) ? __ldg(row + first + NW + k) : 0;
          const int s = (int)(gs % STAGES);
          const uint32_t ph = (gs / STAGES) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u)) {
            report_error(p.err, DEVERR_WAIT_TIMEOUT, 1, it);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], (uint32_t)(cnt * Cfg::PAGE_BYTES));
          uint8_t* dst = smem + s * Cfg::STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < NW; ++k) {
            if (k >= cnt) break;
            const int pid = cur[k];
            if (pid < 0 || (int64_t)pid >= p.num_pages) report_error(p.err, DEVERR_BAD_PAGE, 1, pid);
            // An out-of-range page reads as zeros (TMA bounds-fills), never faults.
#pragma unroll
            for (int h = 0; h < Cfg::HALVES; ++h) {
              const uint64_t pol = first + k < p.keep_pages ? pol_last : pol_first;
              tma_load_4d_hint(dst + k * Cfg::PAGE_BYTES + h * Cfg::TILE_BYTES, &tmk, &full[s], h * 64, w.hk, 0, pid,
                               pol);
              tma_load_4d_hint(dst + k * Cfg::PAGE_BYTES + (Cfg::HALVES + h) * Cfg::TILE_BYTES, &tmv, &full[s],
                               h * 64, w.hk, 0, pid, pol);
            }
          }
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  // This call's epoch.  Unfused, the combine launch that follows advances the
  // stored one.  Fused, thread 0 reads it once for the CTA and counts the CTA in;
  // the last CTA to count stores it for the next call (stream-ordered after this
  // one): every CTA has read it by then, and no CTA's tail waits on the count.
  uint32_t cp_epoch = 0u;
  if (p.cp_state) {
    if (p.cp_fused) {
      volatile uint32_t* s_epoch = reinterpret_cast<volatile uint32_t*>(n_touched + 1);
      if (threadIdx.x == 0) {
        const uint32_t e = __ldcg(p.cp_state) + 1u;
        *s_epoch = e;
        if (atom_add_acq_rel_gpu(p.cp_state + 1, 1u) == gridDim.x - 1) {
          p.cp_state[1] = 0u;
          p.cp_state[0] = e;
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
      cp_epoch = *s_epoch;
    } else {
      cp_epoch = __ldcg(p.cp_state) + 1u;
    }
  }
  const int g = lane >> 2, c = lane & 3;
  // ldmatrix source rows/chunks (see the fragment derivation in the header comment)
  const uint32_t k_row = (lane & 7) + ((lane >> 3) & 1) * 8, k_chunk_hi = lane >> 4;
  const uint32_t v_row = (lane & 7) + (lane >> 4) * 8, v_chunk_hi = (lane >> 3) & 1;
  uint32_t gs = 0;
  bool failed = false;

  for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
    const Item w = item_at(i);
    const int b = w.b, hk = w.hk, n = w.n;
    uint32_t qf[KT][2];
    {
      const bool valid = g < GROUP;
      const __nv_bfloat16* qrow =
          p.q + (int64_t)b * p.q_stride_tok + (int64_t)(hk * GROUP + (valid ? g : 0)) * D;
#pragma unroll
      for (int j = 0; j < KT; ++j) {
        const int d0 = 16 * j + 2 * c;
        qf[j][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + d0) : 0u;
        qf[j][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + d0 + 8) : 0u;
      }
    }
    float o[KT][4];
#pragma unroll
    for (int k = 0; k < KT; ++k) o[k][0] = o[k][1] = o[k][2] = o[k][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int it = 0; it < w.n_iter; ++it, ++gs) {
      const int s = (int)(gs % STAGES);
      const uint32_t ph = (gs / STAGES) & 1u;
      if (!mbar_wait(&full[s], ph)) {
        report_error(p.err, DEVERR_WAIT_TIMEOUT, 1, 1000000 + it);
        failed = true;
        break;
      }
      const int page_idx = w.p0 + it * NW + warp;
      if (page_idx < w.p1) {
        uint8_t* kt = smem + s * Cfg::STAGE_BYTES + warp * Cfg::PAGE_BYTES;
        uint8_t* vt = kt + Cfg::HALVES * Cfg::TILE_BYTES;
        const uint32_t kbase = smem_u32(kt), vbase = smem_u32(vt);
        float sc[4] = {0.f, 0.f, 0.f, 0.f}, sd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < KT; ++j) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(a0, a1, a2, a3,
                      kbase + (j >> 2) * Cfg::TILE_BYTES + swz128(k_row, 2 * (j & 3) + k_chunk_hi));
          if (j & 1) mma_bf16_16816(sd, a0, a1, a2, a3, qf[j][0], qf[j][1]);
          else mma_bf16_16816(sc, a0, a1, a2, a3, qf[j][0], qf[j][1]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[e] += sd[e];
        const int key0 = page_idx * PAGE;
        const int valid_rows = n - key0;  // >= 1
        const bool r0 = g < valid_rows, r1 = g + 8 < valid_rows;
        const float s00 = r0 ? sc[0] * p.scale_log2 : -INFINITY;
        const float s01 = r0 ? sc[1] * p.scale_log2 : -INFINITY;
        const float s10 = r1 ? sc[2] * p.scale_log2 : -INFINITY;
        const float s11 = r1 ? sc[3] * p.scale_log2 : -INFINITY;
        const float mn0 = fmaxf(m0, warp_max_g(fmaxf(s00, s10)));
        const float mn1 = fmaxf(m1, warp_max_g(fmaxf(s01, s11)));
        const float al0 = ex2_approx(m0 - mn0), al1 = ex2_approx(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        const float p00 = ex2_approx(s00 - mn0), p01 = ex2_approx(s01 - mn1);
        const float p10 = ex2_approx(s10 - mn0), p11 = ex2_approx(s11 - mn1);
        l0 = l0 * al0 + p00 + p10;
        l1 = l1 * al1 + p01 + p11;
#pragma unroll
        for (int k = 0; k < KT; ++k) {
          o[k][0] *= al0;
          o[k][1] *= al1;
          o[k][2] *= al0;
          o[k][3] *= al1;
        }
        const uint32_t pb0 = movmatrix_trans(pack_bf16(p00, p01));
        const uint32_t pb1 = movmatrix_trans(pack_bf16(p10, p11));
        if (valid_rows < PAGE) {
          // Rows past the sequence end carry P = 0, but 0 * NaN would still poison
          // O; clear them (a swizzled row stays inside its own 128 bytes).
          const int nz = (PAGE - valid_rows) * 8 * Cfg::HALVES;
          for (int e = lane; e < nz; e += 32) {
            const int hv = e / ((PAGE - valid_rows) * 8);
            const int rem = e % ((PAGE - valid_rows) * 8);
            const int r = valid_rows + rem / 8;
            *reinterpret_cast<uint4*>(vt + hv * Cfg::TILE_BYTES + r * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
          }
          __syncwarp();
        }
#pragma unroll
        for (int k = 0; k < KT; ++k) {
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(a0, a1, a2, a3,
                            vbase + (k >> 2) * Cfg::TILE_BYTES + swz128(v_row, 2 * (k & 3) + v_chunk_hi));
          mma_bf16_16816(o[k], a0, a1, a2, a3, pb0, pb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ------------------------------------------------------------ item merge
    // Only consumer warps write the failure flag, and only before this barrier;
    // every consumer warp reads it after the barrier, so they leave together.
    l0 = warp_sum_g(l0);
    l1 = warp_sum_g(l1);
    if (failed && lane == 0) *fail_flag = 1;
    if (g == 0) {
      mm[warp * 8 + 2 * c] = m0;
      mm[warp * 8 + 2 * c + 1] = m1;
      ml[warp * 8 + 2 * c] = l0;
      ml[warp * 8 + 2 * c + 1] = l1;
    }
    // Heads go through the o area four at a time: thread (g, c) holds heads 2c
    // and 2c + 1, so chunk hc is held by the threads with c >> 1 == hc.
#pragma unroll
    for (int hc = 0; hc < (GROUP + 3) / 4; ++hc) {
      if ((c >> 1) == hc) {
        float* w0 = mo + (warp * 4 + 2 * c - 4 * hc) * Cfg::OSTRIDE;
        float* w1 = w0 + Cfg::OSTRIDE;
#pragma unroll
        for (int k = 0; k < KT; ++k) {
          w0[16 * k + g] = o[k][0];
          w1[16 * k + g] = o[k][1];
          w0[16 * k + g + 8] = o[k][2];
          w1[16 * k + g + 8] = o[k][3];
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
      if (*fail_flag) return;  // uniform across the consumer warps
      constexpr int HC = GROUP < 4 ? GROUP : 4;
      for (int idx = threadIdx.x; idx < HC * D; idx += NW * 32) {
        const int hl = idx / D, d = idx % D, h = 4 * hc + hl;
        float M = -INFINITY;
#pragma unroll
        for (int v = 0; v < NW; ++v) M = fmaxf(M, mm[v * 8 + h]);
        float L = 0.f, acc = 0.f;
        if (M != -INFINITY) {
#pragma unroll
          for (int v = 0; v < NW; ++v) {
            const float f = exp2f(mm[v * 8 + h] - M);
            L += ml[v * 8 + h] * f;
            acc += mo[(v * 4 + hl) * Cfg::OSTRIDE + d] * f;
          }
        }
        const float val = L > 0.f ? acc / L : 0.f;
        const int hq = hk * GROUP + h;
        if (p.final_out) {
          const float sc = p.out_scale ? p.out_scale[hq] : 1.f;
          p.out[(int64_t)b * p.out_stride_tok + (int64_t)hq * D + d] = __float2bfloat16_rn(val * sc);
          if (p.lse && d == 0)
            p.lse[(int64_t)b * p.Hq + hq] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
        } else {
          const int64_t rowi = ((int64_t)b * p.Hq + hq) * p.S + w.split;
          p.part_o[rowi * D + d] = val;
          if (d == 0) p.part_lse[rowi] = L > 0.f ? M + log2f(L) : -INFINITY;
        }
      }
      // the area (and mm / ml) is rewritten by the next chunk or item
      asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
    }
    if (p.cp_fused) {
      // completion after the item loop: remember the unit (the barrier above has
      // ordered this CTA's partial writes; the list is read after the next barrier)
      if (threadIdx.x == 0) touched[(*n_touched)++] = b * p.Hkv + hk;
    } else if (p.cp_state) {
      // Context parallel, more items per CTA than the list holds: count this split
      // now; the unit's last CTA merges the S partials (merge_partials_kernel's
      // arithmetic) and pushes the merged rows, and a cp_combine launch follows.
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
      uint32_t* arrivals = p.cp_state + 2 + (int64_t)b * p.Hkv + hk;
      if (threadIdx.x == 0) *last_flag = atomicAdd(arrivals, 1u) == (uint32_t)(p.S - 1);
      asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
      if (*last_flag) {
        __threadfence();
        for (int h = warp; h < GROUP; h += NW) cp_push_row<D>(p, (int64_t)b * p.Hq + hk * GROUP + h, cp_epoch, lane);
        asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
        if (threadIdx.x == 0) *arrivals = 0u;  // every split has arrived: ready for the next call
      }
    }
  }
  if (!p.cp_fused) return;

  // ---------------------------------------------------------------- fused exchange
  // The arrival counting runs once per CTA, after all its items (counting per
  // item, with its barriers, stalls the consumers while the ring waits).
  // The last CTA to count a unit merges the unit's S split partials
  // (merge_partials_kernel's arithmetic) and pushes the merged rows to every
  // rank; then it polls the unit's rows from every rank and merges them in rank
  // order into `out`.  A CTA polls only after all its items and pushes are done,
  // and only for pushes other GPUs' CTAs make without waiting: no wait cycle.
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));  // this CTA's partial writes are done
  const int n_items_cta = *n_touched;
  uint32_t* counters = p.cp_state + 2;
  // Thread 0's acquire-release counting publishes the CTA's partials (ordered
  // before it by the barrier above) and, for a unit it completes, makes the other
  // CTAs' partials visible to the whole CTA through the barrier below.
  if (threadIdx.x == 0)
    for (int k = 0; k < n_items_cta; ++k)
      last_of[k] = atom_add_acq_rel_gpu(counters + touched[k], 1u) == (uint32_t)(p.S - 1);
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
  for (int k = 0; k < n_items_cta; ++k) {
    if (!last_of[k]) continue;
    const int unit = touched[k];
    const int b = unit / p.Hkv, hk = unit % p.Hkv;
    for (int h = warp; h < GROUP; h += NW) cp_push_row<D>(p, (int64_t)b * p.Hq + hk * GROUP + h, cp_epoch, lane);
  }
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32));
  if (threadIdx.x == 0)
    for (int k = 0; k < n_items_cta; ++k)
      if (last_of[k]) counters[touched[k]] = 0u;  // every split has arrived: ready for the next call
  const int64_t rows = (int64_t)p.B * p.Hq;
  const uint64_t* slot_base = p.cp_recv[p.cp_rank] + (int64_t)(cp_epoch & 1u) * p.cp_world * p.cp_part_words;
  const uint64_t start = global_timer_ns();
  bool fail = false;
  for (int k = 0; k < n_items_cta; ++k) {
    if (!last_of[k]) continue;
    const int unit = touched[k];
    const int b = unit / p.Hkv, hk = unit % p.Hkv;
    for (int h = warp; h < GROUP; h += NW)
      cp_merge_row<D>(slot_base, p.cp_part_words, p.cp_world, p.cp_rank, nullptr, rows,
                      (int64_t)b * p.Hq + hk * GROUP + h, p.Hq, p.out_scale, p.out, p.out_stride_tok, cp_epoch, start,
                      fail, lane);
  }
  if (fail && lane == 0) report_error(p.cp_err, DEVERR_WAIT_TIMEOUT, 1, 2000000 + (int)blockIdx.x);
}

// ------------------------------------------------------------------ merge
// One warp per output row (token, head): merge `parts` normalised partials.
// part_o: [rows, S, D] with row stride S*D when split_major == 0 (decode
// splits), or part s at part_o + s * o_part_stride ([rows, D] each) when
// split_major == 1 (context-parallel ranks; lse likewise with lse_part_stride).
struct MergeParams {
  const float* part_o;
  const float* part_lse;
  int S;
  int64_t rows;
  int split_major;
  int64_t o_part_stride, lse_part_stride;  // elements, split_major == 1
  int lse_log2;  // 1: part_lse in log2 units, 0: natural log
  int Hq;
  const float* out_scale;
  __nv_bfloat16* out;  // bf16 [rows, D] with row index -> (tok = row / Hq, h = row % Hq)
  int64_t out_stride_tok;
  float* lse_out;        // natural log [rows] or null
  float* out_f32;        // fp32 normalised [rows, D] instead of bf16 (partial of partials) or null
  float* out_lse_f32;    // natural log [rows] for out_f32 mode
};

template <int D>
__global__ void __launch_bounds__(128) merge_partials_kernel(const MergeParams p) {
  constexpr int PER = D / 32;
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  if (row >= p.rows) return;
  const float to2 = p.lse_log2 ? 1.f : 1.4426950408889634f;
  auto lse_at = [&](int s) -> float {
    const int64_t i = p.split_major ? (int64_t)s * p.lse_part_stride + row : row * p.S + s;
    return p.part_lse[i] * to2;
  };
  auto o_at = [&](int s) -> const float* {
    return p.split_major ? p.part_o + (int64_t)s * p.o_part_stride + row * D : p.part_o + (row * p.S + s) * D;
  };
  float acc[PER];
  float inv = 0.f, lse2 = -INFINITY;
  if (p.S <= 32) {
    if (p.split_major)
      merge_row_parts<D>(p.part_o + row * D, p.o_part_stride, p.part_lse + row, p.lse_part_stride, p.S, to2, lane,
                         acc, inv, lse2);
    else
      merge_row_parts<D>(p.part_o + row * p.S * D, D, p.part_lse + row * p.S, 1, p.S, to2, lane, acc, inv, lse2);
  } else {
    // general path (more than 32 parts): the same arithmetic, one part at a time
    float M = -INFINITY;
    for (int s = lane; s < p.S; s += 32) M = fmaxf(M, lse_at(s));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.f;
    float L = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < p.S; ++s) {
        const float ls = lse_at(s);
        if (ls == -INFINITY) continue;
        const float w = exp2f(ls - M);
        L += w;
        const float* src = o_at(s) + lane * PER;
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] += w * src[e];
      }
    }
    inv = L > 0.f ? 1.f / L : 0.f;
    lse2 = L > 0.f ? M + log2f(L) : -INFINITY;
  }
  const int h = (int)(row % p.Hq);
  const int64_t tok = row / p.Hq;
  if (p.out_f32) {
#pragma unroll
    for (int e = 0; e < PER; ++e) p.out_f32[row * D + lane * PER + e] = acc[e] * inv;
    if (lane == 0) p.out_lse_f32[row] = lse2 * 0.6931471805599453f;
    return;
  }
  const float sc = (p.out_scale ? p.out_scale[h] : 1.f) * inv;
  __nv_bfloat16* dst = p.out + tok * p.out_stride_tok + (int64_t)h * D + lane * PER;
#pragma unroll
  for (int e = 0; e < PER; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16(acc[e] * sc, acc[e + 1] * sc);
  if (p.lse_out && lane == 0) p.lse_out[row] = lse2 * 0.6931471805599453f;
}

// ------------------------------------------------------------------ host side

namespace {

constexpr int kNW = 4;
constexpr int kMaxSplits = 32;

// LKV_DECODE_L2_KEEP: how many leading block-table columns of every sequence load
// with the L2 evict_last policy - the oldest pages, which in the merged pool are
// shared final-layer pages that every layer of a step reads again - so that
// they fill a quarter of L2 and later calls over the same history hit them.
// Measured on the 8B decode step (batch 8, 8200 keys): a quarter 1850-1857
// tokens/s, 0.15 1832, a half 1826, 0.7 1782, none 1819; more than a quarter
// crowds out the streamed weights and pages.
// At batch 64 (config 2) the same quarter is 3 % of a call's pages and measured
// 0.5 % slower, so only batches up to 16 keep pages.
constexpr double kL2KeepFraction = 0.25;
constexpr int kL2KeepMaxBatch = 16;
int l2_keep_pages(int l2_bytes, int batch, int hkv, int d, int width) {
  const double page_bytes = 16.0 * hkv * d * 2 * 2;  // K and V of one page, all heads
  const double keep = kL2KeepFraction * l2_bytes / (page_bytes * std::max(batch, 1));
  return (int)std::min<double>(width, std::max(0.0, keep));
}

struct DevInfo {
  int sms = 0;
  int l2_bytes = 0;
  int occ[2][4] = {{0}};  // [D==128][log2 GROUP]
  bool attr_done[2][4] = {{false}};
};
DevInfo g_dev[64];

template <int D, int GROUP, int STAGES>
int prepare_kernel(int dev) {
  using Cfg = DecodeCfg<D, kNW, STAGES>;
  auto kern = decode_splitkv_kernel<D, GROUP, kNW, STAGES>;
  const int di = D == 128, gi = GROUP == 1 ? 0 : GROUP == 2 ? 1 : GROUP == 4 ? 2 : 3;
  DevInfo& info = g_dev[dev];
  if (!info.attr_done[di][gi]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES) != cudaSuccess)
      return -1;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (kNW + 1) * 32, Cfg::SMEM_BYTES) != cudaSuccess)
      return -1;
    info.occ[di][gi] = occ > 0 ? occ : 1;
    info.attr_done[di][gi] = true;
  }
  return info.occ[di][gi];
}

// Split count for the persistent grid (min(items, slots) CTAs): minimise the
// busiest CTA's time, (items per CTA) x (pages per item + per-item merge),
// plus one pipeline fill, plus the merge launch when there are splits.
int choose_splits(int units, int max_pages, int slots) {
  if (max_pages <= 0) return 1;
  const int fill = 6;     // pipeline fill, in page-times (once per CTA)
  const int per_item = 1;  // cross-warp merge and output of an item, in page-times
  int best = 1;
  int64_t best_cost = INT64_MAX;
  const int smax = std::min(kMaxSplits, std::max(1, max_pages / 4));
  for (int s = 1; s <= smax; ++s) {
    const int64_t items = (int64_t)units * s;
    const int64_t per_cta = (items + slots - 1) / slots;
    const int64_t per = (max_pages + s - 1) / s;
    const int64_t cost = per_cta * (per + per_item) + fill + (s > 1 ? 2 : 0);
    if (cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

template <int D, int GROUP, int STAGES>
int launch_group(const CUtensorMap& tmk, const CUtensorMap& tmv, DecodeParams prm, int max_pages, int smax, int dev,
                 cudaStream_t stream, bool partial_mode, float* part_o_user, float* part_lse_user,
                 const DecodeArgs* cp) {
  using Cfg = DecodeCfg<D, kNW, STAGES>;
  const int occ = prepare_kernel<D, GROUP, STAGES>(dev);
  if (occ < 0) return LKV_ERR_CUDA;
  const int slots = g_dev[dev].sms * occ;
  const int S = std::min(smax, choose_splits(prm.B * prm.Hkv, max_pages, slots));
  const int64_t rows = (int64_t)prm.B * prm.Hq;
  prm.S = S;
  prm.final_out = (S == 1 && !partial_mode && !cp) ? 1 : 0;
  const int64_t items = (int64_t)S * prm.Hkv * prm.B;
  if (items > INT_MAX) return LKV_ERR_UNSUPPORTED;
  dim3 grid((unsigned)std::min<int64_t>(items, slots));
  // context parallel: fuse the exchange into this launch when no CTA takes more items than it can list
  prm.cp_fused = (cp && (items + grid.x - 1) / grid.x <= kMaxTouched) ? 1 : 0;
  prm.cp_err = cp ? cp->cp_error : nullptr;
  if (launch_pdl(decode_splitkv_kernel<D, GROUP, kNW, STAGES>, grid, dim3((kNW + 1) * 32), Cfg::SMEM_BYTES, stream,
                 tmk, tmv, prm) != cudaSuccess)
    return LKV_ERR_CUDA;
  if (prm.final_out || prm.cp_fused) return LKV_OK;
  if (cp)  // every rank's merged rows are pushed: poll them and merge in rank order
    return cp_combine(nullptr, cp->cp_recv, cp->cp_rank, cp->cp_world, cp->cp_state, rows, D, prm.Hq,
                      cp->out_scale, cp->out, cp->out_stride_tok, cp->cp_error, stream);
  MergeParams mp{};
  mp.part_o = prm.part_o;
  mp.part_lse = prm.part_lse;
  mp.S = S;
  mp.rows = rows;
  mp.split_major = 0;
  mp.lse_log2 = 1;
  mp.Hq = prm.Hq;
  mp.out_scale = prm.out_scale;
  mp.out = prm.out;
  mp.out_stride_tok = prm.out_stride_tok;
  mp.lse_out = prm.lse;
  if (partial_mode) {
    mp.out_f32 = part_o_user;
    mp.out_lse_f32 = part_lse_user;
  }
  return launch_pdl(merge_partials_kernel<D>, dim3((unsigned)((rows + 3) / 4)), dim3(128), 0, stream, mp) ==
                 cudaSuccess
             ? LKV_OK
             : LKV_ERR_CUDA;
}

}  // namespace

// Workspace bytes one KV split takes after the error header: its normalised o
// [rows, D] and LSE [rows] in fp32, plus 256 bytes for the o area's alignment.
size_t decode_split_bytes(int64_t rows, int d) { return (size_t)rows * (size_t)(d + 1) * sizeof(float) + 256; }

size_t decode_workspace_bytes(int batch, int hq, int d, int max_pages) {
  const int64_t rows = (int64_t)std::max(batch, 0) * std::max(hq, 0);
  const int s = std::min(kMaxSplits, std::max(1, max_pages / 4));
  // s splits of decode_paged's per-split layout (o and lse of every row + 256 bytes of alignment slack)
  return kWorkspaceHeader + (size_t)s * decode_split_bytes(rows, std::max(d, 64));
}

int decode_paged(const DecodeArgs& a) {
  if (a.head_dim != 64 && a.head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (a.num_kv_heads <= 0 || a.num_q_heads <= 0 || a.num_q_heads % a.num_kv_heads) return LKV_ERR_INVALID_ARGUMENT;
  const int group = a.num_q_heads / a.num_kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8) return LKV_ERR_UNSUPPORTED;
  if (a.batch < 0 || a.max_pages_per_seq < 0) return LKV_ERR_INVALID_ARGUMENT;
  if (a.batch == 0) return LKV_OK;
  if (!a.q || !a.pool_k || !a.pool_v || !a.block_table || !a.seq_k) return LKV_ERR_INVALID_ARGUMENT;
  const bool partial_mode = a.partial_o != nullptr;
  if (partial_mode != (a.partial_lse != nullptr)) return LKV_ERR_INVALID_ARGUMENT;
  if (!partial_mode && !a.out) return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a.q) & 3) || (a.q_stride_tok & 1)) return LKV_ERR_INVALID_ARGUMENT;
  if (a.out && ((reinterpret_cast<uintptr_t>(a.out) & 3) || (a.out_stride_tok & 1))) return LKV_ERR_INVALID_ARGUMENT;
  if (!a.workspace || a.workspace_bytes < kWorkspaceHeader + 256) return LKV_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(a.workspace) & 255) return LKV_ERR_WORKSPACE;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LKV_ERR_CUDA;
  if (g_dev[dev].sms == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return LKV_ERR_CUDA;
    g_dev[dev].sms = sms;
  }

  CUtensorMap tmk, tmv;
  int st = make_pool_tensor_map(&tmk, a.pool_k, a.num_pages, a.num_kv_heads, a.head_dim);
  if (st != LKV_OK) return st;
  st = make_pool_tensor_map(&tmv, a.pool_v, a.num_pages, a.num_kv_heads, a.head_dim);
  if (st != LKV_OK) return st;

  DecodeParams prm{};
  prm.q = static_cast<const __nv_bfloat16*>(a.q);
  prm.q_stride_tok = a.q_stride_tok;
  prm.bt = a.block_table;
  prm.bt_stride = a.block_table_stride;
  prm.seq_k = a.seq_k;
  prm.out = static_cast<__nv_bfloat16*>(a.out);
  prm.out_stride_tok = a.out_stride_tok;
  prm.lse = a.lse;
  prm.out_scale = a.out_scale;
  prm.err = static_cast<int*>(a.workspace);
  prm.B = a.batch;
  prm.Hq = a.num_q_heads;
  prm.Hkv = a.num_kv_heads;
  prm.W = a.max_pages_per_seq;
  prm.num_pages = a.num_pages;
  prm.scale_log2 = a.softmax_scale * 1.4426950408889634f;
  prm.early = (a.flags & LKV_DECODE_TABLES_READY) ? 1 : 0;
  if ((a.flags & LKV_DECODE_L2_KEEP) && a.batch <= kL2KeepMaxBatch) {
    if (g_dev[dev].l2_bytes == 0) {
      int l2 = 0;
      if (cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev) != cudaSuccess) return LKV_ERR_CUDA;
      g_dev[dev].l2_bytes = l2 > 0 ? l2 : 1;
    }
    prm.keep_pages = l2_keep_pages(g_dev[dev].l2_bytes, a.batch, a.num_kv_heads, a.head_dim, a.max_pages_per_seq);
  }

  // Workspace after the error header: lse [rows * smax] (256-aligned), then o [rows * smax * D].
  uint8_t* ws = static_cast<uint8_t*>(a.workspace) + kWorkspaceHeader;
  const size_t ws_avail = a.workspace_bytes - kWorkspaceHeader;
  const int64_t rows = (int64_t)a.batch * a.num_q_heads;
  const size_t per_split = decode_split_bytes(rows, a.head_dim);
  const int smax = (int)std::min<size_t>(kMaxSplits, ws_avail / per_split);
  if (smax < 1 && (partial_mode || a.max_pages_per_seq > 0)) return LKV_ERR_WORKSPACE;
  prm.part_lse = reinterpret_cast<float*>(ws);
  prm.part_o = reinterpret_cast<float*>(ws + (((size_t)rows * std::max(smax, 1) * sizeof(float) + 255) & ~size_t(255)));
  if (a.cp_state) {
    prm.cp_state = a.cp_state;
    prm.cp_rank = a.cp_rank;
    prm.cp_world = a.cp_world;
    prm.cp_part_words = cp_part_words(rows, a.head_dim);
    for (int r = 0; r < a.cp_world; ++r) prm.cp_recv[r] = reinterpret_cast<uint64_t*>(static_cast<uintptr_t>(a.cp_recv[r]));
  }

  cudaStream_t stream = static_cast<cudaStream_t>(a.stream);
#define LKV_LAUNCH(DD, GG, SS) \
  return launch_group<DD, GG, SS>(tmk, tmv, prm, a.max_pages_per_seq, std::max(smax, 1), dev, stream, \
                                  partial_mode, a.partial_o, a.partial_lse, a.cp_state ? &a : nullptr)
  if (a.head_dim == 128) {
    switch (group) {
      case 1: LKV_LAUNCH(128, 1, 3);
      case 2: LKV_LAUNCH(128, 2, 3);
      case 4: LKV_LAUNCH(128, 4, 3);
      default: LKV_LAUNCH(128, 8, 3);
    }
  } else {
    switch (group) {
      case 1: LKV_LAUNCH(64, 1, 4);
      case 2: LKV_LAUNCH(64, 2, 4);
      case 4: LKV_LAUNCH(64, 4, 4);
      default: LKV_LAUNCH(64, 8, 4);
    }
  }
#undef LKV_LAUNCH
}

// Sequence-sharded decode: this rank's keys with the merged rows pushed to every
// rank (decode_splitkv_kernel, context-parallel push), then cp_combine_kernel
// polling and merging the ranks' rows - two launches, no collective call.
int decode_paged_cp(const DecodeArgs& a) {
  if (a.cp_world < 1 || a.cp_world > kCpMaxRanks || a.cp_rank < 0 || a.cp_rank >= a.cp_world || !a.cp_recv ||
      !a.cp_state || (reinterpret_cast<uintptr_t>(a.cp_state) & 7) || !a.out || a.partial_o || a.partial_lse)
    return LKV_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < a.cp_world; ++r)
    if (!a.cp_recv[r] || (a.cp_recv[r] & 15)) return LKV_ERR_INVALID_ARGUMENT;
  if (a.out_stride_tok < (int64_t)a.num_q_heads * a.head_dim || (a.out_stride_tok % 2)) return LKV_ERR_INVALID_ARGUMENT;
  return decode_paged(a);
}

int decode_plan(int batch, int hq, int hkv, int d, int max_pages, size_t workspace_bytes, int partial, int* splits,
                int* launches) {
  if (!splits || !launches) return LKV_ERR_INVALID_ARGUMENT;
  if ((d != 64 && d != 128) || hkv < 1 || hq % hkv) return LKV_ERR_UNSUPPORTED;
  const int group = hq / hkv;
  if (group != 1 && group != 2 && group != 4 && group != 8) return LKV_ERR_UNSUPPORTED;
  if (batch <= 0) {
    *splits = 0;
    *launches = 0;
    return LKV_OK;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LKV_ERR_CUDA;
  if (g_dev[dev].sms == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return LKV_ERR_CUDA;
    g_dev[dev].sms = sms;
  }
  int occ = -1;
#define LKV_OCC(DD, GG, SS) occ = prepare_kernel<DD, GG, SS>(dev)
  if (d == 128) {
    switch (group) {
      case 1: LKV_OCC(128, 1, 3); break;
      case 2: LKV_OCC(128, 2, 3); break;
      case 4: LKV_OCC(128, 4, 3); break;
      default: LKV_OCC(128, 8, 3); break;
    }
  } else {
    switch (group) {
      case 1: LKV_OCC(64, 1, 4); break;
      case 2: LKV_OCC(64, 2, 4); break;
      case 4: LKV_OCC(64, 4, 4); break;
      default: LKV_OCC(64, 8, 4); break;
    }
  }
#undef LKV_OCC
  if (occ < 0) return LKV_ERR_CUDA;
  const int64_t rows = (int64_t)batch * hq;
  const size_t avail = workspace_bytes > kWorkspaceHeader ? workspace_bytes - kWorkspaceHeader : 0;
  const int smax = (int)std::min<size_t>(kMaxSplits, avail / decode_split_bytes(rows, d));
  const int S = std::min(std::max(smax, 1), choose_splits(batch * hkv, max_pages, g_dev[dev].sms * occ));
  *splits = S;
  *launches = (S == 1 && !partial) ? 1 : 2;
  return LKV_OK;
}

int merge_partials(const float* o_parts, const float* lse_parts, int num_parts, int64_t rows, int head_dim, int hq,
                   int64_t o_part_stride, int64_t lse_part_stride, const float* out_scale, void* out,
                   float* lse_out, cudaStream_t stream, int64_t out_stride_tok) {
  if (head_dim != 64 && head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (num_parts < 1 || rows < 0 || hq < 1 || rows % hq) return LKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return LKV_OK;
  if (!o_parts || !lse_parts || !out) return LKV_ERR_INVALID_ARGUMENT;
  if (o_part_stride == 0) o_part_stride = rows * head_dim;
  if (lse_part_stride == 0) lse_part_stride = rows;
  if (o_part_stride < rows * head_dim || lse_part_stride < rows || (o_part_stride & 3))
    return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(o_parts) & 15) || (reinterpret_cast<uintptr_t>(out) & 3))
    return LKV_ERR_INVALID_ARGUMENT;
  MergeParams mp{};
  mp.part_o = o_parts;
  mp.part_lse = lse_parts;
  mp.S = num_parts;
  mp.rows = rows;
  mp.split_major = 1;
  mp.o_part_stride = o_part_stride;
  mp.lse_part_stride = lse_part_stride;
  mp.lse_log2 = 0;
  mp.Hq = hq;
  mp.out_scale = out_scale;
  mp.out = static_cast<__nv_bfloat16*>(out);
  if (out_stride_tok == 0) out_stride_tok = (int64_t)hq * head_dim;
  if (out_stride_tok < (int64_t)hq * head_dim || (out_stride_tok & 1)) return LKV_ERR_INVALID_ARGUMENT;
  mp.out_stride_tok = out_stride_tok;
  mp.lse_out = lse_out;
  const unsigned blocks = (unsigned)((rows + 3) / 4);
  const cudaError_t e = head_dim == 128 ? launch_pdl(merge_partials_kernel<128>, dim3(blocks), dim3(128), 0, stream, mp)
                                         : launch_pdl(merge_partials_kernel<64>, dim3(blocks), dim3(128), 0, stream, mp);
  return e == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

}  // namespace lkv
