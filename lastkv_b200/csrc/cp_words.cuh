// Context-parallel exchange words and the rank-order merge of one output row,
// shared by cp_combine_kernel and the fused mode of decode_splitkv_kernel so
// both produce the same bits.
//
// A receive buffer holds, per epoch-parity slot and per rank, that rank's
// merged partial as 8-byte words {value (fp32 bits), epoch}: o at row * D + d,
// natural-log LSE at rows * D + row.  An aligned 8-byte store arrives whole,
// so a word is valid once its epoch half matches - no fence or flag needed.
#pragma once

#include "common.cuh"

namespace lkv {

__device__ __forceinline__ uint64_t ll_word(float v, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | (uint64_t)__float_as_uint(v);
}

__device__ __forceinline__ void st_ll2(uint64_t* dst, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ uint64_t ld_ll(const uint64_t* src) {
  uint64_t v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
  return v;
}

__device__ __forceinline__ void ld_ll2(const uint64_t* src, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
}

// Poll one word until it carries `epoch` (or the wall-time limit passes: then `fail` is set).
__device__ __forceinline__ float ll_take(const uint64_t* src, uint32_t epoch, uint64_t start, bool& fail) {
  uint64_t w = ld_ll(src);
  for (uint32_t it = 1; (uint32_t)(w >> 32) != epoch && !fail; ++it) {
    if ((it & 255u) == 0 && global_timer_ns() - start > kWaitLimitNs) fail = true;
    w = ld_ll(src);
  }
  return __uint_as_float((uint32_t)w);
}

// One warp merges output row `row` over the `world` ranks' partials in rank
// order (merge_partials_kernel's arithmetic: log2 weights against the row max,
// fp32 sums, one 1/L), scales by out_scale[head] and writes bf16.  Rank s's
// partial comes from slot_base + s * part_words, polled for `epoch`, except
// that `own` (this rank's packed partial o | lse, or null) replaces the rank
// `rank` entry when given.  The words are requested together - the o words of
// the first four ranks with every rank's LSE (lane s reads rank s), then four
// ranks at a time - and only a word that has not arrived yet is polled again,
// so a row costs a few memory round trips rather than one per word.
template <int D>
__device__ __forceinline__ void cp_merge_row(const uint64_t* slot_base, int64_t part_words, int world, int rank,
                                             const float* own, int64_t rows, int64_t row, int Hq,
                                             const float* out_scale, __nv_bfloat16* out, int64_t out_stride_tok,
                                             uint32_t epoch, uint64_t start, bool& fail, int lane) {
  constexpr int PER = D / 32;
  constexpr int G = 8;  // ranks whose o words are in flight together
  constexpr float to2 = 1.4426950408889634f;
  const int64_t lse_off = rows * D;
  uint64_t wv[G][PER];
  auto load_words = [&](int s0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int s = s0 + g;
#pragma unroll
      for (int e = 0; e < PER; ++e) wv[g][e] = 0;
      if (s < world && !(s == rank && own)) {
        const uint64_t* src = slot_base + (int64_t)s * part_words + row * D + lane * PER;
#pragma unroll
        for (int e = 0; e < PER; e += 2) ld_ll2(src + e, wv[g][e], wv[g][e + 1]);
      }
    }
  };
  load_words(0);            // requested together with the LSE words below
  float my_ls = -INFINITY;  // lane s < world: rank s's LSE in log2 units
  if (lane < world)
    my_ls = ((lane == rank && own) ? own[lse_off + row]
                                   : ll_take(slot_base + (int64_t)lane * part_words + lse_off + row, epoch, start,
                                             fail)) *
            to2;
  float M = my_ls;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float acc[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) acc[e] = 0.f;
  float L = 0.f;
  if (M != -INFINITY) {
    for (int s0 = 0; s0 < world; s0 += G) {
      if (s0 > 0) load_words(s0);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int s = s0 + g;
        if (s >= world) break;
        const float ls = __shfl_sync(0xffffffffu, my_ls, s);
        if (ls == -INFINITY) continue;
        const float w = exp2f(ls - M);
        L += w;
        float v[PER];
        if (s == rank && own) {
#pragma unroll
          for (int e = 0; e < PER; ++e) v[e] = own[row * D + lane * PER + e];
        } else {
          const uint64_t* src = slot_base + (int64_t)s * part_words + row * D + lane * PER;
#pragma unroll
          for (int e = 0; e < PER; ++e)
            v[e] = (uint32_t)(wv[g][e] >> 32) == epoch ? __uint_as_float((uint32_t)wv[g][e])
                                                       : ll_take(src + e, epoch, start, fail);
        }
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] += w * v[e];
      }
    }
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  const int h = (int)(row % Hq);
  const int64_t tok = row / Hq;
  const float sc = (out_scale ? out_scale[h] : 1.f) * inv;
  __nv_bfloat16* dst = out + tok * out_stride_tok + (int64_t)h * D + lane * PER;
#pragma unroll
  for (int e = 0; e < PER; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16(acc[e] * sc, acc[e + 1] * sc);
}

}  // namespace lkv
