// Chunked (varlen) prefill over the shared last-layer paged K/V pool on
// 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Reference semantics: the merged per-layer attention call of the vLLM fast
// path for prefill spans (vllm/src/lastkv/vllm/backends/rmarin_flashinfer/
// fastpath.py:643-650: FA3 varlen, block_table = bt_all[l], seqused_k,
// causal with bottom-right alignment) followed by head_scale_
// (fused_qkv.py:140-155); at the HF level the masked SDPA of
// LastKVAttention.forward (llm/src/lastkv/llm/modeling.py:124-146).  The
// non-causal form serves block attention over a shared history (Wan,
// videogen/src/lastkv/videogen/attention.py:9-32).
//
// Work unit: one CTA = two 128-row query tiles (A, B) x one KV head x one
// sequence.  Rows pack TOK = 128 / GROUP query tokens times the GROUP query
// heads that share the KV head (row r -> token r / GROUP, head r % GROUP);
// tile B holds the TOK tokens after tile A.  Every K/V block brought on chip
// serves 256 rows (the whole GQA group of 2 TOK tokens).
//
// Warp roles (384 threads; warp w runs on SM sub-partition w % 4):
//   warps 0-3  softmax + epilogue of tile A, one thread per row (TMEM lane)
//   warps 4-7  softmax + epilogue of tile B
//   warps 8,10 TMA producers of the K blocks (128 keys = 8 pages): pages 0-3
//              and 4-7 of every block, each arriving with its half of the bytes
//   warp 9     TMA producer: the Q tiles once, then the V blocks
//              (so the first S waits for 8 copies per thread, not Q + 16)
//   warp 11    TMEM allocator and MMA issuer: the whole warp runs the issue
//              loop (warp-uniform descriptors, no per-MMA rebuild) and one
//              elected lane issues every tcgen05.mma / commit
// TMEM columns: S_A [0,128), S_B [128,256), O_A [256,256+D), O_B [256+D, 256+2D).
// Per key block j the MMA thread issues, in order,
//   PV_A(j-1), S_A(j), PV_B(j-1), S_B(j)
// (S = Q K^T: A = Q, B = K, both K-major in smem; PV: A = P read from TMEM,
// B = V MN-major in smem), so while one tile's softmax runs the tensor core
// works on the other tile.  P (bf16, two per column) overwrites the first 64
// columns of its own tile's S; the next S of that tile is issued after the PV
// that reads P, and tcgen05.mma from one thread executes in issue order.
// K and V stream through separate rings (2 and 3 stages).  A bf16 tile whose
// rows are all tokens of the span is written back through shared memory (its Q
// buffer) and one TMA store per warp and 64-column half; ragged tiles and fp32
// split partials store row by row (a warp store then touches 32 rows, which cost ~2,600 cycles per tile, on
// the critical path of the CTA's last tile).  The running max is
// only raised (and O rescaled in TMEM) when a row's max grows by more than
// 2^8; otherwise exp2 is taken against the stale max, which stays exact
// because the final normalisation uses the same reference.  The softmax takes
// a quarter of its exponentials on the FMA pipe (ex2_poly2) and the rest on the
// SFU, and stores P in 32-key chunks as they are ready.
//
// Key splits (non-causal calls, S > 1): blockIdx.z = sequence * S + split and
// a CTA covers its split's share of the key blocks, writing the normalised
// fp32 partial and natural-log LSE of its rows; merge_partials_kernel then
// combines the splits exactly.  With one CTA per SM, this fills the last wave
// of a grid of few, long CTAs (Wan's block attention).

#include <math.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace lkv {

namespace {

constexpr int kBM = 128;  // rows per tile
constexpr int kTiles = 2;  // query tiles per CTA
constexpr int kBN = 128;  // keys per block
constexpr int kPageTok = 16;
constexpr int kPagesPerBlock = kBN / kPageTok;
constexpr int kWarpK = 8, kWarpV = 9, kWarpK2 = 10, kWarpMma = 11;
constexpr int kThreads = 12 * 32;
constexpr int kStagesK = 2, kStagesV = 3;
constexpr float kRescaleLog2 = 8.0f;
constexpr int kMaxKvSplits = 8;

struct PrefillParams {
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* seq_k;
  const int32_t* cu_q;
  __nv_bfloat16* out;
  int64_t out_stride_tok;
  float* lse;
  const float* out_scale;
  int* err;
  int B, Hq, Hkv, W;
  int64_t num_pages;
  int causal;
  float scale_log2;
  int S;                 // key splits: blockIdx.z = sequence * S + split
  float* part_o;         // S > 1: fp32 partials [S][rows][D], rows = token * Hq + head
  float* part_lse;       // S > 1: natural-log LSE [S][rows]
  int64_t part_rows;     // rows per split
  int tma_out;           // S == 1 and the output map is valid: full tiles leave by TMA stores
};

template <int D>
struct PrefillCfg {
  static constexpr int HALVES = D / 64;
  static constexpr int Q_HALF = kBM * 128;   // [128 rows][64 bf16]
  static constexpr int KV_HALF = kBN * 128;  // [128 keys][64 bf16]
  static constexpr int Q_BYTES = HALVES * Q_HALF;  // one tile
  static constexpr int KV_BYTES = HALVES * KV_HALF;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + kTiles * Q_BYTES;
  static constexpr int OFF_V = OFF_K + kStagesK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + kStagesV * KV_BYTES;
  static constexpr int BAR_BYTES = 512;
  // At least 120 KB so a second CTA never shares the SM (each CTA holds all 512 TMEM columns).
  static constexpr int SMEM_BYTES =
      (1024 + OFF_BAR + BAR_BYTES) > 120 * 1024 ? (1024 + OFF_BAR + BAR_BYTES) : 120 * 1024;
  static constexpr uint32_t IDESC_S = umma_idesc_bf16(kBM, kBN, 0, 0);
  static constexpr uint32_t IDESC_PV = umma_idesc_bf16(kBM, D, 0, 1);
  static constexpr uint32_t COL_S = 0;        // + tile * kBN
  static constexpr uint32_t COL_O = 2 * kBN;  // + tile * D
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kStagesK], k_empty[kStagesK];
  uint64_t v_full[kStagesV], v_empty[kStagesV];
  uint64_t s_full[kTiles];   // MMA -> softmax: S_t(j) complete
  uint64_t p_full[kTiles];   // softmax -> MMA: P_t(j) stored in TMEM (4 warp arrivals)
  uint64_t pv_done[kTiles];  // MMA -> softmax: PV_t(j) complete
  uint32_t tmem_addr;
  int fail;
};

template <int D, int GROUP>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tcgen05_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                           const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmo,
                           const PrefillParams p) {
  using Cfg = PrefillCfg<D>;
  constexpr int TOK = kBM / GROUP;  // tokens per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + Cfg::OFF_BAR);

  const int cta_tile = blockIdx.x, hk = blockIdx.y, b = blockIdx.z / p.S, split = blockIdx.z % p.S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = p.cu_q[b];
  const int Lq = p.cu_q[b + 1] - q0;
  const int t0 = cta_tile * kTiles * TOK;
  if (t0 >= Lq) return;
  // A trailing tile with no valid token (the last CTA of a span whose length is
  // not a multiple of the CTA's tokens) is skipped: no Q load, MMAs or softmax.
  const int ntiles = (t0 + TOK < Lq) ? kTiles : 1;
  const int n = p.seq_k[b];
  const int t_end = min(t0 + kTiles * TOK, Lq);
  int lim_max = p.causal ? n - Lq + t_end - 1 : n - 1;
  lim_max = min(lim_max, n - 1);
  // Key blocks [j0, j0 + nb) of this CTA: all visible blocks, or this split's share
  // of them (non-causal calls with S > 1).
  const int nb_all = lim_max >= 0 ? lim_max / kBN + 1 : 0;
  const int per_split = (nb_all + p.S - 1) / p.S;
  const int j0 = min(nb_all, split * per_split);
  const int nb = min(nb_all, j0 + per_split) - j0;
  if (nb == 0) {
    // no visible keys: zero output rows (and -inf LSE), as an empty softmax
    for (int r = threadIdx.x; r < kTiles * TOK * GROUP; r += kThreads) {
      const int tok = t0 + r / GROUP;
      if (tok >= Lq) continue;
      const int hq = hk * GROUP + r % GROUP;
      const int64_t row = (int64_t)(q0 + tok) * p.Hq + hq;
      if (p.S > 1) {
        float* o = p.part_o + ((int64_t)split * p.part_rows + row) * D;
        for (int d = 0; d < D; ++d) o[d] = 0.f;
        p.part_lse[(int64_t)split * p.part_rows + row] = -INFINITY;
        continue;
      }
      __nv_bfloat16* o = p.out + (int64_t)(q0 + tok) * p.out_stride_tok + (int64_t)hq * D;
      for (int d = 0; d < D; ++d) o[d] = __float2bfloat16_rn(0.f);
      if (p.lse) p.lse[row] = -INFINITY;
    }
    return;
  }
  const int npages = min((n + kPageTok - 1) / kPageTok, p.W);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStagesK; ++s) {
      mbar_init(&bars->k_full[s], 2);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < kStagesV; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 4);
      mbar_init(&bars->pv_done[t], 1);
    }
    bars->fail = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(&bars->tmem_addr, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_addr;

  uint8_t* sQ = smem + Cfg::OFF_Q;
  uint8_t* sK = smem + Cfg::OFF_K;
  uint8_t* sV = smem + Cfg::OFF_V;
  const int32_t* btrow = p.bt + (int64_t)b * p.bt_stride;

  if (warp == kWarpK || warp == kWarpK2 || warp == kWarpV) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      const bool is_k = warp != kWarpV;
      const int stages = is_k ? kStagesK : kStagesV;
      const CUtensorMap* map = is_k ? &tmk : &tmv;
      const int pg0 = warp == kWarpK2 ? kPagesPerBlock / 2 : 0;
      const int npg = is_k ? kPagesPerBlock / 2 : kPagesPerBlock;
      tma_prefetch_desc(map);
      if (!is_k) {
        tma_prefetch_desc(&tmq);
        mbar_arrive_expect_tx(&bars->q_full, ntiles * Cfg::Q_BYTES);
        for (int t = 0; t < ntiles; ++t)
#pragma unroll
          for (int h = 0; h < Cfg::HALVES; ++h)
            tma_load_3d(sQ + t * Cfg::Q_BYTES + h * Cfg::Q_HALF, &tmq, &bars->q_full, h * 64, hk * GROUP,
                        q0 + t0 + t * TOK);
      }
      uint64_t* full = is_k ? bars->k_full : bars->v_full;
      uint64_t* empty = is_k ? bars->k_empty : bars->v_empty;
      uint8_t* ring = is_k ? sK : sV;
      for (int j = 0; j < nb; ++j) {
        const int s = j % stages;
        if (!mbar_wait(&empty[s], ((j / stages) & 1) ^ 1)) {
          report_error(p.err, DEVERR_WAIT_TIMEOUT, 4, j);
          bars->fail = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], npg * (Cfg::KV_BYTES / kPagesPerBlock));
        uint8_t* dst = ring + s * Cfg::KV_BYTES;
        for (int pg = pg0; pg < pg0 + npg; ++pg) {
          const int pi = (j0 + j) * kPagesPerBlock + pg;
          int pid = (int)p.num_pages;  // past the pool: TMA fills zeros
          if (pi < npages) {
            pid = btrow[pi];
            if (is_k && (pid < 0 || (int64_t)pid >= p.num_pages)) report_error(p.err, DEVERR_BAD_PAGE, 4, pid);
          }
#pragma unroll
          for (int h = 0; h < Cfg::HALVES; ++h)
            tma_load_4d(dst + h * Cfg::KV_HALF + pg * (kPageTok * 128), map, &full[s], h * 64, hk, 0, pid);
        }
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    const bool leader = elect_one();
    // Descriptors of each operand's first 16-element K slice; the slices and
    // ring stages are constant offsets (16-byte units) from them.
    const uint64_t qd = umma_sdesc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t kd = umma_sdesc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t vd = umma_sdesc_sw128(smem_u32(sV), Cfg::KV_HALF, 1024);
    auto issue_s = [&](int t, int j) {
      const uint64_t kb = kd + (uint64_t)(((j % kStagesK) * Cfg::KV_BYTES) >> 4);
      const uint64_t qb = qd + (uint64_t)((t * Cfg::Q_BYTES) >> 4);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const uint32_t oq = ((ks >> 2) * Cfg::Q_HALF + (ks & 3) * 32) >> 4;
        const uint32_t okv = ((ks >> 2) * Cfg::KV_HALF + (ks & 3) * 32) >> 4;
        if (leader) umma_bf16_ss(tmem + Cfg::COL_S + t * kBN, qb + oq, kb + okv, Cfg::IDESC_S, ks > 0 ? 1u : 0u);
      }
      if (leader) umma_commit(&bars->s_full[t]);
    };
    auto issue_pv = [&](int t, int j) {
      const uint64_t vb = vd + (uint64_t)(((j % kStagesV) * Cfg::KV_BYTES) >> 4);
#pragma unroll
      for (int ks = 0; ks < kBN / 16; ++ks)
        if (leader)
          umma_bf16_ts(tmem + Cfg::COL_O + t * D, tmem + Cfg::COL_S + t * kBN + ks * 8,
                       vb + (uint64_t)((ks * (kPageTok * 128)) >> 4), Cfg::IDESC_PV, (j > 0 || ks > 0) ? 1u : 0u);
      if (leader) umma_commit(&bars->pv_done[t]);
    };
    // Wait results are made warp-uniform so the whole warp leaves together.
    bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->q_full, 0));
    for (int j = 0; ok && j <= nb; ++j) {
      // PV_A(j-1), S_A(j), PV_B(j-1), S_B(j)
      if (j < nb) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->k_full[j % kStagesK], (j / kStagesK) & 1));
        tc_fence_after();
        if (!ok) break;
      }
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->v_full[(j - 1) % kStagesV], ((j - 1) / kStagesV) & 1));
        if (!ok) break;
      }
      for (int t = 0; t < ntiles; ++t) {
        if (j > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(&bars->p_full[t], (j - 1) & 1));
          tc_fence_after();
          if (!ok) break;
          issue_pv(t, j - 1);
        }
        if (j < nb) issue_s(t, j);
      }
      if (!ok) break;
      if (leader) {
        if (j < nb) umma_commit(&bars->k_empty[j % kStagesK]);
        if (j > 0) umma_commit(&bars->v_empty[(j - 1) % kStagesV]);
      }
    }
    if (!ok && leader) {
      report_error(p.err, DEVERR_WAIT_TIMEOUT, 4, 100);
      bars->fail = 1;
    }
  } else if ((warp >> 2) < ntiles) {
    // ------------------------------------------------------------ softmax (rows)
    const int t = warp >> 2;                       // tile
    const int r = (warp & 3) * 32 + lane;          // TMEM lane = row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_s = Cfg::COL_S + t * kBN, col_o = Cfg::COL_O + t * D;
    const int tok = t0 + t * TOK + r / GROUP;
    int lim = p.causal ? n - Lq + tok : n - 1;
    lim = min(lim, n - 1);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    const float sl2 = p.scale_log2;
    // Wait results are made warp-uniform: tcgen05.ld/st below are warp-collective.
    for (int j = 0; j < nb; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bars->s_full[t], j & 1));
      tc_fence_after();
      if (!ok) break;
      // raw scores; the softmax scale is folded into one FFMA per element below
      float x[kBN];
      {
        uint32_t raw[kBN / 32][32];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tmem_ld32(lane_base + col_s + c * 32, raw[c]);
        tmem_wait_ld();  // one wait for all four loads
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(raw[c][e]);
      }
      const int key0 = (j0 + j) * kBN;
      if (key0 + kBN - 1 > lim) {
#pragma unroll
        for (int e = 0; e < kBN; ++e)
          if (key0 + e > lim) x[e] = -INFINITY;
      }
      // 8 independent partial maxima (short dependency chains, three-input max), then a tree
      float mp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mp[u] = fmaxf(x[u], x[kBN - 8 + u]);
#pragma unroll
      for (int e = 8; e + 16 <= kBN - 8; e += 16)
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = fmax3f(mp[u], x[e + u], x[e + 8 + u]);
      float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      mx *= sl2;  // scale > 0, so max commutes with it
      float alpha = 1.f;
      if (mx > m + kRescaleLog2) {
        alpha = (m == -INFINITY) ? 0.f : ex2_approx(m - mx);
        m = mx;
      }
      const float neg_mref = (m == -INFINITY) ? 0.f : -m;
      const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(neg_mref, neg_mref);
      float2 sp[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      // P(j) (bf16 pairs) over the first 64 columns of this tile's S, which is fully
      // read: 16 columns per 32 keys, stored as each chunk is ready.  f32x2 FFMA /
      // FADD halve the issue slots of the scale-and-subtract and the sums; pairs 0
      // and 1 of every 8 take their exponentials on the FMA pipe, the rest on the SFU.
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t pc[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int e = c * 32 + 2 * q;
          const float2 a = __ffma2_rn(make_float2(x[e], x[e + 1]), sl2v, negm);
          const float2 pv = (q & 7) < 2 ? ex2_poly2(a) : make_float2(ex2_approx(a.x), ex2_approx(a.y));
          sp[q & 3] = __fadd2_rn(sp[q & 3], pv);
          pc[q] = pack_bf16(pv.x, pv.y);
        }
        tmem_st16(lane_base + col_s + c * 16, pc);
      }
      const float sum = ((sp[0].x + sp[0].y) + (sp[1].x + sp[1].y)) + ((sp[2].x + sp[2].y) + (sp[3].x + sp[3].y));
      l = l * alpha + sum;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O holds blocks < j once PV(j-1) is complete; rescale it in TMEM
        ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[t], (j - 1) & 1));
        tc_fence_after();
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t raw[32];
          tmem_ld32(lane_base + col_o + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) raw[e] = __float_as_uint(__uint_as_float(raw[e]) * alpha);
          tmem_st32(lane_base + col_o + c * 32, raw);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[t]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars->pv_done[t], (nb - 1) & 1));
    tc_fence_after();
    if (!ok) {
      report_error(p.err, DEVERR_WAIT_TIMEOUT, 4, 200);
      bars->fail = 1;
    }
    // A bf16 tile whose rows are all tokens of this span leaves through shared
    // memory: each thread writes its row into the tile's Q buffer (free now: the
    // tile's last S MMA completed before its last PV) in the 128-byte-swizzled
    // layout of the Q copy, and each warp stores its 32 rows of a 64-column half
    // with one TMA copy as soon as it has written them - whole lines instead of
    // one 16-byte piece of 32 rows per warp store, and no wait for the other
    // warps.  Ragged tiles (and the fp32 split partials) store row by row.
    const bool staged = p.S == 1 && p.tma_out && t0 + (t + 1) * TOK <= Lq;
    uint8_t* swarp = sQ + t * Cfg::Q_BYTES + (warp & 3) * 32 * 128;  // this warp's 32 rows of half 0
    if (ok) {
      const int hq = hk * GROUP + r % GROUP;
      const bool valid = tok < Lq;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const float lse_e = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
      const int64_t row = (int64_t)(q0 + (valid ? tok : 0)) * p.Hq + hq;
      if (p.S > 1) {
        // this split's normalised partial (fp32) and its natural-log LSE
        float* orow = p.part_o + ((int64_t)split * p.part_rows + row) * D;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
          uint32_t raw[2][32];
          tmem_ld32(lane_base + col_o + h * 64, raw[0]);
          tmem_ld32(lane_base + col_o + h * 64 + 32, raw[1]);
          tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int e = 0; e < 64; e += 4)
              *reinterpret_cast<float4*>(orow + h * 64 + e) =
                  make_float4(__uint_as_float(raw[e >> 5][e & 31]) * inv, __uint_as_float(raw[e >> 5][(e & 31) + 1]) * inv,
                              __uint_as_float(raw[e >> 5][(e & 31) + 2]) * inv,
                              __uint_as_float(raw[e >> 5][(e & 31) + 3]) * inv);
          }
        }
        if (valid) p.part_lse[(int64_t)split * p.part_rows + row] = lse_e;
      } else {
        const float sc = inv * (p.out_scale ? p.out_scale[hq] : 1.f);
        __nv_bfloat16* orow = p.out + (int64_t)(q0 + (valid ? tok : 0)) * p.out_stride_tok + (int64_t)hq * D;
#pragma unroll
        for (int h = 0; h < D / 64; ++h) {
          uint32_t raw[2][32];
          tmem_ld32(lane_base + col_o + h * 64, raw[0]);
          tmem_ld32(lane_base + col_o + h * 64 + 32, raw[1]);
          tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const uint32_t* r8 = &raw[c >> 2][(c & 3) * 8];
              uint4 v;
              v.x = pack_bf16(__uint_as_float(r8[0]) * sc, __uint_as_float(r8[1]) * sc);
              v.y = pack_bf16(__uint_as_float(r8[2]) * sc, __uint_as_float(r8[3]) * sc);
              v.z = pack_bf16(__uint_as_float(r8[4]) * sc, __uint_as_float(r8[5]) * sc);
              v.w = pack_bf16(__uint_as_float(r8[6]) * sc, __uint_as_float(r8[7]) * sc);
              if (staged)
                *reinterpret_cast<uint4*>(swarp + h * Cfg::Q_HALF + lane * 128 + ((c ^ (r & 7)) << 4)) = v;
              else
                *reinterpret_cast<uint4*>(orow + h * 64 + c * 8) = v;
            }
          }
          if (staged) {
            fence_proxy_async_smem();  // this lane's rows, visible to the copy
            __syncwarp();
            if (lane == 0)
              tma_store_3d(&tmo, swarp + h * Cfg::Q_HALF, h * 64, hk * GROUP,
                           q0 + t0 + t * TOK + (warp & 3) * (32 / GROUP));
          }
        }
        if (staged && lane == 0) {
          bulk_commit_group();
          bulk_wait_group_read0();  // shared memory is released when the CTA exits
        }
        if (valid && p.lse) p.lse[row] = lse_e;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kWarpMma) tmem_dealloc(tmem, 512);
}

template <int D, int GROUP>
int launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& to,
                   const PrefillParams& prm, int max_q, cudaStream_t stream) {
  using Cfg = PrefillCfg<D>;
  constexpr int TOK = kTiles * kBM / GROUP;  // query tokens per CTA
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    if (cudaFuncSetAttribute(prefill_tcgen05_kernel<D, GROUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::SMEM_BYTES) != cudaSuccess)
      return LKV_ERR_CUDA;
    attr_done[dev] = true;
  }
  dim3 grid((max_q + TOK - 1) / TOK, prm.Hkv, prm.B * prm.S);
  prefill_tcgen05_kernel<D, GROUP><<<grid, kThreads, Cfg::SMEM_BYTES, stream>>>(tq, tk, tv, to, prm);
  return cudaGetLastError() == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

}  // namespace

int prefill_paged(const PrefillArgs& a) {
  if (a.head_dim != 64 && a.head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (a.num_kv_heads <= 0 || a.num_q_heads <= 0 || a.num_q_heads % a.num_kv_heads) return LKV_ERR_INVALID_ARGUMENT;
  const int group = a.num_q_heads / a.num_kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8) return LKV_ERR_UNSUPPORTED;
  if (a.batch < 0 || a.total_q < 0 || a.max_q < 0 || a.max_pages_per_seq < 0) return LKV_ERR_INVALID_ARGUMENT;
  if (a.batch == 0 || a.total_q == 0 || a.max_q == 0) return LKV_OK;
  if (!a.q || !a.pool_k || !a.pool_v || !a.block_table || !a.seq_k || !a.cu_q || !a.out)
    return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a.q) & 15) || ((a.q_stride_tok * 2) & 15)) return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a.out) & 15) || ((a.out_stride_tok * 2) & 15)) return LKV_ERR_INVALID_ARGUMENT;
  if (a.batch > 65535 || a.num_kv_heads > 65535) return LKV_ERR_UNSUPPORTED;
  if (!a.error_word) return LKV_ERR_INVALID_ARGUMENT;
  const int S = a.kv_splits < 1 ? 1 : a.kv_splits;
  if (S > 1) {
    // key splits need a non-causal call (every query sees the same key range)
    if (a.causal || S > kMaxKvSplits || (int64_t)a.batch * S > 65535) return LKV_ERR_UNSUPPORTED;
    if (!a.part_o || !a.part_lse || (reinterpret_cast<uintptr_t>(a.part_o) & 15)) return LKV_ERR_INVALID_ARGUMENT;
  }

  CUtensorMap tq, tk, tv;
  int st = make_query_tensor_map(&tq, a.q, a.total_q, a.q_stride_tok, a.num_q_heads, a.head_dim, group);
  if (st != LKV_OK) return st;
  st = make_pool_tensor_map(&tk, a.pool_k, a.num_pages, a.num_kv_heads, a.head_dim);
  if (st != LKV_OK) return st;
  st = make_pool_tensor_map(&tv, a.pool_v, a.num_pages, a.num_kv_heads, a.head_dim);
  if (st != LKV_OK) return st;
  // The output has the query's [token][head][dim] geometry: full tiles are stored
  // a warp's 32 rows at a time (unused when the map cannot be built).
  CUtensorMap to;
  memset(&to, 0, sizeof(to));
  const int tma_out = S == 1 && make_query_tensor_map(&to, a.out, a.total_q, a.out_stride_tok, a.num_q_heads,
                                                      a.head_dim, group, 32) == LKV_OK;

  PrefillParams prm{};
  prm.bt = a.block_table;
  prm.bt_stride = a.block_table_stride;
  prm.seq_k = a.seq_k;
  prm.cu_q = a.cu_q;
  prm.out = static_cast<__nv_bfloat16*>(a.out);
  prm.out_stride_tok = a.out_stride_tok;
  prm.lse = a.lse;
  prm.out_scale = a.out_scale;
  prm.err = a.error_word;
  prm.B = a.batch;
  prm.Hq = a.num_q_heads;
  prm.Hkv = a.num_kv_heads;
  prm.W = a.max_pages_per_seq;
  prm.num_pages = a.num_pages;
  prm.causal = a.causal ? 1 : 0;
  prm.scale_log2 = a.softmax_scale * 1.4426950408889634f;
  prm.S = S;
  prm.part_o = a.part_o;
  prm.part_lse = a.part_lse;
  prm.part_rows = (int64_t)a.total_q * a.num_q_heads;
  prm.tma_out = tma_out;
  cudaStream_t stream = static_cast<cudaStream_t>(a.stream);
  int rc = LKV_OK;
#define LKV_PF(DD, GG) rc = launch_prefill<DD, GG>(tq, tk, tv, to, prm, a.max_q, stream); break
  if (a.head_dim == 128) {
    switch (group) {
      case 1: LKV_PF(128, 1);
      case 2: LKV_PF(128, 2);
      case 4: LKV_PF(128, 4);
      default: LKV_PF(128, 8);
    }
  } else {
    switch (group) {
      case 1: LKV_PF(64, 1);
      case 2: LKV_PF(64, 2);
      case 4: LKV_PF(64, 4);
      default: LKV_PF(64, 8);
    }
  }
#undef LKV_PF
  if (rc != LKV_OK || S == 1) return rc;
  // exact LSE merge of the splits into out (x out_scale) and lse
  return merge_partials(a.part_o, a.part_lse, S, prm.part_rows, a.head_dim, a.num_q_heads,
                        prm.part_rows * a.head_dim, prm.part_rows, a.out_scale, a.out, a.lse, stream,
                        a.out_stride_tok);
}

// Key splits for a non-causal call: with one CTA per SM, a grid of C CTAs runs
// ceil(C / SMs) waves of equal CTAs of `blocks` key blocks; splitting the keys S
// ways gives S * C CTAs of blocks / S, ceil(S * C / SMs) / S waves, plus per
// extra split the partials' write and merge and the extra CTAs' start-up, about
// 28 block-times (measured on the Wan-1.3B shape: 456 CTAs x 256 blocks ran
// 1.80 / 1.70 / 1.68 / 1.69 / 1.71 / 1.81 ms at S = 1 / 2 / 3 / 4 / 5 / 8).
// Short key ranges (under 16 blocks per split) are not split.
int prefill_split_plan(int batch, int max_q, int num_q_heads, int num_kv_heads, int head_dim, int max_pages,
                       int causal, int* kv_splits) {
  if (!kv_splits) return LKV_ERR_INVALID_ARGUMENT;
  *kv_splits = 1;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads) return LKV_ERR_INVALID_ARGUMENT;
  if (head_dim != 64 && head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (causal || batch <= 0 || max_q <= 0 || max_pages <= 0) return LKV_OK;
  const int group = num_q_heads / num_kv_heads;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return LKV_ERR_CUDA;
  const int64_t tok_per_cta = (int64_t)kTiles * kBM / group;
  const int64_t ctas = (max_q + tok_per_cta - 1) / tok_per_cta * num_kv_heads * batch;
  const int64_t blocks = ((int64_t)max_pages * kPageTok + kBN - 1) / kBN;
  double best = 1e30;
  for (int s = 1; s <= kMaxKvSplits; ++s) {
    if (s > 1 && (blocks / s < 16 || (int64_t)batch * s > 65535)) break;
    const double waves = (double)((ctas * s + sms - 1) / sms) / s;
    const double cost = waves * (double)blocks + 28.0 * (s - 1);
    if (cost < best - 1e-9) {
      best = cost;
      *kv_splits = s;
    }
  }
  return LKV_OK;
}

}  // namespace lkv
