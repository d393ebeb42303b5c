// Decode-shaped weight GEMM on tcgen05 (sm_100a): y[m, n] = sum_k x[m, k] * w[n, k]
// for m <= 16 rows of activations (one decode token per sequence) against a
// bf16 weight matrix w [n_rows, k] (the nn.Linear layout).
//
// At decode batch sizes the GEMM is a weight stream: every weight byte is read
// once and the arithmetic is 16 FLOP per weight element at most.  The tile is
// therefore "swapped": 128 weight rows are the UMMA M side and the (zero-padded)
// 16 activation rows the N side, D = W_tile . X^T accumulates in 16 TMEM columns.
// Both operands are TMA-loaded, 128-byte swizzled and K-major, 64 columns of k
// (one 128-byte row) per pipeline stage; the weight loads carry an evict-first
// L2 hint.  One thread produces, one thread issues tcgen05.mma, then all four
// warps read their 32 TMEM lanes each for the epilogue.  Launched with PDL: the
// first stages' weights stream in while the previous kernel drains; the
// activation loads and every global write wait for it (griddepcontrol.wait).
//
// Split-K inside a thread-block cluster: when the tiles alone do not fill the
// GPU, the k range of each tile is split over the CTAs of one cluster (<= 8,
// co-scheduled by the hardware).  Each CTA leaves its fp32 partial tile in its
// own shared memory; after a cluster barrier every CTA reduces a slice of the
// tile's rows from all partials over distributed shared memory, adding them in
// split order (results do not depend on timing), and a second barrier keeps
// the partials alive until all CTAs are done.  No global scratch, no atomics.
//
// Epilogues (the rounding points of the eager torch modules):
//   LKV_GEMM_PLAIN     y = bf16(acc)                                 (nn.Linear)
//   LKV_GEMM_SILU_MUL  w = [gate (F rows) | up (F rows)]; a tile pairs 64 gate
//                      rows with the matching 64 up rows and writes
//                      y[m, j] = bf16(bf16(silu(bf16(g))) * bf16(u))  for j < F
//                      (F.silu(gate_proj(x)) * up_proj(x) in bf16).

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "tcgen05.cuh"

namespace lkv {

namespace {

constexpr int kRows = 128;    // weight rows per tile (UMMA M)
constexpr int kBatch = 16;    // activation rows (UMMA N), zero-padded
constexpr int kKB = 64;       // k per stage: one 128-byte swizzled row
constexpr int kStages = 5;    // 93 KB: two CTAs share an SM
constexpr int kThreads = 128;
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kWStage = kRows * 128;
constexpr int kXStage = kBatch * 128;
constexpr int kStageBytes = kWStage + kXStage;
constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256;
constexpr int kTmemCols = 32;
constexpr uint32_t kIdesc = umma_idesc_bf16(kRows, kBatch, 0, 0);
constexpr int kKernelId = 7;

struct GemmParams {
  __nv_bfloat16* y;
  int64_t y_row;
  int m;          // activation rows (1..16)
  int n_out;      // output columns
  int half_rows;  // SILU_MUL: F (the up rows start there)
  int kb_total;
  int splits;     // = cluster size along y
  int mode;
  int* err;
};

struct GemmBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc;
  uint32_t tmem;
};

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();  // the barrier is .aligned: every warp arrives converged
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Sum over the cluster's partials (split order) of element `e` of the [kBatch][kRows] partial tile.
__device__ __forceinline__ float cluster_sum(uint32_t part, int splits, int e) {
  float v[kMaxSplits];
#pragma unroll
  for (int s = 0; s < kMaxSplits; ++s) v[s] = s < splits ? dsmem_ld(dsmem_map(part, s) + e * 4) : 0.f;
  float sum = 0.f;
#pragma unroll
  for (int s = 0; s < kMaxSplits; ++s)
    if (s < splits) sum += v[s];
  return sum;
}

__device__ __forceinline__ float silu_mul_round(float g_acc, float u_acc) {
  const float g = bf16_round(g_acc);
  const float s = bf16_round(g / (1.0f + expf(-g)));
  return s * bf16_round(u_acc);
}

__global__ void __launch_bounds__(kThreads, 2)
    decode_gemm_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                       const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmBars* bars = reinterpret_cast<GemmBars*>(smem + kStages * kStageBytes);
  const int tile = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb0 = (int)((int64_t)p.kb_total * split / p.splits);
  const int kb1 = (int)((int64_t)p.kb_total * (split + 1) / p.splits);
  const int nkb = kb1 - kb0;
  // weight rows loaded into the two 64-row halves of the tile
  const int r_lo = p.mode == LKV_GEMM_SILU_MUL ? tile * 64 : tile * kRows;
  const int r_hi = p.mode == LKV_GEMM_SILU_MUL ? p.half_rows + tile * 64 : tile * kRows + 64;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA producer
    tma_prefetch_desc(&tmw);
    tma_prefetch_desc(&tmx);
    const uint64_t pol = policy_evict_first();
    // The weights do not depend on the previous kernel: fill every stage's weight
    // half before waiting for it (PDL), then add the activation tiles.
    const int pre = nkb < kStages ? nkb : kStages;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&bars->full[i], kWStage + p.m * 128);
      tma_load_2d_hint(smem + i * kStageBytes, &tmw, &bars->full[i], (kb0 + i) * kKB, r_lo, pol);
      tma_load_2d_hint(smem + i * kStageBytes + kWStage / 2, &tmw, &bars->full[i], (kb0 + i) * kKB, r_hi, pol);
    }
    pdl_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem + i * kStageBytes + kWStage, &tmx, &bars->full[i], (kb0 + i) * kKB, 0);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&bars->empty[s], ((i / kStages) & 1) ^ 1)) {
        report_error(p.err, DEVERR_WAIT_TIMEOUT, kKernelId, i);
        break;
      }
      mbar_arrive_expect_tx(&bars->full[s], kWStage + p.m * 128);
      uint8_t* st = smem + s * kStageBytes;
      const int kc = (kb0 + i) * kKB;
      tma_load_2d_hint(st, &tmw, &bars->full[s], kc, r_lo, pol);
      tma_load_2d_hint(st + kWStage / 2, &tmw, &bars->full[s], kc, r_hi, pol);
      tma_load_2d(st + kWStage, &tmx, &bars->full[s], kc, 0);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA issuer
    const uint32_t base = smem_u32(smem);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&bars->full[s], (i / kStages) & 1)) {
        report_error(p.err, DEVERR_WAIT_TIMEOUT, kKernelId, 1000000 + i);
        break;
      }
      tc_fence_after();
      const uint32_t a0 = base + s * kStageBytes, b0 = a0 + kWStage;
#pragma unroll
      for (int ks = 0; ks < kKB / 16; ++ks)
        umma_bf16_ss(tmem, umma_sdesc_sw128(a0 + ks * 32, 16, 1024), umma_sdesc_sw128(b0 + ks * 32, 16, 1024),
                     kIdesc, (i > 0 || ks > 0) ? 1u : 0u);
      umma_commit(&bars->empty[s]);
    }
    umma_commit(&bars->acc);  // also when the loop stopped early, so the epilogue never waits in vain
  }
  __syncwarp();

  // -------------------------------------------------------------------- epilogue
  const int r = warp * 32 + lane;  // this thread's weight row within the tile (= TMEM lane)
  const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars->acc, 0));
  if (!ok && lane == 0) report_error(p.err, DEVERR_WAIT_TIMEOUT, kKernelId, 2000000 + warp);
  tc_fence_after();
  float acc[kBatch];
  {
    uint32_t v[kBatch];
    tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16), v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < kBatch; ++j) acc[j] = __uint_as_float(v[j]);
  }
  pdl_wait();  // before any global write (y may still be read by the previous kernel)

  // The stage ring is idle once the accumulator is complete (every TMA load was
  // consumed by an MMA that has finished): the epilogue reuses its first bytes.
  float* xs = reinterpret_cast<float*>(smem);  // [kBatch][kRows] fp32
  if (p.splits == 1) {
    if (p.mode == LKV_GEMM_SILU_MUL) {
      if (r >= 64) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j) xs[j * kRows + r] = acc[j];
      }
      __syncthreads();
      const int n = tile * 64 + r;
      if (r < 64 && n < p.n_out) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          if (j < p.m) p.y[(int64_t)j * p.y_row + n] = __float2bfloat16_rn(silu_mul_round(acc[j], xs[j * kRows + r + 64]));
      }
    } else {
      const int n = tile * kRows + r;
      if (n < p.n_out) {
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          if (j < p.m) p.y[(int64_t)j * p.y_row + n] = __float2bfloat16_rn(acc[j]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (j < p.m) xs[j * kRows + r] = acc[j];
    cluster_sync_all();  // every CTA of the tile has published its partial
    const int rank = (int)cluster_rank();
    const uint32_t part = smem_u32(xs);
    if (p.mode == LKV_GEMM_SILU_MUL) {
      const int g0 = rank * 64 / p.splits, ng = (rank + 1) * 64 / p.splits - g0;
      for (int idx = threadIdx.x; idx < ng * p.m; idx += kThreads) {
        const int j = idx / ng, g = g0 + idx % ng;
        const int n = tile * 64 + g;
        const float gs = cluster_sum(part, p.splits, j * kRows + g);
        const float us = cluster_sum(part, p.splits, j * kRows + g + 64);
        if (n < p.n_out) p.y[(int64_t)j * p.y_row + n] = __float2bfloat16_rn(silu_mul_round(gs, us));
      }
    } else {
      const int r0 = rank * kRows / p.splits, nr = (rank + 1) * kRows / p.splits - r0;
      for (int idx = threadIdx.x; idx < nr * p.m; idx += kThreads) {
        const int j = idx / nr, row = r0 + idx % nr;
        const int n = tile * kRows + row;
        const float s = cluster_sum(part, p.splits, j * kRows + row);
        if (n < p.n_out) p.y[(int64_t)j * p.y_row + n] = __float2bfloat16_rn(s);
      }
    }
    cluster_sync_all();  // the partials stay readable until every CTA has reduced its slice
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

struct GemmDev {
  int sms = 0;
  int occ = 0;
};
GemmDev g_gemm_dev[64];
std::mutex g_gemm_mu;

int gemm_device(int* sms, int* occ) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LKV_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_gemm_mu);
  GemmDev& d = g_gemm_dev[dev];
  if (d.sms == 0) {
    int n = 0, o = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return LKV_ERR_CUDA;
    if (cudaFuncSetAttribute(decode_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
        cudaSuccess)
      return LKV_ERR_CUDA;
    // all of the unified L1 as shared memory, so two CTAs share an SM
    if (cudaFuncSetAttribute(decode_gemm_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return LKV_ERR_CUDA;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, decode_gemm_kernel, kThreads, kSmemBytes) != cudaSuccess)
      return LKV_ERR_CUDA;
    // The occupancy query answers one CTA per SM for any kernel that allocates
    // TMEM; two of these CTAs (32 TMEM columns and 93 KB of shared memory each)
    // do share an SM, so plan for what the shared memory allows.
    int smem_sm = 0, reserved = 0;
    if (cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev) != cudaSuccess)
      return LKV_ERR_CUDA;
    const int by_smem = smem_sm / (kSmemBytes + reserved);
    d.sms = n;
    d.occ = std::max(std::min(by_smem, 2), std::max(o, 1));
  }
  *sms = d.sms;
  *occ = d.occ;
  return LKV_OK;
}

struct GemmPlan {
  int tiles, splits, kb_total, n_out;
};

// Split count (a power of two <= 8): minimise (waves) x (k blocks per CTA +
// pipeline fill), as the decode kernel does for its key splits.
GemmPlan plan_gemm(int64_t n_rows, int64_t k, int mode, int slots) {
  GemmPlan g{};
  g.n_out = (int)(mode == LKV_GEMM_SILU_MUL ? n_rows / 2 : n_rows);
  g.tiles = (int)(mode == LKV_GEMM_SILU_MUL ? (g.n_out + 63) / 64 : (n_rows + kRows - 1) / kRows);
  g.kb_total = (int)((k + kKB - 1) / kKB);
  const int fill = 6;
  int64_t best = INT64_MAX;
  g.splits = 1;
  const int smax = std::min(kMaxSplits, g.kb_total);
  // power-of-two cluster sizes pack onto the GPCs' SM pairs without leftovers
  for (int s = 1; s <= smax; s *= 2) {
    const int64_t ctas = (int64_t)g.tiles * s;
    const int64_t waves = (ctas + slots - 1) / slots;
    const int64_t cost = waves * ((g.kb_total + s - 1) / s + fill) + (s > 1 ? 1 : 0);
    if (cost < best) {
      best = cost;
      g.splits = s;
    }
  }
  return g;
}

bool valid_shape(int64_t n_rows, int64_t k, int mode) {
  if (n_rows < 1 || k < 1 || n_rows > (int64_t)0x7fffffff || k > (int64_t)0x7fffffff) return false;
  if (mode != LKV_GEMM_PLAIN && mode != LKV_GEMM_SILU_MUL) return false;
  if (mode == LKV_GEMM_SILU_MUL && (n_rows % 2)) return false;
  return true;
}

}  // namespace

int decode_gemm_plan(int64_t n_rows, int64_t k, int mode, int* tiles, int* splits, int* ctas_per_sm) {
  if (!valid_shape(n_rows, k, mode)) return LKV_ERR_INVALID_ARGUMENT;
  int sms = 0, occ = 0;
  const int st = gemm_device(&sms, &occ);
  if (st != LKV_OK) return st;
  const GemmPlan g = plan_gemm(n_rows, k, mode, sms * occ);
  if (tiles) *tiles = g.tiles;
  if (splits) *splits = g.splits;
  if (ctas_per_sm) *ctas_per_sm = occ;
  return LKV_OK;
}

int decode_gemm(const void* x, int64_t x_row, const void* w, int64_t w_row, void* y, int64_t y_row, int m,
                int64_t n_rows, int64_t k, int mode, int32_t* error_word, cudaStream_t stream, int* splits_out) {
  if (!valid_shape(n_rows, k, mode) || m < 1 || m > kBatch || !x || !w || !y) return LKV_ERR_INVALID_ARGUMENT;
  int sms = 0, occ = 0;
  int st = gemm_device(&sms, &occ);
  if (st != LKV_OK) return st;
  const GemmPlan g = plan_gemm(n_rows, k, mode, sms * occ);
  if (y_row < g.n_out) return LKV_ERR_INVALID_ARGUMENT;
  if (splits_out) *splits_out = g.splits;
  CUtensorMap tmw, tmx;
  st = make_matrix_tensor_map(&tmw, w, n_rows, k, w_row, 64);
  if (st != LKV_OK) return st;
  st = make_matrix_tensor_map(&tmx, x, m, k, x_row, m);
  if (st != LKV_OK) return st;
  GemmParams p{};
  p.y = static_cast<__nv_bfloat16*>(y);
  p.y_row = y_row;
  p.m = m;
  p.n_out = g.n_out;
  p.half_rows = (int)(n_rows / 2);
  p.kb_total = g.kb_total;
  p.splits = g.splits;
  p.mode = mode;
  p.err = error_word;
  return launch_pdl_cluster(decode_gemm_kernel, dim3(g.tiles, g.splits), dim3(kThreads), kSmemBytes, stream,
                            dim3(1, g.splits, 1), tmw, tmx, p) == cudaSuccess
             ? LKV_OK
             : LKV_ERR_CUDA;
}

}  // namespace lkv
