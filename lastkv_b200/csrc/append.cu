// Cache-append epilogue and boundary commit for the merged paged pool (sm_100a).
//
// rope_norm_append_kernel  - one warp per (token, head): NeoX RoPE, then
//   RMSNorm over head_dim for q and k (norm AFTER RoPE, as the published
//   model; llm/src/lastkv/llm/modeling.py:103-106), V scaled by 1/s_l, and the
//   paged stores: normalised q to q_out, k and V/s_l into the layer ring slot,
//   and - for the top layer - raw k and raw V into the shared-history slot.
//   Arithmetic order follows the vLLM fused epilogue
//   (vllm/src/lastkv/vllm/backends/rmarin_flashinfer/fused_qkv.py:23-90):
//   fp32 math, x*c - y*s as one FMA, one bf16 rounding after RoPE, fp32 sum of
//   squares, rsqrt, x*inv*w with one rounding.
// blend_chunk_kernel - at a chunk boundary, ring = a*raw + (1-a)*ring for every
//   layer ring, K and V (V in V/s units), each product rounded to bf16 like the
//   four eager torch ops (fused_qkv.py:158-201, batching.py:1099-1144).
// append_commit_kernel - the append of a step's first layer and the blend of
//   the chunk the previous step finished, in one launch (the reference runs
//   that commit when the next step starts); the blend's row count may be read
//   on the device, so a captured step carries a commit or none.
// build_block_tables_kernel - bt_all[l][b][c] = bt[b][c] for the older pages and
//   bt[b][c] + ring_base[l] for ring pages (fastpath.py:422-424).

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace lkv {

struct AppendParams {
  const __nv_bfloat16* q;
  int64_t q_row;
  const __nv_bfloat16* k;
  int64_t k_row;
  const __nv_bfloat16* v;
  int64_t v_row;
  const int64_t* pos;
  const void* cos_sin;  // bf16 or fp32 [max_pos, D] = cos | sin halves
  int64_t cs_row;
  int interleaved;  // RoPE pairs (2i, 2i+1) instead of (i, i + D/2)
  int cs_fp32;
  int64_t max_pos;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  float eps;
  const float* inv_scale;
  __nv_bfloat16* q_out;
  int64_t q_out_row;
  const int64_t* ring_slot;
  __nv_bfloat16* ring_k;
  __nv_bfloat16* ring_v;
  int64_t ring_slots;
  const int64_t* src_slot;
  __nv_bfloat16* src_k;
  __nv_bfloat16* src_v;
  int64_t src_slots;
  int T, Hq, Hkv;
  int* err;
};

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One 256-thread block of the append: head group `hg` (8 heads, one per warp) of token `t`.
template <int D>
__device__ __forceinline__ void append_block(const AppendParams& p, int hg, int t) {
  constexpr int HALF = D / 2;
  constexpr int E = HALF / 32;  // rotary pairs per lane (2 for D=128, 1 for D=64)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = hg * 8 + warp;
  if (h >= p.Hq + p.Hkv) return;
  const bool is_q = h < p.Hq;
  const int j = h - p.Hq;  // kv head
  const __nv_bfloat16* src = is_q ? p.q + (int64_t)t * p.q_row + (int64_t)h * D : p.k + (int64_t)t * p.k_row + (int64_t)j * D;
  const int i0 = lane * E;
  // element indices of the two members of rotary pair (i0 + e): NeoX halves or interleaved
  auto ix1 = [&](int e) { return p.interleaved ? 2 * (i0 + e) : i0 + e; };
  auto ix2 = [&](int e) { return p.interleaved ? 2 * (i0 + e) + 1 : HALF + i0 + e; };
  float r1[E], r2[E];
  if (p.cos_sin) {
    const int64_t pos = p.pos[t];
    if (pos < 0 || pos >= p.max_pos) {
      if (lane == 0) report_error(p.err, DEVERR_BAD_SLOT, 2, (int)pos);
      return;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float x = __bfloat162float(src[ix1(e)]);
      const float y = __bfloat162float(src[ix2(e)]);
      float cc, sn;
      if (p.cs_fp32) {
        const float* cs = static_cast<const float*>(p.cos_sin) + pos * p.cs_row;
        cc = cs[i0 + e];
        sn = cs[HALF + i0 + e];
      } else {
        const __nv_bfloat16* cs = static_cast<const __nv_bfloat16*>(p.cos_sin) + pos * p.cs_row;
        cc = __bfloat162float(cs[i0 + e]);
        sn = __bfloat162float(cs[HALF + i0 + e]);
      }
      r1[e] = bf16r(__fmaf_rn(x, cc, -__fmul_rn(y, sn)));
      r2[e] = bf16r(__fmaf_rn(y, cc, __fmul_rn(x, sn)));
    }
  } else {  // use_nope: no rotary embedding
#pragma unroll
    for (int e = 0; e < E; ++e) {
      r1[e] = __bfloat162float(src[ix1(e)]);
      r2[e] = __bfloat162float(src[ix2(e)]);
    }
  }
  const __nv_bfloat16* w = is_q ? p.qw : p.kw;
  __nv_bfloat16 o1[E], o2[E];
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      ss = __fmaf_rn(r1[e], r1[e], ss);
      ss = __fmaf_rn(r2[e], r2[e], ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(__fadd_rn(ss / (float)D, p.eps));
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o1[e] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(r1[e], inv), __bfloat162float(w[ix1(e)])));
      o2[e] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(r2[e], inv), __bfloat162float(w[ix2(e)])));
    }
  } else {  // use_qk_norm = False
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o1[e] = __float2bfloat16_rn(r1[e]);
      o2[e] = __float2bfloat16_rn(r2[e]);
    }
  }
  auto store = [&](__nv_bfloat16* dst, const __nv_bfloat16* a, const __nv_bfloat16* b) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      dst[ix1(e)] = a[e];
      dst[ix2(e)] = b[e];
    }
  };
  if (is_q) {
    store(p.q_out + (int64_t)t * p.q_out_row + (int64_t)h * D, o1, o2);
    return;
  }
  const int64_t slot = p.ring_slot[t];
  const bool ring_ok = slot >= 0 && slot < p.ring_slots;
  if (!ring_ok && lane == 0) report_error(p.err, DEVERR_BAD_SLOT, 2, (int)slot);
  const __nv_bfloat16* vsrc = p.v + (int64_t)t * p.v_row + (int64_t)j * D;
  __nv_bfloat16 va[E], vb[E], vsa[E], vsb[E];
  const float is = p.inv_scale ? p.inv_scale[j] : 1.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    va[e] = vsrc[ix1(e)];
    vb[e] = vsrc[ix2(e)];
    vsa[e] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(va[e]), is));
    vsb[e] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(vb[e]), is));
  }
  if (ring_ok) {
    const int64_t off = (slot * p.Hkv + j) * D;
    store(p.ring_k + off, o1, o2);
    store(p.ring_v + off, vsa, vsb);
  }
  if (p.src_slot) {
    const int64_t ss_ = p.src_slot[t];
    if (ss_ >= 0 && ss_ < p.src_slots) {
      const int64_t off = (ss_ * p.Hkv + j) * D;
      store(p.src_k + off, o1, o2);
      store(p.src_v + off, va, vb);
    } else if (lane == 0) {
      report_error(p.err, DEVERR_BAD_SLOT, 2, (int)ss_);
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256) rope_norm_append_kernel(const AppendParams p) {
  pdl_launch_dependents();
  pdl_wait();  // q/k/v come from the projection GEMM
  append_block<D>(p, blockIdx.x, blockIdx.y);
}

struct BlendParams {
  __nv_bfloat16* pool_k;
  __nv_bfloat16* pool_v;
  int64_t num_pages;
  const int32_t* raw_pages;
  const int32_t* ring_pages;
  int64_t ring_stride;
  const float* alpha;
  int ppc, S, L, Hkv, D;
  const int32_t* count;  // append_commit_kernel: device count of rows of raw/ring to commit (NULL = S)
  int* err;
};

// One 256-thread block of the commit: page `jp` of sequence `seq`'s finished chunk in layer `layer`'s ring.
__device__ __forceinline__ void blend_block(const BlendParams& p, int jp, int seq, int layer) {
  const int64_t raw = p.raw_pages[(int64_t)seq * p.ppc + jp];
  const int64_t ring = (int64_t)p.ring_pages[(int64_t)seq * p.ppc + jp] + (int64_t)layer * p.ring_stride;
  if (raw < 0 || raw >= p.num_pages || ring < 0 || ring >= p.num_pages) {
    if (threadIdx.x == 0) report_error(p.err, DEVERR_BAD_PAGE, 3, (int)(raw < 0 || raw >= p.num_pages ? raw : ring));
    return;
  }
  const int64_t page_elems = (int64_t)16 * p.Hkv * p.D;
  const int vecs = (int)(page_elems / 8);
  // the head of vector vi is (8 vi / D) mod Hkv; D divides the 2048 elements a block
  // covers per iteration (D is 64 or 128), so the head advances by a constant step
  const int head0 = (int)((threadIdx.x * 8) / p.D) % p.Hkv;
  const int hstep = (int)((blockDim.x * 8) / p.D) % p.Hkv;
  const float* alpha = p.alpha + layer * p.Hkv;
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {
    __nv_bfloat16* pool = which ? p.pool_v : p.pool_k;
    const uint4* src = reinterpret_cast<const uint4*>(pool + raw * page_elems);
    uint4* dst = reinterpret_cast<uint4*>(pool + ring * page_elems);
    int head = head0;
    for (int vi = threadIdx.x; vi < vecs; vi += blockDim.x) {
      const float a = alpha[head];
      head += hstep;
      if (head >= p.Hkv) head -= p.Hkv;
      const float ia = bf16r(__fsub_rn(1.f, a));
      uint4 rv = src[vi], gv = dst[vi];
      uint32_t* r = reinterpret_cast<uint32_t*>(&rv);
      uint32_t* g = reinterpret_cast<uint32_t*>(&gv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float t1l = bf16r(__fmul_rn(a, bf16_lo(r[e]))), t1h = bf16r(__fmul_rn(a, bf16_hi(r[e])));
        const float t3l = bf16r(__fmul_rn(ia, bf16_lo(g[e]))), t3h = bf16r(__fmul_rn(ia, bf16_hi(g[e])));
        g[e] = pack_bf16(__fadd_rn(t1l, t3l), __fadd_rn(t1h, t3h));
      }
      dst[vi] = gv;
    }
  }
}

// grid (pages_per_chunk, num_seqs, num_layers); one CTA blends one page of one layer.
__global__ void __launch_bounds__(256) blend_chunk_kernel(const BlendParams p) {
  blend_block(p, blockIdx.x, blockIdx.y, blockIdx.z);
}

// The append of the first layer of a step and the commit of the chunks the
// previous step finished, in one launch (the reference commits lazily at the
// next step's start too, batching.py:1099-1144).  Blocks [0, n_append) append
// (head group i % groups, token i / groups); the other gridDim.x - n_append
// blocks stride over the (page, row, layer) items of the commit, whose row
// count is read on the device when `count` is set, so one captured launch
// serves steps with and without a boundary.  Disjoint addresses: the append
// writes this step's slot of each ring, in the other half of the 2C ring from
// the finished chunk the blend rewrites, and the blend's raw pages belong to
// that finished chunk.
template <int D>
__global__ void __launch_bounds__(256, 8) append_commit_kernel(const AppendParams pa, const BlendParams pb,
                                                               int groups, int n_append) {
  pdl_launch_dependents();
  pdl_wait();  // q/k/v come from the projection GEMM; the rings and the commit count from earlier work
  const int i = blockIdx.x;
  if (i < n_append) {
    append_block<D>(pa, i % groups, i / groups);
    return;
  }
  int rows = pb.S;
  if (pb.count) {
    const int c = *pb.count;
    if (c < 0 || c > pb.S) {
      if (i == n_append && threadIdx.x == 0) report_error(pb.err, DEVERR_BAD_SLOT, 3, c);
      return;
    }
    rows = c;
  }
  const int64_t per_layer = (int64_t)pb.ppc * rows;
  const int64_t items = per_layer * pb.L;
  const int nb = gridDim.x - n_append;
  for (int64_t j = i - n_append; j < items; j += nb) {
    const int layer = (int)(j / per_layer);
    const int64_t r = j - layer * per_layer;
    blend_block(pb, (int)(r % pb.ppc), (int)(r / pb.ppc), layer);
  }
}

struct GatherBlendParams {
  __nv_bfloat16* pool_k;
  __nv_bfloat16* pool_v;
  int64_t num_slots;
  const int64_t* dst;
  const int64_t* src_a;
  const int64_t* src_b;
  const int32_t* alpha_row;
  const float* alpha;
  int Hkv, D;
  int* err;
};

// One CTA per token: copy or blend the token's Hkv x D row of K and of V.
__global__ void __launch_bounds__(128) gather_blend_kernel(const GatherBlendParams p) {
  const int i = blockIdx.x;
  const int64_t dst = p.dst[i], a = p.src_a[i], b = p.src_b[i];
  const bool ok = dst >= 0 && dst < p.num_slots && a < p.num_slots && b < p.num_slots && (a >= 0 || b >= 0);
  if (!ok) {
    if (threadIdx.x == 0) report_error(p.err, DEVERR_BAD_SLOT, 5, i);
    return;
  }
  const int row = p.Hkv * p.D;
  const int vecs = row / 8;
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {
    __nv_bfloat16* pool = which ? p.pool_v : p.pool_k;
    uint4* d = reinterpret_cast<uint4*>(pool + dst * row);
    const uint4* sa = a >= 0 ? reinterpret_cast<const uint4*>(pool + a * row) : nullptr;
    const uint4* sb = b >= 0 ? reinterpret_cast<const uint4*>(pool + b * row) : nullptr;
    for (int vi = threadIdx.x; vi < vecs; vi += blockDim.x) {
      if (!sb) {
        d[vi] = sa[vi];
        continue;
      }
      if (!sa) {
        d[vi] = sb[vi];
        continue;
      }
      const int head = vi * 8 / p.D;
      const float al = p.alpha[(int64_t)p.alpha_row[i] * p.Hkv + head];
      const float ia = bf16r(__fsub_rn(1.f, al));
      uint4 av = sa[vi], bv = sb[vi];
      uint32_t* x = reinterpret_cast<uint32_t*>(&av);
      uint32_t* y = reinterpret_cast<uint32_t*>(&bv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float t1l = bf16r(__fmul_rn(al, bf16_lo(x[e]))), t1h = bf16r(__fmul_rn(al, bf16_hi(x[e])));
        const float t3l = bf16r(__fmul_rn(ia, bf16_lo(y[e]))), t3h = bf16r(__fmul_rn(ia, bf16_hi(y[e])));
        y[e] = pack_bf16(__fadd_rn(t1l, t3l), __fadd_rn(t1h, t3h));
      }
      d[vi] = bv;
    }
  }
}

int gather_blend(void* pool_k, void* pool_v, int64_t num_slots, const int64_t* dst, const int64_t* src_a,
                 const int64_t* src_b, const int32_t* alpha_row, const float* alpha, int num_tokens,
                 int num_kv_heads, int head_dim, int32_t* error_word, cudaStream_t stream) {
  if (head_dim != 64 && head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (num_tokens < 0 || num_kv_heads < 1) return LKV_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return LKV_OK;
  if (!pool_k || !pool_v || !dst || !src_a || !src_b || !alpha_row || !alpha) return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(pool_k) & 15) || (reinterpret_cast<uintptr_t>(pool_v) & 15))
    return LKV_ERR_INVALID_ARGUMENT;
  if (num_tokens > 2147483647) return LKV_ERR_UNSUPPORTED;
  GatherBlendParams p{};
  p.pool_k = static_cast<__nv_bfloat16*>(pool_k);
  p.pool_v = static_cast<__nv_bfloat16*>(pool_v);
  p.num_slots = num_slots;
  p.dst = dst;
  p.src_a = src_a;
  p.src_b = src_b;
  p.alpha_row = alpha_row;
  p.alpha = alpha;
  p.Hkv = num_kv_heads;
  p.D = head_dim;
  p.err = error_word;
  gather_blend_kernel<<<num_tokens, 128, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

__global__ void build_block_tables_kernel(const int32_t* bt, int64_t bt_stride, const int32_t* nsrc,
                                          const int32_t* ring_base, int L, int B, int W, int32_t* bt_all) {
  const int64_t total = (int64_t)L * B * W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % W);
    const int b = (int)((i / W) % B);
    const int l = (int)(i / ((int64_t)W * B));
    const int32_t v = bt[(int64_t)b * bt_stride + c];
    bt_all[i] = c < nsrc[b] ? v : v + ring_base[l];
  }
}

// Host-side checks of an append call; LKV_OK when the bf16 kernel may run.
static int check_append(const AppendArgs& a) {
  if (a.head_dim != 64 && a.head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (a.num_tokens < 0 || a.num_q_heads < 1 || a.num_kv_heads < 1) return LKV_ERR_INVALID_ARGUMENT;
  if (a.num_tokens == 0) return LKV_OK;
  if (!a.q || !a.k || !a.v || !a.q_out || !a.ring_slot || !a.ring_k || !a.ring_v) return LKV_ERR_INVALID_ARGUMENT;
  if (a.cos_sin && !a.positions) return LKV_ERR_INVALID_ARGUMENT;
  if ((a.q_weight == nullptr) != (a.k_weight == nullptr)) return LKV_ERR_INVALID_ARGUMENT;
  if (a.src_slot && (!a.src_k || !a.src_v)) return LKV_ERR_INVALID_ARGUMENT;
  if (a.num_tokens > 65535) return LKV_ERR_UNSUPPORTED;  // grid.y limit; callers split larger spans
  return LKV_OK;
}

static AppendParams append_params(const AppendArgs& a) {
  AppendParams p{};
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_row = a.q_row;
  p.k = static_cast<const __nv_bfloat16*>(a.k);
  p.k_row = a.k_row;
  p.v = static_cast<const __nv_bfloat16*>(a.v);
  p.v_row = a.v_row;
  p.pos = a.positions;
  p.cos_sin = a.cos_sin;
  p.cs_row = a.cos_sin_row;
  p.interleaved = (a.flags & LKV_ROPE_INTERLEAVED) ? 1 : 0;
  p.cs_fp32 = (a.flags & LKV_ROPE_TABLE_FP32) ? 1 : 0;
  p.max_pos = a.max_position;
  p.qw = static_cast<const __nv_bfloat16*>(a.q_weight);
  p.kw = static_cast<const __nv_bfloat16*>(a.k_weight);
  p.eps = a.eps;
  p.inv_scale = a.inv_scale;
  p.q_out = static_cast<__nv_bfloat16*>(a.q_out);
  p.q_out_row = a.q_out_row;
  p.ring_slot = a.ring_slot;
  p.ring_k = static_cast<__nv_bfloat16*>(a.ring_k);
  p.ring_v = static_cast<__nv_bfloat16*>(a.ring_v);
  p.ring_slots = a.ring_slots;
  p.src_slot = a.src_slot;
  p.src_k = static_cast<__nv_bfloat16*>(a.src_k);
  p.src_v = static_cast<__nv_bfloat16*>(a.src_v);
  p.src_slots = a.src_slots;
  p.T = a.num_tokens;
  p.Hq = a.num_q_heads;
  p.Hkv = a.num_kv_heads;
  p.err = a.error_word;
  return p;
}

int rope_norm_append(const AppendArgs& a) {
  const int st = check_append(a);
  if (st != LKV_OK || a.num_tokens == 0) return st;
  if (a.flags & LKV_APPEND_FP32) return rope_norm_append_f32(a);  // fp32 tensors and table (fp32.cu)
  const AppendParams p = append_params(a);
  dim3 grid((a.num_q_heads + a.num_kv_heads + 7) / 8, a.num_tokens);
  cudaStream_t stream = static_cast<cudaStream_t>(a.stream);
  const cudaError_t e = a.head_dim == 128 ? launch_pdl(rope_norm_append_kernel<128>, grid, dim3(256), 0, stream, p)
                                          : launch_pdl(rope_norm_append_kernel<64>, grid, dim3(256), 0, stream, p);
  return e == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

// Host-side checks of a commit call; LKV_OK when the kernel may run.
static int check_blend(const BlendArgs& a) {
  if (a.head_dim != 64 && a.head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (a.num_layers < 0 || a.num_seqs < 0 || a.pages_per_chunk < 0 || a.num_kv_heads < 1)
    return LKV_ERR_INVALID_ARGUMENT;
  if (a.num_layers == 0 || a.num_seqs == 0 || a.pages_per_chunk == 0) return LKV_OK;
  if (!a.pool_k || !a.pool_v || !a.raw_pages || !a.ring_pages || !a.alpha) return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a.pool_k) & 15) || (reinterpret_cast<uintptr_t>(a.pool_v) & 15))
    return LKV_ERR_INVALID_ARGUMENT;
  if (a.num_seqs > 65535 || a.num_layers > 65535) return LKV_ERR_UNSUPPORTED;
  return LKV_OK;
}

static BlendParams blend_params(const BlendArgs& a) {
  BlendParams p{};
  p.pool_k = static_cast<__nv_bfloat16*>(a.pool_k);
  p.pool_v = static_cast<__nv_bfloat16*>(a.pool_v);
  p.num_pages = a.num_pages;
  p.raw_pages = a.raw_pages;
  p.ring_pages = a.ring_pages;
  p.ring_stride = a.ring_layer_stride_pages;
  p.alpha = a.alpha;
  p.ppc = a.pages_per_chunk;
  p.S = a.num_seqs;
  p.L = a.num_layers;
  p.Hkv = a.num_kv_heads;
  p.D = a.head_dim;
  p.err = a.error_word;
  return p;
}

int blend_chunk(const BlendArgs& a) {
  const int st = check_blend(a);
  if (st != LKV_OK || a.num_layers == 0 || a.num_seqs == 0 || a.pages_per_chunk == 0) return st;
  const BlendParams p = blend_params(a);
  dim3 grid(a.pages_per_chunk, a.num_seqs, a.num_layers);
  blend_chunk_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(a.stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

int rope_norm_append_commit(const AppendArgs& a, const BlendArgs& b, const int32_t* commit_count,
                            int commit_blocks) {
  int st = check_append(a);
  if (st != LKV_OK) return st;
  st = check_blend(b);
  if (st != LKV_OK) return st;
  if (a.flags & LKV_APPEND_FP32) return LKV_ERR_UNSUPPORTED;  // fp32 pools: append, then lkv_blend_chunk_f32
  if (a.head_dim != b.head_dim || a.num_kv_heads != b.num_kv_heads || commit_blocks < 0)
    return LKV_ERR_INVALID_ARGUMENT;
  const int groups = (a.num_q_heads + a.num_kv_heads + 7) / 8;
  const int64_t n_append = (int64_t)groups * a.num_tokens;
  const int64_t items = (int64_t)b.pages_per_chunk * b.num_seqs * b.num_layers;
  // commit blocks: by default one per page item when the host knows the rows (as
  // blend_chunk_kernel), else one full wave (8 resident 256-thread blocks per SM at
  // <= 32 registers) striding over the items; an explicit count is capped at the items
  int64_t nb = 0;
  if (items > 0) {
    if (commit_blocks > 0) {
      nb = commit_count ? commit_blocks : std::min<int64_t>(items, commit_blocks);
    } else if (!commit_count) {
      nb = items;
    } else {
      int dev = 0, sms = 0;
      if (cudaGetDevice(&dev) != cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return LKV_ERR_CUDA;
      nb = 8 * sms;
    }
  }
  if (n_append + nb > 0x7fffffffLL) return LKV_ERR_UNSUPPORTED;
  if (n_append + nb == 0) return LKV_OK;
  const AppendParams pa = append_params(a);
  BlendParams pb = blend_params(b);
  pb.count = commit_count;
  cudaStream_t stream = static_cast<cudaStream_t>(a.stream);
  const dim3 grid((unsigned)(n_append + nb));
  const cudaError_t e =
      a.head_dim == 128
          ? launch_pdl(append_commit_kernel<128>, grid, dim3(256), 0, stream, pa, pb, groups, (int)n_append)
          : launch_pdl(append_commit_kernel<64>, grid, dim3(256), 0, stream, pa, pb, groups, (int)n_append);
  return e == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

int build_layer_block_tables(const int32_t* bt, int64_t bt_stride, const int32_t* nsrc, const int32_t* ring_base,
                             int num_layers, int batch, int width, int32_t* bt_all, cudaStream_t stream) {
  if (num_layers < 0 || batch < 0 || width < 0) return LKV_ERR_INVALID_ARGUMENT;
  const int64_t total = (int64_t)num_layers * batch * width;
  if (total == 0) return LKV_OK;
  if (!bt || !nsrc || !ring_base || !bt_all) return LKV_ERR_INVALID_ARGUMENT;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 4096);
  build_block_tables_kernel<<<blocks, 256, 0, stream>>>(bt, bt_stride, nsrc, ring_base, num_layers, batch, width,
                                                        bt_all);
  return cudaGetLastError() == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

}  // namespace lkv
