// fp32 path of the shared-KV attention, for models that run in fp32 (the
// reference's CPU configuration, llm/src/lastkv/llm/modeling.py in fp32:
// fp32 projections, fp32 RoPE / q-k RMSNorm, fp32 SDPA over an fp32 cache).
// Same merged paged layout as the bf16 path - pools [pages, 16, Hkv, D], rings
// holding K and V / s_l, outputs scaled by s_l - with every element fp32:
//
// rope_norm_append_f32_kernel - one warp per (token, head): RoPE as the
//   reference's apply_rotary_pos_emb (q*cos + rotate_half(q)*sin, two rounded
//   products and a rounded sum), RMSNorm as LlamaRMSNorm (mean of squares,
//   1/sqrt, x*inv then *w), V * (1/s_l), paged stores (ring slot; shared slot
//   on the top layer).  Selected by LKV_APPEND_FP32 on lkv_rope_norm_append.
// attention_f32_kernel - one warp per (query token, query head), decode and
//   chunked prefill alike: the visible keys (all seq_k for decode, bottom-right
//   causal for spans, modeling.py:124-146) are taken 32 at a time, one key per
//   lane for the scores (fp32 dot products), then an exact online-softmax
//   update and the P*V accumulation with each lane owning D/32 output columns.
// blend_chunk_f32_kernel - ring = a*raw + (1-a)*ring with the reference's
//   rounding points (a*top and (1-a)*layer rounded, then their rounded sum;
//   modeling.py:115-119 evaluated in fp32), V in V/s units.
//
// These are CUDA-core kernels: at the fp32 configuration's size (124M model,
// batch 1) the work is a few MFLOP per layer and fp32 has no tcgen05 path that
// keeps the reference's arithmetic; the bf16 kernels are the throughput path.

#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace lkv {

struct AppendF32Params {
  const float* q;
  int64_t q_row;
  const float* k;
  int64_t k_row;
  const float* v;
  int64_t v_row;
  const int64_t* pos;
  const float* cos_sin;  // [max_pos, D] = cos | sin halves
  int64_t cs_row;
  int64_t max_pos;
  int interleaved;
  const float* qw;
  const float* kw;
  float eps;
  const float* inv_scale;
  float* q_out;
  int64_t q_out_row;
  const int64_t* ring_slot;
  float* ring_k;
  float* ring_v;
  int64_t ring_slots;
  const int64_t* src_slot;
  float* src_k;
  float* src_v;
  int64_t src_slots;
  int T, Hq, Hkv;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(256) rope_norm_append_f32_kernel(const AppendF32Params p) {
  pdl_launch_dependents();
  pdl_wait();  // q/k/v come from the projection GEMM
  constexpr int HALF = D / 2;
  constexpr int E = HALF / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * 8 + warp;
  const int t = blockIdx.y;
  if (h >= p.Hq + p.Hkv) return;
  const bool is_q = h < p.Hq;
  const int j = h - p.Hq;
  const float* src = is_q ? p.q + (int64_t)t * p.q_row + (int64_t)h * D : p.k + (int64_t)t * p.k_row + (int64_t)j * D;
  const int i0 = lane * E;
  auto ix1 = [&](int e) { return p.interleaved ? 2 * (i0 + e) : i0 + e; };
  auto ix2 = [&](int e) { return p.interleaved ? 2 * (i0 + e) + 1 : HALF + i0 + e; };
  float r1[E], r2[E];
  if (p.cos_sin) {
    const int64_t pos = p.pos[t];
    if (pos < 0 || pos >= p.max_pos) {
      if (lane == 0) report_error(p.err, DEVERR_BAD_SLOT, 7, (int)pos);
      return;
    }
    const float* cs = p.cos_sin + pos * p.cs_row;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float x = src[ix1(e)], y = src[ix2(e)];
      const float cc = cs[i0 + e], sn = cs[HALF + i0 + e];
      // (x, y) -> (x*c + (-y)*s, y*c + x*s): two rounded products, one rounded sum each
      r1[e] = __fadd_rn(__fmul_rn(x, cc), -__fmul_rn(y, sn));
      r2[e] = __fadd_rn(__fmul_rn(y, cc), __fmul_rn(x, sn));
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      r1[e] = src[ix1(e)];
      r2[e] = src[ix2(e)];
    }
  }
  const float* w = is_q ? p.qw : p.kw;
  float o1[E], o2[E];
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      ss = __fadd_rn(ss, __fmul_rn(r1[e], r1[e]));
      ss = __fadd_rn(ss, __fmul_rn(r2[e], r2[e]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)D), p.eps)));
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o1[e] = __fmul_rn(w[ix1(e)], __fmul_rn(r1[e], inv));
      o2[e] = __fmul_rn(w[ix2(e)], __fmul_rn(r2[e], inv));
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o1[e] = r1[e];
      o2[e] = r2[e];
    }
  }
  auto store = [&](float* dst, const float* a, const float* b) {
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
  if (!ring_ok && lane == 0) report_error(p.err, DEVERR_BAD_SLOT, 7, (int)slot);
  const float* vsrc = p.v + (int64_t)t * p.v_row + (int64_t)j * D;
  const float is = p.inv_scale ? p.inv_scale[j] : 1.f;
  float va[E], vb[E], vsa[E], vsb[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    va[e] = vsrc[ix1(e)];
    vb[e] = vsrc[ix2(e)];
    vsa[e] = __fmul_rn(va[e], is);
    vsb[e] = __fmul_rn(vb[e], is);
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
      report_error(p.err, DEVERR_BAD_SLOT, 7, (int)ss_);
    }
  }
}

int rope_norm_append_f32(const AppendArgs& a) {
  AppendF32Params p{};
  p.q = static_cast<const float*>(a.q);
  p.q_row = a.q_row;
  p.k = static_cast<const float*>(a.k);
  p.k_row = a.k_row;
  p.v = static_cast<const float*>(a.v);
  p.v_row = a.v_row;
  p.pos = a.positions;
  p.cos_sin = static_cast<const float*>(a.cos_sin);
  p.cs_row = a.cos_sin_row;
  p.max_pos = a.max_position;
  p.interleaved = (a.flags & LKV_ROPE_INTERLEAVED) ? 1 : 0;
  p.qw = static_cast<const float*>(a.q_weight);
  p.kw = static_cast<const float*>(a.k_weight);
  p.eps = a.eps;
  p.inv_scale = a.inv_scale;
  p.q_out = static_cast<float*>(a.q_out);
  p.q_out_row = a.q_out_row;
  p.ring_slot = a.ring_slot;
  p.ring_k = static_cast<float*>(a.ring_k);
  p.ring_v = static_cast<float*>(a.ring_v);
  p.ring_slots = a.ring_slots;
  p.src_slot = a.src_slot;
  p.src_k = static_cast<float*>(a.src_k);
  p.src_v = static_cast<float*>(a.src_v);
  p.src_slots = a.src_slots;
  p.T = a.num_tokens;
  p.Hq = a.num_q_heads;
  p.Hkv = a.num_kv_heads;
  p.err = a.error_word;
  dim3 grid((a.num_q_heads + a.num_kv_heads + 7) / 8, a.num_tokens);
  cudaStream_t stream = static_cast<cudaStream_t>(a.stream);
  const cudaError_t e = a.head_dim == 128
                            ? launch_pdl(rope_norm_append_f32_kernel<128>, grid, dim3(256), 0, stream, p)
                            : launch_pdl(rope_norm_append_f32_kernel<64>, grid, dim3(256), 0, stream, p);
  return e == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

// ------------------------------------------------------------------ attention

struct AttnF32Params {
  const float* q;
  int64_t q_row;
  const float* pk;
  const float* pv;
  int64_t num_pages;
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* seq_k;
  const int32_t* cu_q;
  float* out;
  int64_t out_row;
  float* lse;  // natural log [T, Hq] or null
  const float* out_scale;
  int B, T, Hq, Hkv, W, causal;
  float scale;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(128) attention_f32_kernel(const AttnF32Params p) {
  pdl_launch_dependents();
  pdl_wait();  // q comes from the append kernel, the newest keys too
  constexpr int E = D / 32;
  __shared__ float qs[4][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  if (row >= (int64_t)p.T * p.Hq) return;  // warp-uniform; no block barrier follows
  const int t = (int)(row / p.Hq), h = (int)(row % p.Hq);
  const int hk = h / (p.Hq / p.Hkv);
  int lo = 0, hi = p.B;  // the sequence b with cu_q[b] <= t < cu_q[b + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (p.cu_q[mid] <= t) lo = mid;
    else hi = mid;
  }
  const int b = lo;
  const int q0 = p.cu_q[b], lq = p.cu_q[b + 1] - q0, i = t - q0;
  const int n = min(max(p.seq_k[b], 0), p.W * 16);
  int nvis = p.causal ? n - lq + i + 1 : n;  // bottom-right aligned: query i sits at key n - lq + i
  nvis = min(max(nvis, 0), n);
  const float* qr = p.q + (int64_t)t * p.q_row + (int64_t)h * D;
  for (int d = lane; d < D; d += 32) qs[warp][d] = qr[d];
  __syncwarp();
  const int32_t* btr = p.bt + (int64_t)b * p.bt_stride;
  float m = -INFINITY, l = 0.f, o[E];
#pragma unroll
  for (int e = 0; e < E; ++e) o[e] = 0.f;
  for (int base = 0; base < nvis; base += 32) {
    const int j = base + lane;
    float s = -INFINITY;
    int pid = 0;
    if (j < nvis) {
      pid = btr[j >> 4];
      if (pid < 0 || (int64_t)pid >= p.num_pages) {
        report_error(p.err, DEVERR_BAD_PAGE, 8, pid);  // the key is skipped
        pid = 0;
      } else {
        const float4* kr = reinterpret_cast<const float4*>(p.pk + (((int64_t)pid * 16 + (j & 15)) * p.Hkv + hk) * D);
        float acc = 0.f;
#pragma unroll 8
        for (int d4 = 0; d4 < D / 4; ++d4) {
          const float4 kv = kr[d4];
          acc = fmaf(qs[warp][4 * d4], kv.x, acc);
          acc = fmaf(qs[warp][4 * d4 + 1], kv.y, acc);
          acc = fmaf(qs[warp][4 * d4 + 2], kv.z, acc);
          acc = fmaf(qs[warp][4 * d4 + 3], kv.w, acc);
        }
        s = acc * p.scale;
      }
    }
    float mb = s;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
    const float mn = fmaxf(m, mb);
    if (mn == -INFINITY) continue;  // every key so far skipped (warp-uniform)
    const float alpha = expf(m - mn);
    const float pj = s == -INFINITY ? 0.f : expf(s - mn);
    float ps = pj;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = l * alpha + ps;
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] *= alpha;
    const int cnt = min(32, nvis - base);
    for (int kk = 0; kk < cnt; ++kk) {
      const float w = __shfl_sync(0xffffffffu, pj, kk);
      const int pg = __shfl_sync(0xffffffffu, pid, kk);
      if (w == 0.f) continue;  // warp-uniform (broadcast value)
      const float* vr = p.pv + (((int64_t)pg * 16 + ((base + kk) & 15)) * p.Hkv + hk) * D + lane * E;
#pragma unroll
      for (int e = 0; e < E; ++e) o[e] = fmaf(w, vr[e], o[e]);
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const float sc = (p.out_scale ? p.out_scale[h] : 1.f) * inv;
  float* dst = p.out + (int64_t)t * p.out_row + (int64_t)h * D + lane * E;
#pragma unroll
  for (int e = 0; e < E; ++e) dst[e] = o[e] * sc;
  if (p.lse && lane == 0) p.lse[(int64_t)t * p.Hq + h] = l > 0.f ? m + logf(l) : -INFINITY;
}

int attention_f32(const AttnF32Args& a) {
  if (a.head_dim != 64 && a.head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (a.num_kv_heads < 1 || a.num_q_heads < 1 || a.num_q_heads % a.num_kv_heads) return LKV_ERR_INVALID_ARGUMENT;
  if (a.batch < 0 || a.total_q < 0 || a.max_pages_per_seq < 0) return LKV_ERR_INVALID_ARGUMENT;
  if (a.batch == 0 || a.total_q == 0) return LKV_OK;
  if (!a.q || !a.pool_k || !a.pool_v || !a.block_table || !a.seq_k || !a.cu_seqlens_q || !a.out || !a.error_word)
    return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a.pool_k) & 15) || (reinterpret_cast<uintptr_t>(a.pool_v) & 15))
    return LKV_ERR_INVALID_ARGUMENT;
  if (a.q_stride_tok < (int64_t)a.num_q_heads * a.head_dim || a.out_stride_tok < (int64_t)a.num_q_heads * a.head_dim)
    return LKV_ERR_INVALID_ARGUMENT;
  AttnF32Params p{};
  p.q = static_cast<const float*>(a.q);
  p.q_row = a.q_stride_tok;
  p.pk = static_cast<const float*>(a.pool_k);
  p.pv = static_cast<const float*>(a.pool_v);
  p.num_pages = a.num_pages;
  p.bt = a.block_table;
  p.bt_stride = a.block_table_stride;
  p.seq_k = a.seq_k;
  p.cu_q = a.cu_seqlens_q;
  p.out = static_cast<float*>(a.out);
  p.out_row = a.out_stride_tok;
  p.lse = a.lse;
  p.out_scale = a.out_scale;
  p.B = a.batch;
  p.T = a.total_q;
  p.Hq = a.num_q_heads;
  p.Hkv = a.num_kv_heads;
  p.W = a.max_pages_per_seq;
  p.causal = a.causal ? 1 : 0;
  p.scale = a.softmax_scale;
  p.err = a.error_word;
  const int64_t rows = (int64_t)a.total_q * a.num_q_heads;
  if ((rows + 3) / 4 > 0x7fffffff) return LKV_ERR_UNSUPPORTED;
  dim3 grid((unsigned)((rows + 3) / 4));
  cudaStream_t stream = static_cast<cudaStream_t>(a.stream);
  const cudaError_t e = a.head_dim == 128 ? launch_pdl(attention_f32_kernel<128>, grid, dim3(128), 0, stream, p)
                                          : launch_pdl(attention_f32_kernel<64>, grid, dim3(128), 0, stream, p);
  return e == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

// ------------------------------------------------------------------ blend

struct BlendF32Params {
  float* pool_k;
  float* pool_v;
  int64_t num_pages;
  const int32_t* raw_pages;
  const int32_t* ring_pages;
  int64_t ring_stride;
  const float* alpha;
  int ppc, Hkv, D;
  int* err;
};

// grid (pages_per_chunk, num_seqs, num_layers); one CTA blends one page of one layer.
__global__ void __launch_bounds__(256) blend_chunk_f32_kernel(const BlendF32Params p) {
  const int jp = blockIdx.x, seq = blockIdx.y, layer = blockIdx.z;
  const int64_t raw = p.raw_pages[(int64_t)seq * p.ppc + jp];
  const int64_t ring = (int64_t)p.ring_pages[(int64_t)seq * p.ppc + jp] + (int64_t)layer * p.ring_stride;
  if (raw < 0 || raw >= p.num_pages || ring < 0 || ring >= p.num_pages) {
    if (threadIdx.x == 0) report_error(p.err, DEVERR_BAD_PAGE, 9, (int)(raw < 0 || raw >= p.num_pages ? raw : ring));
    return;
  }
  const int64_t page_elems = (int64_t)16 * p.Hkv * p.D;
  const int vecs = (int)(page_elems / 4);
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {
    float* pool = which ? p.pool_v : p.pool_k;
    const float4* src = reinterpret_cast<const float4*>(pool + raw * page_elems);
    float4* dst = reinterpret_cast<float4*>(pool + ring * page_elems);
    for (int vi = threadIdx.x; vi < vecs; vi += blockDim.x) {
      const int head = (int)(((int64_t)vi * 4 / p.D) % p.Hkv);
      const float a = p.alpha[layer * p.Hkv + head];
      const float ia = __fsub_rn(1.f, a);
      const float4 r = src[vi];
      float4 g = dst[vi];
      // a*top + (1-a)*layer: two rounded products and a rounded sum (no contraction)
      g.x = __fadd_rn(__fmul_rn(a, r.x), __fmul_rn(ia, g.x));
      g.y = __fadd_rn(__fmul_rn(a, r.y), __fmul_rn(ia, g.y));
      g.z = __fadd_rn(__fmul_rn(a, r.z), __fmul_rn(ia, g.z));
      g.w = __fadd_rn(__fmul_rn(a, r.w), __fmul_rn(ia, g.w));
      dst[vi] = g;
    }
  }
}

int blend_chunk_f32(const BlendArgs& a) {
  if (a.head_dim != 64 && a.head_dim != 128) return LKV_ERR_UNSUPPORTED;
  if (a.num_layers < 0 || a.num_seqs < 0 || a.pages_per_chunk < 0 || a.num_kv_heads < 1)
    return LKV_ERR_INVALID_ARGUMENT;
  if (a.num_layers == 0 || a.num_seqs == 0 || a.pages_per_chunk == 0) return LKV_OK;
  if (!a.pool_k || !a.pool_v || !a.raw_pages || !a.ring_pages || !a.alpha) return LKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a.pool_k) & 15) || (reinterpret_cast<uintptr_t>(a.pool_v) & 15))
    return LKV_ERR_INVALID_ARGUMENT;
  if (a.num_seqs > 65535 || a.num_layers > 65535) return LKV_ERR_UNSUPPORTED;
  BlendF32Params p{};
  p.pool_k = static_cast<float*>(a.pool_k);
  p.pool_v = static_cast<float*>(a.pool_v);
  p.num_pages = a.num_pages;
  p.raw_pages = a.raw_pages;
  p.ring_pages = a.ring_pages;
  p.ring_stride = a.ring_layer_stride_pages;
  p.alpha = a.alpha;
  p.ppc = a.pages_per_chunk;
  p.Hkv = a.num_kv_heads;
  p.D = a.head_dim;
  p.err = a.error_word;
  dim3 grid(a.pages_per_chunk, a.num_seqs, a.num_layers);
  blend_chunk_f32_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(a.stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? LKV_OK : LKV_ERR_CUDA;
}

}  // namespace lkv
