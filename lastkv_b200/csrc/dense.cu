// Dense-layer epilogues around the shared-KV attention for decode steps (sm_100a).
//
// At decode batch sizes the per-layer dense glue (residual adds, RMSNorm,
// SiLU-and-mul) is a few KB per kernel; as separate elementwise launches it
// costs more time per layer than the weights it sits between.  These kernels
// do each step in one launch with the arithmetic of the eager torch modules
// (llm/src/lastkv/llm/modeling.py decoder layer; the vLLM model uses the same
// pair of fused ops, vllm/src/lastkv/vllm/vllm_model.py:756-789):
//
// rmsnorm_kernel  - optional residual add h = bf16(x + r) (written back), then
//   bf16(w * bf16(h * rsqrt(mean(h^2) + eps))) with fp32 accumulation: the
//   rounding points of `weight * (h.float() * rsqrt(...)).to(bf16)`.
// silu_mul_kernel - out = bf16(bf16(silu(g)) * u) for a [gate | up] row, the
//   rounding points of `F.silu(gate) * up` in bf16.
//
// Both read and write 16-byte vectors (8 bf16) and are HBM/latency bound.

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace lkv {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 4;  // hidden <= 256 threads * 4 vectors * 8 = 8192

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

struct RmsParams {
  const __nv_bfloat16* x;
  int64_t x_row;
  const __nv_bfloat16* residual;
  int64_t residual_row;
  __nv_bfloat16* residual_out;
  int64_t residual_out_row;
  const __nv_bfloat16* weight;
  __nv_bfloat16* out;
  int64_t out_row;
  int hidden;
  float eps;
};

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const RmsParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int nvec = p.hidden / 8;
  const uint4* x = reinterpret_cast<const uint4*>(p.x + row * p.x_row);
  const uint4* r = p.residual ? reinterpret_cast<const uint4*>(p.residual + row * p.residual_row) : nullptr;
  uint4* ro = p.residual ? reinterpret_cast<uint4*>(p.residual_out + row * p.residual_out_row) : nullptr;
  float h[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < nvec) {
      unpack8(x[c], h[i]);
      if (r) {
        float rv[8];
        unpack8(r[c], rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[i][j] = bf16_round(h[i][j] + rv[j]);
        ro[c] = pack8(h[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(h[i][j], h[i][j], ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  const float rs = rsqrtf(tot * (1.0f / (float)p.hidden) + p.eps);
  const uint4* w = reinterpret_cast<const uint4*>(p.weight);
  uint4* out = reinterpret_cast<uint4*>(p.out + row * p.out_row);
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int c = threadIdx.x + i * kNormThreads;
    if (c < nvec) {
      float wv[8], o[8];
      unpack8(w[c], wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = wv[j] * bf16_round(h[i][j] * rs);
      out[c] = pack8(o);
    }
  }
}

__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up, int64_t gu_row,
                                                       __nv_bfloat16* __restrict__ out, int64_t out_row,
                                                       int64_t rows, int ffn) {
  pdl_launch_dependents();
  pdl_wait();
  const int nv = ffn / 8;
  const int64_t total = rows * nv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nv;
    const int c = (int)(i - r * nv);
    const __nv_bfloat16* row = gate_up + r * gu_row;
    float g[8], u[8], o[8];
    unpack8(*reinterpret_cast<const uint4*>(row + c * 8), g);
    unpack8(*reinterpret_cast<const uint4*>(row + ffn + c * 8), u);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = bf16_round(g[j] / (1.0f + expf(-g[j]))) * u[j];
    *reinterpret_cast<uint4*>(out + r * out_row + c * 8) = pack8(o);
  }
}

// (value, index) order of torch.argmax: NaN above everything, then larger values,
// and the smaller index between equal values.
struct ArgMax {
  float v;
  int i;
};

__device__ __forceinline__ bool argmax_before(const ArgMax& a, const ArgMax& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (!an && a.v != b.v) return a.v > b.v;
  return a.i < b.i;
}

constexpr int kArgmaxThreads = 1024;

// One CTA per row: 16-byte loads of 8 bf16 logits, a per-thread running best, a
// warp-shuffle and shared-memory reduction, one int64 index written per row.
__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                                     int64_t row_stride, int cols,
                                                                     int64_t* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const __nv_bfloat16* row = x + (int64_t)blockIdx.x * row_stride;
  ArgMax best{-INFINITY, 0x7fffffff};
  const int nvec = cols / 8;
  // Eight independent 16-byte loads per thread and pass (two L2 round trips for
  // a 128K-column row instead of sixteen); the order of the comparisons does not
  // matter, argmax_before being a strict total order.
  constexpr int U = 8;
  for (int c0 = threadIdx.x; c0 < nvec; c0 += U * kArgmaxThreads) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * kArgmaxThreads;
      if (c < nvec) v[u] = *reinterpret_cast<const uint4*>(row + (int64_t)c * 8);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * kArgmaxThreads;
      if (c >= nvec) break;
      float f[8];
      unpack8(v[u], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const ArgMax cand{f[j], c * 8 + j};
        if (argmax_before(cand, best)) best = cand;
      }
    }
  }
  for (int c = nvec * 8 + threadIdx.x; c < cols; c += kArgmaxThreads) {
    const ArgMax cand{__bfloat162float(row[c]), c};
    if (argmax_before(cand, best)) best = cand;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    if (argmax_before(other, best)) best = other;
  }
  __shared__ ArgMax part[kArgmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < kArgmaxThreads / 32 ? part[threadIdx.x] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
      if (argmax_before(other, best)) best = other;
    }
    if (threadIdx.x == 0) out[blockIdx.x] = best.i == 0x7fffffff ? 0 : best.i;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int rmsnorm(const void* x, int64_t x_row, const void* residual, int64_t residual_row, void* residual_out,
            int64_t residual_out_row, const void* weight, void* out, int64_t out_row, int rows, int hidden, float eps,
            cudaStream_t stream) {
  if (rows < 0 || hidden <= 0 || hidden % 8 || hidden > kNormThreads * kNormMaxVec * 8) return LKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return LKV_OK;
  if (!x || !weight || !out || (residual && !residual_out)) return LKV_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || x_row % 8 || out_row % 8 || x_row < hidden ||
      out_row < hidden)
    return LKV_ERR_INVALID_ARGUMENT;
  if (residual && (!aligned16(residual) || !aligned16(residual_out) || residual_row % 8 || residual_out_row % 8 ||
                   residual_row < hidden || residual_out_row < hidden))
    return LKV_ERR_INVALID_ARGUMENT;
  RmsParams p{static_cast<const __nv_bfloat16*>(x),
              x_row,
              static_cast<const __nv_bfloat16*>(residual),
              residual_row,
              static_cast<__nv_bfloat16*>(residual_out),
              residual_out_row,
              static_cast<const __nv_bfloat16*>(weight),
              static_cast<__nv_bfloat16*>(out),
              out_row,
              hidden,
              eps};
  return launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, stream, p) == cudaSuccess ? LKV_OK
                                                                                                  : LKV_ERR_CUDA;
}

int silu_mul(const void* gate_up, int64_t gate_up_row, void* out, int64_t out_row, int64_t rows, int ffn,
             cudaStream_t stream) {
  if (rows < 0 || ffn <= 0 || ffn % 8) return LKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return LKV_OK;
  if (!gate_up || !out || !aligned16(gate_up) || !aligned16(out) || gate_up_row % 8 || out_row % 8 ||
      gate_up_row < 2 * (int64_t)ffn || out_row < ffn)
    return LKV_ERR_INVALID_ARGUMENT;
  const int64_t total = rows * (ffn / 8);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  return launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, stream,
                    static_cast<const __nv_bfloat16*>(gate_up), gate_up_row, static_cast<__nv_bfloat16*>(out),
                    out_row, rows, ffn) == cudaSuccess
             ? LKV_OK
             : LKV_ERR_CUDA;
}

int argmax_rows(const void* x, int64_t row_stride, int rows, int cols, int64_t* out, cudaStream_t stream) {
  if (rows < 0 || cols < 1 || row_stride < cols || (row_stride % 8) || !x || !out || !aligned16(x))
    return LKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return LKV_OK;
  return launch_pdl(argmax_rows_kernel, dim3(rows), dim3(kArgmaxThreads), 0, stream,
                    static_cast<const __nv_bfloat16*>(x), row_stride, cols, out) == cudaSuccess
             ? LKV_OK
             : LKV_ERR_CUDA;
}

}  // namespace lkv
