// Memory-bound model kernels for the transformer families (bf16 activations, fp32 statistics):
// RMSNorm and LayerNorm forward/backward, RoPE (in place, rotate-half convention), SwiGLU and
// GELU forward/backward, and the row-wise softmax cross entropy that overwrites the logits
// with their gradient (the LM-head GEMMs around it are plain library GEMMs).
//
// They replace the ATen chains of the reference's GPT example (examples/train_gpt.py:144-199,
// 261, 350) and provide the Llama-3 pieces (RMSNorm, RoPE theta=500000, SwiGLU).
#include <cuda_bf16.h>

#include <stdexcept>
#include <string>

#include "kernels.h"
#include "tc_common.cuh"

namespace mmf {

namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }

// 8 x bf16 <-> 8 x float through one 16-byte access
__device__ __forceinline__ void ld_bf8(const __nv_bfloat16* p, float* v) {
  uint4 w = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 f = __bfloat1622float2(h[e]);
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}
__device__ __forceinline__ void st_bf8(__nv_bfloat16* p, const float* v) {
  uint4 w;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
  *reinterpret_cast<uint4*>(p) = w;
}

// Block-wide sum for blockDim.x <= 1024 (result broadcast to all threads).
__device__ __forceinline__ float block_allsum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (w == 0) {
    t = warp_sum(t);
    if (l == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// ---------------------------------- RMSNorm ----------------------------------------------
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                          int cols, float eps) {
  __shared__ float red[33];
  const int64_t off = static_cast<int64_t>(blockIdx.x) * cols;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = bf(x[off + c]);
    s = fmaf(v, v, s);
  }
  s = block_allsum(s, red);
  const float r = rsqrtf(s / cols + eps);
  if (threadIdx.x == 0) rstd[blockIdx.x] = r;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) y[off + c] = __float2bfloat16_rn(bf(x[off + c]) * r * bf(w[c]));
}

// Vector variant: the row stays in registers (cols % 8 == 0 and cols <= 256 * 8 * RV).
template <int RV>
__global__ void __launch_bounds__(256) rmsnorm_fwd_vec_kernel(const __nv_bfloat16* __restrict__ x,
                                                              const __nv_bfloat16* __restrict__ w,
                                                              __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                              int cols, float eps) {
  __shared__ float red[33];
  const int64_t off = static_cast<int64_t>(blockIdx.x) * cols;
  float v[RV][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < RV; ++k) {
    const int c = (threadIdx.x + 256 * k) * 8;
    if (c < cols) {
      ld_bf8(x + off + c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[k][e], v[k][e], s);
    }
  }
  s = block_allsum(s, red);
  const float r = rsqrtf(s / cols + eps);
  if (threadIdx.x == 0) rstd[blockIdx.x] = r;
#pragma unroll
  for (int k = 0; k < RV; ++k) {
    const int c = (threadIdx.x + 256 * k) * 8;
    if (c < cols) {
      float wv[8], o[8];
      ld_bf8(w + c, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * r * wv[e];
      st_bf8(y + off + c, o);
    }
  }
}

__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const float* __restrict__ rstd,
                                                          __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part,
                                                          int rows, int cols) {
  extern __shared__ float dw_acc[];  // [cols]
  __shared__ float red[33];
  for (int c = threadIdx.x; c < cols; c += blockDim.x) dw_acc[c] = 0.f;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t off = static_cast<int64_t>(r) * cols;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) dot = fmaf(bf(dy[off + c]) * bf(w[c]), bf(x[off + c]), dot);
    dot = block_allsum(dot, red);
    const float k = dot * rs * rs * rs / cols;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float g = bf(dy[off + c]), xv = bf(x[off + c]);
      dx[off + c] = __float2bfloat16_rn(rs * g * bf(w[c]) - xv * k);
      dw_acc[c] = fmaf(g, xv * rs, dw_acc[c]);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) dw_part[static_cast<int64_t>(blockIdx.x) * cols + c] = dw_acc[c];
}

// Vector variant of the backward (cols % 8 == 0 and cols <= 256 * 8 * RV).  Each block walks its
// rows with the next row's dy and x loaded before the current row's block reduction, so that the
// DRAM latency of one row overlaps the reduction and the stores of the previous one.
template <int RV>
__global__ void __launch_bounds__(256) rmsnorm_bwd_vec_kernel(const __nv_bfloat16* __restrict__ dy,
                                                              const __nv_bfloat16* __restrict__ x,
                                                              const __nv_bfloat16* __restrict__ w,
                                                              const float* __restrict__ rstd,
                                                              __nv_bfloat16* __restrict__ dx,
                                                              float* __restrict__ dw_part, int rows, int cols) {
  __shared__ float red[33];
  float acc[RV][8], wv[RV][8];
#pragma unroll
  for (int k = 0; k < RV; ++k) {
    const int c = (threadIdx.x + 256 * k) * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[k][e] = 0.f;
    if (c < cols) ld_bf8(w + c, wv[k]);
  }
  float g[RV][8], xv[RV][8];  // current row
  float gn[RV][8], xn[RV][8];  // next row (prefetched)
  auto load_row = [&](int r, float (*gd)[8], float (*xd)[8]) {
    const int64_t off = static_cast<int64_t>(r) * cols;
#pragma unroll
    for (int k = 0; k < RV; ++k) {
      const int c = (threadIdx.x + 256 * k) * 8;
      if (c < cols) {
        ld_bf8(dy + off + c, gd[k]);
        ld_bf8(x + off + c, xd[k]);
      }
    }
  };
  int r = blockIdx.x;
  if (r < rows) load_row(r, g, xv);
  for (; r < rows; r += gridDim.x) {
    const int64_t off = static_cast<int64_t>(r) * cols;
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < RV; ++k) {
      const int c = (threadIdx.x + 256 * k) * 8;
      if (c < cols) {
#pragma unroll
        for (int e = 0; e < 8; ++e) dot = fmaf(g[k][e] * wv[k][e], xv[k][e], dot);
      }
    }
    const int rn = r + gridDim.x;
    if (rn < rows) load_row(rn, gn, xn);  // in flight during the reduction below
    dot = block_allsum(dot, red);
    const float k3 = dot * rs * rs * rs / cols;
#pragma unroll
    for (int k = 0; k < RV; ++k) {
      const int c = (threadIdx.x + 256 * k) * 8;
      if (c < cols) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          o[e] = rs * g[k][e] * wv[k][e] - xv[k][e] * k3;
          acc[k][e] = fmaf(g[k][e], xv[k][e] * rs, acc[k][e]);
        }
        st_bf8(dx + off + c, o);
      }
    }
#pragma unroll
    for (int k = 0; k < RV; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        g[k][e] = gn[k][e];
        xv[k][e] = xn[k][e];
      }
  }
#pragma unroll
  for (int k = 0; k < RV; ++k) {
    const int c = (threadIdx.x + 256 * k) * 8;
    if (c < cols) {
      float4* dst = reinterpret_cast<float4*>(dw_part + static_cast<int64_t>(blockIdx.x) * cols + c);
      dst[0] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
      dst[1] = make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
    }
  }
}

// --------------------------------- LayerNorm ---------------------------------------------
__global__ void __launch_bounds__(256) layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ w,
                                                            const __nv_bfloat16* __restrict__ b,
                                                            __nv_bfloat16* __restrict__ y, float* __restrict__ mean,
                                                            float* __restrict__ rstd, int cols, float eps) {
  __shared__ float red[33];
  const int64_t off = static_cast<int64_t>(blockIdx.x) * cols;
  float s = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) s += bf(x[off + c]);
  const float mu = block_allsum(s, red) / cols;
  float v = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const float d = bf(x[off + c]) - mu;
    v = fmaf(d, d, v);
  }
  const float r = rsqrtf(block_allsum(v, red) / cols + eps);
  if (threadIdx.x == 0) {
    mean[blockIdx.x] = mu;
    rstd[blockIdx.x] = r;
  }
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    y[off + c] = __float2bfloat16_rn(fmaf((bf(x[off + c]) - mu) * r, bf(w[c]), b ? bf(b[c]) : 0.f));
}

__global__ void __launch_bounds__(256) layernorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                            const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ w,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ rstd,
                                                            __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part,
                                                            float* __restrict__ db_part, int rows, int cols) {
  extern __shared__ float acc[];  // [2*cols]: dw, db
  __shared__ float red[33];
  float* dw_acc = acc;
  float* db_acc = acc + cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) dw_acc[c] = db_acc[c] = 0.f;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t off = static_cast<int64_t>(r) * cols;
    const float mu = mean[r], rs = rstd[r];
    float s1 = 0.f, s2 = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float gw = bf(dy[off + c]) * bf(w[c]);
      const float xh = (bf(x[off + c]) - mu) * rs;
      s1 += gw;
      s2 = fmaf(gw, xh, s2);
    }
    s1 = block_allsum(s1, red) / cols;
    s2 = block_allsum(s2, red) / cols;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
      const float g = bf(dy[off + c]);
      const float xh = (bf(x[off + c]) - mu) * rs;
      dx[off + c] = __float2bfloat16_rn(rs * (g * bf(w[c]) - s1 - xh * s2));
      dw_acc[c] = fmaf(g, xh, dw_acc[c]);
      db_acc[c] += g;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    dw_part[static_cast<int64_t>(blockIdx.x) * cols + c] = dw_acc[c];
    if (db_part) db_part[static_cast<int64_t>(blockIdx.x) * cols + c] = db_acc[c];
  }
}

template <bool OUT_F32>
__global__ void colsum_kernel(const float* __restrict__ part, int prow, int cols, void* out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int p = 0; p < prow; ++p) s += part[static_cast<int64_t>(p) * cols + c];
  if (OUT_F32)
    reinterpret_cast<float*>(out)[c] = s;
  else
    reinterpret_cast<__nv_bfloat16*>(out)[c] = __float2bfloat16_rn(s);
}

// ------------------------------------ RoPE -----------------------------------------------
// One thread per (token, frequency i): the angle is computed once and applied to every head.
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, int tokens, int heads, int head_dim, int seq_len,
                            float log2_theta, float sign, int64_t token_stride, int64_t head_stride) {
  const int half = head_dim >> 1;
  const int64_t total = static_cast<int64_t>(tokens) * half;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(e % half);
    const int t = static_cast<int>(e / half);
    const int pos = t % seq_len;
    const float inv_freq = exp2f(-log2_theta * (2.f * i) / head_dim);  // theta^(-2i/d)
    float sn, cs;
    sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
    sn *= sign;
    __nv_bfloat16* base = x + t * token_stride + i;
    for (int h = 0; h < heads; ++h) {
      __nv_bfloat16* p = base + h * head_stride;
      const float x1 = bf(p[0]), x2 = bf(p[half]);
      p[0] = __float2bfloat16_rn(x1 * cs - x2 * sn);
      p[half] = __float2bfloat16_rn(x2 * cs + x1 * sn);
    }
  }
}

// ------------------------------- activations ---------------------------------------------
__device__ __forceinline__ float sigmoidf_(float g) { return 1.f / (1.f + expf(-g)); }

__global__ void swiglu_fwd_vec_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u,
                                      __nv_bfloat16* __restrict__ o, int64_t n8) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float gv[8], uv[8], ov[8];
    ld_bf8(g + 8 * i, gv);
    ld_bf8(u + 8 * i, uv);
#pragma unroll
    for (int e = 0; e < 8; ++e) ov[e] = gv[e] * sigmoidf_(gv[e]) * uv[e];
    st_bf8(o + 8 * i, ov);
  }
}
__global__ void swiglu_bwd_vec_kernel(const __nv_bfloat16* __restrict__ d, const __nv_bfloat16* __restrict__ g,
                                      const __nv_bfloat16* __restrict__ u, __nv_bfloat16* __restrict__ dg,
                                      __nv_bfloat16* __restrict__ du, int64_t n8) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float dv[8], gv[8], uv[8], a[8], b[8];
    ld_bf8(d + 8 * i, dv);
    ld_bf8(g + 8 * i, gv);
    ld_bf8(u + 8 * i, uv);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float sg = sigmoidf_(gv[e]);
      a[e] = dv[e] * uv[e] * sg * (1.f + gv[e] * (1.f - sg));
      b[e] = dv[e] * gv[e] * sg;
    }
    st_bf8(dg + 8 * i, a);
    st_bf8(du + 8 * i, b);
  }
}
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u,
                                  __nv_bfloat16* __restrict__ o, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gv = bf(g[i]);
    o[i] = __float2bfloat16_rn(gv * sigmoidf_(gv) * bf(u[i]));
  }
}
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ d, const __nv_bfloat16* __restrict__ g,
                                  const __nv_bfloat16* __restrict__ u, __nv_bfloat16* __restrict__ dg,
                                  __nv_bfloat16* __restrict__ du, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gv = bf(g[i]), uv = bf(u[i]), dv = bf(d[i]);
    const float s = sigmoidf_(gv);
    dg[i] = __float2bfloat16_rn(dv * uv * s * (1.f + gv * (1.f - s)));
    du[i] = __float2bfloat16_rn(dv * gv * s);
  }
}
constexpr float kInvSqrt2 = 0.70710678118654752f;
constexpr float kInvSqrt2Pi = 0.39894228040143268f;
__global__ void gelu_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = bf(x[i]);
    y[i] = __float2bfloat16_rn(0.5f * v * (1.f + erff(v * kInvSqrt2)));
  }
}
__global__ void gelu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                __nv_bfloat16* __restrict__ dx, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float v = bf(x[i]);
    const float cdf = 0.5f * (1.f + erff(v * kInvSqrt2));
    const float pdf = kInvSqrt2Pi * expf(-0.5f * v * v);
    dx[i] = __float2bfloat16_rn(bf(dy[i]) * (cdf + v * pdf));
  }
}

// ------------------------------- scale by a device scalar ---------------------------------
// x (bf16, n elements) *= *s, 16-byte vectors (the tail element-wise); s stays on the device, so
// a loss scale known only to the GPU needs no host synchronisation.
// SM clock probe: one thread per SM spins for `cycles` SM cycles and records the cycles and
// global-timer nanoseconds it took; out[2 * block] = cycles, out[2 * block + 1] = ns.  The
// frequency at that moment is cycles / ns GHz (a diagnostic of power-cap clock changes).
__global__ void clock_probe_kernel(int64_t cycles, long long* __restrict__ out) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  const long long c0 = clock64();
  long long c = c0;
  while (c - c0 < cycles) c = clock64();
  const uint64_t t1 = globaltimer_ns();
  out[2 * blockIdx.x] = c - c0;
  out[2 * blockIdx.x + 1] = static_cast<long long>(t1 - t0);
}

__global__ void scale_bf16_kernel(__nv_bfloat16* __restrict__ x, const float* __restrict__ s, int64_t n) {
  const float f = *s;
  const int64_t n8 = n / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[8];
    ld_bf8(x + 8 * i, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] *= f;
    st_bf8(x + 8 * i, v);
  }
  for (int64_t i = 8 * n8 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = __float2bfloat16_rn(bf(x[i]) * f);
}

// ------------------------------- embedding -----------------------------------------------
// Forward: out[t] = table[tok[t]], one 16-byte vector per thread (D % 8 == 0).
__global__ void embedding_fwd_kernel(const __nv_bfloat16* __restrict__ table, const int64_t* __restrict__ tok,
                                     __nv_bfloat16* __restrict__ out, int64_t tokens, int D, int64_t vocab,
                                     int* __restrict__ err) {
  const int vpr = D / 8;  // vectors per row
  const int64_t total = tokens * vpr;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = e / vpr;
    const int c = static_cast<int>(e - t * vpr) * 8;
    const int64_t v = tok[t];
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (v >= 0 && v < vocab)
      w = *reinterpret_cast<const uint4*>(table + v * D + c);
    else if (c == 0)
      atomicCAS(err, 0, ERR_BAD_ARGUMENT);  // a token outside the table: zeros, and say so
    *reinterpret_cast<uint4*>(out + t * D + c) = w;
  }
}

// Backward, step 1: first[v] = position of vocabulary row v's first occurrence in the sorted
// token list (rows that never occur keep -1 from the memset before).
__global__ void embedding_first_kernel(const int64_t* __restrict__ sorted, int64_t tokens, int64_t vocab,
                                       int* __restrict__ first) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < tokens;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = sorted[i];
    if (v >= 0 && v < vocab && (i == 0 || sorted[i - 1] != v)) first[v] = static_cast<int>(i);
  }
}

// Backward, step 2: every row of the dense table gradient in one pass: zeros for rows without
// tokens, else the fp32 sum of their tokens' output gradients in sorted (then original) order,
// so the result does not depend on scheduling.  One warp per row, 16-byte vectors.
__global__ void embedding_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const int64_t* __restrict__ sorted,
                                     const int64_t* __restrict__ perm, const int* __restrict__ first,
                                     __nv_bfloat16* __restrict__ dtable, int64_t tokens, int64_t vocab, int D) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t v = warp; v < vocab; v += nwarps) {
    const int f = first[v];
    __nv_bfloat16* row = dtable + v * D;
    for (int c = lane * 8; c < D; c += 256) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      if (f >= 0) {
        for (int64_t i = f; i < tokens && sorted[i] == v; ++i) {
          float g[8];
          ld_bf8(dy + perm[i] * D + c, g);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += g[e];
        }
      }
      st_bf8(row + c, acc);
    }
  }
}

// ------------------------------- cross entropy -------------------------------------------
// One block per row.  Online (max, sum-exp) over the row, then the gradient pass.
template <bool VEC>
__global__ void __launch_bounds__(1024) ce_kernel(__nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ tgt,
                                                  float* __restrict__ loss_rows, int vocab, int64_t ld,
                                                  float grad_scale, int ignore_index) {
  __shared__ float red_m[32], red_s[32];
  __shared__ float bc[2];
  const int64_t row = blockIdx.x;
  __nv_bfloat16* L = logits + row * ld;
  const int64_t t = tgt[row];
  float m = -INFINITY, s = 0.f;
  if (VEC) {
    for (int c = threadIdx.x * 8; c < vocab; c += blockDim.x * 8) {
      float v[8];
      ld_bf8(L + c, v);
      float mx = v[0];
#pragma unroll
      for (int e = 1; e < 8; ++e) mx = fmaxf(mx, v[e]);
      if (mx > m) {
        s *= expf(m - mx);
        m = mx;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) s += expf(v[e] - m);
    }
  } else {
    for (int c = threadIdx.x; c < vocab; c += blockDim.x) {
      const float v = bf(L[c]);
      if (v > m) {
        s = s * expf(m - v) + 1.f;
        m = v;
      } else {
        s += expf(v - m);
      }
    }
  }
  // combine (m, s) across the warp then the block
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (mm == -INFINITY) ? 0.f : s * expf(m - mm) + s2 * expf(m2 - mm);
    m = mm;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    red_m[w] = m;
    red_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    m = (l < nw) ? red_m[l] : -INFINITY;
    s = (l < nw) ? red_s[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (mm == -INFINITY) ? 0.f : s * expf(m - mm) + s2 * expf(m2 - mm);
      m = mm;
    }
    if (l == 0) {
      bc[0] = m;
      bc[1] = s;
    }
  }
  __syncthreads();
  const float mx = bc[0], se = bc[1];
  const bool ignored = (t == ignore_index) || t < 0 || t >= vocab;
  if (threadIdx.x == 0) {
    loss_rows[row] = ignored ? 0.f : (logf(se) + mx - bf(L[t]));
  }
  __syncthreads();  // the target logit must be read before it is overwritten
  if (grad_scale != 0.f) {
    const float inv = 1.f / se;
    if (VEC) {
      for (int c = threadIdx.x * 8; c < vocab; c += blockDim.x * 8) {
        float v[8];
        ld_bf8(L + c, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float gv = 0.f;
          if (!ignored) {
            gv = expf(v[e] - mx) * inv;
            if (c + e == t) gv -= 1.f;
            gv *= grad_scale;
          }
          v[e] = gv;
        }
        st_bf8(L + c, v);
      }
    } else {
      for (int c = threadIdx.x; c < vocab; c += blockDim.x) {
        float gv = 0.f;
        if (!ignored) {
          gv = expf(bf(L[c]) - mx) * inv;
          if (c == t) gv -= 1.f;
          gv *= grad_scale;
        }
        L[c] = __float2bfloat16_rn(gv);
      }
    }
  }
}

int grid_for(int64_t work, int threads, int cap) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

void check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: ") + what + " launch failed: " + cudaGetErrorString(e));
}

}  // namespace

void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int rows, int cols, float eps,
                 cudaStream_t stream) {
  if (rows <= 0) return;
  const bool vec = (cols % 8 == 0) && cols <= 256 * 8 * 4 && aligned16(x) && aligned16(w) && aligned16(y);
  if (vec)
    rmsnorm_fwd_vec_kernel<4><<<rows, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                        static_cast<const __nv_bfloat16*>(w),
                                                        static_cast<__nv_bfloat16*>(y), rstd, cols, eps);
  else
    rmsnorm_fwd_kernel<<<rows, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                 static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y),
                                                 rstd, cols, eps);
  check_launch("rmsnorm_fwd");
}

void rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw_partial,
                 int rows, int cols, int partial_rows, cudaStream_t stream) {
  if (rows <= 0) return;
  if ((cols % 8 == 0) && cols <= 256 * 8 * 4 && aligned16(dy) && aligned16(x) && aligned16(w) && aligned16(dx)) {
    auto go = [&](auto kern) {
      kern<<<partial_rows, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
                                             static_cast<const __nv_bfloat16*>(w), rstd, static_cast<__nv_bfloat16*>(dx),
                                             dw_partial, rows, cols);
    };
    if (cols <= 256 * 8 * 2)
      go(rmsnorm_bwd_vec_kernel<2>);
    else
      go(rmsnorm_bwd_vec_kernel<4>);
    check_launch("rmsnorm_bwd");
    return;
  }
  const size_t smem = sizeof(float) * cols;
  if (smem > 200 * 1024) throw std::runtime_error("mmf: rmsnorm_bwd width too large");
  if (smem > 48 * 1024) cudaFuncSetAttribute(rmsnorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  rmsnorm_bwd_kernel<<<partial_rows, 256, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
      rstd, static_cast<__nv_bfloat16*>(dx), dw_partial, rows, cols);
  check_launch("rmsnorm_bwd");
}

void layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd, int rows, int cols,
                   float eps, cudaStream_t stream) {
  if (rows <= 0) return;
  layernorm_fwd_kernel<<<rows, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(b),
      static_cast<__nv_bfloat16*>(y), mean, rstd, cols, eps);
  check_launch("layernorm_fwd");
}

void layernorm_bwd(const void* dy, const void* x, const void* w, const float* mean, const float* rstd, void* dx,
                   float* dw_partial, float* db_partial, int rows, int cols, int partial_rows, cudaStream_t stream) {
  if (rows <= 0) return;
  const size_t smem = sizeof(float) * cols * 2;
  if (smem > 200 * 1024) throw std::runtime_error("mmf: layernorm_bwd width too large");
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(layernorm_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  layernorm_bwd_kernel<<<partial_rows, 256, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
      mean, rstd, static_cast<__nv_bfloat16*>(dx), dw_partial, db_partial, rows, cols);
  check_launch("layernorm_bwd");
}

void colsum_partials(const float* partial, int prow, int cols, void* out, bool out_f32, cudaStream_t stream) {
  if (out_f32)
    colsum_kernel<true><<<(cols + 255) / 256, 256, 0, stream>>>(partial, prow, cols, out);
  else
    colsum_kernel<false><<<(cols + 255) / 256, 256, 0, stream>>>(partial, prow, cols, out);
  check_launch("colsum");
}

void rope_inplace(void* x, int tokens, int heads, int head_dim, int seq_len, float theta, bool inverse,
                  int64_t token_stride, int64_t head_stride, cudaStream_t stream) {
  if (tokens <= 0) return;
  if (head_dim % 2) throw std::runtime_error("mmf: rope needs an even head_dim");
  const int64_t work = static_cast<int64_t>(tokens) * (head_dim / 2);
  rope_kernel<<<grid_for(work, 256, 148 * 16), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), tokens, heads,
                                                                 head_dim, seq_len, log2f(theta),
                                                                 inverse ? -1.f : 1.f, token_stride, head_stride);
  check_launch("rope");
}

void swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, cudaStream_t stream) {
  if (n <= 0) return;
  if (n % 8 == 0 && aligned16(gate) && aligned16(up) && aligned16(out)) {
    swiglu_fwd_vec_kernel<<<grid_for(n / 8, 256, 148 * 16), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up),
        static_cast<__nv_bfloat16*>(out), n / 8);
    check_launch("swiglu_fwd");
    return;
  }
  swiglu_fwd_kernel<<<grid_for(n, 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up), static_cast<__nv_bfloat16*>(out), n);
  check_launch("swiglu_fwd");
}

void swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate, void* dup, int64_t n,
                cudaStream_t stream) {
  if (n <= 0) return;
  if (n % 8 == 0 && aligned16(dout) && aligned16(gate) && aligned16(up) && aligned16(dgate) && aligned16(dup)) {
    swiglu_bwd_vec_kernel<<<grid_for(n / 8, 256, 148 * 16), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(dout), static_cast<const __nv_bfloat16*>(gate),
        static_cast<const __nv_bfloat16*>(up), static_cast<__nv_bfloat16*>(dgate), static_cast<__nv_bfloat16*>(dup),
        n / 8);
    check_launch("swiglu_bwd");
    return;
  }
  swiglu_bwd_kernel<<<grid_for(n, 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(dout), static_cast<const __nv_bfloat16*>(gate),
      static_cast<const __nv_bfloat16*>(up), static_cast<__nv_bfloat16*>(dgate), static_cast<__nv_bfloat16*>(dup), n);
  check_launch("swiglu_bwd");
}

void gelu_fwd(const void* x, void* y, int64_t n, cudaStream_t stream) {
  if (n <= 0) return;
  gelu_fwd_kernel<<<grid_for(n, 256, 148 * 16), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                                  static_cast<__nv_bfloat16*>(y), n);
  check_launch("gelu_fwd");
}

void gelu_bwd(const void* dy, const void* x, void* dx, int64_t n, cudaStream_t stream) {
  if (n <= 0) return;
  gelu_bwd_kernel<<<grid_for(n, 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(dx), n);
  check_launch("gelu_bwd");
}

void clock_probe(int64_t cycles, int blocks, long long* out, cudaStream_t stream) {
  clock_probe_kernel<<<blocks, 32, 0, stream>>>(cycles, out);
  check_launch("clock_probe");
}

void scale_bf16(void* x, const float* s, int64_t n, cudaStream_t stream) {
  if (n <= 0) return;
  if (!aligned16(x)) throw std::runtime_error("mmf: scale_bf16 needs a 16-byte aligned tensor");
  scale_bf16_kernel<<<grid_for(n / 8 + 1, 256, 148 * 8), 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), s, n);
  check_launch("scale_bf16");
}

void embedding_fwd(const void* table, const int64_t* tokens, void* out, int64_t n_tokens, int D, int64_t vocab,
                   cudaStream_t stream) {
  if (n_tokens <= 0) return;
  if (D % 8 || !aligned16(table) || !aligned16(out)) throw std::runtime_error("mmf: embedding needs D % 8 == 0, 16-byte rows");
  int dev = 0;
  cudaGetDevice(&dev);
  embedding_fwd_kernel<<<grid_for(n_tokens * (D / 8), 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(table), tokens, static_cast<__nv_bfloat16*>(out), n_tokens, D, vocab,
      device_error_word(dev));
  check_launch("embedding_fwd");
}

void embedding_bwd(const void* dy, const int64_t* sorted, const int64_t* perm, int* first, void* dtable,
                   int64_t n_tokens, int64_t vocab, int D, cudaStream_t stream) {
  if (D % 8 || !aligned16(dy) || !aligned16(dtable)) throw std::runtime_error("mmf: embedding needs D % 8 == 0, 16-byte rows");
  cudaMemsetAsync(first, 0xff, sizeof(int) * vocab, stream);  // -1: the row has no tokens
  if (n_tokens > 0)
    embedding_first_kernel<<<grid_for(n_tokens, 256, 148 * 4), 256, 0, stream>>>(sorted, n_tokens, vocab, first);
  check_launch("embedding_first");
  embedding_bwd_kernel<<<grid_for(vocab * 32, 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), sorted, perm, first, static_cast<__nv_bfloat16*>(dtable), n_tokens, vocab,
      D);
  check_launch("embedding_bwd");
}

void cross_entropy_fwd_bwd(void* logits, const int64_t* targets, float* loss_rows, int rows, int vocab, int64_t ld,
                           float grad_scale, int ignore_index, cudaStream_t stream) {
  if (rows <= 0) return;
  const bool vec = (vocab % 8 == 0) && (ld % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  if (vec)
    ce_kernel<true><<<rows, 1024, 0, stream>>>(static_cast<__nv_bfloat16*>(logits), targets, loss_rows, vocab, ld,
                                               grad_scale, ignore_index);
  else
    ce_kernel<false><<<rows, 1024, 0, stream>>>(static_cast<__nv_bfloat16*>(logits), targets, loss_rows, vocab, ld,
                                                grad_scale, ignore_index);
  check_launch("cross_entropy");
}

}  // namespace mmf
