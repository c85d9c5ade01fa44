// Optimizer-side memory-bound kernels (multi-tensor, one launch per parameter group):
//   * muon_prep   : momentum / Nesterov / coupled weight decay fused with the bf16 cast of the
//                   NS input, the (optional) transpose into the wide orientation, and the
//                   per-matrix sum of squares for the Frobenius pre-normalisation.
//                   Replaces optimizer.py:142-150 + utils.py:79-89 (several ATen passes).
//   * ns_scale    : 1 / (||G||_F + 1e-7) per matrix (summing per-rank partials when sharded).
//   * ws_to_out   : bf16 workspace -> parameter / output tensors with axpby.
//   * adamw_multi : fused AdamW over all tensors of a group (examples/mixed_adamw.py:310-355
//                   semantics with a correct bias correction).
//   * power_iteration : device-resident power iteration for the spectral norm
//                   (src/muon_fsdp/spectral.py:48-111) without host synchronisation.
#include <cuda_bf16.h>

#include <stdexcept>
#include <string>

#include "kernels.h"
#include "tc_common.cuh"

namespace mmf {

namespace {

template <bool F32>
__device__ __forceinline__ float ld_val(const void* base, int64_t i) {
  if (F32) return reinterpret_cast<const float*>(base)[i];
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
}
template <bool F32>
__device__ __forceinline__ void st_val(void* base, int64_t i, float v) {
  if (F32)
    reinterpret_cast<float*>(base)[i] = v;
  else
    reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.f;
    s = warp_sum(s);
  }
  __syncthreads();
  return s;  // valid in thread 0
}

constexpr int PT = 64;  // prep tile edge

// 8-wide vector helpers (16-byte bf16 / 2 x 16-byte fp32 accesses)
template <bool F32>
__device__ __forceinline__ void ld8(const void* base, int64_t i, float* v) {
  if (F32) {
    const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(h[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
}
template <bool F32>
__device__ __forceinline__ void st8(void* base, int64_t i, const float* v) {
  if (F32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i);
    p[0] = make_float4(v[0], v[1], v[2], v[3]);
    p[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + i) = w;
  }
}

// VEC == 8: each thread handles 8 consecutive columns (requires cols % 8 == 0, 16-byte aligned
// tensors, dst_ld % 8 == 0 and dst_row0 % 8 == 0 — checked on the host).  Loads from peer
// memory (the P2P assembly of the sharded Muon step) are 16-byte requests.
template <bool GRAD_F32, bool PARAM_F32, int VEC>
__global__ void __launch_bounds__(256) muon_prep_kernel(const PrepArgs a) {
  const PrepDesc d = a.descs[blockIdx.y];
  const int tiles_c = (d.cols + PT - 1) / PT;
  const int tiles = ((d.rows + PT - 1) / PT) * tiles_c;
  __shared__ float tile[PT][PT + 1];
  __shared__ float red[8];
  constexpr int TPR = PT / VEC;          // threads per tile row
  constexpr int RPP = 256 / TPR;         // rows per pass
  const int tx = threadIdx.x % TPR;
  const int ty = threadIdx.x / TPR;
  const void* G = reinterpret_cast<const void*>(d.grad);
  float* BUF = reinterpret_cast<float*>(d.buf);
  void* P = reinterpret_cast<void*>(d.param);
  __nv_bfloat16* DST = reinterpret_cast<__nv_bfloat16*>(d.dst);
  const float mu = a.mu;
  float sq = 0.f;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = (t / tiles_c) * PT, c0 = (t % tiles_c) * PT;
    const int c = c0 + tx * VEC;
#pragma unroll 2
    for (int rr = ty; rr < PT; rr += RPP) {
      const int r = r0 + rr;
      float u[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) u[e] = 0.f;
      if (r < d.rows && c < d.cols) {
        const int64_t i = static_cast<int64_t>(r) * d.cols + c;
        float g[VEC];
        if (VEC == 8) {
          ld8<GRAD_F32>(G, i, g);
        } else {
          g[0] = ld_val<GRAD_F32>(G, i);
        }
        if (a.wd_coupled != 0.f && P) {
          float pv[VEC];
          if (VEC == 8) ld8<PARAM_F32>(P, i, pv); else pv[0] = ld_val<PARAM_F32>(P, i);
#pragma unroll
          for (int e = 0; e < VEC; ++e) g[e] = fmaf(a.wd_coupled, pv[e], g[e]);
        }
        if (a.mode == 0) {
#pragma unroll
          for (int e = 0; e < VEC; ++e) u[e] = g[e];
        } else {
          float b[VEC];
          if (VEC == 8) ld8<true>(BUF, i, b); else b[0] = BUF[i];
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            b[e] = (a.mode == 1) ? fmaf(mu, b[e] - g[e], g[e]) : fmaf(mu, b[e], g[e]);
            u[e] = a.nesterov ? fmaf(mu, b[e], g[e]) : b[e];
          }
          if (VEC == 8) st8<true>(BUF, i, b); else BUF[i] = b[0];
        }
        if (!DST) {
          float pv[VEC];
          if (d.p_scale != 0.f) {
            if (VEC == 8) ld8<PARAM_F32>(P, i, pv); else pv[0] = ld_val<PARAM_F32>(P, i);
          } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) pv[e] = 0.f;
          }
#pragma unroll
          for (int e = 0; e < VEC; ++e) pv[e] = fmaf(d.p_scale, pv[e], d.v_scale * u[e]);
          if (VEC == 8) st8<PARAM_F32>(P, i, pv); else st_val<PARAM_F32>(P, i, pv[0]);
        } else if (!d.transposed) {
          const int64_t o = static_cast<int64_t>(d.dst_row0 + r) * d.dst_ld + c;
          if (VEC == 8) st8<false>(DST, o, u); else DST[o] = __float2bfloat16_rn(u[0]);
        }
#pragma unroll
        for (int e = 0; e < VEC; ++e) sq = fmaf(u[e], u[e], sq);
      }
      if (DST && d.transposed) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) tile[rr][tx * VEC + e] = u[e];
      }
    }
    if (DST && d.transposed) {
      __syncthreads();
      // transposed write: destination row (c0 + cc), columns dst_row0 + r0 + [rr0, rr0 + VEC)
#pragma unroll 2
      for (int cc = ty; cc < PT; cc += RPP) {
        const int cg = c0 + cc;
        const int rr0 = tx * VEC;
        if (cg < d.cols) {
          const int64_t o = static_cast<int64_t>(cg) * d.dst_ld + d.dst_row0 + r0 + rr0;
          if (VEC == 8 && r0 + rr0 + 8 <= d.rows) {
            float v8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v8[e] = tile[rr0 + e][cc];
            st8<false>(DST, o, v8);
          } else {
            for (int e = 0; e < VEC; ++e)
              if (r0 + rr0 + e < d.rows) DST[o + e] = __float2bfloat16_rn(tile[rr0 + e][cc]);
          }
        }
      }
      __syncthreads();
    }
  }
  if (a.sumsq) {
    // every block writes its partial (zero included); prep_sumsq_kernel adds them in order
    const float s = block_sum_256(sq, red);
    if (threadIdx.x == 0) a.partials[static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = s;
  }
}

// sumsq[b] += sum_k partials[b * nblk + k], summed in a fixed order: lane-strided, then a fixed
// shuffle tree (one warp per tensor).
__global__ void prep_sumsq_kernel(const float* __restrict__ partials, int nblk, float* __restrict__ sumsq) {
  const int b = blockIdx.x;
  float acc = 0.f;
  for (int k = threadIdx.x; k < nblk; k += 32) acc += partials[static_cast<int64_t>(b) * nblk + k];
  acc = warp_sum(acc);
  if (threadIdx.x == 0) sumsq[b] += acc;
}

__global__ void ns_scale_kernel(const float* sumsq, int n, int nparts, float eps, float* s, float* s2) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  float acc = 0.f;
  for (int p = 0; p < nparts; ++p) acc += sumsq[static_cast<int64_t>(p) * n + b];
  const float v = 1.f / (sqrtf(acc) + eps);
  s[b] = v;
  if (s2) s2[b] = v * v;
}

// T[idx + e] = ps * T[idx + e] + vs * v[e] for e < n (n <= 8); 16-byte vectors when possible.
template <bool OUT_F32>
__device__ __forceinline__ void apply_run8(void* T, int64_t idx, const float* v, int n, float ps, float vs) {
  if (OUT_F32) {
    float* p = reinterpret_cast<float*>(T) + idx;
    if (n == 8 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
      float4* q = reinterpret_cast<float4*>(p);
      float4 o0 = make_float4(0.f, 0.f, 0.f, 0.f), o1 = o0;
      if (ps != 0.f) {
        o0 = q[0];
        o1 = q[1];
      }
      q[0] = make_float4(fmaf(ps, o0.x, vs * v[0]), fmaf(ps, o0.y, vs * v[1]), fmaf(ps, o0.z, vs * v[2]),
                         fmaf(ps, o0.w, vs * v[3]));
      q[1] = make_float4(fmaf(ps, o1.x, vs * v[4]), fmaf(ps, o1.y, vs * v[5]), fmaf(ps, o1.z, vs * v[6]),
                         fmaf(ps, o1.w, vs * v[7]));
      return;
    }
    for (int e = 0; e < n; ++e) p[e] = fmaf(ps, ps != 0.f ? p[e] : 0.f, vs * v[e]);
  } else {
    __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(T) + idx;
    if (n == 8 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (ps != 0.f) w = *reinterpret_cast<const uint4*>(p);
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 o = __bfloat1622float2(h[e]);
        h[e] = __floats2bfloat162_rn(fmaf(ps, o.x, vs * v[2 * e]), fmaf(ps, o.y, vs * v[2 * e + 1]));
      }
      *reinterpret_cast<uint4*>(p) = w;
      return;
    }
    for (int e = 0; e < n; ++e)
      p[e] = __float2bfloat16_rn(fmaf(ps, ps != 0.f ? __bfloat162float(p[e]) : 0.f, vs * v[e]));
  }
}

// Workspace X [batch, Mp, Np] (bf16, the wide orientation) -> destinations, in 64 x 64 tiles.
// A transposed destination goes through a shared-memory tile, so that both the workspace reads
// and the destination read-modify-writes are 16-byte vectors along rows (a direct element-wise
// transposed update would touch a different destination row per element).
template <bool OUT_F32>
__global__ void __launch_bounds__(256) ws_to_out_kernel(const WsOutArgs a) {
  __shared__ float tile[64][65];
  const int b = blockIdx.y;
  const __nv_bfloat16* X = reinterpret_cast<const __nv_bfloat16*>(a.X) + static_cast<int64_t>(b) * a.Mp * a.Np;
  const float sc = a.s_vec ? a.s_vec[b] : 1.f;
  const float ps = a.p_scale * (a.p_scale_vec ? a.p_scale_vec[b] : 1.f);
  const float vs = a.v_scale * (a.v_scale_vec ? a.v_scale_vec[b] : 1.f) * sc;
  int64_t ld = a.out_ld, seg_rows = int64_t(1) << 40;
  int tr = a.out_transposed ? 1 : 0;
  if (a.out_meta) {
    ld = a.out_meta[3 * b];
    tr = static_cast<int>(a.out_meta[3 * b + 1]);
    seg_rows = a.out_meta[3 * b + 2];
  }
  const int64_t* segp = a.out_ptrs + static_cast<int64_t>(b) * (a.nseg < 1 ? 1 : a.nseg);
  auto dest = [&](int64_t r, int64_t c, void*& T) -> int64_t {  // element (r, c) of the destination
    const int seg = (a.nseg > 1) ? static_cast<int>(r / seg_rows) : 0;
    T = reinterpret_cast<void*>(segp[seg]);
    return (r - seg * seg_rows) * ld + c;
  };
  const int tiles_n = (a.n_true + 63) / 64;
  const int tiles = ((a.m_true + 63) / 64) * tiles_n;
  const int tr8 = threadIdx.x >> 3, tc8 = (threadIdx.x & 7) * 8;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int i0 = (t / tiles_n) * 64, j0 = (t % tiles_n) * 64;
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const int ii = tr8 + 32 * pass, i = i0 + ii, j = j0 + tc8;
      float v[8];
      if (i < a.m_true && j < a.n_true) {
        const uint4 w = *reinterpret_cast<const uint4*>(X + static_cast<int64_t>(i) * a.Np + j);  // Np % 8 == 0
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          v[2 * e] = f.x;
          v[2 * e + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      if (!tr) {
        if (i < a.m_true && j < a.n_true) {
          void* T;
          const int64_t idx = dest(i, j, T);
          apply_run8<OUT_F32>(T, idx, v, min(8, a.n_true - j), ps, vs);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) tile[ii][tc8 + e] = v[e];
      }
    }
    if (tr) {
      __syncthreads();
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int rr = tr8 + 32 * pass;      // destination row j0 + rr = workspace column
        const int R = j0 + rr, C = i0 + tc8;  // destination columns = workspace rows
        if (R < a.n_true && C < a.m_true) {
          float v[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = tile[tc8 + e][rr];
          void* T;
          const int64_t idx = dest(R, C, T);
          apply_run8<OUT_F32>(T, idx, v, min(8, a.m_true - C), ps, vs);
        }
      }
      __syncthreads();
    }
  }
}

template <bool F32>
__device__ __forceinline__ void ld4(const void* base, int64_t i, float* v) {
  if (F32) {
    float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
    uint2 w = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(base) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
}
template <bool F32>
__device__ __forceinline__ void st4(void* base, int64_t i, const float* v) {
  if (F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    uint2 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
    h[0] = __floats2bfloat162_rn(v[0], v[1]);
    h[1] = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(base) + i) = w;
  }
}

// VEC == 4 needs numel % 4 == 0 and 16-byte aligned tensors (host-checked per launch).
template <bool P_F32, bool G_F32, int VEC>
__global__ void __launch_bounds__(256) adamw_kernel(const AdamArgs a) {
  const AdamDesc d = a.descs[blockIdx.y];
  void* P = reinterpret_cast<void*>(d.param);
  const void* G = reinterpret_cast<const void*>(d.grad);
  float* M = reinterpret_cast<float*>(d.exp_avg);
  float* V = reinterpret_cast<float*>(d.exp_avg_sq);
  const float step_size = a.lr / a.bias_correction1;
  const float decay = 1.f - a.lr * a.weight_decay;
  const int64_t nv = d.numel / VEC;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < nv;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = j * VEC;
    float g[VEC], m[VEC], v[VEC], p[VEC];
    if (VEC == 4) {
      ld4<G_F32>(G, i, g);
      ld4<true>(M, i, m);
      ld4<true>(V, i, v);
      ld4<P_F32>(P, i, p);
    } else {
      g[0] = ld_val<G_F32>(G, i);
      m[0] = M[i];
      v[0] = V[i];
      p[0] = ld_val<P_F32>(P, i);
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      m[e] = fmaf(a.beta1, m[e] - g[e], g[e]);
      v[e] = fmaf(a.beta2, v[e] - g[e] * g[e], g[e] * g[e]);
      const float denom = sqrtf(v[e]) / a.bias_correction2_sqrt + a.eps;
      p[e] = fmaf(-step_size, m[e] / denom, p[e] * decay);
    }
    if (VEC == 4) {
      st4<true>(M, i, m);
      st4<true>(V, i, v);
      st4<P_F32>(P, i, p);
    } else {
      M[i] = m[0];
      V[i] = v[0];
      st_val<P_F32>(P, i, p[0]);
    }
  }
}

template <bool P_F32, bool G_F32, int VEC>
__global__ void __launch_bounds__(256) muon_moments_kernel(const MomentArgs a) {
  const AdamDesc d = a.descs[blockIdx.y];
  const void* P = reinterpret_cast<const void*>(d.param);
  const void* G = reinterpret_cast<const void*>(d.grad);
  float* B = reinterpret_cast<float*>(d.exp_avg);
  float* S = reinterpret_cast<float*>(d.exp_avg_sq);
  const int64_t nv = d.numel / VEC;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < nv;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = j * VEC;
    float g[VEC], b[VEC], s[VEC], p[VEC];
    if (VEC == 4) {
      ld4<G_F32>(G, i, g);
      ld4<true>(B, i, b);
      ld4<true>(S, i, s);
      if (a.weight_decay != 0.f) ld4<P_F32>(P, i, p);
    } else {
      g[0] = ld_val<G_F32>(G, i);
      b[0] = B[i];
      s[0] = S[i];
      if (a.weight_decay != 0.f) p[0] = ld_val<P_F32>(P, i);
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      if (a.weight_decay != 0.f) g[e] = fmaf(a.weight_decay, p[e], g[e]);
      b[e] = fmaf(a.momentum, b[e], g[e]);
      const float u = a.nesterov ? fmaf(a.momentum, b[e], g[e]) : b[e];
      s[e] = fmaf(a.beta2, s[e], (1.f - a.beta2) * u * u);
    }
    if (VEC == 4) {
      st4<true>(B, i, b);
      st4<true>(S, i, s);
    } else {
      B[i] = b[0];
      S[i] = s[0];
    }
  }
}

// ---------------------------- power iteration helpers ------------------------------------
// y[r] = sum_c W[r, c] x[c]     (one warp per row)
template <bool F32>
__global__ void gemv_rows_kernel(const void* W, int m, int n, const float* x, float* y) {
  const int warps = blockDim.x >> 5;
  const int r = blockIdx.x * warps + (threadIdx.x >> 5);
  const int l = threadIdx.x & 31;
  if (r >= m) return;
  float acc = 0.f;
  for (int c = l; c < n; c += 32) acc = fmaf(ld_val<F32>(W, static_cast<int64_t>(r) * n + c), x[c], acc);
  acc = warp_sum(acc);
  if (l == 0) y[r] = acc;
}
// part[k, c] = sum_{r in row block k} W[r, c] x[r]   (one thread per column, rows split over
// blockIdx.y); y[c] = sum_k part[k, c] in block order (gemv_cols_sum_kernel): no atomics, so the
// result is bitwise reproducible.
template <bool F32>
__global__ void gemv_cols_kernel(const void* W, int m, int n, const float* x, float* part, int rows_per_block) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(m, r0 + rows_per_block);
  float acc = 0.f;
  for (int r = r0; r < r1; ++r) acc = fmaf(ld_val<F32>(W, static_cast<int64_t>(r) * n + c), x[r], acc);
  part[static_cast<int64_t>(blockIdx.y) * n + c] = acc;
}
__global__ void gemv_cols_sum_kernel(const float* part, int nblk, int n, float* y) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float acc = 0.f;
  for (int k = 0; k < nblk; ++k) acc += part[static_cast<int64_t>(k) * n + c];
  y[c] = acc;
}
// x /= max(||x||, eps) in place (single block); optionally also writes ||x|| into *norm_out.
__global__ void normalize_kernel(float* x, int n, float eps, float* norm_out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(x[i], x[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float nrm = sqrtf(red[0]);
  const float inv = 1.f / fmaxf(nrm, eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) x[i] *= inv;
  if (norm_out && threadIdx.x == 0) *norm_out = nrm;
}
__global__ void dot_kernel(const float* a, const float* b, int n, float* out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(a[i], b[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) *out = t;
  }
}

int grid_for(int64_t work, int threads, int cap) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}

void check_launch(const char* what) {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: ") + what + " launch failed: " + cudaGetErrorString(e));
}

}  // namespace

int muon_prep_blocks(int max_tiles) { return max_tiles < 1 ? 1 : (max_tiles > 4096 ? 4096 : max_tiles); }

void muon_prep(const PrepArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  if (a.n > 65535) throw std::runtime_error("mmf: muon_prep supports at most 65535 tensors per launch");
  if (a.sumsq && !a.partials) throw std::runtime_error("mmf: muon_prep needs its partial-sum scratch");
  const int gx = muon_prep_blocks(a.max_tiles);
  dim3 grid(gx, a.n);
#define MMF_PREP(GF, PF, V) muon_prep_kernel<GF, PF, V><<<grid, 256, 0, stream>>>(a)
  if (a.vec8) {
    if (a.grad_f32) {
      if (a.param_f32) MMF_PREP(true, true, 8); else MMF_PREP(true, false, 8);
    } else {
      if (a.param_f32) MMF_PREP(false, true, 8); else MMF_PREP(false, false, 8);
    }
  } else {
    if (a.grad_f32) {
      if (a.param_f32) MMF_PREP(true, true, 1); else MMF_PREP(true, false, 1);
    } else {
      if (a.param_f32) MMF_PREP(false, true, 1); else MMF_PREP(false, false, 1);
    }
  }
#undef MMF_PREP
  check_launch("muon_prep");
  if (a.sumsq) {
    prep_sumsq_kernel<<<a.n, 32, 0, stream>>>(a.partials, gx, a.sumsq);
    check_launch("muon_prep (sum of squares)");
  }
}

void ns_scale(const float* sumsq, int n, int nparts, float eps, float* s, float* s2, cudaStream_t stream) {
  if (n <= 0) return;
  ns_scale_kernel<<<(n + 127) / 128, 128, 0, stream>>>(sumsq, n, nparts, eps, s, s2);
  check_launch("ns_scale");
}

void ws_to_out(const WsOutArgs& a, cudaStream_t stream) {
  if (a.batch <= 0) return;
  if (a.Np % 8 != 0) throw std::runtime_error("mmf: ws_to_out needs Np % 8 == 0");
  const int64_t tiles = static_cast<int64_t>((a.m_true + 63) / 64) * ((a.n_true + 63) / 64);
  dim3 grid(static_cast<unsigned>(tiles < 1184 ? tiles : 1184), a.batch);
  if (a.out_f32)
    ws_to_out_kernel<true><<<grid, 256, 0, stream>>>(a);
  else
    ws_to_out_kernel<false><<<grid, 256, 0, stream>>>(a);
  check_launch("ws_to_out");
}

void adamw_multi(const AdamArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  if (a.n > 65535) throw std::runtime_error("mmf: adamw_multi supports at most 65535 tensors per launch");
  const int vec = a.vec4 ? 4 : 1;
  dim3 grid(grid_for(a.max_numel / vec, 256, 1184), a.n);
#define MMF_ADAM(PF, GF)                                                      \
  do {                                                                        \
    if (a.vec4)                                                               \
      adamw_kernel<PF, GF, 4><<<grid, 256, 0, stream>>>(a);                   \
    else                                                                      \
      adamw_kernel<PF, GF, 1><<<grid, 256, 0, stream>>>(a);                   \
  } while (0)
  if (a.param_f32) {
    if (a.grad_f32) MMF_ADAM(true, true); else MMF_ADAM(true, false);
  } else {
    if (a.grad_f32) MMF_ADAM(false, true); else MMF_ADAM(false, false);
  }
#undef MMF_ADAM
  check_launch("adamw_multi");
}

void muon_moments_multi(const MomentArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  if (a.n > 65535) throw std::runtime_error("mmf: muon_moments_multi supports at most 65535 tensors per launch");
  const int vec = a.vec4 ? 4 : 1;
  dim3 grid(grid_for(a.max_numel / vec, 256, 1184), a.n);
#define MMF_MOM(PF, GF)                                                       \
  do {                                                                        \
    if (a.vec4)                                                               \
      muon_moments_kernel<PF, GF, 4><<<grid, 256, 0, stream>>>(a);            \
    else                                                                      \
      muon_moments_kernel<PF, GF, 1><<<grid, 256, 0, stream>>>(a);            \
  } while (0)
  if (a.param_f32) {
    if (a.grad_f32) MMF_MOM(true, true); else MMF_MOM(true, false);
  } else {
    if (a.grad_f32) MMF_MOM(false, true); else MMF_MOM(false, false);
  }
#undef MMF_MOM
  check_launch("muon_moments_multi");
}

// work must hold max(m, n) + 1 floats.  u [m], v [n] (v holds the start vector on entry).
int power_iteration_col_blocks(int m) { return (m + 255) / 256; }

void power_iteration(const void* W, bool w_f32, int m, int n, float* u, float* v, float* sigma, int iters, float eps,
                     float* work, float* col_part, cudaStream_t stream) {
  const int rows_per_block = 256;
  auto rows = [&](const float* x, float* y) {
    if (w_f32)
      gemv_rows_kernel<true><<<(m + 7) / 8, 256, 0, stream>>>(W, m, n, x, y);
    else
      gemv_rows_kernel<false><<<(m + 7) / 8, 256, 0, stream>>>(W, m, n, x, y);
    check_launch("gemv_rows");
  };
  auto cols = [&](const float* x, float* y) {
    dim3 g((n + 255) / 256, (m + rows_per_block - 1) / rows_per_block);
    if (w_f32)
      gemv_cols_kernel<true><<<g, 256, 0, stream>>>(W, m, n, x, col_part, rows_per_block);
    else
      gemv_cols_kernel<false><<<g, 256, 0, stream>>>(W, m, n, x, col_part, rows_per_block);
    check_launch("gemv_cols");
    gemv_cols_sum_kernel<<<(n + 255) / 256, 256, 0, stream>>>(col_part, static_cast<int>(g.y), n, y);
    check_launch("gemv_cols_sum");
  };
  normalize_kernel<<<1, 1024, 0, stream>>>(v, n, eps, nullptr);
  check_launch("normalize");
  for (int it = 0; it < iters; ++it) {
    rows(v, u);
    normalize_kernel<<<1, 1024, 0, stream>>>(u, m, eps, nullptr);
    check_launch("normalize");
    cols(u, v);
    normalize_kernel<<<1, 1024, 0, stream>>>(v, n, eps, nullptr);
    check_launch("normalize");
  }
  // sigma = u^T W v
  rows(v, work);
  dot_kernel<<<1, 1024, 0, stream>>>(u, work, m, sigma);
  check_launch("dot");
}

}  // namespace mmf
