// Grouped bf16 GEMM for the transformer linears, on CTA pairs (cta_group::2), with the
// neighbouring elementwise work fused into the epilogue.
//
// It replaces the library GEMMs behind the reference's nn.Linear layers under fully_shard
// (examples/train_gpt.py:182-199 GPT-2 block, :261 LM head) and the Llama-3 linears of the
// 8B workload, for all three GEMMs of a training step:
//   forward      Y  = X W^T        A = X [M, K] (K-major), B = W [N, K] (K-major)
//   input grad   dX = dY W         A = dY [M, N'] (K-major), B = W [N', K] read MN-major
//   weight grad  dW = dY^T X       A = dY^T (MN-major), B = X (MN-major), fp32 or bf16, += allowed
//
// One launch may concatenate up to three operands along one axis ("segments"):
//   rows (M)      the weight gradients of wq / wk / wv (or w1 / w3) against the same X
//   columns (N)   the q / k / v projections of one input (RoPE fused on q and k)
//   reduction (K) dX = dQ Wq + dK Wk + dV Wv (or dG W1 + dU W3) as one accumulation
// Segments start on tile (or 64-deep k-block) boundaries; ragged extents are zero-filled by
// TMA on load and bounds-checked on store, so any M, N, K with 16-byte row pitches works.
//
// Epilogues (template EPI):
//   STORE       out = alpha acc (+ bias[col]) (+ C) (+ out, when accumulating); bf16 or fp32
//   ROPE        STORE, then rotary embedding (rotate-half, theta^(-2i/d)) on flagged segments
//   SWIGLU      the two CTAs of a pair load W1 and W3 rows of the same 128 hidden units, so
//               each TMEM row holds gate | up: writes h = silu(g) u, g and u
//   SWIGLU_BWD  dH = dY W2 in TMEM; reads g, u; writes dg = dh u s (1 + g (1 - s)), du = dh g s
//   GELU        z = acc + bias; writes gelu(z) (erf form) and z
//   GELU_BWD    dA = dY Wproj in TMEM; reads z; writes dz = da (Phi(z) + z phi(z))
//   SCATTER     weight gradient (+ C) stored straight into each row's owner (GEMM -> reduce-
//               scatter): every warp stages 32 rows x 64 columns in shared memory (XOR-swizzled)
//               and stores whole 128-byte row segments, four rows per instruction, to the owner
//               addresses (peer-mapped receive slots over NVLink)
//
// Warp roles per CTA (192 threads): warp 0 TMA producer, warp 1 TMEM allocator and (leader CTA)
// MMA issuer, warps 2..5 epilogue.  6-stage ring of 32 KB per CTA, 2 x 256 TMEM columns so the
// epilogue of one tile overlaps the main loop of the next.  Persistent grid, one pair per two
// SMs.  No TMA multicast; every wait is bounded (tc_common.cuh) and records an error code.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <utility>
#include <cmath>
#include <mutex>
#include <type_traits>
#include <stdexcept>
#include <string>

#include "kernels.h"
#include "tc_common.cuh"
#include "tma_host.h"

namespace mmf {

namespace {

constexpr int L_BK = 64;
constexpr int L_HALF = 128;  // rows of A staged by each CTA of the pair
constexpr int L_TM = 256;    // output rows per pair tile
constexpr int L_THREADS = 192;
constexpr uint32_t L_TMEM_COLS = 512;

// Tile geometry for TN output columns per pair tile (MMA N, 256).  Each CTA stages 128 rows of
// A and TN/2 rows of B per 64-deep k-block; the ring takes as many stages as fit in 192 KB of
// shared memory (6).
template <int TN>
struct LinTile {
  static constexpr int BH = TN / 2;
  static constexpr int A_BYTES = L_HALF * L_BK * 2;
  static constexpr int B_BYTES = BH * L_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int STAGING_BYTES = 4 * 32 * 128;  // SCATTER: 32 rows x 64 bf16 per epilogue warp
};
template <int TN, int EPI>
constexpr int lin_smem_bytes() {
  // SCATTER: 1 KB reserved after the barriers, then the 1 KB-aligned staging
  return LinTile<TN>::SMEM_BYTES + (EPI == LIN_EPI_SCATTER ? 1024 + LinTile<TN>::STAGING_BYTES : 0);
}

struct LinMaps {
  CUtensorMap a[3];
  CUtensorMap b[3];
};

struct LinDev {
  int M, N;  // output extents (rows, columns of the concatenated problem; SWIGLU: N = hidden units)
  int tiles_m, tiles_n, num_tiles, band;
  int row_bands;     // raster: 1 = bands of `band` tile rows with columns fastest, 0 = column bands
  int axis, nseg;    // segment axis (LIN_SEG_*) and count
  int seg_tile[4];   // segment s covers tiles (K: k-blocks) [seg_tile[s], seg_tile[s+1])
  int seg_len[3];    // true rows / columns of each segment (axis M / N)
  int total_kb;      // k-blocks of one tile (all K segments)
  void* out[3];
  int64_t ldo[3];
  int vec_ok[3];     // 16-byte vector stores allowed for output s
  int in_vec;        // 16-byte vector loads allowed for C / aux0 / aux1
  int out_f32, accumulate;
  float alpha;
  const __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* aux0;
  const __nv_bfloat16* aux1;
  int64_t ld_aux;
  const __nv_bfloat16* bias;
  int rope_mask, seq_len, head_dim;
  float log2_theta;
  const int64_t* scatter_ptrs;
  int scatter_nseg;
  int64_t scatter_rows;
  // Split last wave: work items [0, full_tiles) are whole tiles; the remaining tiles are each
  // split into `split` parts along K (items full_tiles + j * split + part).  Part 0 owns the
  // tile's epilogue; parts 1.. write fp32 partial sums to part_ws and count up part_flags.
  int full_tiles, split, num_items;
  float* part_ws;
  uint32_t* part_flags;
  int* err;
};

// Work item w -> tile t, split part (-1 = whole tile), and its k-block range [kb0, kb1).
__device__ __forceinline__ void lin_item(const LinDev& p, int w, int& t, int& part, int& kb0, int& kb1) {
  if (w < p.full_tiles) {
    t = w;
    part = -1;
    kb0 = 0;
    kb1 = p.total_kb;
    return;
  }
  const int r = w - p.full_tiles;
  const int j = r / p.split;
  part = r - j * p.split;
  t = p.full_tiles + j;
  kb0 = static_cast<int>((static_cast<int64_t>(part) * p.total_kb) / p.split);
  kb1 = static_cast<int>((static_cast<int64_t>(part + 1) * p.total_kb) / p.split);
}

constexpr int64_t L_PART_FLOATS = static_cast<int64_t>(L_TM) * 256;  // one fp32 partial tile

// The accumulator of one thread's row for the epilogue: its TMEM lane, plus (when this is the
// owning part of a split tile) the other parts' fp32 partial rows, added on every load.
struct AccRow {
  uint32_t t_row;
  const float* part;  // this thread's row in the first partial slot of the tile, or nullptr
  int nparts;
};
__device__ __forceinline__ void acc_ld(const AccRow& a, int col, float* v) {
  tmem_ld_32cols(a.t_row + col, v);
  for (int q = 0; q < a.nparts; ++q) {
    const float4* src = reinterpret_cast<const float4*>(a.part + q * L_PART_FLOATS + col);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 w = src[i];
      v[4 * i] += w.x;
      v[4 * i + 1] += w.y;
      v[4 * i + 2] += w.z;
      v[4 * i + 3] += w.w;
    }
  }
}

__device__ __forceinline__ int seg_of(const LinDev& p, int tile) {
  int s = 0;
  while (s + 1 < p.nseg && tile >= p.seg_tile[s + 1]) ++s;
  return s;
}

__device__ __forceinline__ void lin_tile(const LinDev& p, int t, int& tm, int& tn) {
  // Bands of `band` tile columns with rows fastest inside a band (the pairs running at the same
  // time share a narrow slab of B and walk all of A), or the transpose: bands of tile rows with
  // columns fastest (they share a slab of A and walk all of B).  The host picks the order that
  // keeps the walked operand in L2, so each operand comes from DRAM about once.
  const int n_inner = p.row_bands ? p.tiles_n : p.tiles_m;
  const int n_outer = p.row_bands ? p.tiles_m : p.tiles_n;
  const int span = p.band * n_inner;
  const int bi = t / span;
  const int rr = t - bi * span;
  const int w = min(p.band, n_outer - bi * p.band);
  const int outer = bi * p.band + rr % w;
  const int inner = rr / w;
  tm = p.row_bands ? outer : inner;
  tn = p.row_bands ? inner : outer;
}

__device__ __forceinline__ void ld_bf16x32(const __nv_bfloat16* src, float* v, bool vec, int n) {
  if (vec && n >= 32) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w = s[q];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        v[q * 8 + 2 * e] = f.x;
        v[q * 8 + 2 * e + 1] = f.y;
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = (i < n) ? __bfloat162float(src[i]) : 0.f;
}

__device__ __forceinline__ void st_bf16x32(__nv_bfloat16* dst, const float* v, bool vec, int n) {
  if (vec && n >= 32) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
      d[q] = w;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < n) dst[i] = __float2bfloat16_rn(v[i]);
}

__device__ __forceinline__ float sigmoid_f(float g) { return 1.f / (1.f + expf(-g)); }

// Output address helpers: row r (segment-local), column c (segment-local) of output s.
__device__ __forceinline__ __nv_bfloat16* out_bf(const LinDev& p, int s, int64_t r, int c) {
  return static_cast<__nv_bfloat16*>(p.out[s]) + r * p.ldo[s] + c;
}

// STORE / ROPE epilogue of one 32-column chunk already in v (fp32), for output s.
__device__ __forceinline__ void store_chunk(const LinDev& p, int s, int64_t r, int col, int ncols, float* v) {
  const int n = min(32, ncols - col);
  if (n <= 0) return;
  const bool vec = p.vec_ok[s] != 0;
  if (p.out_f32) {
    float* o = static_cast<float*>(p.out[s]) + r * p.ldo[s] + col;
    if (vec && n >= 32) {
      float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        if (p.accumulate) {
          const float4 old = o4[q];
          w.x += old.x;
          w.y += old.y;
          w.z += old.z;
          w.w += old.w;
        }
        o4[q] = w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < n) o[i] = p.accumulate ? o[i] + v[i] : v[i];
    }
    return;
  }
  __nv_bfloat16* o = out_bf(p, s, r, col);
  if (p.accumulate) {
    float old[32];
    ld_bf16x32(o, old, vec, n);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += old[i];
  }
  st_bf16x32(o, v, vec, n);
}

template <int EPI, int TN>
__device__ __forceinline__ void lin_epilogue(const LinDev& p, int tm, int tn, int row_in_tile, const AccRow& t_row,
                                             uint8_t* staging) {
  const int grow = tm * L_TM + row_in_tile;  // row of the concatenated output
  int s = 0;
  int64_t r = grow;
  int rlim = p.M;
  int cbase = tn * TN;
  int clim = p.N;
  if (p.axis == LIN_SEG_M) {
    s = seg_of(p, tm);
    r = grow - static_cast<int64_t>(p.seg_tile[s]) * L_TM;
    rlim = p.seg_len[s];
  } else if (p.axis == LIN_SEG_N) {
    s = seg_of(p, tn);
    cbase = (tn - p.seg_tile[s]) * TN;
    clim = p.seg_len[s];
  }
  const bool row_ok = r < rlim;

  if constexpr (EPI == LIN_EPI_SWIGLU) {
    // TMEM columns [0, TN/2): gate of hidden units tn*TN/2 + c; [TN/2, TN): up of the same units
    const int h0 = tn * (TN / 2);
#pragma unroll 1
    for (int c = 0; c < TN / 64; ++c) {
      const int col = h0 + c * 32;
      if (col >= p.N) break;  // uniform across the warp
      float g[32], u[32];
      acc_ld(t_row, c * 32, g);
      acc_ld(t_row, TN / 2 + c * 32, u);
      if (!row_ok) continue;
      const int n = min(32, p.N - col);
      float h[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        g[i] *= p.alpha;
        u[i] *= p.alpha;
        h[i] = g[i] * sigmoid_f(g[i]) * u[i];
      }
      st_bf16x32(out_bf(p, 0, r, col), h, p.vec_ok[0] != 0, n);
      st_bf16x32(out_bf(p, 1, r, col), g, p.vec_ok[1] != 0, n);
      st_bf16x32(out_bf(p, 2, r, col), u, p.vec_ok[2] != 0, n);
    }
    return;
  } else if constexpr (EPI == LIN_EPI_SWIGLU_BWD || EPI == LIN_EPI_GELU_BWD) {
#pragma unroll 1
    for (int c = 0; c < TN / 32; ++c) {
      const int col = cbase + c * 32;
      if (col >= clim) break;
      float d[32];
      acc_ld(t_row, c * 32, d);
      if (!row_ok) continue;
      const int n = min(32, clim - col);
      const bool vin = p.in_vec != 0;
      float g[32];
      ld_bf16x32(p.aux0 + r * p.ld_aux + col, g, vin, n);
      if constexpr (EPI == LIN_EPI_SWIGLU_BWD) {
        float u[32], du[32];
        ld_bf16x32(p.aux1 + r * p.ld_aux + col, u, vin, n);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float dv = d[i] * p.alpha;
          const float sg = sigmoid_f(g[i]);
          d[i] = dv * u[i] * sg * (1.f + g[i] * (1.f - sg));
          du[i] = dv * g[i] * sg;
        }
        st_bf16x32(out_bf(p, 0, r, col), d, p.vec_ok[0] != 0, n);
        st_bf16x32(out_bf(p, 1, r, col), du, p.vec_ok[1] != 0, n);
      } else {
        constexpr float kInvSqrt2 = 0.70710678118654752f;
        constexpr float kInvSqrt2Pi = 0.39894228040143268f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float z = g[i];
          const float cdf = 0.5f * (1.f + erff(z * kInvSqrt2));
          const float pdf = kInvSqrt2Pi * expf(-0.5f * z * z);
          d[i] = d[i] * p.alpha * (cdf + z * pdf);
        }
        st_bf16x32(out_bf(p, 0, r, col), d, p.vec_ok[0] != 0, n);
      }
    }
    return;
  } else if constexpr (EPI == LIN_EPI_GELU) {
#pragma unroll 1
    for (int c = 0; c < TN / 32; ++c) {
      const int col = cbase + c * 32;
      if (col >= clim) break;
      float z[32];
      acc_ld(t_row, c * 32, z);
      if (!row_ok) continue;
      const int n = min(32, clim - col);
      float a[32];
      constexpr float kInvSqrt2 = 0.70710678118654752f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        z[i] *= p.alpha;
        if (p.bias != nullptr && i < n) z[i] += __bfloat162float(p.bias[col + i]);
        // the saved pre-activation is rounded to bf16; the activation uses the same value
        z[i] = __bfloat162float(__float2bfloat16_rn(z[i]));
        a[i] = 0.5f * z[i] * (1.f + erff(z[i] * kInvSqrt2));
      }
      st_bf16x32(out_bf(p, 0, r, col), a, p.vec_ok[0] != 0, n);
      st_bf16x32(out_bf(p, 1, r, col), z, p.vec_ok[1] != 0, n);
    }
    return;
  } else if constexpr (EPI == LIN_EPI_SCATTER) {
    // stage[row][unit ^ (row & 7)]: 32 rows x 8 units of 16 bytes (64 bf16) for this warp
    uint8_t* stage = staging;
    const int lane = row_in_tile & 31;
    const int64_t warp_row0 = grow - lane;  // first output row of this warp
#pragma unroll 1
    for (int c64 = 0; c64 < TN / 64; ++c64) {
      const int col = cbase + c64 * 64;
      if (col >= clim) break;  // uniform across the warp
      float v[64];
      acc_ld(t_row, c64 * 64, v);
      acc_ld(t_row, c64 * 64 + 32, v + 32);
      const int n = min(64, clim - col);
      if (row_ok && p.C != nullptr) {
        float c_[32];
        ld_bf16x32(p.C + r * p.ldc + col, c_, p.in_vec != 0, n);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += c_[i];
        if (n > 32) {
          ld_bf16x32(p.C + r * p.ldc + col + 32, c_, p.in_vec != 0, n - 32);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[32 + i] += c_[i];
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        uint4 w;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[u * 8 + 2 * e] * p.alpha, v[u * 8 + 2 * e + 1] * p.alpha);
        *reinterpret_cast<uint4*>(stage + lane * 128 + ((u ^ (lane & 7)) * 16)) = w;
      }
      __syncwarp();
      const int u = lane & 7;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = (lane >> 3) + 4 * i;  // row of the warp's 32 this lane stores now
        const uint4 w = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((u ^ (rr & 7)) * 16));
        const int64_t orow = warp_row0 + rr;
        const int c = col + u * 8;
        if (orow < p.M && c < clim) {
          const int owner = static_cast<int>(orow / p.scatter_rows);
          if (MMF_DCHECK(owner < p.scatter_nseg, p.err, ERR_CHECK_BOUNDS)) {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.scatter_ptrs[owner]) +
                                 (orow - static_cast<int64_t>(owner) * p.scatter_rows) * p.ldo[0] + c;
            *reinterpret_cast<uint4*>(dst) = w;
          }
        }
      }
      __syncwarp();
    }
    return;
  } else {
    // STORE and ROPE
    const bool rope = (EPI == LIN_EPI_ROPE) && ((p.rope_mask >> s) & 1);
    if (rope) {
      // rotate-half pairs (i, i + d/2) inside each head; a 256-column tile holds whole heads
      const int hc = p.head_dim / 32;  // 32-column chunks per head (2 or 4)
      const int half_c = hc / 2;
      const float pos = static_cast<float>(r % p.seq_len);
#pragma unroll 1
      for (int a = 0; a < TN / 32; ++a) {
        if ((a % hc) >= half_c) continue;
        const int b = a + half_c;
        const int col_a = cbase + a * 32;
        if (col_a >= clim) break;
        float x1[32], x2[32];
        acc_ld(t_row, a * 32, x1);
        acc_ld(t_row, b * 32, x2);
        if (!row_ok) continue;
        const int i0 = (a % hc) * 32;
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float inv_freq = exp2f(-p.log2_theta * (2.f * (i0 + e)) / p.head_dim);  // theta^(-2i/d)
          float sn, cs;
          sincosf(pos * inv_freq, &sn, &cs);
          const float v1 = x1[e] * p.alpha, v2 = x2[e] * p.alpha;
          x1[e] = v1 * cs - v2 * sn;
          x2[e] = v2 * cs + v1 * sn;
        }
        store_chunk(p, s, r, col_a, clim, x1);
        store_chunk(p, s, r, cbase + b * 32, clim, x2);
      }
      return;
    }
#pragma unroll 1
    for (int c = 0; c < TN / 32; ++c) {
      const int col = cbase + c * 32;
      if (col >= clim) break;
      float v[32];
      acc_ld(t_row, c * 32, v);
      if (!row_ok) continue;
      const int n = min(32, clim - col);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= p.alpha;
      if (p.bias != nullptr) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < n) v[i] += __bfloat162float(p.bias[col + i]);
      }
      if (p.C != nullptr) {
        float c_[32];
        ld_bf16x32(p.C + r * p.ldc + col, c_, p.in_vec != 0, n);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += c_[i];
      }
      store_chunk(p, s, r, col, clim, v);
    }
  }
}

template <bool A_MN, bool B_MN, int EPI, int TN>
__global__ void __launch_bounds__(L_THREADS, 1)
    linear_gemm_kernel(const __grid_constant__ LinMaps maps, const LinDev p) {
  using G = LinTile<TN>;
  constexpr int L_STAGES = G::STAGES, L_A_BYTES = G::A_BYTES, L_B_BYTES = G::B_BYTES;
  constexpr int L_STAGE_BYTES = G::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + L_STAGES * L_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + L_STAGES * L_B_BYTES);
  uint64_t* empty = full + L_STAGES;
  uint64_t* tfull = empty + L_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  // SCATTER staging after the barriers (1 KB reserved for them), 1 KB-aligned
  uint8_t* staging = sB + L_STAGES * L_B_BYTES + 1024;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  int* err = p.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&tfull[j], 1);
      mbar_init(&tempty[j], 8);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < 3; ++s) {
      tma_prefetch_desc(&maps.a[s]);
      tma_prefetch_desc(&maps.b[s]);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L_TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrive / TMA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) -------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = cluster; w < p.num_items && ok; w += nclusters) {
        int t, part, kb0, kb1;
        lin_item(p, w, t, part, kb0, kb1);
        int tm, tn;
        lin_tile(p, t, tm, tn);
        // rows of A this CTA stages, and which A map (row segments)
        int am = 0, a_row = tm * L_TM + static_cast<int>(rank) * L_HALF;
        if (p.axis == LIN_SEG_M) {
          am = seg_of(p, tm);
          a_row -= p.seg_tile[am] * L_TM;
        }
        // rows (K-major) or columns (MN-major) of B this CTA stages, and which B map
        int bm = 0, b_row = tn * TN + static_cast<int>(rank) * G::BH;
        if (EPI == LIN_EPI_SWIGLU) {
          bm = static_cast<int>(rank);  // CTA 0: W1 (gate) rows, CTA 1: W3 (up) rows
          b_row = tn * G::BH;
        } else if (p.axis == LIN_SEG_N) {
          bm = seg_of(p, tn);
          b_row -= p.seg_tile[bm] * TN;
        }
        int ks = 0;  // K segment
        int ks_end = (p.axis == LIN_SEG_K) ? p.seg_tile[1] : p.total_kb;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (p.axis == LIN_SEG_K) {
            while (kb >= ks_end) {
              ++ks;
              ks_end = p.seg_tile[ks + 1];
            }
            am = ks;
            bm = ks;
          }
          const int kl = (p.axis == LIN_SEG_K) ? kb - p.seg_tile[ks] : kb;
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, ERR_TMA_EMPTY_TIMEOUT)) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L_STAGE_BYTES);
          // debug builds: every innermost TMA coordinate on its 16-byte boundary and every map
          // index inside the segment tables (a failed check records its code and skips; the
          // bounded wait on the stage's barrier then unwinds the kernel)
          if (!MMF_DCHECK_TMA_X(A_MN ? a_row : kl * L_BK, 2, err) || !MMF_DCHECK_TMA_X(B_MN ? b_row : kl * L_BK, 2, err) ||
              !MMF_DCHECK(am >= 0 && am < 3 && bm >= 0 && bm < 3, err, ERR_CHECK_BOUNDS))
            continue;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
              tma_load_3d_pair(sA + stage * L_A_BYTES + c * (L_BK * 64 * 2), &maps.a[am], fb, a_row + c * 64,
                               kl * L_BK, 0);
          } else {
            tma_load_3d_pair(sA + stage * L_A_BYTES, &maps.a[am], fb, kl * L_BK, a_row, 0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < G::BH / 64; ++c)
              tma_load_3d_pair(sB + stage * L_B_BYTES + c * (L_BK * 64 * 2), &maps.b[bm], fb, b_row + c * 64,
                               kl * L_BK, 0);
          } else {
            tma_load_3d_pair(sB + stage * L_B_BYTES, &maps.b[bm], fb, kl * L_BK, b_row, 0);
          }
          if (++stage == L_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader CTA only) ---------------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(L_TM, TN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int w = cluster; w < p.num_items && ok; w += nclusters) {
        int t, part, kb0, kb1;
        lin_item(p, w, t, part, kb0, kb1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, ERR_MMA_TMEM_EMPTY_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * TN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, ERR_MMA_FULL_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * L_A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * L_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < L_BK / 16; ++kk) {
            const uint64_t ad =
                A_MN ? sdesc_mnmajor(a_addr + kk * 16 * 128, L_BK * 64 * 2) : sdesc_kmajor(a_addr + kk * 32);
            const uint64_t bd =
                B_MN ? sdesc_mnmajor(b_addr + kk * 16 * 128, L_BK * 64 * 2) : sdesc_kmajor(b_addr + kk * 32);
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || kk) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == L_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit_pair(drain, 0x1);
      mbar_wait(drain, 0, err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else {
    // ------------------------------ epilogue (both CTAs) -----------------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    const int row_in_tile = static_cast<int>(rank) * L_HALF + q * 32 + lane;
    for (int w = cluster; w < p.num_items; w += nclusters) {
      int t, part, kb0, kb1;
      lin_item(p, w, t, part, kb0, kb1);
      int tm, tn;
      lin_tile(p, t, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, err, ERR_EPI_TMEM_FULL_TIMEOUT)) break;
      tc_fence_after();
      AccRow ar{tmem_base + static_cast<uint32_t>(acc * TN) + (static_cast<uint32_t>(q * 32) << 16), nullptr, 0};
      bool skip = false;
      if (part >= 0) {
        const int j = t - p.full_tiles;
        uint32_t* flag = p.part_flags + j * 8 + static_cast<int>(rank) * 4 + q;  // one per epilogue warp
        float* rowbase = p.part_ws + static_cast<int64_t>(j) * (p.split - 1) * L_PART_FLOATS +
                         static_cast<int64_t>(row_in_tile) * 256;
        if (part > 0) {
          // a non-owning part: its fp32 partial row to slot (part - 1), then count up the flag
          float* dst = rowbase + static_cast<int64_t>(part - 1) * L_PART_FLOATS;
#pragma unroll 1
          for (int c = 0; c < TN / 32; ++c) {
            float v[32];
            tmem_ld_32cols(ar.t_row + c * 32, v);
            float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
          __threadfence();
          __syncwarp();
          if (lane == 0) red_release_gpu_add(flag, 1u);
          skip = true;
        } else {
          // the owning part: wait (bounded) until the other parts' rows of this warp have landed
          bool ready = true;
          if (lane == 0) {
            const uint64_t t0 = globaltimer_ns();
            while (ld_acquire_gpu(flag) < static_cast<uint32_t>(p.split - 1)) {
              if (globaltimer_ns() - t0 > MMF_WAIT_TIMEOUT_NS) {
                atomicCAS(err, 0, ERR_PEER_FLAG_TIMEOUT);
                ready = false;
                break;
              }
              __nanosleep(32);
            }
            *flag = 0;  // consumed: zero for the next launch
          }
          ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
          if (ready) {
            ar.part = rowbase;
            ar.nparts = p.split - 1;
          }
        }
      }
      if (!skip) lin_epilogue<EPI, TN>(p, tm, tn, row_in_tile, ar, staging + q * (32 * 128));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + static_cast<uint32_t>(acc * sizeof(uint64_t)));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // the leader's MMAs read CTA 1's smem: nobody leaves before both are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L_TMEM_COLS);
  }
}

// Scratch of the split last wave, one per (device, stream) so that launches on different
// streams never share it: fp32 partial tiles (fewer than 74 of the at most 148 / 2 pairs) and one
// flag per epilogue warp of each split tile.  The owning part zeroes its flags after use.
struct SplitScratch {
  float* ws = nullptr;
  uint32_t* flags = nullptr;
};
constexpr int L_MAX_SPLIT_TILES = 128;
SplitScratch& split_scratch(int dev, cudaStream_t stream) {
  static std::map<std::pair<int, cudaStream_t>, SplitScratch> cache;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  SplitScratch& sc = cache[{dev, stream}];
  if (sc.ws == nullptr) {
    const size_t ws_bytes = sizeof(float) * static_cast<size_t>(L_PART_FLOATS) * L_MAX_SPLIT_TILES;
    const size_t fl_bytes = sizeof(uint32_t) * 8 * L_MAX_SPLIT_TILES;
    if (cudaMalloc(&sc.ws, ws_bytes) != cudaSuccess || cudaMalloc(&sc.flags, fl_bytes) != cudaSuccess)
      throw std::runtime_error("mmf: linear_gemm: cannot allocate the split-wave scratch");
    if (cudaMemsetAsync(sc.flags, 0, fl_bytes, stream) != cudaSuccess)
      throw std::runtime_error("mmf: linear_gemm: cannot clear the split-wave flags");
  }
  return sc;
}

std::atomic<int> g_split_tail{1};  // 1: split the last wave (default), 0: whole tiles only

int num_sms(int dev) {
  static int sms[64] = {0};
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return sms[dev];
}

// CTA pairs of this kernel that are resident at the same time (one CTA per SM; a GPC with an
// odd number of free SMs leaves one idle).  The persistent grid never exceeds it, so every pair
// runs concurrently: the owner of a split tile can wait for the other parts without deadlock.
// All instantiations take one CTA per SM; the query uses the largest shared-memory size.
int resident_pairs(int dev) {
  static int pairs[64] = {0};
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (pairs[dev] == 0) {
    auto kern = linear_gemm_kernel<true, true, LIN_EPI_SCATTER, 256>;
    const int smem = lin_smem_bytes<256, LIN_EPI_SCATTER>();
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 512, 1, 1);
    cfg.blockDim = dim3(L_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms(dev) / 2;
    }
    pairs[dev] = std::min(n, num_sms(dev) / 2);
  }
  return pairs[dev];
}

template <bool A_MN, bool B_MN, int EPI, int TN>
cudaError_t launch_lin(const LinMaps& maps, const LinDev& p, int clusters, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(linear_gemm_kernel<A_MN, B_MN, EPI, TN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, lin_smem_bytes<TN, EPI>());
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(L_THREADS, 1, 1);
  cfg.dynamicSmemBytes = lin_smem_bytes<TN, EPI>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, linear_gemm_kernel<A_MN, B_MN, EPI, TN>, maps, p);
}

[[noreturn]] void fail(const std::string& what) { throw std::runtime_error("mmf: linear_gemm: " + what); }



bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace

void set_linear_split_tail(bool on) { g_split_tail.store(on ? 1 : 0); }

int linear_resident_pairs() {
  int dev = 0;
  cudaGetDevice(&dev);
  return resident_pairs(dev);
}

void linear_gemm(const LinearGemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0) fail("empty output");
  if (a.nseg < 1 || a.nseg > 3) fail("1..3 operand segments");
  if (a.axis != LIN_SEG_NONE && a.axis != LIN_SEG_M && a.axis != LIN_SEG_N && a.axis != LIN_SEG_K)
    fail("bad segment axis");
  if (a.axis == LIN_SEG_NONE && a.nseg != 1) fail("segments need a segment axis");
  const int epi = a.epilogue;
  if (epi < LIN_EPI_STORE || epi > LIN_EPI_SCATTER) fail("bad epilogue");
  const bool fwd_kind = !a.a_mn && !a.b_mn;
  const bool dx_kind = !a.a_mn && a.b_mn;
  const bool dw_kind = a.a_mn && a.b_mn;
  if (!fwd_kind && !dx_kind && !dw_kind) fail("unsupported operand majorness (A MN-major needs B MN-major)");
  if ((epi == LIN_EPI_ROPE || epi == LIN_EPI_SWIGLU || epi == LIN_EPI_GELU) && !fwd_kind)
    fail("ROPE / SWIGLU / GELU epilogues are forward epilogues");
  if ((epi == LIN_EPI_SWIGLU_BWD || epi == LIN_EPI_GELU_BWD) && !dx_kind)
    fail("SWIGLU_BWD / GELU_BWD epilogues follow an input-gradient GEMM");
  if (epi == LIN_EPI_SCATTER) {
    if (!dw_kind || a.nseg != 1) fail("SCATTER is the epilogue of one weight-gradient GEMM");
    if (a.out_f32 || a.accumulate) fail("SCATTER stores bf16 without reading the destination");
    if (a.scatter_ptrs == nullptr || a.scatter_nseg < 1 || a.scatter_rows < 1) fail("SCATTER needs its owner table");
    if (a.N % 8 || a.ldo[0] % 8) fail("SCATTER needs N % 8 == 0 and a 16-byte row pitch");
  }
  if (epi == LIN_EPI_SWIGLU && (a.axis != LIN_SEG_N || a.nseg != 2)) fail("SWIGLU takes the two weights W1, W3");
  if (epi != LIN_EPI_STORE && epi != LIN_EPI_ROPE && (a.out_f32 || a.accumulate))
    fail("fp32 / accumulating output only with the STORE epilogue");
  if ((a.C || a.bias) && a.nseg != 1 && a.axis != LIN_SEG_K) fail("residual / bias need one output segment");
  if (epi == LIN_EPI_ROPE && (a.head_dim != 64 && a.head_dim != 128)) fail("fused RoPE needs head_dim 64 or 128");

  int dev = 0;
  cudaGetDevice(&dev);
  LinDev p{};
  p.M = a.M;
  p.N = a.N;
  p.axis = a.axis;
  p.nseg = a.nseg;
  p.alpha = a.alpha;
  p.out_f32 = a.out_f32 ? 1 : 0;
  p.accumulate = a.accumulate ? 1 : 0;
  p.C = static_cast<const __nv_bfloat16*>(a.C);
  p.ldc = a.ldc;
  p.aux0 = static_cast<const __nv_bfloat16*>(a.aux0);
  p.aux1 = static_cast<const __nv_bfloat16*>(a.aux1);
  p.ld_aux = a.ld_aux;
  p.bias = static_cast<const __nv_bfloat16*>(a.bias);
  p.rope_mask = a.rope_mask;
  p.seq_len = a.seq_len > 0 ? a.seq_len : 1;
  p.head_dim = a.head_dim;
  p.log2_theta = a.rope_theta > 0.f ? log2f(a.rope_theta) : 0.f;
  p.scatter_ptrs = a.scatter_ptrs;
  p.scatter_nseg = a.scatter_nseg;
  p.scatter_rows = a.scatter_rows;
  p.err = device_error_word(dev);

  const int elt = a.out_f32 ? 4 : 2;
  for (int s = 0; s < 3; ++s) {
    p.out[s] = a.out[s];
    p.ldo[s] = a.ldo[s];
    p.vec_ok[s] = a.out[s] != nullptr && aligned16(a.out[s]) && (a.ldo[s] * elt) % 16 == 0;
  }
  if (epi == LIN_EPI_SWIGLU_BWD || epi == LIN_EPI_GELU_BWD) {
    if (a.aux0 == nullptr || (epi == LIN_EPI_SWIGLU_BWD && a.aux1 == nullptr)) fail("missing saved activations");
    p.in_vec = aligned16(a.aux0) && (a.aux1 == nullptr || aligned16(a.aux1)) && (a.ld_aux % 8) == 0;
  }
  if (a.C) p.in_vec = aligned16(a.C) && (a.ldc % 8) == 0;

  // k-blocks and K-segment starts (independent of the tile width)
  int total_kb = 0;
  if (a.axis == LIN_SEG_K) {
    for (int s = 0; s < a.nseg; ++s) {
      p.seg_tile[s] = total_kb;
      total_kb += (a.K[s] + L_BK - 1) / L_BK;
    }
    p.seg_tile[a.nseg] = total_kb;
  } else {
    total_kb = (a.K[0] + L_BK - 1) / L_BK;
  }
  if (total_kb <= 0) fail("empty reduction");
  p.total_kb = total_kb;
  const int units = resident_pairs(dev);

  // Tile width: 256 columns.  A 128-wide variant (more tiles, a fuller last wave) measured
  // 0.52-0.65x of the 256-wide kernel on every Llama-3-8B linear (1 B200, bench_gemm.py), so it
  // is not built.
  constexpr int TN = 256;
  // tiles along each axis, row / column segment starts (a segment occupies whole tiles; the
  // part of its last tile past the segment's end is zero-filled on load and never stored)
  int tiles_m = (a.M + L_TM - 1) / L_TM;
  int tiles_n = (epi == LIN_EPI_SWIGLU) ? (a.N + TN / 2 - 1) / (TN / 2) : (a.N + TN - 1) / TN;
  if (a.axis == LIN_SEG_M || a.axis == LIN_SEG_N) {
    int acc = 0;
    const int unit = (a.axis == LIN_SEG_M) ? L_TM : TN;
    for (int s = 0; s < a.nseg; ++s) {
      p.seg_tile[s] = acc;
      p.seg_len[s] = a.seg_len[s];
      acc += (epi == LIN_EPI_SWIGLU) ? 0 : (a.seg_len[s] + unit - 1) / unit;
    }
    if (epi == LIN_EPI_SWIGLU) {
      acc = tiles_n;
      p.seg_tile[1] = 0;
      p.seg_len[0] = p.seg_len[1] = a.N;
    }
    p.seg_tile[a.nseg] = acc;
    if (a.axis == LIN_SEG_M)
      tiles_m = acc;
    else
      tiles_n = acc;
  } else if (a.axis != LIN_SEG_K) {
    p.seg_tile[0] = 0;
    p.seg_tile[1] = 1 << 30;
  }
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.num_tiles = tiles_m * tiles_n;
  // Split last wave: the tiles of a last, partly filled wave of pairs are split along K over the
  // pairs that would otherwise idle; the fp32 partial sums go through a per-(device, stream)
  // scratch area of at most units - 1 tiles.  The fix-up (partials written, then read by the
  // owning part's epilogue) costs a few microseconds, so each part must keep at least 128
  // k-blocks (K >= 8192): on a B200 the split made 4096-deep GEMMs 2-5 % slower and the
  // 128256-deep LM-head input gradient 14 % faster.
  {
    const int tail = p.num_tiles % units;
    int split = tail > 0 ? units / tail : 1;
    split = std::min(split, p.total_kb / 128);
    split = std::min(split, 8);
    if (tail == 0 || split < 2 || g_split_tail.load() == 0 || tail > L_MAX_SPLIT_TILES ||
        tail * (split - 1) > L_MAX_SPLIT_TILES) {
      p.full_tiles = p.num_tiles;
      p.split = 1;
      p.num_items = p.num_tiles;
    } else {
      p.full_tiles = p.num_tiles - tail;
      p.split = split;
      p.num_items = p.full_tiles + tail * split;
      SplitScratch& sc = split_scratch(dev, stream);
      p.part_ws = sc.ws;
      p.part_flags = sc.flags;
    }
  }
  {
    // Operand bytes walked per band: column bands re-read A (all rows) once per band, row bands
    // re-read B.  An operand that fits in half the L2 is read from DRAM once either way.
    auto ceil_div = [](int64_t x, int64_t y) { return (x + y - 1) / y; };
    const int64_t kbytes = static_cast<int64_t>(p.total_kb) * L_BK * 2;
    const int64_t a_bytes = static_cast<int64_t>(tiles_m) * L_TM * kbytes;
    const int64_t b_bytes = static_cast<int64_t>(tiles_n) * TN * kbytes;
    const int64_t l2_half = 60ll << 20;
    const int band_c = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles_n, ceil_div(units, tiles_m))));
    const int band_r = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(tiles_m, ceil_div(units, tiles_n))));
    const int64_t cost_c = (a_bytes <= l2_half ? a_bytes : a_bytes * ceil_div(tiles_n, band_c)) + b_bytes;
    const int64_t cost_r = (b_bytes <= l2_half ? b_bytes : b_bytes * ceil_div(tiles_m, band_r)) + a_bytes;
    p.row_bands = cost_r < cost_c ? 1 : 0;
    p.band = p.row_bands ? band_r : band_c;
  }

  // tensor maps: K-major operands [rows, K] with 64-wide boxes of 128 (A) or TN/2 (B) rows;
  // MN-major [K, cols] with 64 x 64 boxes
  LinMaps maps;
  const int na = (a.axis == LIN_SEG_M || a.axis == LIN_SEG_K) ? a.nseg : 1;
  const int nb = (a.axis == LIN_SEG_N || a.axis == LIN_SEG_K) ? a.nseg : 1;
  // only the maps in use are encoded (host time per launch); unused slots repeat slot 0
  for (int s = 0; s < 3; ++s) {
    if (s < na) {
      if (!aligned16(a.A[s])) fail("operands must be 16-byte aligned");
      if (a.a_inner[s] % 8) fail("operand row pitches must be multiples of 8 elements");
      maps.a[s] = a.a_mn ? make_map_bf16_3d(a.A[s], a.a_inner[s], a.a_outer[s], 1, 64, L_BK)
                         : make_map_bf16_3d(a.A[s], a.a_inner[s], a.a_outer[s], 1, L_BK, L_HALF);
    } else {
      maps.a[s] = maps.a[0];
    }
    if (s < nb) {
      if (!aligned16(a.B[s])) fail("operands must be 16-byte aligned");
      if (a.b_inner[s] % 8) fail("operand row pitches must be multiples of 8 elements");
      maps.b[s] = a.b_mn ? make_map_bf16_3d(a.B[s], a.b_inner[s], a.b_outer[s], 1, 64, L_BK)
                         : make_map_bf16_3d(a.B[s], a.b_inner[s], a.b_outer[s], 1, L_BK, TN / 2);
    } else {
      maps.b[s] = maps.b[0];
    }
  }

  const int clusters = p.num_items < units ? p.num_items : units;
  cudaError_t e = cudaSuccess;
  if (fwd_kind) {
    switch (epi) {
      case LIN_EPI_STORE: e = launch_lin<false, false, LIN_EPI_STORE, TN>(maps, p, clusters, stream); break;
      case LIN_EPI_ROPE: e = launch_lin<false, false, LIN_EPI_ROPE, TN>(maps, p, clusters, stream); break;
      case LIN_EPI_SWIGLU: e = launch_lin<false, false, LIN_EPI_SWIGLU, TN>(maps, p, clusters, stream); break;
      case LIN_EPI_GELU: e = launch_lin<false, false, LIN_EPI_GELU, TN>(maps, p, clusters, stream); break;
      default: fail("epilogue not available for the forward GEMM");
    }
  } else if (dx_kind) {
    switch (epi) {
      case LIN_EPI_STORE: e = launch_lin<false, true, LIN_EPI_STORE, TN>(maps, p, clusters, stream); break;
      case LIN_EPI_SWIGLU_BWD: e = launch_lin<false, true, LIN_EPI_SWIGLU_BWD, TN>(maps, p, clusters, stream); break;
      case LIN_EPI_GELU_BWD: e = launch_lin<false, true, LIN_EPI_GELU_BWD, TN>(maps, p, clusters, stream); break;
      default: fail("epilogue not available for the input-gradient GEMM");
    }
  } else if (epi == LIN_EPI_SCATTER) {
    e = launch_lin<true, true, LIN_EPI_SCATTER, TN>(maps, p, clusters, stream);
  } else if (epi == LIN_EPI_STORE) {
    e = launch_lin<true, true, LIN_EPI_STORE, TN>(maps, p, clusters, stream);
  } else {
    fail("the weight-gradient GEMM takes the STORE or SCATTER epilogue");
  }
  count_launch();
  if (e != cudaSuccess) fail(std::string("launch failed: ") + cudaGetErrorString(e));
}

}  // namespace mmf
