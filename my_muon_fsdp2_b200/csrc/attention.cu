// Causal flash attention (GQA) on the sm_100a 5th-generation tensor core.
//
// Forward, one CTA per (128-query block, query head, batch):
//   warp 0      TMA producer: Q once; K_j / V_j per 128-key block into a 2-stage ring
//   warp 1      single-thread tcgen05.mma issuer:  S_j = Q K_j^T  (TMEM, double buffered)
//                                                   O  += P_j V_j   (TMEM, V read MN-major)
//   warps 2..5  softmax: one query row per thread — S_j from TMEM, causal mask on the diagonal
//               block, online max / sum in the exp2 domain, P_j (bf16) into 128B-swizzled smem,
//               O rescaled in TMEM when the running max grows; epilogue O / l -> bf16, and the
//               row log-sum-exp (natural log) for the backward pass.
// All waits are bounded (tc_common.cuh).  Layouts: q [B, T, Hq, D], k/v [B, T, Hkv, D], o like q,
// lse [B, Hq, T] fp32; T % 128 == 0, D in {64, 128}.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <stdexcept>
#include <string>

#include "attention.h"
#include "kernels.h"
#include "tc_common.cuh"
#include "tma_host.h"

namespace mmf {

namespace {

constexpr int QB = 128;  // query rows per CTA
constexpr int KB = 128;  // keys per block
constexpr int BWD_THREADS = 320;  // TMA warp, MMA warp, 8 elementwise warps (2 per TMEM lane quarter)

struct AttnParams {
  int B, T, Hq, Hkv, D;
  float scale_log2;  // softmax scale * log2(e)
  __nv_bfloat16* o;
  float* lse;
  int* err;
};

// byte offset of element (row, col) inside a K-major 128B-swizzled tile made of [rows x 64]
// chunks of 16 KB each (128 rows): the 16-byte unit index is XORed with (row % 8).
__device__ __forceinline__ uint32_t swz_offset(int row, int col) {
  const int chunk = col >> 6;
  const int c = col & 63;
  const int unit = (c >> 3) ^ (row & 7);
  return static_cast<uint32_t>(chunk * (128 * 128) + row * 128 + unit * 16 + (c & 7) * 2);
}

// ======================================================================================
// Forward with two query tiles per CTA (query blocks 2x and 2x+1 of one head): two softmax
// warpgroups, one per tile, so that the tensor core works on one tile's S / P V while the
// other tile's softmax runs, and K_j / V_j are loaded once for both tiles.
//   warp 0      TMA: Q_A, Q_B once; K_j / V_j per key block into a 2-stage ring
//   warp 1      MMA: S_A(0), S_B(0); per j: P_A(j) V_j, S_A(j+1), P_B(j) V_j, S_B(j+1)
//   warps 2..5  softmax + epilogue of tile A;  warps 6..9 of tile B
// TMEM: S_A | S_B (128 columns each; P_t(j) is written as bf16 pairs over S_t(j)) | O_A | O_B.
// ======================================================================================
template <int D>
struct Attn2Smem {
  static constexpr int CH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int Q_OFF = 0;                 // Q_A, Q_B
  static constexpr int K_OFF = 2 * TILE;          // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * TILE;  // 2 stages
  static constexpr int BAR_OFF = V_OFF + 2 * TILE;
  static constexpr int BYTES = (BAR_OFF + 256 + 1024) > 120 * 1024 ? (BAR_OFF + 256 + 1024) : 120 * 1024;
};
constexpr int ATT2_THREADS = 320;

// Online softmax of one query tile (128 rows, one per thread of the 4 calling warps) over key
// blocks 0..nblk-1; P into TMEM over S; O rescaled in TMEM when the reference max moves;
// epilogue O / l -> bf16 and the row log-sum-exp.  The row max is taken on the raw scores (the
// scale is positive), three at a time; the exponent argument is one packed fma s*scale - m per
// pair of scores; the row sum is a packed add; the causal mask is applied only on the diagonal
// block.  FULL_ROW: the whole row of 128 scores in registers (one TMEM read per key block, for
// the 3-warpgroup kernel whose softmax threads hold 224 registers), else two 64-score halves.
template <int D, bool FULL_ROW>
__device__ __forceinline__ void fwd_softmax_tile_v2(const AttnParams& p, uint32_t tS, uint32_t tO, uint64_t* s_full,
                                                    uint64_t* p_full, uint64_t* pv_done, int qb, int nblk, int h,
                                                    int b, int q, int lane) {
  const int r = q * 32 + lane;
  const int qi = qb * QB + r;
  const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
  const float c = p.scale_log2;
  float m2 = -INFINITY, l = 0.f;  // running max in the scaled log2 domain, running sum
  bool ok = true;
  for (int j = 0; j < nblk && ok; ++j) {
    if (!mbar_wait(s_full, j & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const bool diag = (j == qb);
    constexpr int NV = FULL_ROW ? 128 : 64;
    float sv[NV];
    auto mask = [&](float* v, int k0) {  // keys past the query row are masked (diagonal block only)
      const int lim = qi - k0;
#pragma unroll
      for (int e = 0; e < 64; ++e)
        if (e > lim) v[e] = -INFINITY;
    };
    auto load_half = [&](int hf) {  // raw scores of keys j*KB + hf*64 + 0..63
      tmem_ld_32cols_async(tS + lane_off + hf * 64, sv);
      tmem_ld_32cols_async(tS + lane_off + hf * 64 + 32, sv + 32);
      tmem_ld_wait();
      if (diag) mask(sv, j * KB + hf * 64);
    };
    float mx = -INFINITY;
    if constexpr (FULL_ROW) {
      // the whole row in one TMEM read: keys 0..127 -> sv[0..127]
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld_32cols_async(tS + lane_off + cc * 32, sv + cc * 32);
      tmem_ld_wait();
      if (diag) {
        mask(sv, j * KB);
        mask(sv + 64, j * KB + 64);
      }
#pragma unroll
      for (int e = 0; e < 128; e += 2) mx = fmax3(mx, sv[e], sv[e + 1]);
    } else {
      load_half(1);
#pragma unroll
      for (int e = 0; e < 64; e += 2) mx = fmax3(mx, sv[e], sv[e + 1]);
      load_half(0);
#pragma unroll
      for (int e = 0; e < 64; e += 2) mx = fmax3(mx, sv[e], sv[e + 1]);
    }
    const float mxs = mx * c;
    // the reference max moves only when the row max grows by more than 2^8 (then the exponentials stay below 2^8 and fp32 sums cannot overflow)
    const bool grow = (m2 == -INFINITY) || (mxs > m2 + 8.f);
    const float m_new = grow ? mxs : m2;
    const float alpha = (m2 == -INFINITY) ? 0.f : (grow ? fast_exp2(m2 - m_new) : 1.f);
    if (__any_sync(0xffffffffu, j >= 1 && alpha != 1.f)) {
      if (!mbar_wait(pv_done, (j - 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        float o[32];
        tmem_ld_32cols(tO + lane_off + cc * 32, o);
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] *= alpha;
        tmem_st_32cols_async(tO + lane_off + cc * 32, o);
      }
    }
    const float2 c2 = make_float2(c, c);
    const float2 nm = make_float2(-m_new, -m_new);
    float2 sum2 = make_float2(0.f, 0.f);
    // P of keys hf*64 .. hf*64+63 as bf16 pairs over S columns hf*32 .. hf*32+31
    auto exp_store = [&](const float* v, int hf) {
      float pk[32];
#pragma unroll
      for (int e2 = 0; e2 < 32; ++e2) {
        const float2 x = ffma2(make_float2(v[2 * e2], v[2 * e2 + 1]), c2, nm);
        const float2 pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        sum2 = fadd2(sum2, pp);
        __nv_bfloat162 pb = __floats2bfloat162_rn(pp.x, pp.y);
        pk[e2] = *reinterpret_cast<float*>(&pb);
      }
      tmem_st_32cols_async(tS + lane_off + hf * 32, pk);
    };
    if constexpr (FULL_ROW) {
      exp_store(sv, 0);
      exp_store(sv + 64, 1);
    } else {
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        if (hf == 1) {
          tmem_st_wait();  // keys 0..63 stored over S columns 0..31, which were read already
          load_half(1);
        }
        exp_store(sv, hf);
      }
    }
    tmem_st_wait();
    l = l * alpha + (sum2.x + sum2.y);
    m2 = m_new;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(p_full);
  }
  if (ok && nblk > 0 && mbar_wait(pv_done, (nblk - 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) {
    tc_fence_after();
    const float inv = (l > 0.f) ? 1.f / l : 0.f;
    __nv_bfloat16* orow = p.o + ((static_cast<int64_t>(b) * p.T + qi) * p.Hq + h) * D;
#pragma unroll
    for (int cc = 0; cc < D / 32; ++cc) {
      float o[32];
      tmem_ld_32cols(tO + lane_off + cc * 32, o);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 w;
        __nv_bfloat162* hw = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) hw[e2] = __floats2bfloat162_rn(o[g * 8 + 2 * e2] * inv, o[g * 8 + 2 * e2 + 1] * inv);
        *reinterpret_cast<uint4*>(orow + cc * 32 + g * 8) = w;
      }
    }
    p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.T + qi] = (m2 + log2f(l)) * 0.69314718055994531f;
  }
}

template <int D>
__global__ void __launch_bounds__(ATT2_THREADS, 1)
    attn_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using L = Attn2Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2] per tile
  uint64_t* p_full = bars + 7;    // [2] per tile
  uint64_t* pv_done = bars + 9;   // [2] per tile
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / QB;
  const int npair = (nqb + 1) / 2;
  const int x = npair - 1 - static_cast<int>(blockIdx.x);  // heaviest pairs first
  const int qa = 2 * x, qbb = 2 * x + 1;
  const bool has_b = qbb < nqb;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int nblk_a = qa + 1, nblk_b = has_b ? qbb + 1 : 0;
  const int nblk = has_b ? nblk_b : nblk_a;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S of tile t at tmem + 128 t, O of tile t at tmem + 256 + D t (no runtime-indexed arrays)
  auto ts_of = [tmem](int t) { return tmem + static_cast<uint32_t>(t) * 128u; };
  auto to_of = [tmem](int t) { return tmem + 256u + static_cast<uint32_t>(t * D); };

  if (warp == 0) {
    if (lane == 0) {
      constexpr uint32_t TILE = L::TILE;
      mbar_arrive_expect_tx(q_full, has_b ? 2 * TILE : TILE);
#pragma unroll
      for (int c = 0; c < L::CH; ++c) {
        tma_load_4d(sQ + c * 16384, &tmQ, q_full, c * 64, h, qa * QB, b);
        if (has_b) tma_load_4d(sQ + TILE + c * 16384, &tmQ, q_full, c * 64, h, qbb * QB, b);
      }
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
#pragma unroll
        for (int c = 0; c < L::CH; ++c) {
          tma_load_4d(sK + st * TILE + c * 16384, &tmK, &kv_full[st], c * 64, hk, j * KB, b);
          tma_load_4d(sV + st * TILE + c * 16384, &tmV, &kv_full[st], c * 64, hk, j * KB, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, KB, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D, false, true);
      const uint32_t q_addr0 = smem_u32(sQ);
      // S_t(j) = Q_t K_j^T; its buffer last held P_t(j-1), consumed by P_t(j-1) V issued before
      auto issue_s = [&](int t, int j) {
        const uint32_t q_addr = q_addr0 + t * L::TILE;
        const uint32_t k_addr = smem_u32(sK + (j & 1) * L::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(ts_of(t), sdesc_kmajor(q_addr + off), sdesc_kmajor(k_addr + off), idesc_s, kk ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(&p_full[t], j & 1, p.err, ERR_MMA_FULL_TIMEOUT)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (j & 1) * L::TILE);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk)
          umma_bf16_ts(to_of(t), ts_of(t) + static_cast<uint32_t>(kk * 8), sdesc_mnmajor(v_addr + kk * 16 * 128, 16384),
                       idesc_o, (j | kk) ? 1u : 0u);
        umma_commit(&pv_done[t]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.err, ERR_MMA_FULL_TIMEOUT) &&
                mbar_wait(&kv_full[0], 0, p.err, ERR_MMA_FULL_TIMEOUT);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (has_b) issue_s(1, 0);
      }
      // K/V of block j+1 (the other stage) before the S MMAs that read it
      auto wait_kv = [&](int j1) {
        const bool r = mbar_wait(&kv_full[j1 & 1], (j1 >> 1) & 1, p.err, ERR_MMA_FULL_TIMEOUT);
        tc_fence_after();
        return r;
      };
      for (int j = 0; ok && j < nblk; ++j) {
        if (j < nblk_a) {
          if (!(ok = issue_pv(0, j))) break;
          if (j + 1 < nblk_a) {
            if (!(ok = wait_kv(j + 1))) break;
            issue_s(0, j + 1);
          }
        }
        if (j < nblk_b) {
          if (!(ok = issue_pv(1, j))) break;
          if (j + 1 < nblk_b) {
            if (!(ok = wait_kv(j + 1))) break;
            issue_s(1, j + 1);
          }
        }
        umma_commit(&kv_empty[j & 1]);  // K_j, V_j no longer read once these MMAs complete
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else {
    const int t = (warp - 2) >> 2;  // tile of this warpgroup (one call site keeps the code small)
    const int q = warp & 3;
    if (t == 0 || has_b) {
      fwd_softmax_tile_v2<D, false>(p, ts_of(t), to_of(t), s_full + t, p_full + t, pv_done + t, t ? qbb : qa,
                                    t ? nblk_b : nblk_a, h, b, q, lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
// ======================================================================================
// Forward, 3 warpgroups (384 threads) so that the softmax threads can hold a whole row of 128
// scores: WG0 = warp 0 TMA, warp 1 MMA, warps 2-3 idle, with its registers cut to 56 per thread;
// WG1 / WG2 = softmax + epilogue of query tile A / B with 224 per thread.  Launch allocation:
// 384 x 168 = 64512 registers; after the reallocation 128 x 56 + 256 x 224 = 64512, and each
// SM sub-partition holds one WG0 warp and two softmax warps: (56 + 2 x 224) x 32 = 16128 of
// its 16384.  Same barriers, TMEM layout and MMA schedule as attn_fwd2_kernel.
// ======================================================================================
constexpr int ATT3_THREADS = 384;
constexpr uint32_t ATT3_REGS_CTRL = 56, ATT3_REGS_SOFTMAX = 224, ATT3_REGS_LAUNCH = 168;
static_assert(128 * ATT3_REGS_CTRL + 256 * ATT3_REGS_SOFTMAX <= ATT3_THREADS * ATT3_REGS_LAUNCH,
              "register split exceeds the launch allocation");
static_assert((ATT3_REGS_CTRL + 2 * ATT3_REGS_SOFTMAX) * 32 <= 16384, "register split exceeds a sub-partition");

template <int D>
__global__ void __launch_bounds__(ATT3_THREADS, 1)
    attn_fwd3_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using L = Attn2Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2] per tile
  uint64_t* p_full = bars + 7;    // [2] per tile
  uint64_t* pv_done = bars + 9;   // [2] per tile
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / QB;
  const int npair = (nqb + 1) / 2;
  const int x = npair - 1 - static_cast<int>(blockIdx.x);  // heaviest pairs first
  const int qa = 2 * x, qbb = 2 * x + 1;
  const bool has_b = qbb < nqb;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int nblk_a = qa + 1, nblk_b = has_b ? qbb + 1 : 0;
  const int nblk = has_b ? nblk_b : nblk_a;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto ts_of = [tmem](int t) { return tmem + static_cast<uint32_t>(t) * 128u; };
  auto to_of = [tmem](int t) { return tmem + 256u + static_cast<uint32_t>(t * D); };

  if (warp < 4) {
    reg_dealloc<ATT3_REGS_CTRL>();  // unconditionally: the softmax warpgroups wait for these
    if (warp == 0 && lane == 0) {
      constexpr uint32_t TILE = L::TILE;
      mbar_arrive_expect_tx(q_full, has_b ? 2 * TILE : TILE);
#pragma unroll
      for (int c = 0; c < L::CH; ++c) {
        tma_load_4d(sQ + c * 16384, &tmQ, q_full, c * 64, h, qa * QB, b);
        if (has_b) tma_load_4d(sQ + TILE + c * 16384, &tmQ, q_full, c * 64, h, qbb * QB, b);
      }
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
#pragma unroll
        for (int c = 0; c < L::CH; ++c) {
          tma_load_4d(sK + st * TILE + c * 16384, &tmK, &kv_full[st], c * 64, hk, j * KB, b);
          tma_load_4d(sV + st * TILE + c * 16384, &tmV, &kv_full[st], c * 64, hk, j * KB, b);
        }
      }
    } else if (warp == 1 && lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, KB, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D, false, true);
      const uint32_t q_addr0 = smem_u32(sQ);
      auto issue_s = [&](int t, int j) {
        const uint32_t q_addr = q_addr0 + t * L::TILE;
        const uint32_t k_addr = smem_u32(sK + (j & 1) * L::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(ts_of(t), sdesc_kmajor(q_addr + off), sdesc_kmajor(k_addr + off), idesc_s, kk ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(&p_full[t], j & 1, p.err, ERR_MMA_FULL_TIMEOUT)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (j & 1) * L::TILE);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk)
          umma_bf16_ts(to_of(t), ts_of(t) + static_cast<uint32_t>(kk * 8), sdesc_mnmajor(v_addr + kk * 16 * 128, 16384),
                       idesc_o, (j | kk) ? 1u : 0u);
        umma_commit(&pv_done[t]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, p.err, ERR_MMA_FULL_TIMEOUT) &&
                mbar_wait(&kv_full[0], 0, p.err, ERR_MMA_FULL_TIMEOUT);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (has_b) issue_s(1, 0);
      }
      auto wait_kv = [&](int j1) {
        const bool r = mbar_wait(&kv_full[j1 & 1], (j1 >> 1) & 1, p.err, ERR_MMA_FULL_TIMEOUT);
        tc_fence_after();
        return r;
      };
      for (int j = 0; ok && j < nblk; ++j) {
        if (j < nblk_a) {
          if (!(ok = issue_pv(0, j))) break;
          if (j + 1 < nblk_a) {
            if (!(ok = wait_kv(j + 1))) break;
            issue_s(0, j + 1);
          }
        }
        if (j < nblk_b) {
          if (!(ok = issue_pv(1, j))) break;
          if (j + 1 < nblk_b) {
            if (!(ok = wait_kv(j + 1))) break;
            issue_s(1, j + 1);
          }
        }
        umma_commit(&kv_empty[j & 1]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else {
    reg_alloc<ATT3_REGS_SOFTMAX>();
    const int t = (warp - 4) >> 2;
    const int q = warp & 3;
    if (t == 0 || has_b)
      fwd_softmax_tile_v2<D, true>(p, ts_of(t), to_of(t), s_full + t, p_full + t, pv_done + t, t ? qbb : qa,
                                   t ? nblk_b : nblk_a, h, b, q, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
// ======================================================================================
// Backward, part 1 (dK, dV): one CTA per (128-key block j, query head, batch); loops over the
// query blocks i >= j (causal) in units of 64 queries.  K_j and V_j stay in smem; Q_i / dO_i are
// double-buffered; S^T / dP^T / dS^T are double-buffered per 64-query half, so the tensor core
// computes one half while the elementwise warps work on the other.
//   MMA      S^T = K_j Q_u^T  -> TMEM S(h)      dP^T = V_j dO_u^T -> TMEM dP(h)      (N = 64)
//   softmax  (one key row per TMEM lane) P^T = exp2(S^T*scale*log2e - lse*log2e) (causal mask
//            on the diagonal block), packed back into TMEM as bf16; dS^T = P^T * (dP^T - delta)
//            as bf16 into a swizzled smem tile
//   MMA      dV += P^T dO_u (A from TMEM)      dK += dS^T Q_u   (dO_u, Q_u read MN-major)
// dK and dV of each query head are written once at the end as fp32 and summed over the GQA
// group by gqa_reduce_kernel; no atomics.  dQ is computed by attn_bwd_dq_kernel (part 2).
// ======================================================================================
struct AttnBwdParams {
  int B, T, Hq, Hkv, D;
  float scale, scale_log2;
  const float* lse;    // [B, Hq, T]
  const float* delta;  // [B, Hq, T]
  float* dk_h;         // [B, T, Hq, D] fp32: dK of each query head (summed over the GQA group later)
  float* dv_h;         // [B, T, Hq, D] fp32
  int* err;
};

template <int D>
struct BwdSmem {
  static constexpr int CH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int Q_OFF = 2 * TILE;            // 2 buffers (prefetch of the next query block)
  static constexpr int DO_OFF = 4 * TILE;           // 2 buffers
  static constexpr int DST_OFF = 6 * TILE;          // 2 x dS^T [128 keys x 64 q] bf16 (P^T lives in TMEM)
  static constexpr int STAT_OFF = DST_OFF + 32768;  // lse*log2e [128], delta [128]
  static constexpr int BAR_OFF = STAT_OFF + 1024;
  static constexpr int BYTES0 = BAR_OFF + 256 + 1024;
  static constexpr int BYTES = BYTES0 > 120 * 1024 ? BYTES0 : 120 * 1024;
};

template <int D>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const AttnBwdParams p) {
  using L = BwdSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sDO = smem + L::DO_OFF;
  uint8_t* sDSt = smem + L::DST_OFF;  // 2 buffers of dS^T [128 keys x 64 q] (16 KB each)
  float* sLse = reinterpret_cast<float*>(smem + L::STAT_OFF);
  float* sDelta = sLse + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_empty = bars + 3;   // [2]
  uint64_t* do_full = bars + 5;   // [2]
  uint64_t* do_empty = bars + 7;  // [2]
  uint64_t* sp_full = bars + 9;   // [2] per query half
  uint64_t* ds_full = bars + 11;  // [2]
  uint64_t* ds_empty = bars + 13; // [2]
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / QB;
  const int j = blockIdx.x;  // key block (small j = most work, scheduled first)
  const int hq = blockIdx.y, b = blockIdx.z;
  const int hk = hq / (p.Hq / p.Hkv);
  const int n_iter = nqb - j;   // query blocks i = j .. nqb-1
  const int n_units = 2 * n_iter;  // each query block in two halves of 64 queries

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_full[t], 1);
      mbar_init(&q_empty[t], 1);
      mbar_init(&do_full[t], 1);
      mbar_init(&do_empty[t], 1);
      mbar_init(&sp_full[t], 1);
      mbar_init(&ds_full[t], 8);
      mbar_init(&ds_empty[t], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // S^T / dP^T of the two query halves (64 columns each), then the dV and dK accumulators
  // per-half buffers by arithmetic (a runtime-indexed array would live in local memory)
  auto ts_h = [tmem](int h) { return tmem + static_cast<uint32_t>(h) * 64u; };
  auto tdp_h = [tmem](int h) { return tmem + 128u + static_cast<uint32_t>(h) * 64u; };
  const uint32_t tDV = tmem + 256, tDK = tmem + 256 + D;
  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * L::TILE);
#pragma unroll
      for (int c = 0; c < L::CH; ++c) {
        tma_load_4d(sK + c * 16384, &tmK, kv_full, c * 64, hk, j * KB, b);
        tma_load_4d(sV + c * 16384, &tmV, kv_full, c * 64, hk, j * KB, b);
      }
      for (int n = 0; n < n_iter; ++n) {
        const int i = j + n;
        const int qs = n & 1;
        if (!mbar_wait(&q_empty[qs], ((n >> 1) & 1) ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) break;
        mbar_arrive_expect_tx(&q_full[qs], L::TILE);
#pragma unroll
        for (int c = 0; c < L::CH; ++c)
          tma_load_4d(sQ + qs * L::TILE + c * 16384, &tmQ, &q_full[qs], c * 64, hq, i * QB, b);
        if (!mbar_wait(&do_empty[qs], ((n >> 1) & 1) ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) break;
        mbar_arrive_expect_tx(&do_full[qs], L::TILE);
#pragma unroll
        for (int c = 0; c < L::CH; ++c)
          tma_load_4d(sDO + qs * L::TILE + c * 16384, &tmDO, &do_full[qs], c * 64, hq, i * QB, b);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(128, 64, false, false);  // S^T, dP^T of one query half
      constexpr uint32_t id_kv = idesc_bf16_f32(128, D, false, true);   // dV, dK (B MN-major)
      bool ok = mbar_wait(kv_full, 0, p.err, ERR_MMA_FULL_TIMEOUT);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_base = smem_u32(sQ), do_base = smem_u32(sDO);
      const uint32_t ds_base = smem_u32(sDSt);
      // S^T and dP^T of unit u = (query block n, half h) into the TMEM buffers of half h.  The
      // buffers last held unit u-2, whose P^T was consumed by its dV MMA, issued earlier by this
      // thread (tcgen05 MMAs of one thread execute in order).
      auto issue_sdp = [&](int u) -> bool {
        const int n = u >> 1, h = u & 1, qs = n & 1;
        if (h == 0 && !(mbar_wait(&q_full[qs], (n >> 1) & 1, p.err, ERR_MMA_FULL_TIMEOUT) &&
                        mbar_wait(&do_full[qs], (n >> 1) & 1, p.err, ERR_MMA_FULL_TIMEOUT)))
          return false;
        tc_fence_after();
        const uint32_t q_addr = q_base + qs * L::TILE + h * 8192;
        const uint32_t do_addr = do_base + qs * L::TILE + h * 8192;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(ts_h(h), sdesc_kmajor(k_addr + off), sdesc_kmajor(q_addr + off), id_s, kk ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tdp_h(h), sdesc_kmajor(v_addr + off), sdesc_kmajor(do_addr + off), id_s, kk ? 1u : 0u);
        }
        umma_commit(&sp_full[h]);
        return true;
      };
      ok = ok && issue_sdp(0) && issue_sdp(1);
      for (int u = 0; ok && u < n_units; ++u) {
        const int n = u >> 1, h = u & 1, qs = n & 1;
        if (!mbar_wait(&ds_full[h], (u >> 1) & 1, p.err, ERR_MMA_FULL_TIMEOUT)) break;
        tc_fence_after();
        const uint32_t q_addr = q_base + qs * L::TILE;
        const uint32_t do_addr = do_base + qs * L::TILE;
        const uint32_t ds_addr = ds_base + h * 16384;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // K = the 64 queries of this half
          const uint32_t row = static_cast<uint32_t>(h * 64 + kk * 16) * 128;
          // P^T packed by the elementwise warps: queries [32w, 32w+32) in columns [32w, 32w+16)
          const uint32_t a_tm = ts_h(h) + static_cast<uint32_t>((kk >> 1) * 32 + (kk & 1) * 8);
          umma_bf16_ts(tDV, a_tm, sdesc_mnmajor(do_addr + row, 16384), id_kv, (u | kk) ? 1u : 0u);
          umma_bf16(tDK, sdesc_kmajor(ds_addr + kk * 32), sdesc_mnmajor(q_addr + row, 16384), id_kv,
                    (u | kk) ? 1u : 0u);
        }
        umma_commit(&ds_empty[h]);
        if (h == 1) {
          umma_commit(&q_empty[qs]);
          umma_commit(&do_empty[qs]);
        }
        if (u + 2 < n_units && !issue_sdp(u + 2)) break;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // which 32 queries of a 64-query unit (and D/2 output columns)
    const int kr = q * 32 + lane;      // key row (S^T / dP^T lane)
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int tid = threadIdx.x - 64;  // 0..255
    const int c0 = half * 32;
    // Every warp waits on the same mbarriers with waits that only give up on their own timeout: a
    // phase that completed is seen complete by all of them and one that never completes times
    // out in all of them, so every elementwise warp leaves the loop at the same point and the
    // named barriers stay matched.
    bool ok = true;
    // row statistics of each query block, prefetched one block ahead (one value per thread)
    const float* stat_src = (tid < 128) ? p.lse : p.delta;
    // the statistics are kept negated (-lse*log2e, -delta) so that both enter as addends
    const float stat_mul = (tid < 128) ? -1.4426950408889634f : -1.f;
    const int64_t stat_base = (static_cast<int64_t>(b) * p.Hq + hq) * p.T + (tid & 127);
    float stat_next = stat_src[stat_base + j * QB] * stat_mul;
    for (int u = 0; u < n_units && ok; ++u) {
      const int n = u >> 1, h = u & 1;
      const int i = j + n;
      if (h == 0) {
        // publish this block's statistics (the previous block's readers are past the barrier)
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (tid < 128)
          sLse[tid] = stat_next;
        else
          sDelta[tid - 128] = stat_next;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (n + 1 < n_iter) stat_next = stat_src[stat_base + (i + 1) * QB] * stat_mul;
      }
      if (!mbar_wait(&sp_full[h], (u >> 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT, MMF_WAIT_TIMEOUT_NS, false)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = (i == j);
      float sv[32], dp[32];
      tmem_ld_32cols_async(ts_h(h) + lane_off + c0, sv);
      tmem_ld_32cols_async(tdp_h(h) + lane_off + c0, dp);
      tmem_ld_wait();
      // the dS^T buffer of this half was last read by the dK MMA of unit u-2
      if (u >= 2 && !mbar_wait(&ds_empty[h], ((u - 2) >> 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT,
                               MMF_WAIT_TIMEOUT_NS, false)) {
        ok = false;
        break;
      }
      uint8_t* dst_tile = sDSt + h * 16384;
      float ppk[16];  // P^T as bf16 pairs, reinterpreted as 32-bit TMEM words
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 wd;
        __nv_bfloat162* hd = reinterpret_cast<__nv_bfloat162*>(&wd);
        // the 8 query columns' statistics: same address in every lane (broadcast), 16-byte reads
        const int q0 = h * 64 + c0 + g * 8;
        float st_l[8], st_d[8];
        *reinterpret_cast<float4*>(st_l) = *reinterpret_cast<const float4*>(sLse + q0);
        *reinterpret_cast<float4*>(st_l + 4) = *reinterpret_cast<const float4*>(sLse + q0 + 4);
        *reinterpret_cast<float4*>(st_d) = *reinterpret_cast<const float4*>(sDelta + q0);
        *reinterpret_cast<float4*>(st_d + 4) = *reinterpret_cast<const float4*>(sDelta + q0 + 4);
        // one packed fma per pair for the exponent argument, packed add + mul for dS; the
        // causal mask only on the diagonal block
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const int e = g * 8 + e2 * 2;
          const float2 x = ffma2(make_float2(sv[e], sv[e + 1]), sc2, make_float2(st_l[e2 * 2], st_l[e2 * 2 + 1]));
          float2 pr = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          if (diag) {
            const int qc = q0 + e2 * 2;  // query column inside the block
            if (qc < kr) pr.x = 0.f;
            if (qc + 1 < kr) pr.y = 0.f;
          }
          const float2 dd =
              fmul2(pr, fadd2(make_float2(dp[e], dp[e + 1]), make_float2(st_d[e2 * 2], st_d[e2 * 2 + 1])));
          __nv_bfloat162 pb = __floats2bfloat162_rn(pr.x, pr.y);
          ppk[g * 4 + e2] = *reinterpret_cast<float*>(&pb);
          hd[e2] = __floats2bfloat162_rn(dd.x, dd.y);
        }
        *reinterpret_cast<uint4*>(dst_tile + swz_offset(kr, c0 + g * 8)) = wd;
      }
      // packed P^T over this warp's own (already consumed) S^T columns [c0, c0 + 16)
      tmem_st_16cols_async(ts_h(h) + lane_off + c0, ppk);
      tmem_st_wait();
      tc_fence_before();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[h]);
    }
    // the last dV/dK MMAs: the drain commit of the MMA thread is not visible here, so wait for the
    // final Q/dO release (committed after them)
    if (ok) ok = mbar_wait(&q_empty[(n_iter - 1) & 1], ((n_iter - 1) >> 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT,
                           MMF_WAIT_TIMEOUT_NS, false);
    // dK_j (x scale) and dV_j of this query head
    if (ok) {
      tc_fence_after();
      const int64_t row = (static_cast<int64_t>(b) * p.T + j * KB + kr) * p.Hq + hq;
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        float* dst = (which == 0 ? p.dv_h : p.dk_h) + row * D + half * (D / 2);
        const uint32_t tb = (which == 0 ? tDV : tDK) + lane_off + half * (D / 2);
        const float f = which == 0 ? 1.f : p.scale;
        float v[D / 2];
#pragma unroll
        for (int c = 0; c < D / 64; ++c) tmem_ld_32cols_async(tb + c * 32, v + c * 32);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < D / 8; ++g)
          *reinterpret_cast<float4*>(dst + g * 4) = make_float4(v[g * 4] * f, v[g * 4 + 1] * f, v[g * 4 + 2] * f, v[g * 4 + 3] * f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ======================================================================================
// dQ kernel, one CTA per (128-query block i, query head, batch); loops over key blocks j <= i:
//   MMA      S = Q_i K_j^T -> TMEM (double buffered)      dP = dO_i V_j^T -> TMEM
//   softmax  (one query row per TMEM lane, two warps per lane quarter splitting the key columns)
//            P = exp2(S*scale*log2e - lse*log2e) (causal mask on the diagonal), dS = P (dP - delta),
//            bf16 into a swizzled smem tile
//   MMA      dQ += dS K_j  (K_j read MN-major from its K-major tile)   -> TMEM, written once (bf16)
// No atomics: each CTA owns its dQ rows.  Row statistics are per thread (its query row).
// ======================================================================================
template <int D>
struct DqSmem {
  static constexpr int CH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = TILE;
  static constexpr int K_OFF = 2 * TILE;   // 2 stages
  static constexpr int V_OFF = 4 * TILE;   // 2 stages
  static constexpr int DS_OFF = 6 * TILE;  // dS [128 q x 128 keys] bf16
  static constexpr int BAR_OFF = DS_OFF + 32768;
  static constexpr int BYTES0 = BAR_OFF + 256 + 1024;
  static constexpr int BYTES = BYTES0 > 120 * 1024 ? BYTES0 : 120 * 1024;
};

struct AttnDqParams {
  int B, T, Hq, Hkv;
  float scale, scale_log2;
  const float* lse;
  const float* delta;
  __nv_bfloat16* dq;
  int* err;
};

template <int D>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const AttnDqParams p) {
  using L = DqSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sDO = smem + L::DO_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  uint8_t* sDS = smem + L::DS_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* qdo_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2] S_j (and dP_j) ready
  uint64_t* s_empty = bars + 7;   // [2] softmax done reading S buffer
  uint64_t* dp_empty = bars + 9;  // softmax done reading dP
  uint64_t* ds_full = bars + 10;  // dS written
  uint64_t* ds_empty = bars + 11; // dQ MMA done reading dS
  uint64_t* dq_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / QB;
  const int i = nqb - 1 - static_cast<int>(blockIdx.x);  // heaviest first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int nblk = i + 1;

  if (threadIdx.x == 0) {
    mbar_init(qdo_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&kv_full[t], 1);
      mbar_init(&kv_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&s_empty[t], 8);
    }
    mbar_init(dp_empty, 8);
    mbar_init(ds_full, 8);
    mbar_init(ds_empty, 1);
    mbar_init(dq_done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto tsb = [tmem](int st) { return tmem + static_cast<uint32_t>(st) * 128u; };
  const uint32_t tDP = tmem + 256, tDQ = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(qdo_full, 2 * L::TILE);
#pragma unroll
      for (int c = 0; c < L::CH; ++c) {
        tma_load_4d(sQ + c * 16384, &tmQ, qdo_full, c * 64, h, i * QB, b);
        tma_load_4d(sDO + c * 16384, &tmDO, qdo_full, c * 64, h, i * QB, b);
      }
      for (int j = 0; j < nblk; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::TILE);
#pragma unroll
        for (int c = 0; c < L::CH; ++c) {
          tma_load_4d(sK + st * L::TILE + c * 16384, &tmK, &kv_full[st], c * 64, hk, j * KB, b);
          tma_load_4d(sV + st * L::TILE + c * 16384, &tmV, &kv_full[st], c * 64, hk, j * KB, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(128, KB, false, false);
      constexpr uint32_t id_q = idesc_bf16_f32(128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO), ds_addr = smem_u32(sDS);
      // S_j and dP_j for block j; S is double-buffered, dP single (released by the softmax
      // warps as soon as they have loaded it), so S_{j+1}/dP_{j+1} overlap the softmax of j.
      auto issue_s_dp = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t k_addr = smem_u32(sK + st * L::TILE), v_addr = smem_u32(sV + st * L::TILE);
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, p.err, ERR_MMA_FULL_TIMEOUT)) return false;
        if (!mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1u, p.err, ERR_MMA_TMEM_EMPTY_TIMEOUT)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tsb(st), sdesc_kmajor(q_addr + off), sdesc_kmajor(k_addr + off), id_s, kk ? 1u : 0u);
        }
        if (!mbar_wait(dp_empty, (j & 1) ^ 1u, p.err, ERR_MMA_TMEM_EMPTY_TIMEOUT)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tDP, sdesc_kmajor(do_addr + off), sdesc_kmajor(v_addr + off), id_s, kk ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        return true;
      };
      bool ok = mbar_wait(qdo_full, 0, p.err, ERR_MMA_FULL_TIMEOUT) && issue_s_dp(0);
      for (int j = 0; ok && j < nblk; ++j) {
        const int st = j & 1;
        if (j + 1 < nblk && !issue_s_dp(j + 1)) break;
        if (!mbar_wait(ds_full, j & 1, p.err, ERR_MMA_FULL_TIMEOUT)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * L::TILE);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk) {  // K = keys
          const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tDQ, sdesc_kmajor(ds_addr + aoff), sdesc_mnmajor(k_addr + kk * 2048, 16384), id_q,
                    (j | kk) ? 1u : 0u);
        }
        umma_commit(ds_empty);
        umma_commit(&kv_empty[st]);
      }
      umma_commit(dq_done);
    }
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // which 64 key columns this warp owns
    const int r = q * 32 + lane;       // query row in the block
    const int qi = i * QB + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int64_t so = (static_cast<int64_t>(b) * p.Hq + h) * p.T + qi;
    const float lse2 = p.lse[so] * 1.4426950408889634f;
    const float dlt = p.delta[so];
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = (j == i);
      const int c0 = half * 64;
      float sv[64], dp[64];
      tmem_ld_32cols_async(tsb(st) + lane_off + c0, sv);
      tmem_ld_32cols_async(tsb(st) + lane_off + c0 + 32, sv + 32);
      tmem_ld_32cols_async(tDP + lane_off + c0, dp);
      tmem_ld_32cols_async(tDP + lane_off + c0 + 32, dp + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[st]);
        mbar_arrive(dp_empty);
      }
      // the dS buffer must have been consumed by the previous dQ MMA
      if (j >= 1 && !mbar_wait(ds_empty, (j - 1) & 1, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        uint4 w;
        __nv_bfloat162* hw = reinterpret_cast<__nv_bfloat162*>(&w);
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 nl = make_float2(-lse2, -lse2), nd = make_float2(-dlt, -dlt);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const int e = g * 8 + e2 * 2;
          const float2 x = ffma2(make_float2(sv[e], sv[e + 1]), sc2, nl);
          float2 pr = make_float2(fast_exp2(x.x), fast_exp2(x.y));
          if (diag) {
            const int key = j * KB + c0 + e;
            if (key > qi) pr.x = 0.f;
            if (key + 1 > qi) pr.y = 0.f;
          }
          const float2 dd = fmul2(pr, fadd2(make_float2(dp[e], dp[e + 1]), nd));
          hw[e2] = __floats2bfloat162_rn(dd.x, dd.y);
        }
        *reinterpret_cast<uint4*>(sDS + swz_offset(r, c0 + g * 8)) = w;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && mbar_wait(dq_done, 0, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) {
      tc_fence_after();
      __nv_bfloat16* dst = p.dq + ((static_cast<int64_t>(b) * p.T + qi) * p.Hq + h) * D + half * (D / 2);
      float v[D / 2];
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tmem_ld_32cols_async(tDQ + lane_off + half * (D / 2) + c * 32, v + c * 32);
      tmem_ld_wait();
#pragma unroll
      for (int g = 0; g < D / 16; ++g) {
        uint4 w;
        __nv_bfloat162* hw = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2)
          hw[e2] = __floats2bfloat162_rn(v[g * 8 + 2 * e2] * p.scale, v[g * 8 + 2 * e2 + 1] * p.scale);
        *reinterpret_cast<uint4*>(dst + g * 8) = w;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, t] = sum_d dO * O  (one warp per row)
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dO,
                                      float* __restrict__ delta, int B, int T, int H, int D) {
  const int64_t rows = static_cast<int64_t>(B) * T * H;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* a = o + r * D;
  const __nv_bfloat16* g = dO + r * D;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s = fmaf(__bfloat162float(a[d]), __bfloat162float(g[d]), s);
  s = warp_sum(s);
  if (lane == 0) {
    const int h = static_cast<int>(r % H);
    const int64_t bt = r / H;
    const int t = static_cast<int>(bt % T);
    const int bb = static_cast<int>(bt / T);
    delta[(static_cast<int64_t>(bb) * H + h) * T + t] = s;
  }
}

// dk[b, t, hk, d] = sum_{g < G} dk_h[b, t, hk*G + g, d] (and dv), as bf16.
__global__ void gqa_reduce_kernel(const float* __restrict__ dk_h, const float* __restrict__ dv_h,
                                  __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int64_t rows_kv, int G,
                                  int D) {
  const int64_t n = rows_kv * D;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / D;  // (b, t, hk) row
    const int d = static_cast<int>(e % D);
    const int64_t base = (r * G) * D + d;
    float a = 0.f, c = 0.f;
    for (int g = 0; g < G; ++g) {
      a += dk_h[base + static_cast<int64_t>(g) * D];
      c += dv_h[base + static_cast<int64_t>(g) * D];
    }
    dk[e] = __float2bfloat16_rn(a);
    dv[e] = __float2bfloat16_rn(c);
  }
}

// ------------------------------------ host side ------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (!fn) throw std::runtime_error("mmf: cuTensorMapEncodeTiled unavailable");
  return fn;
}

// [B, T, H, D] bf16 tensor, box {64 (D), 1 (head), 128 (T), 1}
CUtensorMap map_bthd(const void* base, int B, int T, int H, int D) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("mmf: attention tensors must be 16B aligned");
  ensure_context();
  CUtensorMap m;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(H) * D * 2,
                           static_cast<cuuint64_t>(T) * H * D * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("mmf: attention tensor map encode failed: " + std::to_string((int)r));
  return m;
}

// Forward kernel: 0 (default) = the 3-warpgroup kernel (whole score rows in registers; at the
// Llama-3-8B shape 0.1776 ms against 0.1794 ms for the 2-warpgroup kernel, 1 B200), which runs
// only when its compiled register count is the one its register split assumes, else the
// 2-warpgroup kernel; 1 = always the 2-warpgroup kernel.
std::atomic<int> g_fwd_variant{0};
// The backward's elementwise arithmetic is packed (f32x2 fma/add/mul, diagonal-only mask): the
// fastest of the versions swept at the 8B shape (0.742 ms against 0.786 / 0.762 / 0.769 ms for
// the plain, ping-pong and FMA-pipe-exponential versions, which were removed).

template <int D>
void launch_fwd(const AttnArgs& a, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  static int regs3[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaFuncSetAttribute(attn_fwd2_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Attn2Smem<D>::BYTES);
    cudaFuncSetAttribute(attn_fwd3_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Attn2Smem<D>::BYTES);
    // the register split of attn_fwd3_kernel assumes its launch allocation; an increase beyond
    // the block's pool would wait forever, so it only runs when the compiled count matches
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, attn_fwd3_kernel<D>);
    regs3[dev] = fa.numRegs;
    attr_set[dev] = true;
  }
  AttnParams p{};
  p.B = a.B;
  p.T = a.T;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.D = D;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.o = static_cast<__nv_bfloat16*>(a.o);
  p.lse = a.lse;
  p.err = device_error_word(dev);
  CUtensorMap mq = map_bthd(a.q, a.B, a.T, a.Hq, D);
  CUtensorMap mk = map_bthd(a.k, a.B, a.T, a.Hkv, D);
  CUtensorMap mv = map_bthd(a.v, a.B, a.T, a.Hkv, D);
  dim3 grid((a.T / QB + 1) / 2, a.Hq, a.B);
  if (g_fwd_variant.load() == 0 && regs3[dev] == static_cast<int>(ATT3_REGS_LAUNCH))
    attn_fwd3_kernel<D><<<grid, ATT3_THREADS, Attn2Smem<D>::BYTES, stream>>>(mq, mk, mv, p);
  else
    attn_fwd2_kernel<D><<<grid, ATT2_THREADS, Attn2Smem<D>::BYTES, stream>>>(mq, mk, mv, p);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: attention launch failed: ") + cudaGetErrorString(e));
}


template <int D>
void launch_bwd(const AttnBwdArgs& a, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdSmem<D>::BYTES);
    cudaFuncSetAttribute(attn_bwd_dq_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, DqSmem<D>::BYTES);
    attr_set[dev] = true;
  }
  const int64_t rows = static_cast<int64_t>(a.B) * a.T * a.Hq;
  attn_bwd_delta_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(a.o), static_cast<const __nv_bfloat16*>(a.dout), a.delta, a.B, a.T, a.Hq, D);
  count_launch();
  AttnBwdParams p{};
  p.B = a.B;
  p.T = a.T;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.D = D;
  p.scale = a.scale;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.lse = a.lse;
  p.delta = a.delta;
  p.dk_h = a.dk_h;
  p.dv_h = a.dv_h;
  p.err = device_error_word(dev);
  CUtensorMap mq = map_bthd(a.q, a.B, a.T, a.Hq, D);
  CUtensorMap mk = map_bthd(a.k, a.B, a.T, a.Hkv, D);
  CUtensorMap mv = map_bthd(a.v, a.B, a.T, a.Hkv, D);
  CUtensorMap mdo = map_bthd(a.dout, a.B, a.T, a.Hq, D);
  dim3 grid(a.T / KB, a.Hq, a.B);
  attn_bwd_kernel<D><<<grid, BWD_THREADS, BwdSmem<D>::BYTES, stream>>>(mq, mk, mv, mdo, p);
  count_launch();
  AttnDqParams pq{};
  pq.B = a.B;
  pq.T = a.T;
  pq.Hq = a.Hq;
  pq.Hkv = a.Hkv;
  pq.scale = a.scale;
  pq.scale_log2 = p.scale_log2;
  pq.lse = a.lse;
  pq.delta = a.delta;
  pq.dq = static_cast<__nv_bfloat16*>(a.dq);
  pq.err = p.err;
  attn_bwd_dq_kernel<D><<<dim3(a.T / QB, a.Hq, a.B), BWD_THREADS, DqSmem<D>::BYTES, stream>>>(mq, mk, mv, mdo, pq);
  count_launch();
  const int64_t rows_kv = static_cast<int64_t>(a.B) * a.T * a.Hkv;
  gqa_reduce_kernel<<<static_cast<unsigned>(std::min<int64_t>((rows_kv * D + 255) / 256, 148 * 16)), 256, 0, stream>>>(
      a.dk_h, a.dv_h, static_cast<__nv_bfloat16*>(a.dk), static_cast<__nv_bfloat16*>(a.dv), rows_kv, a.Hq / a.Hkv, D);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: attention bwd launch failed: ") + cudaGetErrorString(e));
}

}  // namespace

void attention_fwd(const AttnArgs& a, cudaStream_t stream) {
  if (a.T % QB != 0) throw std::runtime_error("mmf: attention needs T % 128 == 0");
  if (a.Hkv <= 0 || a.Hq % a.Hkv != 0) throw std::runtime_error("mmf: Hq must be a multiple of Hkv");
  if (a.D == 128)
    launch_fwd<128>(a, stream);
  else if (a.D == 64)
    launch_fwd<64>(a, stream);
  else
    throw std::runtime_error("mmf: attention supports head_dim 64 or 128");
}

}  // namespace mmf

namespace mmf {
void attention_bwd(const AttnBwdArgs& a, cudaStream_t stream) {
  if (a.T % KB != 0) throw std::runtime_error("mmf: attention needs T % 128 == 0");
  if (a.Hkv <= 0 || a.Hq % a.Hkv != 0) throw std::runtime_error("mmf: Hq must be a multiple of Hkv");
  if (a.D == 128)
    launch_bwd<128>(a, stream);
  else if (a.D == 64)
    launch_bwd<64>(a, stream);
  else
    throw std::runtime_error("mmf: attention supports head_dim 64 or 128");
}
void set_attention_fwd_variant(int v) { g_fwd_variant.store(v); }

}  // namespace mmf
