// Persistent, warp-specialised bf16 GEMM on the sm_100a 5th-generation tensor core.
//
//   warp 0      : TMA producer (one elected lane) — 4-stage smem ring, 128B-swizzled tiles
//   warp 1      : TMEM allocator + MMA issuer (one lane issues tcgen05.mma, M=128 N=256 K=16)
//   warps 2..5  : epilogue — tcgen05.ld from TMEM, fused axpby / SYRK mirror / param update
//
// The accumulator lives in TMEM (2 x 256 fp32 columns, double buffered), so the epilogue of
// tile t overlaps the main loop of tile t+1.  Every mbarrier wait is bounded (see
// tc_common.cuh); a timeout records an error code and unwinds instead of hanging.
//
// This kernel is the building block of the Newton–Schulz chain that replaces the reference's
// three torch.matmul calls per iteration (src/muon_fsdp/utils.py:96-99):
//   A = X X^T            -> symmetric mode, alpha = Frobenius scale^2 on the first iteration
//   B = c A A + b A      -> symmetric mode, beta term reads A
//   X' = B X + a X       -> B operand read MN-major straight from row-major X
// and the final iteration's epilogue applies the Muon update to the parameters directly
// (src/muon_fsdp/optimizer.py:157-170 semantics) in "output" mode.
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>
#include <stdexcept>
#include <string>

#include "kernels.h"
#include "tc_common.cuh"
#include "tma_host.h"

namespace mmf {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (!fn) throw std::runtime_error("mmf: cuTensorMapEncodeTiled is not available from the CUDA driver");
  return fn;
}

void ensure_context() {
  thread_local int ready_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) throw std::runtime_error("mmf: no CUDA device");
  if (ready_dev != dev) {
    const cudaError_t e = cudaSetDevice(dev);  // initialises and binds the primary context
    if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: cudaSetDevice failed: ") + cudaGetErrorString(e));
    ready_dev = dev;
  }
}

CUtensorMap make_map_bf16_3d(const void* base, uint64_t inner, uint64_t outer, uint64_t batch, uint32_t box_inner,
                             uint32_t box_outer) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("mmf: TMA base must be 16-byte aligned");
  ensure_context();
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {inner * 2, inner * outer * 2};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("mmf: cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  return m;
}

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;

struct GemmParams {
  int M, N, K, batch;
  int tiles_m, tiles_n, tiles_per_batch, num_tiles;
  int band;
  int symmetric;
  int mode;  // 0 workspace, 1 output
  __nv_bfloat16* D;
  const __nv_bfloat16* C;
  const float* alpha_vec;
  float alpha;
  const float* beta_vec;
  float beta;
  const int64_t* out_ptrs;
  int nseg;
  const int64_t* out_meta;
  int64_t out_ld;
  int out_f32, out_transposed, m_true, n_true;
  const float* p_scale_vec;
  float p_scale;
  const float* v_scale_vec;
  float v_scale;
  int* err;
};

__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& b, int& tm, int& tn) {
  b = t / p.tiles_per_batch;
  int r = t - b * p.tiles_per_batch;
  if (!p.symmetric) {
    // Column bands of `band` tile columns, M fastest inside a band: the CTAs running at the
    // same time share a narrow slab of the (large) B operand and all of the (small) A operand,
    // so B is read from DRAM about once instead of once per row block.
    const int span = p.band * p.tiles_m;
    const int bi = r / span;
    const int rr = r - bi * span;
    const int w = min(p.band, p.tiles_n - bi * p.band);
    tn = bi * p.band + rr % w;
    tm = rr / w;
    return;
  }
  // Symmetric output: row block i (BM rows) needs column blocks tn >= i*BM/BN = i/2.
  int i = 0;
#pragma unroll 1
  while (true) {
    const int cnt = p.tiles_n - (i >> 1);
    if (r < cnt) {
      tm = i;
      tn = (i >> 1) + r;
      return;
    }
    r -= cnt;
    ++i;
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float* v) {
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
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[q * 8 + 2 * e], v[q * 8 + 2 * e + 1]);
    d[q] = w;
  }
}

// Epilogue of one output tile for one thread: `row` is the thread's output row, `t_row` the
// TMEM address of its accumulator lane (column 0 of the tile), tn the tile column block.
// Warp-collective (tcgen05.ld): all 32 lanes of the warp must call it together.
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, int b, int row, int tn, uint32_t t_row) {
      const float alpha_b = p.alpha * (p.alpha_vec ? p.alpha_vec[b] : 1.f);
      const float beta_b = p.C ? p.beta * (p.beta_vec ? p.beta_vec[b] : 1.f) : 0.f;
      const int64_t mn = static_cast<int64_t>(p.M) * p.N;
      const __nv_bfloat16* Crow = p.C ? p.C + b * mn + static_cast<int64_t>(row) * p.N : nullptr;
      if (p.mode == 0) {
        __nv_bfloat16* Db = p.D + b * mn;
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          float v[32];
          tmem_ld_32cols(t_row + chunk * 32, v);
          const int col0 = tn * BN + chunk * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha_b;
          if (beta_b != 0.f) {
            float c[32];
            load_bf16x32(Crow + col0, c);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = fmaf(beta_b, c[i], v[i]);
          }
          if (!p.symmetric || col0 >= row) {
            store_bf16x32(Db + static_cast<int64_t>(row) * p.N + col0, v);
          } else if (col0 + 31 >= row) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i >= row) Db[static_cast<int64_t>(row) * p.N + col0 + i] = __float2bfloat16_rn(v[i]);
          }
          if (p.symmetric && col0 + 31 > row) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i > row) Db[static_cast<int64_t>(col0 + i) * p.N + row] = __float2bfloat16_rn(v[i]);
          }
        }
      } else {
        const float ps = p.p_scale * (p.p_scale_vec ? p.p_scale_vec[b] : 1.f);
        const float vs = p.v_scale * (p.v_scale_vec ? p.v_scale_vec[b] : 1.f);
        int64_t ld = p.out_ld, seg_rows = int64_t(1) << 40;
        int tr = p.out_transposed;
        if (p.out_meta) {
          ld = p.out_meta[3 * b];
          tr = static_cast<int>(p.out_meta[3 * b + 1]);
          seg_rows = p.out_meta[3 * b + 2];
        }
        const int64_t* segp = p.out_ptrs + static_cast<int64_t>(b) * p.nseg;
        const bool row_ok = row < p.m_true;
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          float v[32];
          tmem_ld_32cols(t_row + chunk * 32, v);
          const int col0 = tn * BN + chunk * 32;
          if (!row_ok || col0 >= p.n_true) continue;
          float c[32];
          if (beta_b != 0.f) load_bf16x32(Crow + col0, c);
          if (!tr && col0 + 32 <= p.n_true && (ld & 7) == 0) {
            // contiguous 32-element run of one destination row: 16-byte vector accesses
            const int seg = (p.nseg > 1) ? static_cast<int>(row / seg_rows) : 0;
            if (!MMF_DCHECK(seg < p.nseg, p.err, ERR_CHECK_BOUNDS)) continue;
            char* T = reinterpret_cast<char*>(segp[seg]);
            const int64_t idx = (static_cast<int64_t>(row) - seg * seg_rows) * ld + col0;
            float val[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              val[i] = alpha_b * v[i];
              if (beta_b != 0.f) val[i] = fmaf(beta_b, c[i], val[i]);
              val[i] *= vs;
            }
            if (p.out_f32) {
              float4* tp = reinterpret_cast<float4*>(reinterpret_cast<float*>(T) + idx);
              if ((reinterpret_cast<uintptr_t>(tp) & 15) == 0) {
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) {
                  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
                  if (ps != 0.f) o = tp[q4];
                  tp[q4] = make_float4(fmaf(ps, o.x, val[4 * q4]), fmaf(ps, o.y, val[4 * q4 + 1]),
                                       fmaf(ps, o.z, val[4 * q4 + 2]), fmaf(ps, o.w, val[4 * q4 + 3]));
                }
                continue;
              }
            } else {
              __nv_bfloat16* tp = reinterpret_cast<__nv_bfloat16*>(T) + idx;
              if ((reinterpret_cast<uintptr_t>(tp) & 15) == 0) {
                if (ps != 0.f) {
                  float o[32];
                  load_bf16x32(tp, o);
#pragma unroll
                  for (int i = 0; i < 32; ++i) val[i] = fmaf(ps, o[i], val[i]);
                }
                store_bf16x32(tp, val);
                continue;
              }
            }
          }
          // Element-wise path (transposed destination, ragged edge, unaligned rows).  Lanes are
          // consecutive rows, so with a transposed destination each element index i is one
          // contiguous 64/128-byte access across the warp.  All old values are loaded before the
          // first store: interleaving them would serialise every load behind the previous store
          // (the compiler cannot prove the destinations distinct) at full DRAM latency each.
          auto elem = [&](int i) -> char* {  // destination of element i, as a byte address base
            const int col = col0 + i;
            const int64_t r = tr ? col : row;
            const int64_t cc = tr ? row : col;
            const int seg = (p.nseg > 1) ? static_cast<int>(r / seg_rows) : 0;
#ifdef MMF_DEVICE_CHECKS
            if (!MMF_DCHECK(seg < p.nseg, p.err, ERR_CHECK_BOUNDS)) return nullptr;
#endif
            return reinterpret_cast<char*>(segp[seg]) +
                   ((r - seg * seg_rows) * ld + cc) * (p.out_f32 ? 4 : 2);
          };
          float olds[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            olds[i] = 0.f;
            if (ps != 0.f && col0 + i < p.n_true) {
              const char* a = elem(i);
#ifdef MMF_DEVICE_CHECKS
              if (a == nullptr) continue;
#endif
              olds[i] = p.out_f32 ? *reinterpret_cast<const float*>(a)
                                  : __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(a));
            }
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (col0 + i >= p.n_true) break;
            float val = alpha_b * v[i];
            if (beta_b != 0.f) val = fmaf(beta_b, c[i], val);
            const float o = fmaf(ps, olds[i], vs * val);
            char* a = elem(i);
#ifdef MMF_DEVICE_CHECKS
            if (a == nullptr) continue;
#endif
            if (p.out_f32)
              *reinterpret_cast<float*>(a) = o;
            else
              *reinterpret_cast<__nv_bfloat16*>(a) = __float2bfloat16_rn(o);
          }
        }
      }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&tfull[j], 1);
      mbar_init(&tempty[j], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int k_blocks = p.K / BK;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued = 0;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int b, tm, tn;
        tile_coords(p, t, b, tm, tn);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_3d(sA + stage * A_BYTES + c * (BK * 64 * 2), &tmA, &full[stage], tm * BM + c * 64, kb * BK,
                          b);
          } else {
            tma_load_3d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, tm * BM, b);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(sB + stage * B_BYTES + c * (BK * 64 * 2), &tmB, &full[stage], tn * BN + c * 64, kb * BK,
                          b);
          } else {
            tma_load_3d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, tn * BN, b);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Unwinding: let the loads already in flight land before the CTA can exit.
        for (int s = 0; s < STAGES && s < issued; ++s) {
          int st = (stage + STAGES - 1 - s) % STAGES;
          uint32_t ph = (st < stage) ? phase : (phase ^ 1u);
          mbar_wait(&full[st], ph, p.err, ERR_TMA_EMPTY_TIMEOUT, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ---------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err, ERR_MMA_TMEM_EMPTY_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, ERR_MMA_FULL_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_mnmajor(a_addr + kk * 16 * 128, BK * 64 * 2) : sdesc_kmajor(a_addr + kk * 32);
            const uint64_t bd = B_MN ? sdesc_mnmajor(b_addr + kk * 16 * 128, BK * 64 * 2) : sdesc_kmajor(b_addr + kk * 32);
            umma_bf16(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: make sure every issued MMA finished before TMEM can be released.
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else {
    // ------------------------------ epilogue -----------------------------------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int b, tm, tn;
      tile_coords(p, t, b, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) break;
      tc_fence_after();
      epilogue_tile(p, b, tm * BM + q * 32 + lane, tn, tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ======================================================================================
// CTA-pair variant (cta_group::2): a cluster of 2 CTAs computes a 256 x 256 tile; each CTA
// stages its 128 rows of A and its 128-column half of B (6-stage ring, 32 KB/stage), the
// leader CTA (rank 0) issues M=256 N=256 K=16 MMAs that read both CTAs' smem, and each CTA's
// epilogue drains its own 128 TMEM lanes.  Halves the per-SM B traffic of the 1-CTA kernel.
//   full[s]  : leader only; both CTAs' TMA bytes land on it (leader arms 64 KB)
//   empty[s] : both CTAs; the leader's commit arrives on both (multicast commit)
//   tfull[j] : both CTAs; multicast commit after the tile's last MMA
//   tempty[j]: leader only, count 8 (4 epilogue warps x 2 CTAs; CTA 1 arrives remotely)
// ======================================================================================
constexpr int P_BM = 256;           // rows per CTA pair
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = 128 * BK * 2;   // 16 KB per CTA
constexpr int P_B_BYTES = 128 * BK * 2;   // 16 KB per CTA (half of N = 256)
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;

__device__ __forceinline__ void tile_coords_pair(const GemmParams& p, int t, int& b, int& tm, int& tn) {
  b = t / p.tiles_per_batch;
  int r = t - b * p.tiles_per_batch;
  if (!p.symmetric) {
    const int span = p.band * p.tiles_m;
    const int bi = r / span;
    const int rr = r - bi * span;
    const int w = min(p.band, p.tiles_n - bi * p.band);
    tn = bi * p.band + rr % w;
    tm = rr / w;
    return;
  }
  // square 256 x 256 tiles: row block i needs column blocks tn >= i
  int i = 0;
#pragma unroll 1
  while (true) {
    const int cnt = p.tiles_n - i;
    if (r < cnt) {
      tm = i;
      tn = i + r;
      return;
    }
    r -= cnt;
    ++i;
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + P_STAGES * P_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + P_STAGES * P_B_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
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
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrive / TMA signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int k_blocks = p.K / BK;

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) -------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < p.num_tiles && ok; t += nclusters) {
        int b, tm, tn;
        tile_coords_pair(p, t, b, tm, tn);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.err, ERR_TMA_EMPTY_TIMEOUT)) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE_BYTES);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
              tma_load_3d_pair(sA + stage * P_A_BYTES + c * (BK * 64 * 2), &tmA, fb, tm * P_BM + rank * 128 + c * 64,
                               kb * BK, b);
          } else {
            tma_load_3d_pair(sA + stage * P_A_BYTES, &tmA, fb, kb * BK, tm * P_BM + rank * 128, b);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < 2; ++c)
              tma_load_3d_pair(sB + stage * P_B_BYTES + c * (BK * 64 * 2), &tmB, fb, tn * BN + rank * 128 + c * 64,
                               kb * BK, b);
          } else {
            tma_load_3d_pair(sB + stage * P_B_BYTES, &tmB, fb, kb * BK, tn * BN + rank * 128, b);
          }
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer (leader CTA only) ---------------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(P_BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster; t < p.num_tiles && ok; t += nclusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.err, ERR_MMA_TMEM_EMPTY_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, ERR_MMA_FULL_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * P_A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * P_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_mnmajor(a_addr + kk * 16 * 128, BK * 64 * 2) : sdesc_kmajor(a_addr + kk * 32);
            const uint64_t bd = B_MN ? sdesc_mnmajor(b_addr + kk * 16 * 128, BK * 64 * 2) : sdesc_kmajor(b_addr + kk * 32);
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb | kk) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == P_STAGES) {
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
      mbar_wait(drain, 0, p.err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else {
    // ------------------------------ epilogue (both CTAs) -----------------------------
    const int q = warp & 3;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < p.num_tiles; t += nclusters) {
      int b, tm, tn;
      tile_coords_pair(p, t, b, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, p.err, ERR_EPI_TMEM_FULL_TIMEOUT)) break;
      tc_fence_after();
      epilogue_tile(p, b, tm * P_BM + static_cast<int>(rank) * 128 + q * 32 + lane, tn,
                    tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16));
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
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ======================================================================================
// FSDP all-gather fused with the consuming GEMM (Y = X W^T, W row-sharded over the ranks).
//   warp 0      : TMA producer; B tiles are two 128-row panels, each read from this rank's
//                 shard (own panels), from the local gather buffer G (remote panels already
//                 pulled) or, if a panel is not complete within wait_ns, from its owner directly
//   warp 1      : MMA issuer (as tc_gemm_kernel)
//   warps 2..5  : epilogue (bf16 Y)
//   warp 6      : puller: 128x64 pieces of every shard, peer -> smem (TMA load) -> G (TMA
//                 store); per-panel counters published with release semantics
// Output columns are visited starting at this rank's own shard, then ring order, which is
// also the order in which the pullers fetch: the NVLink transfer of shard r+s overlaps the
// tensor-core work on shards r .. r+s-1.  No CTA ever waits without a bound, so the kernel
// cannot deadlock even if some CTAs are not co-resident.  No multicast loads.
// ======================================================================================
constexpr int AG_MAX_WS = 8;
constexpr int AG_PANEL = 128;
constexpr int AG_PIECE_BYTES = AG_PANEL * BK * 2;  // 16 KB
constexpr int AG_THREADS = 224;
constexpr int AG_SMEM_BYTES = STAGES * STAGE_BYTES + 2 * AG_PIECE_BYTES + 1024 + 256;

struct AgMaps {
  CUtensorMap shard[AG_MAX_WS];
};

struct AgParams {
  GemmParams g;  // M, N, K, tiling, epilogue (mode 0, D = Y)
  int rot;       // tile-column rotation that puts this rank's shard first
  int rank, ws, rows_per_shard, pps, ppp;
  uint32_t* ready;
  uint64_t wait_ns;
};

__device__ __forceinline__ void ag_tile(const AgParams& p, int t, int& tm, int& tn) {
  int b;
  tile_coords(p.g, t, b, tm, tn);
  tn += p.rot;
  if (tn >= p.g.tiles_n) tn -= p.g.tiles_n;
}

__global__ void __launch_bounds__(AG_THREADS, 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmG,
                   const __grid_constant__ AgMaps maps, const AgParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sP = sB + STAGES * B_BYTES;  // 2 pull buffers
  uint64_t* full = reinterpret_cast<uint64_t*>(sP + 2 * AG_PIECE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* pfull = drain + 1;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pfull + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = p.g.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&tfull[j], 1);
      mbar_init(&tempty[j], 4);
      mbar_init(&pfull[j], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmG);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int k_blocks = p.g.K / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int issued = 0;
      for (int t = blockIdx.x; t < p.g.num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        ag_tile(p, t, tm, tn);
        // source of each 128-row half of the B tile: -1 = local G, else a shard map index
        int src[2], row[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int panel = 2 * tn + h;
          const int owner = panel / p.pps;
          const int lrow = (panel - owner * p.pps) * AG_PANEL;
          if (!MMF_DCHECK(owner >= 0 && owner < p.ws && owner < 8, err, ERR_CHECK_BOUNDS)) ok = false;
          src[h] = owner;
          row[h] = lrow;
          if (owner != p.rank) {
            const uint32_t* flag = p.ready + panel;
            bool ready = ld_acquire_gpu(flag) >= static_cast<uint32_t>(p.ppp);
            if (!ready) {
              const uint64_t t0 = globaltimer_ns();
              while (!(ready = ld_acquire_gpu(flag) >= static_cast<uint32_t>(p.ppp))) {
                if (globaltimer_ns() - t0 > p.wait_ns) break;  // fall back to the owner's memory
                __nanosleep(64);
              }
            }
            if (ready) {
              fence_proxy_async_global();
              src[h] = -1;
              row[h] = panel * AG_PANEL;
            }
          }
        }
#ifdef MMF_DEVICE_CHECKS
        if (!ok) break;
#endif
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err, ERR_TMA_EMPTY_TIMEOUT)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          tma_load_3d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, tm * BM, 0);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const CUtensorMap* m = src[h] < 0 ? &tmG : &maps.shard[src[h]];
            tma_load_3d(sB + stage * B_BYTES + h * AG_PIECE_BYTES, m, &full[stage], kb * BK, row[h], 0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES && s < issued; ++s) {
          int st = (stage + STAGES - 1 - s) % STAGES;
          uint32_t ph = (st < stage) ? phase : (phase ^ 1u);
          mbar_wait(&full[st], ph, err, ERR_TMA_EMPTY_TIMEOUT, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.g.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, ERR_MMA_TMEM_EMPTY_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, ERR_MMA_FULL_TIMEOUT)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16(d_tmem, sdesc_kmajor(a_addr + kk * 32), sdesc_kmajor(b_addr + kk * 32), idesc,
                      (kb | kk) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, err, ERR_MMA_FULL_TIMEOUT, 200000000ull);
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.g.num_tiles; t += gridDim.x) {
      int tm, tn;
      ag_tile(p, t, tm, tn);
      if (!mbar_wait(&tfull[acc], acc_phase, err, ERR_EPI_TMEM_FULL_TIMEOUT)) break;
      tc_fence_after();
      epilogue_tile(p.g, 0, tm * BM + q * 32 + lane, tn,
                    tmem_base + static_cast<uint32_t>(acc * BN) + (static_cast<uint32_t>(q * 32) << 16));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  } else {
    // ------------------------------ puller -------------------------------------------
    if (lane == 0) {
      const int per_shard = p.pps * p.ppp;
      const int total = p.ws * per_shard;
      int i = 0, prev_panel = -1;
      for (int gi = blockIdx.x; gi < total; gi += gridDim.x, ++i) {
        const int step = gi / per_shard;  // 0 -> shard rank+1, ..., ws-1 -> own shard
        int src = p.rank + 1 + step;
        src -= (src >= p.ws) ? p.ws : 0;
        src -= (src >= p.ws) ? p.ws : 0;
        const int rem = gi - step * per_shard;
        const int lp = rem / p.ppp;
        const int kb = rem - lp * p.ppp;
        const int buf = i & 1;
        uint8_t* dst = sP + buf * AG_PIECE_BYTES;
        if (!MMF_DCHECK(src >= 0 && src < p.ws && src < 8, err, ERR_CHECK_BOUNDS)) break;
        mbar_arrive_expect_tx(&pfull[buf], AG_PIECE_BYTES);
        tma_load_3d(dst, &maps.shard[src], &pfull[buf], kb * BK, lp * AG_PANEL, 0);
        if (!mbar_wait(&pfull[buf], (i >> 1) & 1, err, ERR_TMA_EMPTY_TIMEOUT)) break;
        tma_store_3d(&tmG, dst, kb * BK, src * p.rows_per_shard + lp * AG_PANEL, 0);
        bulk_commit_group();
        bulk_wait_group<1>();  // every store but the newest has completed
        if (prev_panel >= 0) {
          fence_proxy_async_global();
          red_release_gpu_add(p.ready + prev_panel, 1u);
        }
        prev_panel = src * p.pps + lp;
      }
      bulk_wait_group<0>();
      if (prev_panel >= 0) {
        fence_proxy_async_global();
        red_release_gpu_add(p.ready + prev_panel, 1u);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------ host side ------------------------------------------
struct DeviceInfo {
  int sms = 0;
  bool attr_set[12] = {};
};
DeviceInfo& dev_info(int dev) {
  static DeviceInfo infos[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  DeviceInfo& d = infos[dev];
  if (d.sms == 0) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  return d;
}

void check_shape(int batch, int M, int N, int K) {
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) throw std::runtime_error("mmf: empty GEMM");
  if (M % BM || N % BN || K % BK)
    throw std::runtime_error("mmf: tc_gemm needs M%128==0, N%256==0, K%64==0 (got M=" + std::to_string(M) +
                             " N=" + std::to_string(N) + " K=" + std::to_string(K) + ")");
}

std::atomic<int> g_variant{0};  // 0 auto, 1 single-CTA, 2 CTA pair

int pair_tiles(const GemmParams& p) {
  const int tm = p.M / P_BM, tn = p.N / BN;
  return (p.symmetric ? tm * (tm + 1) / 2 : tm * tn) * p.batch;
}

void launch(GemmParams& p, const void* A, const void* B, bool b_mn, cudaStream_t stream, bool a_mn = false) {
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo& di = dev_info(dev);
  p.err = device_error_word(dev);
  int variant = g_variant.load();
  if (variant == 0) {
    // the CTA pair needs 256-row blocks and enough tiles to keep most SMs busy
    variant = (p.M % P_BM == 0 && pair_tiles(p) >= di.sms / 2) ? 2 : 1;
  }
  if (variant == 2 && p.M % P_BM != 0) variant = 1;
  const bool pair = variant == 2;
  const int bm = pair ? P_BM : BM;
  p.tiles_m = p.M / bm;
  p.tiles_n = p.N / BN;
  if (p.symmetric) {
    if (p.M != p.N) throw std::runtime_error("mmf: symmetric GEMM needs M == N");
    int cnt = 0;
    for (int i = 0; i < p.tiles_m; ++i) cnt += pair ? (p.tiles_n - i) : (p.tiles_n - (i >> 1));
    p.tiles_per_batch = cnt;
  } else {
    p.tiles_per_batch = p.tiles_m * p.tiles_n;
  }
  p.num_tiles = p.tiles_per_batch * p.batch;
  {
    const int units = di.sms;  // concurrently running tiles
    int band = (units + p.tiles_m - 1) / p.tiles_m;
    p.band = band < 1 ? 1 : (band > p.tiles_n ? p.tiles_n : band);
  }
  const int a_rows = pair ? 128 : BM;
  const int b_rows = pair ? 128 : BN;
  CUtensorMap ma = a_mn ? make_map_bf16_3d(A, p.M, p.K, p.batch, 64, BK) : make_map_bf16_3d(A, p.K, p.M, p.batch, BK, a_rows);
  CUtensorMap mb = b_mn ? make_map_bf16_3d(B, p.N, p.K, p.batch, 64, BK) : make_map_bf16_3d(B, p.K, p.N, p.batch, BK, b_rows);
  if (!pair) {
    const int grid = p.num_tiles < di.sms ? p.num_tiles : di.sms;
    auto go = [&](auto kern, int slot) {
      if (!di.attr_set[slot]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        di.attr_set[slot] = true;
      }
      kern<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ma, mb, p);
    };
    if (a_mn) {
      if (b_mn) go(tc_gemm_kernel<true, true>, 4);
      else go(tc_gemm_kernel<true, false>, 5);
    } else if (b_mn) {
      go(tc_gemm_kernel<false, true>, 1);
    } else {
      go(tc_gemm_kernel<false, false>, 0);
    }
  } else {
    const int clusters = p.num_tiles < di.sms / 2 ? p.num_tiles : di.sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le;
    auto go = [&](auto kern, int slot) {
      if (!di.attr_set[slot]) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
        di.attr_set[slot] = true;
      }
      return cudaLaunchKernelEx(&cfg, kern, ma, mb, p);
    };
    if (a_mn)
      le = b_mn ? go(tc_gemm_pair_kernel<true, true>, 7) : go(tc_gemm_pair_kernel<true, false>, 8);
    else
      le = b_mn ? go(tc_gemm_pair_kernel<false, true>, 3) : go(tc_gemm_pair_kernel<false, false>, 2);
    if (le != cudaSuccess) throw std::runtime_error(std::string("mmf: tc_gemm pair launch failed: ") + cudaGetErrorString(le));
  }
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: tc_gemm launch failed: ") + cudaGetErrorString(e));
}

}  // namespace

// ------------------------------- error word / counters -----------------------------------
__device__ int g_mmf_error_word;

int* device_error_word(int device) {
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (!ptrs[device]) {
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != device) cudaSetDevice(device);
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mmf_error_word);
    if (cur != device) cudaSetDevice(cur);
    if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    ptrs[device] = static_cast<int*>(p);
  }
  return ptrs[device];
}

int read_and_clear_device_error(int device, cudaStream_t stream) {
  int* p = device_error_word(device);
  int v = 0;
  cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, stream);
  cudaStreamSynchronize(stream);
  if (v != 0) {
    cudaMemsetAsync(p, 0, sizeof(int), stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

static std::atomic<uint64_t> g_launches{0};
uint64_t launch_count() { return g_launches.load(); }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_gemm_variant(int v) { g_variant.store(v); }
int gemm_variant() { return g_variant.load(); }

void tc_gemm_ws(const GemmWsArgs& a, cudaStream_t stream) {
  check_shape(a.batch, a.M, a.N, a.K);
  GemmParams p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.batch = a.batch;
  p.symmetric = a.symmetric ? 1 : 0;
  p.mode = 0;
  p.D = static_cast<__nv_bfloat16*>(a.D);
  p.C = static_cast<const __nv_bfloat16*>(a.C);
  p.alpha_vec = a.alpha_vec;
  p.alpha = a.alpha;
  p.beta_vec = a.beta_vec;
  p.beta = a.beta;
  if ((reinterpret_cast<uintptr_t>(a.D) & 15) || (a.C && (reinterpret_cast<uintptr_t>(a.C) & 15)))
    throw std::runtime_error("mmf: D/C must be 16-byte aligned");
  launch(p, a.A, a.B, a.b_mn_major, stream);
}

void tc_gemm_out(const GemmOutArgs& a, cudaStream_t stream) {
  check_shape(a.batch, a.M, a.N, a.K);
  if (a.m_true > a.M || a.n_true > a.N) throw std::runtime_error("mmf: true extent exceeds padded GEMM extent");
  GemmParams p{};
  p.M = a.M;
  p.N = a.N;
  p.K = a.K;
  p.batch = a.batch;
  p.symmetric = 0;
  p.mode = 1;
  p.C = static_cast<const __nv_bfloat16*>(a.C);
  p.alpha_vec = a.alpha_vec;
  p.alpha = a.alpha;
  p.beta_vec = a.beta_vec;
  p.beta = a.beta;
  p.out_ptrs = a.out_ptrs;
  p.nseg = a.nseg < 1 ? 1 : a.nseg;
  p.out_meta = a.out_meta;
  p.out_ld = a.out_ld;
  p.out_f32 = a.out_f32 ? 1 : 0;
  p.out_transposed = a.out_transposed ? 1 : 0;
  p.m_true = a.m_true;
  p.n_true = a.n_true;
  p.p_scale_vec = a.p_scale_vec;
  p.p_scale = a.p_scale;
  p.v_scale_vec = a.v_scale_vec;
  p.v_scale = a.v_scale;
  launch(p, a.A, a.B, a.b_mn_major, stream, a.a_mn_major);
}

void ag_gemm(const AgGemmArgs& a, cudaStream_t stream) {
  if (a.ws < 1 || a.ws > AG_MAX_WS || a.rank < 0 || a.rank >= a.ws) throw std::runtime_error("mmf: ag_gemm: bad rank/world");
  check_shape(1, a.M, a.N, a.K);
  if (a.N % (AG_PANEL * a.ws) != 0)
    throw std::runtime_error("mmf: ag_gemm needs (N / world) % 128 == 0 (N=" + std::to_string(a.N) + ")");
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo& di = dev_info(dev);
  AgParams p{};
  GemmParams& g = p.g;
  g.M = a.M;
  g.N = a.N;
  g.K = a.K;
  g.batch = 1;
  g.mode = 0;
  g.symmetric = 0;
  g.D = static_cast<__nv_bfloat16*>(a.Y);
  g.C = nullptr;
  g.alpha = 1.f;
  g.beta = 0.f;
  g.err = device_error_word(dev);
  g.tiles_m = a.M / BM;
  g.tiles_n = a.N / BN;
  g.tiles_per_batch = g.tiles_m * g.tiles_n;
  g.num_tiles = g.tiles_per_batch;
  const int units = di.sms;  // concurrently running tiles
  const int band = (units + g.tiles_m - 1) / g.tiles_m;
  g.band = band < 1 ? 1 : (band > g.tiles_n ? g.tiles_n : band);
  p.rank = a.rank;
  p.ws = a.ws;
  p.rows_per_shard = a.N / a.ws;
  p.pps = p.rows_per_shard / AG_PANEL;
  p.ppp = a.K / BK;
  p.rot = (a.rank * p.rows_per_shard) / BN;
  p.ready = a.ready;
  p.wait_ns = a.wait_ns;
  if ((reinterpret_cast<uintptr_t>(a.Y) & 15) || (reinterpret_cast<uintptr_t>(a.G) & 15))
    throw std::runtime_error("mmf: ag_gemm: Y/G must be 16-byte aligned");
  AgMaps maps;
  for (int s = 0; s < AG_MAX_WS; ++s) {
    const void* base = reinterpret_cast<const void*>(a.shard_ptrs[s < a.ws ? s : a.rank]);
    maps.shard[s] = make_map_bf16_3d(base, a.K, p.rows_per_shard, 1, BK, AG_PANEL);
  }
  CUtensorMap ma = make_map_bf16_3d(a.X, a.K, a.M, 1, BK, BM);
  CUtensorMap mg = make_map_bf16_3d(a.G, a.K, a.N, 1, BK, AG_PANEL);
  cudaMemsetAsync(a.ready, 0, sizeof(uint32_t) * (a.N / AG_PANEL), stream);
  if (!di.attr_set[6]) {
    cudaFuncSetAttribute(ag_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AG_SMEM_BYTES);
    di.attr_set[6] = true;
  }
  const int grid = g.num_tiles < di.sms ? g.num_tiles : di.sms;
  ag_gemm_kernel<<<grid, AG_THREADS, AG_SMEM_BYTES, stream>>>(ma, mg, maps, p);
  cudaError_t e = cudaSuccess;
  count_launch();
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: ag_gemm launch failed: ") + cudaGetErrorString(e));
}

}  // namespace mmf
