// Cross-GPU signalling over NVLink peer memory (buffers from PyTorch symmetric memory).
//
// symm_barrier: every rank writes `epoch` into slot [slot_base + my_rank] of every peer's
// signal pad (release, system scope) and then waits until all ws slots of its own pad reach
// `epoch` (acquire, system scope).  Optionally, before signalling, it copies a small fp32
// payload (the per-matrix partial sums of squares of the Muon step) into row `my_rank` of
// every peer's payload buffer, so that after the barrier each rank holds all ranks' rows.
//
// Waits are bounded: after MMF_WAIT_TIMEOUT_NS the kernel records ERR_PEER_FLAG_TIMEOUT in
// the error word and returns (no trap, no hang); the host raises on the next check.
// Plain loads/stores only; no multimem and no TMA here.
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "kernels.h"
#include "symm_comm.h"
#include "tc_common.cuh"

namespace mmf {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void symm_barrier_kernel(const int64_t* __restrict__ pad_ptrs, int rank, int ws, uint32_t epoch,
                                    int slot_base, const float* __restrict__ payload, int n_payload,
                                    const int64_t* __restrict__ payload_ptrs, int* err, uint64_t timeout_ns) {
  // 1. payload rows into every peer (all threads cooperate), then make them visible system-wide
  if (payload != nullptr && n_payload > 0) {
    for (int64_t e = threadIdx.x; e < static_cast<int64_t>(ws) * n_payload; e += blockDim.x) {
      const int peer = static_cast<int>(e / n_payload);
      const int i = static_cast<int>(e % n_payload);
      float* dst = reinterpret_cast<float*>(payload_ptrs[peer]);
      dst[static_cast<int64_t>(rank) * n_payload + i] = payload[i];
    }
  }
  __threadfence_system();
  __syncthreads();
  // 2. signal every peer
  for (int peer = threadIdx.x; peer < ws; peer += blockDim.x) {
    uint32_t* pad = reinterpret_cast<uint32_t*>(pad_ptrs[peer]);
    st_release_sys(pad + slot_base + rank, epoch);
  }
  // 3. wait for every peer's signal in my own pad (bounded)
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(pad_ptrs[rank]);
  for (int peer = threadIdx.x; peer < ws; peer += blockDim.x) {
    const uint32_t* slot = mine + slot_base + peer;
    if (static_cast<int32_t>(ld_acquire_sys(slot) - epoch) >= 0) continue;
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int32_t>(ld_acquire_sys(slot) - epoch) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicCAS(err, 0, ERR_PEER_FLAG_TIMEOUT);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
}

// out = bf16((acc ? out : 0) + scale * sum_s slots[s]) in fp32, ranks in order (deterministic);
// 8 bf16 per thread when n % 8 == 0 and the bases are 16-byte aligned.
template <bool VEC>
__global__ void rs_reduce_kernel(const __nv_bfloat16* __restrict__ slots, int ws, int64_t stride_s, int64_t n,
                                 __nv_bfloat16* __restrict__ out, int accumulate, float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (VEC) {
    const int64_t nv = n / 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
      float acc[8], base[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = base[e] = 0.f;
      if (accumulate) {
        const uint4 w = reinterpret_cast<const uint4*>(out)[i];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          base[2 * e] = f.x;
          base[2 * e + 1] = f.y;
        }
      }
      for (int s = 0; s < ws; ++s) {
        const uint4 w = reinterpret_cast<const uint4*>(slots + static_cast<int64_t>(s) * stride_s)[i];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) oh[e] = __floats2bfloat162_rn(base[2 * e] + scale * acc[2 * e], base[2 * e + 1] + scale * acc[2 * e + 1]);
      reinterpret_cast<uint4*>(out)[i] = o;
    }
  } else {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
      float acc = 0.f;
      for (int s = 0; s < ws; ++s) acc += __bfloat162float(slots[static_cast<int64_t>(s) * stride_s + i]);
      out[i] = __float2bfloat16_rn((accumulate ? __bfloat162float(out[i]) : 0.f) + scale * acc);
    }
  }
}

// out[i] = bf16((acc ? out[i] : 0) + scale * sum_s src_s[offset + i]) with src_s = srcs[s] (one
// pointer per rank, P2P-mapped for peers), fp32 sum in rank order.  8 bf16 per thread (16-byte
// loads over NVLink).
__global__ void rs_pull_reduce_kernel(const int64_t* __restrict__ srcs, int ws, int64_t offset, int64_t n,
                                      __nv_bfloat16* __restrict__ out, int accumulate, float scale) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t nv = n / 8;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    for (int s = 0; s < ws; ++s) {
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(srcs[s]) + offset;
      const uint4 w = reinterpret_cast<const uint4*>(src)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    float base[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) base[e] = 0.f;
    if (accumulate) {
      const uint4 w = reinterpret_cast<const uint4*>(out)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        base[2 * e] = f.x;
        base[2 * e + 1] = f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      oh[e] = __floats2bfloat162_rn(base[2 * e] + scale * acc[2 * e], base[2 * e + 1] + scale * acc[2 * e + 1]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

}  // namespace

void symm_barrier(const int64_t* pad_ptrs, int rank, int ws, uint32_t epoch, int slot_base, const float* payload,
                  int n_payload, const int64_t* payload_ptrs, uint64_t timeout_ns, cudaStream_t stream) {
  if (ws < 1 || rank < 0 || rank >= ws) throw std::runtime_error("mmf: bad rank/world for symm_barrier");
  int dev = 0;
  cudaGetDevice(&dev);
  symm_barrier_kernel<<<1, 256, 0, stream>>>(pad_ptrs, rank, ws, epoch, slot_base, payload, n_payload, payload_ptrs,
                                             device_error_word(dev), timeout_ns);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: symm_barrier launch failed: ") + cudaGetErrorString(e));
}

void rs_reduce(const void* slots, int ws, int64_t slot_stride, int64_t n, void* out, bool accumulate, float scale,
               cudaStream_t stream) {
  if (ws < 1 || n < 0) throw std::runtime_error("mmf: rs_reduce: bad arguments");
  if (n == 0) return;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const bool vec = (n % 8 == 0) && (slot_stride % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(slots) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const int64_t work = vec ? n / 8 : n;
  const int64_t want = (work + 255) / 256;
  const unsigned grid = static_cast<unsigned>(want < sms * 8 ? (want < 1 ? 1 : want) : sms * 8);
  if (vec)
    rs_reduce_kernel<true><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(slots), ws, slot_stride, n,
                                                     static_cast<__nv_bfloat16*>(out), accumulate ? 1 : 0, scale);
  else
    rs_reduce_kernel<false><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(slots), ws, slot_stride, n,
                                                      static_cast<__nv_bfloat16*>(out), accumulate ? 1 : 0, scale);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: rs_reduce launch failed: ") + cudaGetErrorString(e));
}

void rs_pull_reduce(const int64_t* srcs, int ws, int64_t offset, int64_t n, void* out, bool accumulate, float scale,
                    cudaStream_t stream) {
  if (ws < 1 || n < 0 || offset < 0) throw std::runtime_error("mmf: rs_pull_reduce: bad arguments");
  if (n % 8 != 0 || offset % 8 != 0 || (reinterpret_cast<uintptr_t>(out) & 15) != 0)
    throw std::runtime_error("mmf: rs_pull_reduce needs n % 8 == 0, offset % 8 == 0 and a 16-byte aligned output");
  if (n == 0) return;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n / 8 + 255) / 256;
  // a few blocks per SM: enough loads in flight over NVLink while the compute stream keeps running
  const unsigned grid = static_cast<unsigned>(want < sms * 2 ? (want < 1 ? 1 : want) : sms * 2);
  rs_pull_reduce_kernel<<<grid, 256, 0, stream>>>(srcs, ws, offset, n, static_cast<__nv_bfloat16*>(out),
                                                  accumulate ? 1 : 0, scale);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("mmf: rs_pull_reduce launch failed: ") + cudaGetErrorString(e));
}

}  // namespace mmf
