// Allocation-free variant of the RMSNorm backward kernel (see noalloc.h for who needs it).
//
// The regular path (model_kernels.cu + bindings.cpp) allocates a [blocks, cols] fp32 buffer for
// the per-block weight-gradient partials on every call.  Here those partials go to a file-scope
// static device array of MMF_NOALLOC_MAX_PARTS * MMF_NOALLOC_MAX_COLS floats (2 MiB per device).
// Host code never passes the array's name to a kernel (in host code it is only a stand-in for
// the symbol): the device address is looked up once per device with cudaGetSymbolAddress and
// that pointer is what the kernels receive.  Nothing in this file allocates device memory.
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "noalloc.h"

namespace {

static __device__ __align__(256) float g_noalloc_scratch[MMF_NOALLOC_MAX_PARTS * MMF_NOALLOC_MAX_COLS];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_mu;
thread_local std::string g_last_error;

int fail(int code, const char* what, cudaError_t e = cudaSuccess) {
  g_last_error = what;
  if (e != cudaSuccess) {
    g_last_error += ": ";
    g_last_error += cudaGetErrorString(e);
  }
  return code;
}

__device__ __forceinline__ float bfv(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// Blocks stride over rows; block b accumulates its dw partial row in registers-by-column and
// writes all `cols` entries of scratch row b (so scratch needs no clearing between calls).
__global__ void __launch_bounds__(256) rmsnorm_bwd_partials(const __nv_bfloat16* __restrict__ dy,
                                                            const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ w,
                                                            const float* __restrict__ rstd,
                                                            __nv_bfloat16* __restrict__ dx, float* __restrict__ part,
                                                            int rows, int cols) {
  __shared__ float red[33];
  constexpr int kPerThread = MMF_NOALLOC_MAX_COLS / 256;
  float acc[kPerThread];
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) acc[k] = 0.f;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int64_t off = static_cast<int64_t>(r) * cols;
    const float rs = rstd[r];
    float dot = 0.f;
    for (int c = threadIdx.x; c < cols; c += 256) dot = fmaf(bfv(dy[off + c]) * bfv(w[c]), bfv(x[off + c]), dot);
    dot = block_sum(dot, red);
    const float k3 = dot * rs * rs * rs / cols;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      const int c = threadIdx.x + 256 * k;
      if (c < cols) {
        const float g = bfv(dy[off + c]), xv = bfv(x[off + c]);
        dx[off + c] = __float2bfloat16_rn(rs * g * bfv(w[c]) - xv * k3);
        acc[k] = fmaf(g, xv * rs, acc[k]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int c = threadIdx.x + 256 * k;
    if (c < cols) part[static_cast<int64_t>(blockIdx.x) * cols + c] = acc[k];
  }
}

__global__ void colsum_to_bf16(const float* __restrict__ part, int parts, int cols, __nv_bfloat16* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += part[static_cast<int64_t>(p) * cols + c];
  out[c] = __float2bfloat16_rn(s);
}

// Once per device, with that device current: the device address of the static scratch array.
float* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return nullptr;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* mmf_noalloc_last_error(void) {
  return g_last_error.c_str();
}

extern "C" __attribute__((visibility("default"))) int mmf_rmsnorm_bwd_noalloc(const void* dy, const void* x,
                                                                             const void* w, const float* rstd, void* dx,
                                                                             void* dw, int rows, int cols,
                                                                             cudaStream_t stream) {
  if (rows < 1 || cols < 1 || cols > MMF_NOALLOC_MAX_COLS)
    return fail(1, "mmf_rmsnorm_bwd_noalloc: rows must be >= 1 and cols in [1, MMF_NOALLOC_MAX_COLS = 8192]");
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return fail(2, "mmf_rmsnorm_bwd_noalloc: cudaGetDevice failed", e);
  if (stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread) {
    // the scratch address belongs to the current device: a stream of another device cannot use it
    int sdev = -1;
    e = cudaStreamGetDevice(stream, &sdev);
    if (e != cudaSuccess) return fail(4, "mmf_rmsnorm_bwd_noalloc: cudaStreamGetDevice failed", e);
    if (sdev != cur) return fail(4, "mmf_rmsnorm_bwd_noalloc: the stream belongs to another device than the current one");
  }
  float* part = scratch_for_current_device();
  if (part == nullptr)
    return fail(2, "mmf_rmsnorm_bwd_noalloc: cudaGetSymbolAddress for the static scratch array failed");
  const int parts = rows < MMF_NOALLOC_MAX_PARTS ? rows : MMF_NOALLOC_MAX_PARTS;
  // cudaLaunchKernelEx returns the error of this launch (or a sticky error of the context),
  // not an unrelated earlier one left in the per-thread error slot
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(parts);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  e = cudaLaunchKernelEx(&cfg, rmsnorm_bwd_partials, static_cast<const __nv_bfloat16*>(dy),
                         static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w), rstd,
                         static_cast<__nv_bfloat16*>(dx), part, rows, cols);
  if (e != cudaSuccess) return fail(3, "mmf_rmsnorm_bwd_noalloc: partials kernel launch failed", e);
  cfg.gridDim = dim3((cols + 255) / 256);
  e = cudaLaunchKernelEx(&cfg, colsum_to_bf16, static_cast<const float*>(part), parts, cols,
                         static_cast<__nv_bfloat16*>(dw));
  if (e != cudaSuccess) return fail(3, "mmf_rmsnorm_bwd_noalloc: column-sum kernel launch failed", e);
  g_last_error.clear();
  return 0;
}
