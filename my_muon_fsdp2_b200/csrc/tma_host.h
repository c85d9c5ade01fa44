// Host-side construction of TMA tensor maps (shared by the GEMM translation units).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace mmf {

// 3-D bf16 tensor map over a row-major [batch][outer][inner] array with a 128-byte-swizzled
// box of box_inner x box_outer elements.  Checks what cuTensorMapEncodeTiled checks (16-byte
// aligned base, strides multiples of 16 bytes) and throws std::runtime_error on failure.
// Make the current device's primary context current on this thread.  The driver's tensor-map
// encoder needs a current context; a thread that has made no CUDA runtime call yet (autograd's
// backward worker, when one of this library's ops is its first CUDA work) has none.
void ensure_context();

CUtensorMap make_map_bf16_3d(const void* base, uint64_t inner, uint64_t outer, uint64_t batch, uint32_t box_inner,
                             uint32_t box_outer);

}  // namespace mmf
