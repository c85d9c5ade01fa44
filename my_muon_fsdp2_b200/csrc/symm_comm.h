// Cross-GPU barrier over symmetric-memory signal pads (see symm_comm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mmf {
void symm_barrier(const int64_t* pad_ptrs, int rank, int ws, uint32_t epoch, int slot_base, const float* payload,
                  int n_payload, const int64_t* payload_ptrs, uint64_t timeout_ns, cudaStream_t stream);
}  // namespace mmf
