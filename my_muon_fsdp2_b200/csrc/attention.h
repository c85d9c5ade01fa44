// Causal GQA flash attention on tcgen05 (see attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mmf {

struct AttnArgs {
  const void* q;  // [B, T, Hq, D] bf16
  const void* k;  // [B, T, Hkv, D] bf16
  const void* v;  // [B, T, Hkv, D] bf16
  void* o;        // [B, T, Hq, D] bf16
  float* lse;     // [B, Hq, T] fp32 (natural log)
  int B, T, Hq, Hkv, D;
  float scale;
};
void attention_fwd(const AttnArgs& a, cudaStream_t stream);
// Forward kernel choice: 0 = three warpgroups, whole score rows in registers (default; falls
// back to 1 when its compiled register count differs from the one its register split assumes),
// 1 = two softmax warpgroups over score-row halves.  Both take two query tiles per CTA.
void set_attention_fwd_variant(int v);

struct AttnBwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;  // [B, T, Hq, D] bf16
  const float* lse;  // [B, Hq, T]
  float* delta;      // [B, Hq, T] scratch
  float* dk_h;       // [B, T, Hq, D] fp32 scratch (per-query-head dK)
  float* dv_h;       // [B, T, Hq, D] fp32 scratch
  void* dq;          // [B, T, Hq, D] bf16
  void* dk;          // [B, T, Hkv, D] bf16
  void* dv;          // [B, T, Hkv, D] bf16
  int B, T, Hq, Hkv, D;
  float scale;
};
void attention_bwd(const AttnBwdArgs& a, cudaStream_t stream);

}  // namespace mmf
