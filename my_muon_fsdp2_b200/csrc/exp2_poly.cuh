// 2^x on the FMA pipe, for spreading the exponentials of a softmax between the MUFU unit
// (ex2.approx) and the FMA units.
//
// Method: range reduction x = n + f with n = floor(x), f in [0, 1) (the Cody-Waite split for
// base 2, where it is exact), 2^f from a degree-3 polynomial, and 2^n applied by adding n to
// the exponent field.  The coefficients were fitted in this repository by Lawson-weighted least
// squares for relative error on [0, 1] (see tests/test_exp2_poly.py, which refits them); the
// maximum relative error is 7.6e-5, far below the 3.9e-3 resolution of the bf16 probabilities
// the attention kernels store.  Inputs below -125 return 0 (the masked scores are -inf), so
// that every other result is a normal number.
// Host and device share this code so that the CPU tests check the same function.
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define MMF_HD __host__ __device__ __forceinline__
#else
#define MMF_HD inline
#endif

namespace mmf {

constexpr float EXP2_POLY_C0 = 0.99992467893137f;
constexpr float EXP2_POLY_C1 = 0.69583643337042f;
constexpr float EXP2_POLY_C2 = 0.22606565398868f;
constexpr float EXP2_POLY_C3 = 0.07802255922514f;

MMF_HD float exp2_poly(float x) {
  if (x < -125.f) return 0.f;  // masked scores are -inf; results stay normal; NaN stays NaN
  const float n = floorf(x);
  const float f = x - n;
  const float p = fmaf(fmaf(fmaf(EXP2_POLY_C3, f, EXP2_POLY_C2), f, EXP2_POLY_C1), f, EXP2_POLY_C0);
  int32_t bits;
  memcpy(&bits, &p, sizeof(bits));
  bits += static_cast<int32_t>(n) * (1 << 23);
  float r;
  memcpy(&r, &bits, sizeof(r));
  return r;
}

}  // namespace mmf
