// Per-row INT8 activation quantisation: the per-element steps of the
// activation kernels (kernels.cu), shared so that every variant produces the
// same codes and scales.  Every FP32 operation is an explicit IEEE
// round-to-nearest intrinsic so the compiler cannot contract or reorder
// (linear_w8a8.c:34-128).
#pragma once

#include <cstdint>

namespace htpg {

// x' = x * inverse[c] (the per-column smoothing factors), or x.
__device__ __forceinline__ float scaled_input(float x, const float *inverse, int c) {
  return inverse ? __fmul_rn(x, __ldg(inverse + c)) : x;
}
// u = x'*s + 128 (two roundings), clamped to [1,255] by integer max/min on the
// IEEE bits (linear_w8a8.c:44-49), then rounded half to even; returned as the
// signed code u-128 in [-127, 127].
__device__ __forceinline__ int quant_code(float xs, float s) {
  const float u = __fadd_rn(__fmul_rn(xs, s), 128.0f);
  int b = __float_as_int(u);
  b = max(b, 0x3f800000);
  b = min(b, 0x437f0000);
  return __float2int_rn(__int_as_float(b)) - 128;
}
__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | ((static_cast<uint32_t>(d) & 0xffu) << 24);
}
// The row's scale from max |x'| (the maximum ignores NaN: fmaxf from 0) and
// the multiplier the codes use.
__device__ __forceinline__ float row_scale_of(float amax) { return fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f); }
__device__ __forceinline__ float row_inverse_of(float scale) { return __fdiv_rn(1.0f, scale); }

}  // namespace htpg
