// Per-element epilogue shared by the GEMM kernels (kernels.cu) and the
// register-fed decode kernel (decode.cu): one INT32 / FP32 accumulator ->
// output value, and the plane-export byte placement.  Keeping one
// definition makes every kernel of a shape produce identical bits.
#pragma once

#include "kernels.h"
#include "ptx.cuh"

namespace htpg {

// Optional epilogue activation (mat_mul.c:788-826): GELU(tanh) as
// x*sigmoid(z), z = 1.5957691216057308*(x + 0.044715 x^3), QuickGELU as
// x*sigmoid(1.702 x).  x*sigmoid(z) is evaluated as 0.5x*(1 + tanh(z/2)) with
// the hardware tanh (one MUFU operation instead of a 2^x and a reciprocal; the
// epilogue, not the tensor pipe, bounds short-K layers).  The tanh's relative
// error of about 2^-11 becomes an absolute error below 2.5e-4*|x| in the
// output, largest where 1 + tanh cancels (z near -6); against the tensor's
// absolute maximum that stays far inside the 2e-3 / 1e-2 output tolerances.
// Saturation is exact: tanh = -1 gives 0, tanh = 1 gives x.  MODE is a
// template parameter so the per-element code is branch-free and the 32
// elements of a chunk interleave.
template <int MODE>
__device__ __forceinline__ float epilogue_act(float x) {
  if constexpr (MODE != 1 && MODE != 2) {
    return x;
  } else {
    // x * sigmoid(z) = 0.5x * (1 + tanh(z / 2)): one MUFU operation per element
    float h;
    if constexpr (MODE == 1) {
      constexpr float c1 = 0.5f * 1.5957691216057308f, c3 = 0.5f * 1.5957691216057308f * 0.044715f;
      h = x * fmaf(x * x, c3, c1);
    } else {
      h = x * (0.5f * 1.702f);
    }
    const float t = tanh_approx(h);
    const float hx = 0.5f * x;
    return fmaf(hx, t, hx);
  }
}

// One accumulator element -> output value.
//  I8:  v = fl(fl(float(acc + corr) * sw) * rs) (linear_w8a8.c:168-179), bias, act
//  F16: v = acc (FP32 accumulate), bias, act (mat_mul.c:864-882)
//  MODE 4 (diagnostic): the raw accumulator bits.
template <Kind KIND, int MODE, bool BIAS>
__device__ __forceinline__ float finish(uint32_t acc, int32_t corr, float sw, float rs, float bias) {
  float v;
  if constexpr (KIND == Kind::I8) {
    const int32_t y = static_cast<int32_t>(acc + static_cast<uint32_t>(corr));
    if constexpr (MODE == 4 || MODE == 5) return __int_as_float(y);  // 5: corr holds (sum w) << 7
    v = __fmul_rn(__fmul_rn(__int2float_rn(y), sw), rs);
  } else {
    v = __uint_as_float(acc);
    if constexpr (MODE == 4 || MODE == 5) return v;
  }
  if constexpr (BIAS) v = __fadd_rn(v, bias);
  return epilogue_act<MODE>(v);
}

// Packed FP32x2 arithmetic (two output elements per instruction).  Each lane
// is the IEEE round-to-nearest operation of the scalar form, so finish2 gives
// the bits of finish for both elements.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float &a, float &b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// finish<Kind::I8, MODE, BIAS> for two accumulators of the same column
// (column scale sw2 = {sw, sw}, row scales rs0 and rs1, bias2 = {b, b}).  The
// bias add is fma(v, one, b): with one = 1.0 that is the single rounding of
// v + b, the bits of __fadd_rn, in one packed instruction.  `one` must come
// from kernel arguments: a literal 1.0 lets ptxas fold the multiplication and
// contract the add into the preceding multiply, which rounds differently.
template <int MODE, bool BIAS>
__device__ __forceinline__ void finish2(uint32_t a0, uint32_t a1, int32_t cr, uint64_t sw2, float rs0, float rs1,
                                        uint64_t bias2, uint64_t one2, float &o0, float &o1) {
  const int32_t y0 = static_cast<int32_t>(a0 + static_cast<uint32_t>(cr));
  const int32_t y1 = static_cast<int32_t>(a1 + static_cast<uint32_t>(cr));
  if constexpr (MODE == 4) {
    o0 = __int_as_float(y0);
    o1 = __int_as_float(y1);
    return;
  } else {
    uint64_t v = mul2(mul2(pk2(__int2float_rn(y0), __int2float_rn(y1)), sw2), pk2(rs0, rs1));
    if constexpr (BIAS) v = fma2(v, one2, bias2);
    if constexpr (MODE == 1 || MODE == 2) {
      uint64_t h;
      if constexpr (MODE == 1) {
        constexpr float c1 = 0.5f * 1.5957691216057308f, c3 = 0.5f * 1.5957691216057308f * 0.044715f;
        h = mul2(v, fma2(mul2(v, v), pk2(c3, c3), pk2(c1, c1)));
      } else {
        h = mul2(v, pk2(0.5f * 1.702f, 0.5f * 1.702f));
      }
      float h0, h1;
      upk2(h, h0, h1);
      const uint64_t hx = mul2(pk2(0.5f, 0.5f), v);
      v = fma2(hx, pk2(tanh_approx(h0), tanh_approx(h1)), hx);
    }
    upk2(v, o0, o1);
  }
}

// Plane export (the opcode-15 CPU-epilogue form, linear_w8a8.c:205-227): the
// unsigned-code INT32 accumulator of (m, n) is split into its four bytes.  In
// the 64-row tile of m (rows = the tile's valid rows) and the 32-column half of
// n, byte p sits at position p*rows*32 + (m%64)*32 + n%32 of the half's byte
// stream, and that stream fills the half's 128 output bytes of the tile's rows
// in order.  Returns where byte p of (m, n) goes.
__device__ __forceinline__ uint8_t *plane_dst(float *out, long long ldo, int M, int m, int n, int p) {
  const int t = m >> 6;
  const int rows = min(64, M - (t << 6));
  const int o = p * rows * 32 + (m & 63) * 32 + (n & 31);
  return reinterpret_cast<uint8_t *>(out + (static_cast<long long>(t) * 64 + o / 128) * ldo + (n & ~31)) +
         (o & 127);
}

}  // namespace htpg
