// Per-row 8-bit codes (e4m3fn or int8) of fp32 values, bit-exact with the
// reference's quantize_rows (d3trt/model/quant.py:92-100):
//   scale = max(max_k |x|, 1e-12) / 448 (fp8) or / 127 (int8), IEEE division
//   code  = e4m3fn(clamp(x / scale, +-448)) (RNE) or int8(clamp(rint(x / scale), +-127))
// Shared by the activation-quant kernels and the fused producers (add +
// RMSNorm, sigmoid gate) that quantise their own output rows.
#pragma once

#include "common.cuh"

namespace d3b_quant {

// Two fp32 -> two e4m3fn bytes, round-to-nearest-even, saturating to +-448.
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two codes from two quotients (already in the target's range or not: the
// fp8 conversion saturates to +-448 like the reference's clamp, int8 clamps).
template <int MODE>
__device__ __forceinline__ uint32_t codes2(float v0, float v1) {
  if (MODE == D3B_MODE_FP8) return e4m3x2(v0, v1);
  const int i0 = min(max(__float2int_rn(v0), -127), 127);
  const int i1 = min(max(__float2int_rn(v1), -127), 127);
  return (static_cast<uint32_t>(i0) & 0xFFu) | ((static_cast<uint32_t>(i1) & 0xFFu) << 8);
}

// The codes of the exact IEEE quotients, out of line: it runs only for the
// rare pairs whose fast quotient lies next to a rounding boundary.
template <int MODE>
__device__ __noinline__ uint32_t exact_codes2(float x0, float x1, float scale) {
  float v0 = __fdiv_rn(x0, scale), v1 = __fdiv_rn(x1, scale);
  if (MODE == D3B_MODE_FP8) {
    v0 = fminf(fmaxf(v0, -448.f), 448.f);
    v1 = fminf(fmaxf(v1, -448.f), 448.f);
  }
  return codes2<MODE>(v0, v1);
}

// Codes of RN(x / scale) for two elements, given rcp = RN(1 / scale).
// v = RN(x * rcp) is within 1.5 * 2^-23 |v| of RN(x / scale). Rounding to the
// target format is monotone, so if v * (1 - 2^-21) and v * (1 + 2^-21) (each
// still at least 1.75 * 2^-22 |v| away from v after rounding) give the same
// code, every value between them does, RN(x / scale) included. Otherwise the
// pair is recomputed with IEEE division.
template <int MODE>
__device__ __forceinline__ uint32_t quant2(float x0, float x1, float scale, float rcp) {
  constexpr float kLo = 1.0f - 0x1p-21f, kHi = 1.0f + 0x1p-21f;
  const float v0 = __fmul_rn(x0, rcp), v1 = __fmul_rn(x1, rcp);
  const uint32_t lo = codes2<MODE>(__fmul_rn(v0, kLo), __fmul_rn(v1, kLo));
  const uint32_t hi = codes2<MODE>(__fmul_rn(v0, kHi), __fmul_rn(v1, kHi));
  if (__builtin_expect(lo == hi, 1)) return lo;
  return exact_codes2<MODE>(x0, x1, scale);
}

// ---- bf16 rows: packed arithmetic (the common case) ----
// Non-negative bf16 bit patterns order like unsigned integers, so max|x| of a
// pair word is a packed u16 max of (w & 0x7FFF7FFF).
__device__ __forceinline__ uint32_t umax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// (d0, d1) = (a0, a1) * (b, b), one packed fp32x2 multiply, round to nearest
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b) {
  asm("{.reg .b64 x, y; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %4}; mul.rn.f32x2 x, x, y; mov.b64 {%0, %1}, x;}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b));
}
// The bracket codes (see quant2) of one word of two bf16 values.
template <int MODE>
__device__ __forceinline__ void pair_codes(uint32_t w, float rcp, uint32_t& lo, uint32_t& hi) {
  constexpr float kLo = 1.0f - 0x1p-21f, kHi = 1.0f + 0x1p-21f;
  float v0, v1, l0, l1, h0, h1;
  mul2(v0, v1, __uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u), rcp);
  mul2(l0, l1, v0, v1, kLo);
  mul2(h0, h1, v0, v1, kHi);
  if (MODE == D3B_MODE_FP8) {
    lo = e4m3x2(l0, l1);
    hi = e4m3x2(h0, h1);
  } else {
    // |v| <= 127 (1 + 2^-21) because |x| <= amax: the reference's clamp to
    // +-127 never changes a code here
    lo = (static_cast<uint32_t>(__float2int_rn(l0)) & 0xFFu) | ((static_cast<uint32_t>(__float2int_rn(l1)) & 0xFFu) << 8);
    hi = (static_cast<uint32_t>(__float2int_rn(h0)) & 0xFFu) | ((static_cast<uint32_t>(__float2int_rn(h1)) & 0xFFu) << 8);
  }
}
template <int MODE>
__device__ __noinline__ uint2 exact_codes8_bf16(uint4 raw, float scale) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = exact_codes2<MODE>(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u), scale);
  return make_uint2(c[0] | (c[1] << 16), c[2] | (c[3] << 16));
}
// (d0, d1) = (a0, a1) * (k, k) + (c, c), one packed fp32x2 FMA, one rounding
__device__ __forceinline__ void fma2_kc(float& d0, float& d1, float a0, float a1, float k, float c) {
  asm("{.reg .b64 x, y, z; mov.b64 x, {%2, %3}; mov.b64 y, {%4, %4}; mov.b64 z, {%5, %5}; "
      "fma.rn.f32x2 x, x, y, z; mov.b64 {%0, %1}, x;}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(k), "f"(c));
}

// int8 bracket codes of eight bf16 values, without float-to-int conversions:
// RN(y + 1.5 * 2^23) for |y| < 2^22 is the integer nearest y (ties to even, the
// shifter's last bit being even) plus 0x4B400000 in its bit pattern, so the low
// byte of the bits is rint(y) as a two's-complement int8. The bracket ends are
// the exact products v * (1 -+ 2^-21), each rounded once, straight to an
// integer, by the fused multiply-add; byte permutes gather four codes a word.
__device__ __forceinline__ void int8_bracket8(uint4 raw, float rcp, uint2& lo, uint2& hi) {
  constexpr float kLo = 1.0f - 0x1p-21f, kHi = 1.0f + 0x1p-21f, kShift = 12582912.f;
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t a[8], b[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v0, v1, l0, l1, h0, h1;
    mul2(v0, v1, __uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u), rcp);
    fma2_kc(l0, l1, v0, v1, kLo, kShift);
    fma2_kc(h0, h1, v0, v1, kHi, kShift);
    a[2 * i] = __float_as_uint(l0);
    a[2 * i + 1] = __float_as_uint(l1);
    b[2 * i] = __float_as_uint(h0);
    b[2 * i + 1] = __float_as_uint(h1);
  }
  lo.x = __byte_perm(__byte_perm(a[0], a[1], 0x0040), __byte_perm(a[2], a[3], 0x0040), 0x5410);
  lo.y = __byte_perm(__byte_perm(a[4], a[5], 0x0040), __byte_perm(a[6], a[7], 0x0040), 0x5410);
  hi.x = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
  hi.y = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
}

// Eight codes of eight bf16 values (one 16-byte load -> one 8-byte store).
template <int MODE>
__device__ __forceinline__ uint2 quant8_bf16(uint4 raw, float scale, float rcp) {
  if (MODE == D3B_MODE_INT8) {
    // |v| <= 127 (1 + 2^-21) because |x| <= amax: the reference's clamp to +-127
    // never changes a code here, and the shifter's range holds
    uint2 lo, hi;
    int8_bracket8(raw, rcp, lo, hi);
    if (__builtin_expect((lo.x == hi.x) & (lo.y == hi.y), 1)) return lo;
    return exact_codes8_bf16<MODE>(raw, scale);
  }
  uint32_t l0, l1, l2, l3, h0, h1, h2, h3;
  pair_codes<MODE>(raw.x, rcp, l0, h0);
  pair_codes<MODE>(raw.y, rcp, l1, h1);
  pair_codes<MODE>(raw.z, rcp, l2, h2);
  pair_codes<MODE>(raw.w, rcp, l3, h3);
  const uint32_t w0 = l0 | (l1 << 16), w1 = l2 | (l3 << 16);
  if (__builtin_expect((w0 == (h0 | (h1 << 16))) & (w1 == (h2 | (h3 << 16))), 1)) return make_uint2(w0, w1);
  return exact_codes8_bf16<MODE>(raw, scale);
}

__device__ __forceinline__ float row_scale(float amax, int mode) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  amax = fmaxf(amax, 1e-12f);
  return __fdiv_rn(amax, mode == D3B_MODE_FP8 ? 448.f : 127.f);
}

}  // namespace d3b_quant
