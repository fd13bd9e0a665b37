// Elementwise numerics shared by the kernels.  Every function here is a fixed
// sequence of IEEE-rounded float operations (explicit __fmul_rn/__fadd_rn/
// __fdiv_rn/__fmaf_rn, no contraction, no fast-math), so a CPU program that
// performs the same sequence reproduces the GPU result bit for bit.  The CPU
// restatement under oracle/ does exactly that.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace kb {

// 2^k for -126 <= k <= 127, built from its exponent bits.
__device__ __forceinline__ float pow2i(int k) { return __int_as_float((k + 127) << 23); }

// exp(x): Cody-Waite range reduction x = n*ln2 + r with ln2 split as
// 0.693359375 - 2.12194440e-4 (the two-constant split used by Cephes expf),
// then the degree-7 Taylor polynomial sum r^i/i! on |r| <= ~0.35 in Horner
// form with fused multiply-adds, then an exact two-step scaling by 2^n.
// Truncation error of the polynomial is below 6e-9 relative.
__device__ __forceinline__ float kb_expf(float x) {
  if (x != x) return x;
  if (x > 0x1.62e42ep+6f) return __int_as_float(0x7f800000);
  if (x < -0x1.9fe36ap+6f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 0x1.715476p+0f /* log2(e) */));
  float r = __fmaf_rn(-n, 0x1.63p-1f /* 0.693359375 */, x);
  r = __fmaf_rn(n, 0x1.bd0106p-13f /* 2.12194440e-4 */, r);
  float p = 0x1.a01a02p-13f /* 1/5040 */;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f /* 1/720 */);
  p = __fmaf_rn(p, r, 0x1.111112p-7f /* 1/120 */);
  p = __fmaf_rn(p, r, 0x1.555556p-5f /* 1/24 */);
  p = __fmaf_rn(p, r, 0x1.555556p-3f /* 1/6 */);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = static_cast<int>(n);
  const int n1 = ni / 2;
  const int n2 = ni - n1;
  return __fmul_rn(__fmul_rn(p, pow2i(n1)), pow2i(n2));
}

// SiLU exactly as the reference writes it inside its SwiGLU: g / (1 + e^-g)
// (cuda-kernels/int8_ops.cu:111-113), with kb_expf in place of expf.
__device__ __forceinline__ float kb_silu(float g) {
  return __fdiv_rn(g, __fadd_rn(1.0f, kb_expf(-g)));
}

// GELU, erf form: 0.5 * x * (1 + erf(x / sqrt 2)).  erf(z) for z >= 0 uses
// Abramowitz & Stegun 7.1.26 (Hastings' rational approximation,
// |error| <= 1.5e-7): erf(z) = 1 - t*(a1 + t*(a2 + t*(a3 + t*(a4 + t*a5)))) * e^(-z^2),
// t = 1 / (1 + p z).
__device__ __forceinline__ float kb_gelu(float x) {
  const float z = __fmul_rn(fabsf(x), 0x1.6a09e6p-1f /* 1/sqrt(2) */);
  const float t = __fdiv_rn(1.0f, __fmaf_rn(0x1.4f740ap-2f /* p = 0.3275911 */, z, 1.0f));
  float poly = __fmaf_rn(0x1.0fb844p+0f /* a5 */, t, -0x1.7401c6p+0f /* a4 */);
  poly = __fmaf_rn(poly, t, 0x1.6be1c6p+0f /* a3 */);
  poly = __fmaf_rn(poly, t, -0x1.23531cp-2f /* a2 */);
  poly = __fmaf_rn(poly, t, 0x1.04f20cp-2f /* a1 */);
  const float e = kb_expf(-__fmul_rn(z, z));
  const float erf_abs = __fadd_rn(1.0f, -__fmul_rn(__fmul_rn(poly, t), e));
  const float erf = x < 0.0f ? -erf_abs : erf_abs;
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erf));
}

enum Act : int { kActNone = 0, kActGelu = 1, kActSilu = 2 };

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == kActGelu) return kb_gelu(v);
  if (act == kActSilu) return kb_silu(v);
  return v;
}

// Round a float through a 16-bit storage type (RNE) and back.
__device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
__device__ __forceinline__ uint16_t bits_f16(float v) {
  return __half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ uint16_t bits_bf16(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float from_f16(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ float from_bf16(uint16_t b) {
  return __bfloat162float(__ushort_as_bfloat16(b));
}
__device__ __forceinline__ uint16_t bits16(float v, bool f16) { return f16 ? bits_f16(v) : bits_bf16(v); }
__device__ __forceinline__ float from16(uint16_t b, bool f16) { return f16 ? from_f16(b) : from_bf16(b); }

// Absolute-value bits: for |v| the IEEE ordering equals unsigned integer
// ordering, and every NaN/Inf compares above every finite value, so an
// integer max over these bits is both the reference's fmaxf(|v|) for finite
// rows and its "row contains a non-finite value" flag.
__device__ __forceinline__ uint32_t abs_bits(float v) { return __float_as_uint(v) & 0x7fffffffu; }

// Per-token symmetric INT8 scale from an absolute-maximum bit pattern:
// NaN when the row held a non-finite value, 1 for an all-zero row, amax/127
// otherwise (cuda-kernels/int8_ops.cu:40, :80).
__device__ __forceinline__ float int8_scale_from_amax(uint32_t amax_bits) {
  if (amax_bits >= 0x7f800000u) return __int_as_float(0x7fc00000);
  if (amax_bits == 0) return 1.0f;
  return __fdiv_rn(__uint_as_float(amax_bits), 127.0f);
}

// q = clamp(rne(v / scale), -127, 127) with IEEE division (int8_ops.cu:44).
__device__ __forceinline__ int quant_i8(float v, float scale) {
  const int q = __float2int_rn(__fdiv_rn(v, scale));
  return max(-127, min(127, q));
}

}  // namespace kb
