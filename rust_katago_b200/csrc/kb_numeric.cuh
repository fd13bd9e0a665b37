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
// Branch-free: the input is clamped into the finite range for the arithmetic
// and the out-of-range results (inf, 0, NaN) are selected at the end.
__device__ __forceinline__ float kb_expf(float x) {
  const float xc = fminf(fmaxf(x, -0x1.9fe36ap+6f), 0x1.62e42ep+6f);
  const float n = rintf(__fmul_rn(xc, 0x1.715476p+0f /* log2(e) */));
  float r = __fmaf_rn(-n, 0x1.63p-1f /* 0.693359375 */, xc);
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
  float y = __fmul_rn(__fmul_rn(p, pow2i(n1)), pow2i(n2));
  y = x > 0x1.62e42ep+6f ? __int_as_float(0x7f800000) : y;
  y = x < -0x1.9fe36ap+6f ? 0.0f : y;
  return x != x ? x : y;
}

// Round a pair to the 16-bit type (binary16 or bfloat16, round to nearest
// even); element 0 in the low half.
__device__ __forceinline__ uint32_t pack16x2(float2 v, bool f16) {
  if (f16) {
    const __half2 h = __floats2half2_rn(v.x, v.y);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// SiLU exactly as the reference writes it inside its SwiGLU: g / (1 + e^-g)
// (cuda-kernels/int8_ops.cu:111-113), with kb_expf in place of expf.
__device__ __forceinline__ float kb_silu(float g) {
  return __fdiv_rn(g, __fadd_rn(1.0f, kb_expf(-g)));
}

// GELU(x) = x * Phi(x) with Phi the standard normal CDF:
//   s   = min(x^2/8 - 1, 1)                      (rounded: RN(RN(x*x)*0.125 - 1))
//   P   = degree-10 polynomial in s (Horner, fused multiply-adds)
//   Phi = saturate(fma(x, P, 0.5)) to [0, 1]
// P is the least-squares Chebyshev fit of 0.5*erf(sqrt(t/2))/sqrt(t) on
// t = x^2 in [0, 16] (rust_katago_b200/gelu_fit.py).  For |x| <= 4 this is
// 0.5 + x*P(x^2); beyond, s stays at 1 and the saturation pins Phi to 0 or 1
// (exactly, once |x| exceeds 4 by 2e-4).  |error| <= 3.2e-5 * max(1, |x|).
// NaN propagates (Phi = 0, x * 0 = NaN).  Only fused multiply-adds, one min
// and a saturating FMA: no division, no exp, no compare-and-select.
#define KB_GELU_COEFFS                                                                      \
  0x1.68585ap-3f, -0x1.5961f4p-4f, 0x1.ca3788p-5f, -0x1.2df2f6p-5f, 0x1.70d728p-6f,        \
      -0x1.9ab164p-7f, 0x1.9a7b1cp-8f, -0x1.5eeeecp-9f, 0x1.229b08p-10f, -0x1.31c494p-11f, \
      0x1.a02d8ap-13f

__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float r;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float kb_gelu(float x) {
  constexpr float c[11] = {KB_GELU_COEFFS};
  const float s = fminf(__fmaf_rn(__fmul_rn(x, x), 0.125f, -1.0f), 1.0f);
  float p = c[10];
#pragma unroll
  for (int i = 9; i >= 0; --i) p = __fmaf_rn(p, s, c[i]);
  return __fmul_rn(x, fma_sat(x, p, 0.5f));
}

// ------------------------------------------------------------------ f32x2
// Packed pairs of IEEE fp32 operations (sm_100 f32x2 instructions): each lane
// of the pair rounds exactly like the scalar __fmul_rn/__fadd_rn/__fmaf_rn.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2pack(a.x, a.y)), "l"(f2pack(b.x, b.y)));
  return f2unpack(r);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2pack(a.x, a.y)), "l"(f2pack(b.x, b.y)));
  return f2unpack(r);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(f2pack(a.x, a.y)), "l"(f2pack(b.x, b.y)), "l"(f2pack(c.x, c.y)));
  return f2unpack(r);
}

// kb_gelu on a pair, bit-identical to two scalar calls.
__device__ __forceinline__ float2 kb_gelu2(float2 x) {
  constexpr float c[11] = {KB_GELU_COEFFS};
  float2 s = fma2(mul2(x, x), make_float2(0.125f, 0.125f), make_float2(-1.0f, -1.0f));
  s.x = fminf(s.x, 1.0f);
  s.y = fminf(s.y, 1.0f);
  float2 p = make_float2(c[10], c[10]);
#pragma unroll
  for (int i = 9; i >= 0; --i) p = fma2(p, s, make_float2(c[i], c[i]));
  // (the packed FMA has no saturating form: two scalar saturating FMAs)
  return mul2(x, make_float2(fma_sat(x.x, p.x, 0.5f), fma_sat(x.y, p.y, 0.5f)));
}

enum Act : int { kActNone = 0, kActGelu = 1, kActSilu = 2 };

template <int ACT>
__device__ __forceinline__ float2 apply_act2(float2 v) {
  if constexpr (ACT == kActGelu) return kb_gelu2(v);
  else if constexpr (ACT == kActSilu) return make_float2(kb_silu(v.x), kb_silu(v.y));
  else return v;
}

template <int ACT>
__device__ __forceinline__ float apply_act(float v) {
  if constexpr (ACT == kActGelu) return kb_gelu(v);
  else if constexpr (ACT == kActSilu) return kb_silu(v);
  else return v;
}

// Division of 32-bit dividends n < 2^31 by a runtime-invariant divisor d >= 1
// without a division instruction (the round-up multiplier method of Granlund &
// Montgomery, "Division by invariant integers using multiplication", 1994):
// with s = ceil(log2 d) and m = floor(2^32 * (2^s - d) / d) + 1,
// n / d = (umulhi(n, m) + n) >> s.
struct FastDiv {
  uint32_t d = 1, m = 0, s = 0;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t div) : d(div) {
    while ((1ull << s) < d) ++s;
    m = static_cast<uint32_t>((((1ull << s) - d) << 32) / d + 1);
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> s; }
};

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
