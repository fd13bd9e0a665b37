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


// GELU(x) = x * Phi(x) with Phi the standard normal CDF:
//   t   = min(x^2, 16)                           (rounded: RN(x*x))
//   P   = degree-7 polynomial in t (Horner, fused multiply-adds)
//   Phi = saturate(fma(x, P, 0.5)) to [0, 1]
// P is the weighted minimax fit of 0.5*erf(sqrt(t/2))/sqrt(t) on t in
// [0, 16], weight min(t, sqrt(t)), so that the GELU error relative to
// max(1, |x|) is what is minimised (rust_katago_b200/gelu_fit.py).  For
// |x| <= 4 this is 0.5 + x*P(x^2); beyond, t stays at 16 and the saturation
// pins Phi to 0 or 1 (exactly, once |x| exceeds 4 by 2e-4).
// |error| <= 3.2e-5 * max(1, |x|).  NaN propagates (t = 16, Phi = 0,
// x * 0 = NaN).  Only fused multiply-adds, one min and a saturating FMA: no
// division, no exp, no compare-and-select.
#define KB_GELU_COEFFS                                                                       \
  0x1.985bf8p-2f, -0x1.0eb09cp-4f, 0x1.3b2a38p-7f, -0x1.0fadb6p-10f, 0x1.4b96f4p-14f,        \
      -0x1.0b18b6p-18f, 0x1.f68866p-24f, -0x1.9e1896p-30f

__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float r;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float kb_gelu(float x) {
  constexpr float c[8] = {KB_GELU_COEFFS};
  const float t = fminf(__fmul_rn(x, x), 16.0f);
  float p = c[7];
#pragma unroll
  for (int i = 6; i >= 0; --i) p = __fmaf_rn(p, t, c[i]);
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

// e^x for the SiLU denominator 1 + e^x (x = -g), without conversion or
// transcendental instructions: Cody-Waite reduction x = n*ln2 + r with ln2
// split as 0.693359375 - 2.12194440e-4 (the two-constant split of Cephes
// expf), the degree-7 Taylor polynomial sum r^i/i! on |r| <= ~0.35 in Horner
// form with fused multiply-adds (truncation below 6e-9 relative), and 2^n
// applied as (p * 2^(n-1)) * 2.  n is the exact product x*log2(e) rounded to
// the nearest integer (ties to even) by one fused multiply-add with the
// shifter 1.5 * 2^23, whose result also holds n in its low mantissa bits.
// x is clamped to [-20, 89], which leaves 1 + e^x unchanged: below -17.4,
// e^x < 2^-25 and 1 + e^x rounds to 1 for the clamped value as for the true
// one; above ln(FLT_MAX) = 88.7228 the true e^x overflows, and so does
// (p * 2^127) * 2 for every float x in (88.7228, 89] (p > 1 there).  A NaN
// g reaches the division unchanged.
constexpr float kSiluLog2e = 0x1.715476p+0f;
constexpr float kSiluShifter = 0x1.8p+23f;  // 1.5 * 2^23
#define KB_SILU_EXP_POLY(FMA, P, R)                       \
  P = FMA(P, R, C2(0x1.6c16c2p-10f)); /* 1/720 */        \
  P = FMA(P, R, C2(0x1.111112p-7f));  /* 1/120 */        \
  P = FMA(P, R, C2(0x1.555556p-5f));  /* 1/24 */         \
  P = FMA(P, R, C2(0x1.555556p-3f));  /* 1/6 */          \
  P = FMA(P, R, C2(0.5f));                               \
  P = FMA(P, R, C2(1.0f));                               \
  P = FMA(P, R, C2(1.0f));

// 2^(n-1) from the shifter sum k = 1.5 * 2^23 + n (bits 0x4B400000 + n):
// its bits shifted left by 23 are n << 23 (mod 2^32).
__device__ __forceinline__ float silu_exp_scale(float k) {
  return __int_as_float((__float_as_int(k) << 23) + (126 << 23));
}

__device__ __forceinline__ float silu_exp(float x) {
#define C2(v) (v)
  const float xc = fminf(fmaxf(x, -20.0f), 89.0f);
  const float k = __fmaf_rn(xc, kSiluLog2e, kSiluShifter);
  const float n = __fadd_rn(k, -kSiluShifter);
  float r = __fmaf_rn(-n, 0x1.63p-1f /* 0.693359375 */, xc);
  r = __fmaf_rn(n, 0x1.bd0106p-13f /* 2.12194440e-4 */, r);
  float p = 0x1.a01a02p-13f /* 1/5040 */;
  KB_SILU_EXP_POLY(__fmaf_rn, p, r)
  return __fmul_rn(__fmul_rn(p, silu_exp_scale(k)), 2.0f);
#undef C2
}

// silu_exp on a pair, bit-identical to two scalar calls.
__device__ __forceinline__ float2 silu_exp2(float2 x) {
#define C2(v) make_float2(v, v)
  const float2 xc = make_float2(fminf(fmaxf(x.x, -20.0f), 89.0f), fminf(fmaxf(x.y, -20.0f), 89.0f));
  const float2 k = fma2(xc, C2(kSiluLog2e), C2(kSiluShifter));
  const float2 n = add2(k, C2(-kSiluShifter));
  float2 r = fma2(n, C2(-0x1.63p-1f), xc);
  r = fma2(n, C2(0x1.bd0106p-13f), r);
  float2 p = C2(0x1.a01a02p-13f);
  KB_SILU_EXP_POLY(fma2, p, r)
  return mul2(mul2(p, make_float2(silu_exp_scale(k.x), silu_exp_scale(k.y))), C2(2.0f));
#undef C2
}
#undef KB_SILU_EXP_POLY

// SiLU exactly as the reference writes it inside its SwiGLU: g / (1 + e^-g)
// (cuda-kernels/int8_ops.cu:111-113), with silu_exp in place of expf.
__device__ __forceinline__ float kb_silu(float g) {
  return __fdiv_rn(g, __fadd_rn(1.0f, silu_exp(-g)));
}

// kb_silu on a pair, bit-identical to two scalar calls.  (The one packed
// multiply that feeds a packed add, e^x's final * 2, is exact, so contracting
// the two into a fused multiply-add leaves every result unchanged.)
__device__ __forceinline__ float2 kb_silu2(float2 g) {
  const float2 d = add2(make_float2(1.0f, 1.0f), silu_exp2(make_float2(-g.x, -g.y)));
  return make_float2(__fdiv_rn(g.x, d.x), __fdiv_rn(g.y, d.y));
}

// kb_gelu on a pair, bit-identical to two scalar calls.
__device__ __forceinline__ float2 kb_gelu2(float2 x) {
  constexpr float c[8] = {KB_GELU_COEFFS};
  float2 t = mul2(x, x);
  t.x = fminf(t.x, 16.0f);
  t.y = fminf(t.y, 16.0f);
  float2 p = make_float2(c[7], c[7]);
#pragma unroll
  for (int i = 6; i >= 0; --i) p = fma2(p, t, make_float2(c[i], c[i]));
  // (the packed FMA has no saturating form: two scalar saturating FMAs)
  return mul2(x, make_float2(fma_sat(x.x, p.x, 0.5f), fma_sat(x.y, p.y, 0.5f)));
}

enum Act : int { kActNone = 0, kActGelu = 1, kActSilu = 2 };

template <int ACT>
__device__ __forceinline__ float2 apply_act2(float2 v) {
  if constexpr (ACT == kActGelu) return kb_gelu2(v);
  else if constexpr (ACT == kActSilu) return kb_silu2(v);
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
