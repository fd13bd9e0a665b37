// Per-token dynamic INT8 activation quantisers.
//
// Replaces the reference's row quantisers and its fused RMSNorm quantiser
// (crates/kata_nn/cuda-kernels/int8_ops.cu:8-89, :140-176).  One warp owns one
// token row, eight rows per 256-thread CTA, and the row stays in registers:
// lane l holds the 8-element groups g = l, l+32, l+64, ... (columns 8g..8g+7),
// brought in with one 16-byte load per group (fp32 rows: two).  Per row:
//   * RMS (optional): sum = fma(x, x, sum) over the lane's columns in group
//     order, then an xor butterfly over 16, 8, 4, 2, 1 (the reference's
//     per-lane partial sums and butterfly, int8_ops.cu:17-25, with 8-wide
//     groups instead of 1-wide lane striding); rstd = 1/sqrt(sum/W + eps)
//     correctly rounded (rsqrtf in the reference); v = T16((x*rstd)*gamma);
//   * scale = NaN if the row holds a non-finite value, 1 if all zero,
//     amax/127 otherwise (int8_ops.cu:36-40); amax is an integer max over
//     |16-bit| bit patterns, which orders exactly like fmaxf(|v|);
//   * q = clamp(rne(v / scale), +-127) with IEEE division, 0 for a bad row,
//     zero padding up to kp (int8_ops.cu:42-46, :80-88); 8-byte stores.
#include "kb_internal.h"
#include "kb_mxfp8.cuh"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

enum InType : int { kInF32 = 0, kInF16 = 1, kInBF16 = 2 };

__device__ __forceinline__ float warp_sum_xor(float v) {
#pragma unroll
  for (int step = 16; step; step >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, step));
  return v;
}

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
  for (int step = 16; step; step >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, step));
  return v;
}

// Load group g (columns 8g..8g+7) of a row as 8 floats; columns >= width read 0.
template <int IN>
__device__ __forceinline__ void load_group(const void* row, int g, int width, bool vec, float (&x)[8]) {
  const int c0 = 8 * g;
  if constexpr (IN == kInF32) {
    const float* s = static_cast<const float*>(row) + c0;
    if (vec && c0 + 8 <= width) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(s));
      const float4 b = __ldg(reinterpret_cast<const float4*>(s) + 1);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) x[t] = c0 + t < width ? __ldg(s + t) : 0.0f;
    }
  } else {
    const bool f16 = IN == kInF16;
    const uint16_t* s = static_cast<const uint16_t*>(row) + c0;
    if (vec && c0 + 8 <= width) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(s));
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        x[2 * t] = from16(static_cast<uint16_t>(w[t] & 0xffffu), f16);
        x[2 * t + 1] = from16(static_cast<uint16_t>(w[t] >> 16), f16);
      }
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) x[t] = c0 + t < width ? from16(s[t], f16) : 0.0f;
    }
  }
}

// rne(v / s) as an integer, clamped to +-127, with the quotient rounded
// exactly as IEEE division rounds it: q0 = RN(v*r), e = v - q0*s (exact by
// FMA), q = RN(q0 + e*r) with r = RN(1/s) is the correctly rounded v/s when
// nothing underflows (Markstein's division theorem).  The caller uses it only
// for rows whose scale and amax are normal numbers, where |v/s| <= 127 and the
// residual e is exact or its quotient contribution rounds away below 0.5.
__device__ __forceinline__ int quant_i8_rcp(float v, float s, float r) {
  const float q0 = __fmul_rn(v, r);
  const float e = __fmaf_rn(-q0, s, v);
  const float q = __fmaf_rn(e, r, q0);
  return __float2int_rn(fminf(fmaxf(q, -127.0f), 127.0f));
}

__device__ __forceinline__ uint32_t pack4_i8(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xffu) | ((static_cast<uint32_t>(b) & 0xffu) << 8) |
         ((static_cast<uint32_t>(c) & 0xffu) << 16) | (static_cast<uint32_t>(d) << 24);
}

// IEEE-division fallback for one group of 8 packed 16-bit values.
__device__ __noinline__ void quantize_group_slow(uint4 w4, bool f16, float scale, bool bad,
                                                 int8_t* dst) {
  const uint32_t w[4] = {w4.x, w4.y, w4.z, w4.w};
  int qi[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float v = from16(static_cast<uint16_t>(t & 1 ? w[t / 2] >> 16 : w[t / 2] & 0xffffu), f16);
    qi[t] = bad ? 0 : quant_i8(v, scale);
  }
  *reinterpret_cast<uint2*>(dst) =
      make_uint2(pack4_i8(qi[0], qi[1], qi[2], qi[3]), pack4_i8(qi[4], qi[5], qi[6], qi[7]));
}

__device__ __noinline__ void quantize_group_slow_f32(float4 a, float4 b, float scale, bool bad,
                                                     int8_t* dst) {
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  int qi[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) qi[t] = bad ? 0 : quant_i8(v[t], scale);
  *reinterpret_cast<uint2*>(dst) =
      make_uint2(pack4_i8(qi[0], qi[1], qi[2], qi[3]), pack4_i8(qi[4], qi[5], qi[6], qi[7]));
}

// Round-to-nearest-even to an integer by adding 1.5 * 2^23: for |q| < 2^22 the
// sum is exactly representable only at integers, so the add rounds q as rint
// does, and the low byte of the sum's bits is the two's-complement int8 of
// the result (the constant's low 22 bits are zero).  One FMA-pipe add per value
// instead of a float-to-int conversion.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

// Low bytes of four such sums -> one packed int8x4 word (two byte permutes).
__device__ __forceinline__ uint32_t pack4_magic(float a, float b, float c, float d) {
  const uint32_t ab = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x0040);
  const uint32_t cd = __byte_perm(__float_as_uint(c), __float_as_uint(d), 0x0040);
  return __byte_perm(ab, cd, 0x5410);
}

template <bool F16>
__device__ __forceinline__ uint2 quant_group_fast(const uint32_t (&w)[4], float scale, float r) {
  float m[8];
#pragma unroll
  for (int t = 0; t < 8; t += 2) {
    // Pair of values through packed fp32: q0 = v*r, e = v - q0*s, q = q0 + e*r
    // (correctly rounded v/s), then rint(q) by the magic add.  A packed
    // multiply feeding only multiplicands or an FMA cannot be contracted.
    // |v/scale| <= 127 for a normal scale = amax/127, so no clamp is needed.
    const uint32_t pw = w[t / 2];
    const float2 v = make_float2(from16(static_cast<uint16_t>(pw & 0xffffu), F16), from16(static_cast<uint16_t>(pw >> 16), F16));
    const float2 q0 = mul2(v, make_float2(r, r));
    const float2 e = fma2(make_float2(-q0.x, -q0.y), make_float2(scale, scale), v);
    const float2 q = fma2(e, make_float2(r, r), q0);
    const float2 mq = add2(q, make_float2(kRoundMagic, kRoundMagic));
    m[t] = mq.x;
    m[t + 1] = mq.y;
  }
  return make_uint2(pack4_magic(m[0], m[1], m[2], m[3]), pack4_magic(m[4], m[5], m[6], m[7]));
}


// Quantise a warp-held row of packed 16-bit values (lane l holds groups
// l, l+32, ...; amax2 = this lane's packed |bits| maximum).
template <bool F16, int G>
__device__ __forceinline__ void quantize_packed_row(const uint32_t (&w)[G][4], uint32_t amax2, int kp, int lane,
                                                    int8_t* dst, float* scale_out, unsigned* status,
                                                    unsigned layer) {
  const uint32_t m16 = max(amax2 & 0xffffu, amax2 >> 16);
  const uint32_t amax = warp_max_u32(F16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m16))) : (m16 << 16));
  const float scale = int8_scale_from_amax(amax);
  const bool bad = amax >= 0x7f800000u;
  if (lane == 0) {
    *scale_out = scale;
    if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
  }
  // The reciprocal path needs a normal scale and a normal amax; other rows
  // (all zero, tiny, non-finite) take the IEEE-division loop, kept out of line.
  const bool fast = !bad && amax >= 0x00800000u && __float_as_uint(scale) >= 0x00800000u;
  const int out_groups = kp / 8;
  if (fast) {
    const float r = __frcp_rn(scale);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j;
      if (g < out_groups) *reinterpret_cast<uint2*>(dst + 8 * g) = quant_group_fast<F16>(w[j], scale, r);
    }
  } else {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j;
      if (g < out_groups)
        quantize_group_slow(make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]), F16, scale, bad, dst + 8 * g);
    }
  }
}

// Plain 16-bit rows (no RMS): the row stays packed (two values per register),
// the absolute maximum is a packed unsigned max over |bits|.
template <bool F16, int G>
__device__ __forceinline__ void quantize_row16(const uint16_t* src, bool vec, int width, int kp,
                                               int lane, int8_t* dst, float* scale_out,
                                               unsigned* status, unsigned layer) {
  const int groups = (width + 7) / 8;
  uint32_t w[G][4];
  uint32_t amax2 = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = lane + 32 * j;
    const int c0 = 8 * g;
    if (g < groups && vec && c0 + 8 <= width) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(src + c0));
      w[j][0] = a.x; w[j][1] = a.y; w[j][2] = a.z; w[j][3] = a.w;
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t lo = (g < groups && c0 + 2 * t < width) ? src[c0 + 2 * t] : 0u;
        const uint32_t hi = (g < groups && c0 + 2 * t + 1 < width) ? src[c0 + 2 * t + 1] : 0u;
        w[j][t] = lo | (hi << 16);
      }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) amax2 = __vmaxu2(amax2, w[j][t] & 0x7fff7fffu);
  }
  quantize_packed_row<F16, G>(w, amax2, kp, lane, dst, scale_out, status, layer);
}

// Raw 16-bit groups (lane l: groups l, l+32, ...) of one row, zero past
// `width`; loaded one row ahead of use by the RMS quantisers.
template <int G>
__device__ __forceinline__ void load_raw16(const uint16_t* __restrict__ src, int width, int lane, uint4 (&raw)[G]) {
  const int groups = (width + 7) / 8;
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = lane + 32 * j;
    const int c0 = 8 * g;
    if (g < groups && vec && c0 + 8 <= width) {
      raw[j] = __ldg(reinterpret_cast<const uint4*>(src + c0));
    } else {
      uint32_t w[4] = {0, 0, 0, 0};
      if (g < groups) {
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (c0 + t < width) w[t / 2] |= static_cast<uint32_t>(__ldg(src + c0 + t)) << (16 * (t & 1));
      }
      raw[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <bool F16, int G>
__device__ __forceinline__ void raw16_to_float(const uint4 (&raw)[G], float (&v)[G][8]) {
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      v[j][2 * t] = from16(static_cast<uint16_t>(w[t] & 0xffffu), F16);
      v[j][2 * t + 1] = from16(static_cast<uint16_t>(w[t] >> 16), F16);
    }
  }
}

// RMSNorm of a warp-held row (lane l holds groups l, l+32, ...):
// sum = fma(x, x, sum) over the lane's columns in group order, xor butterfly,
// rstd = 1/sqrt(sum/W + eps) correctly rounded, v = T16((x*rstd)*gamma) packed;
// columns past `width` are 0.  amax2: the lane's packed |16-bit| maximum.
template <int G>
__device__ __forceinline__ void rms_normalize(const float (&v)[G][8], const float* __restrict__ gamma, float eps,
                                              int width, int lane, bool f16, uint32_t (&nw)[G][4],
                                              uint32_t& amax2) {
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < G; ++j)
#pragma unroll
    for (int t = 0; t < 8; ++t) sum = __fmaf_rn(v[j][t], v[j][t], sum);
  sum = warp_sum_xor(sum);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(width)), eps)));
  amax2 = 0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int c0 = 8 * (lane + 32 * j);
    float gm[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c0 < width)
      load_group<kInF32>(gamma, lane + 32 * j, width, (reinterpret_cast<uintptr_t>(gamma) & 15) == 0, gm);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const float2 n2 = mul2(mul2(make_float2(v[j][2 * t], v[j][2 * t + 1]), make_float2(rstd, rstd)),
                             make_float2(gm[2 * t], gm[2 * t + 1]));
      nw[j][t] = pack16x2(n2, f16);
      amax2 = __vmaxu2(amax2, nw[j][t] & 0x7fff7fffu);
    }
  }
}

// MXFP8 block-32 quantisation of a warp-held packed 16-bit row: the four lanes
// 4q..4q+3 of group index j hold one 32-column block, whose amax is a quad
// reduction.  Same scale / rounding / non-finite rules as mxfp8.cu.
template <bool F16, int G>
__device__ __forceinline__ void mx_quantize_packed_row(const uint32_t (&w)[G][4], int row, int kp, int blocks4,
                                                       int lane, uint8_t* __restrict__ dst,
                                                       uint8_t* __restrict__ scales, unsigned* status,
                                                       unsigned layer) {
  const uint32_t inf16 = F16 ? 0x7c00u : 0x7f80u;
  const int nblocks = kp >> 5;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = lane + 32 * j;
    uint32_t m2 = 0;
#pragma unroll
    for (int t = 0; t < 4; ++t) m2 = __vmaxu2(m2, w[j][t] & 0x7fff7fffu);
    const uint32_t m16 = max(m2 & 0xffffu, m2 >> 16);
    unsigned bad = 0;
    if (m16 >= inf16) {
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t h = ((t & 1) ? w[j][t / 2] >> 16 : w[j][t / 2]) & 0x7fffu;
        if (h > inf16) bad |= KB_STATUS_NAN;
        else if (h == inf16) bad |= KB_STATUS_INF;
      }
      record_status(status, bad, layer);
    }
    // Finite |v| bits of the block (non-finite lanes contribute 0, the block is zeroed).
    uint32_t a = bad ? 0u : (F16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m16))) : (m16 << 16));
    unsigned any_bad = bad;
    a = max(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = max(a, __shfl_xor_sync(0xffffffffu, a, 2));
    any_bad |= __shfl_xor_sync(0xffffffffu, any_bad, 1);
    any_bad |= __shfl_xor_sync(0xffffffffu, any_bad, 2);
    const int blk = g >> 2;
    if (blk >= nblocks) continue;  // quad-uniform
    const bool zero = a == 0u || any_bad != 0;
    const uint32_t scale = zero ? 127u : ue8m0_ceil(__fdiv_rn(__uint_as_float(a), 448.0f));
    const float rcp = ue8m0_reciprocal(scale);
    uint32_t out[2] = {0u, 0u};
    if (!zero) {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float lo = from16(static_cast<uint16_t>(w[j][t] & 0xffffu), F16);
        const float hi = from16(static_cast<uint16_t>(w[j][t] >> 16), F16);
        out[t >> 1] |= e4m3x2(__fmul_rn(lo, rcp), __fmul_rn(hi, rcp)) << (16 * (t & 1));
      }
    }
    *reinterpret_cast<uint2*>(dst + 8 * g) = make_uint2(out[0], out[1]);
    if ((lane & 3) == 0) scales[mx_scale_offset(row, blk, blocks4)] = static_cast<uint8_t>(scale);
  }
}

// Fused RMSNorm -> 16-bit boundary -> MXFP8 (E4M3 + UE8M0 per 32 columns).
template <int IN, int G>
__global__ void __launch_bounds__(256) rms_mxfp8_kernel(
    const void* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows, int width, int kp,
    int blocks4, int bound_f16, uint8_t* __restrict__ q, uint8_t* __restrict__ scales, unsigned* status,
    unsigned layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;  // warp-uniform
  constexpr int kEsize = IN == kInF32 ? 4 : 2;
  const uint8_t* src = static_cast<const uint8_t*>(x) + static_cast<size_t>(row) * ldx * kEsize;
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  const int groups = (width + 7) / 8;
  float v[G][8];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = lane + 32 * j;
    if (g < groups) {
      load_group<IN>(src, g, width, vec, v[j]);
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[j][t] = 0.0f;
    }
  }
  uint32_t nw[G][4];
  uint32_t amax2;
  rms_normalize<G>(v, gamma, eps, width, lane, bound_f16 != 0, nw, amax2);
  uint8_t* dst = q + static_cast<size_t>(row) * kp;
  if (bound_f16)
    mx_quantize_packed_row<true, G>(nw, row, kp, blocks4, lane, dst, scales, status, layer);
  else
    mx_quantize_packed_row<false, G>(nw, row, kp, blocks4, lane, dst, scales, status, layer);
}

// Fused RMSNorm quantisers for 16-bit rows, persistent over rows: each warp
// walks rows warp_id, warp_id + stride, ... and loads the next row while it
// normalises and quantises the current one (the single-row form is bound by
// the load latency of its one row).  MX = false: INT8 per-token output
// (q int8 [rows, kp] + fp32 scales); MX = true: MXFP8 (q E4M3 + packed scales).
// Up to 4 groups per lane (rows of <= 1024) the registers are capped so that
// three CTAs (24 warps) share an SM: more rows in flight per SM.
template <bool F16IN, bool MX, int G>
__global__ void __launch_bounds__(256, G <= 4 ? 3 : 1) rms_rows16_kernel(
    const uint16_t* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows, int width,
    int kp, int blocks4, int bound_f16, void* __restrict__ q, void* __restrict__ scales, unsigned* status,
    unsigned layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int step = gridDim.x * 8;
  int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;  // warp-uniform
  uint4 raw[G];
  load_raw16<G>(x + static_cast<size_t>(row) * ldx, width, lane, raw);
  for (; row < rows; row += step) {
    float v[G][8];
    raw16_to_float<F16IN, G>(raw, v);
    if (row + step < rows) load_raw16<G>(x + static_cast<size_t>(row + step) * ldx, width, lane, raw);
    uint32_t nw[G][4];
    uint32_t amax2;
    rms_normalize<G>(v, gamma, eps, width, lane, bound_f16 != 0, nw, amax2);
    if constexpr (MX) {
      uint8_t* dst = static_cast<uint8_t*>(q) + static_cast<size_t>(row) * kp;
      if (bound_f16)
        mx_quantize_packed_row<true, G>(nw, row, kp, blocks4, lane, dst, static_cast<uint8_t*>(scales), status, layer);
      else
        mx_quantize_packed_row<false, G>(nw, row, kp, blocks4, lane, dst, static_cast<uint8_t*>(scales), status, layer);
    } else {
      int8_t* dst = static_cast<int8_t*>(q) + static_cast<size_t>(row) * kp;
      float* sc = static_cast<float*>(scales) + row;
      if (bound_f16)
        quantize_packed_row<true, G>(nw, amax2, kp, lane, dst, sc, status, layer);
      else
        quantize_packed_row<false, G>(nw, amax2, kp, lane, dst, sc, status, layer);
    }
  }
}

// Rows of exactly 256*G columns (kp == width, rows and gamma 16-byte aligned),
// INT8 output: rms_rows16_kernel without any per-group bounds check, the
// output type a template parameter, and the row's absolute maximum a packed
// max(|a|, |b|) per pair (one instruction; NaN still wins, so a non-finite
// row is classified as before).
//
// Two rows per warp: half-warp h = lane / 16 holds row 2w + h of warp w's
// pair, lane l = lane % 16 the groups l + 16j (j < 2G).  The sum of squares
// runs as the warp-per-row layout's lanes l and l + 16 run it: chain A over
// groups l, l + 32, ... and chain B over l + 16, l + 48, ..., each in group
// order, then A + B (the first step of the 32-lane xor butterfly, offset 16)
// and the butterfly over offsets 8, 4, 2, 1 inside the half: the same
// additions in the same order, so the bytes and scales are identical to the
// generic kernel's.  The per-row work (both reductions, the correctly rounded
// 1/sqrt, the scale and its reciprocal) is issued once for two rows.
// Row count from which the two-rows-per-warp RMS quantisers are used (below it,
// a few positions' rows, one row per warp keeps more warps on the short pass).
constexpr int kPairRows = 2048;

template <bool F16IN, bool F16OUT, int G>
__global__ void __launch_bounds__(256, 2) rms_rows16_full_kernel(
    const uint16_t* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows,
    int8_t* __restrict__ q, float* __restrict__ scales, unsigned* status, unsigned layer) {
  constexpr int kW = 256 * G;
  constexpr int kJ = 2 * G;  // groups per lane
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int step = gridDim.x * 16;
  int row0 = (blockIdx.x * 8 + warp) * 2;  // the pair's first row (warp-uniform)
  if (row0 >= rows) return;
  uint4 raw[kJ];
  auto load = [&](int r) {
#pragma unroll
    for (int j = 0; j < kJ; ++j)
      raw[j] = r < rows ? __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * ldx + 8 * (hl + 16 * j)))
                        : make_uint4(0, 0, 0, 0);
  };
  load(row0 + half);
  for (; row0 < rows; row0 += step) {
    const int row = row0 + half;
    const bool ok = row < rows;
    float v[kJ][8];
    raw16_to_float<F16IN, kJ>(raw, v);
    if (row0 + step < rows) load(row + step);
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int j = 0; j < kJ; j += 2)
#pragma unroll
      for (int t = 0; t < 8; ++t) sa = __fmaf_rn(v[j][t], v[j][t], sa);
#pragma unroll
    for (int j = 1; j < kJ; j += 2)
#pragma unroll
      for (int t = 0; t < 8; ++t) sb = __fmaf_rn(v[j][t], v[j][t], sb);
    float sum = __fadd_rn(sa, sb);
#pragma unroll
    for (int o = 8; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(kW)), eps)));
    uint32_t nw[kJ][4];
    uint32_t amax2 = 0;
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const float4* gp = reinterpret_cast<const float4*>(gamma + 8 * (hl + 16 * j));
      const float4 ga = __ldg(gp), gb = __ldg(gp + 1);
      const float gm[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 n2 = mul2(mul2(make_float2(v[j][2 * t], v[j][2 * t + 1]), make_float2(rstd, rstd)),
                               make_float2(gm[2 * t], gm[2 * t + 1]));
        nw[j][t] = pack16x2(n2, F16OUT);
        amax2 = hmax_abs2<F16OUT>(amax2, nw[j][t]);
      }
    }
    // The half's absolute maximum, its scale (quantize_packed_row's rule).
    amax2 &= 0x7fff7fffu;
    const uint32_t m16 = max(amax2 & 0xffffu, amax2 >> 16);
    uint32_t amax = F16OUT ? __float_as_uint(from_f16(static_cast<uint16_t>(m16))) : (m16 << 16);
#pragma unroll
    for (int o = 8; o; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = int8_scale_from_amax(amax);
    const bool bad = amax >= 0x7f800000u;
    if (ok && hl == 0) {
      scales[row] = scale;
      if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
    }
    if (!ok) continue;
    int8_t* dst = q + static_cast<size_t>(row) * kW;
    if (!bad && amax >= 0x00800000u && __float_as_uint(scale) >= 0x00800000u) {
      const float r = __frcp_rn(scale);
#pragma unroll
      for (int j = 0; j < kJ; ++j)
        *reinterpret_cast<uint2*>(dst + 8 * (hl + 16 * j)) = quant_group_fast<F16OUT>(nw[j], scale, r);
    } else {
#pragma unroll
      for (int j = 0; j < kJ; ++j)
        quantize_group_slow(make_uint4(nw[j][0], nw[j][1], nw[j][2], nw[j][3]), F16OUT, scale, bad,
                            dst + 8 * (hl + 16 * j));
    }
  }
}

// The same rows one per warp (lane l holds groups l, l + 32, ...), for small
// row counts (a batch of a few positions), where two rows per warp would halve
// the warps on the critical path; bit-identical to the pair kernel above.
template <bool F16IN, bool F16OUT, int G>
__global__ void __launch_bounds__(256, 3) rms_rows16_row_kernel(
    const uint16_t* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows,
    int8_t* __restrict__ q, float* __restrict__ scales, unsigned* status, unsigned layer) {
  constexpr int kW = 256 * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int step = gridDim.x * 8;
  int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;  // warp-uniform
  uint4 raw[G];
#pragma unroll
  for (int j = 0; j < G; ++j)
    raw[j] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * ldx + 8 * (lane + 32 * j)));
  for (; row < rows; row += step) {
    float v[G][8];
    raw16_to_float<F16IN, G>(raw, v);
    if (row + step < rows) {
      const uint16_t* nxt = x + static_cast<size_t>(row + step) * ldx;
#pragma unroll
      for (int j = 0; j < G; ++j) raw[j] = __ldg(reinterpret_cast<const uint4*>(nxt + 8 * (lane + 32 * j)));
    }
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < G; ++j)
#pragma unroll
      for (int t = 0; t < 8; ++t) sum = __fmaf_rn(v[j][t], v[j][t], sum);
    sum = warp_sum_xor(sum);
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(kW)), eps)));
    uint32_t nw[G][4];
    uint32_t amax2 = 0;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const float4* gp = reinterpret_cast<const float4*>(gamma + 8 * (lane + 32 * j));
      const float4 ga = __ldg(gp), gb = __ldg(gp + 1);
      const float gm[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 n2 = mul2(mul2(make_float2(v[j][2 * t], v[j][2 * t + 1]), make_float2(rstd, rstd)),
                               make_float2(gm[2 * t], gm[2 * t + 1]));
        nw[j][t] = pack16x2(n2, F16OUT);
        amax2 = hmax_abs2<F16OUT>(amax2, nw[j][t]);
      }
    }
    quantize_packed_row<F16OUT, G>(nw, amax2 & 0x7fff7fffu, kW, lane, q + static_cast<size_t>(row) * kW,
                                   scales + row, status, layer);
  }
}

template <int G>
int launch_rms16_full(bool f16in, bool f16out, const uint16_t* x, long ldx, const float* gamma, float eps, int rows,
                      int8_t* q, float* scales, unsigned* status, unsigned layer, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  const bool pair = rows >= kPairRows;
  const auto k = pair ? (f16in ? (f16out ? rms_rows16_full_kernel<true, true, G> : rms_rows16_full_kernel<true, false, G>)
                               : (f16out ? rms_rows16_full_kernel<false, true, G> : rms_rows16_full_kernel<false, false, G>))
                      : (f16in ? (f16out ? rms_rows16_row_kernel<true, true, G> : rms_rows16_row_kernel<true, false, G>)
                               : (f16out ? rms_rows16_row_kernel<false, true, G> : rms_rows16_row_kernel<false, false, G>));
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 256, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
  const int want = pair ? (rows + 15) / 16 : (rows + 7) / 8, cap = per_sm * num_sms(dev);
  k<<<want < cap ? want : cap, 256, 0, s>>>(x, ldx, gamma, eps, rows, q, scales, status, layer);
  return check_cuda(cudaGetLastError(), "rms quantiser launch");
}

template <bool MX, int G>
int launch_rms16(int dtype, const void* x, long ldx, const float* gamma, float eps, int rows, int width, int kp,
                 int blocks4, int bound_f16, void* q, void* scales, unsigned* status, unsigned layer, cudaStream_t s) {
  if constexpr (!MX && G <= 4) {
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx & 7) == 0 &&
                         (reinterpret_cast<uintptr_t>(gamma) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 15) == 0;
    if (width == 256 * G && kp == width && aligned)
      return launch_rms16_full<G>(dtype == kInF16, bound_f16 != 0, static_cast<const uint16_t*>(x), ldx, gamma, eps,
                                  rows, static_cast<int8_t*>(q), static_cast<float*>(scales), status, layer, s);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  // Persistent: as many CTAs as stay resident together, no second wave.
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      &per_sm, dtype == kInF16 ? rms_rows16_kernel<true, MX, G> : rms_rows16_kernel<false, MX, G>, 256, 0);
  if (e != cudaSuccess || per_sm < 1) per_sm = 1;
  const int want = (rows + 7) / 8;
  const int cap = per_sm * num_sms(dev);
  const int grid = want < cap ? want : cap;
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  if (dtype == kInF16)
    rms_rows16_kernel<true, MX, G><<<grid, 256, 0, s>>>(xs, ldx, gamma, eps, rows, width, kp, blocks4, bound_f16, q,
                                                        scales, status, layer);
  else
    rms_rows16_kernel<false, MX, G><<<grid, 256, 0, s>>>(xs, ldx, gamma, eps, rows, width, kp, blocks4, bound_f16, q,
                                                         scales, status, layer);
  return check_cuda(cudaGetLastError(), "rms quantiser launch");
}

// One warp per row; G = groups of 8 per lane (W <= 256 * G).
template <int IN, bool RMS, int G>
__global__ void __launch_bounds__(256) quantize_rows_kernel(
    const void* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows,
    int width, int kp, int bound_f16, int8_t* __restrict__ q, float* __restrict__ scales,
    unsigned* status, unsigned layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= rows) return;  // warp-uniform
  constexpr int kEsize = IN == kInF32 ? 4 : 2;
  const uint8_t* src = static_cast<const uint8_t*>(x) + static_cast<size_t>(row) * ldx * kEsize;
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  if constexpr (!RMS && IN != kInF32) {
    quantize_row16<IN == kInF16, G>(reinterpret_cast<const uint16_t*>(src), vec, width, kp, lane,
                                    q + static_cast<size_t>(row) * kp, scales + row, status, layer);
    return;
  }
  const int groups = (width + 7) / 8;
  float v[G][8];
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int g = lane + 32 * j;
    if (g < groups) {
      load_group<IN>(src, g, width, vec, v[j]);
    } else {
#pragma unroll
      for (int t = 0; t < 8; ++t) v[j][t] = 0.0f;
    }
  }
  if constexpr (RMS) {
    uint32_t nw[G][4];
    uint32_t amax2 = 0;
    rms_normalize<G>(v, gamma, eps, width, lane, bound_f16 != 0, nw, amax2);
    int8_t* dst = q + static_cast<size_t>(row) * kp;
    if (bound_f16)
      quantize_packed_row<true, G>(nw, amax2, kp, lane, dst, scales + row, status, layer);
    else
      quantize_packed_row<false, G>(nw, amax2, kp, lane, dst, scales + row, status, layer);
    return;
  }
  uint32_t amax = 0;
#pragma unroll
  for (int j = 0; j < G; ++j)
#pragma unroll
    for (int t = 0; t < 8; ++t) amax = max(amax, abs_bits(v[j][t]));
  amax = warp_max_u32(amax);
  const float scale = int8_scale_from_amax(amax);
  const bool bad = amax >= 0x7f800000u;
  if (lane == 0) {
    scales[row] = scale;
    if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
  }
  int8_t* dst = q + static_cast<size_t>(row) * kp;
  const int out_groups = kp / 8;
  const bool fast = !bad && amax >= 0x00800000u && __float_as_uint(scale) >= 0x00800000u;
  if (fast) {
    const float r = __frcp_rn(scale);
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j;
      if (g < out_groups) {
        int qi[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) qi[t] = quant_i8_rcp(v[j][t], scale, r);
        *reinterpret_cast<uint2*>(dst + 8 * g) =
            make_uint2(pack4_i8(qi[0], qi[1], qi[2], qi[3]), pack4_i8(qi[4], qi[5], qi[6], qi[7]));
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j;
      if (g < out_groups)
        quantize_group_slow_f32(make_float4(v[j][0], v[j][1], v[j][2], v[j][3]),
                                make_float4(v[j][4], v[j][5], v[j][6], v[j][7]), scale, bad, dst + 8 * g);
    }
  }
}

// fp32 rows of exactly 128*J columns (J <= 4; kp == width; rows, stride and
// gamma 16-byte aligned) through RMSNorm -> 16-bit boundary -> INT8: two rows
// per warp, persistent, the next pair's rows loaded while this pair is
// quantised.  Half-warp h = lane / 16 holds row 2w + h of warp w's pair, lane
// l = lane % 16 the groups l + 16k (k < J), so every lane carries J groups
// (the warp-per-row layout leaves lanes idle whenever 32 does not divide the
// row's groups: at 384 columns lanes 16..31 hold one group, lanes 0..15 two).
// The sum of squares is the warp-per-row layout's, bit for bit: that layout's
// lane l holds groups l, l + 32, ... (even k here) and lane l + 16 groups
// l + 16, l + 48, ... (odd k); each chain runs in group order, then A + B is
// the butterfly's offset-16 step and offsets 8, 4, 2, 1 stay inside the half.
// Normalisation, the row maximum and the quantisation are per element, the
// scale per row, so bytes and scales equal quantize_rows_kernel's.
template <bool F16OUT, int J>
__global__ void __launch_bounds__(256, 2) rms_rows32_pair_kernel(
    const float* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows,
    int8_t* __restrict__ q, float* __restrict__ scales, unsigned* status, unsigned layer) {
  constexpr int kW = 128 * J;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int step = gridDim.x * 16;
  int row0 = (blockIdx.x * 8 + warp) * 2;  // the pair's first row (warp-uniform)
  if (row0 >= rows) return;
  float4 raw[J][2];
  auto load = [&](int r) {
#pragma unroll
    for (int k = 0; k < J; ++k) {
      if (r < rows) {
        const float4* src = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * ldx + 8 * (hl + 16 * k));
        raw[k][0] = __ldg(src);
        raw[k][1] = __ldg(src + 1);
      } else {
        raw[k][0] = raw[k][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
  };
  load(row0 + half);
  for (; row0 < rows; row0 += step) {
    const int row = row0 + half;
    const bool ok = row < rows;
    float v[J][8];
#pragma unroll
    for (int k = 0; k < J; ++k) {
      v[k][0] = raw[k][0].x, v[k][1] = raw[k][0].y, v[k][2] = raw[k][0].z, v[k][3] = raw[k][0].w;
      v[k][4] = raw[k][1].x, v[k][5] = raw[k][1].y, v[k][6] = raw[k][1].z, v[k][7] = raw[k][1].w;
    }
    if (row0 + step < rows) load(row + step);
    float sa = 0.0f, sb = 0.0f;
#pragma unroll
    for (int k = 0; k < J; k += 2)
#pragma unroll
      for (int t = 0; t < 8; ++t) sa = __fmaf_rn(v[k][t], v[k][t], sa);
#pragma unroll
    for (int k = 1; k < J; k += 2)
#pragma unroll
      for (int t = 0; t < 8; ++t) sb = __fmaf_rn(v[k][t], v[k][t], sb);
    float sum = __fadd_rn(sa, sb);
#pragma unroll
    for (int o = 8; o; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(kW)), eps)));
    uint32_t nw[J][4];
    uint32_t amax2 = 0;
#pragma unroll
    for (int k = 0; k < J; ++k) {
      const float4* gp = reinterpret_cast<const float4*>(gamma + 8 * (hl + 16 * k));
      const float4 ga = __ldg(gp), gb = __ldg(gp + 1);
      const float gm[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 n2 = mul2(mul2(make_float2(v[k][2 * t], v[k][2 * t + 1]), make_float2(rstd, rstd)),
                               make_float2(gm[2 * t], gm[2 * t + 1]));
        nw[k][t] = pack16x2(n2, F16OUT);
        amax2 = hmax_abs2<F16OUT>(amax2, nw[k][t]);
      }
    }
    amax2 &= 0x7fff7fffu;
    const uint32_t m16 = max(amax2 & 0xffffu, amax2 >> 16);
    uint32_t amax = F16OUT ? __float_as_uint(from_f16(static_cast<uint16_t>(m16))) : (m16 << 16);
#pragma unroll
    for (int o = 8; o; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = int8_scale_from_amax(amax);
    const bool bad = amax >= 0x7f800000u;
    if (ok && hl == 0) {
      scales[row] = scale;
      if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
    }
    if (!ok) continue;
    int8_t* dst = q + static_cast<size_t>(row) * kW;
    if (!bad && amax >= 0x00800000u && __float_as_uint(scale) >= 0x00800000u) {
      const float r = __frcp_rn(scale);
#pragma unroll
      for (int k = 0; k < J; ++k)
        *reinterpret_cast<uint2*>(dst + 8 * (hl + 16 * k)) = quant_group_fast<F16OUT>(nw[k], scale, r);
    } else {
#pragma unroll
      for (int k = 0; k < J; ++k)
        quantize_group_slow(make_uint4(nw[k][0], nw[k][1], nw[k][2], nw[k][3]), F16OUT, scale, bad,
                            dst + 8 * (hl + 16 * k));
    }
  }
}

template <int J>
int launch_rms32_pair(bool f16out, const float* x, long ldx, const float* gamma, float eps, int rows, int8_t* q,
                      float* scales, unsigned* status, unsigned layer, cudaStream_t s) {
  int dev = 0;
  cudaGetDevice(&dev);
  const auto k = f16out ? rms_rows32_pair_kernel<true, J> : rms_rows32_pair_kernel<false, J>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 256, 0) != cudaSuccess || per_sm < 1) per_sm = 1;
  const int want = (rows + 15) / 16, cap = per_sm * num_sms(dev);  // two rows per warp
  k<<<want < cap ? want : cap, 256, 0, s>>>(x, ldx, gamma, eps, rows, q, scales, status, layer);
  return check_cuda(cudaGetLastError(), "rms quantiser launch");
}

template <int IN, bool RMS, int G>
int launch_g(const void* x, long ldx, const float* gamma, float eps, int rows, int width, int kp,
             int bound_f16, int8_t* q, float* scales, unsigned* status, unsigned layer, cudaStream_t s) {
  if constexpr (RMS && IN != kInF32)
    return launch_rms16<false, G>(IN, x, ldx, gamma, eps, rows, width, kp, 0, bound_f16, q, scales, status, layer, s);
  if constexpr (RMS && IN == kInF32 && G <= 2) {
    // full fp32 rows of 128, 256, 384 or 512 columns: the two-rows-per-warp kernel
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx & 3) == 0 &&
                         (reinterpret_cast<uintptr_t>(gamma) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 7) == 0;
    if (aligned && kp == width && width % 128 == 0 && rows >= kPairRows) {
      const float* xf = static_cast<const float*>(x);
      switch (width / 128) {
        case 1: return launch_rms32_pair<1>(bound_f16 != 0, xf, ldx, gamma, eps, rows, q, scales, status, layer, s);
        case 2: return launch_rms32_pair<2>(bound_f16 != 0, xf, ldx, gamma, eps, rows, q, scales, status, layer, s);
        case 3: return launch_rms32_pair<3>(bound_f16 != 0, xf, ldx, gamma, eps, rows, q, scales, status, layer, s);
        case 4: return launch_rms32_pair<4>(bound_f16 != 0, xf, ldx, gamma, eps, rows, q, scales, status, layer, s);
        default: break;
      }
    }
  }
  quantize_rows_kernel<IN, RMS, G><<<(rows + 7) / 8, 256, 0, s>>>(x, ldx, gamma, eps, rows, width, kp,
                                                                  bound_f16, q, scales, status, layer);
  return check_cuda(cudaGetLastError(), "quantiser launch");
}

template <int IN, bool RMS>
int launch_quant(const void* x, long ldx, const float* gamma, float eps, int rows, int width, int kp,
                 int bound_f16, int8_t* q, float* scales, unsigned* status, unsigned layer,
                 cudaStream_t s) {
  const int need = (kp + 255) / 256;  // groups of 8 per lane covering the padded row
#define KB_Q(GG) \
  if (need <= GG) return launch_g<IN, RMS, GG>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q, scales, status, layer, s)
  KB_Q(1);
  KB_Q(2);
  KB_Q(3);
  KB_Q(4);
  KB_Q(6);
  KB_Q(8);
  KB_Q(12);
  KB_Q(16);
#undef KB_Q
  set_error("quantiser row width above 4096 is not supported");
  return KB_E_INVALID;
}

// Streaming quantiser for rows whose absolute maximum was already produced by
// the kernel that wrote them (the GEMM / attention epilogue's row_amax): no row
// reduction.  Same scale and rounding as quantize_row16 (bit-identical results).

// One warp per row, persistent over rows: lane l loads the groups l, l+32, ...
// of the row (all G 16-byte loads issued before any is used, so a warp keeps
// G x 512 bytes in flight), the scale and its reciprocal are computed once per
// row, and 8-byte stores leave the int8 groups.
template <bool F16, int G>
__global__ void __launch_bounds__(256) quantize_rows_amax_kernel(
    const uint16_t* __restrict__ x, long ldx, const uint32_t* __restrict__ row_amax, int rows, int width,
    int kp, int8_t* __restrict__ q, float* __restrict__ scales, unsigned* status, unsigned layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int out_groups = kp / 8;
  const int step = gridDim.x * 8;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += step) {  // warp-uniform
    const uint16_t* src = x + static_cast<size_t>(row) * ldx;
    uint32_t w[G][4];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int c0 = 8 * (lane + 32 * j);
      w[j][0] = w[j][1] = w[j][2] = w[j][3] = 0;
      if (c0 + 8 <= width) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(src + c0));
        w[j][0] = a.x; w[j][1] = a.y; w[j][2] = a.z; w[j][3] = a.w;
      } else if (c0 < width) {
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (c0 + t < width) w[j][t / 2] |= static_cast<uint32_t>(src[c0 + t]) << (16 * (t & 1));
      }
    }
    const uint32_t amax = __ldg(row_amax + row);
    const float scale = int8_scale_from_amax(amax);
    const bool bad = amax >= 0x7f800000u;
    if (lane == 0) {
      scales[row] = scale;
      if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
    }
    int8_t* dst = q + static_cast<size_t>(row) * kp;
    if (!bad && amax >= 0x00800000u && __float_as_uint(scale) >= 0x00800000u) {
      const float r = __frcp_rn(scale);
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const int g = lane + 32 * j;
        if (g < out_groups) *reinterpret_cast<uint2*>(dst + 8 * g) = quant_group_fast<F16>(w[j], scale, r);
      }
    } else {
#pragma unroll
      for (int j = 0; j < G; ++j) {
        const int g = lane + 32 * j;
        if (g < out_groups)
          quantize_group_slow(make_uint4(w[j][0], w[j][1], w[j][2], w[j][3]), F16, scale, bad, dst + 8 * g);
      }
    }
  }
}

// Rows of exactly 128*J columns (J <= 3 or 9, kp == width) from kPairRows rows
// on, two rows per warp: half-warp h holds row 2w + h, lane l = lane % 16 the
// groups l + 16k (k < J).  At 384 columns every lane then carries three
// groups, where one row per warp leaves lanes 16..31 with one and lanes 0..15
// with two; at 1152 (the TF3 SwiGLU hidden) nine, instead of five and four.  Per element the same quantisation as quantize_rows_amax_kernel,
// the scale once per row (no reduction: the producer supplied the maximum).
template <bool F16, int J>
__global__ void __launch_bounds__(256) quantize_rows_amax_pair_kernel(
    const uint16_t* __restrict__ x, long ldx, const uint32_t* __restrict__ row_amax, int rows,
    int8_t* __restrict__ q, float* __restrict__ scales, unsigned* status, unsigned layer) {
  constexpr int kW = 128 * J;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int step = gridDim.x * 16;
  for (int row = (blockIdx.x * 8 + warp) * 2 + half; row - half < rows; row += step) {
    if (row >= rows) continue;  // the halves never exchange data
    const uint16_t* src = x + static_cast<size_t>(row) * ldx;
    uint32_t w[J][4];
#pragma unroll
    for (int k = 0; k < J; ++k) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(src + 8 * (hl + 16 * k)));
      w[k][0] = a.x; w[k][1] = a.y; w[k][2] = a.z; w[k][3] = a.w;
    }
    const uint32_t amax = __ldg(row_amax + row);
    const float scale = int8_scale_from_amax(amax);
    const bool bad = amax >= 0x7f800000u;
    if (hl == 0) {
      scales[row] = scale;
      if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
    }
    int8_t* dst = q + static_cast<size_t>(row) * kW;
    if (!bad && amax >= 0x00800000u && __float_as_uint(scale) >= 0x00800000u) {
      const float r = __frcp_rn(scale);
#pragma unroll
      for (int k = 0; k < J; ++k)
        *reinterpret_cast<uint2*>(dst + 8 * (hl + 16 * k)) = quant_group_fast<F16>(w[k], scale, r);
    } else {
#pragma unroll
      for (int k = 0; k < J; ++k)
        quantize_group_slow(make_uint4(w[k][0], w[k][1], w[k][2], w[k][3]), F16, scale, bad, dst + 8 * (hl + 16 * k));
    }
  }
}

template <bool F16, int J>
int launch_amax_pair(const void* x, long ldx, const uint32_t* row_amax, int rows, int8_t* q, float* scales,
                     unsigned* status, unsigned layer, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_rows_amax_pair_kernel<F16, J>, 256, 0) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int want = (rows + 15) / 16;
  const int cap = per_sm * num_sms(dev);
  quantize_rows_amax_pair_kernel<F16, J><<<want < cap ? want : cap, 256, 0, stream>>>(
      static_cast<const uint16_t*>(x), ldx, row_amax, rows, q, scales, status, layer);
  return check_cuda(cudaGetLastError(), "amax quantiser launch");
}

template <bool F16, int G>
int launch_amax(const void* x, long ldx, const uint32_t* row_amax, int rows, int width, int kp, int8_t* q,
                float* scales, unsigned* status, unsigned layer, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_rows_amax_kernel<F16, G>, 256, 0) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const int want = (rows + 7) / 8;
  const int cap = per_sm * num_sms(dev);
  quantize_rows_amax_kernel<F16, G><<<want < cap ? want : cap, 256, 0, stream>>>(
      static_cast<const uint16_t*>(x), ldx, row_amax, rows, width, kp, q, scales, status, layer);
  return check_cuda(cudaGetLastError(), "amax quantiser launch");
}

}  // namespace

// RMSNorm of 16-bit rows to 16-bit rows, the input of an unquantised (bf16)
// projection: out = T16((x * rstd) * gamma), the same values the fused RMS
// quantisers quantise (rms_normalize); a non-finite row sets the status word
// as the quantisers do.  Persistent warp per row.
template <bool F16IN, int G>
__global__ void __launch_bounds__(256) rms_rows16_out16_kernel(
    const uint16_t* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows, int width,
    int bound_f16, uint16_t* __restrict__ out, long ldo, unsigned* status, unsigned layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (width + 7) / 8;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    uint4 raw[G];
    load_raw16<G>(x + static_cast<size_t>(row) * ldx, width, lane, raw);
    float v[G][8];
    raw16_to_float<F16IN, G>(raw, v);
    uint32_t nw[G][4];
    uint32_t amax2;
    rms_normalize<G>(v, gamma, eps, width, lane, bound_f16 != 0, nw, amax2);
    const uint32_t m16 = warp_max_u32(max(amax2 & 0xffffu, amax2 >> 16));
    const uint32_t inf16 = bound_f16 ? 0x7c00u : 0x7f80u;
    if (lane == 0 && m16 >= inf16) record_status(status, m16 > inf16 ? KB_STATUS_NAN : KB_STATUS_INF, layer);
    uint16_t* dst = out + static_cast<size_t>(row) * ldo;
    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j, c0 = 8 * g;
      if (g >= groups) continue;
      if (vec && c0 + 8 <= width) {
        *reinterpret_cast<uint4*>(dst + c0) = make_uint4(nw[j][0], nw[j][1], nw[j][2], nw[j][3]);
      } else {
        for (int t = 0; t < 8 && c0 + t < width; ++t)
          dst[c0 + t] = static_cast<uint16_t>((t & 1) ? nw[j][t / 2] >> 16 : nw[j][t / 2] & 0xffffu);
      }
    }
  }
}

// The same for fp32 rows (the nested trunk's fp32 inner stream, the input of
// an unquantised attention projection).
template <int G>
__global__ void __launch_bounds__(256) rms_rows32_out16_kernel(
    const float* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows, int width,
    int bound_f16, uint16_t* __restrict__ out, long ldo, unsigned* status, unsigned layer) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (width + 7) / 8;
  for (int row = blockIdx.x * 8 + warp; row < rows; row += gridDim.x * 8) {
    const float* src = x + static_cast<size_t>(row) * ldx;
    const bool vin = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    float v[G][8];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j;
      if (g < groups) {
        load_group<kInF32>(src, g, width, vin, v[j]);
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) v[j][t] = 0.0f;
      }
    }
    uint32_t nw[G][4];
    uint32_t amax2;
    rms_normalize<G>(v, gamma, eps, width, lane, bound_f16 != 0, nw, amax2);
    const uint32_t m16 = warp_max_u32(max(amax2 & 0xffffu, amax2 >> 16));
    const uint32_t inf16 = bound_f16 ? 0x7c00u : 0x7f80u;
    if (lane == 0 && m16 >= inf16) record_status(status, m16 > inf16 ? KB_STATUS_NAN : KB_STATUS_INF, layer);
    uint16_t* dst = out + static_cast<size_t>(row) * ldo;
    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int g = lane + 32 * j, c0 = 8 * g;
      if (g >= groups) continue;
      if (vec && c0 + 8 <= width) {
        *reinterpret_cast<uint4*>(dst + c0) = make_uint4(nw[j][0], nw[j][1], nw[j][2], nw[j][3]);
      } else {
        for (int t = 0; t < 8 && c0 + t < width; ++t)
          dst[c0 + t] = static_cast<uint16_t>((t & 1) ? nw[j][t / 2] >> 16 : nw[j][t / 2] & 0xffffu);
      }
    }
  }
}

// Fused RMSNorm -> 16-bit -> MXFP8 over rows of `width` (<= 4096) columns.
int rms_mxfp8_launch(const void* x, int dtype, long ldx, int rows, int width, const float* gamma, float eps,
                     int bound_f16, uint8_t* q, uint8_t* scales, unsigned* status, unsigned layer,
                     cudaStream_t stream) {
  int kp = 0, blocks4 = 0;
  int rc = mxfp8_dims(rows, width, &kp, &blocks4, nullptr, nullptr);
  if (rc) return rc;
  if (width > 4096 || ldx < width || gamma == nullptr || !(eps > 0.0f) ||
      (reinterpret_cast<uintptr_t>(q) & 15) != 0) {
    set_error("RMS MXFP8 quantiser: width <= 4096, stride >= width, gamma, eps > 0, 16-byte aligned output");
    return KB_E_INVALID;
  }
  const int need = (kp + 255) / 256;
  const int grid = (rows + 7) / 8;
#define KB_MXQ(IN, GG)                                                                                         \
  if (need <= GG) {                                                                                            \
    if (IN != kInF32)                                                                                          \
      return launch_rms16<true, GG>(IN, x, ldx, gamma, eps, rows, width, kp, blocks4, bound_f16, q, scales,     \
                                    status, layer, stream);                                                    \
    rms_mxfp8_kernel<IN, GG><<<grid, 256, 0, stream>>>(x, ldx, gamma, eps, rows, width, kp, blocks4, bound_f16, \
                                                        q, scales, status, layer);                             \
    return check_cuda(cudaGetLastError(), "rms mxfp8 launch");                                                  \
  }
#define KB_MXQ_ALL(IN) \
  KB_MXQ(IN, 1) KB_MXQ(IN, 2) KB_MXQ(IN, 3) KB_MXQ(IN, 4) KB_MXQ(IN, 6) KB_MXQ(IN, 8) KB_MXQ(IN, 12) KB_MXQ(IN, 16)
  switch (dtype) {
    case kInF32: KB_MXQ_ALL(kInF32) break;
    case kInF16: KB_MXQ_ALL(kInF16) break;
    case kInBF16: KB_MXQ_ALL(kInBF16) break;
    default: set_error("unknown activation dtype"); return KB_E_INVALID;
  }
#undef KB_MXQ_ALL
#undef KB_MXQ
  set_error("RMS MXFP8 quantiser width above 4096 is not supported");
  return KB_E_INVALID;
}

// Quantise 16-bit rows given their |value| bit maximum (row_amax, [rows]).
// Row starts must be 16-byte aligned (ldx % 8 == 0).
int quantize_rows_amax_launch(const void* x, int dtype, long ldx, const uint32_t* row_amax, int rows, int width,
                              int kp, int8_t* q, float* scales, unsigned* status, unsigned layer,
                              cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || kp < width || kp % 16 != 0 || ldx < width || ldx % 8 != 0 ||
      (dtype != kInF16 && dtype != kInBF16) || row_amax == nullptr ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q) & 15)) {
    set_error("amax quantiser: need 16-bit rows with 16-byte aligned starts, kp % 16 == 0, and row_amax");
    return KB_E_INVALID;
  }
  if (kp > 4096) {
    set_error("amax quantiser: padded width above 4096 is not supported");
    return KB_E_INVALID;
  }
  const int need = (kp / 8 + 31) / 32;  // 16-byte groups per lane
  const bool f16 = dtype == kInF16;
  if (rows >= kPairRows && kp == width && width % 128 == 0 && (width <= 384 || width == 1152)) {
#define KB_AP(JJ)                                                                                              \
  if (width == 128 * JJ)                                                                                       \
    return f16 ? launch_amax_pair<true, JJ>(x, ldx, row_amax, rows, q, scales, status, layer, stream)          \
               : launch_amax_pair<false, JJ>(x, ldx, row_amax, rows, q, scales, status, layer, stream);
    KB_AP(1) KB_AP(2) KB_AP(3) KB_AP(9)
#undef KB_AP
  }
#define KB_AQ(GG)                                                                                          \
  if (need <= GG)                                                                                          \
    return f16 ? launch_amax<true, GG>(x, ldx, row_amax, rows, width, kp, q, scales, status, layer, stream) \
               : launch_amax<false, GG>(x, ldx, row_amax, rows, width, kp, q, scales, status, layer, stream);
  KB_AQ(1) KB_AQ(2) KB_AQ(3) KB_AQ(4) KB_AQ(6) KB_AQ(8) KB_AQ(12) KB_AQ(16)
#undef KB_AQ
  set_error("amax quantiser: unsupported width");
  return KB_E_INVALID;
}

// dtype: 0 = f32, 1 = f16, 2 = bf16.  rms: apply RMSNorm with gamma/eps and a
// 16-bit boundary (bound_f16: 1 = fp16, 0 = bf16) before quantising.
int quantize_rows_launch(const void* x, int dtype, long ldx, int rows, int width, int kp, bool rms,
                         const float* gamma, float eps, int bound_f16, int8_t* q, float* scales,
                         unsigned* status, unsigned layer, cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || kp < width || kp % 16 != 0 || kp > 4096 || ldx < width) {
    set_error("quantiser shape mismatch (rows, width, padded width <= 4096, stride)");
    return KB_E_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(q) & 15) != 0) {
    set_error("quantised output must be 16-byte aligned");
    return KB_E_INVALID;
  }
  if (rms && (gamma == nullptr || !(eps > 0.0f) || eps != eps)) {
    set_error("RMS quantiser needs gamma and a positive finite epsilon");
    return KB_E_INVALID;
  }
  switch (dtype) {
    case kInF32:
      return rms ? launch_quant<kInF32, true>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q,
                                              scales, status, layer, stream)
                 : launch_quant<kInF32, false>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q,
                                               scales, status, layer, stream);
    case kInF16:
      return rms ? launch_quant<kInF16, true>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q,
                                              scales, status, layer, stream)
                 : launch_quant<kInF16, false>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q,
                                               scales, status, layer, stream);
    case kInBF16:
      return rms ? launch_quant<kInBF16, true>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q,
                                               scales, status, layer, stream)
                 : launch_quant<kInBF16, false>(x, ldx, gamma, eps, rows, width, kp, bound_f16, q,
                                                scales, status, layer, stream);
  }
  set_error("unknown activation dtype");
  return KB_E_INVALID;
}


int rms16_rows_launch(const void* x, int dtype, long ldx, int rows, int width, const float* gamma, float eps,
                      int bound_f16, uint16_t* out, long ldo, unsigned* status, unsigned layer, cudaStream_t s) {
  if ((dtype != kInF16 && dtype != kInBF16 && dtype != kInF32) || width <= 0 || width > 4096 || ldx < width ||
      ldo < width || gamma == nullptr || !(eps > 0.0f)) {
    set_error("RMS to 16-bit rows: fp32 or 16-bit input, width <= 4096, strides >= width, gamma, eps > 0");
    return KB_E_INVALID;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  const int want = (rows + 7) / 8, cap = 8 * num_sms(dev);
  const int grid = want < cap ? want : cap;
  const uint16_t* xs = static_cast<const uint16_t*>(x);
  const int need = (width + 255) / 256;
  if (dtype == kInF32) {
#define KB_R32(GG)                                                                                            \
  if (need <= GG) {                                                                                           \
    rms_rows32_out16_kernel<GG><<<grid, 256, 0, s>>>(static_cast<const float*>(x), ldx, gamma, eps, rows, width, \
                                                     bound_f16, out, ldo, status, layer);                       \
    return check_cuda(cudaGetLastError(), "rms fp32 to 16-bit launch");                                       \
  }
    KB_R32(1) KB_R32(2) KB_R32(4) KB_R32(8) KB_R32(16)
#undef KB_R32
  }
#define KB_R16(GG)                                                                                          \
  if (need <= GG) {                                                                                         \
    if (dtype == kInF16)                                                                                    \
      rms_rows16_out16_kernel<true, GG><<<grid, 256, 0, s>>>(xs, ldx, gamma, eps, rows, width, bound_f16, out, \
                                                             ldo, status, layer);                             \
    else                                                                                                    \
      rms_rows16_out16_kernel<false, GG><<<grid, 256, 0, s>>>(xs, ldx, gamma, eps, rows, width, bound_f16, out, \
                                                              ldo, status, layer);                            \
    return check_cuda(cudaGetLastError(), "rms 16-bit launch");                                             \
  }
  KB_R16(1) KB_R16(2) KB_R16(3) KB_R16(4) KB_R16(6) KB_R16(8) KB_R16(12) KB_R16(16)
#undef KB_R16
  return KB_E_INVALID;
}

}  // namespace kb
