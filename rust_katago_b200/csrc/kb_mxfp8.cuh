// MXFP8 (OCP microscaling, E4M3 elements + UE8M0 scale per 32 K) device helpers.
//
// Semantics follow the reference's block-32 quantiser
// (Rust_KataGo crates/kata_nn/cuda-kernels/mxfp8.cu:36-79):
//   amax  = max |x| over the block (non-finite elements zeroed, block flagged)
//   scale = 127 for an all-zero or flagged block, else the UE8M0 byte of the
//           smallest power of two >= fp32(amax / 448) (round toward +inf,
//           saturating at 2^127)
//   q     = E4M3(x * 2^(127 - scale)), round to nearest even, saturating at 448.
#pragma once

#include <stdint.h>

namespace kb {

// UE8M0 byte of the smallest power of two >= r, for finite r > 0, saturating
// at 254 (2^127).  From the fp32 fields: a normal r = 2^(E-127) * 1.M is a power
// of two iff M == 0; a subnormal r < 2^-126 rounds up to 2^-127 (byte 0) when
// r <= 2^-127 (mantissa <= 2^22), else to 2^-126 (byte 1).
__device__ __forceinline__ uint32_t ue8m0_ceil(float r) {
  const uint32_t b = __float_as_uint(r);
  const uint32_t e = (b >> 23) & 0xffu;
  const uint32_t m = b & 0x7fffffu;
  uint32_t s;
  if (e == 0) {
    s = m <= 0x400000u ? 0u : 1u;
  } else {
    s = e + (m != 0 ? 1u : 0u);
  }
  return s > 254u ? 254u : s;
}

// 2^(127 - scale) as an fp32 value for scale in [0, 254]; 2^-127 is subnormal.
__device__ __forceinline__ float ue8m0_reciprocal(uint32_t scale) {
  const int e = 254 - static_cast<int>(scale);  // biased exponent of 2^(127-scale)
  return e >= 1 ? __uint_as_float(static_cast<uint32_t>(e) << 23) : __uint_as_float(0x00400000u);
}

// Two fp32 values -> two E4M3 bytes (lo in bits 0-7, hi in bits 8-15), round to
// nearest even, saturating to +-448 (hardware conversion).
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// |value| of a finite E4M3 byte as fp32 (exact).
__device__ __forceinline__ float e4m3_magnitude(uint32_t code) {
  const uint32_t e = (code >> 3) & 15u, m = code & 7u;
  // e == 0: m * 2^-9;  else (8 + m) * 2^(e - 10).
  const float mant = static_cast<float>(e == 0 ? m : 8u + m);
  const uint32_t pe = e == 0 ? 118u : 117u + e;  // biased exponent of 2^-9 or 2^(e-10)
  return __fmul_rn(mant, __uint_as_float(pe << 23));
}

// Byte offset of (row, block) in the packed scale layout: 512-byte tiles of
// 128 rows x 4 K blocks, inside a tile (row % 32) * 16 + (row % 128 / 32) * 4 +
// block % 4 (mxfp8.cu:75-77).  This is also the tcgen05 scale-factor layout:
// one tile is one 32-lane x 128-bit tcgen05.cp source.
__device__ __forceinline__ size_t mx_scale_offset(int row, int block, int blocks4) {
  return (static_cast<size_t>(row >> 7) * static_cast<size_t>(blocks4 >> 2) + static_cast<size_t>(block >> 2)) * 512u +
         static_cast<size_t>((row & 31) * 16 + ((row & 127) >> 5) * 4 + (block & 3));
}

}  // namespace kb
