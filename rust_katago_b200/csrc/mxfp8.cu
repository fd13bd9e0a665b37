// MXFP8 block-32 quantiser: fp32 / fp16 / bf16 rows -> E4M3 bytes [rows, kp]
// plus UE8M0 scales in the packed 128-row x 4-block tile layout that the
// tcgen05 block-scaled GEMM copies straight into tensor memory.
//
// Replaces the reference's mxfp8_quantize_{half,float}_kernel and
// mxfp8_clear_scales_kernel (Rust_KataGo crates/kata_nn/cuda-kernels/mxfp8.cu:36-149,
// launched by Mxfp8Kernels::quantize, src/backends/mxfp8.rs:209-270).  The
// reference runs one 32-thread CTA per (row, block); here one thread owns 8
// consecutive elements (a 16-byte load for 16-bit inputs), four threads form a
// block and reduce its amax with two shuffles, and a grid-stride loop walks the
// padded [rows_pad128, blocks4] rectangle so every padding scale byte is
// written (zero) by the same launch.
#include <stdint.h>

#include <string>

#include "../../include/katab200.h"
#include "kb_internal.h"
#include "kb_mxfp8.cuh"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

// Eight values of a row as floats; for 16-bit input also the raw packed
// pairs (zero past k).
template <int IN>
__device__ __forceinline__ void load8(const void* src, long ld, int row, int col0, int k, bool vec,
                                      float (&v)[8], uint32_t (&raw)[4]) {
  if constexpr (IN == KB_DT_F32) {
    const float* p = static_cast<const float*>(src) + static_cast<size_t>(row) * ld + col0;
    if (vec) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p));
      const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = col0 + i < k ? __ldg(p + i) : 0.0f;
    }
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(src) + static_cast<size_t>(row) * ld + col0;
    constexpr bool f16 = IN == KB_DT_F16;
    if (vec) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
      raw[0] = w.x, raw[1] = w.y, raw[2] = w.z, raw[3] = w.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = col0 + 2 * i < k ? __ldg(p + 2 * i) : 0u;
        const uint32_t hi = col0 + 2 * i + 1 < k ? __ldg(p + 2 * i + 1) : 0u;
        raw[i] = lo | (hi << 16);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = from16(static_cast<uint16_t>(raw[i] & 0xffffu), f16);
      v[2 * i + 1] = from16(static_cast<uint16_t>(raw[i] >> 16), f16);
    }
  }
}

template <int IN, bool CHECK_WEIGHT>
__global__ void __launch_bounds__(256)
    mxfp8_quantize_kernel(const void* __restrict__ src, long ld, int rows, int k, int kp, int blocks4,
                          int rows_pad, int vec, uint8_t* __restrict__ q, uint8_t* __restrict__ scales,
                          unsigned* status, unsigned layer, FastDiv per_row) {
  // per_row.d = 8-element groups per padded row; rows_pad * per_row.d < 2^31
  const uint32_t total = static_cast<uint32_t>(rows_pad) * per_row.d;
  const int lane = threadIdx.x & 31;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t warps = (gridDim.x * blockDim.x) >> 5;
  const int nblocks = kp >> 5;
  // Warp-uniform trip count: the quad shuffles below need all 32 lanes.
  for (uint32_t base = warp * 32; base < total; base += warps * 32) {
    const uint32_t gi = base + lane;
    const bool active = gi < total;
    const int row = active ? static_cast<int>(per_row.div(gi)) : 0;
    const int grp = active ? static_cast<int>(gi - static_cast<uint32_t>(row) * per_row.d) : 0;
    const int blk = grp >> 2;
    const int col0 = grp * 8;
    const bool live = active && row < rows && blk < nblocks;
    float v[8];
    uint32_t raw[4] = {0u, 0u, 0u, 0u};
    if (live && col0 < k) {
      load8<IN>(src, ld, row, col0, k, vec != 0, v, raw);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    unsigned bad = 0;
    float a = 0.0f;
    // Non-finite values are flagged and zeroed; a = the largest finite |v|.
    auto classify = [&]() {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t mag = __float_as_uint(v[i]) & 0x7fffffffu;
        if (mag >= 0x7f800000u) {
          bad |= mag > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF;
          v[i] = 0.0f;
        }
        a = fmaxf(a, fabsf(v[i]));
      }
    };
    if constexpr (IN == KB_DT_F32) {
      classify();
    } else {
      // 16-bit input: the group's |max| from the packed pairs (one
      // max.NaN.abs per pair; NaN wins), the per-value pass only for a
      // group holding a NaN or an infinity.
      constexpr bool f16 = IN == KB_DT_F16;
      constexpr uint32_t inf16 = f16 ? 0x7c00u : 0x7f80u;
      uint32_t m2 = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) m2 = hmax_abs2<f16>(m2, raw[i]);
      const uint32_t m16 = max(m2 & 0x7fffu, (m2 >> 16) & 0x7fffu);
      if (m16 >= inf16)
        classify();
      else
        a = from16(static_cast<uint16_t>(m16), f16);
    }
    if (bad) record_status(status, bad, layer);
    unsigned any_bad = bad;
    any_bad |= __shfl_xor_sync(0xffffffffu, any_bad, 1);
    any_bad |= __shfl_xor_sync(0xffffffffu, any_bad, 2);
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    const bool zero = a == 0.0f || any_bad != 0;
    const uint32_t scale = zero ? 127u : ue8m0_ceil(__fdiv_rn(a, 448.0f));
    const float rcp = ue8m0_reciprocal(scale);
    uint32_t w0 = 0, w1 = 0;
    if (!zero) {
      // (packed products feed only the conversions: nothing to contract)
      float2 sv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) sv[i] = mul2(make_float2(v[2 * i], v[2 * i + 1]), make_float2(rcp, rcp));
      w0 = e4m3x2(sv[0].x, sv[0].y) | (e4m3x2(sv[1].x, sv[1].y) << 16);
      w1 = e4m3x2(sv[2].x, sv[2].y) | (e4m3x2(sv[3].x, sv[3].y) << 16);
    }
    if constexpr (CHECK_WEIGHT) {
      // Static weights must decode to finite fp32 values (mxfp8.cu:62-65):
      // |q| * 2^(scale - 127) must stay below 2^128.  The product of a 4-bit
      // significand and a power of two is exact unless it overflows.
      if (live && !zero) {
        const float p2 = scale == 0 ? __uint_as_float(0x00400000u) : __uint_as_float(scale << 23);
        bool over = false;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t c = ((i < 4 ? w0 : w1) >> (8 * (i & 3))) & 0x7fu;
          over |= isinf(__fmul_rn(e4m3_magnitude(c), p2));
        }
        if (over) record_status(status, KB_STATUS_WEIGHT_OVERFLOW, layer);
      }
    }
    if (live) *reinterpret_cast<uint2*>(q + static_cast<size_t>(row) * kp + col0) = make_uint2(w0, w1);
    if (active && (grp & 3) == 0) scales[mx_scale_offset(row, blk, blocks4)] = live ? static_cast<uint8_t>(scale) : 0;
  }
}

template <int IN>
int launch(const void* x, long ld, int rows, int k, int kp, int blocks4, int rows_pad, int vec, bool check_weight,
           uint8_t* q, uint8_t* scales, unsigned* status, unsigned layer, cudaStream_t stream) {
  const long total = static_cast<long>(rows_pad) * blocks4 * 4;
  if (total >= (1L << 31)) {
    set_error("mxfp8 quantiser: rows x padded width / 8 must be below 2^31");
    return KB_E_INVALID;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  const long want = (total + 255) / 256;
  const int grid = static_cast<int>(want < 8L * num_sms(dev) ? want : 8L * num_sms(dev));
  const FastDiv per_row(static_cast<uint32_t>(blocks4) * 4u);
  if (check_weight)
    mxfp8_quantize_kernel<IN, true><<<grid, 256, 0, stream>>>(x, ld, rows, k, kp, blocks4, rows_pad, vec, q,
                                                               scales, status, layer, per_row);
  else
    mxfp8_quantize_kernel<IN, false><<<grid, 256, 0, stream>>>(x, ld, rows, k, kp, blocks4, rows_pad, vec, q,
                                                                scales, status, layer, per_row);
  return check_cuda(cudaGetLastError(), "mxfp8 quantiser launch");
}

}  // namespace

int mxfp8_dims(long rows, long k, int* kp, int* blocks4, size_t* data_bytes, size_t* scale_bytes) {
  if (rows <= 0 || rows > 0x7fffffffL || k <= 0 || k > kMxfp8MaxK) {
    set_error("invalid MXFP8 dimensions rows=" + std::to_string(rows) + " K=" + std::to_string(k) +
              "; K must be 1..=" + std::to_string(kMxfp8MaxK));
    return KB_E_INVALID;
  }
  const long p = (k + 31) / 32 * 32;
  const long b4 = (p / 32 + 3) / 4 * 4;
  const unsigned long long data = static_cast<unsigned long long>(rows) * p;
  const unsigned long long sc = static_cast<unsigned long long>((rows + 127) / 128 * 128) * b4;
  if (data > 0xffffffffull || sc > 0xffffffffull) {
    set_error("MXFP8 data or scale size exceeds the 32-bit indexing limit");
    return KB_E_INVALID;
  }
  if (kp) *kp = static_cast<int>(p);
  if (blocks4) *blocks4 = static_cast<int>(b4);
  if (data_bytes) *data_bytes = static_cast<size_t>(data);
  if (scale_bytes) *scale_bytes = static_cast<size_t>(sc);
  return KB_OK;
}

int mxfp8_quantize_launch(const void* x, int dtype, long ld, int rows, int k, uint8_t* q, uint8_t* scales,
                          size_t scale_capacity, bool check_weight, unsigned* status, unsigned layer,
                          cudaStream_t stream) {
  int kp = 0, blocks4 = 0;
  size_t data_bytes = 0, scale_bytes = 0;
  int rc = mxfp8_dims(rows, k, &kp, &blocks4, &data_bytes, &scale_bytes);
  if (rc) return rc;
  if (x == nullptr || q == nullptr || scales == nullptr) {
    set_error("MXFP8 quantiser pointers must be non-null");
    return KB_E_INVALID;
  }
  if (ld < k) {
    set_error("MXFP8 input stride is smaller than K");
    return KB_E_INVALID;
  }
  if (scale_capacity < scale_bytes) {
    set_error("MXFP8 scale buffer holds " + std::to_string(scale_capacity) + " bytes, the shape needs " +
              std::to_string(scale_bytes));
    return KB_E_INVALID;
  }
  if (reinterpret_cast<uintptr_t>(q) & 15) {
    set_error("MXFP8 quantised output must be 16-byte aligned");
    return KB_E_INVALID;
  }
  const int elem = dtype == KB_DT_F32 ? 4 : 2;
  const int vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ld * elem) % 16 == 0 && k % 8 == 0;
  // Clear the scale capacity beyond this shape (a workspace may switch K
  // between projections; the reference clears its whole scale allocation).
  if (scale_capacity > scale_bytes) {
    rc = check_cuda(cudaMemsetAsync(scales + scale_bytes, 0, scale_capacity - scale_bytes, stream),
                    "mxfp8 scale tail clear");
    if (rc) return rc;
  }
  const int rows_pad = (rows + 127) / 128 * 128;
  switch (dtype) {
    case KB_DT_F32:
      return launch<KB_DT_F32>(x, ld, rows, k, kp, blocks4, rows_pad, vec, check_weight, q, scales, status, layer,
                               stream);
    case KB_DT_F16:
      return launch<KB_DT_F16>(x, ld, rows, k, kp, blocks4, rows_pad, vec, check_weight, q, scales, status, layer,
                               stream);
    case KB_DT_BF16:
      return launch<KB_DT_BF16>(x, ld, rows, k, kp, blocks4, rows_pad, vec, check_weight, q, scales, status, layer,
                                stream);
  }
  set_error("unknown MXFP8 input dtype");
  return KB_E_INVALID;
}

}  // namespace kb
