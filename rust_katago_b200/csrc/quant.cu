// Per-token dynamic INT8 activation quantisers.
//
// Replaces the reference's row quantisers and its fused RMSNorm quantiser
// (crates/kata_nn/cuda-kernels/int8_ops.cu:8-89, :140-176).  One warp owns one
// token row; four rows per 128-thread CTA.  The row is brought into shared
// memory with 16-byte vector loads, then every arithmetic step follows the
// reference's order exactly:
//   * RMS: lane-strided partial sums sum = fma(x, x, sum) over columns
//     lane, lane+32, ... then an xor butterfly over 16, 8, 4, 2, 1
//     (int8_ops.cu:17-25); rstd = 1/sqrt(sum/W + eps) (correctly rounded here,
//     rsqrtf in the reference); v = T16((x * rstd) * gamma);
//   * scale = NaN if the row holds a non-finite value, 1 if it is all zero,
//     amax/127 otherwise; q = clamp(rne(v / scale), +-127), 0 for a bad row,
//     zero padding up to the padded width kp.
// The int8 row is staged in shared memory and written with 16-byte stores.
#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

enum InType : int { kInF32 = 0, kInF16 = 1, kInBF16 = 2 };

template <int IN>
__device__ __forceinline__ void load_row(const void* src, int width, float* buf, int lane) {
  if constexpr (IN == kInF32) {
    const float* s = static_cast<const float*>(src);
    if ((reinterpret_cast<uintptr_t>(s) & 15) == 0) {
      const int nv = width / 4;
      for (int i = lane; i < nv; i += 32) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(s) + i);
        buf[4 * i] = t.x;
        buf[4 * i + 1] = t.y;
        buf[4 * i + 2] = t.z;
        buf[4 * i + 3] = t.w;
      }
      for (int c = nv * 4 + lane; c < width; c += 32) buf[c] = __ldg(s + c);
    } else {
      for (int c = lane; c < width; c += 32) buf[c] = __ldg(s + c);
    }
  } else {
    const uint16_t* s = static_cast<const uint16_t*>(src);
    const bool f16 = IN == kInF16;
    if ((reinterpret_cast<uintptr_t>(s) & 15) == 0) {
      const int nv = width / 8;
      for (int i = lane; i < nv; i += 32) {
        const uint4 t = __ldg(reinterpret_cast<const uint4*>(s) + i);
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          buf[8 * i + 2 * j] = from16(static_cast<uint16_t>(w[j] & 0xffffu), f16);
          buf[8 * i + 2 * j + 1] = from16(static_cast<uint16_t>(w[j] >> 16), f16);
        }
      }
      for (int c = nv * 8 + lane; c < width; c += 32) buf[c] = from16(s[c], f16);
    } else {
      for (int c = lane; c < width; c += 32) buf[c] = from16(s[c], f16);
    }
  }
}

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

// Per-warp shared memory: `wbuf` floats of row values then `kp` int8 bytes.
template <int IN, bool RMS>
__global__ void __launch_bounds__(128) quantize_rows_kernel(
    const void* __restrict__ x, long ldx, const float* __restrict__ gamma, float eps, int rows,
    int width, int kp, int bound_f16, int wbuf, int8_t* __restrict__ q, float* __restrict__ scales,
    unsigned* status, unsigned layer) {
  extern __shared__ __align__(16) uint8_t qsmem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= rows) return;  // warp-uniform; only __syncwarp is used below
  float* buf = reinterpret_cast<float*>(qsmem + static_cast<size_t>(warp) * (wbuf * 4 + kp));
  int8_t* qs = reinterpret_cast<int8_t*>(buf + wbuf);
  const int esize = IN == kInF32 ? 4 : 2;
  load_row<IN>(static_cast<const uint8_t*>(x) + static_cast<size_t>(row) * ldx * esize, width, buf,
               lane);
  __syncwarp();
  if constexpr (RMS) {
    float sum = 0.0f;
    for (int c = lane; c < width; c += 32) sum = __fmaf_rn(buf[c], buf[c], sum);
    sum = warp_sum_xor(sum);
    const float rstd =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, static_cast<float>(width)), eps)));
    const bool f16 = bound_f16 != 0;
    for (int c = lane; c < width; c += 32)
      buf[c] = from16(bits16(__fmul_rn(__fmul_rn(buf[c], rstd), __ldg(gamma + c)), f16), f16);
  }
  uint32_t amax = 0;
  for (int c = lane; c < width; c += 32) amax = max(amax, abs_bits(buf[c]));
  amax = warp_max_u32(amax);
  const float scale = int8_scale_from_amax(amax);
  const bool bad = amax >= 0x7f800000u;
  if (lane == 0) {
    scales[row] = scale;
    if (bad) record_status(status, amax > 0x7f800000u ? KB_STATUS_NAN : KB_STATUS_INF, layer);
  }
  for (int c = lane; c < kp; c += 32)
    qs[c] = static_cast<int8_t>((c < width && !bad) ? quant_i8(buf[c], scale) : 0);
  __syncwarp();
  uint4* dst = reinterpret_cast<uint4*>(q + static_cast<size_t>(row) * kp);
  const uint4* s4 = reinterpret_cast<const uint4*>(qs);
  for (int i = lane; i < kp / 16; i += 32) dst[i] = s4[i];
}

template <int IN, bool RMS>
int launch_quant(const void* x, long ldx, const float* gamma, float eps, int rows, int width,
                 int kp, int bound_f16, int8_t* q, float* scales, unsigned* status, unsigned layer,
                 cudaStream_t stream) {
  const int wbuf = (width + 3) & ~3;
  const size_t smem = 4 * static_cast<size_t>(wbuf * 4 + kp);
  auto kern = quantize_rows_kernel<IN, RMS>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return check_cuda(e, "quantiser smem attribute");
  }
  kern<<<(rows + 3) / 4, 128, smem, stream>>>(x, ldx, gamma, eps, rows, width, kp, bound_f16, wbuf,
                                              q, scales, status, layer);
  return check_cuda(cudaGetLastError(), "quantiser launch");
}

}  // namespace

// dtype: 0 = f32, 1 = f16, 2 = bf16.  rms: apply RMSNorm with gamma/eps and a
// 16-bit boundary (bound_f16: 1 = fp16, 0 = bf16) before quantising.
int quantize_rows_launch(const void* x, int dtype, long ldx, int rows, int width, int kp, bool rms,
                         const float* gamma, float eps, int bound_f16, int8_t* q, float* scales,
                         unsigned* status, unsigned layer, cudaStream_t stream) {
  if (rows <= 0 || width <= 0 || width > 16384 || kp < width || kp % 16 != 0 || ldx < width) {
    set_error("quantiser shape mismatch (rows, width, padded width, stride)");
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

}  // namespace kb
