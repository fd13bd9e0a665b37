// Multi-head self-attention over the 361 board tokens, fused with RoPE.
//
// Replaces the reference's q64 flash attention (crates/kata_nn/cuda-kernels/
// attention_fa2_q64.cu:82-390; launcher src/backends/cuda_exec.rs:3442).
// Semantics follow the reference: packed projection [tokens, 3*C] = [Q | K | V]
// with head h at columns h*D..h*D+D-1 of each part; Q and K rotated in fp32 by
// interleaved pairs (2p, 2p+1) with per-(token, head, pair) cos/sin tables
// (native_model.rs:200-228) and rounded back to the 16-bit type; softmax over
// all S keys of (q.k) * scale in fp32; output [tokens, C] with heads merged.
//
// One CTA per (position, head), 8 warps.  The rotated K and the V of all S
// keys (S <= 384) stay in shared memory for the whole CTA; each warp takes
// 16-query chunks, keeps its rotated Q fragments in registers, and runs an
// online softmax over 64-key blocks with bf16 tensor-core MMAs (fp32
// accumulation): S = Q K^T, P = exp2((S - m) * scale * log2 e), O += P V.
// Scores and probabilities never leave registers.
#include <stdint.h>
#include <stdlib.h>

#include <atomic>

#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {

bool attention_tc_supported(int seq, int head_dim);
int attention_tc_launch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out, int batch,
                        int seq, int heads, int head_dim, float scale, int f16, cudaStream_t stream,
                        uint32_t* row_amax, unsigned* status);

namespace {

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kMaxSeq = 384;
#define kNegInf __int_as_float(0xff800000)

template <bool F16>
__device__ __forceinline__ void mma16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                                  const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Rotate one interleaved pair (x, y) by (c, s) and round to the 16-bit type.
__device__ __forceinline__ uint32_t rope_pair(uint32_t w, float c, float s, bool f16) {
  const float x = from16(static_cast<uint16_t>(w & 0xffffu), f16);
  const float y = from16(static_cast<uint16_t>(w >> 16), f16);
  const float rx = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
  const float ry = __fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c));
  return f16 ? pack_f16x2(rx, ry) : pack_bf16x2(rx, ry);
}

template <int D, bool F16>
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const uint16_t* __restrict__ qkv, const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
    uint16_t* __restrict__ out, int seq, int heads, float scale_log2, uint32_t* __restrict__ row_amax) {
  constexpr int kStride = D + 8;  // bf16 elements per smem row (16 B pad: conflict-free ldmatrix)
  constexpr int kKSteps = D / 16;
  constexpr int kDTiles = D / 8;
  extern __shared__ __align__(16) uint16_t asmem[];
  uint16_t* ks = asmem;                       // [kMaxSeq][kStride] rotated K
  uint16_t* vs = asmem + kMaxSeq * kStride;   // [kMaxSeq][kStride] V

  const int b = blockIdx.x / heads;
  const int h = blockIdx.x % heads;
  const int c = heads * D;
  const size_t row_stride = 3 * static_cast<size_t>(c);
  const uint16_t* base = qkv + static_cast<size_t>(b) * seq * row_stride;
  const int pairs_per_head = D / 2;
  const int seq_pad = (seq + 63) & ~63;

  // ---- stage rotated K and V for all keys (16-byte vectors), zero the padding
  constexpr int kVecs = D / 8;
  for (int t = threadIdx.x; t < seq_pad * kVecs; t += kAttnThreads) {
    const int key = t / kVecs;
    const int d0 = (t % kVecs) * 8;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (key < seq) {
      const uint16_t* kr = base + key * row_stride + c + h * D + d0;
      const uint16_t* vr = base + key * row_stride + 2 * c + h * D + d0;
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(kr));
      vv = __ldg(reinterpret_cast<const uint4*>(vr));
      if (rope_cos != nullptr) {
        const size_t ro = (static_cast<size_t>(key) * heads + h) * pairs_per_head + d0 / 2;
        const float4 co = __ldg(reinterpret_cast<const float4*>(rope_cos + ro));
        const float4 si = __ldg(reinterpret_cast<const float4*>(rope_sin + ro));
        kv.x = rope_pair(raw.x, co.x, si.x, F16);
        kv.y = rope_pair(raw.y, co.y, si.y, F16);
        kv.z = rope_pair(raw.z, co.z, si.z, F16);
        kv.w = rope_pair(raw.w, co.w, si.w, F16);
      } else {
        kv = raw;
      }
    }
    *reinterpret_cast<uint4*>(ks + key * kStride + d0) = kv;
    *reinterpret_cast<uint4*>(vs + key * kStride + d0) = vv;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gr = lane >> 2, q4 = lane & 3;
  const int chunks = (seq + 15) / 16;
  for (int chunk = warp; chunk < chunks; chunk += kAttnWarps) {
    const int r0 = chunk * 16 + gr, r1 = r0 + 8;
    // Rotated Q fragments: a[ks][0..3] = rows (r0, r1) x columns (q4*2, +8) of k-step ks.
    uint32_t qa[kKSteps][4];
#pragma unroll
    for (int kk = 0; kk < kKSteps; ++kk) {
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        const int r = (part & 1) ? r1 : r0;
        const int d = kk * 16 + q4 * 2 + ((part & 2) ? 8 : 0);
        uint32_t w = 0;
        if (r < seq) {
          const uint32_t raw = *reinterpret_cast<const uint32_t*>(base + r * row_stride + h * D + d);
          if (rope_cos != nullptr) {
            const size_t ro = (static_cast<size_t>(r) * heads + h) * pairs_per_head + d / 2;
            w = rope_pair(raw, __ldg(rope_cos + ro), __ldg(rope_sin + ro), F16);
          } else {
            w = raw;
          }
        }
        qa[kk][part] = w;
      }
    }
    float o[kDTiles][4];
#pragma unroll
    for (int n = 0; n < kDTiles; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m0 = kNegInf, m1 = kNegInf, l0 = 0.0f, l1 = 0.0f;

    for (int kb = 0; kb < seq_pad; kb += 64) {
      // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
        const uint16_t* krow = ks + (kb + n * 8 + gr) * kStride + q4 * 2;
#pragma unroll
        for (int kk = 0; kk < kKSteps; ++kk) {
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(krow + kk * 16);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(krow + kk * 16 + 8);
          mma16<F16>(s[n], qa[kk], b0, b1);
        }
      }
      // Mask keys past the sequence (only in the last block).
      if (kb + 64 > seq) {
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int key = kb + n * 8 + q4 * 2;
          if (key >= seq) s[n][0] = s[n][2] = kNegInf;
          if (key + 1 >= seq) s[n][1] = s[n][3] = kNegInf;
        }
      }
      float bm0 = kNegInf, bm1 = kNegInf;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        bm0 = fmaxf(bm0, fmaxf(s[n][0], s[n][1]));
        bm1 = fmaxf(bm1, fmaxf(s[n][2], s[n][3]));
      }
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 1));
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, 2));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 1));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, 2));
      const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
      const float corr0 = fast_exp2((m0 - mn0) * scale_log2);
      const float corr1 = fast_exp2((m1 - mn1) * scale_log2);
      m0 = mn0;
      m1 = mn1;
      const float off0 = mn0 * scale_log2, off1 = mn1 * scale_log2;
      float rs0 = 0.0f, rs1 = 0.0f;
      uint32_t pa[4][4];  // P as A fragments for 4 k-steps of 16 keys
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float p0 = fast_exp2(__fmaf_rn(s[n][0], scale_log2, -off0));
        const float p1 = fast_exp2(__fmaf_rn(s[n][1], scale_log2, -off0));
        const float p2 = fast_exp2(__fmaf_rn(s[n][2], scale_log2, -off1));
        const float p3 = fast_exp2(__fmaf_rn(s[n][3], scale_log2, -off1));
        rs0 += p0 + p1;
        rs1 += p2 + p3;
        pa[n / 2][(n & 1) * 2 + 0] = F16 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
        pa[n / 2][(n & 1) * 2 + 1] = F16 ? pack_f16x2(p2, p3) : pack_bf16x2(p2, p3);
      }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = l0 * corr0 + rs0;
      l1 = l1 * corr1 + rs1;
#pragma unroll
      for (int n = 0; n < kDTiles; ++n) {
        o[n][0] *= corr0;
        o[n][1] *= corr0;
        o[n][2] *= corr1;
        o[n][3] *= corr1;
      }
      // O += P V: k-steps over 16 keys, V fragments through ldmatrix.trans.
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        // a-fragment order for m16n8k16: rows gr/gr+8 x keys (q4*2, +8)
        const uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
        for (int n = 0; n < kDTiles; n += 2) {
          const int mtx = lane >> 3;
          const int key = kb + kk * 16 + (mtx & 1) * 8 + (lane & 7);
          const int dcol = n * 8 + (mtx >> 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(b0, b1, b2, b3, vs + key * kStride + dcol);
          mma16<F16>(o[n], a, b0, b1);
          mma16<F16>(o[n + 1], a, b2, b3);
        }
      }
    }
    const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
    uint32_t am0 = 0, am1 = 0;  // packed |16-bit| maxima of this thread's values in rows r0, r1
#pragma unroll
    for (int n = 0; n < kDTiles; ++n) {
      const int d = n * 8 + q4 * 2;
      const uint32_t w0 =
          F16 ? pack_f16x2(o[n][0] * inv0, o[n][1] * inv0) : pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
      const uint32_t w1 =
          F16 ? pack_f16x2(o[n][2] * inv1, o[n][3] * inv1) : pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
      am0 = __vmaxu2(am0, w0 & 0x7fff7fffu);
      am1 = __vmaxu2(am1, w1 & 0x7fff7fffu);
      if (r0 < seq) *reinterpret_cast<uint32_t*>(out + (static_cast<size_t>(b) * seq + r0) * c + h * D + d) = w0;
      if (r1 < seq) *reinterpret_cast<uint32_t*>(out + (static_cast<size_t>(b) * seq + r1) * c + h * D + d) = w1;
    }
    if (row_amax != nullptr) {
      // Row maxima for the following streaming quantiser: reduce over the 4
      // threads that share a row, one atomic per (row, head).
      uint32_t m0 = max(am0 & 0xffffu, am0 >> 16), m1 = max(am1 & 0xffffu, am1 >> 16);
      m0 = max(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
      m0 = max(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
      m1 = max(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
      m1 = max(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
      if (q4 == 0) {
        const uint32_t f0 = F16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m0))) : (m0 << 16);
        const uint32_t f1 = F16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m1))) : (m1 << 16);
        if (r0 < seq) atomicMax(row_amax + static_cast<size_t>(b) * seq + r0, f0);
        if (r1 < seq) atomicMax(row_amax + static_cast<size_t>(b) * seq + r1, f1);
      }
    }
  }
}

template <int D, bool F16>
int launch_attention(const uint16_t* qkv, const float* cos_t, const float* sin_t, uint16_t* out, int batch,
                     int seq, int heads, float scale, uint32_t* row_amax, cudaStream_t stream) {
  const size_t smem = 2 * static_cast<size_t>(kMaxSeq) * (D + 8) * sizeof(uint16_t);
  auto kern = attention_kernel<D, F16>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return check_cuda(e, "attention smem attribute");
    configured.fetch_or(bit);
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  kern<<<batch * heads, kAttnThreads, smem, stream>>>(qkv, cos_t, sin_t, out, seq, heads, scale_log2, row_amax);
  return check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace

// qkv: [batch*seq, 3*heads*D] 16-bit; cos/sin: [seq, heads, D/2] fp32, or both
// null when Q and K are already rotated; out: [batch*seq, heads*D] 16-bit.
// scale multiplies q.k before the softmax.
int attention_launch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out,
                     int batch, int seq, int heads, int head_dim, float scale, int f16, cudaStream_t stream,
                     uint32_t* row_amax, unsigned* status) {
  if (!qkv || (rope_cos == nullptr) != (rope_sin == nullptr) || !out || batch <= 0 || seq <= 0 ||
      seq > kMaxSeq || heads <= 0 || !(scale > 0.0f)) {
    set_error("attention: invalid arguments (seq must be 1..384)");
    return KB_E_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(rope_cos) & 15) ||
      (reinterpret_cast<uintptr_t>(rope_sin) & 15) || (reinterpret_cast<uintptr_t>(out) & 3)) {
    set_error("attention: qkv/tables must be 16-byte aligned");
    return KB_E_INVALID;
  }
  // The board (seq 361, head_dim 64 or 32) runs on the tcgen05 kernel; short
  // sequences on the mma.sync kernel above.  Tactic
  // switch KB_ATTENTION_MMA_SYNC=1 forces the latter (for A/B timing).
  static const bool force_sync = [] {
    const char* v = getenv("KB_ATTENTION_MMA_SYNC");
    return v != nullptr && v[0] == '1';
  }();
  if (!force_sync && attention_tc_supported(seq, head_dim))
    return attention_tc_launch(qkv, rope_cos, rope_sin, out, batch, seq, heads, head_dim, scale, f16, stream, row_amax,
                               status);
  if (head_dim == 64)
    return f16 ? launch_attention<64, true>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, stream)
               : launch_attention<64, false>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, stream);
  if (head_dim == 32)
    return f16 ? launch_attention<32, true>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, stream)
               : launch_attention<32, false>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, stream);
  set_error("attention: head_dim must be 32 or 64");
  return KB_E_UNSUPPORTED;
}

}  // namespace kb
