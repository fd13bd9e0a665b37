// Trunk kernels around the quantized blocks: the stem's input gather, the
// trunk tip, and the policy / value heads.
//
// Reference semantics (crates/kata_nn/tests/debug_exec_units.rs:101-380, the
// CPU restatement of every LayerGraph layer):
//  * InitialConv: 3x3 conv 22 -> C over the 19x19 board (zero padding) plus a
//    global linear 19 -> C, summed into the raw trunk (:101-129).  Here both
//    become one bf16 tcgen05 GEMM: stem_gather builds A[token, 224] =
//    [22*9 conv taps | 19 global features | 7 zeros].
//  * TrunkFinal: v = x*gamma + beta (BN affine with mean 0, std 1), SiLU (:272-282).
//  * PolicyHead (:283-341) and ValueHead (:342-380): per-token linears (done as
//    one bf16 GEMM to [token, 384] = [p1 96 | g1 96 | v1 192] before this
//    kernel), SiLU, global pooling (mean, mean*0.5, max / mean*0.15), tiny
//    MLPs, per-token policy / ownership projections.
#include <stdint.h>

#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

constexpr int kSide = 19;
constexpr int kSeq = kSide * kSide;
constexpr int kInC = 22;
constexpr int kInG = 19;
constexpr int kStemK = 224;  // 22*9 + 19 = 217, padded to a multiple of 8 (16 bytes of bf16)

// Board symmetry of one position (0..7: bit 2 transpose, bit 1 flip x, bit 0
// flip y).  The network sees copy_inputs_with_symmetry(input, sym)
// (crates/kata_game/src/symmetry.rs:108-224, reverse = false on a square
// board): the input at (row h, col w) lands at network (r, c) with
// r = flip_y' ? 18 - w : w, c = flip_x' ? 18 - h : h under transpose (flips
// swapped), else r = flip_y ? 18 - h : h, c = flip_x ? 18 - w : w.  The gather
// needs the inverse: the input cell that network cell (r, c) reads.
__device__ __forceinline__ int sym_source(int sym, int r, int c) {
  int a = r, b = c;
  if (sym & 4) {
    a = c;
    b = r;
  }
  if (sym & 1) a = kSide - 1 - a;
  if (sym & 2) b = kSide - 1 - b;
  return a * kSide + b;
}

// A[(b*361 + t), k] for the stem GEMM.  spatial: [B, 22, 19, 19] (NCHW) or
// [B, 19, 19, 22] (NHWC), global: [B, 19], both fp32; sym: [B] board
// symmetries (NULL = identity), applied as the input is gathered.
// One thread per (token, group of 8 columns): the 8 values leave as one
// 16-byte store; the tap index (ic, ky, kx) advances incrementally.
constexpr int kStemGroups = kStemK / 8;  // 28
__global__ void stem_gather_kernel(const float* __restrict__ spatial, const float* __restrict__ global,
                                   const int* __restrict__ sym, uint16_t* __restrict__ a, int batch, int nhwc,
                                   int f16) {
  const long total = static_cast<long>(batch) * kSeq * kStemGroups;
  for (long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long>(gridDim.x) * blockDim.x) {
    const int grp = static_cast<int>(idx % kStemGroups);
    const long row = idx / kStemGroups;
    const int b = static_cast<int>(row / kSeq);
    const int t = static_cast<int>(row - static_cast<long>(b) * kSeq);
    const int y = t / kSide, x = t - (t / kSide) * kSide;
    const int sm = sym ? (__ldg(sym + b) & 7) : 0;
    int k = grp * 8;
    int ic = k / 9, r9 = k - 9 * ic;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e, ++k) {
      float val = 0.0f;
      if (k < kInC * 9) {
        const int ky = r9 / 3, kx = r9 - 3 * (r9 / 3);
        const int sy = y + ky - 1, sx = x + kx - 1;
        if (sy >= 0 && sy < kSide && sx >= 0 && sx < kSide) {
          const int cell = sym_source(sm, sy, sx);
          const long off = nhwc ? ((static_cast<long>(b) * kSeq + cell) * kInC + ic)
                                : ((static_cast<long>(b) * kInC + ic) * kSeq + cell);
          val = __ldg(spatial + off);
        }
      } else if (k < kInC * 9 + kInG) {
        val = __ldg(global + static_cast<long>(b) * kInG + (k - kInC * 9));
      }
      v[e] = val;
      if (++r9 == 9) r9 = 0, ++ic;
    }
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = pack16x2(make_float2(v[2 * q], v[2 * q + 1]), f16 != 0);
    reinterpret_cast<uint4*>(a)[idx] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// SiLU for the trunk tip and the fp32 heads (their outputs are compared with
// a tolerance, not bit for bit): x / (1 + e^-x) with the fast exponential and
// division.
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// g = bf16(silu(x * gamma + beta)) over [rows, c] bf16, c a multiple of 8:
// each thread converts 8 consecutive values (one 16-byte load and store) per
// vector, two vectors per loop trip with both loads issued first (more bytes
// in flight per thread: the kernel streams 2 bytes in and out per value).
__device__ __forceinline__ uint4 tip8(uint4 raw, const float* __restrict__ gamma, const float* __restrict__ beta,
                                      int col) {
  const float4 g0 = __ldg(reinterpret_cast<const float4*>(gamma + col));
  const float4 g1 = __ldg(reinterpret_cast<const float4*>(gamma + col) + 1);
  const float4 b0 = __ldg(reinterpret_cast<const float4*>(beta + col));
  const float4 b1 = __ldg(reinterpret_cast<const float4*>(beta + col) + 1);
  const float gm[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const float bt[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = from_bf16(static_cast<uint16_t>(w[j] & 0xffffu));
    const float hi = from_bf16(static_cast<uint16_t>(w[j] >> 16));
    const float v0 = __fadd_rn(__fmul_rn(lo, gm[2 * j]), bt[2 * j]);
    const float v1 = __fadd_rn(__fmul_rn(hi, gm[2 * j + 1]), bt[2 * j + 1]);
    o[j] = static_cast<uint32_t>(bits_bf16(silu_fast(v0))) | (static_cast<uint32_t>(bits_bf16(silu_fast(v1))) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void trunk_tip_kernel(const uint16_t* __restrict__ x, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, uint16_t* __restrict__ g, uint32_t total8,
                                 FastDiv c8) {
  // 32-bit vector indices (total8 < 2^31, checked on the host); the column
  // of vector i is (i mod c8) * 8, by a multiply-shift division
  const uint4* x4 = reinterpret_cast<const uint4*>(x);
  uint4* g4 = reinterpret_cast<uint4*>(g);
  const uint32_t stride = gridDim.x * blockDim.x;
  uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  auto col = [&](uint32_t v) { return static_cast<int>(v - c8.div(v) * c8.d) * 8; };
  for (; i + stride < total8; i += 2 * stride) {
    const uint4 r0 = __ldg(x4 + i), r1 = __ldg(x4 + i + stride);
    g4[i] = tip8(r0, gamma, beta, col(i));
    g4[i + stride] = tip8(r1, gamma, beta, col(i + stride));
  }
  if (i < total8) g4[i] = tip8(__ldg(x4 + i), gamma, beta, col(i));
}

// The nested trunk's gates (BN affine folded to scale/bias, then SiLU):
// out16 = T16(silu(x * scale + bias)) from fp32 rows x [rows, w] (row stride
// ldx), into 16-bit rows (stride ldo), w a multiple of 8.  The affine is two
// rounded operations and the SiLU kb_silu (here on pairs: kb_silu2, the same
// bits), so the CPU oracle reproduces every value; 8 columns per thread (two
// 16-byte loads, one 16-byte store), rows * w / 8 < 2^31 items.
__global__ void gate_silu_kernel(const float* __restrict__ x, long ldx, const float* __restrict__ scale,
                                 const float* __restrict__ bias, uint16_t* __restrict__ out, long ldo, uint32_t total,
                                 FastDiv w8, int f16) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t r = w8.div(i);
    const int c = static_cast<int>(i - r * w8.d) * 8;
    const float4* src = reinterpret_cast<const float4*>(x + r * ldx + c);
    const float4 a = __ldg(src), b = __ldg(src + 1);
    const float4 s0 = __ldg(reinterpret_cast<const float4*>(scale + c)), s1 = __ldg(reinterpret_cast<const float4*>(scale + c) + 1);
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + c)), b1 = __ldg(reinterpret_cast<const float4*>(bias + c) + 1);
    const float2 xv[4] = {make_float2(a.x, a.y), make_float2(a.z, a.w), make_float2(b.x, b.y), make_float2(b.z, b.w)};
    const float2 sv[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w), make_float2(s1.x, s1.y),
                          make_float2(s1.z, s1.w)};
    const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                          make_float2(b1.z, b1.w)};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      // scalar rounded affine: a packed multiply feeding a packed add may be
      // contracted into a fused multiply-add by the assembler
      const float2 v = make_float2(__fadd_rn(__fmul_rn(xv[q].x, sv[q].x), bv[q].x),
                                   __fadd_rn(__fmul_rn(xv[q].y, sv[q].y), bv[q].y));
      o[q] = pack16x2(kb_silu2(v), f16 != 0);
    }
    *reinterpret_cast<uint4*>(out + r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

struct HeadWeights {
  const float* g_matmul;   // [96, 288]
  const float* pass1_w;    // [96, 288]
  const float* pass1_b;    // [96]
  const float* pass2_w;    // [6, 96]
  const float* bias2;      // [96]
  const float* conv2p_w;   // [6, 96]
  const float* v2_w;       // [192, 576]
  const float* v2_b;       // [192]
  const float* value_w;    // [3, 192]
  const float* value_b;    // [3]
  const float* misc_w;     // [10, 192]
  const float* misc_b;     // [10]
  const float* moremisc_w; // [8, 192]
  const float* moremisc_b; // [8]
  const float* own_w;      // [192]
};

constexpr int kHeadThreads = 768;
constexpr int kHeadWarps = kHeadThreads / 32;


// Warp-cooperative dot product of a weight row (k floats, global) with a
// vector in shared memory; every lane returns the sum (fixed reduction order).
__device__ __forceinline__ float warp_dot(const float* __restrict__ wrow, const float* vec, int k, int lane) {
  float a = 0.0f;
  for (int i = lane; i < k; i += 32) a = __fmaf_rn(__ldg(wrow + i), vec[i], a);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  return a;
}

// Four such dot products at once (rows w0 + r * stride, r < 4) over K floats,
// K a multiple of 4: lane l reads the 16-byte pieces l, l + 32, ... of each
// row, all four rows' loads in flight together (the products are
// latency-bound, not bandwidth-bound).
template <int K>
__device__ __forceinline__ void warp_dot4(const float* __restrict__ w0, int stride, const float* vec, int lane,
                                          float (&out)[4]) {
  constexpr int kP = K / 4;             // 16-byte pieces per row
  constexpr int kQ = (kP + 31) / 32;    // pieces per lane (the last one partial)
  float4 wv[4][kQ];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int q = 0; q < kQ; ++q)
      wv[r][q] = lane + 32 * q < kP ? __ldg(reinterpret_cast<const float4*>(w0 + r * stride) + lane + 32 * q)
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    float a = 0.0f;
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
      if (lane + 32 * q >= kP) continue;
      const float4 v = *reinterpret_cast<const float4*>(vec + 4 * (lane + 32 * q));
      a = __fmaf_rn(wv[r][q].x, v.x, a);
      a = __fmaf_rn(wv[r][q].y, v.y, a);
      a = __fmaf_rn(wv[r][q].z, v.z, a);
      a = __fmaf_rn(wv[r][q].w, v.w, a);
    }
    out[r] = a;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] += __shfl_xor_sync(0xffffffffu, out[r], o);
}

// One CTA of 24 warps per position.  Pass 1 pools the SiLU'd head activations
// (two tokens per warp per step), the matrix-vector products run four outputs
// per warp at a time, pass 2 computes each token's policy moves and ownership
// (two tokens per warp per step): everything here is latency-bound, so the
// work is arranged to keep many loads in flight per warp.
__global__ void __launch_bounds__(kHeadThreads) heads_kernel(const float* __restrict__ hp, HeadWeights w,
                                                            float* __restrict__ policy, float* __restrict__ value,
                                                            float* __restrict__ misc, float* __restrict__ moremisc,
                                                            float* __restrict__ ownership, unsigned* status) {
  __shared__ float part_sum[kHeadWarps][288];
  __shared__ float part_max[kHeadWarps][96];
  __shared__ __align__(16) float pooled_p[288];
  __shared__ __align__(16) float pooled_v[576];
  __shared__ float gproj[96];
  __shared__ float pass1[96];
  __shared__ float vhid[192];
  __shared__ float conv2p[6 * 96];
  __shared__ float ownw[192];
  __shared__ int bad_any;
  const int b = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* rows = hp + static_cast<size_t>(b) * kSeq * 384;
  if (tid == 0) bad_any = 0;
  for (int i = tid; i < 6 * 96; i += kHeadThreads) conv2p[i] = w.conv2p_w[i];
  for (int i = tid; i < 192; i += kHeadThreads) ownw[i] = w.own_w[i];
  {
    // ---- pass 1: SiLU then mean (g1 and v1) and max (g1)
    const int nq = lane < 8 ? 3 : 2;  // float4 columns of this lane
    float sum[12], mx[4];
#pragma unroll
    for (int i = 0; i < 12; ++i) sum[i] = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) mx[i] = __int_as_float(0xff800000);
    for (int t0 = warp; t0 < kSeq; t0 += 2 * kHeadWarps) {
      float4 v[2][3];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = t0 + u * kHeadWarps;
        const float4* r4 = reinterpret_cast<const float4*>(rows + static_cast<size_t>(t) * 384 + 96);
#pragma unroll
        for (int q = 0; q < 3; ++q)
          v[u][q] = (t < kSeq && q < nq) ? __ldg(r4 + lane + 32 * q) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (t0 + u * kHeadWarps >= kSeq) continue;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          if (q < nq) {
            const float a[4] = {silu_fast(v[u][q].x), silu_fast(v[u][q].y), silu_fast(v[u][q].z),
                                silu_fast(v[u][q].w)};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              sum[4 * q + e] += a[e];
              if (q == 0) mx[e] = fmaxf(mx[e], a[e]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
      if (q < nq)
#pragma unroll
        for (int e = 0; e < 4; ++e) part_sum[warp][4 * (lane + 32 * q) + e] = sum[4 * q + e];
    if (lane < 24)
#pragma unroll
      for (int e = 0; e < 4; ++e) part_max[warp][4 * lane + e] = mx[e];
  }
  __syncthreads();
  if (tid < 288) {
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kHeadWarps; ++i) s += part_sum[i][tid];
    const float mean = s * (1.0f / static_cast<float>(kSeq));
    if (tid < 96) {
      float m = part_max[0][tid];
#pragma unroll
      for (int i = 1; i < kHeadWarps; ++i) m = fmaxf(m, part_max[i][tid]);
      pooled_p[tid] = mean;
      pooled_p[96 + tid] = mean * 0.5f;
      pooled_p[192 + tid] = m;
    } else {
      const int ch = tid - 96;
      pooled_v[ch] = mean;
      pooled_v[192 + ch] = mean * 0.5f;
      pooled_v[384 + ch] = mean * 0.15f;
    }
  }
  __syncthreads();
  // ---- matrix-vector products, four outputs per warp at a time: groups 0..23
  // gproj, 24..47 pass1 (288 wide), 48..95 v2 (576 wide)
  for (int grp = warp; grp < 96; grp += kHeadWarps) {
    float a[4];
    if (grp < 48) {
      const bool gp = grp < 24;
      const int o0 = 4 * (gp ? grp : grp - 24);
      warp_dot4<288>((gp ? w.g_matmul : w.pass1_w) + o0 * 288, 288, pooled_p, lane, a);
      if (lane < 4) {
        const int o = o0 + lane;
        const float x = lane == 0 ? a[0] : lane == 1 ? a[1] : lane == 2 ? a[2] : a[3];
        if (gp) gproj[o] = x + w.bias2[o];
        else pass1[o] = silu_fast(x + w.pass1_b[o]);
      }
    } else {
      const int o0 = 4 * (grp - 48);
      warp_dot4<576>(w.v2_w + o0 * 576, 576, pooled_v, lane, a);
      if (lane < 4) {
        const int o = o0 + lane;
        const float x = lane == 0 ? a[0] : lane == 1 ? a[1] : lane == 2 ? a[2] : a[3];
        vhid[o] = silu_fast(x + w.v2_b[o]);
      }
    }
  }
  __syncthreads();
  float* pol = policy + static_cast<size_t>(b) * 6 * 362;
  bool bad = false;
  // ---- pass logits (6) and value / misc / moremisc (21), one warp per output
  for (int o = warp; o < 27; o += kHeadWarps) {
    if (o < 6) {
      const float a = warp_dot(w.pass2_w + o * 96, pass1, 96, lane);
      if (lane == 0) {
        pol[o * 362 + 361] = a;
        bad |= !isfinite(a);
      }
    } else {
      const int v = o - 6;
      const float* wr;
      float bias;
      float* dst;
      if (v < 3) {
        wr = w.value_w + v * 192, bias = w.value_b[v], dst = value + b * 3 + v;
      } else if (v < 13) {
        wr = w.misc_w + (v - 3) * 192, bias = w.misc_b[v - 3], dst = misc + b * 10 + (v - 3);
      } else {
        wr = w.moremisc_w + (v - 13) * 192, bias = w.moremisc_b[v - 13], dst = moremisc + b * 8 + (v - 13);
      }
      const float a = warp_dot(wr, vhid, 192, lane) + bias;
      if (lane == 0) {
        *dst = a;
        bad |= !isfinite(a);
      }
    }
  }
  // ---- pass 2: per token, policy moves (6) and ownership, two tokens per step
  {
    float gp[4], cw[6][4], ow[8];
    if (lane < 24)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        gp[e] = gproj[4 * lane + e];
#pragma unroll
        for (int o = 0; o < 6; ++o) cw[o][e] = conv2p[o * 96 + 4 * lane + e];
      }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ow[e] = ownw[4 * lane + e];
      ow[4 + e] = lane < 16 ? ownw[128 + 4 * lane + e] : 0.0f;
    }
    for (int t0 = warp; t0 < kSeq; t0 += 2 * kHeadWarps) {
      float4 pq[2], vq[2], uq[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = t0 + u * kHeadWarps;
        const float* r = rows + static_cast<size_t>(t < kSeq ? t : t0) * 384;
        pq[u] = lane < 24 ? __ldg(reinterpret_cast<const float4*>(r) + lane) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        vq[u] = __ldg(reinterpret_cast<const float4*>(r + 192) + lane);
        uq[u] = lane < 16 ? __ldg(reinterpret_cast<const float4*>(r + 320) + lane)
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
      float acc[2][7];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
#pragma unroll
        for (int o = 0; o < 7; ++o) acc[u][o] = 0.0f;
        if (lane < 24) {
          const float pv[4] = {pq[u].x, pq[u].y, pq[u].z, pq[u].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float pa = silu_fast(pv[e] + gp[e]);
#pragma unroll
            for (int o = 0; o < 6; ++o) acc[u][o] = __fmaf_rn(pa, cw[o][e], acc[u][o]);
          }
        }
        acc[u][6] = __fmaf_rn(silu_fast(vq[u].x), ow[0], acc[u][6]);
        acc[u][6] = __fmaf_rn(silu_fast(vq[u].y), ow[1], acc[u][6]);
        acc[u][6] = __fmaf_rn(silu_fast(vq[u].z), ow[2], acc[u][6]);
        acc[u][6] = __fmaf_rn(silu_fast(vq[u].w), ow[3], acc[u][6]);
        if (lane < 16) {
          acc[u][6] = __fmaf_rn(silu_fast(uq[u].x), ow[4], acc[u][6]);
          acc[u][6] = __fmaf_rn(silu_fast(uq[u].y), ow[5], acc[u][6]);
          acc[u][6] = __fmaf_rn(silu_fast(uq[u].z), ow[6], acc[u][6]);
          acc[u][6] = __fmaf_rn(silu_fast(uq[u].w), ow[7], acc[u][6]);
        }
      }
#pragma unroll
      for (int sh = 16; sh > 0; sh >>= 1)
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int o = 0; o < 7; ++o) acc[u][o] += __shfl_xor_sync(0xffffffffu, acc[u][o], sh);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = t0 + u * kHeadWarps;
        if (t >= kSeq) continue;
        if (lane < 6) {
          float a = acc[u][0];
#pragma unroll
          for (int o = 1; o < 6; ++o)
            if (lane == o) a = acc[u][o];
          pol[lane * 362 + t] = a;
          bad |= !isfinite(a);
        } else if (lane == 6) {
          ownership[static_cast<size_t>(b) * kSeq + t] = acc[u][6];
          bad |= !isfinite(acc[u][6]);
        }
      }
    }
  }
  // Sticky status: a non-finite value reached an output (reference
  // mxfp8_check_final_outputs_kernel, cuda-kernels/mxfp8.cu:162-177).
  if (bad) atomicOr(&bad_any, 1);
  __syncthreads();
  if (tid == 0 && bad_any) record_status(status, KB_STATUS_OUTPUT_NONFINITE, 0xfffffffeu);
}

}  // namespace

int stem_gather_launch(const float* spatial, const float* global, const int* sym, uint16_t* a, int batch,
                       int nhwc, cudaStream_t s, int f16) {
  if (reinterpret_cast<uintptr_t>(a) & 15) {
    set_error("stem gather: the operand must be 16-byte aligned");
    return KB_E_INVALID;
  }
  const long total = static_cast<long>(batch) * kSeq * kStemGroups;
  int dev = 0;
  cudaGetDevice(&dev);
  const long want = (total + 255) / 256, cap = 16L * num_sms(dev);
  stem_gather_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, s>>>(spatial, global, sym, a, batch,
                                                                                     nhwc, f16);
  return check_cuda(cudaGetLastError(), "stem gather launch");
}

int trunk_tip_launch(const uint16_t* x, const float* gamma, const float* beta, uint16_t* g, long rows, int c,
                     cudaStream_t s) {
  if (c % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(g) & 15) ||
      (reinterpret_cast<uintptr_t>(gamma) & 15) || (reinterpret_cast<uintptr_t>(beta) & 15)) {
    set_error("trunk tip: channels must be a multiple of 8 and buffers 16-byte aligned");
    return KB_E_INVALID;
  }
  const long total8 = rows * c / 8;
  if (total8 >= (1L << 30)) {  // i + stride stays below 2^31
    set_error("trunk tip: rows * channels / 8 must be below 2^30");
    return KB_E_INVALID;
  }
  if (total8 == 0) return KB_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const long want = (total8 + 255) / 256, cap = 8L * num_sms(dev);
  trunk_tip_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, s>>>(
      x, gamma, beta, g, static_cast<uint32_t>(total8), FastDiv(static_cast<uint32_t>(c / 8)));
  return check_cuda(cudaGetLastError(), "trunk tip launch");
}

int gate_silu_launch(const float* x, long ldx, const float* scale, const float* bias, uint16_t* out, long ldo,
                     long rows, int w, int f16, cudaStream_t s) {
  if (w % 8 != 0 || ldx % 4 != 0 || ldo % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(scale) & 15) ||
      (reinterpret_cast<uintptr_t>(bias) & 15)) {
    set_error("gate: width a multiple of 8, 16-byte aligned rows and vectors");
    return KB_E_INVALID;
  }
  const long total = rows * (w / 8);
  if (rows < 0 || total >= (1L << 31)) {
    set_error("gate: rows * width / 8 must be below 2^31");
    return KB_E_INVALID;
  }
  if (total == 0) return KB_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  const long want = (total + 255) / 256, cap = 8L * num_sms(dev);
  gate_silu_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, s>>>(
      x, ldx, scale, bias, out, ldo, static_cast<uint32_t>(total), FastDiv(static_cast<uint32_t>(w / 8)), f16);
  return check_cuda(cudaGetLastError(), "gate launch");
}

int heads_launch(const float* hp, const float* const* wts, float* policy, float* value, float* misc,
                 float* moremisc, float* ownership, int batch, unsigned* status, cudaStream_t s) {
  HeadWeights w{wts[0], wts[1], wts[2], wts[3], wts[4], wts[5], wts[6], wts[7],
                wts[8], wts[9], wts[10], wts[11], wts[12], wts[13], wts[14]};
  heads_kernel<<<batch, kHeadThreads, 0, s>>>(hp, w, policy, value, misc, moremisc, ownership, status);
  return check_cuda(cudaGetLastError(), "heads launch");
}

}  // namespace kb
