// Self-attention over the 361 board tokens on the tcgen05 tensor cores, fused
// with RoPE (head_dim 64).
//
// Replaces the reference's q64 flash attention (crates/kata_nn/cuda-kernels/
// attention_fa2_q64.cu:82-390; launcher src/backends/cuda_exec.rs:3442) with the
// same semantics as attention.cu: packed [tokens, 3C] = [Q | K | V], Q and K
// rotated by interleaved pairs with per-(token, head, pair) tables and rounded
// to the 16-bit type, softmax of (q.k) * scale over all keys in fp32, P rounded
// to the 16-bit type for the P.V product, output [tokens, C] heads merged.
//
// One CTA per (position, head); two CTAs share an SM (112 KB shared memory and
// 256 TMEM columns each).  All 361 keys fit on chip, so there is no streaming:
//   shared memory  K and V of the board, 368 rows x 128 B (keys padded to a
//                  multiple of 16), and one 128-query Q tile, all in the UMMA
//                  128-byte-swizzled layout (written by the CTA's threads,
//                  with RoPE applied on the way in);
//   TMEM           S (128 lanes x 192 fp32 columns) and O (64 columns).
// Per 128-query tile, keys in two halves A = [0, 192) and B = [192, 368):
//   MMA  S = Q K_A^T          softmax warps: row max, P_A = exp2((S - m) c) in
//                             place over S as packed 16-bit (A operand), sum
//   MMA  O = P_A V_A          (A from TMEM, V as an MN-major B operand)
//   MMA  S = Q K_B^T          softmax: m' = max(m, max S_B), P_B, rescale O by
//                             exp2((m - m') c) when the maximum moved
//   MMA  O += P_B V_B         epilogue: O / sum -> 16-bit, row |max| for the
//                             next quantiser.
// Warps 0-3 (one TMEM lane quarter each, thread = query row) load, run the
// softmax and the epilogue; warp 4 issues the MMAs.  Every wait is bounded;
// the softmax warps leave together (warp-collective TMEM accesses follow).
#include <stdint.h>

#include <atomic>

#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

constexpr int kD = 64;
constexpr int kKeysPad = 368;             // >= 361, multiple of 16
constexpr int kHalfA = 192, kHalfB = kKeysPad - kHalfA;  // 176
constexpr int kTileQ = 128;
constexpr int kRowBytes = kD * 2;         // 128 B: one swizzle row
constexpr int kKBytes = kKeysPad * kRowBytes;
constexpr int kQBytes = kTileQ * kRowBytes;
constexpr int kSoftThreads = 128;
constexpr int kTcThreads = kSoftThreads + 32;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kOCol = 192;
constexpr int kSmemBytes = 2 * kKBytes + kQBytes + 128 /*barriers*/ + 1024 /*alignment*/;

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool f16) {
  if (f16) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Rotate one interleaved pair (x, y) by (c, s), rounded to the 16-bit type.
__device__ __forceinline__ uint32_t rope2(uint32_t w, float c, float s, bool f16) {
  const float x = from16(static_cast<uint16_t>(w & 0xffffu), f16);
  const float y = from16(static_cast<uint16_t>(w >> 16), f16);
  return pack2(__fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s)), __fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c)), f16);
}

// Byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * kRowBytes + ((c ^ (r & 7)) << 4));
}

// Rows [r0, r0 + nrows) of Q or K (part = 0 / 1) or V (part = 2) of head h of
// one position into a swizzled tile; rows at or past `seq` are zero.  Each
// thread handles kBatch 16-byte chunks per step with all their global loads
// issued before any is used, so the copy is not bound by one load's latency.
constexpr int kBatch = 4;

template <bool F16>
__device__ __forceinline__ void stage_rows(uint8_t* dst, const uint16_t* base, size_t row_stride, int part, int h,
                                           int heads, const float* cos_t, const float* sin_t, int r0, int nrows,
                                           int seq, int tid, int nthreads) {
  const int c = heads * kD;
  const int total = nrows * 8;
  for (int t0 = tid; t0 < total; t0 += kBatch * nthreads) {
    uint4 raw[kBatch];
    float4 co[kBatch], si[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = t0 + u * nthreads;
      const int r = t >> 3, ch = t & 7;
      const int tok = r0 + r;
      raw[u] = make_uint4(0, 0, 0, 0);
      if (t < total && tok < seq) {
        raw[u] = __ldg(reinterpret_cast<const uint4*>(base + tok * row_stride + part * c + h * kD + ch * 8));
        if (part != 2) {
          const size_t ro = (static_cast<size_t>(tok) * heads + h) * (kD / 2) + ch * 4;
          co[u] = __ldg(reinterpret_cast<const float4*>(cos_t + ro));
          si[u] = __ldg(reinterpret_cast<const float4*>(sin_t + ro));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = t0 + u * nthreads;
      if (t >= total) break;
      const int r = t >> 3, ch = t & 7;
      uint4 v = raw[u];
      if (part != 2 && r0 + r < seq)
        v = make_uint4(rope2(raw[u].x, co[u].x, si[u].x, F16), rope2(raw[u].y, co[u].y, si[u].y, F16),
                       rope2(raw[u].z, co[u].z, si[u].z, F16), rope2(raw[u].w, co[u].w, si[u].w, F16));
      *reinterpret_cast<uint4*>(dst + sw128(r, ch)) = v;
    }
  }
}

template <bool F16>
__global__ void __launch_bounds__(kTcThreads, 2) attention_tc_kernel(
    const uint16_t* __restrict__ qkv, const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
    uint16_t* __restrict__ out, int seq, int heads, float scale_log2, uint32_t* __restrict__ row_amax,
    unsigned* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ks = smem;
  uint8_t* vs = smem + kKBytes;
  uint8_t* qs = smem + 2 * kKBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(qs + kQBytes);
  uint64_t* s_full = bars + 0;  // S ready (tcgen05.commit), twice per tile
  uint64_t* p_full = bars + 1;  // P in TMEM (128 softmax threads), twice per tile
  uint64_t* o_full = bars + 2;  // P.V done (tcgen05.commit), twice per tile
  uint64_t* q_full = bars + 3;  // next Q tile staged (128 threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int b = blockIdx.x / heads;
  const int h = blockIdx.x % heads;
  const int c = heads * kD;
  const size_t row_stride = 3 * static_cast<size_t>(c);
  const uint16_t* base = qkv + static_cast<size_t>(b) * seq * row_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (seq + kTileQ - 1) / kTileQ;

  if (threadIdx.x == 0) {
    mbar_init(s_full, 1);
    mbar_init(p_full, kSoftThreads);
    mbar_init(o_full, 1);
    mbar_init(q_full, kSoftThreads);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  // Stage K (rotated), V and the first Q tile with every thread of the CTA.
  stage_rows<F16>(ks, base, row_stride, 1, h, heads, rope_cos, rope_sin, 0, kKeysPad, seq, threadIdx.x, kTcThreads);
  stage_rows<F16>(vs, base, row_stride, 2, h, heads, rope_cos, rope_sin, 0, kKeysPad, seq, threadIdx.x, kTcThreads);
  stage_rows<F16>(qs, base, row_stride, 0, h, heads, rope_cos, rope_sin, 0, kTileQ, seq, threadIdx.x, kTcThreads);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = F16 ? 0u : 1u;
      const uint32_t id_common = (1u << 4) | (kFmt << 7) | (kFmt << 10) | (static_cast<uint32_t>(128 >> 4) << 24);
      const uint32_t id_sa = id_common | (static_cast<uint32_t>(kHalfA >> 3) << 17);
      const uint32_t id_sb = id_common | (static_cast<uint32_t>(kHalfB >> 3) << 17);
      const uint32_t id_pv = id_common | (1u << 16) /* B MN-major */ | (static_cast<uint32_t>(kD >> 3) << 17);
      const uint64_t qdesc = sw128_desc(smem_u32(qs));
      const uint64_t kdesc = sw128_desc(smem_u32(ks));
      const uint64_t vdesc = sw128_desc(smem_u32(vs));
      // Half B starts 192 rows (192 * 128 B, >> 4 in the address field) further.
      constexpr uint64_t kHalfBOff = (kHalfA * kRowBytes) >> 4;
      constexpr uint64_t kKStep16 = (16 * kRowBytes) >> 4;  // 16 keys of V along K
      for (int t = 0; t < tiles; ++t) {
        if (t > 0 && !mbar_wait(q_full, (t - 1) & 1, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)  // 16 elements = 32 bytes of K per MMA
          mma_issue<kKindBF16>(tmem, qdesc + 2 * kk, kdesc + 2 * kk, id_sa, kk != 0, 0, 0);
        tc_commit(s_full);
        if (!mbar_wait(p_full, 0, abort_flag)) break;
        tc_fence_after();
        for (int i = 0; i < kHalfA / 16; ++i)
          mma_f16_ts(tmem + kOCol, tmem + 8 * i, vdesc + kKStep16 * i, id_pv, i != 0);
        tc_commit(o_full);
        if (!mbar_wait(o_full, 0, abort_flag)) break;  // P_A consumed before S is overwritten
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_issue<kKindBF16>(tmem, qdesc + 2 * kk, kdesc + kHalfBOff + 2 * kk, id_sb, kk != 0, 0, 0);
        tc_commit(s_full);
        if (!mbar_wait(p_full, 1, abort_flag)) break;
        tc_fence_after();
        for (int i = 0; i < kHalfB / 16; ++i)
          mma_f16_ts(tmem + kOCol, tmem + 8 * i, vdesc + kHalfBOff + kKStep16 * i, id_pv, 1);
        tc_commit(o_full);
        if (!mbar_wait(o_full, 1, abort_flag)) break;  // P_B consumed before the next tile's S
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int row = warp * 32 + lane;
    for (int t = 0; t < tiles; ++t) {
      const int query = t * kTileQ + row;
      // -- half A: keys [0, 192), all valid (seq > 192 is required by the launcher)
      if (!__all_sync(0xffffffffu, mbar_wait(s_full, 0, abort_flag))) break;
      tc_fence_after();
      float m = __int_as_float(0xff800000);
      for (int ch = 0; ch < kHalfA / 32; ++ch) {
        uint32_t v[32];
        tmem_ld32(lane_base + ch * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) m = fmaxf(m, __uint_as_float(v[i]));
      }
      float mc = m * scale_log2;
      float l = 0.0f;
      for (int ch = 0; ch < kHalfA / 32; ++ch) {
        uint32_t v[32], pk[16];
        tmem_ld32(lane_base + ch * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2(__fmaf_rn(__uint_as_float(v[2 * i]), scale_log2, -mc));
          const float p1 = ex2(__fmaf_rn(__uint_as_float(v[2 * i + 1]), scale_log2, -mc));
          l += p0 + p1;
          pk[i] = pack2(p0, p1, F16);
        }
        tmem_st16(lane_base + ch * 16, pk);  // P over the S columns already read
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
      // -- half B: keys [192, 368), valid below seq
      if (!__all_sync(0xffffffffu, mbar_wait(s_full, 1, abort_flag))) break;
      tc_fence_after();
      const int valid_b = seq - kHalfA;
      float mb = __int_as_float(0xff800000);
      for (int ch = 0; ch < (kHalfB + 31) / 32; ++ch) {
        uint32_t v[32];
        tmem_ld32(lane_base + ch * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (ch * 32 + i < valid_b) mb = fmaxf(mb, __uint_as_float(v[i]));
      }
      const float mn = fmaxf(m, mb);
      const float alpha = mn == m ? 1.0f : ex2(__fmul_rn(__fsub_rn(m, mn), scale_log2));
      mc = mn * scale_log2;
      float lb = 0.0f;
      for (int ch = 0; ch < (kHalfB + 31) / 32; ++ch) {
        uint32_t v[32], pk[16];
        tmem_ld32(lane_base + ch * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k0 = ch * 32 + 2 * i;
          const float p0 = k0 < valid_b ? ex2(__fmaf_rn(__uint_as_float(v[2 * i]), scale_log2, -mc)) : 0.0f;
          const float p1 = k0 + 1 < valid_b ? ex2(__fmaf_rn(__uint_as_float(v[2 * i + 1]), scale_log2, -mc)) : 0.0f;
          lb += p0 + p1;
          pk[i] = pack2(p0, p1, F16);
        }
        tmem_st16(lane_base + ch * 16, pk);
      }
      l = l * alpha + lb;
      // O holds P_A.V_A scaled to the old maximum: rescale where it moved.
      if (!__all_sync(0xffffffffu, mbar_wait(o_full, 0, abort_flag))) break;
      tc_fence_after();
      if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t v[32];
          tmem_ld32(lane_base + kOCol + half * 32, v);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
          tmem_st32(lane_base + kOCol + half * 32, v);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
      // -- the next Q tile: S_B has consumed this one
      if (t + 1 < tiles) {
        stage_rows<F16>(qs, base, row_stride, 0, h, heads, rope_cos, rope_sin, (t + 1) * kTileQ, kTileQ, seq,
                        threadIdx.x, kSoftThreads);
        fence_proxy_async_smem();
        mbar_arrive(q_full);
      }
      // -- epilogue: O / l -> 16-bit output row, row |max|
      if (!__all_sync(0xffffffffu, mbar_wait(o_full, 1, abort_flag))) break;
      tc_fence_after();
      const float inv = 1.0f / l;
      uint32_t am = 0;
      uint16_t* dst = out + (static_cast<size_t>(b) * seq + query) * c + h * kD;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t v[32], w[16];
        tmem_ld32(lane_base + kOCol + half * 32, v);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          w[i] = pack2(__uint_as_float(v[2 * i]) * inv, __uint_as_float(v[2 * i + 1]) * inv, F16);
          am = __vmaxu2(am, w[i] & 0x7fff7fffu);
        }
        if (query < seq) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(dst + half * 32)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
      if (row_amax != nullptr && query < seq) {
        const uint32_t m16 = max(am & 0xffffu, am >> 16);
        atomicMax(row_amax + static_cast<size_t>(b) * seq + query,
                  F16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m16))) : (m16 << 16));
      }
      tc_fence_before();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && *abort_flag) record_status(status, KB_STATUS_TIMEOUT, KB_NO_LAYER);
  if (warp == 4) tmem_dealloc(tmem, kTmemCols);
}

template <bool F16>
int launch_tc(const uint16_t* qkv, const float* cos_t, const float* sin_t, uint16_t* out, int batch, int seq,
              int heads, float scale, uint32_t* row_amax, unsigned* status, cudaStream_t stream) {
  auto kern = attention_tc_kernel<F16>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "attention smem attribute");
    configured.fetch_or(bit);
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  kern<<<batch * heads, kTcThreads, kSmemBytes, stream>>>(qkv, cos_t, sin_t, out, seq, heads, scale_log2, row_amax,
                                                          status);
  return check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace

// head_dim 64 and 192 < seq <= 368 (the 361-token board): tcgen05 kernel.
bool attention_tc_supported(int seq, int head_dim) { return head_dim == kD && seq > kHalfA && seq <= kKeysPad; }

int attention_tc_launch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out, int batch,
                        int seq, int heads, float scale, int f16, cudaStream_t stream, uint32_t* row_amax,
                        unsigned* status) {
  return f16 ? launch_tc<true>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, status, stream)
             : launch_tc<false>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, status, stream);
}

}  // namespace kb
