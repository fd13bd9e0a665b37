// tcgen05 GEMM for sm_100a: C[m,n] = A[m,k] * B[n,k]^T, both operands K-major.
//
// This is the B200 replacement for the reference's projection GEMMs: the
// cuBLASLt INT8 call (crates/kata_nn/src/backends/int8.rs:383-599), its
// dequant kernels (cuda-kernels/int8_ops.cu:178-238) and the FP16 outer
// linears.  One persistent CTA per SM runs three warp roles:
//   warp 0      TMA producer: 128-byte-swizzled {128 B x rows} tiles of A and B
//               into a STAGES-deep shared-memory ring (one mbarrier pair per slot);
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, 32 B of K
//               per instruction) into one of two TMEM accumulators and commits
//               ring slots / accumulators back through mbarriers;
//   warps 2-17  epilogue: tcgen05.ld of the accumulator (one TMEM lane = one
//               output row per thread; four warps per 32-lane quarter, each taking
//               a quarter of the tile's columns, 16 columns per step), dequant /
//               bias / activation / rotary / residual / row-amax, then 16-bit
//               results go through a swizzled 2 KiB shared-memory staging tile
//               per warp and a TMA store.
// The double-buffered accumulator lets the epilogue of tile i overlap the MMAs
// of tile i+1.  Every wait is bounded (kb_ptx.cuh); a timeout records
// KB_STATUS_TIMEOUT in the status word and the kernel returns.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>

#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

constexpr int kBM = 128;
constexpr int kBKBytes = 128;  // one 128-byte swizzle row of K per stage
// Epilogue warps: 16 (four per TMEM lane quarter) for the arithmetic-heavy
// 16-bit epilogues (bias + activation, rotary, SwiGLU) and for the residual
// adds of short-K projections, where draining the epilogue bounds the tile; 8
// for the others (long-K residual adds keep the deeper operand ring; plain
// fp32 / int32 outputs).  64-column tiles (small M) always take 8: one
// 32-column chunk per warp.
template <int EPI, int DEEP, int BN>
constexpr int epi_warps() {
  return BN > 64 && (EPI == 3 /* kEpi16 */ || EPI == 7 /* kEpiRope16 */ || EPI == 5 /* kEpiSwiGLU16 */ ||
                     ((EPI == 4 /* kEpiRes16 */ || EPI == 2 /* kEpiResF32 */) && DEEP))
             ? 16
             : 8;
}
constexpr int gemm_threads(int ew) { return 64 + 32 * ew; }
constexpr int kStageTile = 32 * 64;  // one 32x32 16-bit staging tile (2 KiB)
constexpr int kSmemLimit = 227 * 1024;

// SB = staging tiles per epilogue warp (stores in flight per warp).  Short-K
// GEMMs are bound by how fast the epilogue can drain results, so they trade
// one ring stage for two staging tiles per warp; long-K GEMMs keep the deeper
// ring and one staging tile.
constexpr uint32_t pow2_cols(uint32_t c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }

template <int KIND, int BN, int SB, int EW>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = BN * kBKBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // MXFP8: one 512-byte scale tile of A (128 rows x 4 K blocks) and BN/128 of B
  // per stage, each copied to 4 TMEM columns by tcgen05.cp.
  static constexpr int kSfBytes = KIND == kGemmMXF8 ? 512 + 512 * (BN / 128) : 0;
  static constexpr int kSfCols = KIND == kGemmMXF8 ? 4 + 4 * (BN / 128) : 0;
  static constexpr int kStagingBytes = EW * SB * kStageTile;
  static constexpr int kStages = (kSmemLimit - kStagingBytes - 1024 - 512) / (kStageBytes + kSfBytes);
  static constexpr int kRingBytes = kStages * kStageBytes;
  static constexpr int kSfRingBytes = kStages * kSfBytes;
  static constexpr uint32_t kTmemCols = pow2_cols(2 * BN + kStages * kSfCols);
  static constexpr int kSmemBytes =
      kRingBytes + kStagingBytes + kSfRingBytes + 1024 /*align*/ + 512 /*barriers*/;
  static_assert(kStages >= 3, "ring too shallow");
  static_assert(2 * BN + kStages * kSfCols <= 512, "TMEM columns exceeded");
};

// Shared-memory descriptor of one 512-byte scale tile for tcgen05.cp
// .32x128b: 32 rows of 16 bytes, no swizzle, 8-row core groups 128 bytes apart.
__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(128 >> 4) << 32) |
         (1ull << 46);
}

template <int KIND>
__device__ __forceinline__ float acc_value(uint32_t bits, float sa, float sw) {
  if constexpr (KIND == kGemmI8) {
    return __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(bits)), sa), sw);
  } else {
    return __uint_as_float(bits);
  }
}

template <int N>
__device__ __forceinline__ void load_vecn(const float* p, int col0, int n, float (&dst)[N]) {
  if (p == nullptr) {
#pragma unroll
    for (int i = 0; i < N; ++i) dst[i] = 0.0f;
    return;
  }
  if (col0 + N <= n && (reinterpret_cast<uintptr_t>(p + col0) & 15) == 0) {
    const float4* q = reinterpret_cast<const float4*>(p + col0);
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const float4 t = __ldg(q + i);
      dst[4 * i] = t.x;
      dst[4 * i + 1] = t.y;
      dst[4 * i + 2] = t.z;
      dst[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) dst[i] = col0 + i < n ? __ldg(p + col0 + i) : 0.0f;
  }
}

// Eight floats from a 32-byte aligned global address in one 256-bit load
// (read-only path): one L1 wavefront per 32-byte sector instead of one per
// 16 bytes when the lanes of a warp read different rows.
__device__ __forceinline__ void ldg256(const float* p, float* r) {
  asm volatile("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7])
               : "l"(p));
}

// N floats (N a multiple of 8) from a 32-byte aligned address, no checks
// (GemmArgs::cols_vec), in 256-bit loads.
template <int N>
__device__ __forceinline__ void load_vec_aligned(const float* p, float (&dst)[N]) {
#pragma unroll
  for (int i = 0; i < N / 8; ++i) ldg256(p + 8 * i, dst + 8 * i);
}


template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 16) tmem_ld16(taddr, r);
  else tmem_ld32(taddr, r);
}

__device__ __forceinline__ void load_vec32(const float* p, int col0, int n, float (&dst)[32]) {
  if (p == nullptr) {
#pragma unroll
    for (int i = 0; i < 32; ++i) dst[i] = 0.0f;
    return;
  }
  if (col0 + 32 <= n && (reinterpret_cast<uintptr_t>(p + col0) & 15) == 0) {
    const float4* q = reinterpret_cast<const float4*>(p + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = __ldg(q + i);
      dst[4 * i] = t.x;
      dst[4 * i + 1] = t.y;
      dst[4 * i + 2] = t.z;
      dst[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) dst[i] = col0 + i < n ? __ldg(p + col0 + i) : 0.0f;
  }
}


__device__ __forceinline__ float2 unpack16x2(uint32_t w, bool f16) {
  if (f16) return make_float2(from_f16(static_cast<uint16_t>(w & 0xffffu)), from_f16(static_cast<uint16_t>(w >> 16)));
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// 32-bit float bits of the larger |half| held in a packed pair of |16-bit| values.
__device__ __forceinline__ uint32_t amax16_to_f32bits(uint32_t m2, bool f16) {
  const uint32_t m = max(m2 & 0xffffu, m2 >> 16);
  return f16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m))) : (m << 16);
}

__device__ __forceinline__ void store16x32(uint16_t* dst, const uint32_t (&hw)[16], int valid,
                                           bool vec) {
  if (vec && valid == 32) {
    uint4* q = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = static_cast<uint16_t>(i & 1 ? hw[i / 2] >> 16 : hw[i / 2] & 0xffffu);
  }
}

__device__ __forceinline__ void load16x32(const uint16_t* src, uint32_t (&hw)[16], int valid,
                                          bool vec) {
  if (vec && valid == 32) {
    const uint4* q = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 t = q[i];
      hw[4 * i] = t.x;
      hw[4 * i + 1] = t.y;
      hw[4 * i + 2] = t.z;
      hw[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t lo = 2 * i < valid ? src[2 * i] : 0u;
      const uint32_t hi = 2 * i + 1 < valid ? src[2 * i + 1] : 0u;
      hw[i] = lo | (hi << 16);
    }
  }
}

// Per-warp output path for 32 rows x 32 columns of 16-bit results.  With a TMA
// output map the thread's row goes into a 64-byte-swizzled staging tile (16-byte
// chunk c of row r at c ^ ((r >> 1) & 3): conflict-free, and exactly the layout a
// SWIZZLE_64B tensor store reads), then lane 0 issues one bulk tensor store.
// With two staging tiles per warp a store overlaps the next chunk.
struct Out16 {
  const CUtensorMap* map;
  uint8_t* stage;  // this warp's SB staging tiles
  int sb;          // staging tile to use next
};

template <int SB>
__device__ __forceinline__ void emit16(Out16& o, const GemmArgs& g, const uint32_t (&hw)[16], int row,
                                       int row0q, int col0, int lane, bool row_ok, int valid) {
  if (o.map != nullptr) {
    uint8_t* buf = o.stage + o.sb * kStageTile;
    if (lane == 0) bulk_wait_read<SB - 1>();
    __syncwarp();
    const int sw = (lane >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(buf + lane * 64 + ((c ^ sw) << 4)) =
          make_uint4(hw[4 * c], hw[4 * c + 1], hw[4 * c + 2], hw[4 * c + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(o.map, buf, col0, row0q);
      bulk_commit();
    }
    o.sb = o.sb + 1 == SB ? 0 : o.sb + 1;
  } else if (row_ok) {
    uint16_t* dst = static_cast<uint16_t*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
    store16x32(dst, hw, valid, (reinterpret_cast<uintptr_t>(dst) & 15) == 0);
  }
}

// Dequantised pair (i, i+1) of a 32-column chunk: (f32(dot) * sa) * sw, or the
// fp32 accumulator itself for the bf16 / MXFP8 kinds.
template <int KIND>
__device__ __forceinline__ float2 acc_pair(const uint32_t (&v)[32], int i, float sa, const float (&sw)[32]) {
  if constexpr (KIND == kGemmI8) {
    // Scalar rounded multiplies: a packed multiply followed by the bias add
    // may be contracted into a fused multiply-add by the assembler, which
    // would change the rounding.
    return make_float2(
        __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[2 * i])), sa), sw[2 * i]),
        __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[2 * i + 1])), sa), sw[2 * i + 1]));
  } else {
    return make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
  }
}

// Pair (i, i+1) of an N-column piece of a chunk (same arithmetic as acc_pair).
// Scalar rounded multiplies: a packed multiply followed by an add (a bias, the
// residual) may be fused by the assembler, which changes the rounding of a few
// outputs (measured).
template <int KIND, int N>
__device__ __forceinline__ float2 acc_pairn(const uint32_t (&v)[N], int i, float sa, const float (&sw)[N]) {
  if constexpr (KIND == kGemmI8) {
    return make_float2(
        __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[2 * i])), sa), sw[2 * i]),
        __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[2 * i + 1])), sa), sw[2 * i + 1]));
  } else {
    return make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
  }
}

// Pair (i, i+1) plus the bias.  INT8: fma(f32(dot)*sa, sw, bias): the first
// product rounded, then one fused multiply-add (packed; a multiply feeding an
// explicit FMA leaves nothing for the assembler to contract).  Other kinds:
// acc + bias.
template <int KIND, int N>
__device__ __forceinline__ float2 acc_bias_pairn(const uint32_t (&v)[N], int i, float sa, const float (&sw)[N],
                                                 const float (&bias)[N]) {
  if constexpr (KIND == kGemmI8) {
    const float2 d = make_float2(static_cast<float>(static_cast<int>(v[2 * i])),
                                 static_cast<float>(static_cast<int>(v[2 * i + 1])));
    return fma2(mul2(d, make_float2(sa, sa)), make_float2(sw[2 * i], sw[2 * i + 1]),
                make_float2(bias[2 * i], bias[2 * i + 1]));
  } else {
    return make_float2(__fadd_rn(__uint_as_float(v[2 * i]), bias[2 * i]),
                       __fadd_rn(__uint_as_float(v[2 * i + 1]), bias[2 * i + 1]));
  }
}

template <int KIND, int BN, int EPI, int ACT, int SB, int EW>
__global__ void __launch_bounds__(gemm_threads(EW), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_out, const GemmArgs g, const int use_tma_out) {
  constexpr int kEpiWarps = EW;
  constexpr int kParts = kEpiWarps / 4;  // epilogue warps per TMEM lane quarter
  // Columns per accumulator read: 16 with 16 epilogue warps (register budget), else 32.
  constexpr int kSub = kEpiWarps == 16 ? 16 : 32;
  constexpr int kHalves = 32 / kSub;
  using Cfg = GemmCfg<KIND, BN, SB, kEpiWarps>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kElemBytes = (KIND == kGemmBF16) ? 2 : 1;
  constexpr int kBKElems = kBKBytes / kElemBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint8_t* staging = smem + Cfg::kRingBytes;
  uint8_t* sf_ring = staging + Cfg::kStagingBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sf_ring + Cfg::kSfRingBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* res_bar = tempty + 3;  // [epilogue warp][SB]: residual tiles landed (residuals through TMA)
  static_assert((2 * kStages + 5 + kEpiWarps * SB) * 8 <= 512, "barrier area exceeded");

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k_blocks = (g.k + kBKElems - 1) / kBKElems;
  const int tiles_m = (g.m + kBM - 1) / kBM;
  const int tiles_n = (g.n + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const uint64_t wlim = g.wait_limit_ns ? g.wait_limit_ns : kWaitLimitNs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    if constexpr (EPI == kEpiRes16 || EPI == kEpiResF32 || EPI == kEpiF32)
      for (int i = 0; i < kEpiWarps * SB; ++i) mbar_init(&res_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (use_tma_out) tma_prefetch_desc(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t issued = 0, issued_par = 0;  // per ring slot: load issued, its phase parity
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mb = tile / tiles_n, nb = tile % tiles_n;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, wlim)) {
            ok = false;
            break;
          }
          uint8_t* sa = ring + s * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes + Cfg::kSfBytes);
          tma_load_2d(sa, &tmap_a, &full[s], kb * kBKElems, mb * kBM);
          tma_load_2d(sa + Cfg::kABytes, &tmap_b, &full[s], kb * kBKElems, nb * BN);
          if constexpr (KIND == kGemmMXF8) {
            // Scale tiles: tile (row/128, kblock) of the packed layout is 512
            // contiguous bytes; k_blocks tiles per 128-row band.
            uint8_t* sf = sf_ring + s * Cfg::kSfBytes;
            bulk_load(sf, g.sfa + (static_cast<size_t>(mb) * k_blocks + kb) * 512u, 512u, &full[s]);
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              bulk_load(sf + 512 * (j + 1),
                        g.sfb + (static_cast<size_t>(nb * (BN / 128) + j) * k_blocks + kb) * 512u, 512u, &full[s]);
          }
          issued |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {
        // Aborted: let the copies already in flight land before the CTA exits
        // (each wait is bounded again by its own time limit).
        int local_abort = 0;
        for (int t = 0; t < kStages; ++t)
          if (issued & (1u << t)) mbar_wait(&full[t], (issued_par >> t) & 1u, &local_abort);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      // kGemmBF16 with ab_f16: both operands binary16 (format 0) instead of
      // bfloat16 (format 1); A and B always share one type.
      const uint32_t idesc =
          make_idesc<KIND>(BN) & ~(KIND == kGemmBF16 && g.ab_f16 ? ((7u << 7) | (7u << 10)) : 0u);
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      int last_s = -1;  // ring slot and phase of the last MMA commit
      uint32_t last_ph = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag, wlim)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, wlim)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + s * Cfg::kStageBytes);
          const uint64_t adesc = sw128_desc(a_addr);
          const uint64_t bdesc = sw128_desc(a_addr + Cfg::kABytes);
          if constexpr (KIND == kGemmMXF8) {
            // Scale tiles -> TMEM (4 columns each, replicated to all four lane
            // quarters); tcgen05.cp and tcgen05.mma from this thread execute in
            // issue order.  Column c, byte b of lane l then holds the scale of
            // row 32c + l%32, K block b: the MMA of K block kk selects byte kk.
            const uint32_t tsf = tmem_base + static_cast<uint32_t>(2 * BN + s * Cfg::kSfCols);
            const uint32_t sf_addr = smem_u32(sf_ring + s * Cfg::kSfBytes);
#pragma unroll
            for (int j = 0; j < 1 + BN / 128; ++j) tmem_cp_32x128_warpx4(tsf + 4 * j, sf_desc(sf_addr + 512 * j));
#pragma unroll
            for (int kk = 0; kk < kBKBytes / 32; ++kk) {
              const uint32_t id = idesc | (static_cast<uint32_t>(kk) << 29) | (static_cast<uint32_t>(kk) << 4);
              mma_issue<KIND>(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, id, (kb | kk) != 0, tsf, tsf + 4);
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < kBKBytes / 32; ++kk) {
              // +32 bytes along K inside the swizzle atom = +2 in the address field.
              mma_issue<KIND>(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0, 0, 0);
            }
          }
          tc_commit(&empty[s]);
          last_s = s;
          last_ph = ph;
          if (++s == kStages) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1;
      }
      if (!ok && last_s >= 0) {
        // Aborted: the MMAs already issued must finish before the TMEM is
        // freed.  The last commit (to empty[last_s], phase last_ph) tracks
        // every MMA this thread issued before it.
        int local_abort = 0;
        mbar_wait(&empty[last_s], last_ph, &local_abort);
      }
    }
  } else {
    // ---------------- epilogue warps: kParts per TMEM lane quarter, each
    // 1/kParts of the tile's columns, processed 16 columns at a time
    const int e = warp - 2;          // 0..kEpiWarps-1
    const int quarter = warp & 3;    // TMEM lanes this warp may access: 32*quarter..+31
    const int part = e >> 2;         // which share of the tile's columns
    Out16 o{use_tma_out ? &tmap_out : nullptr, staging + e * SB * kStageTile, 0};
    const bool f16 = (EPI == kEpiF16) ? true : (g.out_f16 != 0);
    int acc = 0;
    uint32_t aph = 0;
    bool handled = false;
    if constexpr (EPI == kEpiRes16 || EPI == kEpiResF32 || EPI == kEpiF32) {
      // (kEpiF32 takes this path only with a residual, which the host has
      // checked is the output itself)
      if (use_tma_out && (EPI != kEpiF32 || g.residual != nullptr)) {
        handled = true;
        // ---- residual through shared memory.  Each warp walks a stream of
        // chunks of 32 rows x 64 bytes (32 16-bit or 16 fp32 columns; its
        // columns of each tile, tile after tile); the residual of a chunk is
        // TMA-loaded into a staging tile kLook chunks ahead (the stream runs
        // across tiles, so the next tile's first residuals are in flight while
        // this one finishes), the dequantised accumulator is added in place and
        // the tile is TMA-stored back with the same tensor map (64-byte
        // swizzle, out-of-range rows and columns read as zero and are clipped
        // on the store).
        constexpr bool kF32 = EPI != kEpiRes16;
        constexpr int kCC = kF32 ? 16 : 32;  // columns per chunk
        constexpr int kLook = SB >= 4 ? 2 : 1;
        static_assert(SB - kLook - 1 >= 0, "residual staging needs SB > kLook");
        constexpr int kChunksR = BN / kCC / kParts;
        uint8_t* stage = staging + e * SB * kStageTile;
        uint64_t* rbar = res_bar + e * SB;
        auto chunk_col = [&](int t, int jj) { return (t % tiles_n) * BN + (part * kChunksR + jj) * kCC; };
        int ld_tile = blockIdx.x, ld_jj = 0, ld_n = 0;  // next chunk to load; loads issued
        auto issue_load = [&]() {  // lane 0
          while (ld_tile < num_tiles && chunk_col(ld_tile, ld_jj) >= g.n)
            if (++ld_jj == kChunksR) ld_jj = 0, ld_tile += gridDim.x;
          if (ld_tile >= num_tiles) return;
          const int b = ld_n % SB;
          mbar_arrive_expect_tx(&rbar[b], kStageTile);
          tma_load_2d(stage + b * kStageTile, &tmap_out, &rbar[b], chunk_col(ld_tile, ld_jj),
                      (ld_tile / tiles_n) * kBM + quarter * 32);
          ++ld_n;
          if (++ld_jj == kChunksR) ld_jj = 0, ld_tile += gridDim.x;
        };
        if (lane == 0)
          for (int i = 0; i < kLook; ++i) issue_load();
        int sq = 0;  // chunks processed
        bool ok = true;
        const bool with_bias = g.bias != nullptr;
        for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
          const int mb = tile / tiles_n;
          const int row0q = mb * kBM + quarter * 32;
          const int row = row0q + lane;
          const bool row_ok = row < g.m;
          float sa = 1.0f;
          if constexpr (KIND == kGemmI8) sa = row_ok ? __ldg(g.row_scale + row) : 0.0f;
          if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aph, abort_flag, wlim))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 static_cast<uint32_t>(acc * BN);
          bool nonfinite = false;
#pragma unroll 1
          for (int jj = 0; jj < kChunksR; ++jj) {
            const int j = part * kChunksR + jj;
            const int col0 = chunk_col(tile, jj);
            if (col0 >= g.n) continue;  // warp-uniform
            // the load kLook chunks ahead reuses the staging tile of chunk
            // sq + kLook - SB, whose store must have read it
            if (lane == 0) {
              bulk_wait_read<SB - kLook - 1>();
              issue_load();
            }
            uint8_t* buf = stage + (sq % SB) * kStageTile;
            const int swz = (lane >> 1) & 3;
            uint32_t amax2 = 0;
            if constexpr (kF32) {
              // 16 fp32 columns: four 16-byte cells of four values.  The same
              // arithmetic as the direct-store fp32 epilogues.
              uint32_t v[16];
              tmem_ldn<16>(taddr + j * kCC, v);
              float sw[16], bias[16];
              const bool add_bias = EPI == kEpiF32 && with_bias;  // warp-uniform
              if (g.cols_vec) {  // warp-uniform
                if constexpr (KIND == kGemmI8) load_vec_aligned<16>(g.col_scale + col0, sw);
                if (add_bias) load_vec_aligned<16>(g.bias + col0, bias);
              } else {
                if constexpr (KIND == kGemmI8) load_vecn<16>(g.col_scale, col0, g.n, sw);
                if (add_bias) load_vecn<16>(g.bias, col0, g.n, bias);
              }
              tmem_ld_wait();
              if (!__all_sync(0xffffffffu, mbar_wait(&rbar[sq % SB], (sq / SB) & 1, abort_flag, wlim))) {
                ok = false;
                break;
              }
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                float4* cell = reinterpret_cast<float4*>(buf + lane * 64 + ((c ^ swz) << 4));
                const float4 r4 = *cell;
                const float r[4] = {r4.x, r4.y, r4.z, r4.w};
                float y[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const int i = 4 * c + q;
                  float x;
                  if (EPI == kEpiResF32 || !add_bias)
                    x = acc_value<KIND>(v[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f);
                  else if (KIND == kGemmI8)
                    x = __fmaf_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[i])), sa), sw[i], bias[i]);
                  else
                    x = __fadd_rn(acc_value<KIND>(v[i], sa, 1.0f), bias[i]);
                  y[q] = __fadd_rn(r[q], x);
                  if constexpr (KIND == kGemmMXF8) nonfinite |= row_ok && col0 + i < g.n && !isfinite(y[q]);
                }
                *cell = make_float4(y[0], y[1], y[2], y[3]);
              }
            } else {
            // The chunk's 32 columns in kHalves pieces of kSub (16 with 16
            // epilogue warps: the register budget of a 576-thread CTA).
#pragma unroll
            for (int hh = 0; hh < kHalves; ++hh) {
              const int c0 = col0 + hh * kSub;
              uint32_t v[kSub];
              tmem_ldn<kSub>(taddr + j * 32 + hh * kSub, v);
              float sw[kSub], bias[kSub];
              if (g.cols_vec) {  // warp-uniform
                if constexpr (KIND == kGemmI8) load_vec_aligned<kSub>(g.col_scale + c0, sw);
                if (with_bias) load_vec_aligned<kSub>(g.bias + c0, bias);
              } else {
                if constexpr (KIND == kGemmI8) load_vecn<kSub>(g.col_scale, c0, g.n, sw);
                if (with_bias) load_vecn<kSub>(g.bias, c0, g.n, bias);
              }
              tmem_ld_wait();
              if (hh == 0 && !__all_sync(0xffffffffu, mbar_wait(&rbar[sq % SB], (sq / SB) & 1, abort_flag, wlim))) {
                ok = false;
                break;
              }
#pragma unroll
              for (int c = 0; c < kSub / 8; ++c) {
                const int cc = hh * (kSub / 8) + c;  // 16-byte cell of the 32-column chunk
                uint4* cell = reinterpret_cast<uint4*>(buf + lane * 64 + ((cc ^ swz) << 4));
                const uint4 r4 = *cell;
                const uint32_t rw[4] = {r4.x, r4.y, r4.z, r4.w};
                uint32_t ow[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const int i = 4 * c + q;
                  const float2 x = with_bias ? acc_bias_pairn<KIND, kSub>(v, i, sa, sw, bias)
                                             : acc_pairn<KIND, kSub>(v, i, sa, sw);
                  const float2 r = unpack16x2(rw[q], f16);
                  ow[q] = pack16x2(make_float2(__fadd_rn(r.x, x.x), __fadd_rn(r.y, x.y)), f16);
                  if constexpr (KIND == kGemmMXF8) amax2 = __vmaxu2(amax2, ow[q] & 0x7fff7fffu);
                }
                *cell = make_uint4(ow[0], ow[1], ow[2], ow[3]);
              }
            }
            }
            if (!ok) break;
            if constexpr (KIND == kGemmMXF8)
              nonfinite |= row_ok && max(amax2 & 0xffffu, amax2 >> 16) >= (f16 ? 0x7c00u : 0x7f80u);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_out, buf, col0, row0q);
              bulk_commit();
            }
            ++sq;
          }
          if (!ok) break;
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
          if constexpr (KIND == kGemmMXF8) {
            if (__any_sync(0xffffffffu, nonfinite) && lane == 0)
              record_status(g.status, KB_STATUS_OUTPUT_NONFINITE, g.layer);
          }
          acc ^= 1;
          if (acc == 0) aph ^= 1;
        }
        if (lane == 0) {
          // residual loads still in flight (an aborted walk) land before exit
          int local_abort = 0;
          for (int i = sq; i < ld_n; ++i) mbar_wait(&rbar[i % SB], (i / SB) & 1, &local_abort);
          bulk_wait_all();
        }
      }
    }
    if (!handled) {
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mb = tile / tiles_n, nb = tile % tiles_n;
      const int row0q = mb * kBM + quarter * 32;
      const int row = row0q + lane;
      const bool row_ok = row < g.m;
      int token = 0;
      if constexpr (EPI == kEpiRope16) token = row_ok ? row % g.rope_seq : 0;
      // the row scale is loaded while the accumulator is still being computed
      float sa = 1.0f;
      if constexpr (KIND == kGemmI8 && EPI != kEpiI32) sa = row_ok ? __ldg(g.row_scale + row) : 0.0f;
      // Rotary tables (kEpiRope16) of the next kSub-column piece, loaded one
      // piece ahead, the tile's first while the accumulator is being computed:
      // they come from L2, and a piece of arithmetic covers most of that latency.
      // (256-column tiles only: the narrower tiles' epilogues would spill with
      // the second set of table registers, and load each piece's own tables.)
      constexpr bool kRopeAhead = BN == 256;
      float rc_n[kSub / 2], rs_n[kSub / 2];
      auto rope_load = [&](int c0) {
        if constexpr (EPI == kEpiRope16) {
          if (row_ok && c0 < g.rope_cols) {
            // [head * pairs + pair][token]: pair q of Q or K column cc (even)
            // is entry cc / 2 + q; the warp's 32 rows are consecutive tokens,
            // so each load reads one contiguous run.
            const int half_cols = g.rope_cols / 2;
            const int cc = c0 < half_cols ? c0 : c0 - half_cols;
            const float* pc = g.rope_cos + static_cast<size_t>(cc / 2) * g.rope_seq + token;
            const float* ps = g.rope_sin + static_cast<size_t>(cc / 2) * g.rope_seq + token;
#pragma unroll
            for (int i = 0; i < kSub / 2; ++i) {
              rc_n[i] = __ldg(pc + static_cast<size_t>(i) * g.rope_seq);
              rs_n[i] = __ldg(ps + static_cast<size_t>(i) * g.rope_seq);
            }
          } else {
#pragma unroll
            for (int i = 0; i < kSub / 2; ++i) rc_n[i] = 1.0f, rs_n[i] = 0.0f;
          }
        }
      };
      if constexpr (EPI == kEpiRope16 && kRopeAhead) rope_load(nb * BN + part * (BN / 32 / kParts) * 32);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aph, abort_flag, wlim))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      uint32_t amax = 0;
      bool nonfinite = false;  // MXFP8: output finite check (mxfp8.cu:81-88 in the reference)
      if constexpr (EPI == kEpiSwiGLU16) {
        // Tile columns [0, BN/2) are gate channels, [BN/2, BN) the matching up
        // channels (the dual weight is interleaved per tile at load).
        constexpr int kChunks = BN / 64 / kParts;
#pragma unroll 1
        for (int jj = 0; jj < kChunks; ++jj) {
          const int j = part * kChunks + jj;
          const int gcol0 = nb * BN + j * 32;
          const int ocol0 = nb * (BN / 2) + j * 32;
          if (ocol0 >= g.n_out) continue;  // warp-uniform
          const int valid = min(32, g.n_out - ocol0);
          uint32_t hw[16];
#pragma unroll
          for (int hh = 0; hh < kHalves; ++hh) {
            uint32_t vg[kSub], vu[kSub];
            tmem_ldn<kSub>(taddr + j * 32 + hh * kSub, vg);
            tmem_ldn<kSub>(taddr + BN / 2 + j * 32 + hh * kSub, vu);
            float swg[kSub], swu[kSub];
            if constexpr (KIND == kGemmI8) {
              if (g.cols_vec) {  // warp-uniform
                load_vec_aligned<kSub>(g.col_scale + gcol0 + hh * kSub, swg);
                load_vec_aligned<kSub>(g.col_scale + gcol0 + BN / 2 + hh * kSub, swu);
              } else {
                load_vecn<kSub>(g.col_scale, gcol0 + hh * kSub, g.n, swg);
                load_vecn<kSub>(g.col_scale, gcol0 + BN / 2 + hh * kSub, g.n, swu);
              }
            }
            tmem_ld_wait();
            // Pairs of columns: gate and up dequantised and rounded to binary16
            // (the reference's fp16 boundary), SiLU of the gate, the product
            // rounded to binary16.  The output is always binary16.
#pragma unroll
            for (int i = 0; i < kSub / 2; ++i) {
              const float2 gq = acc_pairn<KIND, kSub>(vg, i, sa, swg);
              const float2 uq = acc_pairn<KIND, kSub>(vu, i, sa, swu);
              const float2 gv = unpack16x2(pack16x2(gq, true), true);
              const float2 uv = unpack16x2(pack16x2(uq, true), true);
              hw[hh * (kSub / 2) + i] = pack16x2(mul2(uv, kb_silu2(gv)), true);
            }
          }
          if (g.row_amax != nullptr) {  // warp-uniform
            // Columns past the matrix edge (a partial chunk, warp-uniform) are
            // zeroed first (the tensor store clips them anyway), so one
            // max-of-|x| per pair covers every chunk; sign bits masked once.
            if (valid < 32) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                hw[i] &= 2 * i + 1 < valid ? 0xffffffffu : (2 * i < valid ? 0x0000ffffu : 0u);
            }
            uint32_t amax2 = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) amax2 = hmax_abs2<true>(amax2, hw[i]);
            amax = max(amax, amax16_to_f32bits(amax2 & 0x7fff7fffu, true));
          }
          emit16<SB>(o, g, hw, row, row0q, ocol0, lane, row_ok, valid);
        }
      } else {
        constexpr int kChunks = BN / 32 / kParts;
        // Residual epilogue: the 16-bit residual of the next chunk is loaded
        // while the current one is computed (one chunk of prefetch).
        uint32_t res_next[16];
        auto load_res = [&](int jj2) {
          const int c = nb * BN + (part * kChunks + jj2) * 32;
          if (row_ok && c < g.n) {
            const uint16_t* src = static_cast<const uint16_t*>(g.out) + static_cast<size_t>(row) * g.ldo + c;
            load16x32(src, res_next, min(32, g.n - c), (reinterpret_cast<uintptr_t>(src) & 15) == 0);
          }
        };
        if constexpr (EPI == kEpiRes16) load_res(0);
#pragma unroll 1
        for (int jj = 0; jj < kChunks; ++jj) {
          const int j = part * kChunks + jj;
          const int col0 = nb * BN + j * 32;
          if (col0 >= g.n) continue;  // warp-uniform
          const int valid = min(32, g.n - col0);
          if constexpr (EPI == kEpiF16 || EPI == kEpi16 || EPI == kEpiRes16 || EPI == kEpiRope16) {
            uint32_t hw[16];
            if constexpr (EPI == kEpiRes16) {
#pragma unroll
              for (int i = 0; i < 16; ++i) hw[i] = res_next[i];
              if (jj + 1 < kChunks) load_res(jj + 1);
            }
            // (the rotary epilogue takes no bias: its registers hold the tables)
            const bool with_bias = EPI != kEpiF16 && EPI != kEpiRope16 && g.bias != nullptr;  // warp-uniform
#pragma unroll
            for (int hh = 0; hh < kHalves; ++hh) {
              const int c0 = col0 + hh * kSub;
              // The accumulator read and this piece's column scales, bias and
              // rotary tables are all in flight before the wait.
              uint32_t v[kSub];
              tmem_ldn<kSub>(taddr + j * 32 + hh * kSub, v);
              float sw[kSub];
              float bias[kSub];
              if (g.cols_vec) {  // warp-uniform
                if constexpr (KIND == kGemmI8) load_vec_aligned<kSub>(g.col_scale + c0, sw);
                if (with_bias) load_vec_aligned<kSub>(g.bias + c0, bias);
              } else {
                if constexpr (KIND == kGemmI8) load_vecn<kSub>(g.col_scale, c0, g.n, sw);
                if (with_bias) load_vecn<kSub>(g.bias, c0, g.n, bias);
              }
              // Rotary tables of these kSub / 2 pairs (kEpiRope16, Q and K
              // columns; loaded one piece ahead), then the next piece's loads:
              // the other half of this chunk, or the next chunk's first.
              float rc[kSub / 2], rs[kSub / 2];
              bool rope = false;
              if constexpr (EPI == kEpiRope16) {
                rope = col0 < g.rope_cols;  // warp-uniform
                if constexpr (!kRopeAhead) rope_load(c0);
#pragma unroll
                for (int i = 0; i < kSub / 2; ++i) rc[i] = rc_n[i], rs[i] = rs_n[i];
                if constexpr (kRopeAhead) {
                  if (hh + 1 < kHalves) rope_load(c0 + kSub);
                  else if (jj + 1 < kChunks) rope_load(col0 + 32);
                }
              }
              tmem_ld_wait();
              // Separate unrolled bodies with and without bias (warp-uniform
              // choice), so a bias-free projection issues no adds.
              auto finish = [&](auto bias_tag) {
                constexpr bool kBias = decltype(bias_tag)::value;
#pragma unroll
                for (int i = 0; i < kSub / 2; ++i) {
                  float2 x = kBias ? acc_bias_pairn<KIND, kSub>(v, i, sa, sw, bias) : acc_pairn<KIND, kSub>(v, i, sa, sw);
                  uint32_t& out = hw[hh * (kSub / 2) + i];
                  if constexpr (EPI == kEpiRes16) {
                    const float2 r = unpack16x2(out, f16);
                    out = pack16x2(make_float2(__fadd_rn(r.x, x.x), __fadd_rn(r.y, x.y)), f16);
                  } else if constexpr (EPI == kEpiRope16) {
                    if (rope) {
                      // (x, y) -> (x c - y s, x s + y c), each product and sum rounded
                      const float c = rc[i], sn = rs[i];
                      x = make_float2(__fsub_rn(__fmul_rn(x.x, c), __fmul_rn(x.y, sn)),
                                      __fadd_rn(__fmul_rn(x.x, sn), __fmul_rn(x.y, c)));
                    }
                    out = pack16x2(x, f16);
                  } else {
                    out = pack16x2(apply_act2<ACT>(x), f16);
                  }
                }
              };
              if constexpr (EPI == kEpiRope16)
                finish(std::false_type{});
              else if (with_bias)
                finish(std::true_type{});
              else
                finish(std::false_type{});
            }
            // |16-bit| maximum of the stored values: the next quantiser's row
            // amax, and the MXFP8 output finite check (Inf/NaN sort highest).
            if (KIND == kGemmMXF8 || (EPI != kEpiRes16 && g.row_amax != nullptr)) {
              uint32_t amax2 = 0;
              if (valid == 32) {
                // max(|a|, |b|) per 16-bit lane in one instruction (NaN wins;
                // the sign bits are masked off below)
                if (f16) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) amax2 = hmax_abs2<true>(amax2, hw[i]);
                } else {
#pragma unroll
                  for (int i = 0; i < 16; ++i) amax2 = hmax_abs2<false>(amax2, hw[i]);
                }
                amax2 &= 0x7fff7fffu;
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const uint32_t mask = 2 * i + 1 < valid ? 0x7fff7fffu : (2 * i < valid ? 0x00007fffu : 0u);
                  amax2 = __vmaxu2(amax2, hw[i] & mask);
                }
              }
              if constexpr (EPI != kEpiRes16) amax = max(amax, amax16_to_f32bits(amax2, f16));
              if constexpr (KIND == kGemmMXF8)
                nonfinite |= row_ok && max(amax2 & 0xffffu, amax2 >> 16) >= (f16 ? 0x7c00u : 0x7f80u);
            }
            emit16<SB>(o, g, hw, row, row0q, col0, lane, row_ok, valid);
          } else if (EPI == kEpiF32 && o.map != nullptr) {
            // fp32 results through the staging tiles: 16 columns (64 bytes) of
            // the warp's 32 rows per TMA store (the tensor map clips the
            // tile's edges), the same arithmetic as the plain-store path.
#pragma unroll
            for (int hh = 0; hh < kHalves; ++hh) {
              const int c0 = col0 + hh * kSub;
              uint32_t v[kSub];
              tmem_ldn<kSub>(taddr + j * 32 + hh * kSub, v);
              float sw[kSub], bias[kSub];
              if constexpr (KIND == kGemmI8) load_vecn<kSub>(g.col_scale, c0, g.n, sw);
              load_vecn<kSub>(g.bias, c0, g.n, bias);
              tmem_ld_wait();
              uint32_t w[kSub];
#pragma unroll
              for (int i = 0; i < kSub; ++i) {
                float x;
                if (g.bias && KIND == kGemmI8)
                  x = __fmaf_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[i])), sa), sw[i], bias[i]);
                else if (g.bias)
                  x = __fadd_rn(acc_value<KIND>(v[i], sa, 1.0f), bias[i]);
                else
                  x = acc_value<KIND>(v[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f);
                if constexpr (KIND == kGemmMXF8) nonfinite |= row_ok && c0 + i < g.n && !isfinite(x);
                w[i] = __float_as_uint(x);
              }
#pragma unroll
              for (int q = 0; q < kSub / 16; ++q) {
                uint32_t piece[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) piece[i] = w[16 * q + i];
                emit16<SB>(o, g, piece, row, row0q, c0 + 16 * q, lane, row_ok, 0);
              }
            }
          } else {
#pragma unroll
            for (int hh = 0; hh < kHalves; ++hh) {
              const int c0 = col0 + hh * kSub;
              const int vh = valid - hh * kSub;  // valid columns of this piece (may be <= 0)
              uint32_t v[kSub];
              tmem_ldn<kSub>(taddr + j * 32 + hh * kSub, v);
              tmem_ld_wait();
              if (!row_ok || vh <= 0) continue;
              float sw[kSub], bias[kSub];
              if constexpr (KIND == kGemmI8 && EPI != kEpiI32) load_vecn<kSub>(g.col_scale, c0, g.n, sw);
              if constexpr (EPI == kEpiF32) load_vecn<kSub>(g.bias, c0, g.n, bias);
              if constexpr (EPI == kEpiI32) {
                int32_t* dst = static_cast<int32_t*>(g.out) + static_cast<size_t>(row) * g.ldo + c0;
                if (vh >= kSub && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                  int4* q = reinterpret_cast<int4*>(dst);
#pragma unroll
                  for (int i = 0; i < kSub / 4; ++i)
                    q[i] = make_int4(int(v[4 * i]), int(v[4 * i + 1]), int(v[4 * i + 2]), int(v[4 * i + 3]));
                } else {
#pragma unroll
                  for (int i = 0; i < kSub; ++i)
                    if (i < vh) dst[i] = static_cast<int32_t>(v[i]);
                }
              } else if constexpr (EPI == kEpiResF32) {
                float* dst = static_cast<float*>(g.out) + static_cast<size_t>(row) * g.ldo + c0;
#pragma unroll
                for (int i = 0; i < kSub; ++i)
                  if (i < vh) {
                    const float x = __fadd_rn(dst[i], acc_value<KIND>(v[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f));
                    dst[i] = x;
                    if constexpr (KIND == kGemmMXF8) nonfinite |= !isfinite(x);
                  }
              } else if constexpr (EPI == kEpiF32) {
                float* dst = static_cast<float*>(g.out) + static_cast<size_t>(row) * g.ldo + c0;
                const float* res = g.residual ? static_cast<const float*>(g.residual) +
                                                    static_cast<size_t>(row) * g.ldr + c0
                                              : nullptr;
                float x[kSub];
#pragma unroll
                for (int i = 0; i < kSub; ++i) {
                  if (g.bias && KIND == kGemmI8)
                    x[i] = __fmaf_rn(__fmul_rn(static_cast<float>(static_cast<int>(v[i])), sa), sw[i], bias[i]);
                  else if (g.bias)
                    x[i] = __fadd_rn(acc_value<KIND>(v[i], sa, 1.0f), bias[i]);
                  else
                    x[i] = acc_value<KIND>(v[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f);
                }
                // A full, 16-byte-aligned piece leaves by 16-byte stores (the row's
                // kSub * 4 bytes are contiguous); edges element by element.
                const bool vec = vh >= kSub && ((reinterpret_cast<uintptr_t>(dst) |
                                                 reinterpret_cast<uintptr_t>(res)) & 15) == 0;
                if (vec) {
#pragma unroll
                  for (int i = 0; i < kSub / 4; ++i) {
                    float4 y = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
                    if (res) {
                      const float4 r = *reinterpret_cast<const float4*>(res + 4 * i);
                      y = make_float4(__fadd_rn(r.x, y.x), __fadd_rn(r.y, y.y), __fadd_rn(r.z, y.z),
                                      __fadd_rn(r.w, y.w));
                    }
                    *reinterpret_cast<float4*>(dst + 4 * i) = y;
                    if constexpr (KIND == kGemmMXF8)
                      nonfinite |= !isfinite(y.x) || !isfinite(y.y) || !isfinite(y.z) || !isfinite(y.w);
                  }
                } else {
#pragma unroll
                  for (int i = 0; i < kSub; ++i) {
                    if (i < vh) {
                      float y = x[i];
                      if (res) y = __fadd_rn(res[i], y);
                      dst[i] = y;
                      if constexpr (KIND == kGemmMXF8) nonfinite |= !isfinite(y);
                    }
                  }
                }
              }
            }
          }
        }
      }
      // Accumulator fully read: hand it back to the MMA warp before the
      // stores of this tile drain.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (g.row_amax != nullptr && row_ok) atomicMax(g.row_amax + row, amax);
      if constexpr (KIND == kGemmMXF8) {
        if (__any_sync(0xffffffffu, nonfinite) && lane == 0)
          record_status(g.status, KB_STATUS_OUTPUT_NONFINITE, g.layer);
      }
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
    if (lane == 0 && use_tma_out) bulk_wait_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && *abort_flag) record_status(g.status, KB_STATUS_TIMEOUT, g.layer);
  if (warp == 1) tmem_dealloc(tmem_base, Cfg::kTmemCols);
}

// ------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Row-major [rows, k] operand, box {128 bytes of K, box_rows}, 128-byte swizzle.
int make_operand_map(CUtensorMap* map, const void* base, int kind, long rows, long k, int box_rows) {
  const int elem = kind == kGemmBF16 ? 2 : 1;
  const CUtensorMapDataType dt =
      kind == kGemmBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  return encode_2d(map, dt, base, k, rows, k * elem, kBKBytes / elem, box_rows,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

bool epi_16bit(int epi) {
  return epi == kEpiF16 || epi == kEpi16 || epi == kEpiRes16 || epi == kEpiSwiGLU16 || epi == kEpiRope16;
}

// DEEP: short K, where draining the epilogue bounds the tile time: more
// staging tiles per warp (4 with 8 epilogue warps, 2 with 16), fewer otherwise.
template <int KIND, int BN, int EPI, int ACT, int DEEP>
int launch_one(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, int use_tma_out,
               const GemmArgs& g, cudaStream_t stream) {
  constexpr int EW = epi_warps<EPI, DEEP, BN>();
  constexpr int SB = DEEP ? (EW == 16 ? 2 : 4) : (EW == 16 ? 1 : 2);
  using Cfg = GemmCfg<KIND, BN, SB, EW>;
  auto kern = gemm_kernel<KIND, BN, EPI, ACT, SB, EW>;
  int dev = 0;
  cudaGetDevice(&dev);
  // Function attributes live in each device's context: set once per device.
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "gemm smem attribute");
    configured.fetch_or(bit);
  }
  const int tiles = ((g.m + kBM - 1) / kBM) * ((g.n + BN - 1) / BN);
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  kern<<<grid, gemm_threads(EW), Cfg::kSmemBytes, stream>>>(ma, mb, mo, g, use_tma_out);
  return check_cuda(cudaGetLastError(), "gemm launch");
}

template <int KIND, int BN, int DEEP>
int dispatch_epi(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, int tma_out,
                 const GemmArgs& g, cudaStream_t s) {
  switch (epi) {
    case kEpiI32:
      if constexpr (KIND != kGemmMXF8) return launch_one<KIND, BN, kEpiI32, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
      break;
    case kEpiF16: return launch_one<KIND, BN, kEpiF16, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
    case kEpiResF32: return launch_one<KIND, BN, kEpiResF32, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
    case kEpi16:
      if (g.act == kActGelu) return launch_one<KIND, BN, kEpi16, kActGelu, DEEP>(ma, mb, mo, tma_out, g, s);
      if (g.act == kActSilu) return launch_one<KIND, BN, kEpi16, kActSilu, DEEP>(ma, mb, mo, tma_out, g, s);
      return launch_one<KIND, BN, kEpi16, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
    case kEpiRes16: return launch_one<KIND, BN, kEpiRes16, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
    case kEpiRope16: return launch_one<KIND, BN, kEpiRope16, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
    case kEpiSwiGLU16:
      if constexpr (KIND != kGemmMXF8) return launch_one<KIND, BN, kEpiSwiGLU16, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
      break;
    case kEpiF32: return launch_one<KIND, BN, kEpiF32, kActNone, DEEP>(ma, mb, mo, tma_out, g, s);
  }
  set_error("unknown GEMM epilogue");
  return KB_E_INVALID;
}

template <int KIND, int BN>
int dispatch_sb(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, int tma_out,
                const GemmArgs& g, cudaStream_t s) {
  // Deep staging when the epilogue, not the K loop, bounds the tile time.
  const int k_bytes = g.k * (KIND == kGemmBF16 ? 2 : 1);
  if (tma_out && k_bytes <= 1024) return dispatch_epi<KIND, BN, 1>(epi, ma, mb, mo, tma_out, g, s);
  return dispatch_epi<KIND, BN, 0>(epi, ma, mb, mo, tma_out, g, s);
}

}  // namespace

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, long cols, long rows,
              long row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return KB_E_CUDA;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (code " + std::to_string(int(r)) + ")");
    return KB_E_CUDA;
  }
  return KB_OK;
}

int encode_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, long d0, long d1, long d2, long stride1_bytes,
              long stride2_bytes, int box0, int box1, int box2, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return KB_E_CUDA;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride1_bytes), static_cast<cuuint64_t>(stride2_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), static_cast<cuuint32_t>(box2)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string(int(r)) + ")");
    return KB_E_CUDA;
  }
  return KB_OK;
}

int gemm_pick_bn(int kind, int epi, int m, int n) {
  (void)kind;
  if (epi == kEpiSwiGLU16) return 256;
  // Wider tiles once N is past four 256-column tiles, even with a partial
  // last one: the short-K projections are bound by per-tile epilogue work.
  int bn = (n % 256 == 0 || n > 1024) ? 256 : 128;
  // Small M (a few positions): narrower tiles while the grid leaves SMs idle.
  int dev = 0;
  cudaGetDevice(&dev);
  const long mt = (m + kBM - 1) / kBM;
  while (bn > 64 && mt * ((n + bn - 1) / bn) < num_sms(dev)) bn /= 2;
  return bn;
}

int gemm_launch(int kind, int epi, const void* a, const void* b, const GemmArgs& g,
                cudaStream_t stream, int bn_hint) {
  if (g.m <= 0 || g.n <= 0 || g.k <= 0) {
    set_error("GEMM shape must be positive");
    return KB_E_INVALID;
  }
  const int elem = kind == kGemmBF16 ? 2 : 1;
  if ((static_cast<long>(g.k) * elem) % 16 != 0) {
    set_error("GEMM K row stride must be a multiple of 16 bytes");
    return KB_E_INVALID;
  }
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15)) {
    set_error("GEMM operands must be 16-byte aligned");
    return KB_E_INVALID;
  }
  if (kind == kGemmMXF8) {
    if (epi == kEpiI32 || epi == kEpiSwiGLU16) {
      set_error("MXFP8 GEMM supports the f16 / 16-bit / residual / f32 epilogues");
      return KB_E_INVALID;
    }
    if (g.sfa == nullptr || g.sfb == nullptr || (reinterpret_cast<uintptr_t>(g.sfa) & 15) ||
        (reinterpret_cast<uintptr_t>(g.sfb) & 15)) {
      set_error("MXFP8 GEMM needs 16-byte aligned scale-factor tiles for A and B");
      return KB_E_INVALID;
    }
    if (g.k % 32 != 0) {
      set_error("MXFP8 GEMM K must be padded to a multiple of 32");
      return KB_E_INVALID;
    }
  }
  if (kind == kGemmI8 && epi != kEpiI32 && (g.row_scale == nullptr || g.col_scale == nullptr)) {
    set_error("INT8 dequant epilogue needs row and column scales");
    return KB_E_INVALID;
  }
  if (epi == kEpiRope16 &&
      (g.rope_cos == nullptr || g.rope_sin == nullptr || g.rope_seq <= 0 || g.rope_heads <= 0 ||
       (g.rope_hd != 32 && g.rope_hd != 64) || g.rope_cols != 2 * g.rope_heads * g.rope_hd || g.rope_cols > g.n ||
       (reinterpret_cast<uintptr_t>(g.rope_cos) & 3) || (reinterpret_cast<uintptr_t>(g.rope_sin) & 3))) {
    set_error("rotary epilogue: needs fp32 tables, head_dim 32 or 64, rope_cols = 2 * heads * head_dim <= N");
    return KB_E_INVALID;
  }
  if (epi == kEpiSwiGLU16 && !g.out_f16) {
    set_error("SwiGLU epilogue: the output is binary16 (out_f16 = 1)");
    return KB_E_INVALID;
  }
  if (epi == kEpiRope16 && g.bias != nullptr) {
    set_error("rotary epilogue: the QKV projection takes no bias");
    return KB_E_INVALID;
  }
  if (g.act < kActNone || g.act > kActSilu) {
    set_error("unknown activation");
    return KB_E_INVALID;
  }
  // MXFP8 keeps BN = 128: two 128-column accumulators plus the per-stage
  // scale-factor columns fill the 512 TMEM columns.
  // The SwiGLU tile is 128 gate + 128 up columns: BN = 256 always.
  const int bn = kind == kGemmMXF8 ? 128 : epi == kEpiSwiGLU16 ? 256 : bn_hint ? bn_hint : gemm_pick_bn(kind, epi, g.m, g.n);
  CUtensorMap ma, mb, mo;
  memset(&mo, 0, sizeof(mo));
  int rc = make_operand_map(&ma, a, kind, g.m, g.k, kBM);
  if (rc) return rc;
  rc = make_operand_map(&mb, b, kind, g.n, g.k, bn);
  if (rc) return rc;
  // 16-bit outputs leave through TMA stores when the row stride allows it.
  int tma_out = 0;
  // Tactic switch (like the reference's KATAGO_CUDA_* keys): KB_GEMM_DIRECT_STORE=1
  // writes 16-bit outputs with plain vector stores instead of TMA stores.
  static const bool direct_store = [] {
    const char* v = getenv("KB_GEMM_DIRECT_STORE");
    return v != nullptr && v[0] == '1';
  }();
  if (!direct_store && epi_16bit(epi) && (g.ldo * 2) % 16 == 0 &&
      (reinterpret_cast<uintptr_t>(g.out) & 15) == 0) {
    const long cols = epi == kEpiSwiGLU16 ? g.n_out : g.n;
    rc = encode_2d(&mo, CU_TENSOR_MAP_DATA_TYPE_UINT16, g.out, cols, g.m, g.ldo * 2, 32, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    tma_out = 1;
  }
  // fp32 outputs leave through the staging tiles too (16 fp32 columns are 64
  // bytes, the same box as 32 16-bit columns), and an fp32 residual that is
  // the output itself (kEpiResF32 always; kEpiF32 when residual == out) comes
  // in through them.
  const bool f32_in_place = epi == kEpiResF32 ||
                            (epi == kEpiF32 && (g.residual == nullptr || (g.residual == g.out && g.ldr == g.ldo)));
  if (!direct_store && f32_in_place && (g.ldo * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(g.out) & 15) == 0) {
    rc = encode_2d(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, g.out, g.n, g.m, g.ldo * 4, 16, 32,
                   CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    tma_out = 1;
  }
  GemmArgs ga = g;
  ga.cols_vec = g.n % 32 == 0 && (reinterpret_cast<uintptr_t>(g.col_scale) & 31) == 0 &&
                (reinterpret_cast<uintptr_t>(g.bias) & 31) == 0;
  if (kind == kGemmI8) {
    return bn == 256   ? dispatch_sb<kGemmI8, 256>(epi, ma, mb, mo, tma_out, ga, stream)
           : bn == 128 ? dispatch_sb<kGemmI8, 128>(epi, ma, mb, mo, tma_out, ga, stream)
                       : dispatch_sb<kGemmI8, 64>(epi, ma, mb, mo, tma_out, ga, stream);
  }
  if (kind == kGemmBF16) {
    return bn == 256   ? dispatch_sb<kGemmBF16, 256>(epi, ma, mb, mo, tma_out, ga, stream)
           : bn == 128 ? dispatch_sb<kGemmBF16, 128>(epi, ma, mb, mo, tma_out, ga, stream)
                       : dispatch_sb<kGemmBF16, 64>(epi, ma, mb, mo, tma_out, ga, stream);
  }
  if (kind == kGemmMXF8) return dispatch_sb<kGemmMXF8, 128>(epi, ma, mb, mo, tma_out, ga, stream);
  set_error("GEMM kind not supported");
  return KB_E_UNSUPPORTED;
}

}  // namespace kb
