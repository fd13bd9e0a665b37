// Self-attention over the 361 board tokens on the tcgen05 tensor cores, fused
// with RoPE (head_dim 64 or 32).
//
// Replaces the reference's q64 flash attention (crates/kata_nn/cuda-kernels/
// attention_fa2_q64.cu:82-390; launcher src/backends/cuda_exec.rs:3442) with the
// same semantics as attention.cu: packed [tokens, 3C] = [Q | K | V], Q and K
// rotated by interleaved pairs with per-(token, head, pair) tables and rounded
// to the 16-bit type, softmax of (q.k) * scale over all keys in fp32, P rounded
// to the 16-bit type for the P.V product, output [tokens, C] heads merged.
//
// Persistent: one CTA per SM walks jobs, each a (position, head) pair with all
// its query tiles, or, at small batch (SPLIT), one query tile of a pair, so the
// grid fills more SMs.  All 361 keys fit on chip, so nothing streams inside a
// job:
//   shared memory  K and V of two pairs (double buffer, 368 keys x 2D bytes
//                  each, keys padded to a multiple of 16) and one 128-query Q
//                  tile, all in the UMMA swizzled layout (rows of 128 bytes
//                  with the 128-byte swizzle for D = 64, rows of 64 bytes with
//                  the 64-byte swizzle for D = 32), loaded by TMA (or by three
//                  staging warps that rotate on the way in);
//   TMEM (512 col) S_A = Q K[0:192]^T (192 columns), S_B = Q K[192:368]^T (176),
//                  O_A = P_A V[0:192] and O_B = P_B V[192:368] (D each), and
//                  the row sums: for D = 64 the softmax's slice sums of two
//                  tiles (16 columns); for D = 32 l_A = P_A . 1 and
//                  l_B = P_B . 1 on the tensor cores (a 16-column MMA each
//                  against a tile of ones: no per-score add in the softmax).
// The two key halves keep their own maxima (no rescaling: the epilogue
// combines them), so they form a two-stage pipeline.  All 16 softmax warps
// (four per TMEM lane quarter, one query row per thread, 48 keys of each half
// per warp) take half A of a tile, then half B; meanwhile warp 16 runs the
// tensor cores on the other half: PV_A of this tile and S_A of the next while
// the softmax works on half B, PV_B and S_B of the next while it works on the
// next half A.  Within a half the four warps of a lane quarter exchange their
// slice maxima through shared memory, then write P = exp2((S - m) c) as packed
// 16-bit pairs over their own, already read S columns (the A operand of the
// P.V MMA, read from TMEM).  Between the halves the softmax warps finish the
// previous tile: O = (O_A 2^((m_A-m)c) + O_B 2^((m_B-m)c)) /
// (l_A 2^((m_A-m)c) + l_B 2^((m_B-m)c)), each warp writing D/4 of the D dims
// by TMA, plus the row |max| for the next quantiser.  Every exponential is the
// same FMA-pipe polynomial (exp2_poly2), so the softmax is a fixed sequence of
// IEEE operations that the CPU oracle restates exactly.  Every wait is bounded.
#include <stdint.h>
#include <string.h>

#include <atomic>

#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

constexpr int kKeysPad = 368;             // >= 361, multiple of 16
constexpr int kHalfA = 192, kHalfB = kKeysPad - kHalfA;  // 176
constexpr int kTileQ = 128;
constexpr int kSoftWarps = 16;
constexpr int kMmaWarp = kSoftWarps;
// Loader warps: two issuing TMA copies (K/V and Q; Q and K arrive rotated),
// or three staging and rotating with the CTA's threads (the table-driven RoPE
// path).
template <bool ROPE>
constexpr int load_warps() { return ROPE ? 3 : 2; }
template <bool ROPE>
constexpr int fa_threads() { return 32 * (kSoftWarps + 1 + load_warps<ROPE>()); }  // 640 / 608
constexpr int kKvBox = 184;               // rows per K/V TMA box (2 boxes = 368 rows)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSB = kHalfA, kOA = kHalfA + kHalfB;  // TMEM columns
constexpr int kBarBytes = 256;
// Slice maxima exchanged between the 4 warps of a TMEM lane quarter:
// [tile parity][half][slice][row] floats.
constexpr int kMlBytes = 2 * 2 * 4 * kTileQ * 4;

// Geometry for head_dim D (64 or 32).
template <int D>
struct Geo {
  static_assert(D == 64 || D == 32, "head_dim 64 or 32");
  static constexpr int kRowBytes = D * 2;  // one Q/K/V row: 128 B (D 64) or 64 B (D 32)
  static constexpr int kChunks = D / 8;    // 16-byte chunks per row
  static constexpr int kKBytes = kKeysPad * kRowBytes;
  static constexpr int kKVBytes = 2 * kKBytes;  // K then V of one pair
  static constexpr int kQBytes = kTileQ * kRowBytes;
  static constexpr int kDimsW = D / 4;          // output dims per softmax warp (4 warps per lane quarter)
  static constexpr int kPieceBytes = 32 * kDimsW * 2;  // one warp's output piece: 32 rows x kDimsW dims
  static constexpr uint32_t kOB = kOA + D;
  // Row sums l of the 8 key slices of a tile (4 per half), double-buffered by
  // tile parity, in 16 TMEM columns after O_B.
  static constexpr uint32_t kLCol = kOB + D;
  static_assert(kLCol + 16 <= kTmemCols, "TMEM budget");
  // D = 32: each half's row sum comes from the tensor cores instead, P times a
  // tile of ones (N = 16, all 16 columns equal) into LA / LB after O_B, so the
  // softmax adds nothing per score; D = 64 has no TMEM room for the 32 columns.
  static constexpr bool kMmaSums = D == 32;
  static constexpr uint32_t kLA = kOB + D, kLB = kLA + 16;
  static_assert(!kMmaSums || kLB + 16 <= kTmemCols, "TMEM budget");
  // The ones tile: K-major without swizzle, two 8-row core matrices along N
  // (256 bytes apart) by two along K (128 bytes apart), 512 bytes read.
  static constexpr int kOnesBytes = kMmaSums ? 512 : 0;
  // K/V double buffer, one Q tile (loaded as soon as the previous tile's S MMAs
  // are done, several microseconds before it is needed), the output pieces.
  static constexpr int kSmemBytes =
      2 * kKVBytes + kQBytes + kSoftWarps * kPieceBytes + kBarBytes + kMlBytes + kOnesBytes + 1024 /*alignment*/;
};

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool f16) {
  if (f16) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// 2^x for a pair of x <= 0 on the FMA pipe, the kernel's one definition of
// the exponential (a fixed sequence of IEEE operations, so the CPU oracle
// reproduces every P bit for bit; the special-function unit's approximation
// would not be reproducible): x clamped to -126,
// n = rint(x) by the 1.5 * 2^23 magic add, f = x - n in [-0.5, 0.5], 2^f by a
// degree-3 polynomial (least-squares Chebyshev fit of 2^f on [-0.5, 0.5],
// relative error 1.4e-4: below the 16-bit rounding of P), and 2^n added to
// the exponent field (the magic sum's low bits are n, shifted by 23).
__device__ __forceinline__ float2 exp2_poly2(float x0, float x1) {
  constexpr float kMagic = 12582912.0f;
  const float2 x = make_float2(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const float2 j = add2(x, make_float2(kMagic, kMagic));
  const float2 n = add2(j, make_float2(-kMagic, -kMagic));
  const float2 f = fma2(n, make_float2(-1.0f, -1.0f), x);
  float2 p = fma2(make_float2(0x1.c2ccd4p-5f, 0x1.c2ccd4p-5f), f, make_float2(0x1.f02456p-3f, 0x1.f02456p-3f));
  p = fma2(p, f, make_float2(0x1.62f21p-1f, 0x1.62f21p-1f));
  p = fma2(p, f, make_float2(0x1.fff9ap-1f, 0x1.fff9ap-1f));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(j.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(j.y) << 23)));
}

// Three-input maximum (fmaxf semantics: NaN operands are ignored).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Rotate one interleaved pair (x, y) by (c, s), rounded to the 16-bit type.
__device__ __forceinline__ uint32_t rope2(uint32_t w, float c, float s, bool f16) {
  const float x = from16(static_cast<uint16_t>(w & 0xffffu), f16);
  const float y = from16(static_cast<uint16_t>(w >> 16), f16);
  return pack2(__fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s)), __fadd_rn(__fmul_rn(x, s), __fmul_rn(y, c)), f16);
}

// Byte offset of 16-byte chunk `c` of row `r` in a swizzled tile: 128-byte
// rows with the 128-byte swizzle (chunk ^ row % 8) for D = 64, 64-byte rows
// with the 64-byte swizzle (chunk ^ (row / 2) % 4) for D = 32.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  if constexpr (D == 64) return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
  else return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// UMMA shared-memory descriptor of a Q, K or V tile in that layout.
template <int D>
__device__ __forceinline__ uint64_t tile_desc(uint32_t saddr) {
  if constexpr (D == 64) return sw128_desc(saddr);
  else return sw64_desc(saddr);
}

// Rows [r0, r0 + nrows) of Q, K or V (part = 0, 1, 2) of head h of one position
// into a swizzled tile, rotated when `rotate`; rows at or past `seq` are zero.  Each
// thread handles kBatch 16-byte chunks per step with all their global loads
// issued before any is used, so the copy is not bound by one load's latency.
constexpr int kBatch = 3;

template <int D, bool F16>
__device__ __forceinline__ void stage_rows(uint8_t* dst, const uint16_t* base, size_t row_stride, int part, int h,
                                           int heads, const float* cos_t, const float* sin_t, int r0, int nrows,
                                           int seq, int tid, int nthreads, bool rotate) {
  constexpr int kCh = Geo<D>::kChunks;
  const int c = heads * D;
  const int total = nrows * kCh;
  for (int t0 = tid; t0 < total; t0 += kBatch * nthreads) {
    uint4 raw[kBatch];
    float4 co[kBatch], si[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = t0 + u * nthreads;
      const int r = t / kCh, ch = t % kCh;
      const int tok = r0 + r;
      raw[u] = make_uint4(0, 0, 0, 0);
      if (t < total && tok < seq) {
        raw[u] = __ldg(reinterpret_cast<const uint4*>(base + tok * row_stride + part * c + h * D + ch * 8));
        if (rotate) {
          const size_t ro = (static_cast<size_t>(tok) * heads + h) * (D / 2) + ch * 4;
          co[u] = __ldg(reinterpret_cast<const float4*>(cos_t + ro));
          si[u] = __ldg(reinterpret_cast<const float4*>(sin_t + ro));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int t = t0 + u * nthreads;
      if (t >= total) break;
      const int r = t / kCh, ch = t % kCh;
      uint4 v = raw[u];
      if (rotate && r0 + r < seq)
        v = make_uint4(rope2(raw[u].x, co[u].x, si[u].x, F16), rope2(raw[u].y, co[u].y, si[u].y, F16),
                       rope2(raw[u].z, co[u].z, si[u].z, F16), rope2(raw[u].w, co[u].w, si[u].w, F16));
      *reinterpret_cast<uint4*>(dst + swz<D>(r, ch)) = v;
    }
  }
}

// Softmax of one key slice for this thread's query row: NK keys (48, or 32
// for the last slice of half B) at S columns [col, col + NK), `valid` of them
// below seq.  The slice maxima of the half's four warps are exchanged through
// shared memory (mx: [slice][row] of this parity and half, barrier `mx_bar`
// with 128 arrivals), then P = 2^((S - m) c) is written as packed 16-bit
// pairs over columns [col, col + NK/2) (keys 2j, 2j+1 at column col + j:
// columns this thread has already read), and (SUMS) the slice's row sum l to
// TMEM column `lcol`.  Returns false if a wait gave up.
template <int NK, bool F16, bool SUMS>
__device__ __forceinline__ bool softmax_slice(uint32_t lane_base, uint32_t col, int valid, float scale_log2, float* mx,
                                              int sub, int row, uint64_t* mx_bar, uint32_t parity,
                                              volatile int* abort_flag, uint32_t lcol, float& m_out) {
  uint32_t v[NK];
  {
    uint32_t (&v0)[32] = *reinterpret_cast<uint32_t(*)[32]>(v);
    tmem_ld32(lane_base + col, v0);
    if constexpr (NK == 48) {
      uint32_t (&v1)[16] = *reinterpret_cast<uint32_t(*)[16]>(v + 32);
      tmem_ld16(lane_base + col + 32, v1);
    }
    tmem_ld_wait();
  }
  // Row maximum over the slice: 8 independent partial maxima (short chains).
  float mp[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) mp[j] = __int_as_float(0xff800000);
  if (valid >= NK) {
#pragma unroll
    for (int i = 0; i < NK / 2; ++i)
      mp[i & 7] = max3(mp[i & 7], __uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
  } else {
#pragma unroll
    for (int i = 0; i < NK; ++i)
      if (i < valid) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(v[i]));
  }
  float m = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
  mx[sub * kTileQ + row] = m;
  mbar_arrive(mx_bar);
  if (!__all_sync(0xffffffffu, mbar_wait(mx_bar, parity, abort_flag))) return false;
  m = fmaxf(fmaxf(mx[row], mx[kTileQ + row]), fmaxf(mx[2 * kTileQ + row], mx[3 * kTileQ + row]));
  m_out = m;
  const float mc = __fmul_rn(m, scale_log2);
  float lp[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // partial sums (short chains)
  uint32_t pk[NK / 2];
  if (valid >= NK) {
#pragma unroll
    for (int i = 0; i < NK / 2; ++i) {
      const float2 x = fma2(make_float2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])),
                            make_float2(scale_log2, scale_log2), make_float2(-mc, -mc));
      const float2 p = exp2_poly2(x.x, x.y);
      if constexpr (SUMS) lp[i & 3] = __fadd_rn(lp[i & 3], __fadd_rn(p.x, p.y));
      pk[i] = pack2(p.x, p.y, F16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < NK / 2; ++i) {
      const float2 e = exp2_poly2(__fmaf_rn(__uint_as_float(v[2 * i]), scale_log2, -mc),
                                  __fmaf_rn(__uint_as_float(v[2 * i + 1]), scale_log2, -mc));
      const float p0 = 2 * i < valid ? e.x : 0.0f;
      const float p1 = 2 * i + 1 < valid ? e.y : 0.0f;
      if constexpr (SUMS) lp[i & 3] = __fadd_rn(lp[i & 3], __fadd_rn(p0, p1));
      pk[i] = pack2(p0, p1, F16);
    }
  }
  tmem_st16(lane_base + col, *reinterpret_cast<const uint32_t(*)[16]>(pk));
  if constexpr (NK == 48) tmem_st8(lane_base + col + 16, *reinterpret_cast<const uint32_t(*)[8]>(pk + 16));
  if constexpr (SUMS)
    tmem_st1(lane_base + lcol, __float_as_uint(__fadd_rn(__fadd_rn(lp[0], lp[1]), __fadd_rn(lp[2], lp[3]))));
  tmem_st_wait();
  tc_fence_before();
  return true;
}

template <int D, bool F16, bool ROPE, bool SPLIT>
__global__ void __launch_bounds__(fa_threads<ROPE>(), 1) attention_fa_kernel(
    const __grid_constant__ CUtensorMap map_kv, const __grid_constant__ CUtensorMap map_q,
    const __grid_constant__ CUtensorMap map_out,
    const uint16_t* __restrict__ qkv, const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
    uint16_t* __restrict__ out, int pairs, int seq, int heads, float scale_log2, uint32_t* __restrict__ row_amax,
    unsigned* status) {
  constexpr int kLoadThreads = 32 * load_warps<ROPE>();
  using G = Geo<D>;
  constexpr int kRowBytes = G::kRowBytes, kKBytes = G::kKBytes, kKVBytes = G::kKVBytes, kQBytes = G::kQBytes;
  constexpr uint32_t kOB = G::kOB, kLCol = G::kLCol;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kv_buf = smem;                    // [2][K | V]
  uint8_t* q_buf = smem + 2 * kKVBytes;      // Q tile
  uint8_t* o_buf = q_buf + kQBytes;          // output pieces: one per softmax warp (32 rows x D/4 dims)
  uint64_t* bars = reinterpret_cast<uint64_t*>(o_buf + kSoftWarps * G::kPieceBytes);
  uint64_t* kv_full = bars + 0;   // [2] loaders staged K/V           (128 arrivals)
  uint64_t* kv_empty = bars + 2;  // [2] MMAs done with K/V            (commit)
  uint64_t* q_full = bars + 4;    // loaders staged the Q tile          (tx bytes, or 96 arrivals)
  uint64_t* q_empty = bars + 5;   // S MMAs done with the Q tile        (commit)
  uint64_t* pva_done = bars + 6;  // PV_A done: P_A consumed           (commit)
  uint64_t* o_free = bars + 7;    // O of the previous tile read back  (512 arrivals)
  uint64_t* sa_full = bars + 8;   // S_A ready                         (commit)
  uint64_t* sb_full = bars + 9;   // S_B ready                         (commit)
  uint64_t* pa_full = bars + 10;  // P_A and its row sums written      (512 arrivals)
  uint64_t* pb_full = bars + 11;  // P_B and its row sums written      (512 arrivals)
  uint64_t* o_full = bars + 12;   // O_A and O_B ready                 (commit)
  uint64_t* kv_tma = bars + 13;   // [2] K/V TMA copies landed         (tx bytes)
  // [half][quarter]: slice maxima of the 4 warps holding the same query rows
  uint64_t* mx_full = bars + 16;  // (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 28);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* mx_ex = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + kBarBytes);  // [2][2][4][128]
  uint8_t* ones_buf = reinterpret_cast<uint8_t*>(bars) + kBarBytes + kMlBytes;  // D = 32: B of P . 1

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = heads * D;
  const size_t row_stride = 3 * static_cast<size_t>(c);
  const int tiles = (seq + kTileQ - 1) / kTileQ;
  // Jobs: a (position, head) pair with tpj of its query tiles, K and V loaded
  // once per job: all tiles, or (SPLIT, when the pairs alone would leave SMs
  // idle) one tile per job.
  const int tpj = SPLIT ? 1 : tiles;
  const int jpp = SPLIT ? tiles : 1;  // jobs per pair
  const int jobs = pairs * jpp;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], ROPE ? kLoadThreads : 32);  // the K/V loader warp (or every staging thread)
      mbar_init(&kv_empty[i], 1);
      mbar_init(&kv_tma[i], 1);
    }
    mbar_init(q_full, ROPE ? kLoadThreads : 1);
    mbar_init(q_empty, 1);

    mbar_init(pva_done, 1);
    mbar_init(o_free, 32 * kSoftWarps);
    mbar_init(sa_full, 1);
    mbar_init(sb_full, 1);
    mbar_init(pa_full, 32 * kSoftWarps);
    mbar_init(pb_full, 32 * kSoftWarps);
    mbar_init(o_full, 1);
    for (int i = 0; i < 8; ++i) mbar_init(&mx_full[i], 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if constexpr (G::kMmaSums) {
    const uint32_t one2 = F16 ? 0x3c003c00u : 0x3f803f80u;  // 1.0 in both 16-bit halves
    for (int i = threadIdx.x; i < G::kOnesBytes / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(ones_buf)[i] = make_uint4(one2, one2, one2, one2);
    fence_proxy_async_smem();  // visible to the tensor cores after the barrier
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp > kMmaWarp && !ROPE) {
    // ------------------------------------------------------------ TMA loaders
    // Q and K arrive rotated.  Warp kMmaWarp + 1 loads K and V of each pair
    // (two 184-row boxes each) into the free half of the double buffer as soon
    // as it is released; warp kMmaWarp + 2 loads the 128-row Q tiles, each as
    // soon as the S MMAs of the previous tile have read the Q buffer.  Both
    // land in the UMMA 128-byte-swizzled layout.
    const bool kv_loader = warp == kMmaWarp + 1;
    if (lane == 0) tma_prefetch_desc(kv_loader ? &map_kv : &map_q);
    int g = 0;  // global Q tile counter
    for (int it = 0, j = blockIdx.x; j < jobs; ++it, j += gridDim.x) {
      const int kb = it & 1;
      const int p = j / jpp, t0 = (j % jpp) * tpj;
      const int b = p / heads, h = p % heads;
      if (kv_loader) {
        if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[kb], ((it >> 1) & 1) ^ 1, abort_flag))) break;
        uint8_t* ks = kv_buf + kb * kKVBytes;
        if (lane == 0) {
          mbar_arrive_expect_tx(&kv_tma[kb], 2 * kKBytes);
          tma_load_2d(ks, &map_kv, &kv_tma[kb], c + h * D, b * seq);
          tma_load_2d(ks + kKvBox * kRowBytes, &map_kv, &kv_tma[kb], c + h * D, b * seq + kKvBox);
          tma_load_2d(ks + kKBytes, &map_kv, &kv_tma[kb], 2 * c + h * D, b * seq);
          tma_load_2d(ks + kKBytes + kKvBox * kRowBytes, &map_kv, &kv_tma[kb], 2 * c + h * D,
                      b * seq + kKvBox);
          // the job's Q tiles into L2, so each later Q load is an L2 hit
          for (int t = t0; t < t0 + tpj; ++t) tma_prefetch_2d(&map_q, h * D, b * seq + t * kTileQ);
        }
        // V rows [seq, 368) hold the next position's values (or TMA zeros):
        // clear them, their P is zero but 0 * Inf would not be.
        if (!__all_sync(0xffffffffu, mbar_wait(&kv_tma[kb], (it >> 1) & 1, abort_flag))) break;
        for (int i = lane; i < (kKeysPad - seq) * G::kChunks; i += 32)
          *reinterpret_cast<uint4*>(ks + kKBytes + swz<D>(seq + i / G::kChunks, i % G::kChunks)) =
              make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();
        mbar_arrive(&kv_full[kb]);
      } else {
        bool ok = true;
        for (int t = t0; t < t0 + tpj; ++t, ++g) {
          if (!__all_sync(0xffffffffu, mbar_wait(q_empty, (g & 1) ^ 1, abort_flag))) {
            ok = false;
            break;
          }
          if (lane == 0) {
            mbar_arrive_expect_tx(q_full, kQBytes);
            tma_load_2d(q_buf, &map_q, q_full, h * D, b * seq + t * kTileQ);
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp > kMmaWarp) {
    // ------------------------------------------------------------ staging loaders (RoPE here)
    const int tid = threadIdx.x - 32 * (kMmaWarp + 1);
    int g = 0;  // global Q tile counter
    for (int it = 0, j = blockIdx.x; j < jobs; ++it, j += gridDim.x) {
      const int kb = it & 1;
      const int p = j / jpp, t0 = (j % jpp) * tpj;
      const int b = p / heads, h = p % heads;
      const uint16_t* base = qkv + static_cast<size_t>(b) * seq * row_stride;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[kb], ((it >> 1) & 1) ^ 1, abort_flag))) break;
      uint8_t* ks = kv_buf + kb * kKVBytes;
      stage_rows<D, F16>(ks, base, row_stride, 1, h, heads, rope_cos, rope_sin, 0, kKeysPad, seq, tid,
                         kLoadThreads, true);
      stage_rows<D, F16>(ks + kKBytes, base, row_stride, 2, h, heads, rope_cos, rope_sin, 0, kKeysPad, seq, tid,
                         kLoadThreads, false);
      fence_proxy_async_smem();
      mbar_arrive(&kv_full[kb]);
      bool ok = true;
      for (int t = t0; t < t0 + tpj; ++t, ++g) {
        if (!__all_sync(0xffffffffu, mbar_wait(q_empty, (g & 1) ^ 1, abort_flag))) {
          ok = false;
          break;
        }
        stage_rows<D, F16>(q_buf, base, row_stride, 0, h, heads, rope_cos, rope_sin, t * kTileQ, kTileQ, seq, tid,
                           kLoadThreads, true);
        fence_proxy_async_smem();
        mbar_arrive(q_full);
      }
      if (!ok) break;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // Per tile g: S_A(g), S_B(g), then PV_A(g) once P_A(g) is written and the
    // previous tile's O has been read, then PV_B(g).  The next tile's S_A is
    // issued as soon as PV_A(g) has consumed P_A(g) (it overwrites those
    // columns), and its S_B once PV_B(g) has consumed P_B(g); so the softmax
    // of one half always overlaps the tensor-core work of the other.
    if (lane == 0) {
      constexpr uint32_t kFmt = F16 ? 0u : 1u;
      const uint32_t id_common = (1u << 4) | (kFmt << 7) | (kFmt << 10) | (static_cast<uint32_t>(128 >> 4) << 24);
      const uint32_t id_sa = id_common | (static_cast<uint32_t>(kHalfA >> 3) << 17);
      const uint32_t id_sb = id_common | (static_cast<uint32_t>(kHalfB >> 3) << 17);
      const uint32_t id_pv = id_common | (1u << 16) /* B MN-major */ | (static_cast<uint32_t>(D >> 3) << 17);
      // P . 1 (D = 32): B K-major, N = 16, the ones tile (built where used)
      constexpr uint32_t kIdOnesN = static_cast<uint32_t>(16 >> 3) << 17;
      constexpr uint64_t kHalfOff = (kHalfA * kRowBytes) >> 4;  // 192 rows, descriptor units
      constexpr uint64_t kStep16 = (16 * kRowBytes) >> 4;       // 16 keys of V along K
      const int my_jobs = blockIdx.x < jobs ? (jobs - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1 : 0;
      const int n = my_jobs * tpj;
      auto issue_sa = [&](int g) -> bool {
        const int it = g / tpj, t = g % tpj, kb = it & 1;
        if (t == 0 && !mbar_wait(&kv_full[kb], (it >> 1) & 1, abort_flag)) return false;
        if (!mbar_wait(q_full, g & 1, abort_flag)) return false;
        tc_fence_after();
        const uint64_t kdesc = tile_desc<D>(smem_u32(kv_buf + kb * kKVBytes));
        const uint64_t qdesc = tile_desc<D>(smem_u32(q_buf));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_issue<kKindBF16>(tmem, qdesc + 2 * kk, kdesc + 2 * kk, id_sa, kk != 0, 0, 0);
        tc_commit(sa_full);
        return true;
      };
      auto issue_sb = [&](int g) {
        const int kb = (g / tpj) & 1;
        const uint64_t kdesc = tile_desc<D>(smem_u32(kv_buf + kb * kKVBytes));
        const uint64_t qdesc = tile_desc<D>(smem_u32(q_buf));
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_issue<kKindBF16>(tmem + kSB, qdesc + 2 * kk, kdesc + kHalfOff + 2 * kk, id_sb, kk != 0, 0, 0);
        tc_commit(sb_full);
        tc_commit(q_empty);
      };
      bool ok = n == 0 || issue_sa(0);
      if (ok && n > 0) issue_sb(0);
      for (int g = 0; g < n && ok; ++g) {
        const int kb = (g / tpj) & 1;
        const uint64_t vdesc = tile_desc<D>(smem_u32(kv_buf + kb * kKVBytes + kKBytes));
        if (!mbar_wait(pa_full, g & 1, abort_flag) || (g > 0 && !mbar_wait(o_free, (g - 1) & 1, abort_flag))) break;
        tc_fence_after();
        // P of keys 16i..16i+15 of a half: softmax warp i/3 holds 48 keys at
        // its own S columns 48(i/3).., two keys per column.
        for (int i = 0; i < kHalfA / 16; ++i)
          mma_f16_ts(tmem + kOA, tmem + 48 * (i / 3) + 8 * (i % 3), vdesc + kStep16 * i, id_pv, i != 0);
        if constexpr (G::kMmaSums)  // l_A = P_A . 1, the same 16-key accumulation steps as O_A
          for (int i = 0; i < kHalfA / 16; ++i)
            mma_f16_ts(tmem + G::kLA, tmem + 48 * (i / 3) + 8 * (i % 3),
                       noswizzle_desc(smem_u32(ones_buf), 128, 256), id_common | kIdOnesN, i != 0);
        tc_commit(pva_done);
        if (g + 1 < n && (!mbar_wait(pva_done, g & 1, abort_flag) || !issue_sa(g + 1))) break;
        if (!mbar_wait(pb_full, g & 1, abort_flag)) break;
        tc_fence_after();
        for (int i = 0; i < kHalfB / 16; ++i)
          mma_f16_ts(tmem + kOB, tmem + kSB + 48 * (i / 3) + 8 * (i % 3), vdesc + kHalfOff + kStep16 * i, id_pv,
                     i != 0);
        if constexpr (G::kMmaSums)
          for (int i = 0; i < kHalfB / 16; ++i)
            mma_f16_ts(tmem + G::kLB, tmem + kSB + 48 * (i / 3) + 8 * (i % 3),
                       noswizzle_desc(smem_u32(ones_buf), 128, 256), id_common | kIdOnesN, i != 0);
        tc_commit(o_full);
        if (g % tpj == tpj - 1) tc_commit(&kv_empty[kb]);
        if (g + 1 < n) {
          if (!mbar_wait(o_full, g & 1, abort_flag)) break;
          issue_sb(g + 1);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    // Warp (sub, quarter): TMEM lanes 32*quarter.. (one query row per thread),
    // keys 48*sub.. of half A and 192 + 48*sub.. of half B (32 keys for sub 3).
    const int sub = warp >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t col_a = 48 * sub, col_b = kSB + 48 * sub;
    const int valid_a = min(48, seq - 48 * sub);
    const int valid_b = min(sub == 3 ? 32 : 48, seq - kHalfA - 48 * sub);
    // previous tile, whose epilogue runs between this tile's two halves
    int pb = 0, ph = 0, pt = 0, pg = -1;
    float pma = 0.0f, pmb = 0.0f;
    // The epilogue of tile pg: O = (O_A 2^((m_A-m)c) + O_B 2^((m_B-m)c)) /
    // (l_A 2^((m_A-m)c) + l_B 2^((m_B-m)c)), D/4 of the D dims per warp.
    auto epilogue = [&]() -> bool {
      constexpr int kDW = G::kDimsW;
      if (!__all_sync(0xffffffffu, mbar_wait(o_full, pg & 1, abort_flag))) return false;
      tc_fence_after();
      uint32_t lv[8], oa[kDW], ob[kDW], w[kDW / 2];
      const int dim0 = sub * kDW;
      if constexpr (G::kMmaSums) {
        tmem_ld1(lane_base + G::kLA, lv[0]);
        tmem_ld1(lane_base + G::kLB, lv[1]);
      } else {
        tmem_ld8(lane_base + kLCol + (pg & 1) * 8, lv);
      }
      if constexpr (kDW == 16) {
        tmem_ld16(lane_base + kOA + dim0, oa);
        tmem_ld16(lane_base + kOB + dim0, ob);
      } else {
        tmem_ld8(lane_base + kOA + dim0, oa);
        tmem_ld8(lane_base + kOB + dim0, ob);
      }
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(o_free);
      float la, lb;
      if constexpr (G::kMmaSums) {
        la = __uint_as_float(lv[0]);
        lb = __uint_as_float(lv[1]);
      } else {
        la = __fadd_rn(__fadd_rn(__uint_as_float(lv[0]), __uint_as_float(lv[1])),
                       __fadd_rn(__uint_as_float(lv[2]), __uint_as_float(lv[3])));
        lb = __fadd_rn(__fadd_rn(__uint_as_float(lv[4]), __uint_as_float(lv[5])),
                       __fadd_rn(__uint_as_float(lv[6]), __uint_as_float(lv[7])));
      }
      const float mx = fmaxf(pma, pmb);
      const float2 fab = exp2_poly2(__fmul_rn(__fsub_rn(pma, mx), scale_log2), __fmul_rn(__fsub_rn(pmb, mx), scale_log2));
      const float fa = pma == mx ? 1.0f : fab.x;
      const float fb = pmb == mx ? 1.0f : fab.y;
      // Every operation rounded on its own (no contraction), so the CPU
      // restatement of this combination reproduces it exactly.
      const float inv = __fdiv_rn(1.0f, __fadd_rn(__fmul_rn(la, fa), __fmul_rn(lb, fb)));
      const float wa = __fmul_rn(fa, inv), wb = __fmul_rn(fb, inv);
      uint32_t am = 0;
#pragma unroll
      for (int i = 0; i < kDW / 2; ++i) {
        const float x0 = __fadd_rn(__fmul_rn(__uint_as_float(oa[2 * i]), wa), __fmul_rn(__uint_as_float(ob[2 * i]), wb));
        const float x1 =
            __fadd_rn(__fmul_rn(__uint_as_float(oa[2 * i + 1]), wa), __fmul_rn(__uint_as_float(ob[2 * i + 1]), wb));
        w[i] = pack2(x0, x1, F16);
        am = __vmaxu2(am, w[i] & 0x7fff7fffu);
      }
      // Each warp's 32 rows x D/4 dims leave by one TMA store of its own piece
      // (rows past `seq` are clipped by the tensor map): wait until the warp's
      // previous store has read the piece, write it, store it.
      uint8_t* piece = o_buf + warp * G::kPieceBytes;
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      if constexpr (kDW == 16) {
        // 32-byte rows with the 32-byte swizzle
        *reinterpret_cast<uint4*>(piece + lane * 32 + (((0 ^ (lane >> 2)) & 1) << 4)) =
            make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(piece + lane * 32 + (((1 ^ (lane >> 2)) & 1) << 4)) =
            make_uint4(w[4], w[5], w[6], w[7]);
      } else {
        // 16-byte rows, no swizzle
        *reinterpret_cast<uint4*>(piece + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(&map_out, piece, ph * D + dim0, pt * kTileQ + quarter * 32, pb);
        bulk_commit();
      }
      const int query = pt * kTileQ + row;
      if (row_amax != nullptr && query < seq) {
        const uint32_t m16 = max(am & 0xffffu, am >> 16);
        atomicMax(row_amax + static_cast<size_t>(pb) * seq + query,
                  F16 ? __float_as_uint(from_f16(static_cast<uint16_t>(m16))) : (m16 << 16));
      }
      return true;
    };
    int g = 0;
    bool ok = true;
    for (int j = blockIdx.x; j < jobs && ok; j += gridDim.x) {
      const int p = j / jpp, t0 = (j % jpp) * tpj;
      const int b = p / heads, h = p % heads;
      for (int t = t0; t < t0 + tpj; ++t, ++g) {
        float* mxg = mx_ex + (g & 1) * (2 * 4 * kTileQ);
        const uint32_t lcol = kLCol + (g & 1) * 8;
        // half A
        if (!__all_sync(0xffffffffu, mbar_wait(sa_full, g & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float ma;
        if (!softmax_slice<48, F16, !G::kMmaSums>(lane_base, col_a, valid_a, scale_log2, mxg, sub, row, &mx_full[quarter],
                                    g & 1, abort_flag, lcol + sub, ma)) {
          ok = false;
          break;
        }
        mbar_arrive(pa_full);
        if (pg >= 0 && !epilogue()) {
          ok = false;
          break;
        }
        // half B
        if (!__all_sync(0xffffffffu, mbar_wait(sb_full, g & 1, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        float mb;
        const bool done = sub == 3 ? softmax_slice<32, F16, !G::kMmaSums>(lane_base, col_b, valid_b, scale_log2, mxg + 4 * kTileQ,
                                                            sub, row, &mx_full[4 + quarter], g & 1, abort_flag,
                                                            lcol + 4 + sub, mb)
                                   : softmax_slice<48, F16, !G::kMmaSums>(lane_base, col_b, valid_b, scale_log2, mxg + 4 * kTileQ,
                                                            sub, row, &mx_full[4 + quarter], g & 1, abort_flag,
                                                            lcol + 4 + sub, mb);
        if (!done) {
          ok = false;
          break;
        }
        mbar_arrive(pb_full);
        pb = b, ph = h, pt = t, pg = g, pma = ma, pmb = mb;
      }
    }
    if (ok && pg >= 0) epilogue();
  }
  if (lane == 0 && warp < kSoftWarps) bulk_wait_all();  // output stores complete before the CTA exits
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && *abort_flag) record_status(status, KB_STATUS_TIMEOUT, KB_NO_LAYER);
  if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
}

template <int D, bool F16, bool ROPE>
int launch_tc(const uint16_t* qkv, const float* cos_t, const float* sin_t, uint16_t* out, int batch, int seq,
              int heads, float scale, uint32_t* row_amax, unsigned* status, cudaStream_t stream) {
  auto k_pairs = attention_fa_kernel<D, F16, ROPE, false>;
  auto k_split = attention_fa_kernel<D, F16, ROPE, true>;
  constexpr int kSmemBytes = Geo<D>::kSmemBytes;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    for (auto k : {k_pairs, k_split}) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
      if (e != cudaSuccess) return check_cuda(e, "attention smem attribute");
    }
    configured.fetch_or(bit);
  }
  CUtensorMap map_kv, map_q, map_out;
  memset(&map_kv, 0, sizeof(map_kv));
  memset(&map_q, 0, sizeof(map_q));
  // out [batch, seq, C]: boxes of D/4 dims x 32 tokens of one position (32-byte
  // rows with the 32-byte swizzle for D = 64, 16-byte rows for D = 32)
  const long c = static_cast<long>(heads) * D;
  int rc0 = encode_3d(&map_out, CU_TENSOR_MAP_DATA_TYPE_UINT16, out, c, seq, batch, c * 2,
                      static_cast<long>(seq) * c * 2, D / 4, 32, 1,
                      D == 64 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc0) return rc0;
  if (!ROPE) {
    // [batch * seq rows, 3C columns] 16-bit; boxes of D columns (one head) x rows
    const long cols = 3 * c, rows = static_cast<long>(batch) * seq;
    const CUtensorMapSwizzle swz_mode = D == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    int rc = encode_2d(&map_kv, CU_TENSOR_MAP_DATA_TYPE_UINT16, qkv, cols, rows, cols * 2, D, kKvBox, swz_mode);
    if (!rc) rc = encode_2d(&map_q, CU_TENSOR_MAP_DATA_TYPE_UINT16, qkv, cols, rows, cols * 2, D, kTileQ, swz_mode);
    if (rc) return rc;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  const int pairs = batch * heads;
  // Few pairs (small batches): one query tile per job, so the grid fills more
  // SMs evenly (each job loads its pair's K and V itself).
  const int tiles = (seq + kTileQ - 1) / kTileQ;
  // One tile per job when the pairs fill at most two rounds over the SMs and
  // single tiles take fewer rounds than whole pairs (B = 1 and 16 with 12
  // heads); larger batches keep one K / V load per pair.
  const long sms = num_sms(dev);
  const bool split = pairs < 2 * sms &&
                     (static_cast<long>(pairs) * tiles + sms - 1) / sms < (pairs + sms - 1) / sms * tiles;
  const int jobs = pairs * (split ? tiles : 1);
  auto kern = split ? k_split : k_pairs;
  const int grid = jobs < num_sms(dev) ? jobs : num_sms(dev);
  kern<<<grid, fa_threads<ROPE>(), kSmemBytes, stream>>>(map_kv, map_q, map_out, qkv, cos_t, sin_t, out, pairs, seq,
                                                        heads, scale_log2, row_amax, status);
  return check_cuda(cudaGetLastError(), "attention launch");
}

}  // namespace

// head_dim 64 or 32 and 192 < seq <= 368 (the 361-token board): tcgen05 kernel.
bool attention_tc_supported(int seq, int head_dim) {
  return (head_dim == 64 || head_dim == 32) && seq > kHalfA && seq <= kKeysPad;
}

template <int D>
int attention_tc_dispatch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out, int batch,
                          int seq, int heads, float scale, int f16, cudaStream_t stream, uint32_t* row_amax,
                          unsigned* status) {
  // Null tables: Q and K arrive already rotated (by the QKV projection's epilogue).
  if (rope_cos == nullptr)
    return f16 ? launch_tc<D, true, false>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, status,
                                           stream)
               : launch_tc<D, false, false>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, status,
                                            stream);
  return f16 ? launch_tc<D, true, true>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, status,
                                        stream)
             : launch_tc<D, false, true>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, row_amax, status,
                                         stream);
}

int attention_tc_launch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out, int batch,
                        int seq, int heads, int head_dim, float scale, int f16, cudaStream_t stream,
                        uint32_t* row_amax, unsigned* status) {
  if (head_dim == 64)
    return attention_tc_dispatch<64>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, f16, stream, row_amax,
                                     status);
  return attention_tc_dispatch<32>(qkv, rope_cos, rope_sin, out, batch, seq, heads, scale, f16, stream, row_amax,
                                   status);
}

}  // namespace kb
