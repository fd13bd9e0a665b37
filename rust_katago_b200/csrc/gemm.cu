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
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (one TMEM lane = one
//               output row per thread), dequant / bias / activation / residual /
//               row-amax, 16-byte global stores.
// The double-buffered accumulator lets the epilogue of tile i overlap the MMAs
// of tile i+1.  Every wait is bounded (kb_ptx.cuh); a timeout records
// KB_STATUS_TIMEOUT in the status word and the kernel returns.
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <string>

#include "kb_internal.h"
#include "kb_numeric.cuh"
#include "kb_ptx.cuh"

namespace kb {
namespace {

constexpr int kBM = 128;
constexpr int kBKBytes = 128;  // one 128-byte swizzle row of K per stage
constexpr int kThreads = 192;

template <int BN>
struct GemmCfg {
  static constexpr int kABytes = kBM * kBKBytes;
  static constexpr int kBBytes = BN * kBKBytes;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes;
  static constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

template <int KIND>
__device__ __forceinline__ float acc_value(uint32_t bits, float sa, float sw) {
  if constexpr (KIND == kGemmI8) {
    return __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(bits)), sa), sw);
  } else {
    return __uint_as_float(bits);
  }
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

__device__ __forceinline__ void store16x32(uint16_t* dst, const uint16_t (&h)[32], int valid,
                                           bool vec) {
  if (vec && valid == 32) {
    uint4* q = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 t;
      t.x = h[8 * i] | (uint32_t(h[8 * i + 1]) << 16);
      t.y = h[8 * i + 2] | (uint32_t(h[8 * i + 3]) << 16);
      t.z = h[8 * i + 4] | (uint32_t(h[8 * i + 5]) << 16);
      t.w = h[8 * i + 6] | (uint32_t(h[8 * i + 7]) << 16);
      q[i] = t;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i < valid) dst[i] = h[i];
  }
}

__device__ __forceinline__ void load16x32(const uint16_t* src, uint16_t (&h)[32], int valid,
                                          bool vec) {
  if (vec && valid == 32) {
    const uint4* q = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 t = q[i];
      const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        h[8 * i + 2 * j] = static_cast<uint16_t>(w[j] & 0xffffu);
        h[8 * i + 2 * j + 1] = static_cast<uint16_t>(w[j] >> 16);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) h[i] = i < valid ? src[i] : 0;
  }
}

// Epilogue of one 32-column chunk held by this thread (row `row`, columns
// col0..col0+31).  `amax` accumulates |value| bits for the row-amax output.
template <int KIND, int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, const uint32_t (&acc)[32], int row,
                                               int col0, float sa, uint32_t& amax) {
  const int valid = min(32, g.n - col0);
  float sw[32], bias[32];
  if constexpr (KIND == kGemmI8) {
    load_vec32(g.col_scale, col0, g.n, sw);
  }
  if constexpr (EPI == kEpi16 || EPI == kEpiRes16 || EPI == kEpiF32) {
    load_vec32(g.bias, col0, g.n, bias);
  }
  if constexpr (EPI == kEpiI32) {
    int32_t* dst = static_cast<int32_t*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
    const bool vec = valid == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    if (vec) {
      int4* q = reinterpret_cast<int4*>(dst);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        q[i] = make_int4(int(acc[4 * i]), int(acc[4 * i + 1]), int(acc[4 * i + 2]),
                         int(acc[4 * i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < valid) dst[i] = static_cast<int32_t>(acc[i]);
    }
  } else if constexpr (EPI == kEpiF16 || EPI == kEpi16) {
    uint16_t h[32];
    const bool f16 = (EPI == kEpiF16) ? true : (g.out_f16 != 0);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float v = acc_value<KIND>(acc[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f);
      if constexpr (EPI == kEpi16) {
        if (g.bias) v = __fadd_rn(v, bias[i]);
        v = apply_act(v, g.act);
      }
      h[i] = bits16(v, f16);
      if (i < valid) amax = max(amax, abs_bits(from16(h[i], f16)));
    }
    uint16_t* dst = static_cast<uint16_t*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
    store16x32(dst, h, valid, (reinterpret_cast<uintptr_t>(dst) & 15) == 0);
  } else if constexpr (EPI == kEpiResF32) {
    float* dst = static_cast<float*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
    const bool vec = valid == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    if (vec) {
      float4* q = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float4 r = q[i];
        r.x = __fadd_rn(r.x, acc_value<KIND>(acc[4 * i], sa, sw[4 * i]));
        r.y = __fadd_rn(r.y, acc_value<KIND>(acc[4 * i + 1], sa, sw[4 * i + 1]));
        r.z = __fadd_rn(r.z, acc_value<KIND>(acc[4 * i + 2], sa, sw[4 * i + 2]));
        r.w = __fadd_rn(r.w, acc_value<KIND>(acc[4 * i + 3], sa, sw[4 * i + 3]));
        q[i] = r;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < valid) dst[i] = __fadd_rn(dst[i], acc_value<KIND>(acc[i], sa, sw[i]));
    }
  } else if constexpr (EPI == kEpiRes16) {
    const bool f16 = g.out_f16 != 0;
    uint16_t* dst = static_cast<uint16_t*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    uint16_t h[32];
    load16x32(dst, h, valid, vec);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float v = acc_value<KIND>(acc[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f);
      if (g.bias) v = __fadd_rn(v, bias[i]);
      h[i] = bits16(__fadd_rn(from16(h[i], f16), v), f16);
    }
    store16x32(dst, h, valid, vec);
  } else if constexpr (EPI == kEpiF32) {
    float* dst = static_cast<float*>(g.out) + static_cast<size_t>(row) * g.ldo + col0;
    const float* res = g.residual ? static_cast<const float*>(g.residual) +
                                        static_cast<size_t>(row) * g.ldr + col0
                                  : nullptr;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < valid) {
        float v = acc_value<KIND>(acc[i], sa, KIND == kGemmI8 ? sw[i] : 1.0f);
        if (g.bias) v = __fadd_rn(v, bias[i]);
        if (res) v = __fadd_rn(res[i], v);
        dst[i] = v;
      }
    }
  }
}

template <int KIND, int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                const __grid_constant__ CUtensorMap tmap_b, const GemmArgs g) {
  using Cfg = GemmCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  constexpr int kElemBytes = (KIND == kGemmBF16) ? 2 : 1;
  constexpr int kBKElems = kBKBytes / kElemBytes;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * Cfg::kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k_blocks = (g.k + kBKElems - 1) / kBKElems;
  const int tiles_m = (g.m + kBM - 1) / kBM;
  const int tiles_n = (g.n + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
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
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = ring + s * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
          tma_load_2d(sa, &tmap_a, &full[s], kb * kBKElems, mb * kBM);
          tma_load_2d(sa + Cfg::kABytes, &tmap_b, &full[s], kb * kBKElems, nb * BN);
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
      const uint32_t idesc = make_idesc<KIND>(BN);
      int s = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t aph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], aph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + s * Cfg::kStageBytes);
          const uint64_t adesc = sw128_desc(a_addr);
          const uint64_t bdesc = sw128_desc(a_addr + Cfg::kABytes);
#pragma unroll
          for (int kk = 0; kk < kBKBytes / 32; ++kk) {
            // +32 bytes along K inside the swizzle atom = +2 in the address field.
            mma_issue<KIND>(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0, 0, 0);
          }
          tc_commit(&empty[s]);
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
    }
  } else {
    // ---------------- epilogue warps (TMEM lane quarter = warp % 4)
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t aph = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aph, abort_flag))) break;
      tc_fence_after();
      const int mb = tile / tiles_n, nb = tile % tiles_n;
      const int row = mb * kBM + quarter * 32 + lane;
      const bool row_ok = row < g.m;
      float sa = 1.0f;
      if constexpr (KIND == kGemmI8 && EPI != kEpiI32) sa = row_ok ? __ldg(g.row_scale + row) : 0.0f;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      uint32_t amax = 0;
      if constexpr (EPI == kEpiSwiGLU16) {
        // Tile columns [0, BN/2) are gate channels, [BN/2, BN) the matching up
        // channels (the dual weight is interleaved per tile at load).
        const bool f16 = g.out_f16 != 0;
#pragma unroll 1
        for (int j = 0; j < BN / 64; ++j) {
          uint32_t vg[32], vu[32];
          tmem_ld32(taddr + j * 32, vg);
          tmem_ld32(taddr + BN / 2 + j * 32, vu);
          tmem_ld_wait();
          const int gcol0 = nb * BN + j * 32;
          const int ocol0 = nb * (BN / 2) + j * 32;
          if (row_ok && ocol0 < g.n_out) {
            float swg[32], swu[32];
            if constexpr (KIND == kGemmI8) {
              load_vec32(g.col_scale, gcol0, g.n, swg);
              load_vec32(g.col_scale, gcol0 + BN / 2, g.n, swu);
            }
            const int valid = min(32, g.n_out - ocol0);
            uint16_t h[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float gv = from16(bits16(acc_value<KIND>(vg[i], sa, KIND == kGemmI8 ? swg[i] : 1.0f), f16), f16);
              const float uv = from16(bits16(acc_value<KIND>(vu[i], sa, KIND == kGemmI8 ? swu[i] : 1.0f), f16), f16);
              h[i] = bits16(__fmul_rn(uv, kb_silu(gv)), f16);
              if (i < valid) amax = max(amax, abs_bits(from16(h[i], f16)));
            }
            uint16_t* dst = static_cast<uint16_t*>(g.out) + static_cast<size_t>(row) * g.ldo + ocol0;
            store16x32(dst, h, valid, (reinterpret_cast<uintptr_t>(dst) & 15) == 0);
          }
        }
      } else {
#pragma unroll 1
        for (int j = 0; j < BN / 32; ++j) {
          uint32_t v[32];
          tmem_ld32(taddr + j * 32, v);
          tmem_ld_wait();
          const int col0 = nb * BN + j * 32;
          if (row_ok && col0 < g.n) epilogue_chunk<KIND, EPI>(g, v, row, col0, sa, amax);
        }
      }
      if (g.row_amax != nullptr && row_ok) atomicMax(g.row_amax + row, amax);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1;
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
int make_map(CUtensorMap* map, const void* base, int kind, long rows, long k, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return KB_E_CUDA;
  }
  const int elem = kind == kGemmBF16 ? 2 : 1;
  const CUtensorMapDataType dt =
      kind == kGemmBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * elem};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBKBytes / elem), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (code " + std::to_string(int(r)) + ")");
    return KB_E_CUDA;
  }
  return KB_OK;
}

template <int KIND, int BN, int EPI>
int launch_one(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_kernel<KIND, BN, EPI>;
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
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ma, mb, g);
  return check_cuda(cudaGetLastError(), "gemm launch");
}

template <int KIND, int BN>
int dispatch_epi(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g,
                 cudaStream_t s) {
  switch (epi) {
    case kEpiI32: return launch_one<KIND, BN, kEpiI32>(ma, mb, g, s);
    case kEpiF16: return launch_one<KIND, BN, kEpiF16>(ma, mb, g, s);
    case kEpiResF32: return launch_one<KIND, BN, kEpiResF32>(ma, mb, g, s);
    case kEpi16: return launch_one<KIND, BN, kEpi16>(ma, mb, g, s);
    case kEpiRes16: return launch_one<KIND, BN, kEpiRes16>(ma, mb, g, s);
    case kEpiSwiGLU16: return launch_one<KIND, BN, kEpiSwiGLU16>(ma, mb, g, s);
    case kEpiF32: return launch_one<KIND, BN, kEpiF32>(ma, mb, g, s);
  }
  set_error("unknown GEMM epilogue");
  return KB_E_INVALID;
}

}  // namespace

int gemm_pick_bn(int kind, int epi, int n) {
  (void)kind;
  if (epi == kEpiSwiGLU16) return 256;
  if (n % 256 == 0 || n > 2048) return 256;
  return 128;
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
  if (kind == kGemmI8 && epi != kEpiI32 && (g.row_scale == nullptr || g.col_scale == nullptr)) {
    set_error("INT8 dequant epilogue needs row and column scales");
    return KB_E_INVALID;
  }
  const int bn = bn_hint ? bn_hint : gemm_pick_bn(kind, epi, g.n);
  CUtensorMap ma, mb;
  int rc = make_map(&ma, a, kind, g.m, g.k, kBM);
  if (rc) return rc;
  rc = make_map(&mb, b, kind, g.n, g.k, bn);
  if (rc) return rc;
  if (kind == kGemmI8) {
    return bn == 256 ? dispatch_epi<kGemmI8, 256>(epi, ma, mb, g, stream)
                     : dispatch_epi<kGemmI8, 128>(epi, ma, mb, g, stream);
  }
  if (kind == kGemmBF16) {
    return bn == 256 ? dispatch_epi<kGemmBF16, 256>(epi, ma, mb, g, stream)
                     : dispatch_epi<kGemmBF16, 128>(epi, ma, mb, g, stream);
  }
  set_error("GEMM kind not supported");
  return KB_E_UNSUPPORTED;
}

}  // namespace kb
