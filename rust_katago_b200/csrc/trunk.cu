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
__global__ void stem_gather_kernel(const float* __restrict__ spatial, const float* __restrict__ global,
                                   const int* __restrict__ sym, uint16_t* __restrict__ a, int batch, int nhwc) {
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long total = static_cast<long>(batch) * kSeq * (kStemK / 2);
  if (idx >= total) return;
  const int kpair = static_cast<int>(idx % (kStemK / 2));
  const long row = idx / (kStemK / 2);
  const int b = static_cast<int>(row / kSeq);
  const int t = static_cast<int>(row % kSeq);
  const int y = t / kSide, x = t % kSide;
  const int sm = sym ? (__ldg(sym + b) & 7) : 0;
  float v[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = 2 * kpair + h;
    float val = 0.0f;
    if (k < kInC * 9) {
      const int ic = k / 9, ky = (k % 9) / 3, kx = k % 3;
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
    v[h] = val;
  }
  const __nv_bfloat162 p = __floats2bfloat162_rn(v[0], v[1]);
  reinterpret_cast<uint32_t*>(a)[idx] = *reinterpret_cast<const uint32_t*>(&p);
}

// g = bf16(silu(x * gamma + beta)) over [rows, c] bf16.
__global__ void trunk_tip_kernel(const uint16_t* __restrict__ x, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, uint16_t* __restrict__ g, long total, int c) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int col = static_cast<int>(i % c);
  const float v = __fadd_rn(__fmul_rn(from_bf16(x[i]), __ldg(gamma + col)), __ldg(beta + col));
  g[i] = bits_bf16(kb_silu(v));
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

constexpr int kHeadThreads = 384;

// One CTA per position.  hp: [B*361, 384] fp32 = [p1 | g1 + bias | v1 + bias].
__global__ void __launch_bounds__(kHeadThreads) heads_kernel(const float* __restrict__ hp, HeadWeights w,
                                                            float* __restrict__ policy, float* __restrict__ value,
                                                            float* __restrict__ misc, float* __restrict__ moremisc,
                                                            float* __restrict__ ownership, unsigned* status) {
  bool bad = false;
  __shared__ float pooled_p[288];
  __shared__ float pooled_v[576];
  __shared__ float gproj[96];
  __shared__ float pass1[96];
  __shared__ float vhid[192];
  __shared__ float conv2p[6 * 96];
  __shared__ float ownw[192];
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const float* rows = hp + static_cast<size_t>(b) * kSeq * 384;
  // Pooling: thread c < 96 handles g1 channel c (SiLU then mean, max);
  // threads 96..287 handle v1 channels (SiLU then mean).
  if (tid < 96) {
    float sum = 0.0f, mx = __int_as_float(0xff800000);
    for (int t = 0; t < kSeq; ++t) {
      const float a = kb_silu(rows[t * 384 + 96 + tid]);
      sum += a;
      mx = fmaxf(mx, a);
    }
    const float mean = sum / static_cast<float>(kSeq);
    pooled_p[tid] = mean;
    pooled_p[96 + tid] = mean * 0.5f;
    pooled_p[192 + tid] = mx;
  } else if (tid < 288) {
    const int ch = tid - 96;
    float sum = 0.0f;
    for (int t = 0; t < kSeq; ++t) sum += kb_silu(rows[t * 384 + 192 + ch]);
    const float mean = sum / static_cast<float>(kSeq);
    pooled_v[ch] = mean;
    pooled_v[192 + ch] = mean * 0.5f;
    pooled_v[384 + ch] = mean * 0.15f;
  }
  for (int i = tid; i < 6 * 96; i += kHeadThreads) conv2p[i] = w.conv2p_w[i];
  for (int i = tid; i < 192; i += kHeadThreads) ownw[i] = w.own_w[i];
  __syncthreads();
  // Small matrix-vector products.
  if (tid < 96) {
    float a = 0.0f, p = 0.0f;
    for (int k = 0; k < 288; ++k) {
      a += pooled_p[k] * w.g_matmul[tid * 288 + k];
      p += pooled_p[k] * w.pass1_w[tid * 288 + k];
    }
    gproj[tid] = a + w.bias2[tid];
    pass1[tid] = kb_silu(p + w.pass1_b[tid]);
  } else if (tid < 288) {
    const int ch = tid - 96;
    float a = 0.0f;
    for (int k = 0; k < 576; ++k) a += pooled_v[k] * w.v2_w[ch * 576 + k];
    vhid[ch] = kb_silu(a + w.v2_b[ch]);
  }
  __syncthreads();
  float* pol = policy + static_cast<size_t>(b) * 6 * 362;
  if (tid < 6) {
    float a = 0.0f;
    for (int k = 0; k < 96; ++k) a += pass1[k] * w.pass2_w[tid * 96 + k];
    pol[tid * 362 + 361] = a;
    bad |= !isfinite(a);
  } else if (tid >= 32 && tid < 32 + 21) {
    const int o = tid - 32;
    const float* wr;
    float bias;
    float* dst;
    if (o < 3) {
      wr = w.value_w + o * 192, bias = w.value_b[o], dst = value + b * 3 + o;
    } else if (o < 13) {
      wr = w.misc_w + (o - 3) * 192, bias = w.misc_b[o - 3], dst = misc + b * 10 + (o - 3);
    } else {
      wr = w.moremisc_w + (o - 13) * 192, bias = w.moremisc_b[o - 13], dst = moremisc + b * 8 + (o - 13);
    }
    float a = 0.0f;
    for (int k = 0; k < 192; ++k) a += vhid[k] * wr[k];
    *dst = a + bias;
    bad |= !isfinite(a + bias);
  }
  // Per-token policy moves and ownership.
  for (int t = tid; t < kSeq; t += kHeadThreads) {
    const float* r = rows + t * 384;
    float mv[6] = {0, 0, 0, 0, 0, 0};
    for (int ch = 0; ch < 96; ++ch) {
      const float pa = kb_silu(r[ch] + gproj[ch]);
#pragma unroll
      for (int o = 0; o < 6; ++o) mv[o] += pa * conv2p[o * 96 + ch];
    }
#pragma unroll
    for (int o = 0; o < 6; ++o) {
      pol[o * 362 + t] = mv[o];
      bad |= !isfinite(mv[o]);
    }
    float own = 0.0f;
    for (int ch = 0; ch < 192; ++ch) own += kb_silu(r[192 + ch]) * ownw[ch];
    ownership[static_cast<size_t>(b) * kSeq + t] = own;
    bad |= !isfinite(own);
  }
  // Sticky status: a non-finite value reached an output (reference
  // mxfp8_check_final_outputs_kernel, cuda-kernels/mxfp8.cu:162-177).
  if (bad) record_status(status, KB_STATUS_OUTPUT_NONFINITE, 0xfffffffeu);
}

}  // namespace

int stem_gather_launch(const float* spatial, const float* global, const int* sym, uint16_t* a, int batch,
                       int nhwc, cudaStream_t s) {
  const long total = static_cast<long>(batch) * kSeq * (kStemK / 2);
  stem_gather_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(spatial, global, sym, a, batch,
                                                                                 nhwc);
  return check_cuda(cudaGetLastError(), "stem gather launch");
}

int trunk_tip_launch(const uint16_t* x, const float* gamma, const float* beta, uint16_t* g, long rows, int c,
                     cudaStream_t s) {
  const long total = rows * c;
  trunk_tip_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(x, gamma, beta, g, total, c);
  return check_cuda(cudaGetLastError(), "trunk tip launch");
}

int heads_launch(const float* hp, const float* const* wts, float* policy, float* value, float* misc,
                 float* moremisc, float* ownership, int batch, unsigned* status, cudaStream_t s) {
  HeadWeights w{wts[0], wts[1], wts[2], wts[3], wts[4], wts[5], wts[6], wts[7],
                wts[8], wts[9], wts[10], wts[11], wts[12], wts[13], wts[14]};
  heads_kernel<<<batch, kHeadThreads, 0, s>>>(hp, w, policy, value, misc, moremisc, ownership, status);
  return check_cuda(cudaGetLastError(), "heads launch");
}

}  // namespace kb
