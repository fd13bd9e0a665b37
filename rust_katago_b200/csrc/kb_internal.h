// Internal C++ interface between the kernels (*.cu) and the host runtime
// (model, workspace and C-ABI layers).  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/katab200.h"
#include "kb_status.h"

namespace kb {

// Thread-local last error, surfaced through kb_last_error().
void set_error(const std::string& msg);
const char* last_error();

// Returns 0, or sets the thread-local error and returns a KB_E_* code.
int check_cuda(cudaError_t e, const char* what);

int num_sms(int device);

// ------------------------------------------------------------------ GEMM
// Epilogue variants of the tcgen05 GEMM.  `dot` below is the 32-bit TMEM
// accumulator of one output element: an exact int32 for kind::i8, an fp32 sum
// for kind::f16 (bf16 operands) and kind::mxf8f6f4.
enum Epi : int {
  kEpiI32 = 0,       // out_i32 = dot                                (LtPlan::run, int8.rs:542-599)
  kEpiF16 = 1,       // out_f16 = half((f32(dot)*sa)*sw)             (int8_ops.cu:178-185)
  kEpiResF32 = 2,    // res_f32 = res + (f32(dot)*sa)*sw             (int8_ops.cu:187-194)
  kEpi16 = 3,        // out16 = T16(act(v + bias)), optional row amax
  kEpiRes16 = 4,     // res16 = T16(f32(res16) + (v + bias))
  kEpiSwiGLU16 = 5,  // dual tile [gate|up] -> T16(u*(g/(1+e^-g))), gate/up rounded to T16 first
  kEpiF32 = 6,       // out_f32 = v + bias (+ res_f32 when residual != null)
  kEpiRope16 = 7,    // QKV projection: out16 = T16(rot(v)) on columns < rope_cols (Q and K), T16(v) after
};

struct GemmArgs {
  int m = 0, n = 0, k = 0;   // k: padded K in elements of the operand type
  void* out = nullptr;       // output base
  long ldo = 0;              // output row stride in elements
  const float* row_scale = nullptr;  // [m] activation scales (int8 only)
  const float* col_scale = nullptr;  // [n] weight scales (int8 only)
  const float* bias = nullptr;       // [n] or null
  void* residual = nullptr;          // kEpiF32 optional residual input
  long ldr = 0;
  unsigned* row_amax = nullptr;      // [m] |v| bit maximum, or null
  int act = 0;                       // Act
  int out_f16 = 0;                   // 16-bit outputs: 1 = fp16, 0 = bf16
  int n_out = 0;                     // SwiGLU: logical output columns (hidden)
  unsigned* status = nullptr;        // sticky status word (timeouts)
  unsigned layer = KB_NO_LAYER;
  // kGemmBF16 only: the 16-bit operands are binary16 (f16 x f16 -> f32)
  // instead of bfloat16.
  int ab_f16 = 0;
  // Limit of the kernel's bounded waits on work (0 = the default two
  // seconds); only the abort-path test sets it.  Waits that drain copies or
  // MMAs already issued keep the default.
  unsigned long long wait_limit_ns = 0;
  // MXFP8 only: block-scale factors, 1 byte per (row, 32-element K block),
  // stored as [rows_padded/128][k/128][32 rows][4 row groups][4 K blocks].
  const uint8_t* sfa = nullptr;
  const uint8_t* sfb = nullptr;
  // kEpiRope16: rotary tables [rope_heads * rope_hd / 2, rope_seq] (cos, sin of
  // each pair (2p, 2p+1) of a head, token fastest); the row's token is row % rope_seq, columns
  // [0, rope_cols) hold Q then K, rope_cols / 2 = rope_heads * rope_hd wide each.
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int rope_cols = 0, rope_heads = 0, rope_seq = 0, rope_hd = 0;
  // Set by gemm_launch: n % 32 == 0 and col_scale / bias 32-byte aligned, so
  // the epilogue reads their pieces with unchecked 32-byte loads.
  int cols_vec = 0;
};

enum GemmKind : int { kGemmI8 = 0, kGemmBF16 = 1, kGemmMXF8 = 2 };

// Launch C[m,n] = A[m,k] * B[n,k]^T with the selected epilogue.  A and B are
// row-major with K contiguous (K-major), row strides k elements.  Returns 0 or
// a KB_E_* code with the error text set.
int gemm_launch(int kind, int epi, const void* a, const void* b, const GemmArgs& args,
                cudaStream_t stream, int bn_hint = 0);

// Activation quantisers (quant.cu).
int quantize_rows_launch(const void* x, int dtype, long ldx, int rows, int width, int kp, bool rms,
                         const float* gamma, float eps, int bound_f16, int8_t* q, float* scales,
                         unsigned* status, unsigned layer, cudaStream_t stream);
int quantize_rows_amax_launch(const void* x, int dtype, long ldx, const uint32_t* row_amax, int rows, int width,
                              int kp, int8_t* q, float* scales, unsigned* status, unsigned layer,
                              cudaStream_t stream);
// RMSNorm of 16-bit rows to 16-bit rows (the bf16 projection's input):
// out = T16((x * rstd) * gamma), bound_f16 selecting the output type.
int rms16_rows_launch(const void* x, int dtype, long ldx, int rows, int width, const float* gamma, float eps,
                      int bound_f16, uint16_t* out, long ldo, unsigned* status, unsigned layer, cudaStream_t s);

// MXFP8 (mxfp8.cu).  Largest K the block-scaled path accepts (the reference's
// MAX_K, crates/kata_nn/src/backends/mxfp8.rs:31).
constexpr int kMxfp8MaxK = 8192;
// kp = ceil(K/32)*32, blocks4 = ceil(kp/32/4)*4, data = rows*kp bytes,
// scales = ceil(rows/128)*128*blocks4 bytes (mxfp8.rs:56-76).
int mxfp8_dims(long rows, long k, int* kp, int* blocks4, size_t* data_bytes, size_t* scale_bytes);
// Block-32 quantiser of fp32/fp16/bf16 rows (dtype KB_DT_*) into E4M3 [rows, kp]
// and packed UE8M0 scales; clears scale bytes in [scale_bytes, scale_capacity).
int mxfp8_quantize_launch(const void* x, int dtype, long ld, int rows, int k, uint8_t* q, uint8_t* scales,
                          size_t scale_capacity, bool check_weight, unsigned* status, unsigned layer,
                          cudaStream_t stream);
// Fused RMSNorm -> 16-bit boundary -> MXFP8 (quant.cu); row width <= 4096.
int rms_mxfp8_launch(const void* x, int dtype, long ldx, int rows, int width, const float* gamma, float eps,
                     int bound_f16, uint8_t* q, uint8_t* scales, unsigned* status, unsigned layer,
                     cudaStream_t stream);

// Encode a 2-D tensor map (innermost dimension `cols`, row pitch `row_bytes`).
int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, long cols, long rows,
              long row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swz);

// 3-D tensor map: dims (d0 innermost, d1, d2), byte strides of d1 and d2.
int encode_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, long d0, long d1, long d2, long stride1_bytes,
              long stride2_bytes, int box0, int box1, int box2, CUtensorMapSwizzle swz);

// Columns per N tile chosen for a given N (the SwiGLU dual-weight packing
// depends on it).
int gemm_pick_bn(int kind, int epi, int m, int n);

// Output decoding (decode.cu): decode n rows of packed raw heads into the
// decoded layout, post-processed when `legal` is non-null.
kb_postprocess_params default_postprocess_params();
int check_row_params(const kb_row_params* h_rows, int n);
int decode_rows_launch(int n, const float* raw, const kb_row_params* rows, const uint8_t* legal,
                       const kb_postprocess_params& pp, float* out, cudaStream_t s);

}  // namespace kb

// Error codes returned by every C-ABI entry point (0 = success).
#define KB_OK 0
#define KB_E_INVALID 1
#define KB_E_CUDA 2
#define KB_E_STATE 3
#define KB_E_NONFINITE 4
#define KB_E_UNSUPPORTED 5
