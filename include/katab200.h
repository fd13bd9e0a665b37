/* katab200 — C ABI of the B200-native (sm_100a) quantized KataGo trunk forward.
 *
 * Plain C: opaque handles, plain pointers and sizes, `int` status codes
 * (0 = success, see KB_E_*), a thread-local kb_last_error() string.  The style
 * follows the reference's own C-ABI shims
 * (crates/kata_nn/cuda-host/dual_ffn_cutlass.cu:142-216, cpp-shim/src/trt_shim.h:15-202),
 * so a Rust `extern "C"` block binds it the same way the reference binds those.
 *
 * Device pointers are CUDA device addresses on the current device.  `stream`
 * is a cudaStream_t passed as uintptr_t (0 = legacy default stream).
 * Every entry point validates shapes and buffers on the host and fails closed:
 * there is no CPU or FP16 fallback (reference: int8.rs:471, mxfp8.rs:40).
 */
#ifndef KATAB200_H
#define KATAB200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KB_API __attribute__((visibility("default")))
#else
#define KB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define KB_OK 0
#define KB_E_INVALID 1     /* bad shape, pointer, stream or argument */
#define KB_E_CUDA 2        /* a CUDA runtime/driver call failed */
#define KB_E_STATE 3       /* object used from the wrong stream/device or not ready */
#define KB_E_NONFINITE 4   /* the status word reported NaN/Inf (outputs withheld) */
#define KB_E_UNSUPPORTED 5 /* device is not sm_100 or feature not built */

/* Activation / output element types. */
#define KB_DT_F32 0
#define KB_DT_F16 1
#define KB_DT_BF16 2

/* Epilogues of kb_int8_linear (all start from the exact int32 dot). */
#define KB_EPI_I32 0     /* out_i32 = dot */
#define KB_EPI_F16 1     /* out_f16 = half((f32(dot)*sa)*sw) */
#define KB_EPI_RES_F32 2 /* res_f32 = res + (f32(dot)*sa)*sw */
#define KB_EPI_16 3      /* out16 = T16(act((f32(dot)*sa)*sw + bias)) */
#define KB_EPI_RES16 4   /* res16 = T16(f32(res16) + ((f32(dot)*sa)*sw + bias)) */
#define KB_EPI_SWIGLU16 5 /* dual weight: out16 = T16(T16(u) * silu(T16(g))) */
#define KB_EPI_F32 6     /* out_f32 = (f32(dot)*sa)*sw + bias */

#define KB_ACT_NONE 0
#define KB_ACT_GELU 1
#define KB_ACT_SILU 2

/* Weight layouts for kb_int8_weight_upload. */
#define KB_LAYOUT_PLAIN 0       /* [N, kp] rows as given */
#define KB_LAYOUT_SWIGLU_DUAL 1 /* input [gate(H); up(H)] x K, stored tile-interleaved */

/* ------------------------------------------------------------------ misc */

/* Last error message of this thread ("" if none).
 * Replaces: katago_trt_last_error (cpp-shim/src/trt_shim.h:33). */
KB_API const char* kb_last_error(void);

/* ABI version of this library (major*10000 + minor*100 + patch). */
KB_API int kb_version(void);

/* Checks that `device` is an sm_100 GPU usable by this library.
 * Replaces: the architecture gate of CudaRuntime::new (src/backends/cuda.rs:454-506)
 * and mxfp8.rs:117-127. */
KB_API int kb_device_check(int device);

/* ------------------------------------------------------------------ INT8 weights */

/* CPU per-output-channel symmetric weight quantisation (load time).
 * w: fp32 [n, k] row-major (out-first).  Writes q [n, kp] (kp = ceil(k/16)*16,
 * zero padded) and scales [n]: s = max(amax/127, FLT_MIN) (1 for a zero row),
 * q = clamp(rne(w/s), +-127).  Rejects NaN/Inf, n % 4 != 0, k > 8192.
 * Replaces: QuantizedWeights::new (src/backends/int8.rs:171-211). */
KB_API int kb_int8_quantize_weights(const float* w, int n, int k, int8_t* q, float* scales);

typedef struct kb_int8_weight kb_int8_weight;

/* Quantise on the CPU and upload to the current device.  layout: KB_LAYOUT_*.
 * For KB_LAYOUT_SWIGLU_DUAL, w is [2H, k] = [gate; up] and n = 2H.
 * Replaces: Int8Weight::upload (src/backends/int8.rs:222-236) and the dual
 * packing of cuda_exec.rs:2004-2009. */
KB_API int kb_int8_weight_upload(const float* w, int n, int k, int layout, kb_int8_weight** out);

/* Shape and device buffers of an uploaded weight (q: [n_stored, kp] int8,
 * scales: [n_stored] fp32; n_stored > n only for padded SwiGLU layouts). */
KB_API int kb_int8_weight_info(const kb_int8_weight* w, int* n, int* k, int* kp, int* n_stored,
                        const int8_t** q, const float** scales);

KB_API void kb_int8_weight_destroy(kb_int8_weight* w);

/* ------------------------------------------------------------------ INT8 kernels */

/* dots[m, n] (int32) = a[m, kp] (int8) * w[n, kp]^T, exact integer arithmetic.
 * Replaces: LtPlan::run / Int8Workspace::integer_gemm (src/backends/int8.rs:542-599, :925-1010). */
KB_API int kb_int8_gemm_i32(const int8_t* a, const int8_t* w, int32_t* dots, int m, int n, int kp,
                     uintptr_t stream);

/* tcgen05 INT8 GEMM with a fused epilogue (KB_EPI_*).  out has row stride ldo
 * elements; for KB_EPI_RES_* it is read and written in place.  The dequantised
 * value is (f32(dot) * sa) * sw with two rounded multiplies (the reference's
 * order); with a bias (nullable, [n]) it is fma(f32(dot) * sa, sw, bias), the
 * bias added by the same fused multiply-add.  out_dtype selects
 * fp16/bf16 for the 16-bit epilogues.  row_amax (nullable, [m] uint32) receives
 * an atomic max of |output| bits for a following per-token quantiser.
 * n_out: logical output width for KB_EPI_SWIGLU16 (hidden), ignored otherwise.
 * Replaces: integer_gemm + int8_dequantize_{half,residual}_kernel
 * (int8_ops.cu:178-194) + int8_swiglu_quantize's dequant/SwiGLU half (int8_ops.cu:93-138). */
KB_API int kb_int8_linear(const int8_t* a, const float* sa, const int8_t* w, const float* sw,
                   const float* bias, int m, int n, int kp, int epilogue, int act, int out_dtype,
                   void* out, int ldo, int n_out, uint32_t* row_amax, uintptr_t stream);

/* Per-token dynamic quantisation of rows x[rows, width] (row stride `stride`
 * elements, dtype KB_DT_*) into q[rows, kp] + scales[rows].
 * Replaces: int8_quantize_rows{_warp,}_kernel (int8_ops.cu:62-89, :140-176). */
KB_API int kb_int8_quantize_rows(const void* x, int dtype, int rows, int width, int stride, int kp,
                          int8_t* q, float* scales, uintptr_t stream);

/* Streaming variant for 16-bit rows whose |value| bit maximum is already known
 * (row_amax [rows], uint32 = max of (bits & 0x7fffffff) of the fp32 values,
 * as written by a GEMM epilogue's row_amax): same scales and integers as
 * kb_int8_quantize_rows, one pass, no row reduction.  Row starts must be
 * 16-byte aligned (stride % 8 == 0).  No single reference counterpart: it
 * splits int8_swiglu_quantize's row reduction (int8_ops.cu:93-138) into the
 * producing GEMM. */
KB_API int kb_int8_quantize_rows_amax(const void* x, int dtype, int rows, int width, int stride, int kp,
                                      const uint32_t* row_amax, int8_t* q, float* scales, uintptr_t stream);

/* Fused RMSNorm -> 16-bit boundary (boundary_dtype KB_DT_F16 or KB_DT_BF16)
 * -> per-token INT8 quantisation.
 * Replaces: int8_rms_quantize{384,512}_kernel (int8_ops.cu:8-57) and
 * rms_norm_f32_w4_kernel (executor.cu:478-519) + quantiser. */
KB_API int kb_int8_rms_quantize(const void* x, int dtype, int rows, int width, int stride,
                         const float* gamma, float eps, int boundary_dtype, int kp, int8_t* q,
                         float* scales, uintptr_t stream);

/* ------------------------------------------------------------------ INT8 workspace */

typedef struct kb_int8_workspace kb_int8_workspace;

/* Scratch buffers for `rows` tokens bound to one stream: quantised activations
 * [rows, max_k], scales [rows], 16-bit hidden [rows, max_n].
 * Replaces: Int8Workspace::new (src/backends/int8.rs:830-869). */
KB_API int kb_int8_workspace_create(uintptr_t stream, int rows, int max_k, int max_n,
                             kb_int8_workspace** out);
KB_API void kb_int8_workspace_destroy(kb_int8_workspace* ws);

/* Device buffers of the workspace (for tests and diagnostics). */
KB_API int kb_int8_workspace_buffers(kb_int8_workspace* ws, int8_t** quantized, float** scales,
                              void** hidden);

/* fp16 input [rows, stride] -> quantise -> GEMM -> half((dot*sa)*sw) into
 * output [rows, n].  Replaces: Int8Workspace::project_half (int8.rs:1012-1050). */
KB_API int kb_int8_project_half(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input,
                         int stride, const kb_int8_weight* w, uint16_t* output, int rows);

/* Same, adding into an fp32 residual [rows, n].
 * Replaces: Int8Workspace::project_residual (int8.rs:1052-1102). */
KB_API int kb_int8_project_residual(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input,
                             int stride, const kb_int8_weight* w, float* residual, int rows);

/* SwiGLU FFN with the reference's fp16 boundaries: input fp16 [rows, mid]
 * -> dual GEMM + SwiGLU -> requant -> down GEMM -> fp32 residual add.
 * dual: KB_LAYOUT_SWIGLU_DUAL weight [2H, mid]; down: [mid, H].
 * Replaces: Int8Workspace::ffn (int8.rs:1104-1125). */
KB_API int kb_int8_ffn(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input,
                const kb_int8_weight* dual, const kb_int8_weight* down, float* output, int rows);

/* RMSNorm(residual fp32) -> fp16 -> quant -> SwiGLU FFN -> residual add.
 * Replaces: Int8Workspace::ffn_rms (int8.rs:1135-1172). */
KB_API int kb_int8_ffn_rms(kb_int8_workspace* ws, uintptr_t stream, const float* gamma, float eps,
                    const kb_int8_weight* dual, const kb_int8_weight* down, float* residual,
                    int rows);

/* BASELINE-topology FFN block on a bf16 residual stream [rows, C]:
 * RMSNorm -> bf16 -> quant -> up GEMM (+bias) + GELU -> bf16 hidden -> requant
 * -> down GEMM (+bias) -> residual add.  up: [F, C], down: [C, F].
 * No reference counterpart (the reference FFN is SwiGLU); built from the same
 * pieces as kb_int8_ffn_rms. */
KB_API int kb_int8_ffn_gelu_rms(kb_int8_workspace* ws, uintptr_t stream, const float* gamma, float eps,
                         const kb_int8_weight* up, const float* up_bias,
                         const kb_int8_weight* down, const float* down_bias, uint16_t* residual,
                         int rows);

/* The same GELU FFN block as kb_int8_ffn_gelu_rms, for callers that cannot
 * allocate device memory where they evaluate (a search thread evaluating a few
 * positions mid-move, where cudaMalloc may synchronise the device; a host that
 * owns all device memory under a fixed budget).  It takes no workspace and
 * allocates nothing: its scratch is one static 8 MiB device array per device
 * (reserved when the library is loaded, held until exit), so `rows` is limited
 * to what fits (about 900 tokens, 2 positions, for C=768, F=3072); larger
 * calls fail with KB_E_INVALID and say the limit.  The weights must live on
 * the current device (KB_E_STATE otherwise).  The first call on each device
 * (or kb_int8_noalloc_prepare) looks the array's address up
 * (cudaGetSymbolAddress) and should come before any stream capture.  All calls on a device share the array: calls
 * that overlap on the GPU race; nothing in it needs clearing between calls.
 * No counterpart in the reference. */
KB_API int kb_int8_ffn_gelu_rms_noalloc(uintptr_t stream, const float* gamma, float eps,
                                        const kb_int8_weight* up, const float* up_bias,
                                        const kb_int8_weight* down, const float* down_bias,
                                        uint16_t* residual, int rows);

/* Looks up the current device's no-alloc scratch address now, so that a caller
 * that captures kb_int8_ffn_gelu_rms_noalloc into a CUDA graph can do the
 * lookup before the capture begins.  Allocates nothing.  Optional: the first
 * kb_int8_ffn_gelu_rms_noalloc call on a device does the same.
 * No counterpart in the reference. */
KB_API int kb_int8_noalloc_prepare(void);

/* ------------------------------------------------------------------ bf16 GEMM */

/* out = a[m,k] (bf16) * w[n,k]^T (bf16) with fp32 accumulation on tcgen05
 * (kind::f16) and a fused epilogue: KB_EPI_16 (bf16/fp16 out, bias, act),
 * KB_EPI_RES16 (16-bit residual add) or KB_EPI_F32 (fp32 out + bias [+ residual]).
 * Replaces: the FP16 hgemm_* linears of the outer trunk (gemm_v2.cu:397-1153). */
KB_API int kb_bf16_linear(const uint16_t* a, const uint16_t* w, const float* bias, int m, int n, int k,
                   int epilogue, int act, int out_dtype, void* out, int ldo, uintptr_t stream);

/* The same GEMM with binary16 operands (f16 x f16, fp32 accumulation): the
 * nested trunk's outer linears and unquantised projections.
 * Replaces: the FP16 hgemm / hgemm_residual linears of the outer trunk
 * (cuda_exec.rs:1170-1240, gemm_v2.cu:397-1153). */
KB_API int kb_f16_linear(const uint16_t* a, const uint16_t* w, const float* bias, int m, int n, int k,
                         int epilogue, int act, int out_dtype, void* out, int ldo, uintptr_t stream);

/* ------------------------------------------------------------------ attention */

/* Multi-head attention over the 361 board tokens with RoPE on Q and K:
 * qkv [batch*361, 3*heads*head_dim] ([Q | K | V], 16-bit, dtype KB_DT_BF16 or
 * KB_DT_F16), rope_cos/rope_sin fp32 [361, heads, head_dim/2] (interleaved
 * pairs), out [batch*361, heads*head_dim]; softmax(q.k * scale) over all keys.
 * rope_cos and rope_sin may both be NULL when Q and K are already rotated (the
 * trunk rotates them in the QKV projection's epilogue).
 * head_dim 32 or 64.  Replaces: attention_fa2_q64_kernel
 * (cuda-kernels/attention_fa2_q64.cu:82-390) via cuda_exec.rs:3442. */
KB_API int kb_attention(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out,
                        int batch, int heads, int head_dim, float scale, int dtype, uintptr_t stream);

/* The trunk's attention launch: Q and K already rotated, and row_amax
 * [batch*361] (zeroed by the caller) raised with atomicMax to the fp32 bits of
 * each output row's largest |16-bit value|, the input of
 * kb_int8_quantize_rows_amax for the out-projection.
 * Replaces: attention_fa2_q64_kernel (attention_fa2_q64.cu:82-390) followed by
 * the row maximum of int8_quantize_rows_kernel (int8_ops.cu:62-89). */
KB_API int kb_attention_amax(const uint16_t* qkv, uint16_t* out, uint32_t* row_amax, int batch, int heads,
                             int head_dim, float scale, int dtype, uintptr_t stream);

/* ------------------------------------------------------------------ MXFP8 (block-scaled E4M3) */

/* Status word [flags, first_layer]: flags OR-ed, first_layer = first layer
 * that reported (0xffffffff = none); same protocol as mxfp8.rs:22-30. */
#define KB_STATUS_NAN 1u               /* NaN input to a quantiser */
#define KB_STATUS_INF 2u               /* infinite input to a quantiser */
#define KB_STATUS_OUTPUT_NONFINITE 4u  /* a non-finite value reached an output */
#define KB_STATUS_WEIGHT_OVERFLOW 8u   /* an MXFP8 weight decodes to a non-finite value */
#define KB_STATUS_UNSUPPORTED_ARCH 16u /* kernel ran on a device other than sm_100 */
#define KB_STATUS_TIMEOUT 32u          /* a bounded device wait gave up (no hang, no trap) */

/* MXFP8 projection outputs (Mxfp8Output, src/backends/mxfp8.rs:382-400, plus bf16). */
#define KB_MX_OUT_HALF 0           /* out f16 [rows, n] = half(acc) */
#define KB_MX_OUT_FLOAT 1          /* out f32 = acc */
#define KB_MX_OUT_FLOAT_RESIDUAL 2 /* out f32 = out + acc (beta = 1) */
#define KB_MX_OUT_BF16 3           /* out bf16 = bf16(act(acc + bias)) */
#define KB_MX_OUT_BF16_RESIDUAL 4  /* out bf16 = bf16(f32(out) + (acc + bias)) */

/* Reset a status word to [0, 0xffffffff] on `stream`.
 * Replaces: mxfp8_begin_forward_kernel (cuda-kernels/mxfp8.cu:91-96) via
 * Mxfp8Workspace::begin_forward (src/backends/mxfp8.rs:977). */
KB_API int kb_status_reset(uint32_t* status, uintptr_t stream);

/* kp = ceil(k/32)*32; blocks4 = ceil(kp/128)*4; data bytes = rows*kp; scale bytes
 * = ceil(rows/128)*128*blocks4.  Rejects rows <= 0, k outside 1..8192 and sizes
 * beyond 32-bit indexing.  Replaces: dimensions (src/backends/mxfp8.rs:56-76). */
KB_API int kb_mxfp8_dimensions(int rows, int k, int* kp, int* blocks4, size_t* data_bytes, size_t* scale_bytes);

/* Block-32 quantiser: x [rows, stride] (dtype KB_DT_F32/F16/BF16) -> q E4M3
 * [rows, kp] and scales (UE8M0, packed 512-byte tiles of 128 rows x 4 blocks:
 * byte ((row/128)*(blocks4/4) + block/4)*512 + (row%32)*16 + (row%128/32)*4 +
 * block%4).  Scale bytes of padding rows/blocks and of [scale bytes,
 * scale_capacity) are zeroed.  NaN/Inf inputs set KB_STATUS_NAN/INF with `layer`
 * and give their block scale 127 and zero bytes.
 * Replaces: mxfp8_quantize_{half,float}_kernel + mxfp8_clear_scales_kernel
 * (cuda-kernels/mxfp8.cu:36-149) via Mxfp8Kernels::quantize (mxfp8.rs:209-270). */
KB_API int kb_mxfp8_quantize(const void* x, int dtype, int rows, int k, int stride, uint8_t* q, uint8_t* scales,
                             size_t scale_capacity, uint32_t* status, uint32_t layer, uintptr_t stream);

/* Fused RMSNorm -> 16-bit boundary (boundary_dtype KB_DT_F16 or KB_DT_BF16) ->
 * MXFP8: v = T16((x * rstd) * gamma) with the same rstd and rounding as
 * kb_int8_rms_quantize, then the block-32 quantiser of kb_mxfp8_quantize on v.
 * width <= 4096.  The whole scale buffer (scale_capacity bytes) is cleared first.
 * Replaces: rms_norm_f32_w4_kernel (cuda-kernels/executor.cu:478-519) followed by
 * mxfp8_quantize_half_kernel (cuda-kernels/mxfp8.cu:103-108). */
KB_API int kb_mxfp8_rms_quantize(const void* x, int dtype, int rows, int width, int stride, const float* gamma,
                                 float eps, int boundary_dtype, uint8_t* q, uint8_t* scales, size_t scale_capacity,
                                 uint32_t* status, uint32_t layer, uintptr_t stream);

typedef struct kb_mxfp8_weight kb_mxfp8_weight;

/* Quantise an original fp32 weight [n, stride] (first k columns used) on the
 * current device and keep it resident (immutable).  Rejects NaN/Inf (host
 * scan) and weights whose decoded value overflows fp32 (device check).
 * Replaces: Mxfp8Weight::upload_from_f32 (src/backends/mxfp8.rs:290-350). */
KB_API int kb_mxfp8_weight_upload(const float* w, int n, int k, int stride, kb_mxfp8_weight** out);

KB_API int kb_mxfp8_weight_info(const kb_mxfp8_weight* w, int* n, int* k, int* kp, const uint8_t** q,
                                const uint8_t** scales, size_t* scale_bytes);

KB_API void kb_mxfp8_weight_destroy(kb_mxfp8_weight* w);

/* Block-scaled GEMM on quantised activations: out[rows, n] from a_q [rows, kp]
 * and a_scales (packed, as produced by kb_mxfp8_quantize for this kp) against
 * the weight, fp32 accumulation on tcgen05 (kind::mxf8f6f4.block_scale,
 * UE8M0 x 32).  out_kind KB_MX_OUT_*; bias (n fp32, or NULL) and act
 * (KB_ACT_*) apply to KB_MX_OUT_BF16 / KB_MX_OUT_BF16_RESIDUAL only (act: BF16).  A non-finite output sets
 * KB_STATUS_OUTPUT_NONFINITE with `layer`.  ldo: output row stride in elements.
 * Replaces: LtPlan::run (src/backends/mxfp8.rs:683-720) + mxfp8_check_*_output_kernel
 * (cuda-kernels/mxfp8.cu:151-159). */
KB_API int kb_mxfp8_gemm(const uint8_t* a_q, const uint8_t* a_scales, int rows, const kb_mxfp8_weight* w,
                         const float* bias, int act, int out_kind, void* out, long ldo, uint32_t* status,
                         uint32_t layer, uintptr_t stream);

/* One MXFP8 projection: quantise x [rows, stride] (16-bit, dtype KB_DT_F16 or
 * KB_DT_BF16) into the caller's scratch (q: rows*kp bytes, scales: at least the
 * scale bytes of (rows, kp), cleared beyond), then kb_mxfp8_gemm.
 * Replaces: Mxfp8Workspace::project{,_half,_f32} (src/backends/mxfp8.rs:1055-1159). */
KB_API int kb_mxfp8_project(const kb_mxfp8_weight* w, const void* x, int dtype, int rows, int stride,
                            uint8_t* q_scratch, uint8_t* scale_scratch, size_t scale_capacity, int out_kind,
                            void* out, long ldo, uint32_t* status, uint32_t layer, uintptr_t stream);

/* ------------------------------------------------------------------ tests of the abort path */

/* Test entry points for the bounded device waits (no reference counterpart;
 * the reference's kernels do not wait on one another).  Every wait inside this
 * library's kernels gives up after two seconds, records KB_STATUS_TIMEOUT in
 * the status word, lets the copies and MMAs it has issued finish, frees its
 * tensor memory and returns, so a fault never hangs the GPU. */

/* One CTA waits `limit_ns` (1 ns .. 1 s) on a barrier that nothing arrives at,
 * then records KB_STATUS_TIMEOUT in status[2]. */
KB_API int kb_test_wait_timeout(unsigned long long limit_ns, uint32_t* status, uintptr_t stream);

/* kb_int8_gemm_i32 with the limit of its waits on work shortened to
 * wait_limit_ns (1 ns .. 2 s): with a limit shorter than the GEMM the kernel
 * aborts, records KB_STATUS_TIMEOUT in status[2] and returns (dots are then
 * partial); the stream and the device stay usable. */
KB_API int kb_test_int8_gemm_i32_wait_limit(const int8_t* a, const int8_t* w, int32_t* dots, int m, int n, int kp,
                                            unsigned long long wait_limit_ns, uint32_t* status, uintptr_t stream);

/* ------------------------------------------------------------------ model and evaluator */

#define KB_PREC_INT8 0  /* W8A8: every trunk linear INT8 x INT8 -> INT32 */
#define KB_PREC_MXFP8 1 /* every trunk linear E4M3 x E4M3 with UE8M0 scales per 32 K, fp32 accumulate */

/* Per-projection precision (the reference's LayerPrecision of a precision
 * recipe, crates/kata_nn/src/quantization_plan.rs:36-80): */
#define KB_PROJ_FOLLOW 0 /* the model's `precision` */
#define KB_PROJ_INT8 1   /* W8A8, per-token / per-channel absmax scales, int32 accumulate */
#define KB_PROJ_MXFP8 2  /* block-32 E4M3 + UE8M0, fp32 accumulate */
#define KB_PROJ_BF16 3   /* unquantised 16-bit projection, fp32 accumulate: bf16 weights and activations
                            in the flat topology, binary16 (the reference's FP16) in the nested one */
#define KB_PROJ_QKV 0
#define KB_PROJ_OUT 1
#define KB_PROJ_FFN_UP 2
#define KB_PROJ_FFN_DOWN 3

/* Trunk topologies. */
#define KB_TOPO_FLAT 0   /* BASELINE: num_blocks x [RMSNorm, attention, RMSNorm, GELU FFN] on a bf16
                            residual stream of width C (below) */
#define KB_TOPO_NESTED 1 /* the reference's TF3 nested bottleneck (native_model.rs:79-124): per outer
                            block, gate-SiLU of the fp32 raw trunk, C -> mid linear, pairs_per_block x
                            [RMSNorm, attention (head_dim 32), RMSNorm, SwiGLU FFN mid -> 2H -> mid] on an
                            fp32 stream of width mid, gate-SiLU, mid -> C linear added to the raw trunk;
                            binary16 at every 16-bit boundary, INT8 FFN */

/* Trunk shape (BASELINE b11c768: C=768, 11 blocks, 12 heads x 64, F=3072;
 * the reference's TF3 b11c768: nested, C=768, mid 384, 11 blocks of 3 pairs,
 * 12 heads x 32, F = SwiGLU hidden 1152). */
typedef struct kb_model_desc {
  int trunk_channels; /* C; multiple of 64, <= 4096 */
  int num_blocks;     /* 1..64 */
  int num_heads;      /* heads * head_dim == C */
  int head_dim;       /* 32 or 64 */
  int ffn_channels;   /* F; multiple of 64, <= 4096 */
  int precision;      /* KB_PREC_INT8 or KB_PREC_MXFP8 */
  /* KB_PROJ_* per projection, indexed by KB_PROJ_QKV .. KB_PROJ_FFN_DOWN; all
   * zero = every projection in `precision` (a zero-initialised descriptor). */
  int proj_precision[4];
  /* cudaInt8MinFfnWidth (crates/kata_nn/src/backends/int8.rs:73-83): FFN
   * projections that resolve to INT8 run in bf16 when ffn_channels is below
   * this width; 0 = no threshold; a multiple of 8, <= 8192. */
  int int8_min_ffn_width;
  /* Appended fields (all zero = the flat topology with epsilon 1e-6). */
  int topology;        /* KB_TOPO_FLAT or KB_TOPO_NESTED */
  int mid_channels;    /* nested: inner width; num_heads * head_dim == mid_channels, multiple of 32,
                          < trunk_channels */
  int pairs_per_block; /* nested: attention / FFN pairs per outer block, 1..8 */
  float norm_eps;      /* RMSNorm epsilon (RmsNormLayer::eps), 0 = 1e-6 */
} kb_model_desc;

/* Weight blob: fp32, out-first [N, K] row-major matrices, in this order:
 *   stem [C, 217]: 3x3 conv taps (ic*9 + ky*3 + kx, 22 input planes) then the
 *                  19 global-input weights;
 *   per block: rms1 [C], qkv [3C, C] ([Q; K; V]), out [C, C], rms2 [C],
 *              up [F, C], up_bias [F], down [C, F], down_bias [C],
 *              rope_freqs [heads, head_dim/2, 2] (x, y frequency per pair);
 *   trunk tip: gamma [C], beta [C];
 *   heads: p1 [96, C], g1 [96, C], g1_bias [96], v1 [192, C], v1_bias [192],
 *          gpool_to_bias [96, 288], pass1 [96, 288], pass1_bias [96], pass2 [6, 96],
 *          bias2 [96], conv2p [6, 96], v2 [192, 576], v2_bias [192], value [3, 192],
 *          value_bias [3], misc [10, 192], misc_bias [10], moremisc [8, 192],
 *          moremisc_bias [8], ownership [192].
 * KB_TOPO_NESTED (the reference's lowered TF3 graph, native_model.rs:79-165;
 * M = mid_channels, H = ffn_channels, all matrices [out, in]):
 *   stem [C, 217] as above;
 *   per outer block: pre_gate_scale [C], pre_gate_bias [C] (the block's
 *     pre_bn, applied to the raw trunk), pre_conv [M, C];
 *     per pair: rms1 [M], qkv [3M, M] ([Q; K; V]), out [M, M],
 *       rope_freqs [heads, 16, 2], rms2 [M], ffn_gate [H, M] (linear1: the
 *       SiLU branch), ffn_up [H, M] (linear_gate), ffn_down [M, H];
 *     post_gate_scale [M], post_gate_bias [M] (post_bn), post_conv [C, M];
 *   trunk tip and heads as above.
 * Same roles as the reference's LayerGraph layers (src/native_model.rs:21-165,
 * tests/debug_exec_units.rs:101-380). */
KB_API int kb_model_blob_floats(const kb_model_desc* desc, size_t* count);

typedef struct kb_model kb_model;
typedef struct kb_handle kb_handle;

/* Quantise and upload a model to `device`.
 * Replaces: CudaBackend::load_model_file + the deferred upload
 * (src/backends/cuda.rs:2618-2680, cuda_exec.rs:674-815). */
KB_API int kb_model_load(const kb_model_desc* desc, const float* blob, size_t count, int device,
                         kb_model** out);
KB_API void kb_model_destroy(kb_model* model);


/* A compute handle: one stream, a workspace for max_batch positions, two
 * pipeline slots with pinned staging.  Not thread-safe: one thread per handle.
 * Replaces: CudaBackend::create_compute_handle (src/backends/cuda.rs:2926). */
KB_API int kb_handle_create(kb_model* model, int max_batch, int inputs_nhwc, kb_handle** out);
KB_API void kb_handle_destroy(kb_handle* handle);
KB_API int kb_handle_stream(kb_handle* handle, uintptr_t* stream);

/* Run forwards for each batch size once uncaptured and once captured into a
 * CUDA graph.  Replaces: Backend::warmup_batches (backend.rs:206-410). */
KB_API int kb_warmup(kb_handle* handle, const int* batches, int count);

/* Asynchronous evaluation of n positions from host memory: spatial fp32
 * [n, 22, 19, 19] (NCHW, or [n, 19, 19, 22] if the handle is NHWC), global
 * fp32 [n, 19], symmetry int [n] in 0..7 (bit 2 transpose, bit 1 flip x,
 * bit 0 flip y; NULL = identity for every row).  Each row's symmetry is applied
 * on the device as the stem gathers its input, with the result of
 * copy_inputs_with_symmetry (crates/kata_game/src/symmetry.rs:108-224), which
 * the reference runs on the host at cuda.rs:2234-2245; outputs stay in the
 * network's frame, as the reference's raw heads do (decode_raw_outputs,
 * output_postprocess.rs:29-112, reverses them).  Returns a token.
 * Replaces: Backend::submit_output (cuda.rs:2196-2480). */
KB_API int kb_submit(kb_handle* handle, int n, const float* spatial, const float* global,
                     const int* symmetry, uint64_t* token);

/* 1 if the token's outputs are ready, 0 if not, negative KB_E_* on error.
 * Replaces: Backend::query_output_done. */
KB_API int kb_query(kb_handle* handle, uint64_t token);

/* Wait for a token and copy its raw outputs (no final activation, like the
 * reference): policy [n, 6, 362], value [n, 3], misc [n, 10], moremisc [n, 8],
 * ownership [n, 361] (any may be NULL).  status receives the sticky status word;
 * if it holds any flag the outputs are withheld and KB_E_NONFINITE returned.
 * Replaces: Backend::finish_output (cuda.rs:2510). */
KB_API int kb_finish(kb_handle* handle, uint64_t token, float* policy, float* value, float* misc,
                     float* moremisc, float* ownership, uint32_t status[2]);

/* Device-resident forward on the handle's stream (inputs and the packed
 * output [policy | value | misc | moremisc | ownership] in device memory),
 * optionally through the per-batch-size CUDA graph.
 * Replaces: CudaModel::apply (src/backends/cuda_exec.rs:913). */
KB_API int kb_forward_device(kb_handle* handle, int n, const float* d_spatial, const float* d_global,
                             float* d_out, int use_graph);

/* kb_forward_device without a graph that also copies intermediates into
 * d_trace, 16-bit [(num_blocks + 2), n*361, C]: flat topology (bf16): the stem
 * output, each block's attention output, the final residual stream; nested
 * topology (binary16): the gated stem output (block 0's pre_bn), after each
 * outer block the gated raw trunk that follows it (the next block's pre_bn,
 * or the trunk tip after the last), then the trunk tip again.  For parity
 * tests and debugging; plays the role of the reference's per-layer debug runs
 * (tests/debug_exec_units.rs). */
KB_API int kb_forward_trace(kb_handle* handle, int n, const float* d_spatial, const float* d_global,
                            float* d_out, uint16_t* d_trace);

/* Synchronise the handle's stream and read its status word [flags, first_layer].
 * Replaces: mxfp8.rs validate_completed_status (:1181). */
KB_API int kb_read_status(kb_handle* handle, uint32_t status[2]);

/* ---- Output decoding on the device -------------------------------------- */

/* One row's decoding parameters: the NNResultBuf fields that
 * decode_raw_outputs reads (crates/kata_nn/src/output_postprocess.rs:29-112)
 * and the MiscNNInputParams / board / rules facts that postprocess_output
 * reads (:140-330).  24 bytes, no padding. */
typedef struct kb_row_params {
  int32_t symmetry;          /* 0..7, the symmetry the row was evaluated under */
  float policy_optimism;     /* [0, 1] (NNResultBuf::policy_optimism as f32, :66) */
  float policy_temperature;  /* nn_policy_temperature, clamped to [1e-6, 1e6] (:150) */
  int32_t board_x, board_y;  /* board size, 1..19: ownership outside it reads 0 (:316-320) */
  uint8_t include_owner_map; /* 0: ownership not decoded (zeros) */
  uint8_t next_player_white; /* 1: white to move (:282) */
  uint8_t passing_hacks;     /* enable_passing_hacks (:170-184) */
  uint8_t no_result_off;     /* ko_rule != Simple and scoring_rule != Territory (:228-242) */
} kb_row_params;

/* ModelPostProcessParams (crates/kata_nn/src/desc.rs:671-695) and the model
 * version.  64 bytes. */
typedef struct kb_postprocess_params {
  int32_t model_version;
  float output_scale_multiplier;
  double td_score_multiplier, score_mean_multiplier, score_stdev_multiplier, lead_multiplier,
      variance_time_multiplier, shortterm_value_error_multiplier, shortterm_score_error_multiplier;
} kb_postprocess_params;

/* Decode n rows of raw heads (the packed kb_forward_device output, head-major:
 * policy [n, 6, 362] | value [n, 3] | misc [n, 10] | moremisc [n, 8] |
 * ownership [n, 361]) into d_decoded, head-major: policy [n, 362] | value
 * [n, 3] | misc [n, 4] (score_mean, score_mean_sq, lead, var_time_left) |
 * moremisc [n, 2] (shortterm_winloss_error, shortterm_score_error) | ownership
 * [n, 361].  All pointers are device memory except pp (host, NULL = the
 * reference defaults with model version 17); enqueued on `stream`.
 * d_legal NULL: decode_raw_outputs only (output_postprocess.rs:29-112: the
 * symmetry reversed, channels 0 and 5 blended by the optimism, exact).
 * d_legal [n, 362] bytes (nonzero = legal, pass last): postprocess_output
 * (:140-330) applied too, as the evaluator does per row (eval.rs:675-690).
 * Replaces: the host decode in CudaBackend::finish_output (cuda.rs:2510-2600)
 * and SharedState::postprocess_output (eval.rs:675). */
KB_API int kb_decode_device(int n, const float* d_raw, const kb_row_params* d_rows, const uint8_t* d_legal,
                            const kb_postprocess_params* pp, float* d_decoded, uintptr_t stream);

/* Post-processing parameters that kb_submit_rows applies (default: the
 * reference defaults with model version 17). */
KB_API int kb_set_postprocess(kb_handle* handle, const kb_postprocess_params* pp);

/* ---- Model files ------------------------------------------------------- */

/* Parse a native KataGo model file of the reference's TF3 family (.bin.gz,
 * .bin, .txt.gz or .txt: text tokens with "@BIN@" little-endian fp32 weight
 * arrays) into the nested topology's descriptor and weight blob: model
 * version 17, nested bottleneck blocks of attention (12 x 32 heads at mid
 * 384 in the shipped b11c768) / SwiGLU FFN pairs, SiLU, standard trunk-tip
 * BN, unit BN scales in the heads; anything else fails with the reason.  BN
 * layers are folded to scale / bias in fp32, matrices transposed to
 * out-first, head channels remapped as the reference lowers them.  blob may
 * be NULL (size query: *count receives the float count); the descriptor's
 * precision fields are INT8.  pp (nullable) receives the file's
 * post-processing multipliers and model version.
 * Replaces: model_parser.rs load_model_file / parse_model (:1002-1160) and
 * native_model.rs lower_model (:21-165). */
KB_API int kb_model_file_parse(const char* path, kb_model_desc* desc, float* blob, size_t capacity, size_t* count,
                               kb_postprocess_params* pp);

/* kb_model_file_parse then kb_model_load on `device`; the precision fields
 * (precision, proj_precision, int8_min_ffn_width) come from `recipe`
 * (NULL = every projection INT8).
 * Replaces: Backend::load_model_file (backend.rs:206-410, cuda.rs:2618-2680). */
KB_API int kb_model_load_file(const char* path, const kb_model_desc* recipe, int device, kb_model** out,
                              kb_postprocess_params* pp);

/* kb_submit with per-row decoding: each row is evaluated under rows[i].symmetry,
 * then decoded on the device as kb_decode_device does (legal NULL: decode only;
 * else host [n, 362] legality bytes and post-processing too); only the
 * decoded outputs are copied back.  Replaces: submit_output + finish_output's
 * decode (cuda.rs:2196-2600) and, with legal, postprocess_output. */
KB_API int kb_submit_rows(kb_handle* handle, int n, const float* spatial, const float* global,
                          const kb_row_params* rows, const uint8_t* legal, uint64_t* token);

/* Wait for a kb_submit_rows token and copy its decoded outputs: policy [n, 362],
 * value [n, 3], misc [n, 4], moremisc [n, 2], ownership [n, 361] (any may be
 * NULL); status as in kb_finish (outputs withheld on a status flag). */
KB_API int kb_finish_rows(kb_handle* handle, uint64_t token, float* policy, float* value, float* misc,
                          float* moremisc, float* ownership, uint32_t status[2]);

#ifdef __cplusplus
}
#endif

#endif /* KATAB200_H */
