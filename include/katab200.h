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
 * elements; for KB_EPI_RES_* it is read and written in place.  out_dtype selects
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
 * calls fail with KB_E_INVALID and say the limit.  The first call on each
 * device looks the array's address up (cudaGetSymbolAddress) and should come
 * before any stream capture.  All calls on a device share the array: calls
 * that overlap on the GPU race; nothing in it needs clearing between calls.
 * No counterpart in the reference. */
KB_API int kb_int8_ffn_gelu_rms_noalloc(uintptr_t stream, const float* gamma, float eps,
                                        const kb_int8_weight* up, const float* up_bias,
                                        const kb_int8_weight* down, const float* down_bias,
                                        uint16_t* residual, int rows);

/* ------------------------------------------------------------------ bf16 GEMM */

/* out = a[m,k] (bf16) * w[n,k]^T (bf16) with fp32 accumulation on tcgen05
 * (kind::f16) and a fused epilogue: KB_EPI_16 (bf16/fp16 out, bias, act),
 * KB_EPI_RES16 (16-bit residual add) or KB_EPI_F32 (fp32 out + bias [+ residual]).
 * Replaces: the FP16 hgemm_* linears of the outer trunk (gemm_v2.cu:397-1153). */
KB_API int kb_bf16_linear(const uint16_t* a, const uint16_t* w, const float* bias, int m, int n, int k,
                   int epilogue, int act, int out_dtype, void* out, int ldo, uintptr_t stream);

#ifdef __cplusplus
}
#endif

#endif /* KATAB200_H */
