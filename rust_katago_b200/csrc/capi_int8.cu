// C ABI: INT8 weights, INT8 kernels, the INT8 workspace (the reference's
// Int8Workspace API, crates/kata_nn/src/backends/int8.rs:830-1259) and the
// bf16 linear.  Every entry point validates on the host and fails closed.
#include <math.h>
#include <string.h>

#include <cfloat>
#include <new>
#include <string>
#include <vector>

#include "../../include/katab200.h"
#include "kb_handles.h"
#include "kb_internal.h"

namespace kb {
int quantize_rows_launch(const void* x, int dtype, long ldx, int rows, int width, int kp, bool rms,
                         const float* gamma, float eps, int bound_f16, int8_t* q, float* scales,
                         unsigned* status, unsigned layer, cudaStream_t stream);
}

using namespace kb;

struct kb_int8_workspace {
  int device = 0;
  cudaStream_t stream = nullptr;
  int rows = 0, max_k = 0, max_n = 0;
  int8_t* q = nullptr;
  float* scales = nullptr;
  uint16_t* hidden = nullptr;
};

namespace {

constexpr int kSwigluHalfTile = 128;  // gate (or up) channels per 256-column GEMM tile

int padded16(int k) { return (k + 15) / 16 * 16; }

bool stream_ok(const kb_int8_workspace* ws, uintptr_t stream) {
  return ws != nullptr && reinterpret_cast<cudaStream_t>(stream) == ws->stream;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

extern "C" {

const char* kb_last_error(void) { return kb::last_error(); }

int kb_version(void) { return 100; }

int kb_device_check(int device) {
  cudaDeviceProp p;
  int rc = check_cuda(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
  if (rc) return rc;
  if (p.major != 10 || p.minor != 0) {
    set_error("device " + std::to_string(device) + " is sm_" + std::to_string(p.major) +
              std::to_string(p.minor) + "; this library is built for sm_100a only");
    return KB_E_UNSUPPORTED;
  }
  return KB_OK;
}

int kb_int8_quantize_weights(const float* w, int n, int k, int8_t* q, float* scales) {
  if (w == nullptr || q == nullptr || scales == nullptr || n <= 0 || k <= 0 || k > 8192 ||
      n % 4 != 0) {
    set_error("invalid INT8 weight shape N=" + std::to_string(n) + " K=" + std::to_string(k));
    return KB_E_INVALID;
  }
  const size_t total = static_cast<size_t>(n) * k;
  for (size_t i = 0; i < total; ++i) {
    if (!std::isfinite(w[i])) {
      set_error("INT8 weights contain NaN or infinity");
      return KB_E_INVALID;
    }
  }
  const int kp = padded16(k);
  for (int r = 0; r < n; ++r) {
    const float* row = w + static_cast<size_t>(r) * k;
    float amax = 0.0f;
    for (int c = 0; c < k; ++c) amax = fmaxf(amax, fabsf(row[c]));
    float s = 1.0f;
    if (amax != 0.0f) {
      s = amax / 127.0f;
      if (s < FLT_MIN) s = FLT_MIN;
    }
    scales[r] = s;
    int8_t* qr = q + static_cast<size_t>(r) * kp;
    for (int c = 0; c < kp; ++c) {
      if (c < k) {
        float v = nearbyintf(row[c] / s);
        v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
        qr[c] = static_cast<int8_t>(v);
      } else {
        qr[c] = 0;
      }
    }
  }
  return KB_OK;
}

int kb_int8_weight_upload(const float* w, int n, int k, int layout, kb_int8_weight** out) {
  if (out == nullptr) {
    set_error("null output handle");
    return KB_E_INVALID;
  }
  *out = nullptr;
  if (layout != KB_LAYOUT_PLAIN && layout != KB_LAYOUT_SWIGLU_DUAL) {
    set_error("unknown INT8 weight layout");
    return KB_E_INVALID;
  }
  if (layout == KB_LAYOUT_SWIGLU_DUAL && (n % 2 != 0)) {
    set_error("SwiGLU dual weight needs an even row count [gate; up]");
    return KB_E_INVALID;
  }
  const int kp = padded16(k > 0 ? k : 1);
  std::vector<int8_t> q(static_cast<size_t>(n > 0 ? n : 0) * kp);
  std::vector<float> s(n > 0 ? n : 0);
  int rc = kb_int8_quantize_weights(w, n, k, q.data(), s.data());
  if (rc) return rc;
  int n_stored = n;
  std::vector<int8_t> qs;
  std::vector<float> ss;
  if (layout == KB_LAYOUT_SWIGLU_DUAL) {
    // Tile t of the 256-column dual GEMM holds gate channels [128t, 128t+128)
    // followed by the matching up channels; padding rows are zero, scale 1.
    const int h = n / 2;
    const int tiles = (h + kSwigluHalfTile - 1) / kSwigluHalfTile;
    n_stored = tiles * 2 * kSwigluHalfTile;
    qs.assign(static_cast<size_t>(n_stored) * kp, 0);
    ss.assign(n_stored, 1.0f);
    for (int t = 0; t < tiles; ++t) {
      for (int i = 0; i < kSwigluHalfTile; ++i) {
        const int ch = t * kSwigluHalfTile + i;
        if (ch >= h) break;
        const int gdst = t * 2 * kSwigluHalfTile + i;
        const int udst = gdst + kSwigluHalfTile;
        memcpy(&qs[static_cast<size_t>(gdst) * kp], &q[static_cast<size_t>(ch) * kp], kp);
        memcpy(&qs[static_cast<size_t>(udst) * kp], &q[static_cast<size_t>(h + ch) * kp], kp);
        ss[gdst] = s[ch];
        ss[udst] = s[h + ch];
      }
    }
  } else {
    qs.swap(q);
    ss.swap(s);
  }
  kb_int8_weight* wt = new (std::nothrow) kb_int8_weight;
  if (!wt) {
    set_error("out of host memory");
    return KB_E_INVALID;
  }
  wt->device = current_device();
  wt->n = n;
  wt->k = k;
  wt->kp = kp;
  wt->n_stored = n_stored;
  wt->layout = layout;
  rc = check_cuda(cudaMalloc(&wt->q, qs.size()), "cudaMalloc(int8 weight)");
  if (!rc) rc = check_cuda(cudaMalloc(&wt->scales, ss.size() * sizeof(float)), "cudaMalloc(weight scales)");
  if (!rc) rc = check_cuda(cudaMemcpy(wt->q, qs.data(), qs.size(), cudaMemcpyHostToDevice), "upload weight");
  if (!rc)
    rc = check_cuda(cudaMemcpy(wt->scales, ss.data(), ss.size() * sizeof(float), cudaMemcpyHostToDevice),
                    "upload weight scales");
  if (rc) {
    kb_int8_weight_destroy(wt);
    return rc;
  }
  *out = wt;
  return KB_OK;
}

int kb_int8_weight_info(const kb_int8_weight* w, int* n, int* k, int* kp, int* n_stored,
                        const int8_t** q, const float** scales) {
  if (w == nullptr) {
    set_error("null weight");
    return KB_E_INVALID;
  }
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (kp) *kp = w->kp;
  if (n_stored) *n_stored = w->n_stored;
  if (q) *q = w->q;
  if (scales) *scales = w->scales;
  return KB_OK;
}

void kb_int8_weight_destroy(kb_int8_weight* w) {
  if (!w) return;
  if (w->q) cudaFree(w->q);
  if (w->scales) cudaFree(w->scales);
  delete w;
}

int kb_int8_gemm_i32(const int8_t* a, const int8_t* w, int32_t* dots, int m, int n, int kp,
                     uintptr_t stream) {
  if (!a || !w || !dots || m <= 0 || n <= 0 || kp <= 0 || kp % 16 != 0) {
    set_error("kb_int8_gemm_i32: invalid arguments (kp must be a positive multiple of 16)");
    return KB_E_INVALID;
  }
  GemmArgs g;
  g.m = m;
  g.n = n;
  g.k = kp;
  g.out = dots;
  g.ldo = n;
  return gemm_launch(kGemmI8, kEpiI32, a, w, g, reinterpret_cast<cudaStream_t>(stream));
}

int kb_test_int8_gemm_i32_wait_limit(const int8_t* a, const int8_t* w, int32_t* dots, int m, int n, int kp,
                                     unsigned long long wait_limit_ns, uint32_t* status, uintptr_t stream) {
  if (!a || !w || !dots || !status || m <= 0 || n <= 0 || kp <= 0 || kp % 16 != 0 || wait_limit_ns == 0 ||
      wait_limit_ns > 2000000000ull) {
    set_error("kb_test_int8_gemm_i32_wait_limit: invalid arguments");
    return KB_E_INVALID;
  }
  GemmArgs g;
  g.m = m;
  g.n = n;
  g.k = kp;
  g.out = dots;
  g.ldo = n;
  g.status = status;
  g.wait_limit_ns = wait_limit_ns;
  return gemm_launch(kGemmI8, kEpiI32, a, w, g, reinterpret_cast<cudaStream_t>(stream));
}

int kb_int8_linear(const int8_t* a, const float* sa, const int8_t* w, const float* sw,
                   const float* bias, int m, int n, int kp, int epilogue, int act, int out_dtype,
                   void* out, int ldo, int n_out, uint32_t* row_amax, uintptr_t stream) {
  if (!a || !w || !out || m <= 0 || n <= 0 || kp <= 0 || kp % 16 != 0 || epilogue < 0 ||
      epilogue > KB_EPI_F32 || act < 0 || act > KB_ACT_SILU) {
    set_error("kb_int8_linear: invalid arguments");
    return KB_E_INVALID;
  }
  if (epilogue != KB_EPI_I32 && (!sa || !sw)) {
    set_error("kb_int8_linear: dequant epilogues need activation and weight scales");
    return KB_E_INVALID;
  }
  const int width = epilogue == KB_EPI_SWIGLU16 ? n_out : n;
  if (ldo < width || (epilogue == KB_EPI_SWIGLU16 && (n_out <= 0 || n % 256 != 0 || n_out * 2 > n))) {
    set_error("kb_int8_linear: output stride / SwiGLU width mismatch");
    return KB_E_INVALID;
  }
  GemmArgs g;
  g.m = m;
  g.n = n;
  g.k = kp;
  g.out = out;
  g.ldo = ldo;
  g.row_scale = sa;
  g.col_scale = sw;
  g.bias = bias;
  g.act = act;
  g.out_f16 = out_dtype == KB_DT_F16;
  g.n_out = n_out;
  g.row_amax = row_amax;
  return gemm_launch(kGemmI8, epilogue, a, w, g, reinterpret_cast<cudaStream_t>(stream));
}

int kb_int8_quantize_rows(const void* x, int dtype, int rows, int width, int stride, int kp,
                          int8_t* q, float* scales, uintptr_t stream) {
  if (!x || !q || !scales) {
    set_error("kb_int8_quantize_rows: null pointer");
    return KB_E_INVALID;
  }
  return quantize_rows_launch(x, dtype, stride, rows, width, kp, false, nullptr, 0.0f, 0, q, scales,
                              nullptr, KB_NO_LAYER, reinterpret_cast<cudaStream_t>(stream));
}

int kb_int8_quantize_rows_amax(const void* x, int dtype, int rows, int width, int stride, int kp,
                               const uint32_t* row_amax, int8_t* q, float* scales, uintptr_t stream) {
  if (!x || !q || !scales || !row_amax) {
    set_error("kb_int8_quantize_rows_amax: null pointer");
    return KB_E_INVALID;
  }
  return quantize_rows_amax_launch(x, dtype, stride, row_amax, rows, width, kp, q, scales, nullptr, KB_NO_LAYER,
                                   reinterpret_cast<cudaStream_t>(stream));
}

int kb_int8_rms_quantize(const void* x, int dtype, int rows, int width, int stride,
                         const float* gamma, float eps, int boundary_dtype, int kp, int8_t* q,
                         float* scales, uintptr_t stream) {
  if (!x || !q || !scales || (boundary_dtype != KB_DT_F16 && boundary_dtype != KB_DT_BF16)) {
    set_error("kb_int8_rms_quantize: invalid arguments");
    return KB_E_INVALID;
  }
  return quantize_rows_launch(x, dtype, stride, rows, width, kp, true, gamma, eps,
                              boundary_dtype == KB_DT_F16, q, scales, nullptr, KB_NO_LAYER,
                              reinterpret_cast<cudaStream_t>(stream));
}

int kb_int8_workspace_create(uintptr_t stream, int rows, int max_k, int max_n,
                             kb_int8_workspace** out) {
  if (!out || rows <= 0 || max_k <= 0 || max_n <= 0) {
    set_error("kb_int8_workspace_create: invalid arguments");
    return KB_E_INVALID;
  }
  *out = nullptr;
  kb_int8_workspace* ws = new (std::nothrow) kb_int8_workspace;
  if (!ws) {
    set_error("out of host memory");
    return KB_E_INVALID;
  }
  ws->device = current_device();
  ws->stream = reinterpret_cast<cudaStream_t>(stream);
  ws->rows = rows;
  ws->max_k = padded16(max_k);
  ws->max_n = max_n;
  int rc = check_cuda(cudaMalloc(&ws->q, static_cast<size_t>(rows) * ws->max_k), "cudaMalloc(ws q)");
  if (!rc) rc = check_cuda(cudaMalloc(&ws->scales, static_cast<size_t>(rows) * sizeof(float)), "cudaMalloc(ws scales)");
  if (!rc)
    rc = check_cuda(cudaMalloc(&ws->hidden, static_cast<size_t>(rows) * max_n * sizeof(uint16_t)),
                    "cudaMalloc(ws hidden)");
  if (rc) {
    kb_int8_workspace_destroy(ws);
    return rc;
  }
  *out = ws;
  return KB_OK;
}

void kb_int8_workspace_destroy(kb_int8_workspace* ws) {
  if (!ws) return;
  if (ws->q) cudaFree(ws->q);
  if (ws->scales) cudaFree(ws->scales);
  if (ws->hidden) cudaFree(ws->hidden);
  delete ws;
}

int kb_int8_workspace_buffers(kb_int8_workspace* ws, int8_t** quantized, float** scales,
                              void** hidden) {
  if (!ws) {
    set_error("null workspace");
    return KB_E_INVALID;
  }
  if (quantized) *quantized = ws->q;
  if (scales) *scales = ws->scales;
  if (hidden) *hidden = ws->hidden;
  return KB_OK;
}

static int validate_ws(kb_int8_workspace* ws, uintptr_t stream, int rows) {
  if (!ws) {
    set_error("null workspace");
    return KB_E_INVALID;
  }
  if (!stream_ok(ws, stream)) {
    set_error("INT8 workspace belongs to another CUDA stream");
    return KB_E_STATE;
  }
  if (rows <= 0 || rows > ws->rows) {
    set_error("INT8 rows must be in 1..workspace rows");
    return KB_E_INVALID;
  }
  if (current_device() != ws->device) {
    set_error("INT8 workspace belongs to another device");
    return KB_E_STATE;
  }
  return KB_OK;
}

static int project(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input, int stride,
                   const kb_int8_weight* w, void* output, int rows, int epi) {
  int rc = validate_ws(ws, stream, rows);
  if (rc) return rc;
  if (!input || !w || !output || stride < w->k || w->kp > ws->max_k ||
      w->layout != KB_LAYOUT_PLAIN) {
    set_error("INT8 projection buffer/stride mismatch");
    return KB_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = quantize_rows_launch(input, KB_DT_F16, stride, rows, w->k, w->kp, false, nullptr, 0.0f, 0,
                            ws->q, ws->scales, nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  GemmArgs g;
  g.m = rows;
  g.n = w->n;
  g.k = w->kp;
  g.out = output;
  g.ldo = w->n;
  g.row_scale = ws->scales;
  g.col_scale = w->scales;
  return gemm_launch(kGemmI8, epi, ws->q, w->q, g, s);
}

int kb_int8_project_half(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input,
                         int stride, const kb_int8_weight* w, uint16_t* output, int rows) {
  return project(ws, stream, input, stride, w, output, rows, kEpiF16);
}

int kb_int8_project_residual(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input,
                             int stride, const kb_int8_weight* w, float* residual, int rows) {
  return project(ws, stream, input, stride, w, residual, rows, kEpiResF32);
}

static int validate_ffn(kb_int8_workspace* ws, const kb_int8_weight* dual,
                        const kb_int8_weight* down, const void* out) {
  if (!dual || !down || !out || dual->layout != KB_LAYOUT_SWIGLU_DUAL ||
      down->layout != KB_LAYOUT_PLAIN || dual->n != 2 * down->k || dual->k != down->n ||
      dual->kp > ws->max_k || down->kp > ws->max_k || down->k > ws->max_n) {
    set_error("INT8 FFN shape/buffer mismatch");
    return KB_E_INVALID;
  }
  return KB_OK;
}

// dual GEMM + SwiGLU (fp16 boundaries) -> requant -> down GEMM + fp32 residual.
static int finish_ffn(kb_int8_workspace* ws, cudaStream_t s, const kb_int8_weight* dual,
                      const kb_int8_weight* down, float* output, int rows) {
  const int hidden = down->k;
  GemmArgs g;
  g.m = rows;
  g.n = dual->n_stored;
  g.k = dual->kp;
  g.out = ws->hidden;
  g.ldo = hidden;
  g.row_scale = ws->scales;
  g.col_scale = dual->scales;
  g.out_f16 = 1;
  g.n_out = hidden;
  int rc = gemm_launch(kGemmI8, kEpiSwiGLU16, ws->q, dual->q, g, s, 256);
  if (rc) return rc;
  rc = quantize_rows_launch(ws->hidden, KB_DT_F16, hidden, rows, hidden, down->kp, false, nullptr,
                            0.0f, 0, ws->q, ws->scales, nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  GemmArgs d;
  d.m = rows;
  d.n = down->n;
  d.k = down->kp;
  d.out = output;
  d.ldo = down->n;
  d.row_scale = ws->scales;
  d.col_scale = down->scales;
  return gemm_launch(kGemmI8, kEpiResF32, ws->q, down->q, d, s);
}

int kb_int8_ffn(kb_int8_workspace* ws, uintptr_t stream, const uint16_t* input,
                const kb_int8_weight* dual, const kb_int8_weight* down, float* output, int rows) {
  int rc = validate_ws(ws, stream, rows);
  if (rc) return rc;
  rc = validate_ffn(ws, dual, down, output);
  if (rc) return rc;
  if (!input) {
    set_error("null FFN input");
    return KB_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = quantize_rows_launch(input, KB_DT_F16, dual->k, rows, dual->k, dual->kp, false, nullptr, 0.0f,
                            0, ws->q, ws->scales, nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  return finish_ffn(ws, s, dual, down, output, rows);
}

int kb_int8_ffn_rms(kb_int8_workspace* ws, uintptr_t stream, const float* gamma, float eps,
                    const kb_int8_weight* dual, const kb_int8_weight* down, float* residual,
                    int rows) {
  int rc = validate_ws(ws, stream, rows);
  if (rc) return rc;
  rc = validate_ffn(ws, dual, down, residual);
  if (rc) return rc;
  if (!gamma || !(eps > 0.0f) || !std::isfinite(eps)) {
    set_error("INT8 RMS shape/epsilon mismatch");
    return KB_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = quantize_rows_launch(residual, KB_DT_F32, dual->k, rows, dual->k, dual->kp, true, gamma, eps,
                            1, ws->q, ws->scales, nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  return finish_ffn(ws, s, dual, down, residual, rows);
}

int kb_int8_ffn_gelu_rms(kb_int8_workspace* ws, uintptr_t stream, const float* gamma, float eps,
                         const kb_int8_weight* up, const float* up_bias,
                         const kb_int8_weight* down, const float* down_bias, uint16_t* residual,
                         int rows) {
  int rc = validate_ws(ws, stream, rows);
  if (rc) return rc;
  if (!up || !down || !residual || up->layout != KB_LAYOUT_PLAIN || down->layout != KB_LAYOUT_PLAIN ||
      up->n != down->k || up->k != down->n || up->kp > ws->max_k || down->kp > ws->max_k ||
      up->n > ws->max_n) {
    set_error("INT8 GELU FFN shape/buffer mismatch");
    return KB_E_INVALID;
  }
  if (!gamma || !(eps > 0.0f) || !std::isfinite(eps)) {
    set_error("INT8 RMS shape/epsilon mismatch");
    return KB_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int c = up->k, f = up->n;
  rc = quantize_rows_launch(residual, KB_DT_BF16, c, rows, c, up->kp, true, gamma, eps, 0, ws->q,
                            ws->scales, nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  GemmArgs g;
  g.m = rows;
  g.n = f;
  g.k = up->kp;
  g.out = ws->hidden;
  g.ldo = f;
  g.row_scale = ws->scales;
  g.col_scale = up->scales;
  g.bias = up_bias;
  g.act = 1;
  g.out_f16 = 0;
  rc = gemm_launch(kGemmI8, kEpi16, ws->q, up->q, g, s);
  if (rc) return rc;
  rc = quantize_rows_launch(ws->hidden, KB_DT_BF16, f, rows, f, down->kp, false, nullptr, 0.0f, 0,
                            ws->q, ws->scales, nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  GemmArgs d;
  d.m = rows;
  d.n = c;
  d.k = down->kp;
  d.out = residual;
  d.ldo = c;
  d.row_scale = ws->scales;
  d.col_scale = down->scales;
  d.bias = down_bias;
  d.out_f16 = 0;
  return gemm_launch(kGemmI8, kEpiRes16, ws->q, down->q, d, s);
}

int kb_bf16_linear(const uint16_t* a, const uint16_t* w, const float* bias, int m, int n, int k,
                   int epilogue, int act, int out_dtype, void* out, int ldo, uintptr_t stream) {
  if (!a || !w || !out || m <= 0 || n <= 0 || k <= 0 || k % 8 != 0 || ldo < n ||
      (epilogue != KB_EPI_16 && epilogue != KB_EPI_RES16 && epilogue != KB_EPI_F32) || act < 0 ||
      act > KB_ACT_SILU) {
    set_error("kb_bf16_linear: invalid arguments (k must be a multiple of 8)");
    return KB_E_INVALID;
  }
  GemmArgs g;
  g.m = m;
  g.n = n;
  g.k = k;
  g.out = out;
  g.ldo = ldo;
  g.bias = bias;
  g.act = act;
  g.out_f16 = out_dtype == KB_DT_F16;
  return gemm_launch(kGemmBF16, epilogue, a, w, g, reinterpret_cast<cudaStream_t>(stream));
}

int kb_f16_linear(const uint16_t* a, const uint16_t* w, const float* bias, int m, int n, int k, int epilogue,
                  int act, int out_dtype, void* out, int ldo, uintptr_t stream) {
  if (!a || !w || !out || m <= 0 || n <= 0 || k <= 0 || k % 8 != 0 || ldo < n ||
      (epilogue != KB_EPI_16 && epilogue != KB_EPI_RES16 && epilogue != KB_EPI_F32) || act < 0 ||
      act > KB_ACT_SILU) {
    set_error("kb_f16_linear: invalid arguments (k must be a multiple of 8)");
    return KB_E_INVALID;
  }
  GemmArgs g;
  g.m = m;
  g.n = n;
  g.k = k;
  g.out = out;
  g.ldo = ldo;
  g.bias = bias;
  g.act = act;
  g.out_f16 = out_dtype == KB_DT_F16;
  g.ab_f16 = 1;
  return gemm_launch(kGemmBF16, epilogue, a, w, g, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
