// C ABI of the MXFP8 path: status reset, block-32 quantiser, resident weights,
// block-scaled tcgen05 GEMM and the fused projection.  Mirrors the reference's
// Mxfp8Kernels / Mxfp8Weight / Mxfp8Workspace (Rust_KataGo
// crates/kata_nn/src/backends/mxfp8.rs:101-1200) on the B200: no cuBLASLt plan,
// the GEMM is this library's kind::mxf8f6f4.block_scale kernel (gemm.cu).
#include <math.h>
#include <stdint.h>

#include <new>
#include <string>
#include <vector>

#include "../../include/katab200.h"
#include "kb_handles.h"
#include "kb_internal.h"

using namespace kb;

namespace {

int device_now() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int out_epilogue(int out_kind, int* epi, int* out_f16, int* elem) {
  switch (out_kind) {
    case KB_MX_OUT_HALF: *epi = kEpiF16, *out_f16 = 1, *elem = 2; return KB_OK;
    case KB_MX_OUT_FLOAT: *epi = kEpiF32, *out_f16 = 0, *elem = 4; return KB_OK;
    case KB_MX_OUT_FLOAT_RESIDUAL: *epi = kEpiResF32, *out_f16 = 0, *elem = 4; return KB_OK;
    case KB_MX_OUT_BF16: *epi = kEpi16, *out_f16 = 0, *elem = 2; return KB_OK;
    case KB_MX_OUT_BF16_RESIDUAL: *epi = kEpiRes16, *out_f16 = 0, *elem = 2; return KB_OK;
  }
  set_error("unknown MXFP8 output kind");
  return KB_E_INVALID;
}

}  // namespace

extern "C" {

int kb_status_reset(uint32_t* status, uintptr_t stream) {
  if (status == nullptr) {
    set_error("null status word");
    return KB_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = check_cuda(cudaMemsetAsync(status, 0, sizeof(uint32_t), s), "status reset");
  if (!rc) rc = check_cuda(cudaMemsetAsync(status + 1, 0xff, sizeof(uint32_t), s), "status reset");
  return rc;
}

int kb_mxfp8_dimensions(int rows, int k, int* kp, int* blocks4, size_t* data_bytes, size_t* scale_bytes) {
  return mxfp8_dims(rows, k, kp, blocks4, data_bytes, scale_bytes);
}

int kb_mxfp8_quantize(const void* x, int dtype, int rows, int k, int stride, uint8_t* q, uint8_t* scales,
                      size_t scale_capacity, uint32_t* status, uint32_t layer, uintptr_t stream) {
  if (layer >= 0xfffffffeu) {
    set_error("MXFP8 layer IDs 0xfffffffe/0xffffffff are reserved");
    return KB_E_INVALID;
  }
  return mxfp8_quantize_launch(x, dtype, stride, rows, k, q, scales, scale_capacity, false, status, layer,
                               reinterpret_cast<cudaStream_t>(stream));
}

int kb_mxfp8_rms_quantize(const void* x, int dtype, int rows, int width, int stride, const float* gamma,
                          float eps, int boundary_dtype, uint8_t* q, uint8_t* scales, size_t scale_capacity,
                          uint32_t* status, uint32_t layer, uintptr_t stream) {
  size_t scale_bytes = 0;
  int rc = mxfp8_dims(rows, width, nullptr, nullptr, nullptr, &scale_bytes);
  if (rc) return rc;
  if (x == nullptr || q == nullptr || scales == nullptr || scale_capacity < scale_bytes) {
    set_error("MXFP8 RMS quantiser: null buffer or scale buffer smaller than the shape needs");
    return KB_E_INVALID;
  }
  if (boundary_dtype != KB_DT_F16 && boundary_dtype != KB_DT_BF16) {
    set_error("boundary dtype must be KB_DT_F16 or KB_DT_BF16");
    return KB_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = check_cuda(cudaMemsetAsync(scales, 0, scale_capacity, s), "mxfp8 scale clear");
  if (rc) return rc;
  return rms_mxfp8_launch(x, dtype, stride, rows, width, gamma, eps, boundary_dtype == KB_DT_F16 ? 1 : 0, q, scales,
                          status, layer, s);
}

int kb_mxfp8_weight_upload(const float* w, int n, int k, int stride, kb_mxfp8_weight** out) {
  if (out == nullptr || w == nullptr) {
    set_error("null weight source or output handle");
    return KB_E_INVALID;
  }
  *out = nullptr;
  int kp = 0, blocks4 = 0;
  size_t data_bytes = 0, scale_bytes = 0;
  int rc = mxfp8_dims(n, k, &kp, &blocks4, &data_bytes, &scale_bytes);
  if (rc) return rc;
  if (stride < k) {
    set_error("MXFP8 weight stride is smaller than K");
    return KB_E_INVALID;
  }
  for (int r = 0; r < n; ++r) {
    const float* row = w + static_cast<size_t>(r) * stride;
    for (int c = 0; c < k; ++c) {
      if (!isfinite(row[c])) {
        set_error("MXFP8 original FP32 weights contain NaN or infinity in row " + std::to_string(r));
        return KB_E_NONFINITE;
      }
    }
  }
  kb_mxfp8_weight* wt = new (std::nothrow) kb_mxfp8_weight;
  if (!wt) {
    set_error("out of host memory");
    return KB_E_INVALID;
  }
  wt->device = device_now();
  wt->n = n, wt->k = k, wt->kp = kp, wt->blocks4 = blocks4, wt->scale_bytes = scale_bytes;
  const size_t src_floats = static_cast<size_t>(n - 1) * stride + k;
  float* d_src = nullptr;
  uint32_t* d_status = nullptr;
  cudaStream_t s = nullptr;
  rc = check_cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "upload stream");
  if (!rc) rc = check_cuda(cudaMalloc(&wt->q, data_bytes), "cudaMalloc(mxfp8 weight)");
  if (!rc) rc = check_cuda(cudaMalloc(&wt->scales, scale_bytes), "cudaMalloc(mxfp8 weight scales)");
  if (!rc) rc = check_cuda(cudaMalloc(&d_src, src_floats * sizeof(float)), "cudaMalloc(weight staging)");
  if (!rc) rc = check_cuda(cudaMalloc(&d_status, 2 * sizeof(uint32_t)), "cudaMalloc(status)");
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(d_src, w, src_floats * sizeof(float), cudaMemcpyHostToDevice, s),
                    "upload weight");
  if (!rc) rc = kb_status_reset(d_status, reinterpret_cast<uintptr_t>(s));
  if (!rc)
    rc = mxfp8_quantize_launch(d_src, KB_DT_F32, stride, n, k, wt->q, wt->scales, scale_bytes, true, d_status, 0,
                               s);
  uint32_t st[2] = {0, 0};
  if (!rc) rc = check_cuda(cudaMemcpyAsync(st, d_status, sizeof(st), cudaMemcpyDeviceToHost, s), "status");
  if (!rc) rc = check_cuda(cudaStreamSynchronize(s), "MXFP8 static weight upload");
  if (!rc && (st[0] != 0 || st[1] != 0xffffffffu)) {
    set_error("MXFP8 weight rejected: flags=" + std::to_string(st[0]) +
              " (NaN=1 infinity=2 weight_overflow=8): an element decodes beyond fp32");
    rc = KB_E_NONFINITE;
  }
  if (d_src) cudaFree(d_src);
  if (d_status) cudaFree(d_status);
  if (s) cudaStreamDestroy(s);
  if (rc) {
    kb_mxfp8_weight_destroy(wt);
    return rc;
  }
  *out = wt;
  return KB_OK;
}

int kb_mxfp8_weight_info(const kb_mxfp8_weight* w, int* n, int* k, int* kp, const uint8_t** q,
                         const uint8_t** scales, size_t* scale_bytes) {
  if (w == nullptr) {
    set_error("null weight");
    return KB_E_INVALID;
  }
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (kp) *kp = w->kp;
  if (q) *q = w->q;
  if (scales) *scales = w->scales;
  if (scale_bytes) *scale_bytes = w->scale_bytes;
  return KB_OK;
}

void kb_mxfp8_weight_destroy(kb_mxfp8_weight* w) {
  if (!w) return;
  if (w->q) cudaFree(w->q);
  if (w->scales) cudaFree(w->scales);
  delete w;
}

int kb_mxfp8_gemm(const uint8_t* a_q, const uint8_t* a_scales, int rows, const kb_mxfp8_weight* w,
                  const float* bias, int act, int out_kind, void* out, long ldo, uint32_t* status, uint32_t layer,
                  uintptr_t stream) {
  if (w == nullptr || a_q == nullptr || a_scales == nullptr || out == nullptr) {
    set_error("null MXFP8 GEMM argument");
    return KB_E_INVALID;
  }
  if (w->device != device_now()) {
    set_error("MXFP8 weight belongs to another device");
    return KB_E_STATE;
  }
  int rc = mxfp8_dims(rows, w->k, nullptr, nullptr, nullptr, nullptr);
  if (rc) return rc;
  int epi = 0, out_f16 = 0, elem = 0;
  rc = out_epilogue(out_kind, &epi, &out_f16, &elem);
  if (rc) return rc;
  if (ldo < w->n || (reinterpret_cast<uintptr_t>(out) & 15)) {
    set_error("MXFP8 output must be 16-byte aligned with a row stride of at least N");
    return KB_E_INVALID;
  }
  if ((out_kind != KB_MX_OUT_BF16 && bias != nullptr && out_kind != KB_MX_OUT_BF16_RESIDUAL) ||
      (out_kind != KB_MX_OUT_BF16 && act != KB_ACT_NONE)) {
    set_error("bias applies to the bf16 outputs only, the activation to KB_MX_OUT_BF16 only");
    return KB_E_INVALID;
  }
  GemmArgs g;
  g.m = rows;
  g.n = w->n;
  g.k = w->kp;
  g.out = out;
  g.ldo = ldo;
  g.bias = bias;
  g.act = act;
  g.out_f16 = out_f16;
  g.status = status;
  g.layer = layer;
  g.sfa = a_scales;
  g.sfb = w->scales;
  return gemm_launch(kGemmMXF8, epi, a_q, w->q, g, reinterpret_cast<cudaStream_t>(stream));
}

int kb_mxfp8_project(const kb_mxfp8_weight* w, const void* x, int dtype, int rows, int stride, uint8_t* q_scratch,
                     uint8_t* scale_scratch, size_t scale_capacity, int out_kind, void* out, long ldo,
                     uint32_t* status, uint32_t layer, uintptr_t stream) {
  if (w == nullptr) {
    set_error("null weight");
    return KB_E_INVALID;
  }
  if (dtype != KB_DT_F16 && dtype != KB_DT_BF16) {
    set_error("MXFP8 projections take 16-bit activations (the reference's half boundary)");
    return KB_E_INVALID;
  }
  int rc = kb_mxfp8_quantize(x, dtype, rows, w->k, stride, q_scratch, scale_scratch, scale_capacity, status, layer,
                             stream);
  if (rc) return rc;
  return kb_mxfp8_gemm(q_scratch, scale_scratch, rows, w, nullptr, KB_ACT_NONE, out_kind, out, ldo, status, layer,
                       stream);
}

}  // extern "C"
