// kb_int8_ffn_gelu_rms_noalloc: the GELU FFN block of kb_int8_ffn_gelu_rms
// with its scratch (16-bit hidden activations, INT8 activations, per-token
// scales) in one fixed, statically reserved device array instead of a
// caller-created workspace, so the call itself allocates nothing.
//
// Who needs it: callers that cannot call cudaMalloc at the point where they
// evaluate, e.g. a search thread that evaluates a handful of positions in the
// middle of a move (cudaMalloc can synchronise the device and stall every
// other stream), or an embedding host that owns all device memory under a
// fixed budget and forbids allocations by plugins.
//
// Limits and rules (also in include/katab200.h):
//   * the array is kNoAllocScratchBytes (8 MiB) on every device that loads the
//     library, held until process exit; calls that need more are rejected;
//   * its device address is looked up with cudaGetSymbolAddress once per
//     device, on the first call made with that device current (or by
//     kb_int8_noalloc_prepare): make that first call before any stream capture
//     begins.  The address is kept per device together with the CUDA context it
//     belongs to; after a device reset the new context triggers a new lookup;
//   * every call on a device shares the one array and it keeps the previous
//     call's contents: nothing in it needs to start at zero (every byte the
//     block reads is written earlier in the same call), and calls that overlap
//     on the GPU (different streams, or different host threads) race on it.
#include <math.h>

#include <mutex>
#include <string>

#include "../../include/katab200.h"
#include "kb_handles.h"
#include "kb_internal.h"
#include "kb_numeric.cuh"

namespace kb {
int quantize_rows_launch(const void* x, int dtype, long ldx, int rows, int width, int kp, bool rms,
                         const float* gamma, float eps, int bound_f16, int8_t* q, float* scales,
                         unsigned* status, unsigned layer, cudaStream_t stream);
}

using namespace kb;

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
// Per device: the CUDA context the address was looked up in, and the address.
// A device reset (cudaDeviceReset) gives the device a new primary context, in
// which the array lives at a new address: the lookup is then repeated.
struct ScratchSlot {
  CUcontext ctx = nullptr;
  void* ptr = nullptr;
};
ScratchSlot g_scratch[kMaxDevices];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of the current device's scratch array; looked up once per
// device (and again only if the device's context has changed).
int scratch_address(void** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device index out of range for the no-alloc scratch table");
    return KB_E_INVALID;
  }
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr) {
    set_error("no-alloc scratch: cuCtxGetCurrent is not available");
    return KB_E_CUDA;
  }
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  if (slot.ptr == nullptr || ctx == nullptr || slot.ctx != ctx) {
    // The lookup binds the device's primary context to this thread if none is
    // current yet; the context is read again afterwards.
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)");
    if (rc) return rc;
    if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    slot.ctx = ctx;
    slot.ptr = p;
  }
  *out = slot.ptr;
  return KB_OK;
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

}  // namespace

extern "C" int kb_int8_ffn_gelu_rms_noalloc(uintptr_t stream, const float* gamma, float eps,
                                            const kb_int8_weight* up, const float* up_bias,
                                            const kb_int8_weight* down, const float* down_bias,
                                            uint16_t* residual, int rows) {
  if (!up || !down || !residual || up->layout != KB_LAYOUT_PLAIN || down->layout != KB_LAYOUT_PLAIN ||
      up->n != down->k || up->k != down->n) {
    set_error("INT8 GELU FFN shape/buffer mismatch");
    return KB_E_INVALID;
  }
  if (!gamma || !(eps > 0.0f) || !std::isfinite(eps)) {
    set_error("INT8 RMS shape/epsilon mismatch");
    return KB_E_INVALID;
  }
  if (rows <= 0) {
    set_error("INT8 rows must be positive");
    return KB_E_INVALID;
  }
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (up->device != dev || down->device != dev) {
    set_error("INT8 weight belongs to another device");
    return KB_E_STATE;
  }
  const int c = up->k, f = up->n;
  const int kq = up->kp > down->kp ? up->kp : down->kp;
  // Layout: hidden 16-bit [rows, f] | int8 [rows, kq] | scales f32 [rows].
  const size_t per_row = 2 * static_cast<size_t>(f) + kq + 4;
  const size_t need = align256(2 * static_cast<size_t>(rows) * f) + align256(static_cast<size_t>(rows) * kq) +
                      align256(4 * static_cast<size_t>(rows));
  if (need > kNoAllocScratchBytes) {
    const size_t max_rows = (kNoAllocScratchBytes - 3 * 256) / per_row;
    set_error("no-alloc FFN: " + std::to_string(rows) + " rows need " + std::to_string(need) +
              " bytes of scratch; the fixed scratch is " + std::to_string(kNoAllocScratchBytes) +
              " bytes (at most " + std::to_string(max_rows) + " rows for this shape)");
    return KB_E_INVALID;
  }
  void* base = nullptr;
  rc = scratch_address(&base);
  if (rc) return rc;
  uint8_t* p = static_cast<uint8_t*>(base);
  uint16_t* hidden = reinterpret_cast<uint16_t*>(p);
  int8_t* q = reinterpret_cast<int8_t*>(p + align256(2 * static_cast<size_t>(rows) * f));
  float* scales = reinterpret_cast<float*>(p + align256(2 * static_cast<size_t>(rows) * f) +
                                           align256(static_cast<size_t>(rows) * kq));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = quantize_rows_launch(residual, KB_DT_BF16, c, rows, c, up->kp, true, gamma, eps, 0, q, scales,
                            nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  GemmArgs g;
  g.m = rows;
  g.n = f;
  g.k = up->kp;
  g.out = hidden;
  g.ldo = f;
  g.row_scale = scales;
  g.col_scale = up->scales;
  g.bias = up_bias;
  g.act = kActGelu;
  g.out_f16 = 0;
  rc = gemm_launch(kGemmI8, kEpi16, q, up->q, g, s);
  if (rc) return rc;
  rc = quantize_rows_launch(hidden, KB_DT_BF16, f, rows, f, down->kp, false, nullptr, 0.0f, 0, q, scales,
                            nullptr, KB_NO_LAYER, s);
  if (rc) return rc;
  GemmArgs d;
  d.m = rows;
  d.n = c;
  d.k = down->kp;
  d.out = residual;
  d.ldo = c;
  d.row_scale = scales;
  d.col_scale = down->scales;
  d.bias = down_bias;
  d.out_f16 = 0;
  return gemm_launch(kGemmI8, kEpiRes16, q, down->q, d, s);
}

extern "C" int kb_int8_noalloc_prepare(void) {
  void* base = nullptr;
  return scratch_address(&base);
}
