// C ABI: kernel-level entry points of the trunk (attention), used by tests and
// by callers that sequence the trunk themselves.
#include "../../include/katab200.h"
#include "kb_internal.h"
#include "kb_ptx.cuh"

namespace kb {
int attention_launch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out,
                     int batch, int seq, int heads, int head_dim, float scale, int f16, cudaStream_t stream,
                     uint32_t* row_amax = nullptr, unsigned* status = nullptr);
}

extern "C" int kb_attention(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out,
                            int batch, int heads, int head_dim, float scale, int dtype, uintptr_t stream) {
  if (dtype != KB_DT_BF16 && dtype != KB_DT_F16) {
    kb::set_error("kb_attention: dtype must be KB_DT_BF16 or KB_DT_F16");
    return KB_E_INVALID;
  }
  return kb::attention_launch(qkv, rope_cos, rope_sin, out, batch, 361, heads, head_dim, scale,
                              dtype == KB_DT_F16, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int kb_attention_amax(const uint16_t* qkv, uint16_t* out, uint32_t* row_amax, int batch, int heads,
                                 int head_dim, float scale, int dtype, uintptr_t stream) {
  if ((dtype != KB_DT_BF16 && dtype != KB_DT_F16) || row_amax == nullptr) {
    kb::set_error("kb_attention_amax: dtype must be KB_DT_BF16 or KB_DT_F16, row_amax non-null");
    return KB_E_INVALID;
  }
  return kb::attention_launch(qkv, nullptr, nullptr, out, batch, 361, heads, head_dim, scale, dtype == KB_DT_F16,
                              reinterpret_cast<cudaStream_t>(stream), row_amax);
}

namespace {

// One CTA waits, with the given limit, on an mbarrier that nothing ever
// arrives at; the wait gives up, the kernel records KB_STATUS_TIMEOUT and
// returns.  The form every bounded wait of this library takes on a fault.
__global__ void wait_timeout_kernel(unsigned long long limit_ns, unsigned* status) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    kb::mbar_init(&bar, 1);
    abort_flag = 0;
    kb::fence_mbar_init();
  }
  __syncthreads();
  const bool ok = kb::mbar_wait(&bar, 0, &abort_flag, limit_ns);
  __syncthreads();
  if (threadIdx.x == 0 && (!ok || abort_flag)) kb::record_status(status, KB_STATUS_TIMEOUT, KB_NO_LAYER);
}

}  // namespace

extern "C" int kb_test_wait_timeout(unsigned long long limit_ns, uint32_t* status, uintptr_t stream) {
  if (!status || limit_ns == 0 || limit_ns > 1000000000ull) {
    kb::set_error("kb_test_wait_timeout: status must be non-null and the limit in 1 ns .. 1 s");
    return KB_E_INVALID;
  }
  wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns, status);
  return kb::check_cuda(cudaGetLastError(), "wait timeout kernel launch");
}
