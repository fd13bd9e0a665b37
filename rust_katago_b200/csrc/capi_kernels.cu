// C ABI: kernel-level entry points of the trunk (attention), used by tests and
// by callers that sequence the trunk themselves.
#include "../../include/katab200.h"
#include "kb_internal.h"

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
