// Host runtime pieces shared by every entry point: thread-local error text,
// CUDA error mapping and cached device properties.
#include <mutex>
#include <string>
#include <vector>

#include "kb_internal.h"

namespace kb {

namespace {
thread_local std::string g_error;
}

void set_error(const std::string& msg) { g_error = msg; }
const char* last_error() { return g_error.c_str(); }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KB_OK;
  set_error(std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
  return KB_E_CUDA;
}

int num_sms(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0) device = 0;
  if (static_cast<int>(cache.size()) <= device) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    cache[device] = v;
  }
  return cache[device];
}

}  // namespace kb
