// common.cu — library-wide state: the device error word that bounded waits
// write on timeout, and version / error introspection entry points.
#include <atomic>

#include <cuda_runtime.h>

#include "host_common.h"

namespace nl {

// One word per device context: 0 = ok, otherwise the first error code.
__device__ int g_device_error;

int* device_error_word() {
  constexpr int kMaxDev = 64;
  static int* cached[kMaxDev] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

}  // namespace nl

extern "C" long long nl_launch_count(void) { return nl::g_launches.load(std::memory_order_relaxed); }

extern "C" const char* nl_version(void) { return "nlearn-b200 0.1 (sm_100a)"; }

extern "C" int nl_get_device_error(cudaStream_t stream) {
  int* w = nl::device_error_word();
  if (!w) return NL_ERR_CUDA;
  int h = 0;
  if (cudaMemcpyAsync(&h, w, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return NL_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return NL_ERR_CUDA;
  if (h != 0) {
    const int zero = 0;
    cudaMemcpyAsync(w, &zero, sizeof(int), cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return h;
}
