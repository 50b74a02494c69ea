// Library-wide entry points: version, last-error text, device checks and the device
// error word that kernels with bounded waits set.
#include <stdarg.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace tob {

static thread_local char g_err[1024] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TO_ECUDA, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

int sm_count() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace tob

// Written by kernels whose bounded waits expired (see tcgen05 GEMMs); read by the host.
// Kernels in other translation units receive its address from tob::device_error_ptr().
__device__ int g_tob_device_error = 0;

namespace tob {
int* device_error_ptr() {
  static std::mutex mu;
  static int* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tob_device_error) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

static std::atomic<int> g_launch_overlap{0};
bool launch_overlap() { return g_launch_overlap.load(std::memory_order_relaxed) != 0; }
}  // namespace tob

extern "C" {

const char* to_version(void) { return "tileops_b200 0.1.0 (sm_100a)"; }

const char* to_last_error_string(void) { return tob::g_err; }

int to_device_check(int device) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_device_check");
  if (prop.major != 10 || prop.minor != 0)
    return tob::fail(TO_EUNSUPPORTED,
                     "device %d is sm_%d%d (%s); libtileops_b200 is built for sm_100a only",
                     device, prop.major, prop.minor, prop.name);
  return TO_OK;
}

int to_set_launch_overlap(int enable) {
  if (enable < 0) return tob::g_launch_overlap.load();
  return tob::g_launch_overlap.exchange(enable ? 1 : 0);
}

int to_device_error_word(int* value, int clear) {
  if (!value) return tob::fail(TO_EINVAL, "to_device_error_word: null output pointer");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_device_error_word: synchronize");
  e = cudaMemcpyFromSymbol(value, g_tob_device_error, sizeof(int));
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_device_error_word: read");
  if (clear) {
    int zero = 0;
    e = cudaMemcpyToSymbol(g_tob_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return tob::cuda_fail(e, "to_device_error_word: clear");
  }
  return TO_OK;
}

}  // extern "C"
