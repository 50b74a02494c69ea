// Library-wide entry points: version, last-error text, device checks and the device
// error word that kernels with bounded waits set.
#include <stdarg.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "sm100.cuh"

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

cudaError_t ensure_smem_attr(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, cudaError_t> done;
  int dev = 0;
  const cudaError_t ge = cudaGetDevice(&dev);
  if (ge != cudaSuccess) return ge;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(func, dev);
  const auto it = done.find(key);
  if (it != done.end()) return it->second;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  done.emplace(key, e);
  return e;
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

// One warp waits on an mbarrier of arrival count 1 through the same bounded wait the GEMM
// pipelines use. With `arrive` set, lane 0 arrives first and the wait completes at once; without
// it nothing arrives, so the wait runs to `limit_ns`, records the timeout in the device error
// word and returns. `out[0]` receives 1 when the wait completed and 0 when it gave up, `out[1]`
// the nanoseconds the wait took.
__global__ void k_wait_limit_selftest(uint64_t limit_ns, int arrive, int* err,
                                      unsigned long long* out) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && arrive) sm100::mbar_arrive(&bar);
  const uint64_t t0 = sm100::globaltimer_ns();
  const bool ok = sm100::mbar_wait(&bar, 0, &abort_flag, err, limit_ns);
  const uint64_t t1 = sm100::globaltimer_ns();
  __syncwarp();
  if (threadIdx.x == 0) {
    out[0] = ok ? 1ull : 0ull;
    out[1] = t1 - t0;
  }
}
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

int to_wait_limit_selftest(int limit_us, int arrive, unsigned long long* out, void* stream) {
  if (limit_us < 1 || limit_us > 1000000)
    return tob::fail(TO_EINVAL, "to_wait_limit_selftest: limit_us %d outside [1, 1000000]",
                     limit_us);
  if (!out) return tob::fail(TO_EINVAL, "to_wait_limit_selftest: null output pointer");
  int* err = tob::device_error_ptr();
  if (!err) return tob::fail(TO_ECUDA, "to_wait_limit_selftest: device error word unavailable");
  tob::k_wait_limit_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      (uint64_t)limit_us * 1000ull, arrive ? 1 : 0, err, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_wait_limit_selftest: launch");
  return TO_OK;
}

int to_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return tob::fail(TO_EINVAL, "to_ipc_alloc: invalid argument");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_ipc_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return tob::cuda_fail(e, "to_ipc_alloc: cudaIpcGetMemHandle");
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return TO_OK;
}

int to_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return tob::fail(TO_EINVAL, "to_ipc_open: invalid argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_ipc_open: cudaIpcOpenMemHandle");
  return TO_OK;
}

int to_ipc_close(void* ptr) {
  if (!ptr) return TO_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_ipc_close: cudaIpcCloseMemHandle");
  return TO_OK;
}

int to_ipc_free(void* ptr) {
  if (!ptr) return TO_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return tob::cuda_fail(e, "to_ipc_free: cudaFree");
  return TO_OK;
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
