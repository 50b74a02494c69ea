// Shared host/device helpers for libtileops_b200: status handling, dtype dispatch,
// exact conversions and vector memory access. sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "../../include/tileops_b200.h"

namespace tob {

// ---------------------------------------------------------------- host error plumbing
// Records a formatted message for to_last_error_string() and returns `code`.
int fail(int code, const char* fmt, ...);
// Converts a CUDA runtime error into TO_ECUDA with context.
int cuda_fail(cudaError_t e, const char* what);
// Checks the launch that just happened on this thread.
inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TO_OK : cuda_fail(e, what);
}
// Number of SMs of the current device (cached per device).
int sm_count();
// Raises the dynamic shared-memory limit of kernel `func` to `bytes` on the current device, once
// per (kernel, device): the attribute belongs to the kernel in that device's context. Returns the
// status of the first call.
cudaError_t ensure_smem_attr(const void* func, int bytes);
// Device address of the library's error word on the current device (nullptr on failure).
int* device_error_ptr();
// Process-wide launch-overlap switch (programmatic dependent launch for streaming kernels).
bool launch_overlap();
// Measurement overrides of the kernel dispatch (tile shapes, splits, stage counts) are read from
// the environment only in a build compiled with -DTOB_TUNING; the product library dispatches on
// shapes alone, so a stray environment variable cannot change its kernels or numerics.
inline const char* tuning_env(const char* name) {
#ifdef TOB_TUNING
  return getenv(name);
#else
  (void)name;
  return nullptr;
#endif
}
// Codes kernels write into the error word.
enum DeviceError : int { kErrNone = 0, kErrWaitTimeout = 1, kErrTmemAlloc = 2, kErrSmemAlign = 3 };

inline const char* dtype_name(int dt) {
  switch (dt) {
    case TO_F32: return "float32";
    case TO_F16: return "float16";
    case TO_BF16: return "bfloat16";
    case TO_I8: return "int8";
    case TO_E4M3: return "float8_e4m3fn";
    case TO_I32: return "int32";
    case TO_I64: return "int64";
  }
  return "unknown";
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline unsigned grid_for(int64_t work_items, int threads, int per_sm = 8) {
  int64_t blocks = ceil_div(work_items, threads);
  int64_t cap = (int64_t)sm_count() * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

// Dispatches a runtime float dtype code to a C++ type alias `T`.
#define TOB_DISPATCH_FLOAT(code, T, ...)                                              \
  switch (code) {                                                                     \
    case TO_F32: { using T = float; __VA_ARGS__; } break;                             \
    case TO_F16: { using T = __half; __VA_ARGS__; } break;                            \
    case TO_BF16: { using T = __nv_bfloat16; __VA_ARGS__; } break;                    \
    default:                                                                          \
      return ::tob::fail(TO_EUNSUPPORTED, "unsupported floating dtype %s",            \
                         ::tob::dtype_name(code));                                    \
  }

// ---------------------------------------------------------------- device conversions
// All conversions round to nearest even, the rounding torch's CPU kernels use.
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Round an fp32 value to the storage type T and back (the value torch holds after a
// reduced-precision op).
template <typename T> __device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// Two fp32 lanes per instruction (sm_100 packed f32x2 arithmetic): each lane rounds exactly
// like the scalar mul.rn / fma.rn.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 sub2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// fp32 -> e4m3fn, round to nearest even, saturating to +-448 (cvt.rn.satfinite).
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}
// Two values at once: low byte = a, high byte = b.
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)v, __NV_E4M3);
  return __half2float(__half(h));
}

// Round-half-even then clamp to int8, as torch.clamp(torch.round(v), -128, 127).to(int8). A NaN
// (0 / 0 with a zero scale) passes torch's clamp and its int8 cast makes it 0.
__device__ __forceinline__ int8_t rne_clamp_i8(float v) {
  float r = rintf(v);
  if (isnan(r)) return 0;
  r = fminf(fmaxf(r, -128.f), 127.f);
  return (int8_t)(int)r;
}

// ---------------------------------------------------------------- vector memory access
template <int BYTES> struct VecT;
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<8> { using type = uint2; };
template <> struct VecT<16> { using type = uint4; };

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Streaming 8-byte global load that does not allocate in L1. Volatile so that it stays where
// a prefetching loop issues it (ahead of the arithmetic on the previous block).
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}

// Programmatic dependent launch: wait for the preceding grid's memory, and let the next grid
// (launched with the overlap attribute) start its prologue. Both are no-ops without it.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename T, int N> struct alignas(sizeof(T) * N) Pack {
  T v[N];
};

// Ordering key of |v|: the bit pattern of v with the sign cleared. Keys of non-negative floats
// order like the floats, and every NaN key lies above +inf's, so an unsigned maximum over keys
// is NaN as soon as one input is NaN -- the result torch's amax / aminmax give (fmaxf would
// skip the NaN instead).
__device__ __forceinline__ unsigned abs_key(float v) { return __float_as_uint(v) & 0x7FFFFFFFu; }

// Unsigned maximum across aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ unsigned warp_max_key(unsigned v, int width) {
  for (int o = width >> 1; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace tob
