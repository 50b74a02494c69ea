// AWQ int4 decoding shared by the streaming GEMV (awq.cu) and the tensor-core GEMM
// (awq_gemm_sm100.cu).
//
// Packed layout (tileops/quant_awq.py:22): word c of a row holds logical columns 8c..8c+7 with
// column 8c+i in nibble ORDER[i], ORDER = (0,4,1,5,2,6,3,7); nibble j holds column
// [0,2,4,6,1,3,5,7][j], so (word >> 4i) & 0x000F000F puts the adjacent column pair (2i, 2i+1)
// into the two 16-bit halves, ready for the magic-bias conversion to half2 / bfloat162.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace tob {

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <typename T> struct Half2Of;
template <> struct Half2Of<__half> {
  using type = __half2;
  static constexpr uint32_t kMagic = 0x64006400u;  // 1024.0 in each half
  static __device__ __forceinline__ __half2 from_bits(uint32_t b) {
    return *reinterpret_cast<__half2*>(&b);
  }
  static __device__ __forceinline__ __half2 sixteenth() { return __float2half2_rn(0.0625f); }
  static __device__ __forceinline__ float magic_f() { return 1024.f; }
  static __device__ __forceinline__ float2 to_float2(__half2 v) { return __half22float2(v); }
  static __device__ __forceinline__ __half2 from_floats(float a, float b) {
    return __floats2half2_rn(a, b);
  }
};
template <> struct Half2Of<__nv_bfloat16> {
  using type = __nv_bfloat162;
  static constexpr uint32_t kMagic = 0x43004300u;  // 128.0 in each bf16
  static __device__ __forceinline__ __nv_bfloat162 from_bits(uint32_t b) {
    return *reinterpret_cast<__nv_bfloat162*>(&b);
  }
  static __device__ __forceinline__ __nv_bfloat162 sixteenth() {
    return __float2bfloat162_rn(0.0625f);
  }
  static __device__ __forceinline__ float magic_f() { return 128.f; }
  static __device__ __forceinline__ float2 to_float2(__nv_bfloat162 v) {
    return __bfloat1622float2(v);
  }
  static __device__ __forceinline__ __nv_bfloat162 from_floats(float a, float b) {
    return __floats2bfloat162_rn(a, b);
  }
};

// Exact (w - z) for the four column pairs of one word: d[i] holds columns (2i, 2i+1).
// fp16: the 10-bit mantissa of 1024.0 holds a nibble at bits 0-3 or 4-7 of each half, so
//   two masks per byte suffice; the bits-4-7 pairs come out as 1024 + 16 v and are folded
//   back with one fma: (1024 + 16 v)/16 - (64 + z) = v - z (exact).
//   zc[0], zc[2] = (1024 + z) pairs for columns 01/45; zc[1], zc[3] = -(64 + z) for 23/67.
// bf16: the 7-bit mantissa of 128.0 only holds bits 0-3, so every pair is shifted down first
//   and zc[i] = (128 + z) pairs for all four.
template <typename T>
__device__ __forceinline__ void awq_word_diff(uint32_t word, const typename Half2Of<T>::type* zc,
                                              typename Half2Of<T>::type* d) {
  using H = Half2Of<T>;
  if constexpr (std::is_same<T, __half>::value) {
    const uint32_t w8 = word >> 8;
    const auto p01 = H::from_bits(lop3_and_or(word, 0x000F000Fu, H::kMagic));
    const auto p23 = H::from_bits(lop3_and_or(word, 0x00F000F0u, H::kMagic));
    const auto p45 = H::from_bits(lop3_and_or(w8, 0x000F000Fu, H::kMagic));
    const auto p67 = H::from_bits(lop3_and_or(w8, 0x00F000F0u, H::kMagic));
    const auto q = H::sixteenth();
    d[0] = __hsub2(p01, zc[0]);
    d[1] = __hfma2(p23, q, zc[1]);
    d[2] = __hsub2(p45, zc[2]);
    d[3] = __hfma2(p67, q, zc[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      d[i] = __hsub2(H::from_bits(lop3_and_or(word >> (4 * i), 0x000F000Fu, H::kMagic)), zc[i]);
  }
}

template <typename T>
__device__ __forceinline__ void awq_zero_consts(uint32_t zw, typename Half2Of<T>::type* zc) {
  using H = Half2Of<T>;
  if constexpr (std::is_same<T, __half>::value) {
    const uint32_t z8 = zw >> 8;
    const auto q = H::sixteenth();
    // -(64 + z) = -(p * 1/16) with p = 1024 + 16 z (the product is exact)
    zc[0] = H::from_bits(lop3_and_or(zw, 0x000F000Fu, H::kMagic));
    zc[1] = __hneg2(__hmul2(H::from_bits(lop3_and_or(zw, 0x00F000F0u, H::kMagic)), q));
    zc[2] = H::from_bits(lop3_and_or(z8, 0x000F000Fu, H::kMagic));
    zc[3] = __hneg2(__hmul2(H::from_bits(lop3_and_or(z8, 0x00F000F0u, H::kMagic)), q));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      zc[i] = H::from_bits(lop3_and_or(zw >> (4 * i), 0x000F000Fu, H::kMagic));
  }
}

template <typename H2>
__device__ __forceinline__ uint32_t bits_of(H2 v) {
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace tob
