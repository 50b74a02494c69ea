// Elementwise and row-wise quantisation kernels (HBM-bound streams):
//   symmetric INT8 per-tensor / per-channel quantise + dequantise   (tileops/quant.py)
//   per-token(-group) dynamic INT8 and FP8 e4m3 quantise            (quant_int8.py, quant_fp8.py)
//   tensor-wide dynamic INT8 / FP8 quantise (amax pass + quantise)  (quant_int8.py:29, quant_fp8.py:52)
//   block dequantisation of INT8 / FP8 weights                      (quant_int8.py:136, quant_fp8.py:143)
// Every kernel reads its input once with 16-byte vector loads and a grid sized to the SM
// count; all float arithmetic is IEEE round-to-nearest-even so results match the
// reference's torch expressions bit for bit.
#include <mutex>
#include <type_traits>

#include "act.cuh"
#include "common.cuh"

namespace tob {
namespace {

constexpr int kThreads = 256;

inline bool aligned_to(const void* p, size_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

template <typename T, int V>
__device__ __forceinline__ Pack<T, V> ld_pack(const T* p) {
  return *reinterpret_cast<const Pack<T, V>*>(p);
}
template <typename T, int V>
__device__ __forceinline__ void st_pack(T* p, const Pack<T, V>& v) {
  *reinterpret_cast<Pack<T, V>*>(p) = v;
}

// Splits a flat index of a [outer, channels, inner] tensor into (channel, position in inner).
struct ChannelCursor {
  int64_t c, r;
  __device__ __forceinline__ ChannelCursor(int64_t idx, int64_t channels, int64_t inner) {
    int64_t t = idx / inner;
    r = idx - t * inner;
    c = t % channels;
  }
  __device__ __forceinline__ void next(int64_t channels, int64_t inner) {
    if (++r == inner) {
      r = 0;
      if (++c == channels) c = 0;
    }
  }
};

// ------------------------------------------------------------------ symmetric INT8
// q = clamp(rint(float(x) / s), -128, 127). Per-tensor when channels == 1.
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) k_quant_sym(const T* __restrict__ x,
                                                       const float* __restrict__ scale,
                                                       int8_t* __restrict__ q, int64_t n,
                                                       int64_t channels, int64_t inner) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nvec = n / V;
  const float s0 = __ldg(scale);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    Pack<T, V> v = ld_pack<T, V>(x + i * V);
    Pack<int8_t, V> o;
    if (channels == 1) {
#pragma unroll
      for (int j = 0; j < V; ++j) o.v[j] = rne_clamp_i8(__fdiv_rn(to_f32(v.v[j]), s0));
    } else {
      ChannelCursor cur(i * V, channels, inner);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        o.v[j] = rne_clamp_i8(__fdiv_rn(to_f32(v.v[j]), __ldg(scale + cur.c)));
        cur.next(channels, inner);
      }
    }
    st_pack<int8_t, V>(q + i * V, o);
  }
  for (int64_t i = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float s = channels == 1 ? s0 : __ldg(scale + (i / inner) % channels);
    q[i] = rne_clamp_i8(__fdiv_rn(to_f32(x[i]), s));
  }
}

// y = T(float(q) * s).
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) k_dequant_sym(const int8_t* __restrict__ q,
                                                         const float* __restrict__ scale,
                                                         T* __restrict__ y, int64_t n,
                                                         int64_t channels, int64_t inner) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nvec = n / V;
  const float s0 = __ldg(scale);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    Pack<int8_t, V> v = ld_pack<int8_t, V>(q + i * V);
    Pack<T, V> o;
    if (channels == 1) {
#pragma unroll
      for (int j = 0; j < V; ++j) o.v[j] = from_f32<T>(__fmul_rn((float)v.v[j], s0));
    } else {
      ChannelCursor cur(i * V, channels, inner);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        o.v[j] = from_f32<T>(__fmul_rn((float)v.v[j], __ldg(scale + cur.c)));
        cur.next(channels, inner);
      }
    }
    st_pack<T, V>(y + i * V, o);
  }
  for (int64_t i = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float s = channels == 1 ? s0 : __ldg(scale + (i / inner) % channels);
    y[i] = from_f32<T>(__fmul_rn((float)q[i], s));
  }
}

template <typename T>
int launch_quant_sym(const void* x, const float* scale, int8_t* q, int64_t n, int64_t channels,
                     int64_t inner, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  unsigned grid = grid_for(ceil_div(n, V), kThreads);
  if (aligned16(x) && aligned_to(q, V))
    k_quant_sym<T, V><<<grid, kThreads, 0, st>>>((const T*)x, scale, q, n, channels, inner);
  else
    k_quant_sym<T, 1><<<grid, kThreads, 0, st>>>((const T*)x, scale, q, n, channels, inner);
  return check_launch("quantize int8 (symmetric)");
}

template <typename T>
int launch_dequant_sym(const int8_t* q, const float* scale, void* y, int64_t n, int64_t channels,
                       int64_t inner, cudaStream_t st) {
  constexpr int V = 8;
  unsigned grid = grid_for(ceil_div(n, V), kThreads);
  if (aligned_to(q, V) && aligned_to(y, V * sizeof(T)))
    k_dequant_sym<T, V><<<grid, kThreads, 0, st>>>(q, scale, (T*)y, n, channels, inner);
  else
    k_dequant_sym<T, 1><<<grid, kThreads, 0, st>>>(q, scale, (T*)y, n, channels, inner);
  return check_launch("dequantize int8 (symmetric)");
}

// ------------------------------------------------------------------ per-token-group quant
// One "team" of 2^team_log2 threads per group of G contiguous elements. Each thread keeps up
// to MAXV vectors of its slice in registers, so x is read from HBM exactly once; groups too
// large for the register cache re-read the tail (served from L2).
struct ScaleLayout {
  int64_t cm_rows;    // > 0: the reference's column_major_scales layout (see scale_offset)
  int64_t cm_groups;  // groups per row
  int64_t tma_ld = 0;  // > 0: TMA-aligned column-major scales, cm_groups groups per row
};

// Position of group g's scale. Natural order is g. With column_major_scales the reference
// returns s_flat.reshape(..., G_, M).transpose(-2, -1).contiguous() (quant_fp8.py:129-136):
// within each batch of M rows x G_ groups, flat scale t lands at row t % M, column t / M of
// a contiguous [M, G_] tensor.
// With tma_ld > 0 (the layout DeepGEMM-style kernels load with TMA): the scale of row r, group
// j of a 2-D input sits at j * tma_ld + r, tma_ld being the row count rounded up to 4 floats
// (16 bytes) so that every column starts 16-byte aligned.
__device__ __forceinline__ int64_t scale_offset(int64_t g, const ScaleLayout& sl) {
  if (sl.tma_ld > 0) {
    const int64_t r = g / sl.cm_groups;
    return (g - r * sl.cm_groups) * sl.tma_ld + r;
  }
  if (sl.cm_rows <= 0) return g;
  const int64_t per_batch = sl.cm_rows * sl.cm_groups;
  const int64_t b = g / per_batch;
  const int64_t t = g - b * per_batch;
  return b * per_batch + (t % sl.cm_rows) * sl.cm_groups + t / sl.cm_rows;
}

// 2^ceil(log2(max(s, 1e-30))) with log2 rounded to fp32 first, as torch evaluates
// torch.exp2(torch.ceil(torch.log2(s))) (quant_fp8.py:48-49).
__device__ __forceinline__ float ue8m0_round(float s) {
  if (isinf(s)) return s;
  s = fmaxf(s, 1e-30f);
  const float l = (float)log2((double)s);
  return ldexpf(1.0f, (int)ceilf(l));
}

// Output codes of the quantisers: int8, OCP float8_e4m3fn, or float8_e4m3fnuz (the encoding
// with exponent bias 8, no infinities, no negative zero and one NaN, 0x80; the reference's
// `dtype` argument accepts it, tileops/quant_fp8.py:19-45).
enum QKind : int { kQI8 = 0, kQE4M3 = 1, kQE4M3Fnuz = 2 };

// fp32 -> e4m3fnuz, round to nearest even, for |v| <= 240 (the quantisers clamp first). The
// fnuz grid is the e4m3fn grid halved (bias 8 against 7, same mantissa), so the code is the
// e4m3fn code of 2v, except: above 232 (the tie between 224 and 240) the nearest fnuz value is
// 240, code 0x7F, which e4m3fn spends on NaN; and e4m3fn's -0 (0x80) is fnuz's NaN, so a
// result of zero is +0.
__device__ __forceinline__ uint8_t f32_to_e4m3fnuz(float v) {
  uint8_t b = f32_to_e4m3(2.0f * v);
  if (fabsf(v) > 232.0f) b = (uint8_t)(((__float_as_uint(v) >> 24) & 0x80u) | 0x7Fu);
  return b == 0x80 ? (uint8_t)0 : b;
}
__device__ __forceinline__ float e4m3fnuz_to_f32(uint8_t b) {
  if (b == 0x80) return __uint_as_float(0x7FC00000u);
  if ((b & 0x7F) == 0x7F) return (b & 0x80) ? -240.0f : 240.0f;
  return 0.5f * e4m3_to_f32(b);
}

// e4m3 code of a NaN quotient x / scale, as the reference's fp32 division and cast produce it
// on the x86 host it is pinned to: with a NaN scale (a NaN in the group) the quotient is the
// NaN operand that comes first -- x itself when x is NaN, else the scale's sign-clear NaN --
// and the cast keeps its sign (0x7F or 0xFF); with a numeric scale the NaN comes from an
// invalid operation (inf / inf, 0 / 0), whose default NaN has the sign set (0xFF).
// `neg_x` is the sign bit of x as stored: the conversion of a 16-bit NaN to fp32 does not
// keep its sign on the GPU.
__device__ __forceinline__ uint8_t nan_code_div(float x, bool neg_x, bool nan_scale) {
  if (!nan_scale) return 0xFF;
  return (isnan(x) && neg_x) ? (uint8_t)0xFF : (uint8_t)0x7F;
}

// Codes of x / scale without a division per element: the bracket test. With r = 1 / scale
// rounded to fp32, lo = r (1 - 2^-21) and hi = r (1 + 2^-21), each rounded, the products x lo
// and x hi enclose both the exact quotient and its fp32 rounding: r, lo, hi and a rounded
// product are each off by at most 2^-24 relatively, 4 x 2^-24 in all, inside the 8 x 2^-24
// margin. Rounding onto the code grid (e4m3fn RNE with saturation, or RNE to an integer) is
// monotone, so when both products give the same code the correctly rounded quotient gives it
// too; a pack where they differ takes the IEEE division for every value. The test holds on the
// e4m3 subnormal grid and at saturation alike. It needs a scale whose reciprocal is a normal
// fp32 number and a group without NaN or infinity (a finite absmax); a scale within
// [1.2e-38, 8e37] implies both.
struct Bracket {
  float lo, hi;
};
__device__ __forceinline__ Bracket make_bracket(float scale) {
  const float r = __frcp_rn(scale);
  return {__fmul_rn(r, 1.0f - 0x1p-21f), __fmul_rn(r, 1.0f + 0x1p-21f)};
}

// RNE integer of the exact product x * m plus 1.5 x 2^23: for |x m| < 2^22 the sum's low bits
// are the integer in two's complement (its low byte is the int8 code).
__device__ __forceinline__ uint32_t rne_int_bits(float x, float m) {
  return __float_as_uint(__fmaf_rn(x, m, 12582912.0f));
}

// The code of the IEEE quotient x / scale (a finite x, a normal scale: no NaN can arise).
template <int Q> __device__ __forceinline__ uint32_t exact_code(float x, float scale) {
  const float y = __fdiv_rn(x, scale);
  if constexpr (Q == kQE4M3) return f32_to_e4m3(fminf(fmaxf(y, -448.f), 448.f));
  else return (uint8_t)rne_clamp_i8(y);
}

// Four codes from the two ends' codes wl, wh (byte j for x[j]): where they differ -- a quotient
// on or next to a rounding boundary, which bf16 inputs hit often since x / scale is then
// frequently an exact e4m3 midpoint -- that value alone divides.
template <int Q>
__device__ __noinline__ uint32_t fix_codes(uint32_t wl, uint32_t wh, float x0, float x1, float x2,
                                           float x3, float scale) {
  const float x[4] = {x0, x1, x2, x3};
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (((wl ^ wh) >> (8 * j)) & 0xFFu)
      wl = (wl & ~(0xFFu << (8 * j))) | (exact_code<Q>(x[j], scale) << (8 * j));
  return wl;
}

// Codes of a pack by the bracket test, the products two lanes per instruction (mul.rn.f32x2 /
// fma.rn.f32x2 round each lane like the scalar forms). e4m3fn: a pair converts in one
// cvt.rn.satfinite.e4m3x2. int8: |x / scale| <= 127 (1 + 2^-22) on this path (scale =
// max(absmax, eps) / 127 rounded), so no value reaches the clamp, and the two ends differ by at
// most one, so their low bytes tell whether they differ. One branch per pack leads to the
// per-value fix-ups.
template <int Q, typename T, int V>
__device__ __forceinline__ void bracket_codes(const Pack<T, V>& t, const Bracket& b, float scale,
                                              Pack<uint8_t, V>& o) {
  if constexpr (V == 1) {
    const float x = to_f32(t.v[0]);
    uint32_t l, h;
    if constexpr (Q == kQE4M3) {
      const uint32_t c = f32x2_to_e4m3x2(__fmul_rn(x, b.lo), __fmul_rn(x, b.hi));
      l = c & 0xFFu;
      h = c >> 8;
    } else {
      l = rne_int_bits(x, b.lo) & 0xFFu;
      h = rne_int_bits(x, b.hi) & 0xFFu;
    }
    o.v[0] = (uint8_t)(l == h ? l : exact_code<Q>(x, scale));
  } else {
    static_assert(V % 4 == 0, "bracket_codes packs four codes to a word");
    constexpr int W = V / 4;
    const float2 lo2 = make_float2(b.lo, b.lo), hi2 = make_float2(b.hi, b.hi);
    uint32_t wl[W], wh[W], diff = 0u;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const float2 x01 = make_float2(to_f32(t.v[4 * k]), to_f32(t.v[4 * k + 1]));
      const float2 x23 = make_float2(to_f32(t.v[4 * k + 2]), to_f32(t.v[4 * k + 3]));
      if constexpr (Q == kQE4M3) {
        const float2 l01 = mul2_rn(x01, lo2), h01 = mul2_rn(x01, hi2);
        const float2 l23 = mul2_rn(x23, lo2), h23 = mul2_rn(x23, hi2);
        wl[k] = __byte_perm(f32x2_to_e4m3x2(l01.x, l01.y), f32x2_to_e4m3x2(l23.x, l23.y), 0x5410);
        wh[k] = __byte_perm(f32x2_to_e4m3x2(h01.x, h01.y), f32x2_to_e4m3x2(h23.x, h23.y), 0x5410);
      } else {
        const float2 m2 = make_float2(12582912.0f, 12582912.0f);
        const float2 l01 = fma2_rn(x01, lo2, m2), h01 = fma2_rn(x01, hi2, m2);
        const float2 l23 = fma2_rn(x23, lo2, m2), h23 = fma2_rn(x23, hi2, m2);
        wl[k] = __byte_perm(__byte_perm(__float_as_uint(l01.x), __float_as_uint(l01.y), 0x0040),
                            __byte_perm(__float_as_uint(l23.x), __float_as_uint(l23.y), 0x0040),
                            0x5410);
        wh[k] = __byte_perm(__byte_perm(__float_as_uint(h01.x), __float_as_uint(h01.y), 0x0040),
                            __byte_perm(__float_as_uint(h23.x), __float_as_uint(h23.y), 0x0040),
                            0x5410);
      }
      diff |= wl[k] ^ wh[k];
    }
    if (diff != 0u) {
#pragma unroll
      for (int k = 0; k < W; ++k)
        if (wl[k] != wh[k])
          wl[k] = fix_codes<Q>(wl[k], wh[k], to_f32(t.v[4 * k]), to_f32(t.v[4 * k + 1]),
                               to_f32(t.v[4 * k + 2]), to_f32(t.v[4 * k + 3]), scale);
    }
    uint32_t* w = reinterpret_cast<uint32_t*>(o.v);
#pragma unroll
    for (int k = 0; k < W; ++k) w[k] = wl[k];
  }
}

// Running maximum of |x| over packs, read out as the abs_key of the largest |x|. 16-bit types
// keep the sign-cleared bit patterns two to a word and take halfword-wise unsigned maxima
// (max.u16x2): patterns of non-negative values order as the values, with NaNs above infinity,
// and the largest converts to the same fp32 key the per-value path finds.
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename T> struct AbsMax {
  unsigned k = 0u;
  template <int V> __device__ __forceinline__ void add(const Pack<T, V>& p) {
#pragma unroll
    for (int j = 0; j < V; ++j) k = max(k, abs_key(to_f32(p.v[j])));
  }
  __device__ __forceinline__ unsigned key() const { return k; }
};
__device__ __forceinline__ unsigned short bits16(__half v) { return __half_as_ushort(v); }
__device__ __forceinline__ unsigned short bits16(__nv_bfloat16 v) { return __bfloat16_as_ushort(v); }
template <typename T> struct AbsMax16 {
  uint32_t k2 = 0u;
  template <int V> __device__ __forceinline__ void add(const Pack<T, V>& p) {
    if constexpr (V % 2 == 0) {
      const uint32_t* w = reinterpret_cast<const uint32_t*>(p.v);
#pragma unroll
      for (int i = 0; i < V / 2; ++i) k2 = max_u16x2(k2, w[i] & 0x7FFF7FFFu);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j)
        k2 = max(k2, (uint32_t)(bits16(p.v[j]) & 0x7FFFu));
    }
  }
  __device__ __forceinline__ unsigned key() const {
    const unsigned short m = (unsigned short)max(k2 & 0xFFFFu, k2 >> 16);
    if constexpr (std::is_same<T, __half>::value) return abs_key(__half2float(__ushort_as_half(m)));
    else return abs_key(__bfloat162float(__ushort_as_bfloat16(m)));
  }
};
template <> struct AbsMax<__half> : AbsMax16<__half> {};
template <> struct AbsMax<__nv_bfloat16> : AbsMax16<__nv_bfloat16> {};

// Sign bit of a stored value.
__device__ __forceinline__ bool sign_of(float v) { return __float_as_uint(v) >> 31; }
__device__ __forceinline__ bool sign_of(__half v) { return __half_as_ushort(v) >> 15; }
__device__ __forceinline__ bool sign_of(__nv_bfloat16 v) { return __bfloat16_as_ushort(v) >> 15; }

// Where the quantiser's groups come from: a contiguous x (groups back to back), or the gated
// activation act(gate) * up of a gate_up output given as [rows, cols] views with row strides
// (cols = groups per row x G), each value rounded to T exactly as the activation kernel writes
// it -- the activation that produces the next layer's input, fused into its quantiser.
template <typename T, int ACT> struct GroupSrc {
  const T* a;
  const T* b;
  int64_t lda, ldb, gpr;  // row strides, groups per row
  template <int V>
  __device__ __forceinline__ Pack<T, V> load(int64_t g, int G, int v) const {
    const int64_t r = g / gpr;
    const int64_t c = (g - r * gpr) * G + (int64_t)v * V;
    const Pack<T, V> pa = ld_pack<T, V>(a + r * lda + c), pb = ld_pack<T, V>(b + r * ldb + c);
    Pack<T, V> o;
#pragma unroll
    for (int j = 0; j < V; ++j) o.v[j] = act_mul<T, ACT>(pa.v[j], pb.v[j]);
    return o;
  }
};
template <typename T> struct GroupSrc<T, -1> {
  const T* x;
  template <int V>
  __device__ __forceinline__ Pack<T, V> load(int64_t g, int G, int v) const {
    return ld_pack<T, V>(x + g * (int64_t)G + (int64_t)v * V);
  }
};

template <typename T, int Q, int V, int MAXV, int ACT = -1>
__global__ void __launch_bounds__(1024) k_group_quant(const GroupSrc<T, ACT> src,
                                                     uint8_t* __restrict__ qout,
                                                     float* __restrict__ scales, int64_t n_groups,
                                                     int G, int team_log2, float eps, int ue8m0,
                                                     ScaleLayout sl) {
  const int team = 1 << team_log2;
  const int lane = threadIdx.x & (team - 1);
  const int teams_per_cta = blockDim.x >> team_log2;
  const int team_id = threadIdx.x >> team_log2;
  const int nvec = G / V;
  __shared__ unsigned red[32];
  constexpr bool FP8 = Q != kQI8;
  // clamp bounds: int8 127; e4m3fn 448; e4m3fnuz 224 (get_fp8_min_max's override)
  const float qmax = Q == kQE4M3 ? 448.0f : (Q == kQE4M3Fnuz ? 224.0f : 127.0f);

  for (int64_t g0 = (int64_t)blockIdx.x * teams_per_cta; g0 < n_groups;
       g0 += (int64_t)gridDim.x * teams_per_cta) {
    const int64_t g = g0 + team_id;
    const bool active = g < n_groups;
    Pack<T, V> cache[MAXV];
    AbsMax<T> am;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int v = lane + i * team;
      if (active && v < nvec) {
        cache[i] = src.template load<V>(g, G, v);
        am.add(cache[i]);
      }
    }
    for (int v = lane + MAXV * team; active && v < nvec; v += team)
      am.add(src.template load<V>(g, G, v));
    unsigned amax = am.key();  // abs_key of the group's largest |x|; a NaN anywhere makes it NaN
    if (team <= 32) {
      amax = warp_max_key(amax, team);
    } else {
      amax = warp_max_key(amax, 32);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
      __syncthreads();
      // Several teams of 64..1024 threads can share a CTA; each reads only its own warps.
      unsigned m = 0u;
      const int w0 = (team_id * team) >> 5;
      for (int w = 0; w < (team >> 5); ++w) m = max(m, red[w0 + w]);
      amax = m;
      __syncthreads();
    }
    // scale = clamp(absmax, min=eps) / qmax  (fp32, IEEE division). A NaN absmax passes the
    // reference's clamp, division and UE8M0 rounding unchanged (quiet NaN, sign clear).
    const float amax_f = __uint_as_float(amax);
    const bool nan_group = isnan(amax_f);
    float scale = nan_group ? amax_f : __fdiv_rn(fmaxf(amax_f, eps), qmax);
    if (FP8 && ue8m0 && !nan_group) scale = ue8m0_round(scale);
    if (active && lane == 0) scales[scale_offset(g, sl)] = scale;
    uint8_t* qg = qout + g * (int64_t)G;
    // e4m3fn and int8 codes come from the bracket test when the scale allows it; otherwise
    // (NaN, inf, 0 or extreme scales, e4m3fnuz, a pack whose bracket straddles a rounding
    // boundary) every value divides.
    const bool fast = (Q == kQE4M3 || Q == kQI8) && scale >= 1.2e-38f && scale <= 8.0e37f;
    const Bracket br = fast ? make_bracket(scale) : Bracket{0.0f, 0.0f};
    auto emit = [&](int v, const Pack<T, V>& t) {
      Pack<uint8_t, V> o;
      if constexpr (Q == kQE4M3 || Q == kQI8) {
        if (fast) {
          bracket_codes<Q>(t, br, scale, o);
          st_pack<uint8_t, V>(qg + (int64_t)v * V, o);
          return;
        }
      }
      {
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float xv = to_f32(t.v[j]);
          const float y = __fdiv_rn(xv, scale);
          if (Q == kQE4M3) {
            o.v[j] = isnan(y) ? nan_code_div(xv, sign_of(t.v[j]), nan_group)
                              : f32_to_e4m3(fminf(fmaxf(y, -448.f), 448.f));
          } else if (Q == kQE4M3Fnuz) {
            o.v[j] = isnan(y) ? (uint8_t)0x80 : f32_to_e4m3fnuz(fminf(fmaxf(y, -224.f), 224.f));
          } else {
            o.v[j] = (uint8_t)rne_clamp_i8(y);
          }
        }
      }
      st_pack<uint8_t, V>(qg + (int64_t)v * V, o);
    };
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int v = lane + i * team;
      if (active && v < nvec) emit(v, cache[i]);
    }
    for (int v = lane + MAXV * team; active && v < nvec; v += team)
      emit(v, src.template load<V>(g, G, v));
  }
}

// Threads per group (a power of two up to 1024) and grid for n_groups groups of nvec vectors.
struct GroupGrid {
  int team_log2, threads;
  int64_t blocks;
};
inline GroupGrid group_grid(int64_t n_groups, int64_t nvec, int maxv) {
  GroupGrid gg;
  const int64_t want = ceil_div(nvec, maxv);
  gg.team_log2 = 0;
  while ((1 << gg.team_log2) < want && gg.team_log2 < 10) ++gg.team_log2;
  const int team = 1 << gg.team_log2;
  gg.threads = team > kThreads ? team : kThreads;
  const int64_t teams_per_cta = gg.threads / team;
  gg.blocks = ceil_div(n_groups, teams_per_cta);
  const int64_t cap = (int64_t)sm_count() * 64;
  if (gg.blocks > cap) gg.blocks = cap;
  if (gg.blocks < 1) gg.blocks = 1;
  return gg;
}

template <typename T, int Q>
int launch_group_quant(const void* x, int64_t n_groups, int64_t G, float eps, int ue8m0,
                       ScaleLayout sl, void* q, float* scales, cudaStream_t st) {
  constexpr int VV = 16 / sizeof(T);
  const bool vec = (G % VV == 0) && aligned16(x) && aligned_to(q, VV);
  const GroupGrid gg = group_grid(n_groups, G / (vec ? VV : 1), vec ? 4 : 8);
  GroupSrc<T, -1> src{(const T*)x};
  if (vec)
    k_group_quant<T, Q, VV, 4><<<(unsigned)gg.blocks, gg.threads, 0, st>>>(
        src, (uint8_t*)q, scales, n_groups, (int)G, gg.team_log2, eps, ue8m0, sl);
  else
    k_group_quant<T, Q, 1, 8><<<(unsigned)gg.blocks, gg.threads, 0, st>>>(
        src, (uint8_t*)q, scales, n_groups, (int)G, gg.team_log2, eps, ue8m0, sl);
  return check_launch(Q != kQI8 ? "per_token_group_quant_fp8" : "per_token_group_quant_int8");
}

// The quantiser of act(gate) * up ([rows, cols] views a, b with row strides lda, ldb).
template <typename T, int Q, int ACT>
int launch_act_group_quant(const void* a, const void* b, int64_t rows, int64_t cols, int64_t lda,
                           int64_t ldb, int64_t G, float eps, int ue8m0, ScaleLayout sl, void* q,
                           float* scales, cudaStream_t st) {
  constexpr int VV = 16 / sizeof(T);
  const bool vec = (G % VV == 0) && lda % VV == 0 && ldb % VV == 0 && aligned16(a) &&
                   aligned16(b) && aligned_to(q, VV);
  const int64_t n_groups = rows * (cols / G);
  // Two cached vectors per thread: the activation's arithmetic leaves no registers for four.
  const GroupGrid gg = group_grid(n_groups, G / (vec ? VV : 1), vec ? 2 : 8);
  GroupSrc<T, ACT> src{(const T*)a, (const T*)b, lda, ldb, cols / G};
  if (vec)
    k_group_quant<T, Q, VV, 2, ACT><<<(unsigned)gg.blocks, gg.threads, 0, st>>>(
        src, (uint8_t*)q, scales, n_groups, (int)G, gg.team_log2, eps, ue8m0, sl);
  else
    k_group_quant<T, Q, 1, 8, ACT><<<(unsigned)gg.blocks, gg.threads, 0, st>>>(
        src, (uint8_t*)q, scales, n_groups, (int)G, gg.team_log2, eps, ue8m0, sl);
  return check_launch("act_and_mul_group_quant");
}

// ------------------------------------------------------------------ tensor-wide dynamic quant
// Pass 1: amax = max |x| folded into one word with atomicMax on abs_key (NaN above every number,
// so a NaN anywhere makes the tensor's amax NaN, as the reference's aminmax does).
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) k_absmax(const T* __restrict__ x, int64_t n,
                                                    unsigned* __restrict__ amax_bits) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nvec = n / V;
  AbsMax<T> am;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // Four loads in flight per thread (64 bytes): one 16-byte load at a time leaves too few
  // bytes in flight per SM to cover DRAM latency.
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    Pack<T, V> p[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) p[u] = ld_pack<T, V>(x + (i + u * stride) * V);
#pragma unroll
    for (int u = 0; u < 4; ++u) am.add(p[u]);
  }
  for (; i < nvec; i += stride) am.add(ld_pack<T, V>(x + i * V));
  for (int64_t j = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += stride)
    am.add(ld_pack<T, 1>(x + j));
  unsigned m = warp_max_key(am.key(), 32);
  __shared__ unsigned red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned b = 0u;
    for (int w = 0; w < kThreads / 32; ++w) b = max(b, red[w]);
    atomicMax(amax_bits, b);
  }
}

// e4m3 code of a NaN product T(x * s) in the reference's tensor-wide quantiser, as its x86 run
// gives it. bfloat16: torch's vectorised bf16 rounding writes every NaN as 0xFFFF (sign set)
// in whole 32-element blocks from the start of the tensor, its scalar tail rounding as the
// sign-clear 0x7FC0. float32 / float16: a NaN scale (a NaN in the tensor) gives a sign-clear
// NaN; with a numeric scale the NaN comes from 0 * inf, the sign-set default NaN.
template <typename T>
__device__ __forceinline__ uint8_t nan_code_mul(int64_t i, int64_t n_blocked, bool nan_scale) {
  if (std::is_same<T, __nv_bfloat16>::value) return i < n_blocked ? (uint8_t)0xFF : (uint8_t)0x7F;
  return nan_scale ? (uint8_t)0x7F : (uint8_t)0xFF;
}

// Pass 2, in the input dtype T exactly as the reference's expression evaluates:
//   amax = T(max(amax, 1e-12)); s = T(T(1/amax) * qmax); q = cast(clamp(T(x*s), qmin, qmax)).
// A NaN amax passes the clamp, so s and every product are NaN. NaN products survive the clamp;
// the int8 cast makes them 0, the e4m3 cast a NaN code (nan_code_mul). In float16 the 1e-12
// floor rounds to 0, so an all-zero tensor has s = inf and NaN products 0 * inf.
// The int8 cast truncates toward zero (torch .to(int8)); the fp8 cast rounds to nearest even.
template <typename T, int Q, int V>
__global__ void __launch_bounds__(kThreads) k_tensor_quant(const T* __restrict__ x, int64_t n,
                                                          const unsigned* __restrict__ amax_bits,
                                                          uint8_t* __restrict__ q,
                                                          float* __restrict__ dq_scale) {
  constexpr bool FP8 = Q != kQI8;
  // finfo bounds: int8 [-128, 127]; e4m3fn +-448; e4m3fnuz +-240
  const float qmax = Q == kQE4M3 ? 448.0f : (Q == kQE4M3Fnuz ? 240.0f : 127.0f);
  const float qmin = Q == kQE4M3 ? -448.0f : (Q == kQE4M3Fnuz ? -240.0f : -128.0f);
  const float amax_raw = __uint_as_float(*amax_bits);
  const bool nan_scale = isnan(amax_raw);
  const float amax = nan_scale ? amax_raw : round_to<T>(fmaxf(amax_raw, 1e-12f));
  const float r = round_to<T>(__frcp_rn(amax));
  const float s = round_to<T>(__fmul_rn(r, qmax));
  const int64_t n_blocked = n & ~(int64_t)31;
  if (blockIdx.x == 0 && threadIdx.x == 0) *dq_scale = __frcp_rn(s);
  auto quant1 = [&](float xv, int64_t i) -> uint8_t {
    float y = round_to<T>(__fmul_rn(xv, s));
    if (isnan(y)) {
      if (Q == kQE4M3Fnuz) return (uint8_t)0x80;  // fnuz's only NaN
      return FP8 ? nan_code_mul<T>(i, n_blocked, nan_scale) : (uint8_t)0;
    }
    y = fminf(fmaxf(y, qmin), qmax);
    if (Q == kQE4M3Fnuz) return f32_to_e4m3fnuz(y);
    if (FP8) return f32_to_e4m3(y);
    return (uint8_t)(int8_t)(int)y;  // truncation toward zero
  };
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t nvec = n / V;
  auto quant_pack = [&](const Pack<T, V>& v, int64_t i) {
    Pack<uint8_t, V> o;
#pragma unroll
    for (int j = 0; j < V; ++j) o.v[j] = quant1(to_f32(v.v[j]), i * V + j);
    st_pack<uint8_t, V>(q + i * V, o);
  };
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + stride < nvec; i += 2 * stride) {  // two loads in flight per thread
    const Pack<T, V> v0 = ld_pack<T, V>(x + i * V);
    const Pack<T, V> v1 = ld_pack<T, V>(x + (i + stride) * V);
    quant_pack(v0, i);
    quant_pack(v1, i + stride);
  }
  for (; i < nvec; i += stride) quant_pack(ld_pack<T, V>(x + i * V), i);
  for (int64_t j = nvec * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += stride)
    q[j] = quant1(to_f32(x[j]), j);
}

template <typename T, int Q>
int launch_tensor_quant(const void* x, int64_t n, void* q, float* dq_scale, unsigned* ws,
                        cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(unsigned), st);
  if (e != cudaSuccess) return cuda_fail(e, "tensor-wide quant: clear amax word");
  unsigned grid = grid_for(ceil_div(n, V), kThreads, 4);
  const bool vec = aligned16(x) && aligned_to(q, V);
  if (vec)
    k_absmax<T, V><<<grid, kThreads, 0, st>>>((const T*)x, n, ws);
  else
    k_absmax<T, 1><<<grid, kThreads, 0, st>>>((const T*)x, n, ws);
  int rc = check_launch("tensor-wide quant: amax");
  if (rc) return rc;
  grid = grid_for(ceil_div(n, V), kThreads, 8);
  if (vec)
    k_tensor_quant<T, Q, V><<<grid, kThreads, 0, st>>>((const T*)x, n, ws, (uint8_t*)q, dq_scale);
  else
    k_tensor_quant<T, Q, 1><<<grid, kThreads, 0, st>>>((const T*)x, n, ws, (uint8_t*)q, dq_scale);
  return check_launch("tensor-wide quant: quantize");
}

// ------------------------------------------------------------------ block dequant
template <int Q>
__global__ void __launch_bounds__(kThreads) k_block_dequant(const uint8_t* __restrict__ q,
                                                           const float* __restrict__ s,
                                                           float* __restrict__ y, int64_t n,
                                                           int64_t k, int64_t bn, int64_t bk,
                                                           int64_t k_tiles) {
  const int64_t total = n * k;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / k;
    const int64_t c = i - r * k;
    const uint8_t v = q[i];
    const float f = Q == kQE4M3 ? e4m3_to_f32(v)
                                : (Q == kQE4M3Fnuz ? e4m3fnuz_to_f32(v) : (float)(int8_t)v);
    y[i] = __fmul_rn(f, __ldg(s + (r / bn) * k_tiles + c / bk));
  }
}

int launch_block_dequant(int kind, const void* q, const float* s, float* y, int64_t n, int64_t k,
                         int64_t bn, int64_t bk, cudaStream_t st) {
  if (n < 0 || k < 0 || bn <= 0 || bk <= 0)
    return fail(TO_EINVAL, "block_dequant: invalid sizes n=%lld k=%lld block=[%lld,%lld]",
                (long long)n, (long long)k, (long long)bn, (long long)bk);
  if (n == 0 || k == 0) return TO_OK;
  const int64_t kt = ceil_div(k, bk);
  unsigned grid = grid_for(n * k, kThreads, 8);
  if (kind == kQE4M3)
    k_block_dequant<kQE4M3><<<grid, kThreads, 0, st>>>((const uint8_t*)q, s, y, n, k, bn, bk, kt);
  else if (kind == kQE4M3Fnuz)
    k_block_dequant<kQE4M3Fnuz><<<grid, kThreads, 0, st>>>((const uint8_t*)q, s, y, n, k, bn, bk,
                                                          kt);
  else
    k_block_dequant<kQI8><<<grid, kThreads, 0, st>>>((const uint8_t*)q, s, y, n, k, bn, bk, kt);
  return check_launch("block_dequant");
}

// ------------------------------------------------------------------ no-allocation variant
// Scratch of to_input_to_fp8_noalloc: one partial |x| maximum (float bits) per chunk of
// kNoAllocChunk elements, then the final maximum at index kNoAllocSlots. It is part of the
// library image, so every GPU that loads the library holds these 33 KB until the process
// exits. Each call writes every slot it later reads, so nothing needs clearing between calls;
// two calls that run at the same time on the GPU (different streams or threads) overwrite each
// other's slots and must not overlap.
constexpr int kNoAllocSlots = 8192;
constexpr int64_t kNoAllocChunk = 16384;
constexpr int64_t kNoAllocMaxElems = (int64_t)kNoAllocSlots * kNoAllocChunk;  // 134,217,728
static __device__ __align__(256) unsigned g_noalloc_amax[kNoAllocSlots + 64];

// CTA b: max |x| (as abs_key) over elements [b * kNoAllocChunk, min(n, (b + 1) * kNoAllocChunk)).
template <typename T, int V>
__global__ void __launch_bounds__(kThreads) k_absmax_chunks(const T* __restrict__ x, int64_t n,
                                                           unsigned* __restrict__ partial) {
  const int64_t beg = (int64_t)blockIdx.x * kNoAllocChunk;
  const int64_t end = min(n, beg + kNoAllocChunk);
  unsigned m = 0u;
  const int64_t vbeg = (beg + V - 1) / V, vend = end / V;
  for (int64_t i = vbeg + threadIdx.x; i < vend; i += blockDim.x) {
    Pack<T, V> v = ld_pack<T, V>(x + i * V);
#pragma unroll
    for (int j = 0; j < V; ++j) m = max(m, abs_key(to_f32(v.v[j])));
  }
  for (int64_t i = beg + threadIdx.x; i < min(end, vbeg * V); i += blockDim.x)
    m = max(m, abs_key(to_f32(x[i])));  // head before the first full vector
  for (int64_t i = max(vend * V, beg) + threadIdx.x; i < end; i += blockDim.x)
    m = max(m, abs_key(to_f32(x[i])));  // tail after the last full vector
  m = warp_max_key(m, 32);
  __shared__ unsigned red[kThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned b = 0u;
    for (int w = 0; w < kThreads / 32; ++w) b = max(b, red[w]);
    partial[blockIdx.x] = b;
  }
}

// One CTA folds the nparts partial maxima into *out.
__global__ void __launch_bounds__(1024) k_absmax_final(const unsigned* __restrict__ partial,
                                                      int nparts, unsigned* __restrict__ out) {
  unsigned m = 0u;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = max(m, partial[i]);
  m = warp_max_key(m, 32);
  __shared__ unsigned red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned b = 0u;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = max(b, red[w]);
    *out = b;
  }
}

// Device address of g_noalloc_amax on the current device, looked up once per device with
// that device current (a host-side reference to the array itself is not a device address).
int noalloc_scratch(unsigned** out) {
  static std::mutex mu;
  static unsigned* cached[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "input_to_float8 (no-alloc): cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(TO_EUNSUPPORTED, "input_to_float8 (no-alloc): device %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_amax);
    if (e != cudaSuccess) return cuda_fail(e, "input_to_float8 (no-alloc): cudaGetSymbolAddress");
    cached[dev] = static_cast<unsigned*>(p);
  }
  *out = cached[dev];
  return TO_OK;
}

template <typename T>
int launch_tensor_quant_fp8_noalloc(const void* x, int64_t n, void* q, float* dq_scale,
                                    unsigned* scratch, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int nparts = (int)ceil_div(n, kNoAllocChunk);
  const bool vec = aligned16(x) && aligned_to(q, V);
  if (vec)
    k_absmax_chunks<T, V><<<nparts, kThreads, 0, st>>>((const T*)x, n, scratch);
  else
    k_absmax_chunks<T, 1><<<nparts, kThreads, 0, st>>>((const T*)x, n, scratch);
  int rc = check_launch("input_to_float8 (no-alloc): partial amax");
  if (rc) return rc;
  unsigned* amax = scratch + kNoAllocSlots;
  k_absmax_final<<<1, 1024, 0, st>>>(scratch, nparts, amax);
  rc = check_launch("input_to_float8 (no-alloc): final amax");
  if (rc) return rc;
  const unsigned grid = grid_for(ceil_div(n, V), kThreads, 8);
  if (vec)
    k_tensor_quant<T, kQE4M3, V><<<grid, kThreads, 0, st>>>((const T*)x, n, amax, (uint8_t*)q,
                                                           dq_scale);
  else
    k_tensor_quant<T, kQE4M3, 1><<<grid, kThreads, 0, st>>>((const T*)x, n, amax, (uint8_t*)q,
                                                           dq_scale);
  return check_launch("input_to_float8 (no-alloc): quantize");
}

}  // namespace
}  // namespace tob

using namespace tob;

extern "C" {

int to_quant_per_tensor_i8(const void* x, int x_dtype, const float* scale, int8_t* q, int64_t n,
                           void* stream) {
  if (n < 0) return fail(TO_EINVAL, "quantize_per_tensor: negative size");
  if (n == 0) return TO_OK;
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_quant_sym<T>(x, scale, q, n, 1, 1, (cudaStream_t)stream));
  return TO_OK;
}

int to_dequant_per_tensor_i8(const int8_t* q, const float* scale, void* y, int y_dtype, int64_t n,
                             void* stream) {
  if (n < 0) return fail(TO_EINVAL, "dequantize_per_tensor: negative size");
  if (n == 0) return TO_OK;
  TOB_DISPATCH_FLOAT(y_dtype, T,
                     return launch_dequant_sym<T>(q, scale, y, n, 1, 1, (cudaStream_t)stream));
  return TO_OK;
}

int to_quant_per_channel_i8(const void* x, int x_dtype, const float* scale, int8_t* q,
                            int64_t outer, int64_t channels, int64_t inner, void* stream) {
  if (outer < 0 || channels <= 0 || inner < 0)
    return fail(TO_EINVAL, "quantize_per_channel: invalid view [%lld,%lld,%lld]",
                (long long)outer, (long long)channels, (long long)inner);
  const int64_t n = outer * channels * inner;
  if (n == 0) return TO_OK;
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_quant_sym<T>(x, scale, q, n, channels, inner,
                                                (cudaStream_t)stream));
  return TO_OK;
}

int to_dequant_per_channel_i8(const int8_t* q, const float* scale, void* y, int y_dtype,
                              int64_t outer, int64_t channels, int64_t inner, void* stream) {
  if (outer < 0 || channels <= 0 || inner < 0)
    return fail(TO_EINVAL, "dequantize_per_channel: invalid view [%lld,%lld,%lld]",
                (long long)outer, (long long)channels, (long long)inner);
  const int64_t n = outer * channels * inner;
  if (n == 0) return TO_OK;
  TOB_DISPATCH_FLOAT(y_dtype, T,
                     return launch_dequant_sym<T>(q, scale, y, n, channels, inner,
                                                  (cudaStream_t)stream));
  return TO_OK;
}

size_t to_input_quant_workspace_size(void) { return 256; }

int to_input_to_int8(const void* x, int x_dtype, int64_t n, int8_t* q, float* dq_scale,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (n <= 0) return fail(TO_EINVAL, "input_to_int8: empty input");
  if (!workspace || workspace_bytes < sizeof(unsigned))
    return fail(TO_ENOSPACE, "input_to_int8: workspace of %zu bytes is too small",
                workspace_bytes);
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_tensor_quant<T, kQI8>(x, n, q, dq_scale, (unsigned*)workspace,
                                                          (cudaStream_t)stream));
  return TO_OK;
}

int to_input_to_fp8(const void* x, int x_dtype, int64_t n, void* q, float* dq_scale,
                    void* workspace, size_t workspace_bytes, void* stream) {
  if (n <= 0) return fail(TO_EINVAL, "input_to_float8: empty input");
  if (!workspace || workspace_bytes < sizeof(unsigned))
    return fail(TO_ENOSPACE, "input_to_float8: workspace of %zu bytes is too small",
                workspace_bytes);
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_tensor_quant<T, kQE4M3>(x, n, q, dq_scale,
                                                           (unsigned*)workspace,
                                                           (cudaStream_t)stream));
  return TO_OK;
}

int to_input_to_fp8_fnuz(const void* x, int x_dtype, int64_t n, void* q, float* dq_scale,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (n <= 0) return fail(TO_EINVAL, "input_to_float8: empty input");
  if (!workspace || workspace_bytes < sizeof(unsigned))
    return fail(TO_ENOSPACE, "input_to_float8: workspace of %zu bytes is too small",
                workspace_bytes);
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_tensor_quant<T, kQE4M3Fnuz>(x, n, q, dq_scale,
                                                               (unsigned*)workspace,
                                                               (cudaStream_t)stream));
  return TO_OK;
}

int to_input_to_fp8_noalloc(const void* x, int x_dtype, int64_t n, void* q, float* dq_scale,
                            void* stream) {
  if (n <= 0) return fail(TO_EINVAL, "input_to_float8 (no-alloc): empty input");
  if (n > kNoAllocMaxElems)
    return fail(TO_EINVAL,
                "input_to_float8 (no-alloc): %lld elements exceed the built-in scratch limit of "
                "%lld; use to_input_to_fp8 with a caller workspace for larger tensors",
                (long long)n, (long long)kNoAllocMaxElems);
  unsigned* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_tensor_quant_fp8_noalloc<T>(x, n, q, dq_scale, scratch,
                                                               (cudaStream_t)stream));
  return TO_OK;
}

int to_per_token_group_quant_i8(const void* x, int x_dtype, int64_t n_groups, int64_t group_size,
                                float eps, int8_t* q, float* scales, void* stream) {
  if (n_groups < 0 || group_size <= 0 || group_size > (int64_t)1 << 30)
    return fail(TO_EINVAL, "per_token_group_quant_int8: invalid groups=%lld size=%lld",
                (long long)n_groups, (long long)group_size);
  if (n_groups == 0) return TO_OK;
  ScaleLayout sl{0, 1};
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_group_quant<T, kQI8>(x, n_groups, group_size, eps, 0, sl, q,
                                                         scales, (cudaStream_t)stream));
  return TO_OK;
}

namespace tob {
namespace {
int group_quant_fp8_entry(int kind, const void* x, int x_dtype, int64_t n_groups,
                          int64_t group_size, float eps, int ue8m0, int64_t cm_rows,
                          int64_t cm_groups, void* q, float* scales, cudaStream_t st) {
  if (n_groups < 0 || group_size <= 0 || group_size > (int64_t)1 << 30)
    return fail(TO_EINVAL, "per_token_group_quant_fp8: invalid groups=%lld size=%lld",
                (long long)n_groups, (long long)group_size);
  if (cm_rows > 0 && (cm_groups <= 0 || n_groups % (cm_rows * cm_groups) != 0))
    return fail(TO_EINVAL, "per_token_group_quant_fp8: column-major layout %lld x %lld does not "
                "tile %lld groups", (long long)cm_rows, (long long)cm_groups, (long long)n_groups);
  if (n_groups == 0) return TO_OK;
  ScaleLayout sl{cm_rows, cm_groups > 0 ? cm_groups : 1};
  if (kind == kQE4M3Fnuz) {
    TOB_DISPATCH_FLOAT(x_dtype, T,
                       return launch_group_quant<T, kQE4M3Fnuz>(x, n_groups, group_size, eps,
                                                                ue8m0, sl, q, scales, st));
  } else {
    TOB_DISPATCH_FLOAT(x_dtype, T,
                       return launch_group_quant<T, kQE4M3>(x, n_groups, group_size, eps, ue8m0,
                                                            sl, q, scales, st));
  }
  return TO_OK;
}
}  // namespace
}  // namespace tob

int to_per_token_group_quant_fp8(const void* x, int x_dtype, int64_t n_groups, int64_t group_size,
                                 float eps, int ue8m0, int64_t cm_rows, int64_t cm_groups, void* q,
                                 float* scales, void* stream) {
  return group_quant_fp8_entry(kQE4M3, x, x_dtype, n_groups, group_size, eps, ue8m0, cm_rows,
                               cm_groups, q, scales, (cudaStream_t)stream);
}

int to_per_token_group_quant_fp8_tma(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                     int64_t group_size, float eps, int ue8m0, void* q,
                                     float* scales, int64_t scales_ld, void* stream) {
  if (rows < 0 || cols < 0 || group_size <= 0 || cols % group_size != 0 ||
      scales_ld < ((rows + 3) / 4) * 4)
    return fail(TO_EINVAL, "per_token_group_quant_fp8: TMA-aligned scales need cols %% group == 0 "
                "and a leading dimension >= rows rounded up to 4 (rows=%lld cols=%lld group=%lld "
                "ld=%lld)", (long long)rows, (long long)cols, (long long)group_size,
                (long long)scales_ld);
  if (rows == 0 || cols == 0) return TO_OK;
  ScaleLayout sl{0, cols / group_size, scales_ld};
  TOB_DISPATCH_FLOAT(x_dtype, T,
                     return launch_group_quant<T, kQE4M3>(x, rows * (cols / group_size),
                                                          group_size, eps, ue8m0, sl, q, scales,
                                                          (cudaStream_t)stream));
  return TO_OK;
}

int to_per_token_group_quant_fp8_fnuz(const void* x, int x_dtype, int64_t n_groups,
                                      int64_t group_size, float eps, int ue8m0, int64_t cm_rows,
                                      int64_t cm_groups, void* q, float* scales, void* stream) {
  return group_quant_fp8_entry(kQE4M3Fnuz, x, x_dtype, n_groups, group_size, eps, ue8m0, cm_rows,
                               cm_groups, q, scales, (cudaStream_t)stream);
}

int to_act_and_mul_group_quant(const void* a, const void* b, int dtype, int64_t rows,
                               int64_t cols, int64_t lda, int64_t ldb, int act,
                               int64_t group_size, float eps, int ue8m0, int column_major,
                               int q_dtype, void* q, float* scales, void* stream) {
  if (rows < 0 || cols < 0 || group_size <= 0 || group_size > (int64_t)1 << 30 ||
      (cols % group_size) != 0 || (rows > 1 && (lda < cols || ldb < cols)))
    return fail(TO_EINVAL,
                "act_and_mul_group_quant: invalid shape rows=%lld cols=%lld group=%lld "
                "strides=(%lld, %lld)", (long long)rows, (long long)cols, (long long)group_size,
                (long long)lda, (long long)ldb);
  if (act != kSilu && act != kGeluTanh)
    return fail(TO_EINVAL, "act_and_mul_group_quant: unknown activation %d", act);
  if (q_dtype != TO_E4M3 && q_dtype != TO_I8)
    return fail(TO_EUNSUPPORTED, "act_and_mul_group_quant: codes %s (float8_e4m3fn or int8)",
                dtype_name(q_dtype));
  if (q_dtype == TO_I8 && (ue8m0 || column_major))
    return fail(TO_EINVAL, "act_and_mul_group_quant: ue8m0 / column-major scales are FP8 options");
  if (rows == 0 || cols == 0) return TO_OK;
  if (!a || !b || !q || !scales) return fail(TO_EINVAL, "act_and_mul_group_quant: null pointer");
  ScaleLayout sl{column_major ? rows : 0, column_major ? cols / group_size : 1};
  cudaStream_t st = (cudaStream_t)stream;
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    if (q_dtype == TO_E4M3)
      return act == kSilu
                 ? launch_act_group_quant<T, kQE4M3, kSilu>(a, b, rows, cols, lda, ldb,
                                                            group_size, eps, ue8m0, sl, q,
                                                            scales, st)
                 : launch_act_group_quant<T, kQE4M3, kGeluTanh>(a, b, rows, cols, lda, ldb,
                                                                group_size, eps, ue8m0, sl, q,
                                                                scales, st);
    return act == kSilu
               ? launch_act_group_quant<T, kQI8, kSilu>(a, b, rows, cols, lda, ldb, group_size,
                                                        eps, 0, sl, q, scales, st)
               : launch_act_group_quant<T, kQI8, kGeluTanh>(a, b, rows, cols, lda, ldb,
                                                            group_size, eps, 0, sl, q, scales,
                                                            st);
  };
  switch (dtype) {
    case TO_F32: return run(0.0f);
    case TO_F16: return run(__half{});
    case TO_BF16: return run(__nv_bfloat16{});
  }
  return fail(TO_EUNSUPPORTED, "act_and_mul_group_quant: dtype %s", dtype_name(dtype));
}

int to_block_dequant_i8(const int8_t* q, const float* s, float* y, int64_t n, int64_t k,
                        int64_t block_n, int64_t block_k, void* stream) {
  return launch_block_dequant(kQI8, q, s, y, n, k, block_n, block_k, (cudaStream_t)stream);
}

int to_block_dequant_fp8(const void* q, const float* s, float* y, int64_t n, int64_t k,
                         int64_t block_n, int64_t block_k, void* stream) {
  return launch_block_dequant(kQE4M3, q, s, y, n, k, block_n, block_k, (cudaStream_t)stream);
}

int to_block_dequant_fp8_fnuz(const void* q, const float* s, float* y, int64_t n, int64_t k,
                              int64_t block_n, int64_t block_k, void* stream) {
  return launch_block_dequant(kQE4M3Fnuz, q, s, y, n, k, block_n, block_k, (cudaStream_t)stream);
}

}  // extern "C"
