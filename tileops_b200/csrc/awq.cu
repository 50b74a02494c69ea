// AWQ W4A16 kernels (tileops/quant_awq.py):
//   pack / unpack of the AWQ nibble order (quant_awq.py:41-65)
//   dequantisation (w - z) * s per K-group (quant_awq.py:68-109)
//   y = x @ dequant(W) for small M: a streaming GEMV (quant_awq.py:112-155)
//
// Packed layout (quant_awq.py:22): word c of a row holds logical columns 8c..8c+7 with
// column 8c+i in nibble ORDER[i], ORDER = (0,4,1,5,2,6,3,7). Equivalently nibble j holds
// column [0,2,4,6,1,3,5,7][j], so (word >> 4i) & 0x000F000F puts the adjacent column pair
// (2i, 2i+1) into the two 16-bit halves -- the operand of the magic-number int4 -> fp16/bf16
// conversion used below (one LOP3 per column pair).
#include <cooperative_groups.h>

#include <type_traits>

#include "awq_common.cuh"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace tob {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kTensorCoreMinM = 32;
__constant__ int kAwqOrder[8] = {0, 4, 1, 5, 2, 6, 3, 7};

// ------------------------------------------------------------------ pack / unpack
template <typename Tin>
__global__ void __launch_bounds__(kThreads) k_awq_pack(const Tin* __restrict__ in,
                                                      uint32_t* __restrict__ out, int64_t words) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += stride) {
    const Tin* p = in + w * 8;
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) word |= ((uint32_t)p[i] & 0xFu) << (4 * kAwqOrder[i]);
    out[w] = word;
  }
}

template <typename Tin>
__global__ void __launch_bounds__(kThreads) k_awq_unpack(const Tin* __restrict__ in,
                                                        int64_t* __restrict__ out, int64_t words) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += stride) {
    const uint32_t word = (uint32_t)in[w];
    longlong2* o = reinterpret_cast<longlong2*>(out + w * 8);
#pragma unroll
    for (int i = 0; i < 8; i += 2)
      o[i / 2] = make_longlong2((word >> (4 * kAwqOrder[i])) & 0xF,
                                (word >> (4 * kAwqOrder[i + 1])) & 0xF);
  }
}

// ------------------------------------------------------------------ dequant
// out[k, 8c+i] = T(float(w - z) * s): the subtraction is exact and the product is rounded
// once to T, exactly as the reference evaluates (weights - z_rows) * s_rows in scales.dtype.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_awq_dequant(const uint32_t* __restrict__ qw,
                                                         const T* __restrict__ scales,
                                                         const uint32_t* __restrict__ qz,
                                                         T* __restrict__ out, int64_t K,
                                                         int64_t words_per_row, int64_t G) {
  const int64_t total = K * words_per_row;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total; w += stride) {
    const int64_t k = w / words_per_row;
    const int64_t c = w - k * words_per_row;
    const int64_t g = k / G;
    const uint32_t word = __ldg(qw + w);
    const uint32_t zw = __ldg(qz + g * words_per_row + c);
    const T* s = scales + g * words_per_row * 8 + c * 8;
    Pack<T, 8> o;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int sh = 4 * kAwqOrder[i];
      const int d = (int)((word >> sh) & 0xF) - (int)((zw >> sh) & 0xF);
      o.v[i] = from_f32<T>(__fmul_rn((float)d, to_f32(s[i])));
    }
    *reinterpret_cast<Pack<T, 8>*>(out + w * 8) = o;
  }
}

// ------------------------------------------------------------------ streaming GEMV
// y[m, n] = sum_k x[m,k] * (w[k,n] - z[g,n]) * s[g,n] for M <= 4.
//
// Work split: a CTA owns a column tile of CW packed words (8*CW columns) and a K-chunk; the
// K-chunks of one column tile form a thread-block cluster and are reduced through
// distributed shared memory into cluster rank 0 (deterministic order, no global scratch).
// Inside a CTA, each thread streams WPL consecutive words of RUN consecutive rows; the lanes
// of a row cover CW words so every warp load touches whole 128-byte lines.
//
// Arithmetic: (w - z) is formed exactly in half2 / bfloat162 with the magic-bias trick
// (one LOP3 per column pair) and multiplied by the group scale in the model dtype, which is
// exactly the reference's dequantised weight T((w - z) * s) (quant_awq.py:109). It is then
// multiplied by x and accumulated in fp32 with sm_100's mixed-precision
// fma.rn.f32.{f16,bf16} (exact products, fp32 sums, no conversions).
constexpr int kRun = 16;

// acc0 += lo(d2) * x, acc1 += hi(d2) * x with exact products and one fp32 rounding each.
template <typename T>
__device__ __forceinline__ void fma_pair_mixed(uint32_t d2, uint16_t x, float& a0, float& a1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "fma.rn.f32.f16 %0, lo, %3, %0;\n\tfma.rn.f32.f16 %1, hi, %3, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(d2), "h"(x));
  } else {
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "fma.rn.f32.bf16 %0, lo, %3, %0;\n\tfma.rn.f32.bf16 %1, hi, %3, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(d2), "h"(x));
  }
}

template <typename T, int MT, int WPL, int CW>
__global__ void __launch_bounds__(kThreads) k_awq_gemv(const T* __restrict__ x,
                                                      const uint32_t* __restrict__ qw,
                                                      const T* __restrict__ scales,
                                                      const uint32_t* __restrict__ qz,
                                                      T* __restrict__ y, int M, int K, int N,
                                                      int G, int kchunk, int ksplit) {
  using H = Half2Of<T>;
  using H2 = typename H::type;
  constexpr int LPR = CW / WPL;      // lanes per row
  constexpr int RPW = 32 / LPR;      // rows a warp covers per load
  constexpr int NSLOT = (kThreads / 32) * RPW;
  constexpr int COLS = WPL * 8;      // columns per thread

  extern __shared__ __align__(16) unsigned char smem_raw[];
  // x chunk [MT][kchunk] in T, then the partial sums [MT][CW*8] fp32.
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);
  float* part = reinterpret_cast<float*>(smem_raw + (((size_t)MT * kchunk * sizeof(T) + 15) & ~(size_t)15));

  const int words_per_row = N >> 3;
  const int col_word0 = blockIdx.x * CW;
  const int kz = blockIdx.y;  // K-chunk index == cluster rank along y
  const int kb = kz * kchunk;
  const int ke = min(K, kb + kchunk);
  const int m0 = blockIdx.z * MT;

  const uint16_t* x16 = reinterpret_cast<const uint16_t*>(x);
  for (int i = threadIdx.x; i < MT * kchunk; i += kThreads) {
    const int m = i / kchunk, k = i - m * kchunk;
    xs[i] = (m0 + m < M && kb + k < K) ? x16[(int64_t)(m0 + m) * K + kb + k] : (uint16_t)0;
  }
  for (int i = threadIdx.x; i < MT * CW * 8; i += kThreads) part[i] = 0.f;
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lr = lane / LPR, lw = lane - lr * LPR;
  const int slot = warp * RPW + lr;
  const int word0 = col_word0 + lw * WPL;
  const bool col_ok = word0 < words_per_row;

  float acc[MT][COLS];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < COLS; ++c) acc[m][c] = 0.f;

  if (col_ok) {
    for (int r0 = kb + slot * kRun; r0 < ke; r0 += NSLOT * kRun) {
      const int g = r0 / G;
      // Issue every load of the run first: RUN x WPL words in flight per thread.
      uint32_t wv[kRun][WPL];
#pragma unroll
      for (int i = 0; i < kRun; ++i) {
        const int row = r0 + i;
        const uint32_t* p = qw + (int64_t)row * words_per_row + word0;
        if (row < ke) {
          if constexpr (WPL == 4) {
            uint4 v = ld_stream_v4(p);
            wv[i][0] = v.x; wv[i][1] = v.y; wv[i][2] = v.z; wv[i][3] = v.w;
          } else if constexpr (WPL == 2) {
            uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
            wv[i][0] = v.x; wv[i][1] = v.y;
          } else {
            wv[i][0] = __ldg(p);
          }
        } else {
#pragma unroll
          for (int j = 0; j < WPL; ++j) wv[i][j] = 0;  // x is zero there
        }
      }
      H2 zc[WPL][4], sc[WPL][4];
      const H2* s2 = reinterpret_cast<const H2*>(scales + (int64_t)g * N + (int64_t)word0 * 8);
#pragma unroll
      for (int j = 0; j < WPL; ++j) {
        awq_zero_consts<T>(__ldg(qz + (int64_t)g * words_per_row + word0 + j), zc[j]);
#pragma unroll
        for (int q = 0; q < 4; ++q) sc[j][q] = s2[j * 4 + q];
      }
      const int xo = r0 - kb;
#pragma unroll
      for (int i = 0; i < kRun; ++i) {
        uint16_t xv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) xv[m] = xs[m * kchunk + xo + i];
#pragma unroll
        for (int j = 0; j < WPL; ++j) {
          H2 d[4];
          awq_word_diff<T>(wv[i][j], zc[j], d);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const H2 w = __hmul2(d[q], sc[j][q]);  // the reference's dequantised weight pair
#pragma unroll
            for (int m = 0; m < MT; ++m)
              fma_pair_mixed<T>(bits_of(w), xv[m], acc[m][j * 8 + 2 * q], acc[m][j * 8 + 2 * q + 1]);
          }
        }
      }
    }
  }

  // Reduce over the RPW lane-rows of a warp (lanes that share word0), then over warps.
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < COLS; ++c) {
      float v = acc[m][c];
#pragma unroll
      for (int o = LPR; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[m][c] = v;
    }
  // Warps add into the CTA partial in a fixed order (deterministic).
  for (int w = 0; w < kThreads / 32; ++w) {
    if (warp == w && lr == 0) {
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int c = 0; c < COLS; ++c) part[m * CW * 8 + lw * COLS + c] += acc[m][c];
    }
    __syncthreads();
  }

  // Cluster reduction over the K-chunks of this column tile through distributed shared memory.
  if (ksplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (kz == 0) {
      for (int r = 1; r < ksplit; ++r) {
        const float* rp = cluster.map_shared_rank(part, r);
        for (int i = threadIdx.x; i < MT * CW * 8; i += kThreads) part[i] += rp[i];
      }
    }
    cluster.sync();  // keep every rank's shared memory alive until rank 0 has read it
  }
  if (kz == 0) {
    for (int i = threadIdx.x; i < MT * CW * 8; i += kThreads) {
      const int m = i / (CW * 8), c = i - m * (CW * 8);
      const int col = col_word0 * 8 + c;
      if (m0 + m < M && col < N) y[(int64_t)(m0 + m) * N + col] = from_f32<T>(part[i]);
    }
  }
}

template <typename T, int MT, int WPL, int CW>
int launch_gemv_cfg(const void* x, const int32_t* qw, const void* s, const int32_t* qz, void* y,
                    int64_t M, int64_t K, int64_t N, int64_t G, int ksplit, cudaStream_t st) {
  const int words = (int)(N / 8);
  const int tiles = (words + CW - 1) / CW;
  // Chunks start on multiples of kRun, so every run of rows lies inside one group.
  int kchunk = (int)ceil_div(ceil_div(K, ksplit), kRun) * kRun;
  const size_t smem = (((size_t)MT * kchunk * sizeof(T) + 15) & ~(size_t)15) +
                      (size_t)MT * CW * 8 * sizeof(float);
  auto kern = k_awq_gemv<T, MT, WPL, CW>;
  if (smem > 200 * 1024)
    return fail(TO_EUNSUPPORTED, "awq_gemm: K=%lld too long for the streaming kernel",
                (long long)K);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "awq_gemv: shared memory attribute");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, ksplit, (unsigned)ceil_div(M, MT));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = ksplit;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)x, (const uint32_t*)qw, (const T*)s,
                                     (const uint32_t*)qz, (T*)y, (int)M, (int)K, (int)N, (int)G,
                                     kchunk, ksplit);
  if (e != cudaSuccess) return cuda_fail(e, "awq_gemv launch");
  return check_launch("awq_gemv");
}

// Picks the column tile and the cluster split so that about two CTAs land on every SM.
template <typename T, int MT>
int launch_gemv(const void* x, const int32_t* qw, const void* s, const int32_t* qz, void* y,
                int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st) {
  const int64_t words = N / 8;
  const int64_t sms = sm_count();
  const bool v4 = (words % 4 == 0) && aligned16(qw);
  const bool wide = words >= 32;
  const int cw = wide ? 32 : 16;
  const int64_t tiles = ceil_div(words, cw);
  int ksplit = 1;
  const int64_t rows_per_run_slot = kRun;
  while (ksplit < 8 && tiles * ksplit * 2 <= 2 * sms &&
         K / (ksplit * 2) >= rows_per_run_slot * 8)
    ksplit *= 2;
  // Registers grow with MT x columns per thread: 16 columns per thread up to MT = 2, 8 beyond.
  (void)v4;
  if constexpr (MT <= 2) {
    if ((words % 2 == 0) && ((uintptr_t)qw % 8 == 0)) {
      if (wide) return launch_gemv_cfg<T, MT, 2, 32>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
      return launch_gemv_cfg<T, MT, 2, 16>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
    }
  }
  if (wide) return launch_gemv_cfg<T, MT, 1, 32>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
  return launch_gemv_cfg<T, MT, 1, 16>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
}

template <typename T>
int launch_gemv_any_m(const void* x, const int32_t* qw, const void* s, const int32_t* qz, void* y,
                      int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st) {
  switch (M) {
    case 1: return launch_gemv<T, 1>(x, qw, s, qz, y, M, K, N, G, st);
    case 2: return launch_gemv<T, 2>(x, qw, s, qz, y, M, K, N, G, st);
    case 3: return launch_gemv<T, 3>(x, qw, s, qz, y, M, K, N, G, st);
    default: return launch_gemv<T, 4>(x, qw, s, qz, y, M, K, N, G, st);  // grid.z covers M / 4
  }
}

int check_awq_shapes(const char* op, int64_t K, int64_t N, int64_t G) {
  if (K <= 0 || N <= 0 || N % 8 != 0)
    return fail(TO_EINVAL, "%s: invalid shape K=%lld N=%lld", op, (long long)K, (long long)N);
  if (G <= 0 || K % G != 0)
    return fail(TO_EINVAL, "%s: group size %lld does not divide K=%lld", op, (long long)G,
                (long long)K);
  return TO_OK;
}

}  // namespace

int awq_gemm_tc_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                       const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                       cudaStream_t st);

// Used by the tensor-core GEMM translation unit when it must stream small M.
int awq_gemv_dispatch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                      const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                      cudaStream_t st) {
  if (G % kRun != 0 && G != K)
    return fail(TO_EUNSUPPORTED, "awq_gemm: group size %lld is not a multiple of %d",
                (long long)G, kRun);
  if (K > (1 << 30) || N > (1 << 30))
    return fail(TO_EUNSUPPORTED, "awq_gemm: K or N too large");
  switch (s_dtype) {
    case TO_F16: return launch_gemv_any_m<__half>(x, qw, s, qz, y, M, K, N, G, st);
    case TO_BF16: return launch_gemv_any_m<__nv_bfloat16>(x, qw, s, qz, y, M, K, N, G, st);
    default:
      return fail(TO_EUNSUPPORTED, "awq_gemm: scales dtype %s is not supported (fp16, bf16)",
                  dtype_name(s_dtype));
  }
}

}  // namespace tob

using namespace tob;

extern "C" {

int to_awq_pack(const void* unpacked, int in_dtype, int32_t* packed, int64_t rows, int64_t cols8,
                void* stream) {
  if (rows < 0 || cols8 < 0) return fail(TO_EINVAL, "pack_awq_int4: negative shape");
  const int64_t words = rows * cols8;
  if (words == 0) return TO_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = grid_for(words, kThreads, 8);
  if (in_dtype == TO_I64)
    k_awq_pack<int64_t><<<grid, kThreads, 0, st>>>((const int64_t*)unpacked, (uint32_t*)packed, words);
  else if (in_dtype == TO_I32)
    k_awq_pack<int32_t><<<grid, kThreads, 0, st>>>((const int32_t*)unpacked, (uint32_t*)packed, words);
  else
    return fail(TO_EUNSUPPORTED, "pack_awq_int4: input dtype %s (expected int32/int64)",
                dtype_name(in_dtype));
  return check_launch("pack_awq_int4");
}

int to_awq_unpack(const void* packed, int in_dtype, int64_t* out, int64_t rows, int64_t cols8,
                  void* stream) {
  if (rows < 0 || cols8 < 0) return fail(TO_EINVAL, "unpack_awq_int4: negative shape");
  const int64_t words = rows * cols8;
  if (words == 0) return TO_OK;
  if (!aligned16(out)) return fail(TO_EINVAL, "unpack_awq_int4: output must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = grid_for(words, kThreads, 8);
  if (in_dtype == TO_I32)
    k_awq_unpack<int32_t><<<grid, kThreads, 0, st>>>((const int32_t*)packed, out, words);
  else if (in_dtype == TO_I64)
    k_awq_unpack<int64_t><<<grid, kThreads, 0, st>>>((const int64_t*)packed, out, words);
  else
    return fail(TO_EUNSUPPORTED, "unpack_awq_int4: expected int32 packed tensor, got %s",
                dtype_name(in_dtype));
  return check_launch("unpack_awq_int4");
}

int to_awq_dequant(const int32_t* qweight, const void* scales, int s_dtype, const int32_t* qzeros,
                   void* out, int64_t K, int64_t N, int64_t group_size, void* stream) {
  int rc = check_awq_shapes("awq_dequantize", K, N, group_size);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t words = K * (N / 8);
  const unsigned grid = grid_for(words, kThreads, 8);
  TOB_DISPATCH_FLOAT(s_dtype, T, {
    if ((uintptr_t)out % (8 * sizeof(T)) != 0)
      return fail(TO_EINVAL, "awq_dequantize: output must be %d-byte aligned", (int)(8 * sizeof(T)));
    k_awq_dequant<T><<<grid, kThreads, 0, st>>>((const uint32_t*)qweight, (const T*)scales,
                                                (const uint32_t*)qzeros, (T*)out, K, N / 8,
                                                group_size);
  });
  return check_launch("awq_dequantize");
}

size_t to_awq_gemm_workspace_size(int64_t M, int64_t K, int64_t N, int64_t group_size) {
  (void)M; (void)K; (void)N; (void)group_size;
  return 0;
}

int to_awq_gemm(const void* x, const int32_t* qweight, const void* scales, int s_dtype,
                const int32_t* qzeros, void* y, int64_t M, int64_t K, int64_t N,
                int64_t group_size, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace; (void)workspace_bytes;
  int rc = check_awq_shapes("awq_gemm", K, N, group_size);
  if (rc) return rc;
  if (M <= 0) return fail(TO_EINVAL, "awq_gemm: invalid M=%lld", (long long)M);
  if (!aligned16(scales) || !aligned16(x))
    return fail(TO_EINVAL, "awq_gemm: x and scales must be 16-byte aligned");
  // Prefill-sized M runs on the tensor cores; small M streams the weights once per 4 rows.
  if (M >= kTensorCoreMinM) {
    const int rc = awq_gemm_tc_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N,
                                      group_size, (cudaStream_t)stream);
    if (rc != TO_EUNSUPPORTED) return rc;
  }
  return awq_gemv_dispatch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size,
                           (cudaStream_t)stream);
}

}  // extern "C"
