// Generic block-scaled W8A8 GEMM for INT8 and FP8 e4m3 operands, any M/N/K and any
// block_size (tileops/quant_int8.py:180, tileops/quant_fp8.py:188).
//
//   C[m,n] = sum_kb ( sum_{k in kb} A[m,k] * B[n,k] ) * a_s[m,kb] * b_s[n/bn,kb]
//
// The inner sums are exact (int32 for INT8 via dp4a; fp32 for e4m3 whose products are
// exact in fp32), one k-block at a time, then scaled and accumulated in fp32. This is the
// path for small or ragged shapes (the reference tests use M=6, N=10, K=24, block [4,8]);
// the tcgen05 kernels take the large per-token / per-channel shapes.
#include "common.cuh"

namespace tob {
namespace {

constexpr int kTM = 64, kTN = 64, kTK = 32;
constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ void store_out(void* c, int64_t idx, float v, const void* bias,
                                          int64_t n) {
  T r = from_f32<T>(v);
  if (bias) r = from_f32<T>(to_f32(r) + to_f32(reinterpret_cast<const T*>(bias)[n]));
  reinterpret_cast<T*>(c)[idx] = r;
}

template <bool FP8, typename TC>
__global__ void __launch_bounds__(kThreads) k_w8a8_generic(
    const uint8_t* __restrict__ a, const uint8_t* __restrict__ b, const float* __restrict__ a_s,
    const float* __restrict__ b_s, void* __restrict__ c, const void* __restrict__ bias,
    int32_t* __restrict__ acc_out, int M, int N, int K, int bn, int bk) {
  __shared__ __align__(16) uint8_t As[kTM][kTK + 4];
  __shared__ __align__(16) uint8_t Bs[kTN][kTK + 4];
  const int tm = threadIdx.x / 16, tn = threadIdx.x % 16;  // 16 x 16 threads, 4 x 4 outputs each
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
  const int k_tiles = (K + bk - 1) / bk;

  float accf[4][4] = {};
  int32_t acci_total[4][4] = {};

  for (int kb = 0; kb < k_tiles; ++kb) {
    const int kbeg = kb * bk, kend = min(K, kbeg + bk);
    int32_t pi[4][4] = {};
    float pf[4][4] = {};
    for (int k0 = kbeg; k0 < kend; k0 += kTK) {
      const int kt = min(kTK, kend - k0);
      __syncthreads();
      for (int i = threadIdx.x; i < kTM * kTK; i += kThreads) {
        const int r = i / kTK, kk = i % kTK;
        const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
        As[r][kk] = (gm < M && kk < kt) ? a[(int64_t)gm * K + gk] : 0;
        Bs[r][kk] = (gn < N && kk < kt) ? b[(int64_t)gn * K + gk] : 0;
      }
      __syncthreads();
      if (!FP8) {
#pragma unroll
        for (int kk = 0; kk < kTK; kk += 4) {
          int av[4], bv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) av[i] = *reinterpret_cast<const int*>(&As[tm + 16 * i][kk]);
#pragma unroll
          for (int j = 0; j < 4; ++j) bv[j] = *reinterpret_cast<const int*>(&Bs[tn + 16 * j][kk]);
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) pi[i][j] = __dp4a(av[i], bv[j], pi[i][j]);
        }
      } else {
        for (int kk = 0; kk < kt; ++kk) {
          float av[4], bv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) av[i] = e4m3_to_f32(As[tm + 16 * i][kk]);
#pragma unroll
          for (int j = 0; j < 4; ++j) bv[j] = e4m3_to_f32(Bs[tn + 16 * j][kk]);
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) pf[i][j] = fmaf(av[i], bv[j], pf[i][j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gm = m0 + tm + 16 * i;
      const float sa = gm < M ? __ldg(a_s + (int64_t)gm * k_tiles + kb) : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int gn = n0 + tn + 16 * j;
        const float sb = gn < N ? __ldg(b_s + (int64_t)(gn / bn) * k_tiles + kb) : 0.f;
        const float part = FP8 ? pf[i][j] : (float)pi[i][j];
        accf[i][j] = fmaf(part, sa * sb, accf[i][j]);
        if (!FP8) acci_total[i][j] += pi[i][j];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + tm + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tn + 16 * j;
      if (gn >= N) continue;
      const int64_t idx = (int64_t)gm * N + gn;
      store_out<TC>(c, idx, accf[i][j], bias, gn);
      if (!FP8 && acc_out) acc_out[idx] = acci_total[i][j];
    }
  }
}

// Dense C[M, N] = A[M, K] @ B[K, N] (row-major, T = fp32, fp16 or bf16; fp32 accumulation, C
// rounded once) for the shapes the tcgen05 tiles do not take (N % 64, K % 8, unaligned rows,
// fp32; tileops/blas/gemm.py:31). 64 x 64 output tiles, 16 x 16 threads of 4 x 4 outputs, K in
// steps of 32 through shared memory; every product in fp32 with fmaf in increasing k.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_gemm_dense_simt(const T* __restrict__ a,
                                                             const T* __restrict__ b,
                                                             T* __restrict__ c, int M, int N,
                                                             int K) {
  __shared__ float As[kTK][kTM + 4];  // transposed: As[k][m]
  __shared__ float Bs[kTK][kTN + 4];  // Bs[k][n]
  const int tm = threadIdx.x / 16, tn = threadIdx.x % 16;
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kTK) {
    __syncthreads();
    for (int i = threadIdx.x; i < kTM * kTK; i += kThreads) {
      const int r = i / kTK, kk = i % kTK;  // A: consecutive threads along k of one row
      const int gm = m0 + r, gk = k0 + kk;
      As[kk][r] = (gm < M && gk < K) ? to_f32(a[(int64_t)gm * K + gk]) : 0.f;
    }
    for (int i = threadIdx.x; i < kTK * kTN; i += kThreads) {
      const int kk = i / kTN, cc = i % kTN;  // B: consecutive threads along n of one row
      const int gk = k0 + kk, gn = n0 + cc;
      Bs[kk][cc] = (gk < K && gn < N) ? to_f32(b[(int64_t)gk * N + gn]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kTK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][tm + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tn + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + tm + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tn + 16 * j;
      if (gn < N) c[(int64_t)gm * N + gn] = from_f32<T>(acc[i][j]);
    }
  }
}

}  // namespace

int gemm_dense_simt_launch(const void* a, const void* b, void* c, int dtype, int64_t M, int64_t N,
                           int64_t K, cudaStream_t st) {
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2)
    return fail(TO_EUNSUPPORTED, "gemm: dimensions too large");
  dim3 grid((unsigned)ceil_div(N, kTN), (unsigned)ceil_div(M, kTM));
  if (grid.y > 65535) return fail(TO_EUNSUPPORTED, "gemm: M too large for the SIMT tiles");
  TOB_DISPATCH_FLOAT(dtype, T, {
    k_gemm_dense_simt<T><<<grid, kThreads, 0, st>>>((const T*)a, (const T*)b, (T*)c, (int)M,
                                                     (int)N, (int)K);
  });
  return check_launch("gemm (SIMT tiles)");
}

int w8a8_generic_launch(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                        void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M,
                        int64_t N, int64_t K, int64_t bn, int64_t bk, cudaStream_t st) {
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2)
    return fail(TO_EUNSUPPORTED, "w8a8 generic: dimensions too large");
  dim3 grid((unsigned)ceil_div(N, kTN), (unsigned)ceil_div(M, kTM));
  TOB_DISPATCH_FLOAT(c_dtype, TC, {
    if (fp8)
      k_w8a8_generic<true, TC><<<grid, kThreads, 0, st>>>(
          (const uint8_t*)a, (const uint8_t*)b, a_s, b_s, c, bias, nullptr, (int)M, (int)N,
          (int)K, (int)bn, (int)bk);
    else
      k_w8a8_generic<false, TC><<<grid, kThreads, 0, st>>>(
          (const uint8_t*)a, (const uint8_t*)b, a_s, b_s, c, bias, acc_out, (int)M, (int)N,
          (int)K, (int)bn, (int)bk);
  });
  return check_launch(fp8 ? "w8a8_block_fp8_matmul (generic)" : "w8a8_block_int8_matmul (generic)");
}

}  // namespace tob
