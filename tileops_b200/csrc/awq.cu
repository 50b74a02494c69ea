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

#include <stdlib.h>

#include <type_traits>

#include "act.cuh"
#include "awq_common.cuh"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace tob {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kTensorCoreMinM = 33;
// Below the decode kernel's range (M <= 2 on layers of fewer than 1024 weight units) and on the
// shapes the tensor-core kernels reject, M <= 2 streams on CUDA cores (its cost grows with M);
// 3 <= M <= 64 runs the TMA-fed register-MMA kernel, whose cost is flat in M.
constexpr int64_t kStreamMaxM = 2;
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

template <typename T, int MT>
int launch_gemv_stream(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                       void* y, int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st);

// A/B switches for measurements: TOB_GEMV_GENERAL=1 routes M <= 4 to the general streaming
// kernel instead of the prefetching one; TOB_AWQ_SMALL_M=0 skips the TMA-fed small-M kernel.
bool gemv_stream_enabled() {
  static const bool on = tuning_env("TOB_GEMV_GENERAL") == nullptr;
  return on;
}
bool small_m_enabled() {
  static const bool on = [] {
    const char* v = tuning_env("TOB_AWQ_SMALL_M");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}
// Largest M routed to the register-MMA kernel (measurement override TOB_AWQ_SMALL_M_MAX).
int64_t small_m_max() {
  static const int64_t v = [] {
    const char* e = tuning_env("TOB_AWQ_SMALL_M_MAX");
    const int64_t w = e ? atoll(e) : 0;
    return (w >= 2 && w <= 64) ? w : 64;
  }();
  return v;
}

// 33 <= M <= 64: the tcgen05 kernel wins once its 128 x 256 tiles cover a third of the SMs
// (one M tile: N >= ~12.6K columns); below that the register-MMA kernel, which splits K over
// a cluster, keeps more SMs streaming.
bool tc_for_mid_m(int64_t M, int64_t N) {
  return M >= kTensorCoreMinM && ceil_div(M, 128) * ceil_div(N, 256) * 3 >= sm_count();
}

template <typename T>
int launch_gemv_any_m(const void* x, const int32_t* qw, const void* s, const int32_t* qz, void* y,
                      int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st) {
  if (M <= 4 && gemv_stream_enabled()) {
    int rc = TO_EUNSUPPORTED;
    switch (M) {
      case 1: rc = launch_gemv_stream<T, 1>(x, qw, s, qz, y, M, K, N, G, st); break;
      case 2: rc = launch_gemv_stream<T, 2>(x, qw, s, qz, y, M, K, N, G, st); break;
      case 3: rc = launch_gemv_stream<T, 3>(x, qw, s, qz, y, M, K, N, G, st); break;
      default: rc = launch_gemv_stream<T, 4>(x, qw, s, qz, y, M, K, N, G, st); break;
    }
    if (rc != TO_EUNSUPPORTED) return rc;
  }
  switch (M) {
    case 1: return launch_gemv<T, 1>(x, qw, s, qz, y, M, K, N, G, st);
    case 2: return launch_gemv<T, 2>(x, qw, s, qz, y, M, K, N, G, st);
    case 3: return launch_gemv<T, 3>(x, qw, s, qz, y, M, K, N, G, st);
    default: return launch_gemv<T, 4>(x, qw, s, qz, y, M, K, N, G, st);  // grid.z covers M / 4
  }
}

// ------------------------------------------------------------------ streaming GEMV, prefetching
// The same arithmetic as k_awq_gemv for M <= 4, organised so that the weight stream starts at
// the first instruction and never drains:
//   * a column tile is CW packed words (8*CW columns); each lane reads 2 words (8 bytes) of a
//     row, so a warp load covers RPL = 2*32/CW rows of whole 64- or 128-byte segments;
//   * a CTA owns a K-chunk of the tile; each of its 8 warps owns a contiguous run of rows,
//     walked in blocks of RB = RPL*LPT rows (inside one K-group), with the next block's weights,
//     zeros and scales in flight while the current block is multiplied (two register buffers);
//   * the first two blocks are requested before griddepcontrol.wait: with launch overlap on,
//     they stream while the previous kernel in the stream finishes (x and y are only touched
//     after the wait);
//   * warp sums -> CTA sums in shared memory (fixed order) -> cluster reduction over the
//     K-chunks through distributed shared memory into cluster rank 0 (deterministic).
// The end of both GEMV kernels: each thread holds acc[m][c] for its lane-row's 2 words
// (16 columns) of the CTA's CW-word tile. Sum over the lane-rows of a warp, then over the 8
// warps in a fixed order; with a K split, cluster rank r reduces column slice r over all ranks
// (fixed order) and stores it, so the remote loads and the stores are spread over the cluster.
template <typename T, int MT, int CW>
__device__ __forceinline__ void gemv_reduce_store(const float (&acc)[MT][16], float* part,
                                                  float* tot, T* __restrict__ y, int M, int N,
                                                  int ksplit) {
  constexpr int LPR = CW / 2;  // lanes per row
  constexpr int COLS = CW * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rl = lane / LPR, lw = lane - rl * LPR;
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      float v = acc[m][c];
#pragma unroll
      for (int o = LPR; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (rl == 0) part[(warp * MT + m) * COLS + lw * 16 + c] = v;
    }
  __syncthreads();
  for (int i = threadIdx.x; i < MT * COLS; i += kThreads) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += part[w * MT * COLS + i];
    tot[i] = s;
  }
  const int rows = min(M, MT);
  if (ksplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    // ceil(COLS / ksplit) columns per rank: the K split need not divide the tile (K = 3072
    // in 512-row chunks is a split of 6).
    const int per = (COLS + ksplit - 1) / ksplit;
    const int c0 = blockIdx.y * per;
    const int cn = min(per, COLS - c0);
    for (int i = threadIdx.x; i < rows * cn; i += kThreads) {
      const int m = i / cn, c = c0 + (i - m * cn);
      float v[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) v[r] = r < ksplit ? cluster.map_shared_rank(tot, r)[m * COLS + c] : 0.f;
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) s += v[r];
      const int col = blockIdx.x * COLS + c;
      if (col < N) y[(int64_t)m * N + col] = from_f32<T>(s);
    }
    cluster.sync();  // peers keep their shared memory until every slice has been read
  } else {
    __syncthreads();
    for (int i = threadIdx.x; i < rows * COLS; i += kThreads) {
      const int m = i / COLS, c = i - m * COLS;
      const int col = blockIdx.x * COLS + c;
      if (col < N) y[(int64_t)m * N + col] = from_f32<T>(tot[i]);
    }
  }
}

template <typename T, int CW, int LPT>
struct GemvBlock {
  uint2 w[LPT];
  uint2 z;
  uint4 s[2];
};

template <typename T, int MT, int CW, int LPT>
__global__ void __launch_bounds__(kThreads, 2)
k_awq_gemv_stream(const T* __restrict__ x, const uint32_t* __restrict__ qw,
                  const T* __restrict__ scales, const uint32_t* __restrict__ qz,
                  T* __restrict__ y, int M, int K, int N, int G, int kchunk, int ksplit) {
  using H = Half2Of<T>;
  using H2 = typename H::type;
  constexpr int WPL = 2;
  constexpr int LPR = CW / WPL;   // lanes per row
  constexpr int RPL = 32 / LPR;   // rows per warp load
  constexpr int RB = RPL * LPT;   // rows per block
  constexpr int COLS = CW * 8;    // columns per CTA
  using Blk = GemvBlock<T, CW, LPT>;

  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem_raw);  // [MT][kchunk]
  float* part = reinterpret_cast<float*>(smem_raw + (((size_t)MT * kchunk * 2 + 15) & ~(size_t)15));
  float* tot = part + 8 * MT * COLS;                      // [MT][COLS]

  const int words = N >> 3;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rl = lane / LPR, lw = lane - rl * LPR;
  const int word0 = blockIdx.x * CW + lw * WPL;
  const bool col_ok = word0 < words;
  const int kb = blockIdx.y * kchunk;
  const int rpw = kchunk >> 3;  // rows per warp, a multiple of RB
  const int wb = kb + warp * rpw;
  const int we = min(min(K, kb + kchunk), wb + rpw);
  const int nblk = we > wb ? (we - wb + RB - 1) / RB : 0;

  auto load = [&](Blk& b, int row0) {
#pragma unroll
    for (int i = 0; i < LPT; ++i) {
      const int row = row0 + rl + RPL * i;
      b.w[i] = (col_ok && row < K) ? ld_stream_v2(qw + (int64_t)row * words + word0)
                                   : make_uint2(0u, 0u);
    }
    const int g = row0 / G;
    if (col_ok) {
      b.z = __ldg(reinterpret_cast<const uint2*>(qz + (int64_t)g * words + word0));
      const uint4* sp = reinterpret_cast<const uint4*>(scales + (int64_t)g * N + (int64_t)word0 * 8);
      b.s[0] = __ldg(sp);
      b.s[1] = __ldg(sp + 1);
    } else {
      b.z = make_uint2(0u, 0u);
      b.s[0] = b.s[1] = make_uint4(0u, 0u, 0u, 0u);
    }
  };

  float acc[MT][WPL * 8];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < WPL * 8; ++c) acc[m][c] = 0.f;

  auto compute = [&](const Blk& b, int row0) {
    H2 zc[WPL][4];
    awq_zero_consts<T>(b.z.x, zc[0]);
    awq_zero_consts<T>(b.z.y, zc[1]);
    const H2* sc = reinterpret_cast<const H2*>(&b.s[0]);  // sc[j*4 + q]: columns 8j+2q, +1
#pragma unroll
    for (int i = 0; i < LPT; ++i) {
      const int xo = row0 + rl + RPL * i - kb;
      uint16_t xv[MT];
#pragma unroll
      for (int m = 0; m < MT; ++m) xv[m] = xs[m * kchunk + xo];
      const uint32_t wv[WPL] = {b.w[i].x, b.w[i].y};
#pragma unroll
      for (int j = 0; j < WPL; ++j) {
        H2 d[4];
        awq_word_diff<T>(wv[j], zc[j], d);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const H2 wq = __hmul2(d[q], sc[j * 4 + q]);  // the reference's dequantised pair
#pragma unroll
          for (int m = 0; m < MT; ++m)
            fma_pair_mixed<T>(bits_of(wq), xv[m], acc[m][j * 8 + 2 * q], acc[m][j * 8 + 2 * q + 1]);
        }
      }
    }
  };

  Blk A, B;
  if (nblk > 0) load(A, wb);
  if (nblk > 1) load(B, wb + RB);

  // Everything above reads only the weights; x (and y below) may belong to the previous grid.
  grid_dependency_wait();
  const uint16_t* x16 = reinterpret_cast<const uint16_t*>(x);
  if ((K & 7) == 0) {
    const int vec = kchunk >> 3;
    for (int i = threadIdx.x; i < MT * vec; i += kThreads) {
      const int m = i / vec, k = (i - m * vec) * 8;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (m < M && kb + k < K) v = __ldg(reinterpret_cast<const uint4*>(x16 + (int64_t)m * K + kb + k));
      *reinterpret_cast<uint4*>(xs + m * kchunk + k) = v;
    }
  } else {
    for (int i = threadIdx.x; i < MT * kchunk; i += kThreads) {
      const int m = i / kchunk, k = i - m * kchunk;
      xs[i] = (m < M && kb + k < K) ? x16[(int64_t)m * K + kb + k] : (uint16_t)0;
    }
  }
  __syncthreads();
  grid_dependents_launch();

#pragma unroll 1
  for (int bi = 0; bi < nblk; bi += 2) {
    compute(A, wb + bi * RB);
    if (bi + 2 < nblk) load(A, wb + (bi + 2) * RB);
    if (bi + 1 < nblk) {
      compute(B, wb + (bi + 1) * RB);
      if (bi + 3 < nblk) load(B, wb + (bi + 3) * RB);
    }
  }

  gemv_reduce_store<T, MT, CW>(acc, part, tot, y, M, N, ksplit);
}

template <typename T, int MT, int CW, int LPT>
int launch_gemv_stream_cfg(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                           void* y, int64_t M, int64_t K, int64_t N, int64_t G, int ksplit,
                           cudaStream_t st) {
  constexpr int RB = (64 / CW) * LPT;
  const int words = (int)(N / 8);
  const int tiles = (words + CW - 1) / CW;
  const int per_cta = 8 * RB;
  const int kchunk = (int)(ceil_div(ceil_div(K, ksplit), per_cta) * per_cta);
  ksplit = (int)ceil_div(K, kchunk);
  const size_t smem = (((size_t)MT * kchunk * 2 + 15) & ~(size_t)15) +
                      (size_t)9 * MT * CW * 8 * sizeof(float);
  if (smem > 100 * 1024) return TO_EUNSUPPORTED;
  auto kern = k_awq_gemv_stream<T, MT, CW, LPT>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "awq_gemv: shared memory attribute");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, ksplit, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = 1;
  attr[na].val.clusterDim.y = ksplit;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (launch_overlap()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)x, (const uint32_t*)qw, (const T*)s,
                                     (const uint32_t*)qz, (T*)y, (int)M, (int)K, (int)N, (int)G,
                                     kchunk, ksplit);
  if (e != cudaSuccess) return cuda_fail(e, "awq_gemv launch");
  return check_launch("awq_gemv");
}

// M <= 4 with an even number of packed words per row and aligned rows; returns
// TO_EUNSUPPORTED (nothing launched) for shapes the general streaming kernel must take.
template <typename T, int MT>
int launch_gemv_stream(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                       void* y, int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st) {
  constexpr int LPT = MT <= 2 ? 8 : 4;
  const int64_t words = N / 8;
  if (words % 2 != 0 || (uintptr_t)qw % 8 != 0 || (uintptr_t)qz % 8 != 0 || !aligned16(s))
    return TO_EUNSUPPORTED;
  const int64_t sms = sm_count();
  // Wide tiles (128-byte row segments) when they still give two CTAs per SM at ksplit 8.
  const bool wide = ceil_div(words, 32) * 8 >= 2 * sms;
  const int cw = wide ? 32 : 16;
  const int rb = (64 / cw) * LPT;
  if (G % rb != 0 && G != K) return TO_EUNSUPPORTED;
  const int64_t tiles = ceil_div(words, cw);
  int ksplit = 1;
  while (ksplit < 8 && tiles * ksplit < 2 * sms && K >= (int64_t)ksplit * 2 * 8 * rb) ksplit *= 2;
  if (wide) return launch_gemv_stream_cfg<T, MT, 32, LPT>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
  return launch_gemv_stream_cfg<T, MT, 16, LPT>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
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
int awq_gemm_tc_gather_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                              const int32_t* qz, void* const* y_ranks, int world, int rank,
                              int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st);
int awq_small_m_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                       const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                       cudaStream_t st);
size_t awq_decode_workspace(int64_t M, int64_t K, int64_t N, int64_t G, int s_dtype);
bool awq_decode_wanted(int64_t M, int64_t K, int64_t N);
int awq_decode_gather_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                             const int32_t* qz, void* const* y_ranks, int world, int rank,
                             int64_t M, int64_t K, int64_t N, int64_t G, void* ws,
                             size_t ws_bytes, cudaStream_t st, int act = -1);
int awq_decode_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                      const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                      void* ws, size_t ws_bytes, cudaStream_t st, int act = -1,
                      int64_t ldx = 0);
int act_mul_interleaved_launch(const void* y, void* c, int dtype, int64_t rows, int64_t cols,
                               int64_t ldy, int64_t ldc, int act, cudaStream_t st);
size_t awq_sk_workspace(int64_t M, int64_t K, int64_t N, int64_t G, int s_dtype);
int awq_sk_launch(const void* x, const int32_t* qw, const void* s, int s_dtype, const int32_t* qz,
                  void* y, int64_t M, int64_t K, int64_t N, int64_t G, void* ws, size_t ws_bytes,
                  cudaStream_t st, int act);
int awq_sk_gather_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                         const int32_t* qz, void* const* y_ranks, int world, int rank, int64_t M,
                         int64_t K, int64_t N, int64_t G, void* ws, size_t ws_bytes,
                         cudaStream_t st, int act);

// Measurement switch: TOB_AWQ_DECODE=0 keeps decode-sized M off the stream-K decode kernel.
bool decode_enabled() {
  static const bool on = [] {
    const char* v = tuning_env("TOB_AWQ_DECODE");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

// Shapes the stream-K tensor-core kernel takes: 33-128 tokens on layers of long K (>= 8192)
// and few 256-column tiles (<= 32), where the tile GEMM leaves most SMs idle for the whole K and
// the register-MMA kernel runs out of token tiles. Measured on the 4096 x 14336 down projection:
// 57 us at M = 64 (register-MMA kernel 82 us) and 90 us at M = 128 (tile GEMM 131 us). On the
// other decode layers it is slower than both: each SM expands one 64 x 256 weight block per
// ~1.2 us, so its rate stays near 1.1 TB/s (below, the decode kernel's register-operand MMAs
// stream faster). Measurement switch TOB_AWQ_SK: "0" never, "all" for every M <= 128.
constexpr int64_t kSkMinM = 33, kSkMaxM = 128;
bool sk_wanted(int64_t M, int64_t K, int64_t N) {
  static const int mode = [] {
    const char* v = tuning_env("TOB_AWQ_SK");
    if (v == nullptr) return 1;
    return v[0] == '0' ? 0 : (v[0] == 'a' ? 2 : 1);
  }();
  if (mode == 0 || M > kSkMaxM) return false;
  if (mode == 2) return true;
  return M >= kSkMinM && K >= 8192 && ceil_div(N, 256) <= 32;
}

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
  if (M <= 0 || K <= 0 || N <= 0 || group_size <= 0 || N % 8 != 0 || K % group_size != 0)
    return 0;
  if (sk_wanted(M, K, N)) return awq_sk_workspace(M, K, N, group_size, TO_F16);
  if (!decode_enabled()) return 0;
  return awq_decode_workspace(M, K, N, group_size, TO_F16);
}

int to_awq_gemm(const void* x, const int32_t* qweight, const void* scales, int s_dtype,
                const int32_t* qzeros, void* y, int64_t M, int64_t K, int64_t N,
                int64_t group_size, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_awq_shapes("awq_gemm", K, N, group_size);
  if (rc) return rc;
  if (M <= 0) return fail(TO_EINVAL, "awq_gemm: invalid M=%lld", (long long)M);
  if (!aligned16(scales) || !aligned16(x))
    return fail(TO_EINVAL, "awq_gemm: x and scales must be 16-byte aligned");
  // Decode-sized M (1..32) runs on the stream-K decode kernel; prefill-sized M on the tcgen05
  // GEMM; 33 <= M <= 64 on the TMA-fed register-MMA kernel when the tcgen05 tiles would leave
  // most SMs idle; the shapes none of them takes (ragged N, unaligned rows) on the streaming
  // SIMT kernels.
  if (sk_wanted(M, K, N)) {
    rc = awq_sk_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size, workspace,
                       workspace_bytes, (cudaStream_t)stream, -1);
    if (rc != TO_EUNSUPPORTED) return rc;
  } else if (M <= 32 && decode_enabled() && awq_decode_wanted(M, K, N)) {
    rc = awq_decode_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size,
                           workspace, workspace_bytes, (cudaStream_t)stream);
    if (rc != TO_EUNSUPPORTED) return rc;
  }
  if (M > small_m_max() || tc_for_mid_m(M, N)) {
    const int rc = awq_gemm_tc_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N,
                                      group_size, (cudaStream_t)stream);
    if (rc != TO_EUNSUPPORTED) return rc;
  } else if (M > kStreamMaxM && small_m_enabled()) {
    int rc = awq_small_m_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size,
                                (cudaStream_t)stream);
    if (rc != TO_EUNSUPPORTED) return rc;
    if (M >= kTensorCoreMinM) {  // shapes the register-MMA kernel does not take
      rc = awq_gemm_tc_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size,
                              (cudaStream_t)stream);
      if (rc != TO_EUNSUPPORTED) return rc;
    }
  }
  return awq_gemv_dispatch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size,
                           (cudaStream_t)stream);
}

// The gate_up linear with its activation: the decode and stream-K kernels
// apply it in their epilogue, on the shapes to_awq_gemm routes to them; other shapes run
// to_awq_gemm into the front of the workspace ([M, N] in the scales' dtype, 256-byte aligned
// size) and the activation over it. Either way the result is to_awq_gemm's output on these
// weights, rounded, then the activation.
static size_t act_tmp_bytes(int64_t M, int64_t N) { return ((size_t)(M * N * 2) + 255) & ~(size_t)255; }

size_t to_awq_gemm_act_workspace_size(int64_t M, int64_t K, int64_t N, int64_t group_size) {
  if (M <= 0 || K <= 0 || N <= 0 || group_size <= 0 || N % 16 != 0 || K % group_size != 0)
    return 0;
  return act_tmp_bytes(M, N) + to_awq_gemm_workspace_size(M, K, N, group_size);
}

int to_awq_gemm_act(const void* x, const int32_t* qweight, const void* scales, int s_dtype,
                    const int32_t* qzeros, void* y, int64_t M, int64_t K, int64_t N,
                    int64_t group_size, int act, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int rc = check_awq_shapes("awq_gemm_act", K, N, group_size);
  if (rc) return rc;
  if (M <= 0) return fail(TO_EINVAL, "awq_gemm_act: invalid M=%lld", (long long)M);
  if (act != kSilu && act != kGeluTanh)
    return fail(TO_EINVAL, "awq_gemm_act: unknown activation %d", act);
  if (N % 16 != 0)
    return fail(TO_EINVAL, "awq_gemm_act: N=%lld is not a multiple of 16 (gate and up blocks of 8)",
                (long long)N);
  if (s_dtype != TO_F16 && s_dtype != TO_BF16)
    return fail(TO_EUNSUPPORTED, "awq_gemm_act: scales dtype %s (fp16, bf16)", dtype_name(s_dtype));
  if (!aligned16(scales) || !aligned16(x) || !aligned16(y))
    return fail(TO_EINVAL, "awq_gemm_act: x, scales and y must be 16-byte aligned");
  const size_t need = to_awq_gemm_act_workspace_size(M, K, N, group_size);
  if (workspace_bytes < need || (need > 0 && (workspace == nullptr || !aligned16(workspace))))
    return fail(TO_ENOSPACE, "awq_gemm_act: workspace of %zu bytes, %zu needed (16-byte aligned)",
                workspace_bytes, need);
  cudaStream_t st = (cudaStream_t)stream;
  char* tmp = static_cast<char*>(workspace);
  char* gemm_ws = tmp + act_tmp_bytes(M, N);
  const size_t gemm_ws_bytes = workspace_bytes - act_tmp_bytes(M, N);
  if (sk_wanted(M, K, N)) {
    rc = awq_sk_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size, gemm_ws,
                       gemm_ws_bytes, st, act);
    if (rc != TO_EUNSUPPORTED) return rc;
  } else if (M > 2 && M <= 32 && decode_enabled()) {
    // 1-2 tokens keep the activation as its own launch: the layer after a gate_up of that size
    // streams on the GEMV, whose CTAs (small shared memory) start under programmatic dependent
    // launch while the tiny activation kernel runs, but not while the decode kernel's CTAs
    // (190 KB each) still hold the SMs -- measured on the 32-layer step at one token, 2.10 ms
    // fused against 1.81 ms separate.
    rc = awq_decode_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size, gemm_ws,
                           gemm_ws_bytes, st, act);
    if (rc != TO_EUNSUPPORTED) return rc;
  }
  rc = to_awq_gemm(x, qweight, scales, s_dtype, qzeros, tmp, M, K, N, group_size, gemm_ws,
                   gemm_ws_bytes, stream);
  if (rc) return rc;
  return act_mul_interleaved_launch(tmp, y, s_dtype, M, N, N, N / 2, act, st);
}

int to_awq_gemm_act_gather(const void* x, const int32_t* qweight, const void* scales,
                           int s_dtype, const int32_t* qzeros, void* const* y_ranks, int world,
                           int rank, int64_t M, int64_t K, int64_t N, int64_t group_size, int act,
                           void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_awq_shapes("awq_gemm_act_gather", K, N, group_size);
  if (rc) return rc;
  if (M <= 0) return fail(TO_EINVAL, "awq_gemm_act_gather: invalid M=%lld", (long long)M);
  if (act != kSilu && act != kGeluTanh)
    return fail(TO_EINVAL, "awq_gemm_act_gather: unknown activation %d", act);
  if (N % 16 != 0)
    return fail(TO_EINVAL, "awq_gemm_act_gather: N=%lld is not a multiple of 16", (long long)N);
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(TO_EINVAL, "awq_gemm_act_gather: rank %d of %d (1 to 8 ranks)", rank, world);
  if (!y_ranks) return fail(TO_EINVAL, "awq_gemm_act_gather: null output table");
  for (int r = 0; r < world; ++r)
    if (!y_ranks[r]) return fail(TO_EINVAL, "awq_gemm_act_gather: null output of rank %d", r);
  if (!aligned16(scales) || !aligned16(x))
    return fail(TO_EINVAL, "awq_gemm_act_gather: x and scales must be 16-byte aligned");
  rc = TO_EUNSUPPORTED;
  if (sk_wanted(M, K, N))
    rc = awq_sk_gather_launch(x, qweight, scales, s_dtype, qzeros, y_ranks, world, rank, M, K, N,
                              group_size, workspace, workspace_bytes, (cudaStream_t)stream, act);
  else if (M <= 32 && decode_enabled())
    rc = awq_decode_gather_launch(x, qweight, scales, s_dtype, qzeros, y_ranks, world, rank, M,
                                  K, N, group_size, workspace, workspace_bytes,
                                  (cudaStream_t)stream, act);
  if (rc == TO_EUNSUPPORTED)
    return fail(TO_EUNSUPPORTED,
                "awq_gemm_act_gather: only the decode and stream-K kernels gather the activation; "
                "run to_awq_gemm_act and an all-gather instead");
  return rc;
}

int to_awq_gemm_strided(const void* x, int64_t ldx, const int32_t* qweight, const void* scales,
                        int s_dtype, const int32_t* qzeros, void* y, int64_t M, int64_t K,
                        int64_t N, int64_t group_size, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int rc = check_awq_shapes("awq_gemm", K, N, group_size);
  if (rc) return rc;
  if (M <= 0) return fail(TO_EINVAL, "awq_gemm: invalid M=%lld", (long long)M);
  if (ldx < K) return fail(TO_EINVAL, "awq_gemm: row stride %lld < K=%lld", (long long)ldx,
                           (long long)K);
  // The decode kernel reads x through its tensor map, which takes any 16-byte row stride;
  // shapes routed elsewhere need x contiguous.
  if (M <= 32 && !sk_wanted(M, K, N) && decode_enabled() && awq_decode_wanted(M, K, N)) {
    rc = awq_decode_launch(x, qweight, scales, s_dtype, qzeros, y, M, K, N, group_size, workspace,
                           workspace_bytes, (cudaStream_t)stream, -1, ldx);
    if (rc != TO_EUNSUPPORTED) return rc;
  }
  return TO_EUNSUPPORTED;
}

int to_awq_gemm_gather(const void* x, const int32_t* qweight, const void* scales, int s_dtype,
                       const int32_t* qzeros, void* const* y_ranks, int world, int rank,
                       int64_t M, int64_t K, int64_t N, int64_t group_size, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int rc = check_awq_shapes("awq_gemm_gather", K, N, group_size);
  if (rc) return rc;
  if (M <= 0) return fail(TO_EINVAL, "awq_gemm_gather: invalid M=%lld", (long long)M);
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(TO_EINVAL, "awq_gemm_gather: rank %d of %d (1 to 8 ranks)", rank, world);
  if (!y_ranks) return fail(TO_EINVAL, "awq_gemm_gather: null output table");
  for (int r = 0; r < world; ++r)
    if (!y_ranks[r]) return fail(TO_EINVAL, "awq_gemm_gather: null output of rank %d", r);
  if (!aligned16(scales) || !aligned16(x))
    return fail(TO_EINVAL, "awq_gemm_gather: x and scales must be 16-byte aligned");
  // Decode-sized M on the stream-K decode kernel, the rest on the tensor-core GEMM; both store
  // each finished tile into every rank's output.
  rc = TO_EUNSUPPORTED;
  if (sk_wanted(M, K, N))
    rc = awq_sk_gather_launch(x, qweight, scales, s_dtype, qzeros, y_ranks, world, rank, M, K, N,
                              group_size, workspace, workspace_bytes, (cudaStream_t)stream, -1);
  else if (M <= 32 && decode_enabled())
    rc = awq_decode_gather_launch(x, qweight, scales, s_dtype, qzeros, y_ranks, world, rank, M, K,
                                  N, group_size, workspace, workspace_bytes,
                                  (cudaStream_t)stream);
  if (rc == TO_EUNSUPPORTED)
    rc = awq_gemm_tc_gather_launch(x, qweight, scales, s_dtype, qzeros, y_ranks, world, rank, M,
                                   K, N, group_size, (cudaStream_t)stream);
  if (rc == TO_EUNSUPPORTED)
    return fail(TO_EUNSUPPORTED,
                "awq_gemm_gather: shapes outside the gathering kernels (N %% 32, K %% 8, group "
                "size, alignment); run the local GEMM and an all-gather instead");
  return rc;
}

}  // extern "C"
