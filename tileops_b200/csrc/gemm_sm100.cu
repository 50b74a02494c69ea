// Persistent warp-specialised tcgen05 GEMM for the W8A8 paths on sm_100a:
//   kind::i8      int8 x int8 -> s32 accumulators (exact), INT8 W8A8 (quant_int8.py:180)
//   kind::f8f6f4  e4m3 x e4m3 -> f32 accumulators,         FP8 W8A8  (quant_fp8.py:188)
// with the per-token x per-channel (or per-tensor) scale epilogue
//   C[m, n] = float(acc[m, n]) * (a_s[m] * b_s[n / bn])  (+ bias, rounded like the reference)
// and, for INT8, an optional copy of the raw int32 accumulators.
//
// Layout: A [M, K] and B [N, K] row-major ("K-major"), both streamed by TMA in 128-byte K
// slices with the 128-byte swizzle into a STAGES-deep shared-memory ring.
//
// CTA roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one thread)      full[s]  <- TMA bytes       empty[s] -> wait
//   warp 1      MMA issuer   (one thread)      empty[s] <- tcgen05.commit  tfull[b] <- commit
//   warps 2..5  epilogue: TMEM -> registers -> scales -> global, then arrive on tempty[b]
// Accumulators live in tensor memory, double-buffered when two fit in 512 columns, so the
// epilogue of tile i overlaps the main loop of tile i+1. A tile is BM x BN with BM = 128 or
// 256 (two M=128 MMAs sharing each B slice, for small-M layers that must spread N over all SMs).
//
// Every wait is bounded (sm100.cuh, kWaitLimitNs); on expiry the kernel records the error
// word, unwinds every role, waits (bounded) for its in-flight copies and MMAs, frees its TMEM
// and returns.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "sm100.cuh"

namespace tob {
namespace sm100 {

struct Epi {
  const float* a_s;  // per-row scale, element m at a_s[m * a_s_ld]
  int64_t a_s_ld;
  const float* b_s;  // per column-block scale, column n at b_s[(n / bn) * b_s_ld]
  int64_t b_s_ld;
  int64_t bn;
  void* c;           // [M, N] row-major
  int c_dtype;       // TO_F32 / TO_F16 / TO_BF16
  const void* bias;  // optional [N] in c_dtype, added after rounding to c_dtype
  int32_t* acc_out;  // optional [M, N] raw int32 accumulators (kind::i8 only)
  int policy_a;      // L2 policy for A loads: 0 normal, 1 evict_first, 2 evict_last
  int policy_b;
};

constexpr int kGemmThreads = 192;

__host__ __device__ constexpr int pow2_at_least(int v) {
  int p = 32;
  while (p < v) p <<= 1;
  return p;
}

template <Kind KD, int BM, int BN, int STAGES>
struct GemmCfg {
  static_assert(BM == 128 || BM == 256, "BM");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN");
  static constexpr int kElem = KindTraits<KD>::kElemBytes;
  static constexpr int kBK = 128 / kElem;  // K elements per stage = one 128-byte swizzle row
  static constexpr int kHalves = BM / 128;
  static constexpr int kABytes = BM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccCols = kHalves * BN;
  static constexpr int kAccBufs = (2 * kAccCols <= 512) ? 2 : 1;
  static constexpr int kTmemCols = pow2_at_least(kAccBufs * kAccCols);
  static constexpr size_t kBarrierBytes = 256;
  static constexpr size_t kSmem = 1024 + (size_t)STAGES * kStageBytes + kBarrierBytes;
  static_assert(kTmemCols <= 512, "TMEM");
  static_assert(kSmem <= 232448, "shared memory");
};

__device__ __forceinline__ uint64_t make_policy(int which) {
  if (which == 1) return policy_evict_first();
  if (which == 2) return policy_evict_last();
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

template <typename T>
__device__ __forceinline__ void store_row_chunk16(T* dst, const float* v, const T* bias,
                                                  int valid, bool vec_ok) {
  T o[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    T r = from_f32<T>(v[j]);
    if (bias != nullptr && j < valid) r = from_f32<T>(to_f32(r) + to_f32(bias[j]));
    o[j] = r;
  }
  if (vec_ok && valid == 16) {
    constexpr int kVec = 16 / sizeof(T);
#pragma unroll
    for (int j = 0; j < 16; j += kVec)
      *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(o + j);
  } else {
    for (int j = 0; j < valid; ++j) dst[j] = o[j];
  }
}

template <Kind KD, int BM, int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 int M, int N, int K, Epi ep, int* err) {
  using C = GemmCfg<KD, BM, BN, STAGES>;
  using Tr = KindTraits<KD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + (size_t)STAGES * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + (size_t)STAGES * C::kBBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int kblocks = (K + C::kBK - 1) / C::kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 0) tmem_alloc<C::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a = make_policy(ep.policy_a), pol_b = make_policy(ep.policy_b);
      uint32_t s = 0, ph = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int i = 0; i < STAGES; ++i) issued[i] = false, issued_phase[i] = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mt = t % m_tiles, nt = t / m_tiles;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(empty + s, ph ^ 1, abort_flag, err)) { ok = false; break; }
          mbar_arrive_expect_tx(full + s, C::kStageBytes);
          tma_load_2d(sA + (size_t)s * C::kABytes, &tmA, kb * C::kBK, mt * BM, full + s, pol_a);
          tma_load_2d(sB + (size_t)s * C::kBBytes, &tmB, kb * C::kBK, nt * BN, full + s, pol_b);
          issued[s] = true;
          issued_phase[s] = ph;
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        // Unwinding: let every copy this thread started land before the CTA exits.
        for (int i = 0; i < STAGES; ++i)
          if (issued[i]) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(full + i, issued_phase[i]) &&
                   globaltimer_ns() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 128, BN);
      uint32_t s = 0, ph = 0;
      int i = 0;
      bool ok = true, any = false;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++i) {
        const int buf = i % C::kAccBufs;
        const uint32_t aph = (uint32_t)(i / C::kAccBufs) & 1u;
        if (!mbar_wait(tempty + buf, aph ^ 1, abort_flag, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * C::kAccCols);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(full + s, ph, abort_flag, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + (size_t)s * C::kABytes);
          const uint32_t b0 = smem_u32(sB + (size_t)s * C::kBBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t bdesc = smem_desc_kmajor_sw128(b0 + 32 * k);
#pragma unroll
            for (int h = 0; h < C::kHalves; ++h) {
              const uint64_t adesc = smem_desc_kmajor_sw128(a0 + 16384 * h + 32 * k);
              umma<KD>(d0 + (uint32_t)(h * BN), adesc, bdesc, idesc, (kb | k) != 0);
            }
          }
          any = true;
          umma_commit(empty + s);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull + buf);
      }
      if (!ok && any) {
        // Unwinding: wait (bounded) until the MMAs already issued have finished with TMEM.
        umma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // the TMEM lane quarter this warp may read
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int buf = i % C::kAccBufs;
      const uint32_t aph = (uint32_t)(i / C::kAccBufs) & 1u;
      if (!mbar_wait(tfull + buf, aph, abort_flag, err)) break;
      tc_fence_after();
      const int mt = t % m_tiles, nt = t / m_tiles;
#pragma unroll 1
      for (int h = 0; h < C::kHalves; ++h) {
        const int row = mt * BM + h * 128 + q * 32 + lane;
        const bool row_ok = row < M;
        const float sa = row_ok ? __ldg(ep.a_s + (int64_t)row * ep.a_s_ld) : 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * C::kAccCols + h * BN + c0),
                    r);
          tmem_ld_wait();
          const int col0 = nt * BN + c0;
          if (!row_ok || col0 >= N) continue;
          const int valid = min(16, N - col0);
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int col = min(col0 + j, N - 1);
            const float sb = __ldg(ep.b_s + (ep.bn == 1 ? (int64_t)col : (int64_t)col / ep.bn) * ep.b_s_ld);
            const float a = (KD == Kind::I8) ? (float)(int32_t)r[j] : __uint_as_float(r[j]);
            v[j] = a * (sa * sb);
          }
          const int64_t off = (int64_t)row * N + col0;
          const bool vec_ok = (N % 8) == 0;
          if (KD == Kind::I8 && ep.acc_out != nullptr) {
            int32_t* dst = ep.acc_out + off;
            if (vec_ok && valid == 16) {
#pragma unroll
              for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
            } else {
              for (int j = 0; j < valid; ++j) dst[j] = (int32_t)r[j];
            }
          }
          if (ep.c_dtype == TO_BF16) {
            store_row_chunk16<__nv_bfloat16>(
                reinterpret_cast<__nv_bfloat16*>(ep.c) + off, v,
                ep.bias ? reinterpret_cast<const __nv_bfloat16*>(ep.bias) + col0 : nullptr, valid,
                vec_ok);
          } else if (ep.c_dtype == TO_F16) {
            store_row_chunk16<__half>(reinterpret_cast<__half*>(ep.c) + off, v,
                                      ep.bias ? reinterpret_cast<const __half*>(ep.bias) + col0 : nullptr,
                                      valid, vec_ok);
          } else {
            store_row_chunk16<float>(reinterpret_cast<float*>(ep.c) + off, v,
                                     ep.bias ? reinterpret_cast<const float*>(ep.bias) + col0 : nullptr,
                                     valid, (N % 4) == 0);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + buf);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<C::kTmemCols>(tmem);
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// 2-D K-major operand [rows, cols] (cols contiguous, elem bytes each) tiled as
// box_rows x 128 bytes with the 128-byte swizzle. Cached per (pointer, shape, box).
int make_tmap_kmajor(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int elem,
                     int box_rows) {
  struct Key {
    const void* p;
    int64_t rows, cols;
    int elem, box;
    bool operator==(const Key& o) const {
      return p == o.p && rows == o.rows && cols == o.cols && elem == o.elem && box == o.box;
    }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ (size_t)(k.rows * 1315423911u) ^
             (size_t)(k.cols * 2654435761u) ^ (size_t)(k.box * 97 + k.elem);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{(const char*)ptr + ((int64_t)dev << 56), rows, cols, elem, box_rows};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return TO_OK;
    }
  }
  EncodeFn encode = get_encode();
  if (!encode) return fail(TO_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * elem)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(out, elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                      2, const_cast<void*>(ptr), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TO_ECUDA, "cuTensorMapEncodeTiled failed (%d) for [%lld, %lld] x %d B", (int)r,
                (long long)rows, (long long)cols, elem);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return TO_OK;
}

template <Kind KD, int BM, int BN, int STAGES>
int launch_gemm_cfg(const void* a, const void* b, int64_t M, int64_t N, int64_t K, const Epi& ep,
                    cudaStream_t st) {
  using C = GemmCfg<KD, BM, BN, STAGES>;
  auto kern = k_gemm_sm100<KD, BM, BN, STAGES>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem);
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "tcgen05 gemm: shared memory attribute");
  CUtensorMap ta, tb;
  int rc = make_tmap_kmajor(&ta, a, M, K, C::kElem, BM);
  if (rc) return rc;
  rc = make_tmap_kmajor(&tb, b, N, K, C::kElem, BN);
  if (rc) return rc;
  const int64_t tiles = ceil_div(M, BM) * ceil_div(N, BN);
  const int grid = (int)std::min<int64_t>(tiles, sm_count());
  k_gemm_sm100<KD, BM, BN, STAGES><<<grid, kGemmThreads, C::kSmem, st>>>(
      ta, tb, (int)M, (int)N, (int)K, ep, device_error_ptr());
  return check_launch("tcgen05 gemm");
}

// Tile shapes: large problems take 128 x 256 tiles; small-M layers (M <= 256, the decode /
// small-batch regime, HBM-bound on B) take the narrowest N tile that still fits every tile
// in one wave, so all SMs stream B at once.
template <Kind KD>
int launch_gemm(const void* a, const void* b, int64_t M, int64_t N, int64_t K, const Epi& ep,
                cudaStream_t st) {
  const int64_t sms = sm_count();
  auto tiles = [&](int bm, int bn) { return ceil_div(M, bm) * ceil_div(N, bn); };
  if (M > 256 || tiles(128, 256) >= sms) return launch_gemm_cfg<KD, 128, 256, 4>(a, b, M, N, K, ep, st);
  if (M <= 128) {
    if (tiles(128, 128) <= sms && tiles(128, 64) > sms)
      return launch_gemm_cfg<KD, 128, 128, 6>(a, b, M, N, K, ep, st);
    if (tiles(128, 128) > sms) return launch_gemm_cfg<KD, 128, 256, 4>(a, b, M, N, K, ep, st);
    return launch_gemm_cfg<KD, 128, 64, 8>(a, b, M, N, K, ep, st);
  }
  if (tiles(256, 64) <= sms) return launch_gemm_cfg<KD, 256, 64, 5>(a, b, M, N, K, ep, st);
  if (tiles(256, 80) <= sms) return launch_gemm_cfg<KD, 256, 80, 5>(a, b, M, N, K, ep, st);
  return launch_gemm_cfg<KD, 256, 128, 4>(a, b, M, N, K, ep, st);
}

}  // namespace sm100

// Routes a W8A8 call to the tcgen05 kernel when its scales are per-row x per-column-block
// (block_k >= K) and the operands meet TMA's alignment rules; otherwise TO_EUNSUPPORTED so
// the caller uses the generic kernel.
int w8a8_tc_launch(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                   void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M, int64_t N,
                   int64_t K, int64_t bn, int64_t bk, cudaStream_t st) {
  if (bk < K) return TO_EUNSUPPORTED;
  if (K % 16 != 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return TO_EUNSUPPORTED;
  if (!aligned16(a) || !aligned16(b)) return TO_EUNSUPPORTED;
  if (M * N < 128 * 128) return TO_EUNSUPPORTED;  // tiny problems: the generic kernel is cheaper
  sm100::Epi ep;
  ep.a_s = a_s;
  ep.a_s_ld = 1;
  ep.b_s = b_s;
  ep.b_s_ld = 1;
  ep.bn = bn >= N ? N : bn;
  ep.c = c;
  ep.c_dtype = c_dtype;
  ep.bias = bias;
  ep.acc_out = fp8 ? nullptr : acc_out;
  // Small-M layers re-read A from L2 in every CTA and stream B once: keep A, evict B first.
  const bool small_m = M <= 256;
  ep.policy_a = small_m ? 2 : 0;
  ep.policy_b = small_m ? 1 : 0;
  if (fp8) return sm100::launch_gemm<sm100::Kind::E4M3>(a, b, M, N, K, ep, st);
  return sm100::launch_gemm<sm100::Kind::I8>(a, b, M, N, K, ep, st);
}

}  // namespace tob
