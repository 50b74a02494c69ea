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
// CTA roles (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one thread)      full[s]  <- TMA bytes       empty[s] -> wait
//   warp 1      MMA issuer   (one thread)      empty[s] <- tcgen05.commit  tfull[b] <- commit
//   warps 2..9  epilogue, two warps per TMEM lane quarter taking alternate 32-column chunks:
//               TMEM -> registers -> scales -> staged TMA stores, then arrive on tempty[b]
// The 2-CTA kernel (k_gemm_pair) adds an eleventh warp that issues the B copies.
// Accumulators live in tensor memory, double-buffered when two fit in 512 columns, so the
// epilogue of tile i overlaps the main loop of tile i+1. A tile is BM x BN with BM = 128 or
// 256 (two M=128 MMAs sharing each B slice, for small-M layers that must spread N over all SMs).
//
// Every wait is bounded (sm100.cuh, kWaitLimitNs); on expiry the kernel records the error
// word, unwinds every role, waits (bounded) for its in-flight copies and MMAs, frees its TMEM
// and returns.
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <stdlib.h>
#include <string.h>

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
  int tma_store;     // 16-bit C written through shared-memory staging + TMA stores
  int band = 16;     // M tiles per band of the tile order (tile_band)
};

// warp 0 TMA producer, warp 1 MMA issuer, warps 2..9 epilogue (two per TMEM lane quarter)
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
// The 2-CTA kernel adds an eleventh warp that issues the B copies.
constexpr int kPairBWarp = 2 + kEpiWarps;
constexpr int kPairThreads = kGemmThreads + 32;

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
  // Epilogue staging for TMA stores of 16-bit outputs: one 32 x 32 x 2 B slab per warp.
  static constexpr int kStageOutBytes = 32 * 32 * 2;
  static constexpr size_t kOutBytes = kEpiWarps * kStageOutBytes;
  static constexpr size_t kSmem = (size_t)STAGES * kStageBytes + kOutBytes + kBarrierBytes;
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
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < valid) dst[j] = o[j];
  }
}

// Per-column scales of one tile, preloaded by each epilogue warp while the main loop runs:
// lane l holds b_s for tile columns 32*i + l in sb[i] (broadcast later with shuffles).
template <int BN>
__device__ __forceinline__ void load_tile_col_scales(float (&sb)[(BN + 31) / 32], const Epi& ep,
                                                     int n0, int N, int lane) {
#pragma unroll
  for (int i = 0; i < (BN + 31) / 32; ++i) {
    const int col = min(n0 + 32 * i + lane, N - 1);
    const int64_t idx = ep.bn >= N ? 0 : (ep.bn == 1 ? (int64_t)col : (int64_t)col / ep.bn);
    sb[i] = ep.b_s != nullptr ? __ldg(ep.b_s + idx * ep.b_s_ld) : 1.f;  // null: unscaled
  }
}

// sb[i] for a runtime i < (BN + 31) / 32 without dynamic register indexing.
template <int BN>
__device__ __forceinline__ float pick_scale(const float (&sb)[(BN + 31) / 32], int i) {
  float s = sb[0];
#pragma unroll
  for (int k = 1; k < (BN + 31) / 32; ++k) s = (i == k) ? sb[k] : s;
  return s;
}

// v[j] = acc[j] * (a_s[row] * b_s[col0 + j]) for the 32-column chunk starting at tile column c0.
template <Kind KD, int BN>
__device__ __forceinline__ void scale_chunk32(const uint32_t* r, float* v, float sa,
                                              const float (&sb)[(BN + 31) / 32], int c0) {
  const float mine = pick_scale<BN>(sb, c0 / 32);
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float s = __shfl_sync(0xffffffffu, mine, j);
    const float a = (KD == Kind::I8) ? (float)(int32_t)r[j] : __uint_as_float(r[j]);
    v[j] = a * (sa * s);
  }
}

// Rounds 32 values to the 16-bit output dtype (pairs packed in pk); a bias is added after
// that rounding and rounded again, the order of `output + bias` in apply_w8a8_block_*_linear.
__device__ __forceinline__ void pack_out16(const float* v, uint32_t* pk, const Epi& ep, int col0,
                                           int valid) {
  if (ep.bias == nullptr) {  // common case: one paired conversion per two values
    if (ep.c_dtype == TO_BF16) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        __nv_bfloat162 o = __floats2bfloat162_rn(v[j], v[j + 1]);
        pk[j / 2] = *reinterpret_cast<uint32_t*>(&o);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        __half2 o = __floats2half2_rn(v[j], v[j + 1]);
        pk[j / 2] = *reinterpret_cast<uint32_t*>(&o);
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    uint16_t lo, hi;
    if (ep.c_dtype == TO_BF16) {
      __nv_bfloat16 a = __float2bfloat16_rn(v[j]), b = __float2bfloat16_rn(v[j + 1]);
      if (ep.bias != nullptr) {
        const __nv_bfloat16* bias = reinterpret_cast<const __nv_bfloat16*>(ep.bias) + col0;
        if (j < valid) a = __float2bfloat16_rn(__bfloat162float(a) + __bfloat162float(bias[j]));
        if (j + 1 < valid) b = __float2bfloat16_rn(__bfloat162float(b) + __bfloat162float(bias[j + 1]));
      }
      lo = *reinterpret_cast<uint16_t*>(&a);
      hi = *reinterpret_cast<uint16_t*>(&b);
    } else {
      __half a = __float2half_rn(v[j]), b = __float2half_rn(v[j + 1]);
      if (ep.bias != nullptr) {
        const __half* bias = reinterpret_cast<const __half*>(ep.bias) + col0;
        if (j < valid) a = __float2half_rn(__half2float(a) + __half2float(bias[j]));
        if (j + 1 < valid) b = __float2half_rn(__half2float(b) + __half2float(bias[j + 1]));
      }
      lo = *reinterpret_cast<uint16_t*>(&a);
      hi = *reinterpret_cast<uint16_t*>(&b);
    }
    pk[j / 2] = (uint32_t)lo | ((uint32_t)hi << 16);
  }
}

// Direct row stores of one 32-column chunk (fp32 output, or shapes the TMA path rejects).
template <Kind KD>
__device__ __forceinline__ void store_direct(const float* v, const Epi& ep, int64_t off, int col0,
                                             int valid, int N) {
  if (ep.c_dtype == TO_BF16) {
    const __nv_bfloat16* bias = ep.bias ? reinterpret_cast<const __nv_bfloat16*>(ep.bias) + col0 : nullptr;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.c) + off;
    store_row_chunk16<__nv_bfloat16>(dst, v, bias, min(valid, 16), (N % 8) == 0);
    if (valid > 16) store_row_chunk16<__nv_bfloat16>(dst + 16, v + 16, bias ? bias + 16 : nullptr, valid - 16, (N % 8) == 0);
  } else if (ep.c_dtype == TO_F16) {
    const __half* bias = ep.bias ? reinterpret_cast<const __half*>(ep.bias) + col0 : nullptr;
    __half* dst = reinterpret_cast<__half*>(ep.c) + off;
    store_row_chunk16<__half>(dst, v, bias, min(valid, 16), (N % 8) == 0);
    if (valid > 16) store_row_chunk16<__half>(dst + 16, v + 16, bias ? bias + 16 : nullptr, valid - 16, (N % 8) == 0);
  } else {
    const float* bias = ep.bias ? reinterpret_cast<const float*>(ep.bias) + col0 : nullptr;
    float* dst = reinterpret_cast<float*>(ep.c) + off;
    store_row_chunk16<float>(dst, v, bias, min(valid, 16), (N % 4) == 0);
    if (valid > 16) store_row_chunk16<float>(dst + 16, v + 16, bias ? bias + 16 : nullptr, valid - 16, (N % 4) == 0);
  }
}

// First K block of tile t. Tiles start at different K offsets so that concurrently running
// CTAs, which share the A (or B) operand, do not all request the same lines from L2 at the
// same moment. Integer accumulation is exact in any order; fp32 accumulation order changes
// only within rounding.
__device__ __forceinline__ int k_start(int t, int kblocks) { return (int)(((unsigned)t * 5u) % (unsigned)kblocks); }

// Output tile t -> (M tile, N tile). Tiles run in bands of `band` M tiles, M fastest within a
// band: the ~148 tiles in flight then share the band's M tiles of A and a few N tiles of B, so
// each band streams B once and keeps its A rows in L2, instead of re-reading all of A on every
// wave (the plain M-fastest order does that once M spans more tiles than a wave). Problems of at
// most `band` M tiles keep the plain order.
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int band, int& mt,
                                            int& nt) {
  const int band_tiles = band * n_tiles;
  const int b = t / band_tiles;
  const int rows = min(band, m_tiles - b * band);  // M tiles in this band
  const int local = t - b * band_tiles;
  mt = b * band + local % rows;
  nt = local / rows;
}

// The band: the most M tiles (16 or 32) whose A rows stay within 32 MB, so that they and the
// B blocks in flight stay in L2 next to the output being written. FP8 8192^3 (128-row tiles,
// K = 8192): 32 tiles, B read twice instead of four times (262 MB read per GEMM against 360);
// 64 tiles (all of A, 64 MB) thrashed L2 (733 MB read).
inline int tile_band(int bm, int64_t K, int elem) {
  return (int64_t)32 * bm * K * elem <= ((int64_t)32 << 20) ? 32 : 16;
}

// Bytes of one 128-row half's partial sums in the exchange layout [chunk][j / 4][row][4] (32-bit
// words; 16-column tail chunks leave their upper half unused).
template <int BN>
__host__ __device__ constexpr int ks2_xfer_bytes() {
  return ((BN + 31) / 32) * 8 * 128 * 16;
}

// Epilogue of a K-split pair (see k_gemm_sm100): 8 warps, two per TMEM lane quarter q, taking
// alternate 32-column chunks. Each CTA stages its partial sums of the peer's half in its own
// (idle) operand ring, then one bulk copy moves them into the peer's ring, completing on the
// peer's recv_bar; the staging layout makes every warp store and load one contiguous
// 512-byte row (no bank conflicts).
template <Kind KD, int BM, int BN, int STAGES>
__device__ __forceinline__ void ks2_epilogue(uint32_t tmem, uint8_t* sA, uint64_t* tfull,
                                             uint64_t* recv_bar,
                                             volatile int* abort_flag, int* err, const Epi& ep,
                                             const CUtensorMap* tmC, const CUtensorMap* tmC16,
                                             int M, int N, int m_tiles, int n_tiles, int t,
                                             int rank, int warp, int lane) {
  using C = GemmCfg<KD, BM, BN, STAGES>;
  constexpr int kXfer = ks2_xfer_bytes<BN>();
  constexpr int kRecvOff = (kXfer + 1023) & ~1023;
  // Output slabs for the TMA stores, one per (chunk, lane quarter), after the exchange areas:
  // no store has to wait for an earlier one to release its slab.
  constexpr int kOutOff = kRecvOff + ((kXfer + 1023) & ~1023);
  static_assert((size_t)kOutOff + (size_t)((BN + 31) / 32) * 4 * C::kStageOutBytes <=
                    (size_t)STAGES * C::kStageBytes,
                "the staged and received partial sums and the output slabs must fit in the ring");
  const int q = warp & 3;          // the TMEM lane quarter this warp may read
  const int eg = (warp - 2) >> 2;  // which of the two warps on that quarter
  const int mine = rank, other = rank ^ 1;
  int mt, nt;
  tile_coords(t, m_tiles, n_tiles, ep.band, mt, nt);
  float sbt[(BN + 31) / 32];
  load_tile_col_scales<BN>(sbt, ep, nt * BN, N, lane);
  const int row0 = mt * BM + mine * 128 + q * 32;  // first row of this warp's 32-row slab
  const int row = row0 + lane;
  const bool row_ok = row < M;
  const float sa = row_ok ? __ldg(ep.a_s + (int64_t)row * ep.a_s_ld) : 0.f;
  uint32_t* stage = reinterpret_cast<uint32_t*>(sA);             // partial sums for the peer
  uint32_t* recv = reinterpret_cast<uint32_t*>(sA + kRecvOff);   // the peer's, for this CTA
  auto slot = [&](int c, int jj) { return ((c * 8 + jj) * 128 + q * 32 + lane) * 4; };

  const bool ok = mbar_wait(tfull, 0, abort_flag, err);
  tc_fence_after();
  if (ok) {
    // The main loop is done, so this CTA's ring is free: stage the peer's half.
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (((c0 / 32) & 1) != eg) continue;
      const bool wide = (BN - c0) >= 32;
      uint32_t r[32];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(other * BN + c0);
      tmem_ld16(taddr, r);
      if (wide) tmem_ld16(taddr + 16, r + 16);
      tmem_ld_wait();
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        if (jj < (wide ? 8 : 4))
          *reinterpret_cast<uint4*>(stage + slot(c0 / 32, jj)) =
              make_uint4(r[4 * jj], r[4 * jj + 1], r[4 * jj + 2], r[4 * jj + 3]);
    }
  }
  fence_proxy_async_smem();  // the staged words are read by the bulk copy (async proxy)
  cluster_sync_all();        // 1: both halves staged; both rings free to receive
  if (warp == 2 && lane == 0) {
    const uint32_t dst = mapa_shared(smem_u32(recv), (uint32_t)other);
    const uint32_t bar = mapa_shared(smem_u32(recv_bar), (uint32_t)other);
    constexpr int kPiece = 16384;  // bytes per copy
#pragma unroll 1
    for (int off = 0; off < kXfer; off += kPiece)
      bulk_copy_to_peer(dst + off, reinterpret_cast<uint8_t*>(stage) + off,
                        (uint32_t)min(kPiece, kXfer - off), bar);
  }
  const bool got = mbar_wait(recv_bar, 0, abort_flag, err);
  // 2 (split): this CTA's copy has landed in the peer once the peer arrives; the peer's shared
  // memory may be released only after that, so the wait is at the very end.
  cluster_arrive_release();
  if (ok && got) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      if (((c0 / 32) & 1) != eg) continue;
      const bool wide = (BN - c0) >= 32;
      uint32_t r[32];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(mine * BN + c0);
      tmem_ld16(taddr, r);
      if (wide) tmem_ld16(taddr + 16, r + 16);
      tmem_ld_wait();
      // Rank 0's partial sum comes first in every element, whichever CTA adds it up.
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        if (jj >= (wide ? 8 : 4)) continue;
        const uint4 pv = *reinterpret_cast<const uint4*>(recv + slot(c0 / 32, jj));
        const uint32_t p[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t& d = r[4 * jj + e];
          if (KD == Kind::I8) {
            d = (uint32_t)((int32_t)d + (int32_t)p[e]);
          } else {
            const float lo = rank == 0 ? __uint_as_float(d) : __uint_as_float(p[e]);
            const float hi = rank == 0 ? __uint_as_float(p[e]) : __uint_as_float(d);
            d = __float_as_uint(lo + hi);
          }
        }
      }
      const int col0 = nt * BN + c0;
      if (col0 >= N) continue;
      const int valid = min(wide ? 32 : 16, N - col0);
      float v[32];
      scale_chunk32<KD, BN>(r, v, sa, sbt, c0);
      if (KD == Kind::I8 && ep.acc_out != nullptr && row_ok) {
        int32_t* dst = ep.acc_out + (int64_t)row * N + col0;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < valid) dst[j] = (int32_t)r[j];
      }
      if (ep.tma_store) {
        uint8_t* stg = sA + kOutOff + (size_t)((c0 / 32) * 4 + q) * C::kStageOutBytes;
        uint32_t pk[16];
        pack_out16(v, pk, ep, col0, valid);
        if (wide) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        } else {
#pragma unroll
          for (int c = 0; c < 2; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 32 + (c << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(wide ? tmC : tmC16, col0, row0, stg);
          bulk_commit();
        }
      } else if (row_ok) {
        store_direct<KD>(v, ep, (int64_t)row * N + col0, col0, valid, N);
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  if (ep.tma_store && lane == 0) bulk_wait_read<0>();  // stores have read their slabs
  cluster_wait_acquire();
}

// KS2: the two CTAs of a (2,1,1) cluster share one BM = 256 tile and split its K blocks in
// half, so each SM streams half of the tile's A and B rows. Each CTA then finalises one
// 128-row half: it sends its partial sums of the other half into the peer's (by then idle)
// operand ring through distributed shared memory and adds the peer's partial sums to its own.
// int32 sums stay exact; fp32 sums are added in a fixed order. One tile per CTA pair.
// BMN: B is [K, N] row-major (MN-major for the MMA), as in a dense C = A @ B, copied as
// 64-column strips of BK rows (a 3-D tensor-map view {64 columns, K rows, N / 64 strips}) into
// the 128-byte-swizzled MN-major layout; otherwise B is [N, K] (K-major).
template <Kind KD, int BM, int BN, int STAGES, bool KS2, bool BMN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC16,
                 int M, int N, int K, Epi ep, int* err) {
  static_assert(!KS2 || BM == 256, "the K-split pair finalises one 128-row half per CTA");
  static_assert(!BMN || (!KS2 && BN % 64 == 0 && KindTraits<KD>::kElemBytes == 2),
                "MN-major B: 16-bit operands in whole 64-column strips");
  using C = GemmCfg<KD, BM, BN, STAGES>;
  using Tr = KindTraits<KD>;
  // The swizzled operand tiles need 1024-byte alignment; the dynamic shared memory window
  // is declared with that alignment.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  uint8_t* sA = smem;
  uint8_t* sB = smem + (size_t)STAGES * C::kABytes;
  uint8_t* sOut = sB + (size_t)STAGES * C::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::kOutBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* recv_bar = drain + 1;  // K-split pair: the peer's partial sums have landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int kblocks = (K + C::kBK - 1) / C::kBK;
  // Tiles this CTA visits (t0, t0 + tstride, ...) and its K blocks [kb_lo, kb_lo + kb_n).
  const int rank = KS2 ? (int)(blockIdx.x & 1) : 0;
  const int t0 = KS2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstride = KS2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int kb_lo = KS2 ? rank * (kblocks / 2) : 0;
  const int kb_n = KS2 ? (rank ? kblocks - kblocks / 2 : kblocks / 2) : kblocks;

  // Every role depends on the 1024-byte alignment of the operand ring; without it the kernel
  // records an error and does nothing.
  const bool misaligned = (smem_u32(smem_raw) & 1023u) != 0;
  // The producer thread initialises the barriers and at once requests the first ring of
  // stages of its first tile (no stage has a previous use to wait for), so the operand stream
  // starts while the MMA warp allocates tensor memory.
  int pre = 0;  // stages of the first tile already requested
  uint64_t pol_a = 0, pol_b = 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, kEpiWarps);
    }
    mbar_init(drain, 1);
    mbar_init(recv_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (KS2) mbar_arrive_expect_tx(recv_bar, (uint32_t)ks2_xfer_bytes<BN>());
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (ep.tma_store) {
      prefetch_tmap(&tmC);
      prefetch_tmap(&tmC16);
    }
    if (misaligned) {
      if (err) atomicExch(err, (int)kErrSmemAlign);
    } else if (t0 < tiles) {
      pol_a = make_policy(ep.policy_a);
      pol_b = make_policy(ep.policy_b);
      int mt, nt;
      tile_coords(t0, m_tiles, n_tiles, ep.band, mt, nt);
      // The dense form's B (larger than L2) is shared by the M tiles of a band: they walk K in
      // step, so each B block is read from DRAM once.
      const int k0 = BMN ? 0 : k_start(t0, kb_n);
      pre = min(STAGES, kb_n);
      for (int it = 0; it < pre; ++it) {
        const int kb = kb_lo + (k0 + it) % kb_n;
        mbar_arrive_expect_tx(full + it, C::kStageBytes);
        tma_load_2d(sA + (size_t)it * C::kABytes, &tmA, kb * C::kBK, mt * BM, full + it, pol_a);
        if constexpr (BMN)
          tma_load_3d(sB + (size_t)it * C::kBBytes, &tmB, 0, kb * C::kBK, nt * (BN / 64),
                      full + it, pol_b);
        else
          tma_load_2d(sB + (size_t)it * C::kBBytes, &tmB, kb * C::kBK, nt * BN, full + it, pol_b);
      }
    }
  }
  if (warp == 1) tmem_alloc<C::kTmemCols>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (misaligned) {
    // nothing to do; fall through to the teardown
    if constexpr (KS2) {
      cluster_sync_all();
      cluster_arrive_release();
      cluster_wait_acquire();
    }
  } else if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t s = (uint32_t)(pre % STAGES), ph = pre == STAGES ? 1u : 0u;
      // per stage: loads issued / their phase (the pre-issued ring is phase 0)
      uint32_t issued_mask = (1u << pre) - 1u, issued_phase = 0;
      bool ok = true;
      int step = pre;
      for (int t = t0; ok && t < tiles; t += tstride) {
        int mt, nt;
        tile_coords(t, m_tiles, n_tiles, ep.band, mt, nt);
        const int k0 = BMN ? 0 : k_start(t, kb_n);
        for (int it = (t == t0 ? pre : 0); it < kb_n; ++it, ++step) {
          const int kb = kb_lo + (k0 + it) % kb_n;
          if (!mbar_wait(empty + s, ph ^ 1, abort_flag, err)) { ok = false; break; }
          mbar_arrive_expect_tx(full + s, C::kStageBytes);
          tma_load_2d(sA + (size_t)s * C::kABytes, &tmA, kb * C::kBK, mt * BM, full + s, pol_a);
          if constexpr (BMN)
            tma_load_3d(sB + (size_t)s * C::kBBytes, &tmB, 0, kb * C::kBK, nt * (BN / 64),
                        full + s, pol_b);
          else
            tma_load_2d(sB + (size_t)s * C::kBBytes, &tmB, kb * C::kBK, nt * BN, full + s, pol_b);
          issued_mask |= 1u << s;
          issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        // Unwinding: let every copy this thread started land before the CTA exits.
        for (int i = 0; i < STAGES; ++i)
          if (issued_mask & (1u << i)) {
            const uint64_t tw = globaltimer_ns();
            while (!mbar_try_wait(full + i, (issued_phase >> i) & 1u) &&
                   globaltimer_ns() - tw < kWaitLimitNs) {
            }
          }
      }
    }
    if constexpr (KS2) {  // the pair's epilogue barriers (see ks2_epilogue)
      cluster_sync_all();
      cluster_arrive_release();
      cluster_wait_acquire();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc =
          BMN ? make_idesc_major(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 128, BN, 0, 1)
              : make_idesc(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 128, BN);
      uint32_t s = 0, ph = 0;
      int i = 0, step = 0;
      bool ok = true, any = false;
      for (int t = t0; ok && t < tiles; t += tstride, ++i) {
        const int buf = i % C::kAccBufs;
        const uint32_t aph = (uint32_t)(i / C::kAccBufs) & 1u;
        if (!mbar_wait(tempty + buf, aph ^ 1, abort_flag, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * C::kAccCols);
        for (int it = 0; it < kb_n; ++it, ++step) {
          if (!mbar_wait(full + s, ph, abort_flag, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + (size_t)s * C::kABytes);
          const uint32_t b0 = smem_u32(sB + (size_t)s * C::kBBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // MN-major: 64-column strips BK rows deep (8 KB apart); K step k = 16 rows = 2 KB
            const uint64_t bdesc = BMN ? smem_desc_mnmajor_sw128(b0 + 2048 * k, 8192, 1024)
                                       : smem_desc_kmajor_sw128(b0 + 32 * k);
#pragma unroll
            for (int h = 0; h < C::kHalves; ++h) {
              const uint64_t adesc = smem_desc_kmajor_sw128(a0 + 16384 * h + 32 * k);
              umma<KD>(d0 + (uint32_t)(h * BN), adesc, bdesc, idesc, (it | k) != 0);
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
        const uint64_t tw = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - tw < kWaitLimitNs) {
        }
      }
    }
    if constexpr (KS2) {
      cluster_sync_all();
      cluster_arrive_release();
      cluster_wait_acquire();
    }
  } else if constexpr (KS2) {
    // ------------------------------------------------------------ epilogue, K-split pair
    ks2_epilogue<KD, BM, BN, STAGES>(tmem, sA, tfull, recv_bar, abort_flag, err, ep, &tmC, &tmC16,
                                     M, N, m_tiles, n_tiles, t0, rank, warp, lane);
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;          // the TMEM lane quarter this warp may read
    const int eg = (warp - 2) >> 2;  // which of the two warps on that quarter
    int i = 0;
    for (int t = t0; t < tiles; t += tstride, ++i) {
      const int buf = i % C::kAccBufs;
      const uint32_t aph = (uint32_t)(i / C::kAccBufs) & 1u;
      // Scales of this tile, loaded while the main loop still runs.
      int mt, nt;
      tile_coords(t, m_tiles, n_tiles, ep.band, mt, nt);
      float sbt[(BN + 31) / 32];
      load_tile_col_scales<BN>(sbt, ep, nt * BN, N, lane);
      float sat[C::kHalves];
#pragma unroll
      for (int h = 0; h < C::kHalves; ++h) {
        const int rr = mt * BM + h * 128 + q * 32 + lane;
        sat[h] = rr >= M ? 0.f : ep.a_s != nullptr ? __ldg(ep.a_s + (int64_t)rr * ep.a_s_ld) : 1.f;
      }
      if (!mbar_wait(tfull + buf, aph, abort_flag, err)) break;
      tc_fence_after();
      constexpr int kChunks = (BN + 31) / 32;
#pragma unroll 1
      for (int h = 0; h < C::kHalves; ++h) {
        const int row0 = mt * BM + h * 128 + q * 32;  // first row of this warp's 32-row slab
        const int row = row0 + lane;
        const bool row_ok = row < M;
        const float sa = (C::kHalves == 1 || h == 0) ? sat[0] : sat[C::kHalves - 1];
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          if (((h * kChunks + c0 / 32) & 1) != eg) continue;  // the two warps alternate chunks
          const bool wide = (BN - c0) >= 32;  // BN = 80 ends with a 16-column chunk
          uint32_t r[32];
          const uint32_t taddr =
              tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * C::kAccCols + h * BN + c0);
          tmem_ld16(taddr, r);
          if (wide) tmem_ld16(taddr + 16, r + 16);
          tmem_ld_wait();
          const int col0 = nt * BN + c0;
          if (col0 >= N) continue;
          const int valid = min(wide ? 32 : 16, N - col0);
          float v[32];
          scale_chunk32<KD, BN>(r, v, sa, sbt, c0);
          if (KD == Kind::I8 && ep.acc_out != nullptr && row_ok) {
            int32_t* dst = ep.acc_out + (int64_t)row * N + col0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < valid) dst[j] = (int32_t)r[j];
          }
          if (ep.tma_store) {
            uint8_t* stg = sOut + (size_t)(warp - 2) * C::kStageOutBytes;
            if (lane == 0) bulk_wait_read<0>();  // the previous store has read the slab
            __syncwarp();
            uint32_t pk[16];
            pack_out16(v, pk, ep, col0, valid);
            if (wide) {
              // 64-byte rows, 16-byte chunk c stored at c ^ ((row >> 1) & 3): the layout of a
              // SWIZZLE_64B TMA box, and free of bank conflicts for these row-per-lane stores.
#pragma unroll
              for (int c = 0; c < 4; ++c)
                *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            } else {
#pragma unroll
              for (int c = 0; c < 2; ++c)
                *reinterpret_cast<uint4*>(stg + lane * 32 + (c << 4)) =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(wide ? &tmC : &tmC16, col0, row0, stg);
              bulk_commit();
            }
          } else if (row_ok) {
            store_direct<KD>(v, ep, (int64_t)row * N + col0, col0, valid, N);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + buf);
    }
    if (ep.tma_store && lane == 0) bulk_wait_read<0>();  // stores have read their slabs
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<C::kTmemCols>(tmem);
  }
}

// ------------------------------------------------------------------ block-scaled tiles
// k_gemm_bs: W8A8 with per-(row, K block) activation scales and per-(column block, K block)
// weight scales, block_k = one 128-byte K slice:
//   C[m, n] = sum_kb (A_kb B_kb^T)[m, n] * a_s[m, kb] * b_s[n / bn, kb]
// (tileops/quant_int8.py:180, tileops/quant_fp8.py:188; DeepSeek-style 128 x 128 blocks).
// One 128 x 128 output tile per CTA. The products of each K block land in one of two TMEM
// buffers (the MMA warp alternates); the eight epilogue warps fold each finished buffer into
// fp32 running sums held in registers (64 columns of one row per thread), scaled by that
// block's two scales, and release it, so the tensor core fills one buffer while the other is
// read. The sums then leave like the per-channel kernel's outputs.
template <Kind KD, int STAGES, int KC>
struct BsCfg {
  static constexpr int kElem = KindTraits<KD>::kElemBytes;
  static constexpr int kBK = 128 / kElem;  // K elements per scale block (one 128-byte slice)
  static constexpr int kChunk = 128 * 128;  // one slice of 128 rows
  static constexpr int kABytes = KC * kChunk;  // a stage holds KC K blocks
  static constexpr int kBBytes = KC * kChunk;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStageOutBytes = 32 * 32 * 2;
  static constexpr size_t kOutBytes = kEpiWarps * kStageOutBytes;
  static constexpr size_t kSmem = (size_t)STAGES * kStageBytes + kOutBytes + 256;
  static_assert((2 * STAGES + 5) * 8 + 8 <= 256, "barrier area");
  static_assert(kSmem <= 232448, "shared memory");
};

template <Kind KD, int STAGES, int KC>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_bs(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmC, int M, int N, int K, Epi ep, int* err) {
  using C = BsCfg<KD, STAGES, KC>;
  using Tr = KindTraits<KD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sA = smem_raw;
  uint8_t* sB = smem_raw + (size_t)STAGES * C::kABytes;
  uint8_t* sOut = sB + (size_t)STAGES * C::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + C::kOutBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* pfull = empty + STAGES;  // [2] a K block's products are in TMEM buffer b
  uint64_t* pempty = pfull + 2;      // [2] the epilogue warps have folded buffer b
  uint64_t* drain = pempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + 127) / 128;
  const int mt = (int)(blockIdx.x % (unsigned)m_tiles), nt = (int)(blockIdx.x / (unsigned)m_tiles);
  const int kblocks = (K + C::kBK - 1) / C::kBK;
  const int nstages = (kblocks + KC - 1) / KC;  // stages of KC K blocks (the last may be partial)
  const bool misaligned = (smem_u32(smem_raw) & 1023u) != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(pfull + b, 1);
      mbar_init(pempty + b, kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (ep.tma_store) prefetch_tmap(&tmC);
    if (misaligned && err) atomicExch(err, (int)kErrSmemAlign);
  }
  if (warp == 1) tmem_alloc<256>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (misaligned) {
    // nothing to do; fall through to the teardown
  } else if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_a = make_policy(ep.policy_a), pol_b = make_policy(ep.policy_b);
      uint32_t issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int st = 0; st < nstages; ++st) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (st >= STAGES && !mbar_wait(empty + s, ph ^ 1, abort_flag, err)) { ok = false; break; }
        mbar_arrive_expect_tx(full + s, C::kStageBytes);
        if (KC == 1) {
          tma_load_2d(sA + (size_t)s * C::kABytes, &tmA, st * C::kBK, mt * 128, full + s, pol_a);
          tma_load_2d(sB + (size_t)s * C::kBBytes, &tmB, st * C::kBK, nt * 128, full + s, pol_b);
        } else {  // 3-D views {128 B, rows, K slices}: KC slices per copy
          tma_load_3d(sA + (size_t)s * C::kABytes, &tmA, 0, mt * 128, st * KC, full + s, pol_a);
          tma_load_3d(sB + (size_t)s * C::kBBytes, &tmB, 0, nt * 128, st * KC, full + s, pol_b);
        }
        issued_mask |= 1u << s;
        issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
      }
      if (!ok) {
        // Unwinding: let every copy this thread started land before the CTA exits.
        const uint64_t tw = globaltimer_ns();
        for (int i = 0; i < STAGES; ++i)
          if (issued_mask & (1u << i))
            while (!mbar_try_wait(full + i, (issued_phase >> i) & 1u) &&
                   globaltimer_ns() - tw < kWaitLimitNs) {
            }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 128, 128);
      bool ok = true, any = false;
      for (int st = 0; ok && st < nstages; ++st) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!mbar_wait(full + s, ph, abort_flag, err)) { ok = false; break; }
        for (int sub = 0; sub < KC; ++sub) {
          const int kb = st * KC + sub;
          if (kb >= kblocks) break;
          const int b = kb & 1;
          const uint32_t bph = (uint32_t)(kb >> 1) & 1u;
          if (kb >= 2 && !mbar_wait(pempty + b, bph ^ 1, abort_flag, err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + (size_t)s * C::kABytes + (size_t)sub * C::kChunk);
          const uint32_t b0 = smem_u32(sB + (size_t)s * C::kBBytes + (size_t)sub * C::kChunk);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma<KD>(tmem + (uint32_t)(b * 128), smem_desc_kmajor_sw128(a0 + 32 * k),
                     smem_desc_kmajor_sw128(b0 + 32 * k), idesc, k != 0);
          any = true;
          umma_commit(pfull + b);
        }
        if (ok) umma_commit(empty + s);
      }
      if (!ok && any) {
        // Unwinding: wait (bounded) until the MMAs already issued have finished with TMEM.
        umma_commit(drain);
        const uint64_t tw = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - tw < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ fold + epilogue
    const int q = warp & 3;          // the TMEM lane quarter this warp may read
    const int eg = (warp - 2) >> 2;  // columns [64 eg, 64 eg + 64) of the tile
    const int row0 = mt * 128 + q * 32;
    const int row = row0 + lane;
    const bool row_ok = row < M;
    const float* arow = ep.a_s + (int64_t)min(row, M - 1) * ep.a_s_ld;
    const float* bcol = ep.b_s + (ep.bn >= N ? 0 : (int64_t)(nt * 128) / ep.bn) * ep.b_s_ld;
    float run[64];
#pragma unroll
    for (int j = 0; j < 64; ++j) run[j] = 0.f;
    bool ok = true;
    float sa_next = __ldg(arow), sb_next = __ldg(bcol);
    for (int kb = 0; kb < kblocks; ++kb) {
      const int b = kb & 1;
      const uint32_t bph = (uint32_t)(kb >> 1) & 1u;
      const float sa = sa_next, sb = sb_next;
      if (kb + 1 < kblocks) {
        sa_next = __ldg(arow + kb + 1);
        sb_next = __ldg(bcol + kb + 1);
      }
      if (!mbar_wait(pfull + b, bph, abort_flag, err)) { ok = false; break; }
      tc_fence_after();
      uint32_t r[64];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * 128 + eg * 64);
      tmem_ld16(taddr, r);
      tmem_ld16(taddr + 16, r + 16);
      tmem_ld16(taddr + 32, r + 32);
      tmem_ld16(taddr + 48, r + 48);
      tmem_ld_wait();
      // run += (P * a_s) * b_s with each rounding of the scalar form, two columns per
      // instruction. An int8 block sum |P| <= 128 * 128 * 128 < 2^22 becomes a float exactly as
      // (bits(2^23 + 2^22) + P) - (2^23 + 2^22), which keeps the conversion off the slow pipe.
      const float2 sa2 = make_float2(sa, sa), sb2 = make_float2(sb, sb);
#pragma unroll
      for (int j = 0; j < 64; j += 2) {
        float2 pj;
        if constexpr (KD == Kind::I8) {
          pj = sub2_rn(make_float2(__int_as_float(0x4B400000 + (int32_t)r[j]),
                                   __int_as_float(0x4B400000 + (int32_t)r[j + 1])),
                       make_float2(12582912.0f, 12582912.0f));
        } else {
          pj = make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
        }
        const float2 acc = fma2_rn(mul2_rn(pj, sa2), sb2, make_float2(run[j], run[j + 1]));
        run[j] = acc.x;
        run[j + 1] = acc.y;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pempty + b);
    }
    if (ok) {
      uint8_t* stg = sOut + (size_t)(warp - 2) * C::kStageOutBytes;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col0 = nt * 128 + eg * 64 + h * 32;
        if (col0 >= N) continue;
        const int valid = min(32, N - col0);
        const float* v = run + h * 32;
        if (ep.tma_store) {
          if (lane == 0) bulk_wait_read<0>();  // the previous store has read the slab
          __syncwarp();
          uint32_t pk[16];
          pack_out16(v, pk, ep, col0, valid);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, col0, row0, stg);
            bulk_commit();
          }
        } else if (row_ok) {
          store_direct<KD>(v, ep, (int64_t)row * N + col0, col0, valid, N);
        }
      }
    }
    if (ep.tma_store && lane == 0) bulk_wait_read<0>();  // stores have read their slabs
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<256>(tmem);
  }
}

// ------------------------------------------------------------------ 2-CTA tiles
// k_gemm_pair: one 256 x BN output tile per CTA pair (a (2,1,1) cluster), M <= 256. The pair
// runs tcgen05 with cta_group::2: each CTA streams its 128 rows of A and its BN/2 rows of B
// into its own ring (TMA completing on the leader's barriers), the leader's single thread
// issues M=256 x N=BN MMAs that read both CTAs' halves, and each CTA's TMEM receives the
// full-K sums of its own 128 rows. Per SM that is half of A and half of B of the tile, as in the
// K-split pair, with no partial sums to exchange.
template <Kind KD, int BN, int STAGES, int KC>
struct PairCfg {
  static constexpr int kElem = KindTraits<KD>::kElemBytes;
  static constexpr int kBK = KC * 128 / kElem;         // K elements per stage (KC 128-byte slices)
  static constexpr int kAChunk = 128 * 128;            // one slice of this CTA's 128 rows of A
  static constexpr int kBChunk = (BN / 2) * 128;       // one slice of this CTA's BN/2 rows of B
  static constexpr int kABytes = KC * kAChunk;
  static constexpr int kBBytes = KC * kBChunk;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = pow2_at_least(BN);
  static constexpr int kStageOutBytes = 32 * 32 * 2;
  static constexpr int kOutSlabs = ((BN + 31) / 32) * 4;  // one per (chunk, lane quarter)
  static constexpr size_t kSmem = (size_t)STAGES * kStageBytes + 256;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "2-CTA tiles: N a multiple of 32");
  static_assert(KC == 1 || KC == 2 || KC == 4, "1, 2 or 4 K slices per stage");
  static_assert((size_t)kOutSlabs * kStageOutBytes <= (size_t)STAGES * kStageBytes, "slabs");
  static_assert(kSmem <= 232448, "shared memory");
};

// MINB: CTAs per SM the registers are sized for. Two (a 2-stage ring of 104 KB, so a CTA of the
// next launch could start under launch overlap during this one's tail) measured slower on the
// 256 x 11008 x 4096 INT8 layer: 17.5 us against 14.9 us with one CTA and four stages.
template <Kind KD, int BN, int STAGES, int KC, int MINB>
__global__ void __launch_bounds__(kPairThreads, MINB)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC16,
                int M, int N, int K, Epi ep, int* err) {
  using C = PairCfg<KD, BN, STAGES, KC>;
  using Tr = KindTraits<KD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sA = smem_raw;
  uint8_t* sB = smem_raw + (size_t)STAGES * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + (size_t)STAGES * C::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)(blockIdx.x & 1);  // 0: the leader, which issues the MMAs
  const int t = (int)(blockIdx.x >> 1);    // one tile per pair
  const int n_tiles = (N + BN - 1) / BN;
  const int mt = t / n_tiles, nt = t - mt * n_tiles;
  const int kblocks = (K + C::kBK - 1) / C::kBK;
  const bool misaligned = (smem_u32(smem_raw) & 1023u) != 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);   // the leader's producer arrives; both CTAs' bytes complete it
      mbar_init(empty + s, 1);  // the leader's commit, multicast to both CTAs
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (ep.tma_store) {
      prefetch_tmap(&tmC);
      prefetch_tmap(&tmC16);
    }
    if (misaligned && err) atomicExch(err, (int)kErrSmemAlign);
  }
  // First ring of stages, requested before the tensor-memory allocation: the leader's copies
  // complete on its own barriers, so it starts at once; the peer's complete on the leader's, so
  // it starts right after a cluster barrier that publishes them.
  //
  // Two warps issue the copies: warp 0 those of A (and, on the leader, the expectation of both
  // CTAs' bytes of a stage), warp kPairBWarp those of B. A warp's bulk tensor copies are
  // processed one after another, so two issuing warps keep twice as many requests moving. Under
  // programmatic dependent launch B (the weights) streams in while the previous kernel
  // finishes; A is requested after it has completed.
  const bool a_issuer = threadIdx.x == 0;
  const bool b_issuer = threadIdx.x == kPairBWarp * 32;
  int pre = 0;
  uint64_t pol = 0;
  const int k0 = k_start(t, kblocks);
  // This thread's copy of stage slot s for K block kb: A (a_issuer) or B. With KC = 2 the
  // operand maps are 3-D views {128 bytes, rows, K slices} and one copy brings KC slices.
  auto load_stage = [&](int s, int kb, uint32_t bar) {
    if (a_issuer) {
      if (KC == 1)
        tma_load_2d_pair(sA + (size_t)s * C::kABytes, &tmA, kb * C::kBK, mt * 256 + rank * 128,
                         bar, pol);
      else
        tma_load_3d_pair(sA + (size_t)s * C::kABytes, &tmA, 0, mt * 256 + rank * 128, kb * KC,
                         bar, pol);
    } else {
      if (KC == 1)
        tma_load_2d_pair(sB + (size_t)s * C::kBBytes, &tmB, kb * C::kBK,
                         nt * BN + rank * (BN / 2), bar, pol);
      else
        tma_load_3d_pair(sB + (size_t)s * C::kBBytes, &tmB, 0, nt * BN + rank * (BN / 2),
                         kb * KC, bar, pol);
    }
  };
  auto request_first_ring = [&]() {
    pol = make_policy(a_issuer ? ep.policy_a : ep.policy_b);
    pre = min(STAGES, kblocks);
    const uint32_t lead_full = mapa_shared(smem_u32(full), 0);
    if (a_issuer) grid_dependency_wait();  // A may be the previous kernel's output
    for (int it = 0; it < pre; ++it) {
      const int kb = (k0 + it) % kblocks;
      if (a_issuer) {
        if (rank == 0) mbar_arrive_expect_tx(full + it, 2 * C::kStageBytes);
        load_stage(it, kb, lead_full + it * 8u);
      } else {
        load_stage(it, kb, lead_full + it * 8u);
      }
    }
  };
  // The cluster barrier that publishes both CTAs' barriers is split: every thread arrives at
  // once, the leader's first ring and the tensor-memory allocation run while it completes.
  cluster_arrive_relaxed();
  if ((a_issuer || b_issuer) && !misaligned && rank == 0) request_first_ring();
  if (warp == 1) tmem_alloc_pair<C::kTmemCols>(tmem_holder);
  cluster_wait_acquire();  // both CTAs' barriers exist: copies and commits may signal them
  if ((a_issuer || b_issuer) && !misaligned && rank == 1) request_first_ring();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (misaligned) {
    // nothing to do; fall through to the teardown
  } else if (warp == 0 || warp == kPairBWarp) {
    // ------------------------------------------------------------ TMA producers (both CTAs)
    if (a_issuer || b_issuer) {
      const uint32_t lead_full = mapa_shared(smem_u32(full), 0);
      uint32_t s = (uint32_t)(pre % STAGES), ph = pre == STAGES ? 1u : 0u;
      // the leader's expectations (the pre-requested ring is phase 0), for unwinding
      uint32_t issued_mask = (1u << pre) - 1u, issued_phase = 0;
      bool ok = true;
      for (int it = pre; it < kblocks; ++it) {
        const int kb = (k0 + it) % kblocks;
        if (!mbar_wait(empty + s, ph ^ 1, abort_flag, err)) { ok = false; break; }
        const uint32_t bar = lead_full + (uint32_t)s * 8u;
        if (a_issuer) {
          if (rank == 0) {
            mbar_arrive_expect_tx(full + s, 2 * C::kStageBytes);
            issued_mask |= 1u << s;
            issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
          }
          load_stage((int)s, kb, bar);
        } else {
          load_stage((int)s, kb, bar);
        }
        if (++s == STAGES) { s = 0; ph ^= 1; }
      }
      if (a_issuer) grid_dependents_launch();
      if (!ok && rank == 0 && a_issuer) {
        // Unwinding: the leader's full barriers count both CTAs' bytes; let them land. One
        // deadline for all stages: a stage whose B copy was never issued does not complete.
        const uint64_t tw = globaltimer_ns();
        for (int i = 0; i < STAGES; ++i)
          if (issued_mask & (1u << i))
            while (!mbar_try_wait(full + i, (issued_phase >> i) & 1u) &&
                   globaltimer_ns() - tw < kWaitLimitNs) {
            }
      } else if (!ok && b_issuer) {
        // Unwinding: a B copy of a stage whose expectation the A issuer did not post cannot
        // be observed on the barrier; a copy lands within microseconds, so give it 50 us.
        const uint64_t tw = globaltimer_ns();
        while (globaltimer_ns() - tw < 50000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 256, BN);
      uint32_t s = 0, ph = 0;
      bool ok = true, any = false;
      for (int it = 0; it < kblocks; ++it) {
        if (!mbar_wait(full + s, ph, abort_flag, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + (size_t)s * C::kABytes);
        const uint32_t b0 = smem_u32(sB + (size_t)s * C::kBBytes);
#pragma unroll
        for (int k = 0; k < 4 * KC; ++k)
          umma_pair<KD>(tmem, smem_desc_kmajor_sw128(a0 + (k / 4) * C::kAChunk + 32 * (k % 4)),
                        smem_desc_kmajor_sw128(b0 + (k / 4) * C::kBChunk + 32 * (k % 4)), idesc,
                        (it | k) != 0);
        any = true;
        umma_commit_pair_mc(empty + s, 0x3);
        if (++s == STAGES) { s = 0; ph ^= 1; }
      }
      if (ok) {
        umma_commit_pair_mc(tfull, 0x3);
      } else if (any) {
        // Unwinding: wait (bounded) until the MMAs already issued have finished.
        umma_commit_pair(drain);
        const uint64_t tw = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - tw < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;          // the TMEM lane quarter this warp may read
    const int eg = (warp - 2) >> 2;  // which of the two warps on that quarter
    float sbt[(BN + 31) / 32];
    load_tile_col_scales<BN>(sbt, ep, nt * BN, N, lane);
    const int row0 = mt * 256 + rank * 128 + q * 32;  // first row of this warp's 32-row slab
    const int row = row0 + lane;
    const bool row_ok = row < M;
    grid_dependency_wait();  // A's scales and the output: after the previous kernel
    const float sa = row_ok ? __ldg(ep.a_s + (int64_t)row * ep.a_s_ld) : 0.f;
    const bool ok = mbar_wait(tfull, 0, abort_flag, err);
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        if (((c0 / 32) & 1) != eg) continue;  // the two warps of a quarter alternate chunks
        uint32_t r[32];
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0;
        tmem_ld16(taddr, r);
        tmem_ld16(taddr + 16, r + 16);
        tmem_ld_wait();
        const int col0 = nt * BN + c0;
        if (col0 >= N) continue;
        const int valid = min(32, N - col0);
        float v[32];
        scale_chunk32<KD, BN>(r, v, sa, sbt, c0);
        if (KD == Kind::I8 && ep.acc_out != nullptr && row_ok) {
          int32_t* dst = ep.acc_out + (int64_t)row * N + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < valid) dst[j] = (int32_t)r[j];
        }
        if (ep.tma_store) {
          // After tfull every MMA has read its operands: the ring holds the output slabs.
          uint8_t* stg = smem_raw + (size_t)((c0 / 32) * 4 + q) * C::kStageOutBytes;
          uint32_t pk[16];
          pack_out16(v, pk, ep, col0, valid);
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, col0, row0, stg);
            bulk_commit();
          }
        } else if (row_ok) {
          store_direct<KD>(v, ep, (int64_t)row * N + col0, col0, valid, N);
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (ep.tma_store && lane == 0) bulk_wait_read<0>();  // stores have read their slabs
  }

  tc_fence_before();
  cluster_sync_all();  // both epilogues are done with TMEM; no signal to a peer is pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair<C::kTmemCols>(tmem);
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

// K-major operand [rows, cols] (cols contiguous, elem bytes each) tiled as box_rows x 128
// bytes with the 128-byte swizzle; with slices > 1 a 3-D view {128 bytes, rows, 128-byte K
// slices} whose box lands as `slices` consecutive [box_rows][128 B] tiles. Cached per
// (pointer, shape, box).
int make_tmap_kmajor(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int elem,
                     int box_rows, int slices) {
  struct Key {
    const void* p;
    int64_t rows, cols;
    int elem, box, slices;
    bool operator==(const Key& o) const {
      return p == o.p && rows == o.rows && cols == o.cols && elem == o.elem && box == o.box &&
             slices == o.slices;
    }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ (size_t)(k.rows * 1315423911u) ^
             (size_t)(k.cols * 2654435761u) ^ (size_t)(k.box * 97 + k.elem + k.slices * 7919);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{(const char*)ptr + ((int64_t)dev << 56), rows, cols, elem, box_rows, slices};
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
  if (slices > 1 && (cols * elem) % 128 != 0)
    return fail(TO_EINVAL, "K-slice view needs a row length that is a multiple of 128 bytes");
  const CUtensorMapDataType dt =
      elem == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUresult r;
  if (slices <= 1) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * elem)};
    cuuint32_t box[2] = {(cuuint32_t)(128 / elem), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = encode(out, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[3] = {(cuuint64_t)(128 / elem), (cuuint64_t)rows,
                          (cuuint64_t)(cols * elem / 128)};
    cuuint64_t strides[2] = {(cuuint64_t)(cols * elem), 128};
    cuuint32_t box[3] = {(cuuint32_t)(128 / elem), (cuuint32_t)box_rows, (cuuint32_t)slices};
    cuuint32_t estr[3] = {1, 1, 1};
    r = encode(out, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS)
    return fail(TO_ECUDA, "cuTensorMapEncodeTiled failed (%d) for [%lld, %lld] x %d B", (int)r,
                (long long)rows, (long long)cols, elem);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return TO_OK;
}

// Output map for the staged epilogue: C [rows, cols] of 16-bit elements, box = 32 rows x
// box_cols columns; 32-column boxes read a 64-byte-swizzled staging slab, 16-column (tail)
// boxes a plain one with 32-byte rows.
int make_tmap_out16(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int box_cols,
                    int dtype) {
  EncodeFn encode = get_encode();
  if (!encode) return fail(TO_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(out, dtype == TO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      2, const_cast<void*>(ptr), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      box_cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TO_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return TO_OK;
}

int make_tmap_plain(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int elem,
                    int box_cols, int box_rows) {
  struct Key {
    const void* p;
    int64_t rows, cols;
    int elem, bc, br;
    bool operator==(const Key& o) const {
      return p == o.p && rows == o.rows && cols == o.cols && elem == o.elem && bc == o.bc &&
             br == o.br;
    }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ (size_t)(k.rows * 1315423911u) ^
             (size_t)(k.cols * 2654435761u) ^ (size_t)(k.bc * 131 + k.br * 7 + k.elem);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{(const char*)ptr + ((int64_t)dev << 56), rows, cols, elem, box_cols, box_rows};
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
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(out, elem == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                      2, const_cast<void*>(ptr), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TO_ECUDA, "cuTensorMapEncodeTiled (plain) failed (%d) for [%lld, %lld] x %d B",
                (int)r, (long long)rows, (long long)cols, elem);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return TO_OK;
}

// Activations x [M, K] (16-bit, K % 64 == 0, rows ld elements apart) viewed as 64-element
// blocks: dims {64, M, K/64} with strides {ld*2, 128} bytes; one box {64, box_tokens, box_blocks}
// lands as box_blocks tiles of [box_tokens x 128 B], each in the 128-byte-swizzle layout. Cached.
int make_tmap_x_blocks(CUtensorMap* out, const void* ptr, int64_t M, int64_t K, int box_tokens,
                       int box_blocks, int64_t ld) {
  if (ld <= 0) ld = K;
  struct Key {
    const void* p;
    int64_t m, k, ld;
    int bt, bb;
    bool operator==(const Key& o) const {
      return p == o.p && m == o.m && k == o.k && ld == o.ld && bt == o.bt && bb == o.bb;
    }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ (size_t)(k.m * 1315423911u) ^
             (size_t)(k.k * 2654435761u) ^ (size_t)(k.ld * 40503u) ^ (size_t)(k.bt * 131 + k.bb);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const Key key{(const char*)ptr + ((int64_t)dev << 56), M, K, ld, box_tokens, box_blocks};
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
  cuuint64_t dims[3] = {64, (cuuint64_t)M, (cuuint64_t)(K / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_tokens, (cuuint32_t)box_blocks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(ptr), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TO_ECUDA, "cuTensorMapEncodeTiled (x blocks) failed (%d) for [%lld, %lld]", (int)r,
                (long long)M, (long long)K);
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return TO_OK;
}

// B [K, N] of 16-bit elements, N a multiple of 64, as a 3-D view {64 columns, K rows, N / 64
// strips}: one box brings box_rows rows of `strips` consecutive 64-column strips, landing as
// strips of box_rows x 128 bytes (128-byte swizzle) -- the MN-major operand layout.
int make_tmap_mn_strips(CUtensorMap* out, const void* ptr, int64_t K, int64_t N, int box_rows,
                        int strips) {
  EncodeFn encode = get_encode();
  if (!encode) return fail(TO_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (N % 64 != 0) return fail(TO_EINVAL, "MN-major strips need N a multiple of 64");
  cuuint64_t dims[3] = {64, (cuuint64_t)K, (cuuint64_t)(N / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)(N * 2), 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)strips};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(ptr), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(TO_ECUDA, "cuTensorMapEncodeTiled (MN-major strips) failed (%d) for [%lld, %lld]",
                (int)r, (long long)K, (long long)N);
  return TO_OK;
}

template <Kind KD, int BM, int BN, int STAGES, bool KS2 = false, bool BMN = false>
int launch_gemm_cfg(const void* a, const void* b, int64_t M, int64_t N, int64_t K, const Epi& ep,
                    cudaStream_t st) {
  using C = GemmCfg<KD, BM, BN, STAGES>;
  auto kern = k_gemm_sm100<KD, BM, BN, STAGES, KS2, BMN>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)C::kSmem);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "tcgen05 gemm: shared memory attribute");
  CUtensorMap ta, tb, tc32, tc16;
  int rc = make_tmap_kmajor(&ta, a, M, K, C::kElem, BM);
  if (rc) return rc;
  rc = BMN ? make_tmap_mn_strips(&tb, b, K, N, C::kBK, BN / 64)
           : make_tmap_kmajor(&tb, b, N, K, C::kElem, BN);
  if (rc) return rc;
  Epi e2 = ep;
  e2.band = tile_band(BM, K, C::kElem);
  memset(&tc32, 0, sizeof(tc32));
  memset(&tc16, 0, sizeof(tc16));
  if (e2.tma_store) {
    rc = make_tmap_out16(&tc32, e2.c, M, N, 32, e2.c_dtype);
    if (!rc) rc = make_tmap_out16(&tc16, e2.c, M, N, 16, e2.c_dtype);
    if (rc) return rc;
  }
  const int64_t tiles = ceil_div(M, BM) * ceil_div(N, BN);
  if constexpr (KS2) {
    // One tile per CTA pair: the caller guarantees 2 x tiles <= SMs.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * tiles), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc32, tc16, (int)M, (int)N, (int)K, e2,
                                       device_error_ptr());
    if (e != cudaSuccess) return cuda_fail(e, "tcgen05 gemm (K-split pair) launch");
    return check_launch("tcgen05 gemm (K-split pair)");
  } else {
    const int grid = (int)std::min<int64_t>(tiles, sm_count());
    kern<<<grid, kGemmThreads, C::kSmem, st>>>(ta, tb, tc32, tc16, (int)M, (int)N, (int)K, e2,
                                               device_error_ptr());
    return check_launch("tcgen05 gemm");
  }
}

template <Kind KD, int BN, int STAGES, int KC, int MINB = 1>
int launch_gemm_pair(const void* a, const void* b, int64_t M, int64_t N, int64_t K, const Epi& ep,
                     cudaStream_t st) {
  using C = PairCfg<KD, BN, STAGES, KC>;
  auto kern = k_gemm_pair<KD, BN, STAGES, KC, MINB>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)C::kSmem);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "tcgen05 2-CTA gemm: shared memory attribute");
  CUtensorMap ta, tb, tc32, tc16;
  int rc = make_tmap_kmajor(&ta, a, M, K, C::kElem, 128, KC);
  if (!rc) rc = make_tmap_kmajor(&tb, b, N, K, C::kElem, BN / 2, KC);
  if (rc) return rc;
  Epi e2 = ep;
  memset(&tc32, 0, sizeof(tc32));
  memset(&tc16, 0, sizeof(tc16));
  if (e2.tma_store) {
    rc = make_tmap_out16(&tc32, e2.c, M, N, 32, e2.c_dtype);
    if (rc) return rc;
  }
  const int64_t tiles = ceil_div(M, 256) * ceil_div(N, BN);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * tiles), 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (launch_overlap()) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tc32, tc16, (int)M, (int)N, (int)K, e2,
                                     device_error_ptr());
  if (e != cudaSuccess) return cuda_fail(e, "tcgen05 2-CTA gemm launch");
  return check_launch("tcgen05 2-CTA gemm");
}

// Tile shapes: large problems take 128 x 256 tiles; small-M layers (M <= 256, the decode /
// small-batch regime, HBM-bound on B) take the narrowest N tile that still fits every tile
// in one wave, so all SMs stream B at once.
// TOB_GEMM_TILE=<BM>x<BN> forces one of the compiled tile shapes (tuning and tests).
inline int forced_tile() {
  static int v = [] {
    const char* e = tuning_env("TOB_GEMM_TILE");
    if (!e) return 0;
    int bm = 0, bn = 0;
    if (sscanf(e, "%dx%d", &bm, &bn) != 2) return 0;
    return bm * 1000 + bn;
  }();
  return v;
}

template <Kind KD>
int launch_gemm(const void* a, const void* b, int64_t M, int64_t N, int64_t K, const Epi& ep,
                cudaStream_t st) {
  switch (forced_tile()) {
    case 128256: return launch_gemm_cfg<KD, 128, 256, 4>(a, b, M, N, K, ep, st);
    case 128128: return launch_gemm_cfg<KD, 128, 128, 6>(a, b, M, N, K, ep, st);
    case 128064: return launch_gemm_cfg<KD, 128, 64, 8>(a, b, M, N, K, ep, st);
    case 256128: return launch_gemm_cfg<KD, 256, 128, 4>(a, b, M, N, K, ep, st);
    case 256080: return launch_gemm_cfg<KD, 256, 80, 5>(a, b, M, N, K, ep, st);
    case 256064: return launch_gemm_cfg<KD, 256, 64, 5>(a, b, M, N, K, ep, st);
    case 256160: return launch_gemm_cfg<KD, 256, 160, 4, true>(a, b, M, N, K, ep, st);
    default: break;
  }
  const int64_t sms = sm_count();
  auto tiles = [&](int bm, int bn) { return ceil_div(M, bm) * ceil_div(N, bn); };
  // 128 < M <= 256 with every 256 x 160 tile on a CTA pair in one wave: split K over the pair
  // (half the A and B bytes per SM). TOB_GEMM_KSPLIT=0 disables it (measurements).
  static const bool ks2_on = [] {
    const char* v = tuning_env("TOB_GEMM_KSPLIT");
    return v == nullptr || v[0] != '0';
  }();
  // Those with a 16-bit output (TMA-stored rows) run as 2-CTA (cta_group::2) tiles of
  // 256 x 160: the same halved operand bytes per SM, without the partial-sum exchange.
  // TOB_GEMM_PAIR=0 keeps them on the K-split pair (measurements).
  static const bool pair_on = [] {
    const char* v = tuning_env("TOB_GEMM_PAIR");
    return v == nullptr || v[0] != '0';
  }();
  if (pair_on && M > 128 && M <= 256 && 2 * tiles(256, 160) <= sms && ep.tma_store) {
    // K slices per copy (measurement override TOB_PAIR_SLICES = 1, 2 or 4)
    static const int slices = [] {
      const char* v = tuning_env("TOB_PAIR_SLICES");
      return v == nullptr ? 2 : atoi(v);
    }();
    if ((K * KindTraits<KD>::kElemBytes) % 128 != 0 || slices == 1)
      return launch_gemm_pair<KD, 160, 8, 1>(a, b, M, N, K, ep, st);
    if (slices == 4) return launch_gemm_pair<KD, 160, 2, 4>(a, b, M, N, K, ep, st);
    return launch_gemm_pair<KD, 160, 4, 2>(a, b, M, N, K, ep, st);
  }
  if (ks2_on && M > 128 && M <= 256 && 2 * tiles(256, 160) <= sms && K >= 2 * (128 / KindTraits<KD>::kElemBytes))
    return launch_gemm_cfg<KD, 256, 160, 4, true>(a, b, M, N, K, ep, st);
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

template <Kind KD, int kStages, int KC>
int launch_gemm_bs(const void* a, const void* b, int64_t M, int64_t N, int64_t K, const Epi& ep,
                   cudaStream_t st) {
  using C = BsCfg<KD, kStages, KC>;
  auto kern = k_gemm_bs<KD, kStages, KC>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)C::kSmem);
  if (attr_err != cudaSuccess)
    return cuda_fail(attr_err, "tcgen05 block-scaled gemm: shared memory attribute");
  CUtensorMap ta, tb, tc32;
  int rc = make_tmap_kmajor(&ta, a, M, K, C::kElem, 128, KC);
  if (!rc) rc = make_tmap_kmajor(&tb, b, N, K, C::kElem, 128, KC);
  if (rc) return rc;
  memset(&tc32, 0, sizeof(tc32));
  if (ep.tma_store) {
    rc = make_tmap_out16(&tc32, ep.c, M, N, 32, ep.c_dtype);
    if (rc) return rc;
  }
  const int64_t tiles = ceil_div(M, 128) * ceil_div(N, 128);
  kern<<<(unsigned)tiles, kGemmThreads, C::kSmem, st>>>(ta, tb, tc32, (int)M, (int)N, (int)K, ep,
                                                       device_error_ptr());
  return check_launch("tcgen05 block-scaled gemm");
}

}  // namespace sm100

// Routes a W8A8 call to the tcgen05 kernel when its scales are per-row x per-column-block
// (block_k >= K) and the operands meet TMA's alignment rules; otherwise TO_EUNSUPPORTED so
// the caller uses the generic kernel.
int w8a8_tc_launch(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                   void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M, int64_t N,
                   int64_t K, int64_t bn, int64_t bk, cudaStream_t st) {
  if (bk < K) {
    // Per-K-block scales: the block-scaled tiles take block_k = 128 with column blocks that
    // 128-column tiles do not straddle.
    if (bk != 128 || !(bn % 128 == 0 || bn >= N) || acc_out != nullptr) return TO_EUNSUPPORTED;
    if (K % 16 != 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return TO_EUNSUPPORTED;
    if (!aligned16(a) || !aligned16(b)) return TO_EUNSUPPORTED;
    if (M * N < 128 * 128 || ceil_div(M, 128) * ceil_div(N, 128) > INT32_MAX)
      return TO_EUNSUPPORTED;
    const int64_t kt = ceil_div(K, bk);
    sm100::Epi ep;
    memset(&ep, 0, sizeof(ep));
    ep.a_s = a_s;
    ep.a_s_ld = kt;  // a_s [M, kt]
    ep.b_s = b_s;
    ep.b_s_ld = kt;  // b_s [ceil(N / bn), kt]
    ep.bn = bn >= N ? N : bn;
    ep.c = c;
    ep.c_dtype = c_dtype;
    ep.bias = bias;
    ep.acc_out = nullptr;
    ep.policy_a = 0;
    ep.policy_b = 0;
    ep.tma_store = (c_dtype == TO_BF16 || c_dtype == TO_F16) && (N % 8 == 0) && aligned16(c);
    // Two K blocks per copy when K is whole 128-byte slices (each copy costs a roughly fixed
    // time on top of its bytes), else one.
    if (K % 128 == 0)
      return fp8 ? sm100::launch_gemm_bs<sm100::Kind::E4M3, 3, 2>(a, b, M, N, K, ep, st)
                 : sm100::launch_gemm_bs<sm100::Kind::I8, 3, 2>(a, b, M, N, K, ep, st);
    return fp8 ? sm100::launch_gemm_bs<sm100::Kind::E4M3, 6, 1>(a, b, M, N, K, ep, st)
               : sm100::launch_gemm_bs<sm100::Kind::I8, 6, 1>(a, b, M, N, K, ep, st);
  }
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
  ep.tma_store = (c_dtype == TO_BF16 || c_dtype == TO_F16) && (N % 8 == 0) && aligned16(c);
  if (fp8) return sm100::launch_gemm<sm100::Kind::E4M3>(a, b, M, N, K, ep, st);
  return sm100::launch_gemm<sm100::Kind::I8>(a, b, M, N, K, ep, st);
}

int gemm_dense_simt_launch(const void* a, const void* b, void* c, int dtype, int64_t M, int64_t N,
                           int64_t K, cudaStream_t st);

}  // namespace tob

extern "C" {

int to_gemm(const void* a, const void* b, void* c, int dtype, int64_t M, int64_t N, int64_t K,
            void* stream) {
  using namespace tob;
  if (M < 0 || N < 0 || K < 0)
    return fail(TO_EINVAL, "gemm: invalid shape M=%lld N=%lld K=%lld", (long long)M,
                (long long)N, (long long)K);
  if (dtype != TO_F16 && dtype != TO_BF16 && dtype != TO_F32)
    return fail(TO_EUNSUPPORTED, "gemm: dtype %s (float32, float16 and bfloat16 are supported)",
                dtype_name(dtype));
  if (M == 0 || N == 0) return TO_OK;
  if (!a || !b || !c) return fail(TO_EINVAL, "gemm: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 0) {
    const size_t elem = dtype == TO_F32 ? 4 : 2;
    const cudaError_t e = cudaMemsetAsync(c, 0, (size_t)(M * N) * elem, st);
    return e == cudaSuccess ? TO_OK : cuda_fail(e, "gemm: zero fill");
  }
  // TMA constraints of the tcgen05 tiles: 16-bit operands, 16-byte rows of A, whole 64-column
  // strips of B; everything else on the SIMT tiles.
  if (dtype == TO_F32 || K % 8 != 0 || N % 64 != 0 || M > INT32_MAX || N > INT32_MAX ||
      K > INT32_MAX || !aligned16(a) || !aligned16(b) || !aligned16(c))
    return gemm_dense_simt_launch(a, b, c, dtype, M, N, K, st);
  sm100::Epi ep;
  memset(&ep, 0, sizeof(ep));
  ep.a_s = nullptr;  // unscaled: the epilogue multiplies by 1
  ep.b_s = nullptr;
  ep.bn = N;
  ep.c = c;
  ep.c_dtype = dtype;
  ep.tma_store = 1;
  // 256-row tiles (3 stages of 64 KB, one accumulator buffer) halve the copies per MMA; they
  // pay once they fill the SMs, 128-row tiles (4 stages, two accumulator buffers) below that.
  using sm100::Kind;
  if (ceil_div(M, 256) * ceil_div(N, 256) >= sm_count())
    return dtype == TO_F16
               ? sm100::launch_gemm_cfg<Kind::F16, 256, 256, 3, false, true>(a, b, M, N, K, ep, st)
               : sm100::launch_gemm_cfg<Kind::BF16, 256, 256, 3, false, true>(a, b, M, N, K, ep, st);
  return dtype == TO_F16
             ? sm100::launch_gemm_cfg<Kind::F16, 128, 256, 4, false, true>(a, b, M, N, K, ep, st)
             : sm100::launch_gemm_cfg<Kind::BF16, 128, 256, 4, false, true>(a, b, M, N, K, ep, st);
}

}  // extern "C"
