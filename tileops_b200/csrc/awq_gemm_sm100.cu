// AWQ W4A16 GEMM on the sm_100a tensor cores: y[M, N] = x[M, K] @ dequant(W)[K, N]
// (tileops/quant_awq.py:112-155) for prefill-sized M.
//
// The packed int4 weights never exist in HBM as fp16/bf16: each K block of the weight tile is
// TMA-loaded packed (0.5 B per weight), expanded in shared memory by eight dequantising warps
// into the exact reference weights T((w - z) * s) (quant_awq.py:104-109), and consumed by
// tcgen05.mma kind::f16 straight from there.
//
// Per CTA (persistent, one per SM, 448 threads), tile (128 HALVES) x BN, K blocks of 64:
//   warp 0      TMA producer, 3-5-deep ring: x tile [128 HALVES x 64] (K-major, 128B swizzle),
//               packed weights [64 rows x BN/8 words], the block's scale and zero rows -> full[s]
//   warps 2-9   dequantise into one of two B buffers: one packed word (8 columns at one k) ->
//               one 16-byte store, MN-major with the 128-byte swizzle          -> bready[b]
//   warp 1      MMA: 4 x HALVES tcgen05.mma (M = 128, N = BN, K = 16), the HALVES row halves of
//               x sharing each B slice; A K-major, B MN-major
//               -> empty[s] (ring slot), bfree[b] (B buffer), tfull (tile done)
//   warps 10-13 epilogue: TMEM -> bf16/fp16 -> 64B-swizzled staging -> TMA store -> tempty
// The deep TMA ring hides load latency; the separate B buffers let dequantisation of block
// k+1 overlap the MMAs of block k. 128-row tiles double-buffer their accumulators in TMEM
// (2 x 256 columns); 256-row tiles use all 512 columns for one tile (over a K of thousands, the
// un-overlapped epilogue is about 1% of the tile). The expansion's shared-memory stores and the
// tensor core's reads of B bound the kernel, which is why 256-row tiles pay.
// Waits are bounded (sm100.cuh).
#include <string.h>

#include <mutex>

#include "awq_common.cuh"
#include "sm100.cuh"

namespace tob {
namespace sm100 {
namespace {

constexpr int kAwqBK = 64;
constexpr int kAwqDqWarps = 8;  // dequantising warps
constexpr int kAwqThreads = 64 + 32 * kAwqDqWarps + 128;
constexpr int kAwqEpiWarp0 = 2 + kAwqDqWarps;
constexpr int kAwqSZBytes = 2048;  // scales + zeros of up to 2 group rows, padded
constexpr int kAwqOutBytes = 4 * 32 * 32 * 2;  // 4 epilogue warps x one 32 x 32 slab
// B operand layout (MN-major, 128B swizzle): 1 KB atoms of 8 k-rows x 64 columns; the 8 atoms
// of a 64-column strip are contiguous along K, strips are 8 KB apart.
constexpr uint32_t kAwqBLbo = 8192, kAwqBSbo = 1024;

// Tile shapes. A tile is (128 HALVES) x BN: HALVES M=128 MMAs share every dequantised B tile,
// so each packed weight is expanded once per 128 HALVES rows of x (the expansion's shared-memory
// stores and the tensor core's B reads bound this kernel; 256-row tiles halve them per MMA).
// BN = 256, or 224 when 224-column tiles fill the SMs in fewer rounds.
// BBUFS: dequantised B tiles in flight. Three (one TMA stage fewer for the 256 x 224 tiles) ran
// the M=2048 K=8192 N=28672 layer at 988 TFLOP/s against 1309 with two.
template <int HALVES, int BN, int BBUFS = 2>
struct AwqCfg {
  static constexpr int kBBufs = BBUFS;  // dequantised B tiles in flight
  static constexpr int kBM = 128 * HALVES;
  static constexpr int kABytes = kBM * 128;          // x tile, 64 bf16/fp16 per row
  static constexpr int kWBytes = kAwqBK * BN / 2;    // packed words (64 rows x BN / 8)
  static constexpr int kBBytes = kAwqBK * 256 * 2;   // dequantised B (4 strips, 32 KB)
  static constexpr int kStageBytes = kABytes + kWBytes + kAwqSZBytes;
  // TMEM: HALVES x BN accumulator columns per buffer; two buffers when they fit in 512.
  static constexpr int kAccCols = HALVES * BN;
  static constexpr int kAccBufs = kAccCols <= 256 ? 2 : 1;
  static constexpr int kAccStride = kAccBufs == 2 ? 256 : 0;
  static constexpr int kStages =
      (int)((232448 - 256 - kBBufs * kBBytes - kAwqOutBytes) / kStageBytes) > 5
          ? 5
          : (int)((232448 - 256 - kBBufs * kBBytes - kAwqOutBytes) / kStageBytes);
  static constexpr size_t kSmem =
      (size_t)kStages * kStageBytes + (size_t)kBBufs * kBBytes + kAwqOutBytes + 256;
  // dequantisation: thread dt owns word column dt % kWords of rows dt / kWords + kRowStep i
  static constexpr int kWords = BN / 8;
  static constexpr int kRowStep = (32 * kAwqDqWarps) / kWords;
  static_assert(kStages >= 2 && kSmem <= 232448, "shared memory");
  static_assert(BN % 32 == 0 && BN <= 256, "tile width");
};

// Output tensor maps: one per destination. A plain call has one (this GPU's y); the gathering
// form of an N-sharded layer has one per rank of the group (the peers' [M, N_full] outputs,
// mapped into this process), each tile being stored to all of them at column offset ycol0.
constexpr int kAwqMaxRanks = 8;
struct AwqOutMaps {
  CUtensorMap m[kAwqMaxRanks];
};

__device__ __forceinline__ int awq_k_start(int t, int kblocks) {
  return (int)(((unsigned)t * 5u) % (unsigned)kblocks);
}

template <typename T, int HALVES, int BN, int BBUFS>
__global__ void __launch_bounds__(kAwqThreads, 1)
    k_awq_gemm_sm100(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ,
                     const __grid_constant__ AwqOutMaps ym, int ny, int ycol0, int M, int N,
                     int K, int G, int group_rows, int* err) {
  using H = Half2Of<T>;
  using H2 = typename H::type;
  using C = AwqCfg<HALVES, BN, BBUFS>;
  constexpr int kAwqBBufs = C::kBBufs;
  constexpr Kind KD = std::is_same<T, __half>::value ? Kind::F16 : Kind::BF16;
  using Tr = KindTraits<KD>;
  constexpr int kSBytes = 2 * BN * 2;  // up to 2 scale rows (group 32)
  static_assert(kSBytes + 2 * C::kWords * 4 <= kAwqSZBytes, "scale/zero area");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* stage0 = smem_raw;
  uint8_t* bbase = smem_raw + (size_t)C::kStages * C::kStageBytes;
  uint8_t* sOut = bbase + (size_t)kAwqBBufs * C::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + kAwqOutBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* bready = empty + C::kStages;
  uint64_t* bfree = bready + kAwqBBufs;
  uint64_t* tfull = bfree + kAwqBBufs;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  auto sA = [&](int s) { return stage0 + (size_t)s * C::kStageBytes; };
  auto sW = [&](int s) { return stage0 + (size_t)s * C::kStageBytes + C::kABytes; };
  auto sS = [&](int s) { return stage0 + (size_t)s * C::kStageBytes + C::kABytes + C::kWBytes; };
  auto sZ = [&](int s) { return sS(s) + kSBytes; };
  auto sB = [&](int b) { return bbase + (size_t)b * C::kBBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (M + C::kBM - 1) / C::kBM, n_tiles = (N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles;
  const int kblocks = (K + kAwqBK - 1) / kAwqBK;
  const uint32_t stage_tx = C::kABytes + C::kWBytes + group_rows * (BN * 2 + C::kWords * 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < kAwqBBufs; ++b) {
      mbar_init(bready + b, kAwqDqWarps);
      mbar_init(bfree + b, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
    prefetch_tmap(&tmZ);
    for (int r = 0; r < ny; ++r) prefetch_tmap(&ym.m[r]);
  }
  if (warp == 0) tmem_alloc<512>(tmem_holder);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const bool misaligned = (smem_u32(smem_raw) & 1023u) != 0;
  if (misaligned && threadIdx.x == 0 && err) atomicExch(err, (int)kErrSmemAlign);

  if (misaligned) {
  } else if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();  // x and the weight tile are re-read by other CTAs
      uint32_t s = 0, ph = 0, issued_mask = 0, issued_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mt = t % m_tiles, nt = t / m_tiles;
        const int k0 = awq_k_start(t, kblocks);
        for (int it = 0; it < kblocks; ++it) {
          const int kb = (k0 + it) % kblocks;
          if (!mbar_wait(empty + s, ph ^ 1, abort_flag, err)) { ok = false; break; }
          mbar_arrive_expect_tx(full + s, stage_tx);
          const int g0 = group_rows == 1 ? (kb * kAwqBK) / G : kb * group_rows;
          tma_load_2d(sA(s), &tmX, kb * kAwqBK, mt * C::kBM, full + s, pol);
          tma_load_2d(sW(s), &tmW, nt * C::kWords, kb * kAwqBK, full + s, pol);
          tma_load_2d(sS(s), &tmS, nt * BN, g0, full + s, pol);
          tma_load_2d(sZ(s), &tmZ, nt * C::kWords, g0, full + s, pol);
          issued_mask |= 1u << s;
          issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
          if (++s == C::kStages) { s = 0; ph ^= 1; }
        }
      }
      if (!ok) {
        for (int i = 0; i < C::kStages; ++i)
          if (issued_mask & (1u << i)) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(full + i, (issued_phase >> i) & 1u) &&
                   globaltimer_ns() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_major(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 128, BN, 0, 1);
      uint32_t s = 0, ph = 0, bb = 0, bph = 0;
      int i = 0;
      bool ok = true, any = false;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++i) {
        const int buf = C::kAccBufs == 2 ? (i & 1) : 0;
        const uint32_t aph = (uint32_t)(C::kAccBufs == 2 ? (i >> 1) : i) & 1u;
        if (!mbar_wait(tempty + buf, aph ^ 1, abort_flag, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(buf * C::kAccStride);
        for (int it = 0; it < kblocks; ++it) {
          if (!mbar_wait(full + s, ph, abort_flag, err) ||
              !mbar_wait(bready + bb, bph, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA(s)), b0 = smem_u32(sB(bb));
#pragma unroll
          for (int k = 0; k < kAwqBK / 16; ++k) {
            const uint64_t bdesc = smem_desc_mnmajor_sw128(b0 + 2048 * k, kAwqBLbo, kAwqBSbo);
#pragma unroll
            for (int h = 0; h < HALVES; ++h) {
              const uint64_t adesc = smem_desc_kmajor_sw128(a0 + 16384 * h + 32 * k);
              umma<KD>(d0 + (uint32_t)(h * BN), adesc, bdesc, idesc, (it | k) != 0);
            }
          }
          any = true;
          umma_commit(empty + s);
          umma_commit(bfree + bb);
          if (++s == C::kStages) { s = 0; ph ^= 1; }
          if (++bb == kAwqBBufs) { bb = 0; bph ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull + buf);
      }
      if (!ok && any) {
        umma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp < kAwqEpiWarp0) {
    // ------------------------------------------------------------ dequantise
    // Thread dt owns the 8-column chunk wc = dt % kWords of every row r = dt / kWords +
    // kRowStep i (threads past kWords x kRowStep only take part in the barriers).
    constexpr int kRowStep = C::kRowStep;
    constexpr int kRowsPer = (kAwqBK + kRowStep - 1) / kRowStep;
    const int dt = threadIdx.x - 64;
    const int wc = dt % C::kWords, r0 = dt / C::kWords;
    const bool active = r0 < kRowStep;
    const int an = wc >> 3, cc = wc & 7;  // 64-column strip and 16-byte chunk within it
    uint32_t s = 0, ph = 0, bb = 0, bph = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      for (int it = 0; it < kblocks; ++it) {
        if (!mbar_wait(full + s, ph, abort_flag, err) ||
            !mbar_wait(bfree + bb, bph ^ 1, abort_flag, err)) {
          ok = false;
          break;
        }
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(sW(s));
        const uint4* sp = reinterpret_cast<const uint4*>(sS(s));
        const uint32_t* zp = reinterpret_cast<const uint32_t*>(sZ(s));
        uint8_t* bp = sB(bb);
        if (!active) {
        } else if (group_rows == 1) {
          // One quantisation group covers the whole K block: constants once, then every load
          // of the thread's rows before any arithmetic.
          H2 zc[4], sc[4];
          awq_zero_consts<T>(zp[wc], zc);
          const uint4 sv = sp[wc];
          sc[0] = H::from_bits(sv.x);
          sc[1] = H::from_bits(sv.y);
          sc[2] = H::from_bits(sv.z);
          sc[3] = H::from_bits(sv.w);
          uint32_t wv[kRowsPer];
#pragma unroll
          for (int i = 0; i < kRowsPer; ++i) {
            const int r = r0 + kRowStep * i;
            wv[i] = r < kAwqBK ? wp[r * C::kWords + wc] : 0u;
          }
#pragma unroll
          for (int i = 0; i < kRowsPer; ++i) {
            const int r = r0 + kRowStep * i;
            if (r >= kAwqBK) break;
            H2 d[4];
            awq_word_diff<T>(wv[i], zc, d);
            uint4 o;
            o.x = bits_of(__hmul2(d[0], sc[0]));
            o.y = bits_of(__hmul2(d[1], sc[1]));
            o.z = bits_of(__hmul2(d[2], sc[2]));
            o.w = bits_of(__hmul2(d[3], sc[3]));
            const int rr = r & 7;
            *reinterpret_cast<uint4*>(bp + an * kAwqBLbo + (r >> 3) * kAwqBSbo + rr * 128 +
                                      ((cc ^ rr) << 4)) = o;
          }
        } else {
          int cur_g = -1;
          H2 zc[4], sc[4];
#pragma unroll
          for (int i = 0; i < kRowsPer; ++i) {
            const int r = r0 + kRowStep * i;
            if (r >= kAwqBK) break;
            const int gl = r / G;  // group row of this k within the block
            if (gl != cur_g) {
              cur_g = gl;
              awq_zero_consts<T>(zp[gl * C::kWords + wc], zc);
              const uint4 sv = sp[gl * C::kWords + wc];
              sc[0] = H::from_bits(sv.x);
              sc[1] = H::from_bits(sv.y);
              sc[2] = H::from_bits(sv.z);
              sc[3] = H::from_bits(sv.w);
            }
            H2 d[4];
            awq_word_diff<T>(wp[r * C::kWords + wc], zc, d);
            uint4 o;
            o.x = bits_of(__hmul2(d[0], sc[0]));
            o.y = bits_of(__hmul2(d[1], sc[1]));
            o.z = bits_of(__hmul2(d[2], sc[2]));
            o.w = bits_of(__hmul2(d[3], sc[3]));
            const int rr = r & 7;
            *reinterpret_cast<uint4*>(bp + an * kAwqBLbo + (r >> 3) * kAwqBSbo + rr * 128 +
                                      ((cc ^ rr) << 4)) = o;
          }
        }
        fence_proxy_async_smem();  // make the generic stores visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(bready + bb);
        if (++s == C::kStages) { s = 0; ph ^= 1; }
        if (++bb == kAwqBBufs) { bb = 0; bph ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int buf = C::kAccBufs == 2 ? (i & 1) : 0;
      const uint32_t aph = (uint32_t)(C::kAccBufs == 2 ? (i >> 1) : i) & 1u;
      if (!mbar_wait(tfull + buf, aph, abort_flag, err)) break;
      tc_fence_after();
      const int mt = t % m_tiles, nt = t / m_tiles;
      uint8_t* stg = sOut + (size_t)(warp - kAwqEpiWarp0) * (32 * 32 * 2);
#pragma unroll 1
      for (int h = 0; h < HALVES; ++h) {
        const int row0 = mt * C::kBM + h * 128 + q * 32;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) +
                                 (uint32_t)(buf * C::kAccStride + h * BN + c0);
          tmem_ld16(taddr, r);
          tmem_ld16(taddr + 16, r + 16);
          tmem_ld_wait();
          if (nt * BN + c0 >= N || row0 >= M) continue;
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float a = __uint_as_float(r[j]), b = __uint_as_float(r[j + 1]);
            if constexpr (std::is_same<T, __half>::value) {
              __half2 o = __floats2half2_rn(a, b);
              pk[j / 2] = bits_of(o);
            } else {
              __nv_bfloat162 o = __floats2bfloat162_rn(a, b);
              pk[j / 2] = bits_of(o);
            }
          }
          if (lane < ny) bulk_wait_read<0>();  // the slab's previous stores have read it
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stg + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane < ny) {
            // One destination per lane: copies issued by different threads proceed in
            // parallel. Rotated by tile, so the ranks' stores spread over the links.
            tma_store_2d(&ym.m[(lane + t) % ny], ycol0 + nt * BN + c0, row0, stg);
            bulk_commit();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + buf);
    }
    if (lane < ny) {
      if (ny > 1) {
        // Peers' outputs: the stores have completed and are ordered before whatever this
        // GPU signals to the peers after the kernel.
        bulk_wait_all();
        __threadfence_system();
      } else {
        bulk_wait_read<0>();  // stores have read their slabs
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// Tile rounds of the persistent grid (one CTA per SM) for a tile shape.
inline int64_t awq_rounds(int64_t M, int64_t N, int bm, int bn, int64_t sms) {
  const int64_t tiles = ceil_div(M, bm) * ceil_div(N, bn);
  return ceil_div(tiles, sms);
}

template <typename T, int HALVES, int BN, int BBUFS = 2>
int launch_awq_gemm_cfg(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                        void* const* ys, int ny, int64_t n_full, int64_t ycol0, int64_t M,
                        int64_t K, int64_t N, int64_t G, int dtype, cudaStream_t st) {
  using C = AwqCfg<HALVES, BN, BBUFS>;
  auto kern = k_awq_gemm_sm100<T, HALVES, BN, BBUFS>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)C::kSmem);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "awq tcgen05 gemm: shared memory attribute");
  if (ny < 1 || ny > kAwqMaxRanks) return fail(TO_EINVAL, "awq tcgen05 gemm: %d outputs", ny);
  const int group_rows = G >= kAwqBK ? 1 : (int)(kAwqBK / G);
  CUtensorMap tx, tw, ts, tz;
  AwqOutMaps ym;
  memset(&ym, 0, sizeof(ym));
  int rc = make_tmap_kmajor(&tx, x, M, K, 2, C::kBM);
  if (!rc) rc = make_tmap_plain(&tw, qw, K, N / 8, 4, C::kWords, kAwqBK);
  if (!rc) rc = make_tmap_plain(&ts, s, K / G, N, 2, BN, group_rows);
  if (!rc) rc = make_tmap_plain(&tz, qz, K / G, N / 8, 4, C::kWords, group_rows);
  for (int r = 0; !rc && r < ny; ++r) rc = make_tmap_out16(&ym.m[r], ys[r], M, n_full, 32, dtype);
  if (rc) return rc;
  const int64_t tiles = ceil_div(M, C::kBM) * ceil_div(N, BN);
  const int grid = (int)std::min<int64_t>(tiles, sm_count());
  kern<<<grid, kAwqThreads, C::kSmem, st>>>(tx, tw, ts, tz, ym, ny, (int)ycol0, (int)M, (int)N,
                                            (int)K, (int)G, group_rows, device_error_ptr());
  return check_launch("awq tcgen05 gemm");
}

// Tile shape: 256-row tiles (each B tile expanded once for 256 rows of x) once M reaches 256,
// 224 columns wide instead of 256 when the rounds of tiles over the SMs times the tile width
// is smaller (M=2048, N=28672: 1024 tiles in 7 rounds instead of 896 in 7, the last nearly
// empty); 128-row tiles below (measurement override TOB_AWQ_TILE=1 keeps 128 x 256 tiles).
template <typename T>
int launch_awq_gemm(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                    void* const* ys, int ny, int64_t n_full, int64_t ycol0, int64_t M, int64_t K,
                    int64_t N, int64_t G, int dtype, cudaStream_t st) {
  static const bool narrow = [] {
    const char* v = tuning_env("TOB_AWQ_TILE");
    return v != nullptr && v[0] == '1';
  }();
  const int64_t sms = sm_count();
  if (!narrow && M >= 256) {
    if (awq_rounds(M, N, 256, 224, sms) * 224 < awq_rounds(M, N, 256, 256, sms) * 256)
      return launch_awq_gemm_cfg<T, 2, 224>(x, qw, s, qz, ys, ny, n_full, ycol0, M, K, N, G,
                                            dtype, st);
    return launch_awq_gemm_cfg<T, 2, 256>(x, qw, s, qz, ys, ny, n_full, ycol0, M, K, N, G, dtype,
                                          st);
  }
  return launch_awq_gemm_cfg<T, 1, 256>(x, qw, s, qz, ys, ny, n_full, ycol0, M, K, N, G, dtype,
                                        st);
}

}  // namespace
}  // namespace sm100

// Routes an AWQ GEMM to the tensor-core kernel when the shapes meet its TMA constraints;
// TO_EUNSUPPORTED (no error recorded) otherwise.
int awq_gemm_tc_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                       const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                       cudaStream_t st) {
  if (s_dtype != TO_F16 && s_dtype != TO_BF16) return TO_EUNSUPPORTED;
  if (N % 32 != 0 || K % 8 != 0) return TO_EUNSUPPORTED;  // 16-byte TMA row strides
  if (!(G % 64 == 0 || G == 32 || G == K)) return TO_EUNSUPPORTED;
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return TO_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(qw) || !aligned16(s) || !aligned16(qz) || !aligned16(y))
    return TO_EUNSUPPORTED;
  void* ys[1] = {y};
  if (s_dtype == TO_F16)
    return sm100::launch_awq_gemm<__half>(x, qw, s, qz, ys, 1, N, 0, M, K, N, G, s_dtype, st);
  return sm100::launch_awq_gemm<__nv_bfloat16>(x, qw, s, qz, ys, 1, N, 0, M, K, N, G, s_dtype,
                                               st);
}

// The gathering form for a layer whose N columns are split over `world` ranks: this rank's
// [M, N] slice is stored into the [M, N * world] output of every rank (y_ranks[r], mapped into
// this process) at columns [rank * N, (rank + 1) * N). TO_EUNSUPPORTED when the shapes do not
// meet the kernel's TMA constraints (nothing launched).
int awq_gemm_tc_gather_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                              const int32_t* qz, void* const* y_ranks, int world, int rank,
                              int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st) {
  if (s_dtype != TO_F16 && s_dtype != TO_BF16) return TO_EUNSUPPORTED;
  if (N % 32 != 0 || K % 8 != 0) return TO_EUNSUPPORTED;
  if (!(G % 64 == 0 || G == 32 || G == K)) return TO_EUNSUPPORTED;
  if (M > INT32_MAX || N * world > INT32_MAX || K > INT32_MAX) return TO_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(qw) || !aligned16(s) || !aligned16(qz)) return TO_EUNSUPPORTED;
  for (int r = 0; r < world; ++r)
    if (!aligned16(y_ranks[r])) return TO_EUNSUPPORTED;
  const int64_t n_full = N * world, col0 = N * rank;
  if (s_dtype == TO_F16)
    return sm100::launch_awq_gemm<__half>(x, qw, s, qz, y_ranks, world, n_full, col0, M, K, N,
                                          G, s_dtype, st);
  return sm100::launch_awq_gemm<__nv_bfloat16>(x, qw, s, qz, y_ranks, world, n_full, col0, M, K,
                                               N, G, s_dtype, st);
}

}  // namespace tob
