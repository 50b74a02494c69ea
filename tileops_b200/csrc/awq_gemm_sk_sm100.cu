// AWQ W4A16 GEMM for 1-128 tokens on the sm_100a tensor cores, with the work spread over every
// SM ("stream-K"): y[M, N] = x[M, K] @ dequant(W)[K, N] (tileops/quant_awq.py:112-155).
//
// The prefill kernel (awq_gemm_sm100.cu) gives each CTA whole 128 x 256 output tiles. At these
// token counts a layer has only N / 256 tiles (16 for a 4096-wide layer, 112 for 28672), so
// most SMs would sit idle. This kernel keeps that data path -- a TMA ring bringing the x block
// (128 rows, zero-filled past M) and the packed weights of a 64 x 256 block, eight warps
// expanding the packed words into the exact reference weights T((w - z) * s) in shared memory
// (MN-major, 128-byte swizzle), tcgen05.mma kind::f16 (M = 128, N = 256, K = 16) accumulating
// in TMEM -- and splits the K blocks of every tile over the CTAs:
//   * units are (column tile, 64-row K block), numbered tile-major, K-minor; CTA b of a grid of
//     P <= #SMs takes units [b U / P, (b + 1) U / P), so every SM expands the same number of
//     weight blocks whatever N / 256 is;
//   * a CTA's consecutive units of one tile (a "tile part") accumulate in one of two TMEM
//     buffers; the epilogue warps (lane = row of x) either leave the part's fp32 sums in a
//     caller workspace behind a flag carrying a per-launch epoch (a later K range of a tile), or
//     -- in the CTA holding the tile's first K block, the "owner" -- add the other parts' sums
//     in K order (deterministic), round, and store y (optionally act(gate) * up of a gate_up
//     linear interleaved in blocks of 8 columns, and to every rank's output of an N-sharded
//     layer). The owner reaches that tile at the end of its range and the other CTAs at the
//     start of theirs, so its wait is short; every wait is bounded.
// Roles (448 threads): warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 expansion, warps 10-13
// epilogue. Each SM expands about one 64 x 256 block per 1.2 us here (tensor pipe ~30 % busy,
// 0.4 eligible warps per scheduler), so the kernel pays off only where the alternatives leave
// SMs idle for a long K: the dispatch (awq.cu) sends it 33-128 tokens on layers of K >= 8192 and
// at most 32 column tiles.
#include <string.h>

#include <algorithm>
#include <atomic>
#include <chrono>

#include <unistd.h>

#include "act.cuh"
#include "awq_common.cuh"
#include "sm100.cuh"

namespace tob {
namespace sm100 {
namespace {

constexpr int kSkBK = 64;                                   // K rows per unit
constexpr int kSkBN = 256;                                  // columns per tile
constexpr int kSkWords = kSkBN / 8;                         // packed words per tile row
constexpr int kSkDqWarps = 8;                               // expanding warps
constexpr int kSkThreads = 64 + 32 * kSkDqWarps + 128;      // 448
constexpr int kSkEpiWarp0 = 2 + kSkDqWarps;                 // first epilogue warp
constexpr int kSkABytes = 128 * 128;                        // x block: 128 rows x 64 16-bit
constexpr int kSkWBytes = kSkBK * kSkWords * 4;             // packed block: 8 KB
constexpr int kSkSZBytes = 2048;                            // scale + zero rows (up to 2)
constexpr int kSkStageBytes = kSkABytes + kSkWBytes + kSkSZBytes;  // 26 KB
constexpr int kSkBBytes = kSkBK * kSkBN * 2;                // expanded block: 32 KB
// Expanded blocks in flight. Three (with four stages) measured the same as two on the decode
// shapes (89.9 against 89.8 us on 128 x 14336 x 4096): the hand-off depth is not the limit.
constexpr int kSkBBufs = 2;
constexpr int kSkStages = 6;
constexpr size_t kSkSmem = (size_t)kSkStages * kSkStageBytes + (size_t)kSkBBufs * kSkBBytes + 256;
// Expanded-weight layout (MN-major, 128B swizzle): 1 KB atoms of 8 K rows x 64 columns; the 8
// atoms of a 64-column strip are contiguous along K, strips 8 KB apart.
constexpr uint32_t kSkBLbo = 8192, kSkBSbo = 1024;
constexpr int kSkRowStep = (32 * kSkDqWarps) / kSkWords;    // 8 rows apart per thread
constexpr int kSkRowsPer = kSkBK / kSkRowStep;              // 8 rows per thread
constexpr int kSkMaxOut = 8;
// Row stride (floats) of the owner's sum of the later parts in shared memory: 16 bytes of
// padding per row, so a warp's lanes (one row each) read the same columns conflict-free.
constexpr int kSkRedLd = kSkBN + 4;
// (the stage ring and the expanded-weight buffers after it, both idle by then)
static_assert(128 * kSkRedLd * 4 <= kSkStages * kSkStageBytes + kSkBBufs * kSkBBytes,
              "owner sums fit in the ring");
static_assert(kSkSmem <= 232448, "shared memory");
static_assert(kSkStageBytes % 1024 == 0, "stages keep the 1 KB alignment of the swizzled x");

// Where the output goes (as the decode kernel's): this GPU's y, or every rank's [M, ld] output
// at column col0 of an N-sharded layer; act >= 0: a gate_up linear interleaved in blocks of 8
// columns whose output is act(gate) * up, N / 2 columns (col0 and ld count those).
struct SkOut {
  void* y[kSkMaxOut];
  int ny, ld, col0, act;
};

__host__ __device__ __forceinline__ int64_t sk_start(int64_t b, int64_t units, int64_t ctas) {
  return b * units / ctas;
}
__host__ __device__ __forceinline__ int64_t sk_cta_of(int64_t u, int64_t units, int64_t ctas) {
  return ((u + 1) * ctas - 1) / units;
}

__device__ __forceinline__ unsigned long long sk_ld_relaxed(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void sk_st_release(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  return bits_of(Half2Of<T>::from_floats(a, b));
}

template <typename T>
__global__ void __launch_bounds__(kSkThreads, 1)
    k_awq_gemm_sk(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                  const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ,
                  const SkOut out, float* __restrict__ part,
                  unsigned long long* __restrict__ flags, int M, int N, int G, int group_rows,
                  int kbn, int units, int maxc, unsigned long long epoch, int* err) {
  using H = Half2Of<T>;
  using H2 = typename H::type;
  constexpr Kind KD = std::is_same<T, __half>::value ? Kind::F16 : Kind::BF16;
  using Tr = KindTraits<KD>;
  constexpr int kSBytes = 2 * kSkBN * 2;  // up to 2 scale rows (group 32)

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* stage0 = smem_raw;
  uint8_t* bbase = smem_raw + (size_t)kSkStages * kSkStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(bbase + (size_t)kSkBBufs * kSkBBytes);
  uint64_t* empty = full + kSkStages;
  uint64_t* bready = empty + kSkStages;
  uint64_t* bfree = bready + kSkBBufs;
  uint64_t* tfull = bfree + kSkBBufs;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* redbar = drain + 1;  // the epilogue threads' sums of later parts are in place
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(redbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  auto sA = [&](int s) { return stage0 + (size_t)s * kSkStageBytes; };
  auto sW = [&](int s) { return stage0 + (size_t)s * kSkStageBytes + kSkABytes; };
  auto sS = [&](int s) { return stage0 + (size_t)s * kSkStageBytes + kSkABytes + kSkWBytes; };
  auto sZ = [&](int s) { return sS(s) + kSBytes; };
  auto sB = [&](int b) { return bbase + (size_t)b * kSkBBytes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = (int)sk_start(blockIdx.x, units, gridDim.x);
  const int n = (int)sk_start(blockIdx.x + 1, units, gridDim.x) - u0;
  const uint32_t stage_tx = kSkABytes + kSkWBytes + group_rows * (kSkBN * 2 + kSkWords * 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSkStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < kSkBBufs; ++b) {
      mbar_init(bready + b, kSkDqWarps);
      mbar_init(bfree + b, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, 4);
    }
    mbar_init(drain, 1);
    mbar_init(redbar, 128);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
    prefetch_tmap(&tmZ);
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
      const uint64_t pol_w = policy_evict_first();  // each weight block is read once
      const uint64_t pol_x = policy_evict_last();   // x blocks are read by every column tile
      uint32_t s = 0, ph = 0, issued_mask = 0, issued_phase = 0;
      int t = u0 / kbn, kb = u0 % kbn;
      bool ok = true;
      for (int i = 0; i < n; ++i) {
        if (!mbar_wait(empty + s, ph ^ 1, abort_flag, err)) { ok = false; break; }
        mbar_arrive_expect_tx(full + s, stage_tx);
        const int g0 = group_rows == 1 ? (kb * kSkBK) / G : kb * group_rows;
        tma_load_2d(sA(s), &tmX, kb * kSkBK, 0, full + s, pol_x);
        tma_load_2d(sW(s), &tmW, t * kSkWords, kb * kSkBK, full + s, pol_w);
        tma_load_2d(sS(s), &tmS, t * kSkBN, g0, full + s, pol_w);
        tma_load_2d(sZ(s), &tmZ, t * kSkWords, g0, full + s, pol_w);
        issued_mask |= 1u << s;
        issued_phase = (issued_phase & ~(1u << s)) | (ph << s);
        if (++s == kSkStages) { s = 0; ph ^= 1; }
        if (++kb == kbn) { kb = 0; ++t; }
      }
      if (!ok) {
        for (int i = 0; i < kSkStages; ++i)
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
      constexpr uint32_t idesc =
          make_idesc_major(Tr::kDFmt, Tr::kAFmt, Tr::kBFmt, 128, kSkBN, 0, 1);
      uint32_t s = 0, ph = 0, bb = 0, bph = 0;
      int kb = u0 % kbn, p = 0;
      bool ok = true, any = false;
      for (int i = 0; i < n; ++i) {
        const bool first = i == 0 || kb == 0, last = i == n - 1 || kb == kbn - 1;
        const int buf = p & 1;
        if (first) {
          if (!mbar_wait(tempty + buf, ((p >> 1) & 1) ^ 1, abort_flag, err)) { ok = false; break; }
          tc_fence_after();
        }
        if (!mbar_wait(full + s, ph, abort_flag, err) ||
            !mbar_wait(bready + bb, bph, abort_flag, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA(s)), b0 = smem_u32(sB(bb));
        const uint32_t d0 = tmem + (uint32_t)(buf * kSkBN);
#pragma unroll
        for (int k = 0; k < kSkBK / 16; ++k) {
          const uint64_t bdesc = smem_desc_mnmajor_sw128(b0 + 2048 * k, kSkBLbo, kSkBSbo);
          const uint64_t adesc = smem_desc_kmajor_sw128(a0 + 32 * k);
          umma<KD>(d0, adesc, bdesc, idesc, (first && k == 0) ? 0u : 1u);
        }
        any = true;
        umma_commit(empty + s);
        umma_commit(bfree + bb);
        if (last) {
          umma_commit(tfull + buf);
          ++p;
        }
        if (++s == kSkStages) { s = 0; ph ^= 1; }
        if (++bb == kSkBBufs) { bb = 0; bph ^= 1; }
        if (++kb == kbn) kb = 0;
      }
      if (!ok && any) {
        umma_commit(drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp < kSkEpiWarp0) {
    // ------------------------------------------------------------ expansion
    // Thread dt owns the 8-column chunk wc = dt % 32 of rows r0 + 8 i of every block.
    const int dt = threadIdx.x - 64;
    const int wc = dt % kSkWords, r0 = dt / kSkWords;
    const int an = wc >> 3, cc = wc & 7;  // 64-column strip and 16-byte chunk within it
    uint32_t s = 0, ph = 0, bb = 0, bph = 0;
    for (int i = 0; i < n; ++i) {
      if (!mbar_wait(full + s, ph, abort_flag, err) ||
          !mbar_wait(bfree + bb, bph ^ 1, abort_flag, err))
        break;
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(sW(s));
      const uint4* sp = reinterpret_cast<const uint4*>(sS(s));
      const uint32_t* zp = reinterpret_cast<const uint32_t*>(sZ(s));
      uint8_t* bp = sB(bb);
      if (group_rows == 1) {
        H2 zc[4], sc[4];
        awq_zero_consts<T>(zp[wc], zc);
        const uint4 sv = sp[wc];
        sc[0] = H::from_bits(sv.x);
        sc[1] = H::from_bits(sv.y);
        sc[2] = H::from_bits(sv.z);
        sc[3] = H::from_bits(sv.w);
        uint32_t wv[kSkRowsPer];
#pragma unroll
        for (int j = 0; j < kSkRowsPer; ++j) wv[j] = wp[(r0 + kSkRowStep * j) * kSkWords + wc];
#pragma unroll
        for (int j = 0; j < kSkRowsPer; ++j) {
          const int r = r0 + kSkRowStep * j;
          H2 d[4];
          awq_word_diff<T>(wv[j], zc, d);
          uint4 o;
          o.x = bits_of(__hmul2(d[0], sc[0]));
          o.y = bits_of(__hmul2(d[1], sc[1]));
          o.z = bits_of(__hmul2(d[2], sc[2]));
          o.w = bits_of(__hmul2(d[3], sc[3]));
          const int rr = r & 7;
          *reinterpret_cast<uint4*>(bp + an * kSkBLbo + (r >> 3) * kSkBSbo + rr * 128 +
                                    ((cc ^ rr) << 4)) = o;
        }
      } else {
        int cur_g = -1;
        H2 zc[4], sc[4];
#pragma unroll
        for (int j = 0; j < kSkRowsPer; ++j) {
          const int r = r0 + kSkRowStep * j;
          const int gl = r / G;  // group row of this k within the block
          if (gl != cur_g) {
            cur_g = gl;
            awq_zero_consts<T>(zp[gl * kSkWords + wc], zc);
            const uint4 sv = sp[gl * kSkWords + wc];
            sc[0] = H::from_bits(sv.x);
            sc[1] = H::from_bits(sv.y);
            sc[2] = H::from_bits(sv.z);
            sc[3] = H::from_bits(sv.w);
          }
          H2 d[4];
          awq_word_diff<T>(wp[r * kSkWords + wc], zc, d);
          uint4 o;
          o.x = bits_of(__hmul2(d[0], sc[0]));
          o.y = bits_of(__hmul2(d[1], sc[1]));
          o.z = bits_of(__hmul2(d[2], sc[2]));
          o.w = bits_of(__hmul2(d[3], sc[3]));
          const int rr = r & 7;
          *reinterpret_cast<uint4*>(bp + an * kSkBLbo + (r >> 3) * kSkBSbo + rr * 128 +
                                    ((cc ^ rr) << 4)) = o;
        }
      }
      fence_proxy_async_smem();  // the generic stores, visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(bready + bb);
      if (++s == kSkStages) { s = 0; ph ^= 1; }
      if (++bb == kSkBBufs) { bb = 0; bph ^= 1; }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp q reads TMEM lanes 32 q .. 32 q + 31: row m of x (and y) per lane.
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const size_t slab = (size_t)M * kSkBN;  // floats of one part's sums
    int t = u0 / kbn, kb = u0 % kbn, first_kb = kb, p = 0;
    bool ok = true;
    for (int i = 0; ok && i < n; ++i) {
      const bool last = i == n - 1 || kb == kbn - 1;
      const int cur_t = t;
      if (++kb == kbn) { kb = 0; ++t; }
      if (!last) continue;
      const int buf = p & 1;
      if (!mbar_wait(tfull + buf, (p >> 1) & 1, abort_flag, err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kSkBN);
      const int64_t owner = sk_cta_of((int64_t)cur_t * kbn, units, gridDim.x);
      if (first_kb > 0) {
        // A later K range of a tile owned by an earlier CTA: leave the fp32 sums.
        const int slot = (int)(blockIdx.x - owner - 1);
        float* dst = part + ((size_t)cur_t * maxc + slot) * slab + (size_t)m * kSkBN;
#pragma unroll 1
        for (int c0 = 0; c0 < kSkBN; c0 += 32) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld16(tbase + c0, r);
          tmem_ld16(tbase + c0 + 16, r + 16);
          tmem_ld_wait();
          if (m < M && cur_t * kSkBN + c0 < N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<uint4*>(dst + c0 + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) sk_st_release(flags + ((size_t)cur_t * maxc + slot) * 4 + q, epoch);
      } else {
        // The owner. Later parts exist (nc > 0) only in this CTA's last part, when its stage
        // ring and expanded-weight buffers are idle: wait for their flags, then the four epilogue warps add them column-
        // parallel (thread e takes float4 e, e + 128, ... of the [M, 256] tile, the
        // contributors' values of one float4 loaded together and added in K order) into
        // shared memory, and each lane adds its row of that sum to its own TMEM row.
        const int nc = (int)(sk_cta_of((int64_t)cur_t * kbn + kbn - 1, units, gridDim.x) - owner);
        unsigned long long* fl = flags + (size_t)cur_t * maxc * 4;
        float* red = reinterpret_cast<float*>(stage0);
        if (nc > 0) {
          const uint64_t t0 = globaltimer_ns();
          while (true) {
            bool mine = true;
            for (int c = lane; c < 4 * nc; c += 32) mine &= sk_ld_relaxed(fl + c) == epoch;
            if (__all_sync(0xffffffffu, mine)) break;
            if (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs) {
              if (!*abort_flag) {
                *abort_flag = 1;
                if (err) atomicExch(err, (int)kErrWaitTimeout);
              }
              ok = false;
              break;
            }
          }
          __threadfence();
          fence_proxy_async_smem();  // the ring's last TMA writes are ordered before these
          if (ok) {
            const int e = threadIdx.x - kSkEpiWarp0 * 32;
            const float* src0 = part + (size_t)cur_t * maxc * slab;
            const int nf = M * (kSkBN / 4);
            const int cols = min(kSkBN, N - cur_t * kSkBN);
            for (int f = e; f < nf; f += 128) {
              const int mm = f / (kSkBN / 4), c4 = f % (kSkBN / 4);
              if (c4 * 4 >= cols) continue;
              const float4* src = reinterpret_cast<const float4*>(src0) + f;
              const size_t cs = slab / 4;  // float4s per part
              float4 acc = src[0];
              int c = 1;
              for (; c + 3 < nc; c += 4) {
                const float4 a0 = src[c * cs], a1 = src[(c + 1) * cs], a2 = src[(c + 2) * cs],
                             a3 = src[(c + 3) * cs];
                acc.x = (((acc.x + a0.x) + a1.x) + a2.x) + a3.x;
                acc.y = (((acc.y + a0.y) + a1.y) + a2.y) + a3.y;
                acc.z = (((acc.z + a0.z) + a1.z) + a2.z) + a3.z;
                acc.w = (((acc.w + a0.w) + a1.w) + a2.w) + a3.w;
              }
              for (; c < nc; ++c) {
                const float4 a = src[c * cs];
                acc.x += a.x;
                acc.y += a.y;
                acc.z += a.z;
                acc.w += a.w;
              }
              *reinterpret_cast<float4*>(red + (size_t)mm * kSkRedLd + c4 * 4) = acc;
            }
          }
          mbar_arrive(redbar);  // every epilogue thread, once per launch
          if (!mbar_wait(redbar, 0, abort_flag, err)) ok = false;
        }
#pragma unroll 1
        for (int c0 = 0; ok && c0 < kSkBN; c0 += 32) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld16(tbase + c0, r);
          tmem_ld16(tbase + c0 + 16, r + 16);
          tmem_ld_wait();
          const int col = cur_t * kSkBN + c0;  // first column of this chunk
          if (m >= M || col >= N) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (nc > 0) {
            const float4* rs = reinterpret_cast<const float4*>(red + (size_t)m * kSkRedLd + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 a = rs[j];
              v[4 * j] += a.x;
              v[4 * j + 1] += a.y;
              v[4 * j + 2] += a.z;
              v[4 * j + 3] += a.w;
            }
          }
          if (out.act < 0) {
            uint4 o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              o[j] = make_uint4(pack2<T>(v[8 * j], v[8 * j + 1]), pack2<T>(v[8 * j + 2], v[8 * j + 3]),
                                pack2<T>(v[8 * j + 4], v[8 * j + 5]),
                                pack2<T>(v[8 * j + 6], v[8 * j + 7]));
            for (int d = 0; d < out.ny; ++d) {
              uint4* yd = reinterpret_cast<uint4*>(static_cast<T*>(out.y[d]) +
                                                   (size_t)m * out.ld + out.col0 + col);
#pragma unroll
              for (int j = 0; j < 4; ++j) yd[j] = o[j];
            }
          } else {
            // Columns col .. col + 31 are blocks gate, up, gate, up of 8: outputs col / 2 .. + 15.
            alignas(16) T a[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int gi = (j < 8 ? 0 : 16) + (j & 7);
              const T gt = from_f32<T>(v[gi]), ut = from_f32<T>(v[gi + 8]);
              a[j] = out.act == kSilu ? act_mul<T, kSilu>(gt, ut) : act_mul<T, kGeluTanh>(gt, ut);
            }
            const uint4* ap = reinterpret_cast<const uint4*>(a);
            for (int d = 0; d < out.ny; ++d) {
              uint4* yd = reinterpret_cast<uint4*>(static_cast<T*>(out.y[d]) +
                                                   (size_t)m * out.ld + out.col0 + col / 2);
              yd[0] = ap[0];
              yd[1] = ap[1];
            }
          }
        }
        __syncwarp();
        if (q == 0)
          for (int c = lane; c < 4 * nc; c += 32) fl[c] = 0ull;  // ready for the next launch
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + buf);
      ++p;
      first_kb = kb;
    }
    // Stores into the peers' outputs are performed system-wide before the kernel completes (the
    // caller's rank barrier then publishes them).
    if (out.ny > 1) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

struct SkPlan {
  int tiles, kbn, units, grid, maxc, group_rows;
  size_t part_bytes, ws_bytes;
};

// Grid: one CTA per SM, at least four 64-row blocks each; partial-sum slots per tile = the most
// CTAs after a tile's owner that hold part of it.
bool sk_plan(int64_t M, int64_t K, int64_t N, int64_t G, int sms, SkPlan* p) {
  p->tiles = (int)ceil_div(N, kSkBN);
  p->kbn = (int)ceil_div(K, kSkBK);
  if ((int64_t)p->tiles * p->kbn >= ((int64_t)1 << 30)) return false;
  p->units = p->tiles * p->kbn;
  p->grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, p->units / 4));
  int maxc = 0;
  for (int t = 0; t < p->tiles; ++t) {
    const int64_t own = sk_cta_of((int64_t)t * p->kbn, p->units, p->grid);
    const int64_t last = sk_cta_of((int64_t)t * p->kbn + p->kbn - 1, p->units, p->grid);
    maxc = std::max(maxc, (int)(last - own));
  }
  p->maxc = maxc;
  p->group_rows = G >= kSkBK ? 1 : (int)(kSkBK / G);
  p->part_bytes = (size_t)p->tiles * maxc * (size_t)M * kSkBN * 4;
  p->ws_bytes = p->part_bytes + (size_t)p->tiles * maxc * 4 * 8;
  return true;
}

bool sk_supported(int64_t M, int64_t K, int64_t N, int64_t G, int s_dtype) {
  if (M < 1 || M > 128) return false;
  if (s_dtype != TO_F16 && s_dtype != TO_BF16) return false;
  if (N % 32 != 0 || K % 8 != 0) return false;  // 16-byte TMA row strides
  if (G <= 0 || K % G != 0 || !(G % 64 == 0 || G == 32 || G == K)) return false;
  return N <= INT32_MAX / 2 && K <= INT32_MAX / 2;
}

// A launch's flag value: unique per launch within the process (and unlikely to repeat stale
// workspace contents), the same on every replay of a captured launch -- whose flags the owners
// reset after use.
std::atomic<unsigned long long>& sk_epoch() {
  static std::atomic<unsigned long long> e{
      ((unsigned long long)std::chrono::steady_clock::now().time_since_epoch().count() << 21) ^
      ((unsigned long long)getpid() << 2) ^ 3ull};
  return e;
}

template <typename T>
int launch_sk(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
              const SkOut& out, int64_t M, int64_t K, int64_t N, int64_t G, void* ws,
              size_t ws_bytes, cudaStream_t st) {
  SkPlan plan;
  if (!sk_plan(M, K, N, G, sm_count(), &plan)) return TO_EUNSUPPORTED;
  if (plan.ws_bytes > 0 && (ws == nullptr || ws_bytes < plan.ws_bytes))
    return fail(TO_ENOSPACE, "awq_gemm: workspace of %zu bytes, %zu needed", ws_bytes,
                plan.ws_bytes);
  auto kern = k_awq_gemm_sk<T>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)kSkSmem);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "awq stream-K gemm: shared memory attribute");
  CUtensorMap tx, tw, ts, tz;
  int rc = make_tmap_kmajor(&tx, x, M, K, 2, 128);
  if (!rc) rc = make_tmap_plain(&tw, qw, K, N / 8, 4, kSkWords, kSkBK);
  if (!rc) rc = make_tmap_plain(&ts, s, K / G, N, 2, kSkBN, plan.group_rows);
  if (!rc) rc = make_tmap_plain(&tz, qz, K / G, N / 8, 4, kSkWords, plan.group_rows);
  if (rc) return rc;
  float* part = static_cast<float*>(ws);
  unsigned long long* flags =
      reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + plan.part_bytes);
  const unsigned long long epoch = sk_epoch().fetch_add(1) + 1;
  kern<<<plan.grid, kSkThreads, kSkSmem, st>>>(tx, tw, ts, tz, out, part, flags, (int)M, (int)N,
                                               (int)G, plan.group_rows, plan.kbn, plan.units,
                                               plan.maxc, epoch, device_error_ptr());
  return check_launch("awq stream-K gemm");
}

int sk_dispatch(const void* x, const int32_t* qw, const void* s, int s_dtype, const int32_t* qz,
                const SkOut& out, int64_t M, int64_t K, int64_t N, int64_t G, void* ws,
                size_t ws_bytes, cudaStream_t st) {
  if (!sk_supported(M, K, N, G, s_dtype)) return TO_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(qw) || !aligned16(s) || !aligned16(qz)) return TO_EUNSUPPORTED;
  if (ws != nullptr && !aligned16(ws)) return TO_EUNSUPPORTED;
  for (int d = 0; d < out.ny; ++d)
    if (!aligned16(out.y[d])) return TO_EUNSUPPORTED;
  if (s_dtype == TO_F16)
    return launch_sk<__half>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
  return launch_sk<__nv_bfloat16>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
}

}  // namespace
}  // namespace sm100

// Workspace bytes of the stream-K kernel for these shapes (0 when it does not take them).
size_t awq_sk_workspace(int64_t M, int64_t K, int64_t N, int64_t G, int s_dtype) {
  if (!sm100::sk_supported(M, K, N, G, s_dtype)) return 0;
  sm100::SkPlan plan;
  if (!sm100::sk_plan(M, K, N, G, sm_count(), &plan)) return 0;
  return plan.ws_bytes;
}

// y = x @ dequant(W) ([M, N]), or with act >= 0 act(gate) * up ([M, N / 2]) of a gate_up weight
// interleaved in blocks of 8 columns. TO_EUNSUPPORTED (nothing launched, no error recorded) for
// shapes the kernel does not take.
int awq_sk_launch(const void* x, const int32_t* qw, const void* s, int s_dtype, const int32_t* qz,
                  void* y, int64_t M, int64_t K, int64_t N, int64_t G, void* ws, size_t ws_bytes,
                  cudaStream_t st, int act) {
  if (act >= 0 && N % 16 != 0) return TO_EUNSUPPORTED;
  sm100::SkOut out = {};
  out.y[0] = y;
  out.ny = 1;
  out.ld = (int)(act >= 0 ? N / 2 : N);
  out.col0 = 0;
  out.act = act;
  return sm100::sk_dispatch(x, qw, s, s_dtype, qz, out, M, K, N, G, ws, ws_bytes, st);
}

// The gathering form: this rank's [M, N] slice (or [M, N / 2] activation slice) into every
// rank's output (y_ranks[r], the peers' mapped into this process) at its column offset.
int awq_sk_gather_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                         const int32_t* qz, void* const* y_ranks, int world, int rank, int64_t M,
                         int64_t K, int64_t N, int64_t G, void* ws, size_t ws_bytes,
                         cudaStream_t st, int act) {
  if (world < 1 || world > sm100::kSkMaxOut || N * world > INT32_MAX / 2) return TO_EUNSUPPORTED;
  if (act >= 0 && N % 16 != 0) return TO_EUNSUPPORTED;
  sm100::SkOut out = {};
  for (int r = 0; r < world; ++r) out.y[r] = y_ranks[r];
  out.ny = world;
  const int64_t n_out = act >= 0 ? N / 2 : N;
  out.ld = (int)(n_out * world);
  out.col0 = (int)(n_out * rank);
  out.act = act;
  return sm100::sk_dispatch(x, qw, s, s_dtype, qz, out, M, K, N, G, ws, ws_bytes, st);
}

}  // namespace tob
