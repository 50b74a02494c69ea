// AWQ W4A16 GEMM for decode-sized batches (1 <= M <= 32 tokens) on sm_100a:
// y[M, N] = x[M, K] @ dequant(W)[K, N]  (tileops/quant_awq.py:112-155, awq_gemm at small M).
//
// At these sizes the layer streams its packed int4 weights once and does almost no arithmetic
// per byte, so the design goal is the fewest SM instructions per weight and an even split of
// the weight bytes over all SMs:
//   * Work split ("stream-K"). The weights are cut into units of 256 columns (32 packed words)
//     x 256 K rows (32 KB). Units are numbered tile-major, K-minor and CTA b of a grid of one
//     CTA per SM takes the contiguous range [b U / P, (b + 1) U / P): every SM streams the same
//     number of bytes whatever N / 256 is. A column tile whose K range spans several CTAs is
//     summed deterministically: the CTA holding the tile's first K unit (the "owner") adds the
//     others' fp32 partial sums, left in a caller workspace behind a per-launch flag, in K order.
//     The other CTAs reach that tile at the start of their ranges and the owner at the end of
//     its own, so the owner does not wait in practice; every wait is bounded all the same.
//   * Feed. Each unit's packed words, its scale and zero rows and the matching 256 rows of x
//     arrive with four TMA copies (no multicast) in a ring of 3-6 stages (~130-190 KB in flight
//     per SM). There is no producer warp: the last warp to release a stage (a shared counter per
//     stage) issues the copies of the unit that reuses it, so the block is 8 warps and keeps
//     255 registers per thread. The weight copies of the first stages go out before
//     griddepcontrol.wait, so with launch overlap they stream while the previous kernel ends.
//   * Dequantisation. Warp (wc, wk) owns 64 columns (8 words) and one 128-row half of every
//     unit. Per 16-row MMA step a thread loads its word of rows 2q, 2q+1, 2q+8, 2q+9 (the rows
//     of its mma.sync A fragment, natural K order; conflict-free in the 128-byte-swizzled
//     stage). One PRMT pairs the low (or high) halves of two rows, so a LOP3 with the
//     magic-bias constant yields a K pair of one column directly as an fp16/bf16 pair of
//     (bias + w) -- no transposition after conversion.
//   * Tensor cores and scales. mma.sync.m16n8k16 (fp32 accumulate). For fp16 the MMA takes the
//     converted values (bias + w) as they come out of the LOP3, and one more MMA per step with an
//     all-ones A gives the group's sum of x per token; at the end of each quantisation group
//     sum_k x (w - z) = sum_k x (bias + w) - (bias + z) sum_k x is scaled once, in fp32, into
//     the running sums: two FMAs per output element per group instead of a subtraction and a
//     multiply per weight pair. This is the reference's product without its per-weight rounding
//     of T((w - z) * s) to fp16 (2^-11 relative), well inside the GEMM tolerance. For bf16,
//     whose per-weight rounding (2^-8) is as large as that tolerance, each pair is made exact
//     (w - z) and multiplied by its scale in bf16 first: the reference's dequantised weight, bit
//     for bit, accumulated straight into the running sums.
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

// A unit is 256 columns (32 packed words) x 128 WK K rows; its 4 WK warps are 4 column
// warp-tiles of 64 columns x WK row slices of 128 (WK = 2 or 4).
constexpr int kDecWords = 32;  // packed words per unit (256 columns)
template <int WK> struct DecGeom {
  static constexpr int kWarps = 4 * WK;
  static constexpr int kThreads = 32 * kWarps;
  static constexpr int kRows = 128 * WK;                // K rows per unit
  static constexpr int kWBytes = kRows * kDecWords * 4;  // packed weights per unit
};
constexpr size_t kDecSmemMax = 227 * 1024;
constexpr int kDecMaxStages = 6;

// Unit range of CTA b, and the CTA whose range holds unit u (the inverse).
__host__ __device__ __forceinline__ int64_t dec_start(int64_t b, int64_t units, int64_t ctas) {
  return b * units / ctas;
}
__host__ __device__ __forceinline__ int64_t dec_cta_of(int64_t u, int64_t units, int64_t ctas) {
  return ((u + 1) * ctas - 1) / units;
}

// Where the output goes: this GPU's y, or (an N-sharded layer whose all-gather is done here)
// every rank's [M, ld] output at columns [col0, col0 + N), the peers' mapped into this process.
// act >= 0 (kSilu, kGeluTanh): the weights are a gate_up linear whose gate and up columns
// alternate in blocks of 8 (one packed word each), and the output is act(gate) * up, N / 2
// columns wide (col0 and ld count those columns).
constexpr int kDecMaxOut = 8;
struct DecOut {
  void* y[kDecMaxOut];
  int ny, ld, col0, act;
  int64_t ldx;  // row stride of x in elements (0: K); read by the host side only (TMA map)
};

struct DecPlan {
  int tiles, ku, units, grid, maxc, stages, srows;
  int stage_bytes, x_off, s_off, z_off, tx_bytes, red_bytes;
  size_t smem, ws_bytes, part_bytes;
};

// The launch plan: grid (at most one CTA per SM, at least two units per CTA), partial-sum slots
// per tile (the most CTAs after a tile's owner that hold part of it), shared-memory stages.
template <int NT, int GR, int WK>
bool dec_plan(int64_t M, int64_t K, int64_t N, int sms, DecPlan* p) {
  using Geo = DecGeom<WK>;
  p->tiles = (int)ceil_div(N / 8, kDecWords);
  p->ku = (int)ceil_div(K, Geo::kRows);
  if ((int64_t)p->tiles * p->ku >= ((int64_t)1 << 30)) return false;
  p->units = p->tiles * p->ku;
  p->grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, p->units / 2));
  int maxc = 0;
  for (int t = 0; t < p->tiles; ++t) {
    const int64_t own = dec_cta_of((int64_t)t * p->ku, p->units, p->grid);
    const int64_t last = dec_cta_of((int64_t)t * p->ku + p->ku - 1, p->units, p->grid);
    maxc = std::max(maxc, (int)(last - own));
  }
  p->maxc = maxc;
  p->srows = Geo::kRows / GR;
  const int x_bytes = (Geo::kRows / 64) * 1024 * NT;  // 64-row blocks x 8 NT tokens x 128 B
  const int s_bytes = p->srows * 256 * 2;
  const int z_bytes = p->srows * kDecWords * 4;
  p->x_off = Geo::kWBytes;
  p->s_off = p->x_off + x_bytes;
  p->z_off = p->s_off + s_bytes;
  p->tx_bytes = Geo::kWBytes + x_bytes + s_bytes + z_bytes;
  p->stage_bytes = (p->tx_bytes + 1023) & ~1023;
  // one fragment-order tile per column warp-tile and row slice after the first
  p->red_bytes = 4 * (WK - 1) * 16 * NT * 32 * 4;
  const size_t fixed = 1024 + (size_t)p->red_bytes + 512;
  p->stages = (int)std::min<size_t>(kDecMaxStages, (kDecSmemMax - fixed) / p->stage_bytes);
  if (p->stages < 2) return false;
  p->smem = fixed + (size_t)p->stages * p->stage_bytes;
  p->part_bytes = (size_t)p->tiles * p->maxc * (size_t)M * 256 * 4;
  p->ws_bytes = p->part_bytes + (size_t)p->tiles * p->maxc * 4 * 8;
  return true;
}

// --- device helpers -------------------------------------------------------------------
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Magic-bias conversion of the four nibbles of each 16-bit half of v (v already paired, so both
// halves hold the same columns of two K rows): o[i] = the pair of nibble i. fp16: bits 0-3 read
// as 1024 + n under 0x6400 and bits 4-7 as 64 + n under 0x5400, so one shift by 8 serves both
// upper nibbles; bf16 (7 mantissa bits) reads only bits 0-3, as 128 + n under 0x4300.
template <typename T>
__device__ __forceinline__ void nibble_pairs(uint32_t v, uint32_t* o) {
  if constexpr (std::is_same<T, __half>::value) {
    const uint32_t v8 = v >> 8;
    o[0] = lop3_and_or(v, 0x000F000Fu, 0x64006400u);
    o[1] = lop3_and_or(v, 0x00F000F0u, 0x54005400u);
    o[2] = lop3_and_or(v8, 0x000F000Fu, 0x64006400u);
    o[3] = lop3_and_or(v8, 0x00F000F0u, 0x54005400u);
  } else {
    o[0] = lop3_and_or(v, 0x000F000Fu, 0x43004300u);
    o[1] = lop3_and_or(v >> 4, 0x000F000Fu, 0x43004300u);
    o[2] = lop3_and_or(v >> 8, 0x000F000Fu, 0x43004300u);
    o[3] = lop3_and_or(v >> 12, 0x000F000Fu, 0x43004300u);
  }
}

// Per column c of a zero word: the (bias + z_c) pair that nibble_pairs' output for column c
// must lose. Nibble j holds column [0,2,4,6,1,3,5,7][j]: columns 0, 2, 4, 6 sit in the low
// half-word, 1, 3, 5, 7 in the high one.
template <typename T>
__device__ __forceinline__ void zero_pairs(uint32_t zw, uint32_t* zc) {
  uint32_t lo[4], hi[4];
  nibble_pairs<T>(prmt(zw, zw, 0x5410u), lo);
  nibble_pairs<T>(prmt(zw, zw, 0x7632u), hi);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    zc[2 * i] = lo[i];
    zc[2 * i + 1] = hi[i];
  }
}

template <typename T>
__device__ __forceinline__ uint32_t sub_pair(uint32_t a, uint32_t b) {
  using H = Half2Of<T>;
  return bits_of(__hsub2(H::from_bits(a), H::from_bits(b)));
}

// Exact (w - z) K pairs of rows (ra, rb) = (r, r + 1) for the word's 8 columns: out[c] holds
// column c, row ra in the low half.
template <typename T>
__device__ __forceinline__ void word_kpairs(uint32_t ra, uint32_t rb, const uint32_t* zc,
                                            uint32_t* out) {
  uint32_t lo[4], hi[4];
  nibble_pairs<T>(prmt(ra, rb, 0x5410u), lo);
  nibble_pairs<T>(prmt(ra, rb, 0x7632u), hi);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = sub_pair<T>(lo[i], zc[2 * i]);
    out[2 * i + 1] = sub_pair<T>(hi[i], zc[2 * i + 1]);
  }
}

// The K pairs of rows (ra, ra + 1) for the word's 8 columns, still carrying the magic bias:
// out[c] = {bias_c + w[ra][c], bias_c + w[ra + 1][c]} (exact in fp16).
template <typename T>
__device__ __forceinline__ void word_rawpairs(uint32_t ra, uint32_t rb, uint32_t* out) {
  uint32_t lo[4], hi[4];
  nibble_pairs<T>(prmt(ra, rb, 0x5410u), lo);
  nibble_pairs<T>(prmt(ra, rb, 0x7632u), hi);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = lo[i];
    out[2 * i + 1] = hi[i];
  }
}

template <typename T>
__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Shared-memory counter increment with acquire-release ordering at CTA scope: a warp's reads
// of a stage (fenced against the async proxy) happen before the refill the last warp issues.
__device__ __forceinline__ unsigned atom_add_acq_rel_smem(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "r"(smem_u32(p)), "r"(v)
               : "memory");
  return old;
}

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid: one CTA per SM, all resident at once (P <= #SMs); block: 8 warps.
// NT: 8-token tiles of M (1, 2 or 4); GR: rows of one scale (32, 64 or 128; divides G).
// EXACT: multiply each (w - z) pair by its scale in T before the MMA -- the reference's
// dequantised weight T((w - z) * s), bit for bit -- instead of scaling each group's fp32 sums.
template <typename T, int NT, int GR, bool EXACT, int WK>
__global__ void __launch_bounds__(DecGeom<WK>::kThreads, 1) k_awq_decode(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
    const DecOut out, float* __restrict__ part, unsigned long long* __restrict__ flags,
    int M, int N, int G, int g_log2, int ku, int units, int maxc, int stages, int stage_bytes,
    int x_off, int s_off, int z_off, int tx_bytes, unsigned long long epoch, int* err) {
  using H2 = typename Half2Of<T>::type;
  constexpr int kSteps = GR / 16;     // MMA steps per scaled group
  constexpr int kGroups = 128 / GR;   // groups per warp row slice of a unit
  constexpr int kDecWarps = DecGeom<WK>::kWarps;
  constexpr int kDecRows = DecGeom<WK>::kRows;
  constexpr int kXTile = 1024 * NT;   // one 64-row block of x: 8 NT tokens x 128 B
  constexpr int kAcc = 16 * NT;       // accumulators per thread

  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  float* reds = reinterpret_cast<float*>(base + (size_t)stages * stage_bytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(reds) +
                                               4 * (WK - 1) * kAcc * 32 * 4);
  uint64_t* redfull = full + stages;
  uint64_t* redfree = redfull + 4;
  unsigned* released = reinterpret_cast<unsigned*>(redfree + 4);  // per stage, monotonic
  int* last_issue = reinterpret_cast<int*>(released + stages);    // per stage, for unwinding
  volatile int* abort_flag = reinterpret_cast<volatile int*>(last_issue + stages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = dec_start(blockIdx.x, units, gridDim.x);
  const int64_t u1 = dec_start(blockIdx.x + 1, units, gridDim.x);
  const int n = (int)(u1 - u0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      released[s] = 0;
      last_issue[s] = -1;
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(redfull + i, WK - 1);
      mbar_init(redfree + i, 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const uint64_t pol_w = policy_evict_first();  // streamed once
  const uint64_t pol_x = policy_evict_last();   // re-read by every column tile
  auto issue_w = [&](int i, int slot) {
    const int u = (int)(u0 + i);  // units < 2^31 (checked on the host)
    const int t = u / ku, r = u - t * ku;
    unsigned char* st = base + (size_t)slot * stage_bytes;
    const int g0 = (r * kDecRows) / G;
    last_issue[slot] = i;
    mbar_arrive_expect_tx(full + slot, (uint32_t)tx_bytes);
#pragma unroll
    for (int b = 0; b < kDecRows / 256; ++b)  // boxes of 256 rows
      tma_load_2d(st + b * 256 * kDecWords * 4, &tm_w, t * 2 * kDecWords, r * kDecRows + b * 256,
                  full + slot, pol_w);
    tma_load_2d(st + s_off, &tm_s, t * 256, g0, full + slot, pol_w);
    tma_load_2d(st + z_off, &tm_z, t * kDecWords, g0, full + slot, pol_w);
  };
  auto issue_x = [&](int i, int slot) {
    const int r = (int)(u0 + i) % ku;
    tma_load_3d(base + (size_t)slot * stage_bytes + x_off, &tm_x, 0, 0, r * (kDecRows / 64),
                full + slot, pol_x);
  };
  const int pre = min(n, stages);
  if (threadIdx.x == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_s);
    prefetch_tmap(&tm_z);
    prefetch_tmap(&tm_x);
    for (int i = 0; i < pre; ++i) issue_w(i, i);
  }
  // x, y and the workspace may belong to the previous grid in the stream.
  grid_dependency_wait();
  grid_dependents_launch();
  if (threadIdx.x == 0)
    for (int i = 0; i < pre; ++i) issue_x(i, i);

  const int wc = warp & 3, wk = warp >> 2;  // column warp-tile, row slice
  const int g = lane >> 2, q = lane & 3;
  const int word = wc * 8 + g;  // this thread's packed word within the unit
  // Per-thread shared-memory offsets, so that the loads of a step take immediate offsets.
  // Weights (128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7)): rows 2q (+8) and
  // 2q+1 (+9) of every 16-row step have r & 7 = 2q and 2q+1.
  const int w_off0 = (wk * 128 + 2 * q) * kDecWords + ((((word >> 2) ^ (2 * q)) << 2) | (word & 3));
  const int w_off1 =
      (wk * 128 + 2 * q + 1) * kDecWords + ((((word >> 2) ^ (2 * q + 1)) << 2) | (word & 3));
  // x: token g + 8t, K pair 2q of a 16-row step, in the block of 64 rows this half starts at;
  // the swizzled chunk (c ^ g) is formed per step from its compile-time part c.
  const int x_off0 = (wk * 2) * kXTile + g * 128 + 4 * q;
  const uint32_t g16 = (uint32_t)g << 4;

  float acc[4][NT][4];
#pragma unroll
  for (int p = 0; p < 4; ++p)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[p][t][e] = 0.f;

  int flushes = 0;
  // tile and K unit of the current unit, advanced without divisions
  int cur_t = (int)(u0 / ku), cur_r = (int)(u0 % ku);
  int first_r = cur_r;  // K unit where the current tile part began
  bool ok = true;
#pragma unroll 1
  for (int i = 0; ok && i < n; ++i) {
    const int slot = i % stages;
    if (!mbar_wait(full + slot, (i / stages) & 1, abort_flag, err)) {
      ok = false;
      break;
    }
    const int r = cur_r;
    const unsigned char* st = base + (size_t)slot * stage_bytes;
    const uint32_t* ws = reinterpret_cast<const uint32_t*>(st);
    const unsigned char* xs = st + x_off;
    const H2* ss = reinterpret_cast<const H2*>(st + s_off);
    const uint32_t* zs = reinterpret_cast<const uint32_t*>(st + z_off);
    const int row0 = r * kDecRows;
    const int g0 = row0 / G;

#pragma unroll
    for (int gi = 0; gi < kGroups; ++gi) {
      const int lrow = wk * 128 + gi * GR;  // first stage row of the group slice
      // scale row within the stage: by shifts when G is a power of two
      const int srow = g_log2 >= 0 ? ((row0 + lrow) >> g_log2) - (row0 >> g_log2)
                                   : (row0 + lrow) / G - g0;
      uint32_t zc[8];  // per column c: {bias_c + z_c, bias_c + z_c}
      zero_pairs<T>(zs[srow * kDecWords + word], zc);
      // The group's scales for the word's 8 columns (pairs of columns 2j, 2j+1).
      const uint4 sv = *reinterpret_cast<const uint4*>(ss + srow * 128 + word * 4);
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
      uint32_t sp[8];  // EXACT: {s_c, s_c} per column c
      if constexpr (EXACT) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sp[2 * j] = prmt(sw[j], sw[j], 0x1010u);
          sp[2 * j + 1] = prmt(sw[j], sw[j], 0x3232u);
        }
      }
      float ag[4][NT][4];  // !EXACT: sum_k x (bias + w) per output of the group
      float xg[NT][4];     // !EXACT: sum_k x per token (all-ones MMA rows)

      // This thread's weight words and x pairs of step s (loaded one step ahead).
      auto load_step = [&](int s_, uint32_t* w, uint32_t (*bx)[2]) {
        const int r16 = gi * GR + 16 * s_;  // step row within the warp's half (compile time)
        const uint32_t* wr0 = ws + w_off0 + r16 * kDecWords;
        const uint32_t* wr1 = ws + w_off1 + r16 * kDecWords;
        w[0] = wr0[0];
        w[1] = wr1[0];
        w[2] = wr0[8 * kDecWords];
        w[3] = wr1[8 * kDecWords];
        // x[token g + 8t][k 2q, 2q+1] and [k 2q+8, 2q+9]: x rows are 128-byte-swizzled
        // 64-element blocks, so the +8 pair is the next 16-byte chunk.
        const int c0 = (r16 & 63) >> 3;
        const unsigned char* xb = xs + x_off0 + (r16 >> 6) * kXTile;
        const uint32_t o0 = ((uint32_t)c0 << 4) ^ g16, o1 = ((uint32_t)(c0 + 1) << 4) ^ g16;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          bx[t][0] = *reinterpret_cast<const uint32_t*>(xb + t * 1024 + o0);
          bx[t][1] = *reinterpret_cast<const uint32_t*>(xb + t * 1024 + o1);
        }
      };
      uint32_t wcur[4], bcur[NT][2];
      load_step(0, wcur, bcur);
#pragma unroll
      for (int s = 0; s < kSteps; ++s) {
        uint32_t wnext[4], bnext[NT][2];
        if (s + 1 < kSteps) load_step(s + 1, wnext, bnext);
        uint32_t alo[8], ahi[8];
        if constexpr (EXACT) {
          using H = Half2Of<T>;
          word_kpairs<T>(wcur[0], wcur[1], zc, alo);
          word_kpairs<T>(wcur[2], wcur[3], zc, ahi);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            alo[c] = bits_of(__hmul2(H::from_bits(alo[c]), H::from_bits(sp[c])));
            ahi[c] = bits_of(__hmul2(H::from_bits(ahi[c]), H::from_bits(sp[c])));
          }
        } else {
          word_rawpairs<T>(wcur[0], wcur[1], alo);
          word_rawpairs<T>(wcur[2], wcur[3], ahi);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if constexpr (!EXACT) {
            if (s == 0) {
#pragma unroll
              for (int e = 0; e < 4; ++e) xg[t][e] = 0.f;
            }
            constexpr uint32_t kOnes = 0x3C003C00u;  // fp16 1.0 pairs
            mma16816<T>(xg[t], kOnes, kOnes, kOnes, kOnes, bcur[t][0], bcur[t][1]);
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            if constexpr (EXACT) {
              mma16816<T>(acc[p][t], alo[2 * p], alo[2 * p + 1], ahi[2 * p], ahi[2 * p + 1],
                          bcur[t][0], bcur[t][1]);
            } else {
              if (s == 0) {
#pragma unroll
                for (int e = 0; e < 4; ++e) ag[p][t][e] = 0.f;
              }
              mma16816<T>(ag[p][t], alo[2 * p], alo[2 * p + 1], ahi[2 * p], ahi[2 * p + 1],
                          bcur[t][0], bcur[t][1]);
            }
          }
        }
        if (s + 1 < kSteps) {
#pragma unroll
          for (int j = 0; j < 4; ++j) wcur[j] = wnext[j];
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            bcur[t][0] = bnext[t][0];
            bcur[t][1] = bnext[t][1];
          }
        }
      }
      if constexpr (!EXACT) {
        // sum_k x (w - z) = sum_k x (bias + w) - (bias + z) sum_k x, scaled once in fp32.
        float sc[8], zf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = Half2Of<T>::to_float2(Half2Of<T>::from_bits(sw[j]));
          sc[2 * j] = f.x;
          sc[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) zf[c] = Half2Of<T>::to_float2(Half2Of<T>::from_bits(zc[c])).x;
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            acc[p][t][0] = fmaf(fmaf(-zf[2 * p], xg[t][0], ag[p][t][0]), sc[2 * p], acc[p][t][0]);
            acc[p][t][1] = fmaf(fmaf(-zf[2 * p], xg[t][1], ag[p][t][1]), sc[2 * p], acc[p][t][1]);
            acc[p][t][2] =
                fmaf(fmaf(-zf[2 * p + 1], xg[t][0], ag[p][t][2]), sc[2 * p + 1], acc[p][t][2]);
            acc[p][t][3] =
                fmaf(fmaf(-zf[2 * p + 1], xg[t][1], ag[p][t][3]), sc[2 * p + 1], acc[p][t][3]);
          }
      }
    }
    // Release the stage: this thread's generic reads come before the TMA refill, which the
    // last warp to release it issues.
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && i + stages < n &&
        atom_add_acq_rel_smem(released + slot, 1u) % kDecWarps == kDecWarps - 1) {
      issue_w(i + stages, slot);
      issue_x(i + stages, slot);
    }

    const int t = cur_t;
    if (++cur_r == ku) {
      cur_r = 0;
      ++cur_t;
    }
    if (i + 1 < n && cur_r != 0) continue;  // the tile part goes on

    // ---------------------------------------------------------- end of a tile part
    // The row slices of a column warp-tile meet in shared memory (fragment order): slices
    // 1..WK-1 leave their sums, slice 0 adds them in order.
    if (wk > 0) {
      float* red = reds + ((size_t)wc * (WK - 1) + (wk - 1)) * kAcc * 32;
      if (flushes > 0 && !mbar_wait(redfree + wc, (flushes - 1) & 1, abort_flag, err)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
          for (int e = 0; e < 4; ++e) red[((p * NT + tt) * 4 + e) * 32 + lane] = acc[p][tt][e];
      __syncwarp();
      if (lane == 0) mbar_arrive(redfull + wc);
    } else {
      if (!mbar_wait(redfull + wc, flushes & 1, abort_flag, err)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int k = 0; k < WK - 1; ++k) {
        const float* red = reds + ((size_t)wc * (WK - 1) + k) * kAcc * 32;
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
          for (int tt = 0; tt < NT; ++tt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[p][tt][e] += red[((p * NT + tt) * 4 + e) * 32 + lane];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(redfree + wc);

      const int col0 = t * 256 + wc * 64 + g * 8;  // this thread's word's first column
      const int64_t owner = dec_cta_of((int64_t)t * ku, units, gridDim.x);
      if (first_r > 0) {
        // A later K range of a tile owned by an earlier CTA: leave the fp32 partial sums.
        const int slot_c = (int)(blockIdx.x - owner - 1);
        float* dst = part + ((size_t)t * maxc + slot_c) * (size_t)M * 256;
#pragma unroll
        for (int tt = 0; tt < NT; ++tt)
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int c = col0 + 2 * p;
            const int m = 8 * tt + 2 * q;
            if (c < N) {
              if (m < M)
                *reinterpret_cast<float2*>(dst + (size_t)m * 256 + (c - t * 256)) =
                    make_float2(acc[p][tt][0], acc[p][tt][2]);
              if (m + 1 < M)
                *reinterpret_cast<float2*>(dst + (size_t)(m + 1) * 256 + (c - t * 256)) =
                    make_float2(acc[p][tt][1], acc[p][tt][3]);
            }
          }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_u64(flags + ((size_t)t * maxc + slot_c) * 4 + wc, epoch);
      } else {
        // The owner: add the later K ranges' partial sums in K order, then store y. All
        // flags are read together (relaxed) until every one shows this launch, then one fence
        // orders the partial-sum loads after them; the loads go out several contributors at a
        // time.
        const int nc = (int)(dec_cta_of((int64_t)t * ku + ku - 1, units, gridDim.x) - owner);
        unsigned long long* fl = flags + (size_t)t * maxc * 4 + wc;
        if (nc > 0) {
          const uint64_t t0 = globaltimer_ns();
          while (true) {
            bool all = true;
            for (int c = 0; c < nc; ++c) all &= ld_relaxed_u64(fl + 4 * c) == epoch;
            if (all) break;
            if (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs) {
              if (!*abort_flag) {
                *abort_flag = 1;
                if (err) atomicExch(err, (int)kErrWaitTimeout);
              }
              ok = false;
              break;
            }
          }
          if (!ok) break;
          __threadfence();
        }
        const float* src0 = part + (size_t)t * maxc * (size_t)M * 256;
        const size_t cstride = (size_t)M * 256;
        // contributors whose loads are in flight together (bounded by the register budget)
        constexpr int kBatch = NT * (WK == 4 ? 2 : 1) >= 4 ? 2 : 4;
        for (int c0 = 0; c0 < nc; c0 += kBatch) {
          float2 v[kBatch][NT][4][2];
#pragma unroll
          for (int j = 0; j < kBatch; ++j)
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                const int cc = col0 + 2 * p - t * 256;
                const int m = 8 * tt + 2 * q;
                const bool col_ok = c0 + j < nc && col0 + 2 * p < N;
                const float* src = src0 + (size_t)(c0 + j) * cstride;
                v[j][tt][p][0] = (col_ok && m < M)
                                     ? *reinterpret_cast<const float2*>(src + (size_t)m * 256 + cc)
                                     : make_float2(0.f, 0.f);
                v[j][tt][p][1] =
                    (col_ok && m + 1 < M)
                        ? *reinterpret_cast<const float2*>(src + (size_t)(m + 1) * 256 + cc)
                        : make_float2(0.f, 0.f);
              }
#pragma unroll
          for (int j = 0; j < kBatch; ++j)
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                acc[p][tt][0] += v[j][tt][p][0].x;
                acc[p][tt][2] += v[j][tt][p][0].y;
                acc[p][tt][1] += v[j][tt][p][1].x;
                acc[p][tt][3] += v[j][tt][p][1].y;
              }
        }
        __syncwarp();
        if (lane < nc) fl[4 * lane] = 0ull;  // consumed: ready for the next launch's epoch
        for (int c = 32 + lane; c < nc; c += 32) fl[4 * c] = 0ull;
        if (!ok) break;
        if (out.act < 0) {
          // The thread's 8 columns of rows m and m + 1: one 16-byte store per row and
          // destination (the fewest transactions over NVLink for the peers' copies).
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) {
            const int m = 8 * tt + 2 * q;
            uint32_t r0[4], r1[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              r0[p] = bits_of(Half2Of<T>::from_floats(acc[p][tt][0], acc[p][tt][2]));
              r1[p] = bits_of(Half2Of<T>::from_floats(acc[p][tt][1], acc[p][tt][3]));
            }
            if (col0 < N) {
              for (int d = 0; d < out.ny; ++d) {
                T* yd = static_cast<T*>(out.y[d]) + out.col0 + col0;
                if (m < M)
                  *reinterpret_cast<uint4*>(yd + (size_t)m * out.ld) =
                      make_uint4(r0[0], r0[1], r0[2], r0[3]);
                if (m + 1 < M)
                  *reinterpret_cast<uint4*>(yd + (size_t)(m + 1) * out.ld) =
                      make_uint4(r1[0], r1[1], r1[2], r1[3]);
              }
            }
          }
        } else {
          // Gate and up blocks alternate word by word, so this thread's word (g) and the word
          // of lane ^ 4 (g ^ 1) hold the gate and up sums of the same 8 columns. The even lane
          // takes columns 0-3 of the pair, the odd lane columns 4-7; each receives the other
          // half's sums by one exchange. Each sum is rounded to T (the GEMM's output) before
          // the activation, so the result equals the unfused GEMM + silu_and_mul.
          const bool is_gate = (g & 1) == 0;
          const int pair0 = col0 - (is_gate ? 0 : 8);    // the gate word's first column
          const int a_col = (pair0 >> 1) + (is_gate ? 0 : 4);  // first output column here
#pragma unroll
          for (int tt = 0; tt < NT; ++tt) {
            uint32_t w0[2], w1[2];  // rows m, m + 1: outputs a_col .. a_col + 3
#pragma unroll
            for (int pp = 0; pp < 2; ++pp) {
              float gv[4], uv[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float mine = is_gate ? acc[pp + 2][tt][e] : acc[pp][tt][e];
                const float other = __shfl_xor_sync(0xffffffffu, mine, 4);
                gv[e] = is_gate ? acc[pp][tt][e] : other;
                uv[e] = is_gate ? other : acc[pp + 2][tt][e];
              }
              T r[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const T gt = from_f32<T>(gv[e]), ut = from_f32<T>(uv[e]);
                r[e] = out.act == kSilu ? act_mul<T, kSilu>(gt, ut) : act_mul<T, kGeluTanh>(gt, ut);
              }
              H2 v0, v1;
              v0.x = r[0];
              v0.y = r[2];
              v1.x = r[1];
              v1.y = r[3];
              w0[pp] = bits_of(v0);
              w1[pp] = bits_of(v1);
            }
            const int m = 8 * tt + 2 * q;
            if (pair0 < N) {
              for (int d = 0; d < out.ny; ++d) {
                T* yd = static_cast<T*>(out.y[d]) + out.col0 + a_col;
                if (m < M) *reinterpret_cast<uint2*>(yd + (size_t)m * out.ld) = make_uint2(w0[0], w0[1]);
                if (m + 1 < M)
                  *reinterpret_cast<uint2*>(yd + (size_t)(m + 1) * out.ld) = make_uint2(w1[0], w1[1]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[p][tt][e] = 0.f;
    ++flushes;
    first_r = cur_r;
  }
  // Stores into the peers' outputs are performed system-wide before the kernel completes (the
  // caller's rank barrier then publishes them).
  if (out.ny > 1) __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // Unwinding: copies issued into a stage nobody consumed must land before the CTA's shared
    // memory is released.
    const uint64_t t0 = globaltimer_ns();
    for (int sl = 0; sl < stages; ++sl)
      if (last_issue[sl] >= 0)
        while (!mbar_try_wait(full + sl, (last_issue[sl] / stages) & 1) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
  }
}

// A launch's flag value: unique per launch within the process (and unlikely to repeat stale
// workspace contents), the same on every replay of a captured launch -- whose flags the owners
// reset after use.
std::atomic<unsigned long long>& dec_epoch() {
  static std::atomic<unsigned long long> e{
      ((unsigned long long)std::chrono::steady_clock::now().time_since_epoch().count() << 20) ^
      ((unsigned long long)getpid() << 1) ^ 1ull};
  return e;
}

template <typename T, int NT, int GR, bool EXACT, int WK>
int launch_decode(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                  const DecOut& out,
                  int64_t M, int64_t K, int64_t N, int64_t G, void* ws, size_t ws_bytes,
                  cudaStream_t st) {
  DecPlan plan;
  if (!dec_plan<NT, GR, WK>(M, K, N, sm_count(), &plan)) return TO_EUNSUPPORTED;
  if (plan.ws_bytes > 0 && (ws == nullptr || ws_bytes < plan.ws_bytes))
    return fail(TO_ENOSPACE, "awq_gemm: workspace of %zu bytes, %zu needed", ws_bytes,
                plan.ws_bytes);
  auto kern = k_awq_decode<T, NT, GR, EXACT, WK>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)plan.smem);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "awq decode gemm: shared memory attribute");
  CUtensorMap tx, tw, ts, tz;
  int rc = make_tmap_x_blocks(&tx, x, M, K, 8 * NT, DecGeom<WK>::kRows / 64, out.ldx);
  // the packed words as 16-bit pairs, so that a 128-byte swizzled box holds 32 words
  if (!rc) rc = make_tmap_kmajor(&tw, qw, K, N / 4, 2, 256);
  if (!rc) rc = make_tmap_plain(&ts, s, K / G, N, 2, 256, plan.srows);
  if (!rc) rc = make_tmap_plain(&tz, qz, K / G, N / 8, 4, kDecWords, plan.srows);
  if (rc) return rc;
  float* part = static_cast<float*>(ws);
  unsigned long long* flags = reinterpret_cast<unsigned long long*>(
      static_cast<char*>(ws) + plan.part_bytes);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid, 1, 1);
  cfg.blockDim = dim3(DecGeom<WK>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  int na = 0;
  if (launch_overlap()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const unsigned long long epoch = dec_epoch().fetch_add(1) + 1;
  const int g_log2 = (G & (G - 1)) == 0 ? __builtin_ctzll((unsigned long long)G) : -1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, tz, out, part, flags, (int)M,
                                     (int)N, (int)G, g_log2, plan.ku, plan.units, plan.maxc, plan.stages,
                                     plan.stage_bytes, plan.x_off, plan.s_off, plan.z_off,
                                     plan.tx_bytes, epoch, device_error_ptr());
  if (e != cudaSuccess) return cuda_fail(e, "awq decode gemm launch");
  return check_launch("awq decode gemm");
}

// Rows scaled at once: the largest of 128, 64, 32 that divides the group size (0 if none).
inline int dec_group_rows(int64_t G) {
  return G % 128 == 0 ? 128 : G % 64 == 0 ? 64 : G % 32 == 0 ? 32 : 0;
}

bool dec_supported(int64_t M, int64_t K, int64_t N, int64_t G, int s_dtype) {
  if (M < 1 || M > 32) return false;
  if (s_dtype != TO_F16 && s_dtype != TO_BF16) return false;
  if (N % 32 != 0 || K % 64 != 0 || G <= 0 || K % G != 0 || dec_group_rows(G) == 0) return false;
  return N <= INT32_MAX / 2 && K <= INT32_MAX / 2;
}

// Row slices per unit: 2 (8 warps). Four (16 warps of at most 128 registers, NT <= 2) measured
// no faster on the decode shapes: the extra warps queue on the mma.sync pipe (measurement
// override TOB_DECODE_WK=4).
template <int NT>
int dec_wk() {
  static const int v = [] {
    const char* e = tuning_env("TOB_DECODE_WK");
    return (e != nullptr && e[0] == '4' && NT <= 2) ? 4 : 2;
  }();
  return v;
}

template <int NT, int WK>
size_t dec_ws_wk(int64_t M, int64_t K, int64_t N, int64_t G) {
  DecPlan plan;
  bool ok = false;
  switch (dec_group_rows(G)) {
    case 128: ok = dec_plan<NT, 128, WK>(M, K, N, sm_count(), &plan); break;
    case 64: ok = dec_plan<NT, 64, WK>(M, K, N, sm_count(), &plan); break;
    case 32: ok = dec_plan<NT, 32, WK>(M, K, N, sm_count(), &plan); break;
  }
  return ok ? plan.ws_bytes : 0;
}

template <int NT>
size_t dec_ws(int64_t M, int64_t K, int64_t N, int64_t G) {
  if constexpr (NT <= 2) {
    if (dec_wk<NT>() == 4) return dec_ws_wk<NT, 4>(M, K, N, G);
  }
  return dec_ws_wk<NT, 2>(M, K, N, G);
}

// fp16 scales each group's fp32 sums (its per-weight rounding error is 2^-11 relative, far
// inside the GEMM tolerance); bf16 rounds every dequantised weight as the reference does, since
// its 2^-8 weight rounding moves outputs by as much as the tolerance (measurement override
// TOB_DECODE_EXACT=1 makes fp16 exact too).
inline bool dec_exact(bool f16) {
  static const bool force = [] {
    const char* v = tuning_env("TOB_DECODE_EXACT");
    return v != nullptr && v[0] == '1';
  }();
  return !f16 || force;
}

template <typename T, int NT, bool EXACT, int WK>
int dispatch_decode_gr(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                       const DecOut& out, int64_t M, int64_t K, int64_t N, int64_t G, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
  switch (dec_group_rows(G)) {
    case 128:
      return launch_decode<T, NT, 128, EXACT, WK>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
    case 64:
      return launch_decode<T, NT, 64, EXACT, WK>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
    case 32:
      return launch_decode<T, NT, 32, EXACT, WK>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
  }
  return TO_EUNSUPPORTED;
}

template <typename T, int NT, bool EXACT>
int dispatch_decode_wk(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                       const DecOut& out, int64_t M, int64_t K, int64_t N, int64_t G, void* ws,
                       size_t ws_bytes, cudaStream_t st) {
  if constexpr (NT <= 2) {
    if (dec_wk<NT>() == 4)
      return dispatch_decode_gr<T, NT, EXACT, 4>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
  }
  return dispatch_decode_gr<T, NT, EXACT, 2>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
}

template <typename T, int NT>
int dispatch_decode(const void* x, const int32_t* qw, const void* s, const int32_t* qz,
                    const DecOut& out,
                    int64_t M, int64_t K, int64_t N, int64_t G, void* ws, size_t ws_bytes,
                    cudaStream_t st) {
  if constexpr (std::is_same<T, __half>::value) {
    if (!dec_exact(true))
      return dispatch_decode_wk<T, NT, false>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
  }
  return dispatch_decode_wk<T, NT, true>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st);
}

}  // namespace
}  // namespace sm100

// Whether the decode kernel is the faster choice: for 1-2 tokens the streaming GEMV (K split
// over a thread-block cluster, no global partial sums) wins on layers of fewer than 1024 units
// (4096 x 28672 runs 21 us here against 29 us there; 4096 x 4096 9 us against 6 us).
bool awq_decode_wanted(int64_t M, int64_t K, int64_t N) {
  if (M > 2) return true;
  return ceil_div(N / 8, sm100::kDecWords) * ceil_div(K, 256) >= 1024;
}

// Workspace bytes the decode kernel needs for these shapes (0 when it does not take them).
size_t awq_decode_workspace(int64_t M, int64_t K, int64_t N, int64_t G, int s_dtype) {
  if (!sm100::dec_supported(M, K, N, G, s_dtype)) return 0;
  if (M <= 8) return sm100::dec_ws<1>(M, K, N, G);
  if (M <= 16) return sm100::dec_ws<2>(M, K, N, G);
  return sm100::dec_ws<4>(M, K, N, G);
}

// Routes 1 <= M <= 32 to the decode kernel; TO_EUNSUPPORTED (nothing launched, no error
// recorded) for shapes it does not take.
namespace {
int decode_dispatch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                    const int32_t* qz, const sm100::DecOut& out, int64_t M, int64_t K, int64_t N,
                    int64_t G, void* ws, size_t ws_bytes, cudaStream_t st) {
  const bool f16 = s_dtype == TO_F16;
  if (M <= 8)
    return f16 ? sm100::dispatch_decode<__half, 1>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st)
               : sm100::dispatch_decode<__nv_bfloat16, 1>(x, qw, s, qz, out, M, K, N, G, ws,
                                                          ws_bytes, st);
  if (M <= 16)
    return f16 ? sm100::dispatch_decode<__half, 2>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st)
               : sm100::dispatch_decode<__nv_bfloat16, 2>(x, qw, s, qz, out, M, K, N, G, ws,
                                                          ws_bytes, st);
  return f16 ? sm100::dispatch_decode<__half, 4>(x, qw, s, qz, out, M, K, N, G, ws, ws_bytes, st)
             : sm100::dispatch_decode<__nv_bfloat16, 4>(x, qw, s, qz, out, M, K, N, G, ws,
                                                        ws_bytes, st);
}
}  // namespace

// act < 0: y = x @ dequant(W), [M, N]; act >= 0: y = act(gate) * up, [M, N / 2], of a gate_up
// weight interleaved in blocks of 8 columns.
int awq_decode_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                      const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                      void* ws, size_t ws_bytes, cudaStream_t st, int act, int64_t ldx) {
  if (!sm100::dec_supported(M, K, N, G, s_dtype)) return TO_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(qw) || !aligned16(s) || !aligned16(qz) || !aligned16(y))
    return TO_EUNSUPPORTED;
  if (ldx != 0 && (ldx < K || ldx % 8 != 0)) return TO_EUNSUPPORTED;  // 16-byte row strides
  if (ws != nullptr && !aligned16(ws)) return TO_EUNSUPPORTED;
  sm100::DecOut out = {};
  out.y[0] = y;
  out.ny = 1;
  out.ld = (int)(act >= 0 ? N / 2 : N);
  out.col0 = 0;
  out.act = act;
  out.ldx = ldx;
  return decode_dispatch(x, qw, s, s_dtype, qz, out, M, K, N, G, ws, ws_bytes, st);
}

// The gathering form: this rank's [M, N] slice goes into the [M, N x world] output of every
// rank (y_ranks[r], the peers' mapped into this process) at columns [rank N, (rank + 1) N)
// (with act >= 0: its [M, N / 2] activation slice into [M, N / 2 x world]).
int awq_decode_gather_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                             const int32_t* qz, void* const* y_ranks, int world, int rank,
                             int64_t M, int64_t K, int64_t N, int64_t G, void* ws,
                             size_t ws_bytes, cudaStream_t st, int act) {
  if (!sm100::dec_supported(M, K, N, G, s_dtype)) return TO_EUNSUPPORTED;
  if (world < 1 || world > sm100::kDecMaxOut || N * world > INT32_MAX / 2) return TO_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(qw) || !aligned16(s) || !aligned16(qz)) return TO_EUNSUPPORTED;
  if (ws != nullptr && !aligned16(ws)) return TO_EUNSUPPORTED;
  sm100::DecOut out = {};
  for (int r = 0; r < world; ++r) {
    if (!aligned16(y_ranks[r])) return TO_EUNSUPPORTED;
    out.y[r] = y_ranks[r];
  }
  out.ny = world;
  const int64_t n_out = act >= 0 ? N / 2 : N;  // this rank's output columns
  out.ld = (int)(n_out * world);
  out.col0 = (int)(n_out * rank);
  out.act = act;
  return decode_dispatch(x, qw, s, s_dtype, qz, out, M, K, N, G, ws, ws_bytes, st);
}

}  // namespace tob
