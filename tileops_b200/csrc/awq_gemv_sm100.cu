// Small-M AWQ W4A16 GEMM on sm_100a: y = x @ dequant(W) for 1 <= M <= 64 (tileops/quant_awq.py:
// 112-155, awq_gemm with a handful of tokens). The dispatch (awq.cu) sends it 33-64 tokens on
// layers whose tensor-core tiles would leave most SMs idle, and the 1-32-token shapes the
// stream-K decode kernel (awq_decode_sm100.cu) does not take.
//
// At decode sizes the layer is bound by streaming the packed int4 weights from HBM; the
// design keeps every SM's share of them in flight and spends as few instructions as possible
// per weight once it lands:
//   * TMA feed. One producer thread per CTA streams the CTA's K-chunk of packed weights as
//     8-16 KB tensor copies (cp.async.bulk.tensor, no multicast; 128-256 rows of the column tile)
//     through a ring of shared-memory stages with mbarrier completion and bounded waits. The
//     chunk's scales, zeros and x arrive once, one copy each (x through a 3-D view of 64-element
//     blocks that lands in the 128-byte-swizzled layout), so each stage costs one TMA
//     operation: the feed reaches HBM rate only with ~200 KB in flight per SM and few, large
//     copies. The weight copies of the first stages are issued before griddepcontrol.wait, so
//     with launch overlap on they stream while the previous kernel in the stream finishes; x
//     is copied only after that wait.
//   * Dequantisation in registers. Each consumer thread forms (w - z) exactly with the LOP3
//     magic-bias conversion and multiplies by the group scale in the model dtype -- the
//     reference's dequantised weight T((w - z) * s) (quant_awq.py:109), bit for bit.
//   * Register-operand MMA. The dequantised pairs go straight into the A fragments of
//     mma.sync.m16n8k16 (fp32 accumulate) with x as the B fragment, so the weights never make
//     a second trip through shared memory. tcgen05 reads both operands from shared memory
//     or tensor memory: the dequantised weights would cost 4 bytes of shared-memory traffic
//     per weight (store + MMA read), above the ~2.6 bytes per weight that shared memory can
//     serve at HBM rate, so for this HBM-bound shape the register-fed MMA is the faster one.
//     AWQ words hold 8 consecutive N columns of one K row, while an A fragment register holds
//     two consecutive K of one row; one PRMT per register transposes row pairs. The fragment
//     rows are this thread's own columns (any N order is allowed as long as the epilogue
//     follows it) and the K order within a 16-row step is permuted identically in A and B.
//   * Reduction. The 4 consumer warps split the 16-row MMA steps of a stage; their partial sums
//     are added in a fixed order in shared memory, then over the K-chunks of a column tile
//     through distributed shared memory of a thread-block cluster, each CTA of the cluster
//     reducing and storing one slice of the columns (deterministic; no global scratch, no
//     atomics).
#include <cooperative_groups.h>

#include <stdlib.h>

#include <algorithm>
#include <mutex>

#include "awq_common.cuh"
#include "sm100.cuh"

namespace cg = cooperative_groups;

namespace tob {
namespace sm100 {
namespace {

constexpr int kSmConsumers = 4;
constexpr int kSmThreads = 32 * (1 + kSmConsumers);
constexpr int kSmMaxStageBytes = 16384;  // one weight box per stage, at most 256 rows
constexpr int kSmMaxStages = 12;
constexpr size_t kSmSmemLimit = 112 * 1024;  // two CTAs per SM (228 KB, 1 KB reserved per CTA)
constexpr int kSmCtasPerSm = 2;

// Bytes of one stage (one TMA box of CW-word rows): as large as the 256-row box limit allows,
// since every copy costs a roughly fixed time on top of its bytes.
template <int CW>
__host__ __device__ constexpr int sm_stage_bytes() {
  return 256 * 4 * CW < kSmMaxStageBytes ? 256 * 4 * CW : kSmMaxStageBytes;
}

// Shared-memory plan of one CTA (offsets from a 1024-byte-aligned base):
//   x      : kchunk/64 tiles of [NT*8 tokens x 128 B] (128-byte swizzle), one 3-D TMA box
//   ring   : `stages` weight boxes of sm_stage_bytes<CW>() (8 or 16 KB)
//   scales : [szrows x 8CW] 16-bit, zeros : [szrows x CW] words -- the chunk's groups, one box each
//   tot    : fragment-order partial sums [16*WPQ*NT][32] fp32
//   barriers
struct SmPlan {
  int x_bytes, ring_bytes, s_bytes, z_bytes, tot_bytes, stages, szrows;
  size_t total() const {
    return 1024 + (size_t)x_bytes + ring_bytes + s_bytes + z_bytes + tot_bytes +
           (size_t)(2 * stages + 2) * 8 + 16;
  }
};

__host__ __device__ inline int round128(int v) { return (v + 127) & ~127; }

// Volatile so that the MMAs of a stage keep their place ahead of the stage's release.
template <typename T>
__device__ __forceinline__ void mma_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __half>::value) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <int WPQ>
__device__ __forceinline__ void lds_words(const uint32_t* p, uint32_t* out) {
  if constexpr (WPQ == 4) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else if constexpr (WPQ == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    out[0] = v.x; out[1] = v.y;
  } else {
    out[0] = *p;
  }
}

__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kSmConsumers) : "memory");
}


// Grid: (column tiles of CW = 8*WPQ packed words, K-chunks); the K-chunks of a column tile
// form one cluster. NT = 8-token tiles of M (1, 2 or 4 for M <= 8, 16, 32).
template <typename T, int NT, int WPQ>
__global__ void __launch_bounds__(kSmThreads, kSmCtasPerSm) k_awq_small_m(
    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_z,
    T* __restrict__ y, int M, int K, int N, int G, int kchunk, int ksplit, SmPlan plan,
    int* err) {
  using H2 = typename Half2Of<T>::type;
  constexpr int CW = 8 * WPQ;
  constexpr int kStageBytes = sm_stage_bytes<CW>();
  constexpr int kRows = kStageBytes / (4 * CW);      // K rows per stage
  constexpr int kSteps = kRows / 16 / kSmConsumers;  // 16-row MMA steps per warp per stage
  static_assert(kSteps >= 1 && kRows <= 256, "stage shape");
  constexpr int kXTile = 1024 * NT;                  // one 64-row block of x
  constexpr int kCols = CW * 8;
  const int stages = plan.stages;

  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  unsigned char* xarea = base;
  unsigned char* ring = xarea + plan.x_bytes;
  unsigned char* sarea = ring + plan.ring_bytes;
  unsigned char* zarea = sarea + plan.s_bytes;
  float* tot = reinterpret_cast<float*>(zarea + plan.z_bytes);  // [16*WPQ*NT][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(zarea + plan.z_bytes + plan.tot_bytes);
  uint64_t* empty = full + stages;
  uint64_t* szbar = empty + stages;
  uint64_t* xbar = szbar + 1;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(xbar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col0 = blockIdx.x * CW;  // first packed word of the tile
  const int kb = blockIdx.y * kchunk;
  const int ke = min(K, kb + kchunk);
  const int nst = (ke - kb + kRows - 1) / kRows;
  const int g0 = G == K ? 0 : kb / G;  // first group row of the chunk

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, kSmConsumers);
    }
    mbar_init(szbar, 1);
    mbar_init(xbar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_s);
      prefetch_tmap(&tm_z);
      prefetch_tmap(&tm_x);
      const uint64_t pol_w = policy_evict_first();  // streamed once
      const uint64_t pol_x = policy_evict_last();   // re-read by every column tile
      auto issue_w = [&](int st, int slot) {
        mbar_arrive_expect_tx(full + slot, kStageBytes);
        tma_load_2d(ring + slot * kStageBytes, &tm_w, col0, kb + st * kRows, full + slot, pol_w);
      };
      const int pre = min(nst, stages);
      for (int st = 0; st < pre; ++st) issue_w(st, st);
      mbar_arrive_expect_tx(szbar, (uint32_t)(plan.szrows * (8 * CW * 2 + CW * 4)));
      tma_load_2d(sarea, &tm_s, col0 * 8, g0, szbar, pol_w);
      tma_load_2d(zarea, &tm_z, col0, g0, szbar, pol_w);
      grid_dependency_wait();  // x may be the previous kernel's output
      grid_dependents_launch();
      mbar_arrive_expect_tx(xbar, (uint32_t)plan.x_bytes);
      tma_load_3d(xarea, &tm_x, 0, 0, kb / 64, xbar, pol_x);
      for (int st = pre; st < nst; ++st) {
        const int slot = st % stages;
        if (!mbar_wait(empty + slot, ((st / stages) - 1) & 1, abort_flag, err)) break;
        issue_w(st, slot);
      }
    } else {
      grid_dependency_wait();
      grid_dependents_launch();
    }
    __syncwarp();
  } else {
    const int cw = warp - 1;
    const int g = lane >> 2, q = lane & 3;
    grid_dependency_wait();  // y may still be read by the previous kernel
    grid_dependents_launch();

    float acc[WPQ][4][NT][4];
#pragma unroll
    for (int j = 0; j < WPQ; ++j)
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[j][p][t][e] = 0.f;

    bool ok = mbar_wait(szbar, 0, abort_flag, err) && mbar_wait(xbar, 0, abort_flag, err);
#pragma unroll 1
    for (int st = 0; ok && st < nst; ++st) {
      const int slot = st % stages;
      if (!mbar_wait(full + slot, (st / stages) & 1, abort_flag, err)) break;
      const uint32_t* wt = reinterpret_cast<const uint32_t*>(ring + slot * kStageBytes);
#pragma unroll
      for (int u = 0; u < kSteps; ++u) {
        const int step = cw * kSteps + u;           // 16-row step within the stage
        const int krow = st * kRows + 16 * step;    // row within the chunk
        if (kb + krow >= K) break;                  // past the end of K (warp-uniform)
        const int gr = G == K ? 0 : (kb + krow) / G - g0;

        // B fragments: x[token][krow + 4q .. +3] of each 8-token tile (128-byte swizzle).
        const unsigned char* xt = xarea + (krow >> 6) * kXTile;
        uint32_t bx[NT][2];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int row = g + 8 * t;
          const int byte = ((krow & 63) + 4 * q) * 2;
          const int chunk = (byte >> 4) ^ (row & 7);
          const uint2 v = *reinterpret_cast<const uint2*>(xt + row * 128 + chunk * 16 + (byte & 15));
          bx[t][0] = v.x;
          bx[t][1] = v.y;
        }
        // This thread's 4 K rows (16*step + 4q + i) of its WPQ words, and their group's
        // zeros and scales.
        uint32_t wr[4][WPQ];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          lds_words<WPQ>(wt + (16 * step + 4 * q + i) * CW + g * WPQ, wr[i]);
        uint32_t zw[WPQ];
        lds_words<WPQ>(reinterpret_cast<const uint32_t*>(zarea) + gr * CW + g * WPQ, zw);
        const H2* srow = reinterpret_cast<const H2*>(sarea) + gr * 4 * CW;

#pragma unroll
        for (int j = 0; j < WPQ; ++j) {
          H2 zc[4];
          awq_zero_consts<T>(zw[j], zc);
          const H2* sc = srow + (g * WPQ + j) * 4;  // 4 pairs = the word's 8 columns
          H2 s4[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) s4[p] = sc[p];
          uint32_t wq[4][4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            H2 d[4];
            awq_word_diff<T>(wr[i][j], zc, d);
#pragma unroll
            for (int p = 0; p < 4; ++p) wq[i][p] = bits_of(__hmul2(d[p], s4[p]));
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            // Fragment rows g / g+8 = columns 2p / 2p+1 of the word; K pairs (4q,4q+1) and
            // (4q+2,4q+3) sit at MMA k = 2q and 2q+8, as in bx.
            const uint32_t a0 = __byte_perm(wq[0][p], wq[1][p], 0x5410);
            const uint32_t a1 = __byte_perm(wq[0][p], wq[1][p], 0x7632);
            const uint32_t a2 = __byte_perm(wq[2][p], wq[3][p], 0x5410);
            const uint32_t a3 = __byte_perm(wq[2][p], wq[3][p], 0x7632);
#pragma unroll
            for (int t = 0; t < NT; ++t)
              mma_16816<T>(acc[j][p][t], a0, a1, a2, a3, bx[t][0], bx[t][1]);
          }
        }
      }
      // The slot is refilled by TMA (async proxy) once all 4 warps release it: order this
      // thread's generic-proxy reads of the slot before those writes, then release.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(empty + slot);
    }

    // Consumer warps add their partial sums into tot in a fixed order. tot is kept in
    // fragment order, tot[v][lane] with v = ((j*4 + p)*NT + t)*4 + e, so every store of a
    // pass is one conflict-free 128-byte row; coords() below maps it back to (token, column).
#pragma unroll 1
    for (int w = 0; w < kSmConsumers; ++w) {
      if (cw == w) {
#pragma unroll
        for (int j = 0; j < WPQ; ++j)
#pragma unroll
          for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                float* d = tot + (((j * 4 + p) * NT + t) * 4 + e) * 32 + lane;
                if (w == 0) *d = acc[j][p][t][e];
                else *d += acc[j][p][t][e];
              }
      }
      consumer_bar();
    }
  }

  // Only the M real token rows leave the CTA. With a K split, cluster rank r sums slice r of
  // every rank's partials (ranks in a fixed order) and stores it: the reduction and the
  // stores are spread over the cluster, one round of remote loads per element.
  constexpr int kVals = NT * 8 * kCols;  // = 16 * WPQ * NT values x 32 lanes
  auto coords = [&](int idx, int& m, int& n) {
    const int v = idx >> 5, l = idx & 31;
    const int e = v & 3, t = (v >> 2) % NT, jp = (v >> 2) / NT;  // jp = j*4 + p
    const int j = jp >> 2, p = jp & 3;
    m = 8 * t + 2 * (l & 3) + (e & 1);
    n = col0 * 8 + ((l >> 2) * WPQ + j) * 8 + 2 * p + (e >> 1);
  };
  if (ksplit > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster_sync_all();
    // ceil(kVals / ksplit) values per rank: the K split need not divide them.
    const int per = (kVals + ksplit - 1) / ksplit;
    const int i0 = blockIdx.y * per;
    const int i1 = min(kVals, i0 + per);
    for (int i = i0 + threadIdx.x; i < i1; i += kSmThreads) {
      int m, n;
      coords(i, m, n);
      if (m >= M || n >= N) continue;
      float v[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) v[r] = r < ksplit ? cluster.map_shared_rank(tot, r)[i] : 0.f;
      float a = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) a += v[r];
      y[(int64_t)m * N + n] = from_f32<T>(a);
    }
    cluster_sync_all();  // peers keep their shared memory until every slice has been read
  } else {
    __syncwarp();
    __syncthreads();
    for (int i = threadIdx.x; i < kVals; i += kSmThreads) {
      int m, n;
      coords(i, m, n);
      if (m < M && n < N) y[(int64_t)m * N + n] = from_f32<T>(tot[i]);
    }
  }
}

// Shared-memory plan for a K-chunk; returns false when even the smallest ring does not fit.
template <int NT, int WPQ>
bool plan_small_m(int64_t K, int64_t G, int kchunk, SmPlan* p) {
  constexpr int CW = 8 * WPQ;
  constexpr int kRows = sm_stage_bytes<CW>() / (4 * CW);
  p->x_bytes = (kchunk / 64) * 1024 * NT;
  p->szrows = G == K ? 1 : (int)(kchunk / G);
  p->s_bytes = round128(p->szrows * 8 * CW * 2);
  p->z_bytes = round128(p->szrows * CW * 4);
  p->tot_bytes = NT * 8 * CW * 8 * 4;
  p->stages = std::min(kchunk / kRows, kSmMaxStages);
  if (const char* v = tuning_env("TOB_SMALL_M_STAGES")) {  // measurement override
    const int want = atoi(v);
    if (want >= 1) p->stages = std::min(p->stages, want);
  }
  for (;;) {
    p->ring_bytes = p->stages * sm_stage_bytes<CW>();
    if (p->total() <= kSmSmemLimit) return p->szrows <= 256 && kchunk / 64 <= 256;
    if (p->stages <= 2) return false;
    --p->stages;
  }
}

template <typename T, int NT, int WPQ>
int launch_small_m(const void* x, const int32_t* qw, const void* s, const int32_t* qz, void* y,
                   int64_t M, int64_t K, int64_t N, int64_t G, int ksplit, cudaStream_t st) {
  constexpr int CW = 8 * WPQ;
  constexpr int kRows = sm_stage_bytes<CW>() / (4 * CW);
  const int64_t words = N / 8;
  const int tiles = (int)ceil_div(words, CW);
  // K-chunks are whole stages and whole groups; the x, scale and zero slices must fit too.
  const int unit = (G != K && G > kRows) ? (int)G : kRows;
  SmPlan plan;
  int kchunk = 0;
  for (;; ksplit *= 2) {
    kchunk = (int)(ceil_div(ceil_div(K, ksplit), unit) * unit);
    if (plan_small_m<NT, WPQ>(K, G, kchunk, &plan)) break;
    if (ksplit >= 8) return TO_EUNSUPPORTED;
  }
  ksplit = (int)ceil_div(K, kchunk);
  auto kern = k_awq_small_m<T, NT, WPQ>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, (int)kSmSmemLimit);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "awq small-M gemm: shared memory attribute");
  CUtensorMap tx, tw, ts, tz;
  int rc = make_tmap_x_blocks(&tx, x, M, K, 8 * NT, kchunk / 64);
  if (!rc) rc = make_tmap_plain(&tw, qw, K, words, 4, CW, kRows);
  if (!rc) rc = make_tmap_plain(&ts, s, K / G, N, 2, 8 * CW, plan.szrows);
  if (!rc) rc = make_tmap_plain(&tz, qz, K / G, words, 4, CW, plan.szrows);
  if (rc) return rc;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, ksplit, 1);
  cfg.blockDim = dim3(kSmThreads, 1, 1);
  cfg.dynamicSmemBytes = plan.total();
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (ksplit > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = ksplit;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (launch_overlap()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, ts, tz, (T*)y, (int)M, (int)K, (int)N,
                                     (int)G, kchunk, ksplit, plan, device_error_ptr());
  if (e != cudaSuccess) return cuda_fail(e, "awq small-M gemm launch");
  return check_launch("awq small-M gemm");
}

template <typename T, int NT>
int dispatch_small_m(const void* x, const int32_t* qw, const void* s, const int32_t* qz, void* y,
                     int64_t M, int64_t K, int64_t N, int64_t G, cudaStream_t st) {
  const int64_t words = N / 8;
  const int64_t sms = sm_count();
  // Widest column tile that still yields ~1.5 CTAs per SM at the largest K split (the
  // accumulators, 16 x WPQ x NT registers, cap WPQ at 4 / NT).
  int wpq = NT == 1 ? 4 : (NT == 2 ? 2 : 1);
  while (wpq > 1 && ceil_div(words, 8 * wpq) * 8 < sms + sms / 2) wpq >>= 1;
  const int64_t tiles = ceil_div(words, 8 * wpq);
  int ksplit = 1;
  while (ksplit < 8 && tiles * ksplit < 2 * sms && K >= (int64_t)ksplit * 2 * 256) ksplit *= 2;
  if (const char* v = tuning_env("TOB_SMALL_M_KSPLIT")) {  // measurement override: 1, 2, 4 or 8
    const int want = atoi(v);
    if (want == 1 || want == 2 || want == 4 || want == 8) ksplit = want;
  }
  if constexpr (NT == 1) {
    if (wpq == 4) return launch_small_m<T, NT, 4>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
  }
  if constexpr (NT <= 2) {
    if (wpq == 2) return launch_small_m<T, NT, 2>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
  }
  return launch_small_m<T, NT, 1>(x, qw, s, qz, y, M, K, N, G, ksplit, st);
}

}  // namespace
}  // namespace sm100

// Routes 1 <= M <= 64 to the TMA-fed small-M kernel when the shapes meet its TMA constraints;
// TO_EUNSUPPORTED (nothing launched, no error recorded) otherwise.
int awq_small_m_launch(const void* x, const int32_t* qw, const void* s, int s_dtype,
                       const int32_t* qz, void* y, int64_t M, int64_t K, int64_t N, int64_t G,
                       cudaStream_t st) {
  if (M < 1 || M > 64) return TO_EUNSUPPORTED;
  if (s_dtype != TO_F16 && s_dtype != TO_BF16) return TO_EUNSUPPORTED;
  if (N % 32 != 0 || K % 64 != 0) return TO_EUNSUPPORTED;  // TMA strides, whole x blocks
  if (!(G == K || G % 64 == 0 || G == 32)) return TO_EUNSUPPORTED;
  if (N > INT32_MAX || K > INT32_MAX) return TO_EUNSUPPORTED;
  if (!aligned16(x) || !aligned16(qw) || !aligned16(s) || !aligned16(qz)) return TO_EUNSUPPORTED;
  const bool f16 = s_dtype == TO_F16;
  if (M <= 8)
    return f16 ? sm100::dispatch_small_m<__half, 1>(x, qw, s, qz, y, M, K, N, G, st)
               : sm100::dispatch_small_m<__nv_bfloat16, 1>(x, qw, s, qz, y, M, K, N, G, st);
  if (M <= 16)
    return f16 ? sm100::dispatch_small_m<__half, 2>(x, qw, s, qz, y, M, K, N, G, st)
               : sm100::dispatch_small_m<__nv_bfloat16, 2>(x, qw, s, qz, y, M, K, N, G, st);
  int rc = M <= 32
               ? (f16 ? sm100::dispatch_small_m<__half, 4>(x, qw, s, qz, y, M, K, N, G, st)
                      : sm100::dispatch_small_m<__nv_bfloat16, 4>(x, qw, s, qz, y, M, K, N, G,
                                                                  st))
               : (f16 ? sm100::dispatch_small_m<__half, 8>(x, qw, s, qz, y, M, K, N, G, st)
                      : sm100::dispatch_small_m<__nv_bfloat16, 8>(x, qw, s, qz, y, M, K, N, G,
                                                                  st));
  if (rc != TO_EUNSUPPORTED) return rc;
  // The tokens of x for a long K chunk do not fit next to the weight ring: run them as two
  // launches of half the tile (nothing was launched above).
  const int64_t half = M <= 32 ? 16 : 32;
  const char* x2 = static_cast<const char*>(x) + (size_t)half * K * 2;
  char* y2 = static_cast<char*>(y) + (size_t)half * N * 2;
  rc = awq_small_m_launch(x, qw, s, s_dtype, qz, y, half, K, N, G, st);
  if (rc != TO_OK) return rc;
  return awq_small_m_launch(x2, qw, s, s_dtype, qz, y2, M - half, K, N, G, st);
}

}  // namespace tob
