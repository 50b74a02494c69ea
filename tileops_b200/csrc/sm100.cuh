// Inline-PTX building blocks for the sm_100a tensor-core kernels: mbarriers with
// time-bounded waits, TMA tile loads, the tcgen05 (5th-generation tensor core) MMA,
// tensor-memory (TMEM) allocation and loads, and the shared-memory matrix descriptors.
//
// Descriptor formats follow the PTX ISA "tcgen05 matrix descriptors" and "instruction
// descriptor" tables (sm_100a):
//   smem descriptor  : [0,14) start>>4 | [16,30) leading byte offset>>4 | [32,46) stride byte
//                      offset>>4 | [46,48) version = 1 | [49,52) base offset | [61,64) layout
//                      (2 = 128-byte swizzle)
//   instr descriptor : [4,6) D format (0 F16, 1 F32, 2 S32) | [7,10) A format | [10,13) B
//                      format | [15] A major | [16] B major | [17,23) N>>3 | [24,29) M>>4
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace tob {
namespace sm100 {

// Upper bound of any single wait in these kernels. A healthy wait lasts microseconds; a wait
// that reaches this limit records kErrWaitTimeout in the library's device error word and the
// kernel unwinds instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of parity `parity` to complete. Gives up when `*abort` becomes non-zero
// (another role failed) or after `limit_ns`; in the latter case it records the timeout in
// the device error word and raises `*abort` so every role of the CTA unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* err, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort = 1;
      if (err) atomicExch(err, (int)kErrWaitTimeout);
      return false;
    }
  }
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled load of box (x = inner coordinate in elements, y = row) into this CTA's shared
// memory, completing `bytes` on `bar`. x must be a multiple of 16 bytes worth of elements.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 3-D tiled load (coordinates innermost first), completing `bytes` on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, int x, int y, int z,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 2-D tiled store of a box from this CTA's shared memory to global (bulk-group completion).
// Rows / columns outside the tensor are clipped by the hardware.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, int x, int y, const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(x), "r"(y), "r"(smem_u32(src))
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Cluster-wide barrier with release/acquire ordering of shared memory (distributed shared
// memory stores before it are visible to every CTA of the cluster after it). The warp is
// reconverged first so that the aligned barrier counts it once, after all of its lanes' work.
__device__ __forceinline__ void cluster_sync_all() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Split cluster barrier: arrive (release) now, wait (acquire) later; work in between overlaps.
__device__ __forceinline__ void cluster_arrive_release() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
// Arrive without release ordering: enough to publish mbarrier initialisation that a
// fence.mbarrier_init.release.cluster already ordered.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  __syncwarp();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of `addr` (a shared::cta address) in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Bulk copy (no multicast) of `bytes` (multiple of 16) from this CTA's shared memory to a
// peer CTA's shared memory, completing on the peer's mbarrier (both shared::cluster addresses).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, const void* src, uint32_t bytes,
                                                  uint32_t peer_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "r"(smem_u32(src)), "r"(bytes), "r"(peer_bar)
      : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before later async-proxy ones:
// stores before a tensor-core or TMA-store read of them, and loads before a TMA load that
// refills the same buffer once it has been released.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
template <int NCOLS>
__device__ __forceinline__ void tmem_alloc(uint32_t* holder) {
  static_assert(NCOLS >= 32 && NCOLS <= 512 && (NCOLS & (NCOLS - 1)) == 0, "TMEM columns");
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(holder)),
               "r"(NCOLS)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
template <int NCOLS>
__device__ __forceinline__ void tmem_dealloc(uint32_t base) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(NCOLS)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory descriptor of a K-major tile stored as 128-byte rows with the 128-byte
// swizzle, 8-row groups 1024 bytes apart (the layout a TMA load with
// CU_TENSOR_MAP_SWIZZLE_128B and a 128-byte inner box produces). The tile base must be
// 1024-byte aligned; advancing the start address by 32 bytes selects the next 32-byte K slice.
__device__ __forceinline__ uint64_t smem_desc_kmajor_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;               // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;               // descriptor version for sm_100
  d |= (uint64_t)2 << 61;               // 128-byte swizzle
  return d;
}

// Shared-memory descriptor of an MN-major tile in the 128-byte-swizzle canonical layout:
// 1 KB atoms of 8 K-rows x 128 contiguous MN bytes (16-byte chunk c of row r stored at c ^ r),
// atoms along MN `lbo` bytes apart and 8-row K groups `sbo` bytes apart.
__device__ __forceinline__ uint64_t smem_desc_mnmajor_sw128(uint32_t addr, uint32_t lbo,
                                                           uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor with explicit operand majors (0 = K-major, 1 = MN-major).
__host__ __device__ constexpr uint32_t make_idesc_major(uint32_t d_fmt, uint32_t a_fmt,
                                                        uint32_t b_fmt, int M, int N,
                                                        uint32_t a_major, uint32_t b_major) {
  return (d_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_major << 15) | (b_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor: dense, K-major A and B.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t d_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                                  int M, int N) {
  return (d_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

enum class Kind : int { I8 = 0, E4M3 = 1, F16 = 2, BF16 = 3 };

// ------------------------------------------------------------------ host-side tensor maps
// (defined in gemm_sm100.cu)
// K-major operand [rows, cols] of `elem`-byte elements as box_rows x 128-byte boxes with the
// 128-byte swizzle; cached per (pointer, shape, box). slices > 1: a 3-D view {128 bytes, rows,
// cols * elem / 128} whose boxes bring `slices` consecutive 128-byte K slices of box_rows rows
// (cols * elem must be a multiple of 128).
int make_tmap_kmajor(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int elem,
                     int box_rows, int slices = 1);
// 16-bit output [rows, cols] for staged epilogue stores: 32-row boxes of box_cols columns.
int make_tmap_out16(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int box_cols,
                    int dtype);
// Plain row-major 2-D map without swizzle: box_cols x box_rows elements of `elem` bytes
// (elem 2 or 4), inner box bytes a multiple of 16.
int make_tmap_plain(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int elem,
                    int box_cols, int box_rows);
// 16-bit activations [M, K] (K % 64 == 0, rows ld >= K elements apart; ld = 0 means K) as
// {64, M, K/64} blocks: a box of box_tokens rows x box_blocks 64-element blocks lands as
// box_blocks [box_tokens x 128 B] 128-byte-swizzled tiles.
int make_tmap_x_blocks(CUtensorMap* out, const void* ptr, int64_t M, int64_t K, int box_tokens,
                       int box_blocks, int64_t ld = 0);

template <Kind K> struct KindTraits;
template <> struct KindTraits<Kind::I8> {
  static constexpr int kElemBytes = 1;
  static constexpr uint32_t kDFmt = 2, kAFmt = 1, kBFmt = 1;  // S32 <- s8 x s8
};
template <> struct KindTraits<Kind::E4M3> {
  static constexpr int kElemBytes = 1;
  static constexpr uint32_t kDFmt = 1, kAFmt = 0, kBFmt = 0;  // F32 <- e4m3 x e4m3
};
template <> struct KindTraits<Kind::F16> {
  static constexpr int kElemBytes = 2;
  static constexpr uint32_t kDFmt = 1, kAFmt = 0, kBFmt = 0;  // F32 <- f16 x f16
};
template <> struct KindTraits<Kind::BF16> {
  static constexpr int kElemBytes = 2;
  static constexpr uint32_t kDFmt = 1, kAFmt = 1, kBFmt = 1;  // F32 <- bf16 x bf16
};

// D[tmem] (+)= A[smem] * B[smem]^T for one 32-byte K slice; issued by one thread.
template <Kind K>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                     uint32_t idesc, uint32_t accumulate) {
  if constexpr (K == Kind::I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else if constexpr (K == Kind::E4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
  }
}

// Arrives once on `bar` when every tcgen05 operation this thread issued before has completed.
// ---- 2-CTA (cta_group::2) forms: a CTA pair of a (2,1,1) cluster computes one M=256 tile;
// the even ("leader") CTA issues the MMAs, each CTA holds 128 rows of A and half the N rows of
// B at the same shared-memory offsets, and each CTA's TMEM receives its 128 rows.
// Tensor memory is allocated / freed by the same warp of both CTAs, with the same holder offset.
template <int NCOLS>
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* holder) {
  static_assert(NCOLS >= 32 && NCOLS <= 512 && (NCOLS & (NCOLS - 1)) == 0, "TMEM columns");
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(holder)),
               "r"(NCOLS)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
template <int NCOLS>
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t base) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(NCOLS)
               : "memory");
}
template <Kind K>
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;  // disable-output-lane mask: no lane disabled
  if constexpr (K == Kind::I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z));
  } else if constexpr (K == Kind::E4M3) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z));
  }
}
// Arrive (release at cluster scope) on a barrier given by its shared::cluster address, which
// may belong to another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// Arrives on the barrier at `bar`'s offset in every CTA of `cta_mask` once the pair's earlier
// MMAs complete.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// Arrives on this CTA's barrier once the pair's earlier MMAs complete (no multicast).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 2-D tiled load into this CTA's shared memory whose bytes complete on the leader CTA's
// barrier (`leader_bar`: a shared::cluster address); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, int x, int y,
                                                 uint32_t leader_bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(leader_bar), "l"(policy)
      : "memory");
}

// 3-D form of tma_load_2d_pair (coordinates innermost first).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m, int x, int y,
                                                 int z, uint32_t leader_bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(leader_bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns: thread t of the warp receives lane
// (taddr.lane + t), columns taddr.col .. +15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace sm100
}  // namespace tob
