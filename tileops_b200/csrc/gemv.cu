// Dense matrix-vector product (tileops/blas/gemv.py:22, kernel tileops/backend/cuda/blas/gemv.py:10-46):
//   y [M] = A [M, K] @ x [K], A row-major, fp32 accumulation, y rounded once to the dtype.
// HBM-bound: every byte of A is read once, x is re-read out of L1/L2, and 16-bit products are
// accumulated with the mixed-precision FMA (two conversions per element would otherwise bound
// the kernel below the HBM rate). Tall matrices with aligned rows of at least 2 KB stream A
// through per-warp bulk-copy rings (k_gemv_bulk below); every other shape runs k_gemv, where A
// arrives by 16-byte streaming loads (no L1 allocation) and a team of TW warps owns one row. TW
// grows (1, 2, 4, 8) while the teams would leave the SMs short of warps and each lane still has
// at least four vectors of the row, so short-and-wide matrices keep enough loads in flight; each
// lane issues four loads of A before their multiply-adds. The reduction order (lane stride, then
// the warp's shuffle tree, then the team's warps in order) is fixed, so results do not depend on
// the grid. With launch overlap on (to_set_launch_overlap), a launch prefetches its first vectors of
// A into L2 while the previous kernel in the stream finishes, and reads x and writes y only after
// that kernel has completed.
#include "sm100.cuh"

namespace tob {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

template <typename T, int V>
__device__ __forceinline__ Pack<T, V> ld_row(const Pack<T, V>* p) {
  if constexpr (sizeof(Pack<T, V>) == 16) {
    const uint4 r = ld_stream_v4(p);
    return *reinterpret_cast<const Pack<T, V>*>(&r);
  } else {
    return *p;
  }
}

// acc += a[e] * x[e] for e = 0 .. V-1 in order, each step one fused multiply-add in fp32 (the
// product of two 16-bit values is exact in fp32, so each step rounds once). 16-bit pairs use the
// mixed-precision fma.rn.f32.{f16,bf16}, which takes the 16-bit operands directly: the same
// result as converting both and calling fmaf, without the two conversions per element.
__device__ __forceinline__ float fma2_mixed(__half, uint32_t a2, uint32_t x2, float acc) {
  asm("{\n\t.reg .b16 al, ah, xl, xh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.f16 %0, al, xl, %0;\n\tfma.rn.f32.f16 %0, ah, xh, %0;\n\t}"
      : "+f"(acc)
      : "r"(a2), "r"(x2));
  return acc;
}
__device__ __forceinline__ float fma2_mixed(__nv_bfloat16, uint32_t a2, uint32_t x2, float acc) {
  asm("{\n\t.reg .b16 al, ah, xl, xh;\n\tmov.b32 {al, ah}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, al, xl, %0;\n\tfma.rn.f32.bf16 %0, ah, xh, %0;\n\t}"
      : "+f"(acc)
      : "r"(a2), "r"(x2));
  return acc;
}

template <typename T, int V>
__device__ __forceinline__ float dot_pack(const Pack<T, V>& a, const Pack<T, V>& x, float acc) {
  if constexpr (sizeof(T) == 2 && V % 2 == 0) {
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(a.v);
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(x.v);
#pragma unroll
    for (int e = 0; e < V / 2; ++e) acc = fma2_mixed(T(), aw[e], xw[e], acc);
  } else {
#pragma unroll
    for (int e = 0; e < V; ++e) acc = fmaf(to_f32<T>(a.v[e]), to_f32<T>(x.v[e]), acc);
  }
  return acc;
}

// V elements per load (16 bytes when the rows are 16-byte aligned, else 1); nvec = K / V.
template <typename T, int V, int TW>
__global__ void __launch_bounds__(kThreads)
    k_gemv(const T* __restrict__ a, const T* __restrict__ x, T* __restrict__ y, int64_t M,
           int64_t nvec) {
  constexpr int kRows = kWarps / TW;  // rows per block pass
  constexpr int kTeam = 32 * TW;      // threads per row
  __shared__ float part[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = warp / TW;
  const int t = threadIdx.x - slot * kTeam;
  using P = Pack<T, V>;
  const P* xv = reinterpret_cast<const P*>(x);
  // Before waiting on the previous grid (programmatic dependent launch), prefetch into L2 the
  // first vectors of A this thread reads; x may be that grid's output and y may still be read by
  // it, so both are touched only after the wait. Both calls are no-ops without the overlap.
  {
    const int64_t row0 = (int64_t)blockIdx.x * kRows + slot;
    if (row0 < M) {
      const P* ar = reinterpret_cast<const P*>(a) + row0 * nvec;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (t + u * kTeam < nvec) prefetch_l2(ar + t + u * kTeam);
    }
  }
  grid_dependency_wait();
  grid_dependents_launch();
  for (int64_t base = (int64_t)blockIdx.x * kRows; base < M; base += (int64_t)gridDim.x * kRows) {
    const int64_t row = base + slot;
    float acc = 0.f;
    if (row < M) {
      const P* ar = reinterpret_cast<const P*>(a) + row * nvec;
      int64_t j = t;
      for (; j + (kUnroll - 1) * kTeam < nvec; j += kUnroll * kTeam) {
        P pa[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) pa[u] = ld_row<T, V>(ar + j + u * kTeam);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) acc = dot_pack<T, V>(pa[u], xv[j + u * kTeam], acc);
      }
      for (; j < nvec; j += kTeam) acc = dot_pack<T, V>(ld_row<T, V>(ar + j), xv[j], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if constexpr (TW == 1) {
      if (lane == 0 && row < M) y[row] = from_f32<T>(acc);
    } else {
      if (lane == 0) part[warp] = acc;
      __syncthreads();
      if (t == 0 && row < M) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < TW; ++w) s += part[slot * TW + w];
        y[row] = from_f32<T>(s);
      }
      __syncthreads();
    }
  }
}

// ------------------------------------------------------------------ bulk-copy streaming path
// For tall matrices (every warp of the grid gets at least one row) with 16-byte aligned rows of
// at least 2 KB: each warp owns rows gw, gw + W, ... (W warps in the grid) and streams them
// through its own ring of kBulkStages shared-memory stages with one bulk copy (cp.async.bulk,
// no multicast) of up to kBulkChunk bytes per stage, issued by the warp's lane 0 and completed
// on the stage's mbarrier. The bytes in flight per SM are therefore explicit
// (8 warps x 3 stages x 8 KB), not left to the instruction scheduler. Lanes read the stage's
// 16-byte vectors in lane order (conflict-free) against x from L1; the row's sum is the lanes'
// partials in the warp's shuffle tree, the order of the one-warp-per-row register path, so the two
// give identical results.
constexpr int kBulkWarps = 8;
constexpr int kBulkStages = 3;
constexpr int kBulkChunk = 8192;
constexpr int kBulkSmem = kBulkWarps * kBulkStages * kBulkChunk + kBulkWarps * kBulkStages * 8 + 16;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(sm100::smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(sm100::smem_u32(bar)), "l"(policy)
      : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kBulkWarps * 32, 1)
    k_gemv_bulk(const T* __restrict__ a, const T* __restrict__ x, T* __restrict__ y, int64_t M,
                int64_t row_bytes, int* err) {
  using namespace sm100;
  constexpr int V = 16 / sizeof(T);
  using P = Pack<T, V>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* ring = smem_raw + warp * kBulkStages * kBulkChunk;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kBulkWarps * kBulkStages * kBulkChunk) +
                   warp * kBulkStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(
      smem_raw + kBulkWarps * kBulkStages * kBulkChunk + kBulkWarps * kBulkStages * 8);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kBulkWarps * kBulkStages; ++i)
      mbar_init(reinterpret_cast<uint64_t*>(smem_raw + kBulkWarps * kBulkStages * kBulkChunk) + i, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t nwarps = (int64_t)gridDim.x * kBulkWarps;
  const int64_t gw = (int64_t)blockIdx.x * kBulkWarps + warp;
  const int64_t nch = (row_bytes + kBulkChunk - 1) / kBulkChunk;
  const int64_t rows = gw < M ? (M - 1 - gw) / nwarps + 1 : 0;  // rows of this warp
  const int64_t units = rows * nch;                               // (row, chunk) copies
  const unsigned char* a8 = reinterpret_cast<const unsigned char*>(a);
  const uint64_t pol = policy_evict_first();
  auto unit_bytes = [&](int64_t u) -> uint32_t {
    const int64_t off = (u % nch) * kBulkChunk;
    return (uint32_t)(row_bytes - off < kBulkChunk ? row_bytes - off : kBulkChunk);
  };
  auto issue = [&](int64_t u) {
    const int s = (int)(u % kBulkStages);
    const int64_t row = gw + (u / nch) * nwarps;
    const uint32_t bytes = unit_bytes(u);
    mbar_arrive_expect_tx(full + s, bytes);
    bulk_load(ring + s * kBulkChunk, a8 + row * row_bytes + (u % nch) * kBulkChunk, bytes,
              full + s, pol);
  };

  // A only before waiting on the previous grid: x may be its output, y may still be read by it.
  int64_t issued = 0;
  if (lane == 0)
    for (; issued < units && issued < kBulkStages; ++issued) issue(issued);
  grid_dependency_wait();
  grid_dependents_launch();

  const P* xv = reinterpret_cast<const P*>(x);
  float acc = 0.f;
  int64_t u = 0;
  for (; u < units; ++u) {
    const int s = (int)(u % kBulkStages);
    const bool ok = mbar_wait(full + s, (uint32_t)((u / kBulkStages) & 1), abort_flag, err);
    if (!__all_sync(0xffffffffu, ok)) break;  // the warp leaves together
    const int64_t c = u % nch;
    const int nv = (int)(unit_bytes(u) >> 4);
    const P* sv = reinterpret_cast<const P*>(ring + s * kBulkChunk);
    const P* xc = xv + c * (kBulkChunk / 16);
#pragma unroll 4
    for (int v = lane; v < nv; v += 32) acc = dot_pack<T, V>(sv[v], xc[v], acc);
    // The stage is refilled by the async proxy: order this lane's reads of it first.
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && issued < units) issue(issued++);
    if (c == nch - 1) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) y[gw + (u / nch) * nwarps] = from_f32<T>(acc);
      acc = 0.f;
    }
  }
  // After a wait gave up, lane 0 lets its copies still in flight land before the CTA exits.
  if (lane == 0 && u < units) {
    int stop = 0;
    for (int64_t d = u; d < issued; ++d)
      mbar_wait(full + (int)(d % kBulkStages), (uint32_t)((d / kBulkStages) & 1), &stop, nullptr,
                100000000ull);
  }
}

template <typename T>
int launch_gemv_bulk(const void* a, const void* x, void* y, int64_t M, int64_t K,
                     cudaStream_t st) {
  auto kern = k_gemv_bulk<T>;
  const cudaError_t attr_err = ensure_smem_attr((const void*)kern, kBulkSmem);
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "gemv: shared memory attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sm_count(), 1, 1);
  cfg.blockDim = dim3(kBulkWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = kBulkSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (launch_overlap()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, (const T*)a, (const T*)x, (T*)y, M,
                                           K * (int64_t)sizeof(T), device_error_ptr());
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return check_launch("gemv");
}

template <typename T, int V, int TW>
cudaError_t launch_tw(const T* a, const T* x, T* y, int64_t M, int64_t nvec, cudaStream_t st) {
  constexpr int kRows = kWarps / TW;
  int64_t blocks = ceil_div(M, kRows);
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (launch_overlap()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, k_gemv<T, V, TW>, a, x, y, M, nvec);
}

template <typename T, int V>
cudaError_t launch_v(const void* a, const void* x, void* y, int64_t M, int64_t nvec, cudaStream_t st) {
  // Grow the row team while the teams fill less than half of the resident warps (64 per SM)
  // and every lane of the doubled team still loads kUnroll vectors of the row.
  const int64_t want = (int64_t)sm_count() * 32;
  int tw = 1;
  while (tw < 8 && M * tw < want && nvec >= (int64_t)tw * 2 * 32 * kUnroll) tw *= 2;
  const T* pa = (const T*)a;
  const T* px = (const T*)x;
  T* py = (T*)y;
  switch (tw) {
    case 1: return launch_tw<T, V, 1>(pa, px, py, M, nvec, st);
    case 2: return launch_tw<T, V, 2>(pa, px, py, M, nvec, st);
    case 4: return launch_tw<T, V, 4>(pa, px, py, M, nvec, st);
    default: return launch_tw<T, V, 8>(pa, px, py, M, nvec, st);
  }
}

template <typename T>
int launch_gemv(const void* a, const void* x, void* y, int64_t M, int64_t K, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = K % V == 0 && aligned16(a) && aligned16(x);
  if (vec && K * (int64_t)sizeof(T) >= 2048 && M >= (int64_t)sm_count() * kBulkWarps)
    return launch_gemv_bulk<T>(a, x, y, M, K, st);
  const cudaError_t e = vec
                            ? launch_v<T, V>(a, x, y, M, K / V, st)
                            : launch_v<T, 1>(a, x, y, M, K, st);
  if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  return check_launch("gemv");
}

}  // namespace
}  // namespace tob

extern "C" int to_gemv(const void* a, const void* x, void* y, int dtype, int64_t M, int64_t K,
                       void* stream) {
  using namespace tob;
  if (M < 0 || K < 0)
    return fail(TO_EINVAL, "gemv: invalid shape M=%lld K=%lld", (long long)M, (long long)K);
  if (M == 0) return TO_OK;
  if (!y || (K > 0 && (!a || !x))) return fail(TO_EINVAL, "gemv: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 0) {
    // an empty sum: y = 0 (all-zero bits are +0.0 in every float dtype)
    size_t bytes = 0;
    TOB_DISPATCH_FLOAT(dtype, T, bytes = (size_t)M * sizeof(T));
    const cudaError_t e = cudaMemsetAsync(y, 0, bytes, st);
    return e == cudaSuccess ? TO_OK : cuda_fail(e, "gemv: memset");
  }
  TOB_DISPATCH_FLOAT(dtype, T, return launch_gemv<T>(a, x, y, M, K, st));
  return TO_OK;
}
