// Gated activations of an MLP block (tileops/fused.py:97-114, kernels
// tileops/backend/cuda/fused.py:17-43):
//   silu_and_mul: C = silu(A) * B,      silu(x) = x * sigmoid(x)
//   gelu_and_mul: C = gelu_tanh(A) * B, gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
// A, B, C are [rows, cols] with unit column stride and their own row strides, so the gate and
// up halves of a fused gate_up output ([M, 2F], gate in columns [0, F), up in [F, 2F)) are read
// in place. HBM-bound: 16-byte vector loads of A and B, one 16-byte store of C per vector, a
// grid sized to the SM count. Arithmetic in fp32; the activation is rounded to the tensor dtype
// before the multiply and the product rounded again, the two roundings of `act(a) * b` in the
// tensor dtype.
#include "act.cuh"
#include "common.cuh"

namespace tob {
namespace {

constexpr int kThreads = 256;

// Vector form: every row starts 16-byte aligned and cols is a multiple of V. Vector j of a row
// of A and B starts at element j * in_vs (V for plain rows; 2V for a gate_up output whose gate
// and up columns alternate in blocks of V, with B = A + V).
template <typename T, int OP, int V>
__global__ void __launch_bounds__(kThreads)
    k_act_mul_vec(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c,
                  int64_t rows, int64_t vpr, int64_t lda, int64_t ldb, int64_t ldc,
                  int64_t in_vs) {
  const int64_t total = rows * vpr;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / vpr, v = i - r * vpr;
    const Pack<T, V> va = *reinterpret_cast<const Pack<T, V>*>(a + r * lda + v * in_vs);
    const Pack<T, V> vb = *reinterpret_cast<const Pack<T, V>*>(b + r * ldb + v * in_vs);
    Pack<T, V> vc;
#pragma unroll
    for (int j = 0; j < V; ++j) vc.v[j] = act_mul<T, OP>(va.v[j], vb.v[j]);
    *reinterpret_cast<Pack<T, V>*>(c + r * ldc + v * V) = vc;
  }
}

// Any alignment and width.
template <typename T, int OP>
__global__ void __launch_bounds__(kThreads)
    k_act_mul(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c, int64_t rows,
              int64_t cols, int64_t lda, int64_t ldb, int64_t ldc) {
  const int64_t total = rows * cols;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / cols, col = i - r * cols;
    c[r * ldc + col] = act_mul<T, OP>(a[r * lda + col], b[r * ldb + col]);
  }
}

template <typename T, int OP>
int launch_act_mul(const void* a, const void* b, void* c, int64_t rows, int64_t cols,
                   int64_t lda, int64_t ldb, int64_t ldc, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = cols % V == 0 && lda % V == 0 && ldb % V == 0 && ldc % V == 0 &&
                   aligned16(a) && aligned16(b) && aligned16(c);
  if (vec) {
    const int64_t vpr = cols / V;
    k_act_mul_vec<T, OP, V><<<grid_for(rows * vpr, kThreads), kThreads, 0, st>>>(
        (const T*)a, (const T*)b, (T*)c, rows, vpr, lda, ldb, ldc, (int64_t)V);
  } else {
    k_act_mul<T, OP><<<grid_for(rows * cols, kThreads), kThreads, 0, st>>>(
        (const T*)a, (const T*)b, (T*)c, rows, cols, lda, ldb, ldc);
  }
  return check_launch(OP == kSilu ? "silu_and_mul" : "gelu_and_mul");
}

template <int OP>
int act_mul_entry(const char* op, const void* a, const void* b, void* c, int dtype, int64_t rows,
                  int64_t cols, int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  if (rows < 0 || cols < 0 || (rows > 1 && (lda < cols || ldb < cols || ldc < cols)))
    return fail(TO_EINVAL, "%s: invalid shape rows=%lld cols=%lld strides=(%lld, %lld, %lld)",
                op, (long long)rows, (long long)cols, (long long)lda, (long long)ldb,
                (long long)ldc);
  if (rows == 0 || cols == 0) return TO_OK;
  if (!a || !b || !c) return fail(TO_EINVAL, "%s: null pointer", op);
  cudaStream_t st = (cudaStream_t)stream;
  TOB_DISPATCH_FLOAT(dtype, T,
                     return launch_act_mul<T, OP>(a, b, c, rows, cols, lda, ldb, ldc, st));
  return TO_OK;
}

}  // namespace

// C[rows, cols / 2] = act(gate) * up over a gate_up output Y[rows, cols] (row stride ldy) whose
// gate and up columns alternate in blocks of 8: block 2j holds gate columns 8j..8j+7, block
// 2j + 1 the up columns of the same indices. 16-bit dtypes, cols % 16 == 0, 16-byte aligned
// rows (one 16-byte vector is one block).
int act_mul_interleaved_launch(const void* y, void* c, int dtype, int64_t rows, int64_t cols,
                               int64_t ldy, int64_t ldc, int act, cudaStream_t st) {
  if (cols % 16 != 0 || ldy % 8 != 0 || ldc % 8 != 0 || !aligned16(y) || !aligned16(c))
    return fail(TO_EINVAL, "gate_up activation: cols %% 16 and 16-byte aligned rows required");
  if (rows == 0 || cols == 0) return TO_OK;
  const int64_t vpr = cols / 16;
  const unsigned grid = grid_for(rows * vpr, kThreads);
  auto run = [&](auto tag) {
    using T = decltype(tag);
    const T* a = static_cast<const T*>(y);
    if (act == kSilu)
      k_act_mul_vec<T, kSilu, 8><<<grid, kThreads, 0, st>>>(a, a + 8, (T*)c, rows, vpr, ldy,
                                                             ldy, ldc, 16);
    else
      k_act_mul_vec<T, kGeluTanh, 8><<<grid, kThreads, 0, st>>>(a, a + 8, (T*)c, rows, vpr, ldy,
                                                                 ldy, ldc, 16);
  };
  if (dtype == TO_F16)
    run(__half{});
  else if (dtype == TO_BF16)
    run(__nv_bfloat16{});
  else
    return fail(TO_EUNSUPPORTED, "gate_up activation: fp16 or bf16 only");
  return check_launch(act == kSilu ? "awq_gemm_silu_and_mul" : "awq_gemm_gelu_and_mul");
}

}  // namespace tob

extern "C" {

int to_silu_and_mul(const void* a, const void* b, void* c, int dtype, int64_t rows, int64_t cols,
                    int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return tob::act_mul_entry<tob::kSilu>("silu_and_mul", a, b, c, dtype, rows, cols, lda, ldb,
                                        ldc, stream);
}

int to_gelu_and_mul(const void* a, const void* b, void* c, int dtype, int64_t rows, int64_t cols,
                    int64_t lda, int64_t ldb, int64_t ldc, void* stream) {
  return tob::act_mul_entry<tob::kGeluTanh>("gelu_and_mul", a, b, c, dtype, rows, cols, lda,
                                            ldb, ldc, stream);
}

}  // extern "C"
