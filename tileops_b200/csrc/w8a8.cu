// W8A8 entry points: validate, then route each call to the tcgen05 tensor-core kernel when
// the shape and scale layout fit its tiles, else to the generic block-scaled kernel.
#include "common.cuh"

namespace tob {
int w8a8_generic_launch(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                        void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M,
                        int64_t N, int64_t K, int64_t bn, int64_t bk, cudaStream_t st);
// Returns TO_EUNSUPPORTED (without recording an error) when the shape does not fit.
int w8a8_tc_launch(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                   void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M, int64_t N,
                   int64_t K, int64_t bn, int64_t bk, cudaStream_t st);

static int w8a8_entry(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                      void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M,
                      int64_t N, int64_t K, int64_t bn, int64_t bk, void* stream) {
  const char* op = fp8 ? "w8a8_block_fp8_matmul" : "w8a8_block_int8_matmul";
  if (M < 0 || N < 0 || K <= 0 || bn <= 0 || bk <= 0)
    return fail(TO_EINVAL, "%s: invalid M=%lld N=%lld K=%lld block=[%lld,%lld]", op,
                (long long)M, (long long)N, (long long)K, (long long)bn, (long long)bk);
  if (c_dtype != TO_F32 && c_dtype != TO_F16 && c_dtype != TO_BF16)
    return fail(TO_EUNSUPPORTED, "%s: output dtype %s", op, dtype_name(c_dtype));
  if (M == 0 || N == 0) return TO_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int rc = w8a8_tc_launch(fp8, a, b, a_s, b_s, c, c_dtype, bias, acc_out, M, N, K, bn, bk, st);
  if (rc != TO_EUNSUPPORTED) return rc;
  return w8a8_generic_launch(fp8, a, b, a_s, b_s, c, c_dtype, bias, acc_out, M, N, K, bn, bk, st);
}

}  // namespace tob

extern "C" {

int to_w8a8_i8_gemm(const int8_t* a, const int8_t* b, const float* a_s, const float* b_s, void* c,
                    int c_dtype, const void* bias, int32_t* acc_out, int64_t M, int64_t N,
                    int64_t K, int64_t block_n, int64_t block_k, void* stream) {
  return tob::w8a8_entry(false, a, b, a_s, b_s, c, c_dtype, bias, acc_out, M, N, K, block_n,
                         block_k, stream);
}

int to_w8a8_fp8_gemm(const void* a, const void* b, const float* a_s, const float* b_s, void* c,
                     int c_dtype, const void* bias, int64_t M, int64_t N, int64_t K,
                     int64_t block_n, int64_t block_k, void* stream) {
  return tob::w8a8_entry(true, a, b, a_s, b_s, c, c_dtype, bias, nullptr, M, N, K, block_n,
                         block_k, stream);
}

}  // extern "C"
