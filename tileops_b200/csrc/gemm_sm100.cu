// tcgen05 tensor-core GEMMs for sm_100a (placeholder dispatcher: every shape goes to the
// generic kernel until the tcgen05 tiles are enabled).
#include "common.cuh"

namespace tob {

int w8a8_tc_launch(bool fp8, const void* a, const void* b, const float* a_s, const float* b_s,
                   void* c, int c_dtype, const void* bias, int32_t* acc_out, int64_t M, int64_t N,
                   int64_t K, int64_t bn, int64_t bk, cudaStream_t st) {
  (void)fp8; (void)a; (void)b; (void)a_s; (void)b_s; (void)c; (void)c_dtype; (void)bias;
  (void)acc_out; (void)M; (void)N; (void)K; (void)bn; (void)bk; (void)st;
  return TO_EUNSUPPORTED;
}

}  // namespace tob
