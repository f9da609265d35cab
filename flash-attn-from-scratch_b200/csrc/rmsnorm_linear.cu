// rmsnorm_linear.cu — placeholder until the RMSNorm+Linear GEMM lands.
#include "lk_abi.h"

extern "C" int lk_rmsnorm_linear_fold(const void*, int, const void*, void*, int, int64_t, int64_t, void*) {
  return LK_ERR_UNSUPPORTED;
}
extern "C" int lk_rmsnorm_linear(const void*, int64_t, const void*, void*, int64_t, int, int64_t, int64_t, int64_t,
                                 float, float*, void*) {
  return LK_ERR_UNSUPPORTED;
}
extern "C" int lk_fused_rmsnorm_linear(const void*, const void*, const void*, void*, float, int64_t, int64_t,
                                       int64_t, int, void*, float*, void*) {
  return LK_ERR_UNSUPPORTED;
}
