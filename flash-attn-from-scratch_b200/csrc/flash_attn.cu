// flash_attn.cu — placeholder until the tcgen05 attention kernel lands.
#include "lk_abi.h"

extern "C" int lk_flash_attn_fwd(const void*, const void*, const void*, void*, int, int64_t, int64_t, int64_t,
                                 int64_t, int64_t, const int64_t*, const int64_t*, const int64_t*, const int64_t*,
                                 int, float, void*) {
  return LK_ERR_UNSUPPORTED;
}
