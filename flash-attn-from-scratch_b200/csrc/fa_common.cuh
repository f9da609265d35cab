// fa_common.cuh — pieces shared by the flash-attention forward (flash_attn.cu) and backward
// (flash_attn_bwd.cu): exp2 on the MUFU pipe, packed fp32x2 arithmetic, 16-bit packing, and
// the host-side builder of the [B, H, rows, D] TMA maps.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "lk_sm100.cuh"

namespace lk {
namespace fa {

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32x2 arithmetic lives in lk_sm100.cuh.
using lk::add2;
using lk::f2;
using lk::fma2;
using lk::max3;
using lk::uf2;

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kBf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// 4-D TMA map of a [B, H, S, D] tensor (element strides st[0..3], st[3] == 1) with boxes of
// 64 columns x box_rows rows, 128-byte swizzle (flash_attn.cu).
int make_map(CUtensorMap* map, bool bf16, const void* base, int64_t B, int64_t H, int64_t S, int64_t D,
             const int64_t* st, uint32_t box_rows = 128);

}  // namespace fa
}  // namespace lk
