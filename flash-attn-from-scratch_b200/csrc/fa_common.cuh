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

// 2^x0 and 2^x1 on the FMA pipe instead of the MUFU pipe, for a share of the softmax
// exponentials (the MUFU unit does 16 ex2 per clock per SM, as many as the tensor pipe needs
// per clock at D = 128, so moving some of them elsewhere shortens the exp phase).
// Cody-Waite argument reduction (W. J. Cody, W. Waite, Software Manual for the Elementary
// Functions, 1980): x = j + f with j = rint(x) by the 1.5 * 2^23 shifter and |f| <= 1/2 exact;
// 2^f by a cubic whose coefficients were fitted here by Remez exchange for minimax relative
// error on [-1/2, 1/2] (7.5e-5, under half an ulp of bf16's 8-bit significand); 2^j is added
// into the exponent field.  Inputs below -125 (masked keys: -inf) give about 2^-125, not 0,
// which no bf16 / fp16 P or row sum can tell apart from 0 next to the row maximum's 2^0.
__device__ __forceinline__ void exp2_poly_pair(float x0, float x1, float& p0, float& p1) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  const uint64_t xc = lk::f2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = lk::add2(xc, lk::f2(kShift, kShift));   // low bits of t: rint(x)
  const uint64_t j = lk::add2(t, lk::f2(-kShift, -kShift));  // rint(x) as a float, exact
  const uint64_t f = lk::fma2(j, lk::f2(-1.f, -1.f), xc);     // x - rint(x), exact
  uint64_t p = lk::fma2(lk::f2(0x1.c3f760p-5f, 0x1.c3f760p-5f), f, lk::f2(0x1.f0de1ap-3f, 0x1.f0de1ap-3f));
  p = lk::fma2(p, f, lk::f2(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  p = lk::fma2(p, f, lk::f2(0x1.fff692p-1f, 0x1.fff692p-1f));
  float pa, pb, ta, tb;
  lk::uf2(p, pa, pb);
  lk::uf2(t, ta, tb);
  // (bits(t) << 23) == rint(x) << 23 modulo 2^32: the shifter's own bits shift out.
  p0 = __uint_as_float(__float_as_uint(pa) + (__float_as_uint(ta) << 23));
  p1 = __uint_as_float(__float_as_uint(pb) + (__float_as_uint(tb) << 23));
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
