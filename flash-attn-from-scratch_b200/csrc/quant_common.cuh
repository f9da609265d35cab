// quant_common.cuh — the per-row symmetric int8 code arithmetic shared by the quantiser
// (quantize.cu) and the int8 GEMM epilogue that re-quantises its own output
// (gemm_pair_sm100.cuh, Epi::DequantQuant).
//
// Restates kernels/int8_gemm/int8_gemm.py:157-161 (quantize_symmetric) bit for bit:
//     scale = amax(|x|) / 127.0 (IEEE division);  q = clamp(rint(x / scale), -128, 127)
// with ties to even and NaN quotients mapped to code 0.
#pragma once

#include <cstdint>

#include "lk_sm100.cuh"

namespace lk {

// The IEEE division of the rare exact path, kept out of line so unrolled callers stay small.
static __device__ __noinline__ float div_rn_out_of_line(float x, float y) { return __fdiv_rn(x, y); }

// One code: clamp(rint(x / scale), -128, 127) with NaN -> 0.
__device__ __forceinline__ int8_t quant_one(float x, float scale) {
  float t = div_rn_out_of_line(x, scale);
  if (t != t) return 0;
  t = rintf(t);
  t = fminf(fmaxf(t, -128.0f), 127.0f);
  return (int8_t)(int)t;
}

// The row's divisor, with its reciprocal for the fast path.
struct RowScale {
  float scale;
  float rcp;
  bool fast;  // 2^-100 <= scale < inf: the division-free paths below apply
};

__device__ __forceinline__ RowScale make_row_scale(float amax) {
  RowScale s;
  s.scale = __fdiv_rn(amax, 127.0f);
  s.fast = (s.scale >= 0x1p-100f) && (s.scale < INFINITY);
  s.rcp = s.fast ? __frcp_rn(s.scale) : 0.f;
  return s;
}

// Exact code of a 16-bit-float value without a division: Markstein's FMA correction of the
// reciprocal product (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990):
//     q0 = RN(x * r),  e = RN(x - q0 * s) (exact, one FMA),  q = RN(q0 + e * r),  r = RN(1 / s),
// then rint(q) via the 1.5 * 2^23 shifter.  For every fp16 and every bf16 pair (x, absmax)
// with |x| <= absmax and scale = absmax / 127 >= 2^-100, rint(q) equals rint(RN(x / scale))
// -- checked exhaustively on the CPU (tests/exhaustive_codes.c, 2.1e9 pairs) -- so the codes
// are the IEEE-division codes bit for bit, with no near-tie test and no divergent fallback.
// (Below 2^-100 the residual e can underflow; such rows take the division.)

// ---- packed-pair codes of 16-bit-float values -----------------------------------------------
__device__ __forceinline__ uint32_t pack4_codes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// The codes of the 2 * kPairs fp16 / bf16 values in x2[] (packed pairs, as fp32) into the low
// bytes of b[], by the FMA-corrected quotient above, two lanes per FMA-pipe instruction.  A row
// whose scale is not in the fast range (all-zero, inf / NaN, or tiny) takes the division.
template <int kPairs>
__device__ __forceinline__ void codes_x2(const uint64_t (&x2)[kPairs], const RowScale& s, uint32_t (&b)[2 * kPairs]) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  if (s.fast) {
    const uint64_t rcp2 = f2(s.rcp, s.rcp);
    const uint64_t ns2 = f2(-s.scale, -s.scale);
    const uint64_t nz2 = f2(-0.f, -0.f);
    const uint64_t sh2 = f2(kShift, kShift);
#pragma unroll
    for (int j = 0; j < kPairs; ++j) {
      const uint64_t q0 = fma2(x2[j], rcp2, nz2);  // RN(x * r)
      const uint64_t e = fma2(q0, ns2, x2[j]);     // x - q0 * s, exact
      const uint64_t q = fma2(e, rcp2, q0);        // RN(q0 + e * r)
      float lo, hi;
      uf2(add2(q, sh2), lo, hi);
      b[2 * j] = __float_as_uint(lo);
      b[2 * j + 1] = __float_as_uint(hi);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kPairs; ++j) {
      float lo, hi;
      uf2(x2[j], lo, hi);
      b[2 * j] = (uint32_t)(uint8_t)quant_one(lo, s.scale);
      b[2 * j + 1] = (uint32_t)(uint8_t)quant_one(hi, s.scale);
    }
  }
}

}  // namespace lk
