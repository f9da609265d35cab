// Exhaustive check of the division-free quantisation codes used for 16-bit-float values
// (quant_common.cuh: codes_x2, quantize.cu: quant_vec16_store, the int8 GEMM's re-quantising
// epilogue).  For every positive finite absmax of the format and every finite x with
// |x| <= absmax:
//     s = RN(absmax / 127),  r = RN(1 / s),  q0 = RN(x * r),  e = RN(x - q0 * s),
//     q = RN(q0 + e * r)                         (Markstein's FMA-corrected quotient)
// must round to the same integer as the IEEE quotient RN(x / s) (rint, ties to even), which
// is what quantize_symmetric (kernels/int8_gemm/int8_gemm.py:157-161) computes.  Rows whose
// scale is below 2^-100 (where e can underflow) or not finite take the IEEE division in the
// kernels and are skipped here.
//
// Usage: exhaustive_codes f   (fp16)   |   exhaustive_codes b   (bf16)
// Prints "<fmt> pairs=N mismatches=M skipped_scales=S"; exits non-zero on any mismatch.
// Build with -ffp-contract=off so that x * r and x / s are single IEEE operations; fmaf is the
// correctly rounded fused multiply-add.
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static float from_fp16(uint16_t h) {
  const uint32_t sign = h & 0x8000u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  float v;
  if (e == 0)
    v = ldexpf((float)m, -24);
  else if (e == 31)
    v = m ? NAN : INFINITY;
  else
    v = ldexpf((float)(m | 0x400u), (int)e - 25);
  return sign ? -v : v;
}

static float from_bf16(uint16_t h) {
  const uint32_t b = (uint32_t)h << 16;
  float f;
  memcpy(&f, &b, sizeof f);
  return f;
}

int main(int argc, char** argv) {
  const int bf = argc > 1 && argv[1][0] == 'b';
  long long pairs = 0, mismatches = 0, skipped = 0;
  for (uint32_t ha = 1; ha < 0x7F80u; ++ha) {
    const float a = bf ? from_bf16((uint16_t)ha) : from_fp16((uint16_t)ha);
    if (!(a > 0) || isinf(a)) continue;
    volatile float s = a / 127.0f;
    if (!(s >= 0x1p-100f && s < INFINITY)) {
      ++skipped;
      continue;
    }
    volatile float r = 1.0f / s;
    for (uint32_t hx = 0; hx < 0x10000u; ++hx) {
      const float x = bf ? from_bf16((uint16_t)hx) : from_fp16((uint16_t)hx);
      if (isnan(x) || isinf(x) || fabsf(x) > a) continue;
      volatile float q0 = x * r;
      const float e = fmaf(-q0, s, x);
      const float q = fmaf(e, r, q0);
      volatile float qd = x / s;
      ++pairs;
      if (rintf(q) != rintf(qd)) {
        if (mismatches < 10) printf("mismatch absmax=%a x=%a q=%a x/s=%a\n", a, x, q, qd);
        ++mismatches;
      }
    }
  }
  printf("%s pairs=%lld mismatches=%lld skipped_scales=%lld\n", bf ? "bf16" : "fp16", pairs, mismatches, skipped);
  return mismatches != 0;
}
