// quantize.cu — per-row symmetric absmax int8 quantisation (HBM-bound).
//
// Restates kernels/int8_gemm/int8_gemm.py:157-161 (quantize_symmetric) bit for bit:
//     x_f32 = x.float();  scale = amax(|x_f32|, -1) / 127.0
//     q = clamp(round(x_f32 / scale), -128, 127).to(int8)
// with IEEE-rounded divisions (no reciprocal, no fast-math), ties-to-even rounding, a NaN-
// propagating max, and NaN quotients mapped to code 0 (what the reference's CPU cast yields
// for all-zero / non-finite rows).
//
// Design: one warp owns one row.  The row is read ONCE with 16-byte vector loads into
// registers (up to kMaxVecs vectors per lane), the absmax is a register/shuffle reduction on
// the raw magnitude bits (|x| bit patterns order like the values and every NaN sorts above
// +inf, so an integer max propagates NaN for free), then codes are produced from the cached
// registers and written with 4/8-byte stores.  HBM traffic = 1 read of x + 1 write of q.
// fp16 / bf16 codes come from Markstein's FMA-corrected reciprocal product (quant_common.cuh),
// which rounds exactly like the IEEE division for every value of those formats (checked
// exhaustively) -- fp16 inputs put x / scale on a coarse lattice where exact ties are common,
// so a near-tie test with a division fallback would diverge constantly.  fp32 codes use the
// reciprocal product with a near-tie test and the IEEE division for the rare near-tie.
// Rows longer than the register cache take a two-pass path whose second pass is an L2 hit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "lk_abi.h"
#include "lk_sm100.cuh"
#include "quant_common.cuh"

namespace lk {
namespace {

template <typename T>
struct VecTraits;
template <>
struct VecTraits<float> {
  static constexpr int kElems = 4;  // per 16-byte vector
};
template <>
struct VecTraits<__half> {
  static constexpr int kElems = 8;
};
template <>
struct VecTraits<__nv_bfloat16> {
  static constexpr int kElems = 8;
};

// Magnitude bits of every element of a 16-byte vector, reduced to one unsigned max.
template <typename T>
__device__ __forceinline__ uint32_t vec_absmax_bits(const uint4& v);
template <>
__device__ __forceinline__ uint32_t vec_absmax_bits<float>(const uint4& v) {
  uint32_t a = max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu);
  uint32_t b = max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu);
  return max(a, b);
}
__device__ __forceinline__ uint32_t absmax_bits_16(const uint4& v) {
  uint32_t a = __vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu);
  uint32_t b = __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu);
  uint32_t m = __vmaxu2(a, b);
  return max(m & 0xFFFFu, m >> 16);
}
template <>
__device__ __forceinline__ uint32_t vec_absmax_bits<__half>(const uint4& v) {
  return absmax_bits_16(v);
}
template <>
__device__ __forceinline__ uint32_t vec_absmax_bits<__nv_bfloat16>(const uint4& v) {
  return absmax_bits_16(v);
}

template <typename T>
__device__ __forceinline__ float bits_to_float(uint32_t b);
template <>
__device__ __forceinline__ float bits_to_float<float>(uint32_t b) {
  return __uint_as_float(b);
}
template <>
__device__ __forceinline__ float bits_to_float<__half>(uint32_t b) {
  return __half2float(__ushort_as_half((unsigned short)b));
}
template <>
__device__ __forceinline__ float bits_to_float<__nv_bfloat16>(uint32_t b) {
  return __uint_as_float(b << 16);  // bf16 -> fp32 is exact: the bf16 bits are the top half
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ uint32_t mag_bits(T v);
template <>
__device__ __forceinline__ uint32_t mag_bits<float>(float v) {
  return __float_as_uint(v) & 0x7FFFFFFFu;
}
template <>
__device__ __forceinline__ uint32_t mag_bits<__half>(__half v) {
  return (uint32_t)__half_as_ushort(v) & 0x7FFFu;
}
template <>
__device__ __forceinline__ uint32_t mag_bits<__nv_bfloat16>(__nv_bfloat16 v) {
  return (uint32_t)__bfloat16_as_ushort(v) & 0x7FFFu;
}

// Same code as quant_one, usually without the division.  t = x * rcp differs from the
// correctly rounded quotient fl(x / scale) by at most 2.3e-5 (|x / scale| <= 127.1: 2^-23
// relative for the product and reciprocal, half an ulp of 127 for fl), so when t is more
// than 2^-12 away from every half-integer both round to the same integer; only the rare
// near-tie falls back to the IEEE division.
// Rounding uses the 1.5 * 2^23 shifter: t + 1.5*2^23 rounds t to the nearest integer, ties
// to even (exactly rintf), and leaves that integer in the low mantissa bits, so the int8
// code is the low byte of the float's bits — no float->int conversion instruction needed.
// The fast path only runs where |t| <= 127.1, so the code never needs clamping there.
__device__ __forceinline__ int8_t quant_code(float x, const RowScale& s) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  if (s.fast) {
    const float t = x * s.rcp;
    const float tb = t + kShift;
    if (fabsf(t - (tb - kShift)) <= 0.5f - 2.44140625e-4f) return (int8_t)(__float_as_uint(tb) & 0xFFu);
  }
  return quant_one(x, s.scale);
}

// Codes for one 16-byte vector, written to q (kElems bytes).
template <typename T>
__device__ __forceinline__ void quant_vec_store(const uint4& v, const RowScale& s, int8_t* q);
template <>
__device__ __forceinline__ void quant_vec_store<float>(const uint4& v, const RowScale& s, int8_t* q) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  const float f[4] = {__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w)};
  uint32_t b[4];
  bool bad = !s.fast;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float t = f[e] * s.rcp;
    const float tb = t + kShift;
    bad |= !(fabsf(t - (tb - kShift)) <= 0.5f - 2.44140625e-4f);
    b[e] = __float_as_uint(tb);
  }
  if (bad) {
#pragma unroll
    for (int e = 0; e < 4; ++e) b[e] = (uint32_t)(uint8_t)quant_one(f[e], s.scale);
  }  *reinterpret_cast<uint32_t*>(q) =
      __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
}
template <typename T16>
__device__ __forceinline__ float lo16(uint32_t w);
template <>
__device__ __forceinline__ float lo16<__half>(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
}
template <>
__device__ __forceinline__ float lo16<__nv_bfloat16>(uint32_t w) {
  return __uint_as_float(w << 16);
}
template <typename T16>
__device__ __forceinline__ float hi16(uint32_t w);
template <>
__device__ __forceinline__ float hi16<__half>(uint32_t w) {
  return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
template <>
__device__ __forceinline__ float hi16<__nv_bfloat16>(uint32_t w) {
  return __uint_as_float(w & 0xFFFF0000u);
}
// fp16 / bf16 vectors: the FMA-corrected quotient of quant_common.cuh (exact for these types,
// checked exhaustively), so no near-tie test and no per-vector fallback.
template <typename T16>
__device__ __forceinline__ void quant_vec16_store(const uint4& v, const RowScale& s, int8_t* q) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint64_t x2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x2[j] = f2(lo16<T16>(w[j]), hi16<T16>(w[j]));
  uint32_t b[8];
  codes_x2<4>(x2, s, b);
  *reinterpret_cast<uint2*>(q) = make_uint2(pack4_codes(b[0], b[1], b[2], b[3]), pack4_codes(b[4], b[5], b[6], b[7]));
}
template <>
__device__ __forceinline__ void quant_vec_store<__half>(const uint4& v, const RowScale& s, int8_t* q) {
  quant_vec16_store<__half>(v, s, q);
}
template <>
__device__ __forceinline__ void quant_vec_store<__nv_bfloat16>(const uint4& v, const RowScale& s, int8_t* q) {
  quant_vec16_store<__nv_bfloat16>(v, s, q);
}

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

constexpr int kWarpsPerCta = 8;

// Vector path, row cached in registers: requires 16-byte aligned rows and
// cols <= 32 * kVecs * kElems.  kVecs is the per-lane register cache size.
template <typename T, int kVecs>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    quantize_rows_cached(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t x_ld,
                         int8_t* __restrict__ q, int64_t q_ld, float* __restrict__ scale_out) {
  constexpr int E = VecTraits<T>::kElems;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * x_ld;
  const int64_t nvec = cols / E;  // cols % E == 0 on this path
  const uint4* xv = reinterpret_cast<const uint4*>(xr);

  uint4 cache[kVecs];
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < kVecs; ++i) {
    const int64_t vi = (int64_t)i * 32 + lane;
    if (vi < nvec) {
      cache[i] = ld_stream(xv + vi);
      m = max(m, vec_absmax_bits<T>(cache[i]));
    }
  }
  m = warp_max_u32(m);
  const RowScale s = make_row_scale(bits_to_float<T>(m));
  if (lane == 0) scale_out[row] = s.scale;
  int8_t* qr = q + row * q_ld;
#pragma unroll
  for (int i = 0; i < kVecs; ++i) {
    const int64_t vi = (int64_t)i * 32 + lane;
    if (vi < nvec) quant_vec_store<T>(cache[i], s, qr + vi * E);
  }
}

// Vector path for wide rows: one CTA of kRowThreads threads per row, each caching up to
// kVecs 16-byte vectors; the absmax is reduced across warps through shared memory.  Many
// rows stay in flight per SM, which is what an HBM-bound pass needs.
template <typename T, int kRowThreads, int kVecs>
__global__ void __launch_bounds__(kRowThreads)
    quantize_rows_cta(const T* __restrict__ x, int64_t cols, int64_t x_ld, int8_t* __restrict__ q, int64_t q_ld,
                      float* __restrict__ scale_out) {
  constexpr int E = VecTraits<T>::kElems;
  constexpr int kWarps = kRowThreads / 32;
  __shared__ uint32_t warp_max[kWarps];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x + row * x_ld);
  const int64_t nvec = cols / E;
  uint4 cache[kVecs];
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < kVecs; ++i) {
    const int64_t vi = (int64_t)i * kRowThreads + tid;
    if (vi < nvec) {
      cache[i] = ld_stream(xv + vi);
      m = max(m, vec_absmax_bits<T>(cache[i]));
    }
  }
  m = warp_max_u32(m);
  if ((tid & 31) == 0) warp_max[tid >> 5] = m;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kWarps; ++w) m = max(m, warp_max[w]);
  const RowScale s = make_row_scale(bits_to_float<T>(m));
  if (tid == 0) scale_out[row] = s.scale;
  int8_t* qr = q + row * q_ld;
#pragma unroll
  for (int i = 0; i < kVecs; ++i) {
    const int64_t vi = (int64_t)i * kRowThreads + tid;
    if (vi < nvec) quant_vec_store<T>(cache[i], s, qr + vi * E);
  }
}

// Generic path: any alignment / width.  Two passes over the row (the second is an L2 hit).
template <typename T>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    quantize_rows_generic(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t x_ld,
                          int8_t* __restrict__ q, int64_t q_ld, float* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * x_ld;
  uint32_t m = 0;
  for (int64_t c = lane; c < cols; c += 32) m = max(m, mag_bits<T>(xr[c]));
  m = warp_max_u32(m);
  const RowScale s = make_row_scale(bits_to_float<T>(m));
  if (lane == 0) scale_out[row] = s.scale;
  int8_t* qr = q + row * q_ld;
  for (int64_t c = lane; c < cols; c += 32) qr[c] = quant_code(to_f32<T>(xr[c]), s);
}

template <typename T>
int launch_quantize(const void* x, int64_t rows, int64_t cols, int64_t x_ld, int8_t* q, int64_t q_ld, float* scale,
                    cudaStream_t stream) {
  constexpr int E = VecTraits<T>::kElems;
  const dim3 grid((unsigned)((rows + kWarpsPerCta - 1) / kWarpsPerCta));
  const dim3 block(kWarpsPerCta * 32);
  const T* xt = static_cast<const T*>(x);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((x_ld * (int64_t)sizeof(T)) % 16 == 0) &&
                       (cols % E == 0) && ((reinterpret_cast<uintptr_t>(q) & 7) == 0) && (q_ld % 8 == 0);
  const int64_t nvec = cols / E;
  const bool cta_rows = rows <= 0x7FFFFFFF;
  if (aligned && nvec <= 32 * 4) {
    quantize_rows_cached<T, 4><<<grid, block, 0, stream>>>(xt, rows, cols, x_ld, q, q_ld, scale);
  } else if (aligned && cta_rows && nvec <= 128 * 4) {
    quantize_rows_cta<T, 128, 4><<<(unsigned)rows, 128, 0, stream>>>(xt, cols, x_ld, q, q_ld, scale);
  } else if (aligned && cta_rows && nvec <= 256 * 4) {
    quantize_rows_cta<T, 256, 4><<<(unsigned)rows, 256, 0, stream>>>(xt, cols, x_ld, q, q_ld, scale);
  } else if (aligned && cta_rows && nvec <= 512 * 4) {
    quantize_rows_cta<T, 512, 4><<<(unsigned)rows, 512, 0, stream>>>(xt, cols, x_ld, q, q_ld, scale);
  } else if (aligned && cta_rows && nvec <= 512 * 8) {
    quantize_rows_cta<T, 512, 8><<<(unsigned)rows, 512, 0, stream>>>(xt, cols, x_ld, q, q_ld, scale);
  } else {
    quantize_rows_generic<T><<<grid, block, 0, stream>>>(xt, rows, cols, x_ld, q, q_ld, scale);
  }
  return check_launch();
}

}  // namespace
}  // namespace lk

extern "C" int lk_quantize_symmetric(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t x_ld, int8_t* q,
                                     int64_t q_ld, float* scale, void* stream) {
  using namespace lk;
  if (rows < 0 || cols < 0) return LK_ERR_INVALID_ARG;
  if (rows == 0) return LK_OK;
  if (!x || !q || !scale) return LK_ERR_INVALID_ARG;
  if (x_ld < cols || q_ld < cols) return LK_ERR_INVALID_ARG;
  if (rows > (int64_t)0x7FFFFFFF * kWarpsPerCta) return LK_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = bind_stream(s)) return st;
  switch (x_dtype) {
    case LK_F32:
      return launch_quantize<float>(x, rows, cols, x_ld, q, q_ld, scale, s);
    case LK_F16:
      return launch_quantize<__half>(x, rows, cols, x_ld, q, q_ld, scale, s);
    case LK_BF16:
      return launch_quantize<__nv_bfloat16>(x, rows, cols, x_ld, q, q_ld, scale, s);
    default:
      return LK_ERR_UNSUPPORTED;
  }
}
