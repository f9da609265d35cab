// int8_gemm.cu — C-ABI entry points of the tcgen05 kind::i8 GEMM with fused dequant.
//
// Restates kernels/int8_gemm/int8_gemm.py:33-90 (int8_gemm_dequant_kernel):
//   acc[m,n] = sum_k A[m,k] * B[k,n]          int32, exact
//   C[m,n]   = fp16(fp32(acc) * sa[m] * sb[n])  evaluated left to right (:84), RN conversion
// on sm_100a: the int32 accumulator lives in tensor memory and is dequantised straight from
// TMEM in the epilogue, so it never touches HBM.
#include <cstring>

#include "gemm_pair_sm100.cuh"
#include "gemm_split.h"
#include "lk_abi.h"

namespace lk {
namespace {

#ifndef LK_GEMM_TMA_STORE
#define LK_GEMM_TMA_STORE 1
#endif

using gemm::Epi;
using gemm::Kind;

int make_int8_maps(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, bool b_mn, int M, int N, int K,
                   int BN, CUtensorMap* ta, CUtensorMap* tb) {
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)lda};
    const uint32_t box[2] = {128, 128};
    if (int st = make_tmap(ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  if (b_mn) {
    // B row-major [K, N]: innermost N.  Box = 128 N-bytes x 128 k-rows.
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)ldb};
    const uint32_t box[2] = {128, 128};
    return make_tmap(tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    // B row-major [N, K]: innermost K.  Box = 128 K-bytes x BN rows.
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)ldb};
    const uint32_t box[2] = {128, (uint32_t)BN};
    return make_tmap(tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  }
}

// num_dst > 0 (DequantF16 only): no C; each output element goes to dsts[0 .. num_dst), device
// pointers already offset to this GEMM's column block, all with row pitch ldc.
template <Epi kEpi>
int run_int8(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout, const float* sa,
             const float* sb, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, cudaStream_t stream,
             void* const* dsts = nullptr, int num_dst = 0) {
  if (M < 0 || N < 0 || K < 0) return LK_ERR_INVALID_ARG;
  if (b_layout != 0 && b_layout != 1) return LK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return LK_OK;
  if (!A || !B || !C) return LK_ERR_INVALID_ARG;
  if (kEpi == Epi::DequantF16 && (!sa || !sb)) return LK_ERR_INVALID_ARG;
  if (K == 0) return LK_ERR_INVALID_ARG;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return LK_ERR_INVALID_ARG;
  const bool b_mn = (b_layout == 0);
  if (lda < K || ldc < N) return LK_ERR_INVALID_ARG;
  if (b_mn ? (ldb < N) : (ldb < K)) return LK_ERR_INVALID_ARG;
  if (lda % 16 || ldb % 16) return LK_ERR_ALIGNMENT;
  if (num_dst > 0 && (ldc % 8 || kEpi != Epi::DequantF16 || !aligned16(sb))) return LK_ERR_ALIGNMENT;
  for (int d = 0; d < num_dst; ++d)
    if (!aligned16(dsts[d])) return LK_ERR_ALIGNMENT;
  if (int st = bind_stream(stream)) return st;
  auto set_scatter = [&](gemm::Params& p) {
    p.num_dst = num_dst;
    for (int d = 0; d < num_dst; ++d) p.c_dst[d] = dsts[d];
  };

  const int num_sms = sm_count();
#ifndef LK_GEMM_PAIR
#define LK_GEMM_PAIR 1
#endif
  {
    // CTA pairs with 256 x 256 tiles when there are enough of them to occupy every pair.
    const int ptm = (int)((M + 255) / 256), ptn = (int)((N + 255) / 256);
    if (LK_GEMM_PAIR && (int64_t)ptm * ptn >= num_sms / 2) {
      CUtensorMap ta, tb;
      if (int st = make_int8_maps(A, lda, B, ldb, b_mn, (int)M, (int)N, (int)K, 128, &ta, &tb)) return st;
      gemm::Params p{};
      p.M = (int)M;
      p.N = (int)N;
      p.K = (int)K;
      p.tiles_m = ptm;
      p.tiles_n = ptn;
      p.num_tiles = ptm * ptn;
      p.C = C;
      p.ldc = ldc;
      p.sa = sa;
      p.sb = sb;
      p.rstd = nullptr;
#ifndef LK_GEMM_PAIR_GROUP_M
#define LK_GEMM_PAIR_GROUP_M 16
#endif
      p.group_m = LK_GEMM_PAIR_GROUP_M;
      apply_split(p, num_sms / 2, (int)((K + 127) / 128), 4, stream);
      // C through TMA stores of 32-row x 64-byte tiles when its base and row pitch allow it.
      CUtensorMap tc;
      memset(&tc, 0, sizeof(tc));
      {
        constexpr bool kI32 = (kEpi == Epi::RawI32);
        const int64_t elem = kI32 ? 4 : 2;
        const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
        const uint64_t strides[1] = {(uint64_t)(ldc * elem)};
        const uint32_t box[2] = {kI32 ? 16u : 32u, 32u};
        p.c_tma = (LK_GEMM_TMA_STORE && aligned16(C) && (ldc * elem) % 16 == 0 &&
                   make_tmap(&tc, kI32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, C, dims,
                             strides, box, CU_TENSOR_MAP_SWIZZLE_64B) == LK_OK)
                      ? 1
                      : 0;
      }
      if (num_dst > 0) {
        set_scatter(p);
        p.c_tma = 0;  // the scatter stores from registers, to every destination
      }
      const int err = b_mn ? gemm::launch_pair<Kind::I8, true, kEpi>(ta, tb, tc, p, num_sms, stream)
                           : gemm::launch_pair<Kind::I8, false, kEpi>(ta, tb, tc, p, num_sms, stream);
      return cuda_status((cudaError_t)err);
    }
  }
  const int tiles_m = (int)((M + gemm::kBM - 1) / gemm::kBM);
  // Wide tiles halve operand traffic per MMA; narrow ones only when wide ones cannot fill the GPU.
  const int tiles_n256 = (int)((N + 255) / 256);
  const bool narrow = (int64_t)tiles_m * tiles_n256 < num_sms && N > 128;
  const int BN = narrow ? 128 : 256;
  const int tiles_n = (int)((N + BN - 1) / BN);

  CUtensorMap ta, tb;
  if (int st = make_int8_maps(A, lda, B, ldb, b_mn, (int)M, (int)N, (int)K, BN, &ta, &tb)) return st;

  gemm::Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.num_tiles = tiles_m * tiles_n;
  p.C = C;
  p.ldc = ldc;
  p.sa = sa;
  p.sb = sb;
  p.rstd = nullptr;
  set_scatter(p);

  int err;
  if (BN == 256) {
    err = b_mn ? gemm::launch<Kind::I8, 256, true, kEpi>(ta, tb, p, num_sms, stream)
               : gemm::launch<Kind::I8, 256, false, kEpi>(ta, tb, p, num_sms, stream);
  } else {
    err = b_mn ? gemm::launch<Kind::I8, 128, true, kEpi>(ta, tb, p, num_sms, stream)
               : gemm::launch<Kind::I8, 128, false, kEpi>(ta, tb, p, num_sms, stream);
  }
  return cuda_status((cudaError_t)err);
}

}  // namespace
}  // namespace lk

extern "C" int lk_int8_gemm_dequant(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                                    const float* scale_a, const float* scale_b, void* C, int64_t ldc, int64_t M,
                                    int64_t N, int64_t K, void* stream) {
  return lk::run_int8<lk::gemm::Epi::DequantF16>(A, lda, B, ldb, b_layout, scale_a, scale_b, C, ldc, M, N, K,
                                                 static_cast<cudaStream_t>(stream));
}

extern "C" int lk_int8_gemm_i32(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout, int32_t* C,
                                int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream) {
  return lk::run_int8<lk::gemm::Epi::RawI32>(A, lda, B, ldb, b_layout, nullptr, nullptr, C, ldc, M, N, K,
                                             static_cast<cudaStream_t>(stream));
}

extern "C" int lk_int8_gemm_dequant_scatter(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                                            int b_layout, const float* scale_a, const float* scale_b,
                                            void* const* dsts, int num_dst, int64_t ldc, int64_t col_offset,
                                            int64_t M, int64_t N, int64_t K, void* stream) {
  if (num_dst < 1 || num_dst > lk::gemm::kMaxScatter || !dsts || col_offset < 0) return LK_ERR_INVALID_ARG;
  if (N > 0 && ldc < col_offset + N) return LK_ERR_INVALID_ARG;
  void* at[lk::gemm::kMaxScatter];
  for (int d = 0; d < num_dst; ++d) {
    if (!dsts[d]) return LK_ERR_INVALID_ARG;
    at[d] = static_cast<uint16_t*>(dsts[d]) + col_offset;
  }
  return lk::run_int8<lk::gemm::Epi::DequantF16>(A, lda, B, ldb, b_layout, scale_a, scale_b, at[0], ldc, M, N, K,
                                                 static_cast<cudaStream_t>(stream), at, num_dst);
}
