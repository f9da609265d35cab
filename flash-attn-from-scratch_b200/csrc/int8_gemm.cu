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
             void* const* dsts = nullptr, int num_dst = 0, int multimem = 0) {
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
  // Multicast stores are whole 16-byte vectors of whole 32-column chunks.
  if (multimem && (num_dst != 1 || N % 32)) return LK_ERR_ALIGNMENT;
  if (int st = bind_stream(stream)) return st;
  auto set_scatter = [&](gemm::Params& p) {
    p.num_dst = num_dst;
    p.dst_multimem = multimem;
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

// Requant workspace layout: [M] row maxima, [ceil(M/32)] slice counters, then (256-byte
// aligned) the epilogue warps' parking rings, 128 KB per CTA of the largest grid.
int64_t requant_park_offset(int64_t M) { return ((M + (M + 31) / 32) * 4 + 255) / 256 * 256; }
int64_t requant_workspace_bytes(int64_t M, int num_sms) {
  return requant_park_offset(M) + (int64_t)num_sms * 4 * 2 * 1024 * 16;
}

// The int8 GEMM + dequant whose epilogue also quantises its own fp16 output per row
// (Epi::DequantQuant on CTA pairs): codes q [M, N] int8 (row pitch ldq) and scales [M], equal
// bit for bit to quantize_symmetric(C).  C (fp16) is written too when it is not null.
int run_int8_requant(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout, const float* sa,
                     const float* sb, void* C, int64_t ldc, int8_t* q, int64_t ldq, float* q_scale, uint32_t* ws,
                     int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (M < 0 || N < 0 || K < 0) return LK_ERR_INVALID_ARG;
  if (b_layout != 0 && b_layout != 1) return LK_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return LK_OK;
  if (!A || !B || !sa || !sb || !q || !q_scale || !ws || K == 0) return LK_ERR_INVALID_ARG;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return LK_ERR_INVALID_ARG;
  const bool b_mn = (b_layout == 0);
  if (lda < K || ldq < N || (C && ldc < N)) return LK_ERR_INVALID_ARG;
  if (b_mn ? (ldb < N) : (ldb < K)) return LK_ERR_INVALID_ARG;
  if (lda % 16 || ldb % 16 || ldq % 16 || !aligned16(q)) return LK_ERR_ALIGNMENT;
  if (int st = bind_stream(stream)) return st;
  const int num_sms = sm_count();
  const int ptm = (int)((M + 255) / 256), ptn = (int)((N + 255) / 256);
  // Every tile of a row block must sit on its own pair, and every pair of the grid must be
  // resident at once: a tile's epilogue waits for the other tiles of its row block.
  if (ptn > num_sms / 2) return LK_ERR_UNSUPPORTED;
  int npairs = 0;
  {
    const cudaError_t e = b_mn ? gemm::resident_pairs<Kind::I8, true, Epi::DequantQuant>(num_sms, &npairs)
                               : gemm::resident_pairs<Kind::I8, false, Epi::DequantQuant>(num_sms, &npairs);
    if (e != cudaSuccess) return cuda_status(e);
  }
  if (ptn > npairs) return LK_ERR_UNSUPPORTED;
  CUtensorMap ta, tb, tq;
  if (int st = make_int8_maps(A, lda, B, ldb, b_mn, (int)M, (int)N, (int)K, 128, &ta, &tb)) return st;
  {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)ldq};
    const uint32_t box[2] = {64u, 32u};
    if (int st = make_tmap(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B))
      return st;
  }
  const int64_t slices = (M + 31) / 32;
  if (int st = cuda_status(cudaMemsetAsync(ws, 0, (size_t)(M + slices) * sizeof(uint32_t), stream))) return st;
  // The parking ring follows the counters, 256-byte aligned: 4 warps x 2 slots x 16 KB per CTA.
  uint4* park = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(ws) + requant_park_offset(M));
  gemm::Params p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.tiles_m = ptm;
  p.tiles_n = ptn;
  p.num_tiles = ptm * ptn;
  p.full_tiles = p.num_tiles;
  p.split = 1;
  p.num_units = p.num_tiles;
#ifndef LK_REQUANT_GROUP_M
#define LK_REQUANT_GROUP_M 1
#endif
  // Raster groups of g row blocks (N-fastest when g = 1).  A tile's codes are written one
  // tile after its own pass, once its row block has published; with every row block spread
  // over fewer than 2 * pairs consecutive tiles those waits only ever point at earlier work.
  int g = LK_REQUANT_GROUP_M;
  while (g > 1 && (int64_t)g * ptn > 2 * (int64_t)npairs) --g;
  p.group_m = g;
  p.C = C;
  p.ldc = ldc;
  p.sa = sa;
  p.sb = sb;
  p.c_tma = 1;  // the codes' map
  p.q_absmax = ws;
  p.q_slice_ctr = reinterpret_cast<int*>(ws + M);
  p.q_scale = q_scale;
  p.q_park = park;
  const int err = b_mn ? gemm::launch_pair<Kind::I8, true, Epi::DequantQuant>(ta, tb, tq, p, num_sms, stream, npairs)
                       : gemm::launch_pair<Kind::I8, false, Epi::DequantQuant>(ta, tb, tq, p, num_sms, stream, npairs);
  return cuda_status((cudaError_t)err);
}

}  // namespace
}  // namespace lk

extern "C" int64_t lk_int8_gemm_requant_workspace_bytes(int64_t M) {
  return M <= 0 ? 0 : lk::requant_workspace_bytes(M, lk::sm_count());
}

extern "C" int lk_int8_gemm_dequant_requant(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int b_layout,
                                            const float* scale_a, const float* scale_b, void* C, int64_t ldc,
                                            int8_t* q, int64_t ldq, float* q_scale, void* workspace, int64_t M,
                                            int64_t N, int64_t K, void* stream) {
  return lk::run_int8_requant(A, lda, B, ldb, b_layout, scale_a, scale_b, C, ldc, q, ldq, q_scale,
                              static_cast<uint32_t*>(workspace), M, N, K, static_cast<cudaStream_t>(stream));
}

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

extern "C" int lk_int8_gemm_dequant_multicast(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                                              int b_layout, const float* scale_a, const float* scale_b,
                                              void* multicast_dst, int64_t ldc, int64_t col_offset, int64_t M,
                                              int64_t N, int64_t K, void* stream) {
  if (!multicast_dst || col_offset < 0 || col_offset % 8) return LK_ERR_INVALID_ARG;
  if (N > 0 && ldc < col_offset + N) return LK_ERR_INVALID_ARG;
  void* at[1] = {static_cast<uint16_t*>(multicast_dst) + col_offset};
  return lk::run_int8<lk::gemm::Epi::DequantF16>(A, lda, B, ldb, b_layout, scale_a, scale_b, at[0], ldc, M, N, K,
                                                 static_cast<cudaStream_t>(stream), at, 1, 1);
}
