// rmsnorm_linear.cu — fused RMSNorm + Linear on sm_100a.
//
// Restates the reference's fused op (csrc/fused_rmsnorm_linear.cu:37-99 and the fallback
// kernels/fused_rmsnorm_linear/fused_ops.py:27-37):
//     y[r, :] = (x[r, :] * rsqrt(mean_k x[r,k]^2 + eps) * w_norm) @ w_lin^T
// as   y[r, n] = rstd[r] * sum_k x[r,k] * w_fold[n,k],   w_fold = w_lin * w_norm  (folded once)
//
// Three kernels:
//   fold_kernel      w_fold = dtype(w_lin * w_norm), elementwise, once per weight version.
//   row_rstd_kernel  rstd[r] = rsqrt(sum_k x^2 / d_in + eps): one warp per row, 16-byte loads,
//                    warp-shuffle reduction (the reference's per-row reduction,
//                    csrc/fused_rmsnorm_linear.cu:55-81); HBM-bound, reads x once.
//   gemm_kernel<RowRsqrt>  tcgen05 GEMM x @ w_fold^T whose epilogue scales row r by rstd[r].
//                    Launched as a programmatic dependent of row_rstd_kernel: its TMA/MMA
//                    warps start the main loop while the row kernel is still running; only
//                    the epilogue waits (griddepcontrol.wait) before reading rstd.
// The normalised activation is never written to HBM.
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstring>
#include <mutex>

#include "gemm_pair_sm100.cuh"
#include "gemm_split.h"
#include "lk_abi.h"

namespace lk {
namespace {

using gemm::Epi;
using gemm::Kind;

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]);
template <>
__device__ __forceinline__ void unpack8<__half>(const uint4& w, float (&f)[8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __half2float(__ushort_as_half((unsigned short)(ws[j] & 0xFFFFu)));
    f[2 * j + 1] = __half2float(__ushort_as_half((unsigned short)(ws[j] >> 16)));
  }
}
template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4& w, float (&f)[8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = __uint_as_float(ws[j] << 16);
    f[2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  return gemm::pack_half2(a, b);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  return gemm::pack_bf162(a, b);
}

template <typename TN>
__device__ __forceinline__ float load_norm(const void* w, int64_t k);
template <>
__device__ __forceinline__ float load_norm<float>(const void* w, int64_t k) {
  return __ldg(static_cast<const float*>(w) + k);
}
template <>
__device__ __forceinline__ float load_norm<__half>(const void* w, int64_t k) {
  return __half2float(static_cast<const __half*>(w)[k]);
}
template <>
__device__ __forceinline__ float load_norm<__nv_bfloat16>(const void* w, int64_t k) {
  return __bfloat162float(static_cast<const __nv_bfloat16*>(w)[k]);
}

// w_fold[n, k] = T(float(w_lin[n, k]) * float(w_norm[k])), 8 elements per thread.
template <typename T, typename TN>
__global__ void __launch_bounds__(256) fold_kernel(const void* __restrict__ w_norm, const T* __restrict__ w_lin,
                                                   T* __restrict__ w_fold, int64_t d_in, int64_t total_vec) {
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total_vec; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = v * 8;
    const int64_t k0 = e0 % d_in;  // d_in % 8 == 0: a vector never straddles rows
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(w_lin) + v);
    float f[8];
    unpack8<T>(w, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = f[j] * load_norm<TN>(w_norm, k0 + j);
    reinterpret_cast<uint4*>(w_fold)[v] =
        make_uint4(pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
  }
}

constexpr int kRowWarps = 8;

// rstd[r] = rsqrt(mean_k x[r,k]^2 + eps).  One warp per row; d_in % 8 == 0, rows 16B aligned.
template <typename T>
__global__ void __launch_bounds__(kRowWarps * 32)
    row_rstd_kernel(const T* __restrict__ x, int64_t x_ld, int rows, int d_in, float eps, float* __restrict__ rstd) {
  // The GEMM that consumes rstd may begin launching right away; it waits for our completion
  // only in its epilogue.
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xv = reinterpret_cast<const uint4*>(x + (int64_t)row * x_ld);
  const int nvec = d_in >> 3;
  float ss0 = 0.f, ss1 = 0.f;
  int v = lane;
  // Two independent accumulators; 16 loads in flight per lane, so a row of up to 4096 16-bit
  // values costs one memory round trip (the kernel is latency-bound: few rows, short rows).
  for (; v + 480 < nvec; v += 512) {
    uint4 w[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) w[u] = __ldg(xv + v + 32 * u);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      float f[8];
      unpack8<T>(w[u], f);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        ss0 = fmaf(f[j], f[j], ss0);
        ss1 = fmaf(f[j + 1], f[j + 1], ss1);
      }
    }
  }
  for (; v + 96 < nvec; v += 128) {
    uint4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = __ldg(xv + v + 32 * u);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float f[8];
      unpack8<T>(w[u], f);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        ss0 = fmaf(f[j], f[j], ss0);
        ss1 = fmaf(f[j + 1], f[j + 1], ss1);
      }
    }
  }
  for (; v < nvec; v += 32) {
    float f[8];
    unpack8<T>(__ldg(xv + v), f);
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      ss0 = fmaf(f[j], f[j], ss0);
      ss1 = fmaf(f[j + 1], f[j + 1], ss1);
    }
  }
  float ss = ss0 + ss1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) rstd[row] = rsqrtf(ss / (float)d_in + eps);
}

template <typename T>
int run_fold(const void* w_norm, int w_norm_dtype, const void* w_lin, void* w_fold, int64_t d_in, int64_t d_out,
             cudaStream_t s) {
  const int64_t total_vec = d_in * d_out / 8;
  const int64_t want = (total_vec + 255) / 256;
  const int grid = (int)(want < 4 * 148 * 8 ? want : 4 * 148 * 8);
  const T* wl = static_cast<const T*>(w_lin);
  T* wf = static_cast<T*>(w_fold);
  switch (w_norm_dtype) {
    case LK_F32:
      fold_kernel<T, float><<<grid, 256, 0, s>>>(w_norm, wl, wf, d_in, total_vec);
      break;
    case LK_F16:
      fold_kernel<T, __half><<<grid, 256, 0, s>>>(w_norm, wl, wf, d_in, total_vec);
      break;
    case LK_BF16:
      fold_kernel<T, __nv_bfloat16><<<grid, 256, 0, s>>>(w_norm, wl, wf, d_in, total_vec);
      break;
    default:
      return LK_ERR_UNSUPPORTED;
  }
  return check_launch();
}

// may_allocate = false: nothing is allocated (the CTA-pair kernel's split workspace is not
// used), for the no-allocation entry point.
template <Kind kKind>
int run_gemm(const void* x, int64_t x_ld, const void* w_fold, void* y, int64_t y_ld, int64_t rows, int64_t d_in,
             int64_t d_out, float eps, float* rstd, cudaStream_t s, bool may_allocate) {
  using T = typename std::conditional<kKind == Kind::F16, __half, __nv_bfloat16>::type;
  const CUtensorMapDataType tdt = kKind == Kind::F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int num_sms = sm_count();
  const int tiles_m = (int)((rows + gemm::kBM - 1) / gemm::kBM);
  const bool narrow = (int64_t)tiles_m * ((d_out + 255) / 256) < num_sms && d_out > 128;
  const int BN = narrow ? 128 : 256;
  const int tiles_n = (int)((d_out + BN - 1) / BN);

  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)d_in, (uint64_t)rows};
    const uint64_t strides[1] = {(uint64_t)x_ld * 2};
    const uint32_t box[2] = {64, 128};
    if (int st = make_tmap(&ta, tdt, 2, x, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }
  {
    const uint64_t dims[2] = {(uint64_t)d_in, (uint64_t)d_out};
    const uint64_t strides[1] = {(uint64_t)d_in * 2};
    const uint32_t box[2] = {64, (uint32_t)BN};
    if (int st = make_tmap(&tb, tdt, 2, w_fold, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
  }

  // 1) per-row rstd (HBM-bound row kernel)
  row_rstd_kernel<T><<<(unsigned)((rows + kRowWarps - 1) / kRowWarps), kRowWarps * 32, 0, s>>>(
      static_cast<const T*>(x), x_ld, (int)rows, (int)d_in, eps, rstd);
  if (int st = check_launch()) return st;

  // 2) the GEMM, a programmatic dependent of (1).  With enough 256 x 256 tiles to occupy
  //    every SM pair: the CTA-pair kernel (each CTA loads half of every W tile, C leaves
  //    through TMA store tiles); otherwise the one-CTA kernel.
#ifndef LK_RMS_PAIR
#define LK_RMS_PAIR 1
#endif
  {
    // (Fewer tiles than pairs, split along K, measured slower: such problems are bound by the
    // TMA round trip, not by tensor or L2 throughput.)  Leftover tiles of the last round are
    // split in at most 2 parts, so float partial sums do not depend on arrival order.
    const int ptm = (int)((rows + 255) / 256), ptn = (int)((d_out + 255) / 256);
    const int num_kb = (int)((d_in + 63) / 64);
    if (LK_RMS_PAIR && (int64_t)ptm * ptn >= num_sms / 2) {
      CUtensorMap tbp, tc;
      {
        const uint64_t dims[2] = {(uint64_t)d_in, (uint64_t)d_out};
        const uint64_t strides[1] = {(uint64_t)d_in * 2};
        const uint32_t box[2] = {64, 128};
        if (int st = make_tmap(&tbp, tdt, 2, w_fold, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return st;
      }
      gemm::Params p{};
      p.M = (int)rows;
      p.N = (int)d_out;
      p.K = (int)d_in;
      p.tiles_m = ptm;
      p.tiles_n = ptn;
      p.num_tiles = ptm * ptn;
      p.C = y;
      p.ldc = y_ld;
      p.rstd = rstd;
#ifndef LK_GEMM_PAIR_GROUP_M
#define LK_GEMM_PAIR_GROUP_M 16
#endif
      p.group_m = LK_GEMM_PAIR_GROUP_M;
      gemm::apply_split(p, num_sms / 2, num_kb, may_allocate ? 2 : 1, s);
      memset(&tc, 0, sizeof(tc));
      {
        const uint64_t dims[2] = {(uint64_t)d_out, (uint64_t)rows};
        const uint64_t strides[1] = {(uint64_t)y_ld * 2};
        const uint32_t box[2] = {32, 32};
        p.c_tma = (aligned16(y) && (y_ld * 2) % 16 == 0 &&
                   make_tmap(&tc, tdt, 2, y, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B) == LK_OK)
                      ? 1
                      : 0;
      }
      return cuda_status((cudaError_t)gemm::launch_pair<kKind, false, Epi::RowRsqrt>(ta, tbp, tc, p, num_sms, s));
    }
  }
  gemm::Params p{};
  p.M = (int)rows;
  p.N = (int)d_out;
  p.K = (int)d_in;
  p.tiles_m = tiles_m;
  p.tiles_n = tiles_n;
  p.num_tiles = tiles_m * tiles_n;
  p.C = y;
  p.ldc = y_ld;
  p.rstd = rstd;
  const int err = (BN == 256) ? gemm::launch<kKind, 256, false, Epi::RowRsqrt>(ta, tb, p, num_sms, s)
                              : gemm::launch<kKind, 128, false, Epi::RowRsqrt>(ta, tb, p, num_sms, s);
  return cuda_status((cudaError_t)err);
}

bool is16(int dt) { return dt == LK_F16 || dt == LK_BF16; }

}  // namespace
}  // namespace lk

extern "C" int lk_rmsnorm_linear_fold(const void* w_norm, int w_norm_dtype, const void* w_lin, void* w_fold,
                                      int dtype, int64_t d_in, int64_t d_out, void* stream) {
  using namespace lk;
  if (d_in < 0 || d_out < 0) return LK_ERR_INVALID_ARG;
  if (d_in == 0 || d_out == 0) return LK_OK;
  if (!w_norm || !w_lin || !w_fold) return LK_ERR_INVALID_ARG;
  if (!is16(dtype)) return LK_ERR_UNSUPPORTED;
  if (d_in % 8) return LK_ERR_INVALID_ARG;
  if (!aligned16(w_lin) || !aligned16(w_fold)) return LK_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = bind_stream(s)) return st;
  return dtype == LK_F16 ? run_fold<__half>(w_norm, w_norm_dtype, w_lin, w_fold, d_in, d_out, s)
                         : run_fold<__nv_bfloat16>(w_norm, w_norm_dtype, w_lin, w_fold, d_in, d_out, s);
}

namespace lk {
namespace {
int rmsnorm_linear(const void* x, int64_t x_ld, const void* w_fold, void* y, int64_t y_ld, int dtype, int64_t rows,
                   int64_t d_in, int64_t d_out, float eps, float* row_rstd, void* stream, bool may_allocate) {
  if (rows < 0 || d_in < 0 || d_out < 0) return LK_ERR_INVALID_ARG;
  if (rows == 0 || d_out == 0) return LK_OK;
  if (!x || !w_fold || !y || !row_rstd || d_in == 0) return LK_ERR_INVALID_ARG;
  if (!is16(dtype)) return LK_ERR_UNSUPPORTED;
  if (d_in % 8 || x_ld < d_in || x_ld % 8 || y_ld < d_out) return LK_ERR_INVALID_ARG;
  if (rows > INT32_MAX / 2 || d_in > INT32_MAX / 2 || d_out > INT32_MAX / 2) return LK_ERR_INVALID_ARG;
  if (!aligned16(x) || !aligned16(w_fold)) return LK_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (int st = bind_stream(s)) return st;
  return dtype == LK_F16
             ? run_gemm<gemm::Kind::F16>(x, x_ld, w_fold, y, y_ld, rows, d_in, d_out, eps, row_rstd, s, may_allocate)
             : run_gemm<gemm::Kind::BF16>(x, x_ld, w_fold, y, y_ld, rows, d_in, d_out, eps, row_rstd, s,
                                          may_allocate);
}
}  // namespace
}  // namespace lk

extern "C" int lk_rmsnorm_linear(const void* x, int64_t x_ld, const void* w_fold, void* y, int64_t y_ld, int dtype,
                                 int64_t rows, int64_t d_in, int64_t d_out, float eps, float* row_rstd,
                                 void* stream) {
  return lk::rmsnorm_linear(x, x_ld, w_fold, y, y_ld, dtype, rows, d_in, d_out, eps, row_rstd, stream, true);
}

extern "C" int lk_fused_rmsnorm_linear(const void* X, const void* W_norm, const void* W_lin, void* Y, float eps,
                                       int64_t B, int64_t D_in, int64_t D_out, int dtype, void* w_fold,
                                       float* row_rstd, void* stream) {
  if (int st = lk_rmsnorm_linear_fold(W_norm, dtype, W_lin, w_fold, dtype, D_in, D_out, stream)) return st;
  return lk_rmsnorm_linear(X, D_in, w_fold, Y, D_out, dtype, B, D_in, D_out, eps, row_rstd, stream);
}

// ---- RMSNorm + Linear without any caller-provided scratch -----------------------------------
// For callers that cannot allocate device memory at the point of the call (see the header):
// the per-row rsqrt scratch that lk_rmsnorm_linear takes as `row_rstd` lives in this file-scope
// array instead.  Host code must not pass `g_static_rstd` itself to a kernel — on the host that
// name is only a stand-in — so its device address is looked up once per device, with that
// device current, and cached.
namespace lk {
namespace {
constexpr int64_t kStaticRstdRows = 65536;  // 256 KiB of fp32 on every device that loads the library
static __device__ __align__(256) float g_static_rstd[kStaticRstdRows];
constexpr int kStaticDevices = 64;
std::mutex g_static_mu;
float* g_static_rstd_addr[kStaticDevices];
unsigned long long g_static_rstd_ctx[kStaticDevices];  // unique id of the context it belongs to
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;

// Unique id (for the life of the process) of the calling thread's current context, 0 if none.
unsigned long long current_context_id() {
  if (!g_ctx_current || !g_ctx_id) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
        q1 != cudaDriverEntryPointSuccess || cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
        q2 != cudaDriverEntryPointSuccess)
      return 0;
    g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f1);
    g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(f2);
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx || g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// The array's address, looked up once per device with that device current and kept with the
// id of the context it was looked up in.  A device reset replaces the context (and the module
// that holds the array), so a call in a new context looks the address up again.
int static_rstd_address(float** out) {
  int dev = -1;
  if (int st = cuda_status(cudaGetDevice(&dev))) return st;
  if (dev < 0 || dev >= kStaticDevices) return LK_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_static_mu);
  const unsigned long long id = current_context_id();
  if (id == 0 || !g_static_rstd_addr[dev] || g_static_rstd_ctx[dev] != id) {
    void* p = nullptr;
    if (int st = cuda_status(cudaGetSymbolAddress(&p, g_static_rstd))) return st;
    g_static_rstd_addr[dev] = static_cast<float*>(p);
    g_static_rstd_ctx[dev] = current_context_id();  // the lookup made the context current
  }
  *out = g_static_rstd_addr[dev];
  return LK_OK;
}
}  // namespace
}  // namespace lk

extern "C" int lk_rmsnorm_linear_noalloc(const void* x, int64_t x_ld, const void* w_fold, void* y, int64_t y_ld,
                                         int dtype, int64_t rows, int64_t d_in, int64_t d_out, float eps,
                                         void* stream) {
  using namespace lk;
  if (rows < 0 || d_in < 0 || d_out < 0) return LK_ERR_INVALID_ARG;
  if (rows > kStaticRstdRows) return LK_ERR_SCRATCH_LIMIT;
  if (rows == 0 || d_out == 0) return LK_OK;
  if (int st = bind_stream(static_cast<cudaStream_t>(stream))) return st;
  float* rstd = nullptr;
  if (int st = static_rstd_address(&rstd)) return st;
  // Every element of rstd[0, rows) is written by the row kernel before the GEMM reads it, so
  // whatever the previous call left in the array needs no clearing.
  return rmsnorm_linear(x, x_ld, w_fold, y, y_ld, dtype, rows, d_in, d_out, eps, rstd, stream, false);
}
