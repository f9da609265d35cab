// lk_common.cu — status codes, the device status word, device queries and TMA descriptor
// encoding shared by every entry point.
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <utility>

#include "gemm_split.h"
#include "lk_abi.h"
#include "lk_sm100.cuh"

namespace lk {

__device__ int g_status[4];
__device__ unsigned long long g_wait_limit_ns = 1000000000ull;

namespace {
thread_local int t_last_cuda_error = 0;
// Device this library made current on the calling thread with cudaSetDevice (-1: none yet).
// cudaGetDevice alone cannot tell: it reports device 0 on a fresh thread without making any
// context current, and the driver calls of this library (TMA descriptor encoding) need one --
// e.g. on the worker thread that runs autograd's backward.
thread_local int t_bound_device = -1;

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
std::mutex g_mu;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  return g_encode;
}
}  // namespace

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return LK_OK;
  t_last_cuda_error = (int)err;
  return LK_ERR_CUDA;
}

int bind_device(int dev) {
  if (t_bound_device == dev) return LK_OK;
  const int st = cuda_status(cudaSetDevice(dev));  // makes the device's primary context current
  if (st == LK_OK) t_bound_device = dev;
  return st;
}

int bind_stream(cudaStream_t stream) {
  if (stream == nullptr) return t_bound_device >= 0 ? LK_OK : bind_device(0);
  int dev = -1;
  const int st = cuda_status(cudaStreamGetDevice(stream, &dev));
  if (st != LK_OK) return st;
  return bind_device(dev);
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_sm_count[dev] > 0) return g_sm_count[dev];
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  std::lock_guard<std::mutex> lock(g_mu);
  g_sm_count[dev] = n;
  return n;
}

int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle,
              CUtensorMapL2promotion promo) {
  if (!aligned16(base)) return LK_ERR_ALIGNMENT;
  for (int i = 0; i + 1 < rank; ++i)
    if (strides_bytes[i] % 16 != 0) return LK_ERR_ALIGNMENT;
  auto enc = encoder();
  if (!enc) return cuda_status(cudaErrorNotSupported);
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = enc(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = 10000 + (int)r;  // driver error codes are offset to tell them apart
    return LK_ERR_CUDA;
  }
  return LK_OK;
}

namespace {
std::mutex g_inject_mu;
Injection g_inject = {LK_INJECT_NONE, -1, -1};
}  // namespace

Injection take_injection(int kind) {
  std::lock_guard<std::mutex> lock(g_inject_mu);
  if (g_inject.kind != kind || kind == LK_INJECT_NONE) return Injection{LK_INJECT_NONE, -1, -1};
  const Injection r = g_inject;
  g_inject = Injection{LK_INJECT_NONE, -1, -1};
  return r;
}

namespace gemm {
namespace {
std::mutex g_ws_mu;
std::map<std::pair<int, uintptr_t>, SplitWorkspace> g_ws_table;  // (device, stream) -> workspace
}  // namespace

bool split_workspace(cudaStream_t stream, int npairs, SplitWorkspace* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const auto key = std::make_pair(dev, reinterpret_cast<uintptr_t>(stream));
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto it = g_ws_table.find(key);
  if (it != g_ws_table.end()) {
    *out = it->second;
    return true;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return false;
  }
  SplitWorkspace ws;
  const size_t partial_bytes = (size_t)npairs * 8 * 8 * 256 * sizeof(uint4);
  ws.flag_bytes = (size_t)npairs * 16 * sizeof(int);
  if (cudaMalloc(&ws.partial, partial_bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cudaMalloc(&ws.flags, ws.flag_bytes) != cudaSuccess ||
      cudaMemsetAsync(ws.flags, 0, ws.flag_bytes, stream) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(ws.partial);
    if (ws.flags) cudaFree(ws.flags);
    return false;
  }
  g_ws_table[key] = ws;
  *out = ws;
  return true;
}

int reset_split_workspaces() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  std::lock_guard<std::mutex> lock(g_ws_mu);
  for (auto& kv : g_ws_table) {
    if (kv.first.first != dev) continue;
    e = cudaMemset(kv.second.flags, 0, kv.second.flag_bytes);
    if (e != cudaSuccess) return (int)e;
  }
  return (int)cudaDeviceSynchronize();
}
}  // namespace gemm

}  // namespace lk

extern "C" {

const char* lk_status_string(int status) {
  switch (status) {
    case LK_OK:
      return "ok";
    case LK_ERR_INVALID_ARG:
      return "invalid argument";
    case LK_ERR_UNSUPPORTED:
      return "unsupported dtype, head dim or layout";
    case LK_ERR_CUDA:
      return "CUDA error";
    case LK_ERR_TIMEOUT:
      return "device pipeline wait timed out";
    case LK_ERR_ALIGNMENT:
      return "pointer or stride not 16-byte aligned";
    case LK_ERR_SCRATCH_LIMIT:
      return "problem exceeds the fixed scratch of a no-allocation entry point (rows > 65536)";
    default:
      return "unknown status";
  }
}

int lk_last_cuda_error(void) { return lk::t_last_cuda_error; }

int lk_version(void) { return (1 << 16) | 0; }

int lk_set_device(int device) { return lk::bind_device(device); }

int lk_device_status(int* out4) {
  int h[4] = {0, 0, 0, 0};
  int st = lk::cuda_status(cudaDeviceSynchronize());
  if (st != LK_OK) return st;
  st = lk::cuda_status(cudaMemcpyFromSymbol(h, lk::g_status, sizeof(h)));
  if (st != LK_OK) return st;
  if (out4)
    for (int i = 0; i < 4; ++i) out4[i] = h[i];
  return h[0];
}

int lk_debug_set_wait_limit(int64_t ns) {
  const unsigned long long v = ns > 0 ? (unsigned long long)ns : 1000000000ull;
  int st = lk::cuda_status(cudaDeviceSynchronize());
  if (st != LK_OK) return st;
  return lk::cuda_status(cudaMemcpyToSymbol(lk::g_wait_limit_ns, &v, sizeof(v)));
}

int lk_debug_inject(int kind, int block, int item) {
  if (kind < LK_INJECT_NONE || kind > LK_INJECT_REQUANT_SKIP_PUBLISH) return LK_ERR_INVALID_ARG;
  if (kind != LK_INJECT_NONE && (block < 0 || item < 0)) return LK_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(lk::g_inject_mu);
  lk::g_inject = lk::Injection{kind, block, item};
  return LK_OK;
}

int lk_clear_device_status(void) {
  int z[4] = {0, 0, 0, 0};
  int st = lk::cuda_status(cudaDeviceSynchronize());
  if (st != LK_OK) return st;
  // A split GEMM launch that gave up may have left its tail counters non-zero.
  st = lk::cuda_status((cudaError_t)lk::gemm::reset_split_workspaces());
  if (st != LK_OK) return st;
  return lk::cuda_status(cudaMemcpyToSymbol(lk::g_status, z, sizeof(z)));
}

}  // extern "C"
