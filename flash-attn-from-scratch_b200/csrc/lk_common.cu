// lk_common.cu — status codes, the device status word, device queries and TMA descriptor
// encoding shared by every entry point.
#include <cudaTypedefs.h>

#include <mutex>

#include "lk_abi.h"
#include "lk_sm100.cuh"

namespace lk {

__device__ int g_status[4];

namespace {
thread_local int t_last_cuda_error = 0;

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

int bind_stream(cudaStream_t stream) {
  if (stream == nullptr) return LK_OK;
  int dev = -1, cur = -1;
  int st = cuda_status(cudaStreamGetDevice(stream, &dev));
  if (st != LK_OK) return st;
  st = cuda_status(cudaGetDevice(&cur));
  if (st != LK_OK) return st;
  if (cur != dev) return cuda_status(cudaSetDevice(dev));
  return LK_OK;
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

int lk_set_device(int device) {
  int cur = -1;
  if (cudaGetDevice(&cur) == cudaSuccess && cur == device) return LK_OK;
  return lk::cuda_status(cudaSetDevice(device));
}

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

int lk_clear_device_status(void) {
  int z[4] = {0, 0, 0, 0};
  int st = lk::cuda_status(cudaDeviceSynchronize());
  if (st != LK_OK) return st;
  return lk::cuda_status(cudaMemcpyToSymbol(lk::g_status, z, sizeof(z)));
}

}  // extern "C"
