// lk_abi.h — host-side helpers shared by the C-ABI entry points (internal).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/llm_kernels_b200.h"

namespace lk {

// Records err as this host thread's last CUDA error and returns LK_ERR_CUDA (or LK_OK).
int cuda_status(cudaError_t err);

// cudaGetLastError() after a launch, mapped to a status.
inline int check_launch() { return cuda_status(cudaGetLastError()); }

// Makes `dev` current in this library's runtime on the calling thread, with its primary
// context (cached per thread).
int bind_device(int dev);

// Binds to the stream's device (for the NULL stream: to the device set with lk_set_device, or
// device 0).
int bind_stream(cudaStream_t stream);

// Streaming multiprocessor count of the current device (cached per device).
int sm_count();

// Builds a tiled TMA descriptor (row-major tensor, dims/strides innermost first; strides in
// bytes for dims 1..rank-1).  Returns LK_OK, LK_ERR_ALIGNMENT or LK_ERR_CUDA.
int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle,
              CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Test-hook injection armed by lk_debug_inject.  take_injection(kind) returns it (and disarms
// it) if it is of that kind; otherwise {LK_INJECT_NONE, -1, -1}.
struct Injection {
  int kind, block, item;
};
Injection take_injection(int kind);

}  // namespace lk
