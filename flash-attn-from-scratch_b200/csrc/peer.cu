// peer.cu — mapping another rank's device buffer into this process (CUDA IPC), so a kernel on
// this GPU can store into it over NVLink.  Host-side plumbing only: the column-sharded int8
// GEMM's scatter epilogue (lk_int8_gemm_dequant_scatter) writes every rank's replicated
// output through these mappings.
//
// An exported handle names the whole allocation that holds the pointer (a caching allocator
// hands out pieces of larger allocations), so the export also returns the pointer's offset
// inside it and the importer adds it back.  Two buffers a peer carved out of one allocation
// therefore arrive with the same handle: the importer opens each (device, handle) once and
// counts its users, and only the last lk_peer_close of a mapping unmaps it.
#include <cudaTypedefs.h>

#include <array>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "lk_abi.h"

namespace lk {
namespace {

std::mutex g_peer_mu;
PFN_cuMemGetAddressRange_v3020 g_range = nullptr;

// Open mappings of this process: (device, handle bytes) -> (base address, users), and the
// reverse index (device, base) -> handle for lk_peer_close.
using HandleKey = std::pair<int, std::array<char, LK_PEER_HANDLE_BYTES>>;
struct Mapping {
  void* base;
  int users;
};
std::mutex g_map_mu;
std::map<HandleKey, Mapping> g_open;
std::map<std::pair<int, uintptr_t>, HandleKey> g_by_base;

PFN_cuMemGetAddressRange_v3020 address_range() {
  std::lock_guard<std::mutex> lock(g_peer_mu);
  if (!g_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  return g_range;
}

}  // namespace
}  // namespace lk

extern "C" int lk_peer_export(int device, const void* ptr, void* handle_out, int64_t* offset_out) {
  using namespace lk;
  if (!ptr || !handle_out || !offset_out) return LK_ERR_INVALID_ARG;
  if (int st = lk_set_device(device)) return st;
  auto range = address_range();
  if (!range) return LK_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return LK_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (int st = cuda_status(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)))) return st;
  static_assert(sizeof(h) == LK_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
  return LK_OK;
}

extern "C" int lk_peer_open(int device, const void* handle, int64_t offset, void** ptr_out) {
  using namespace lk;
  if (!handle || !ptr_out || offset < 0) return LK_ERR_INVALID_ARG;
  if (int st = lk_set_device(device)) return st;
  HandleKey key;
  key.first = device;
  memcpy(key.second.data(), handle, LK_PEER_HANDLE_BYTES);
  std::lock_guard<std::mutex> lock(g_map_mu);
  auto it = g_open.find(key);
  if (it != g_open.end()) {
    ++it->second.users;
    *ptr_out = static_cast<uint8_t*>(it->second.base) + offset;
    return LK_OK;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (int st = cuda_status(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess))) return st;
  g_open[key] = Mapping{base, 1};
  g_by_base[std::make_pair(device, reinterpret_cast<uintptr_t>(base))] = key;
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return LK_OK;
}

extern "C" int lk_peer_close(int device, void* ptr, int64_t offset) {
  using namespace lk;
  if (!ptr || offset < 0) return LK_ERR_INVALID_ARG;
  if (int st = lk_set_device(device)) return st;
  void* base = static_cast<uint8_t*>(ptr) - offset;
  std::lock_guard<std::mutex> lock(g_map_mu);
  auto bit = g_by_base.find(std::make_pair(device, reinterpret_cast<uintptr_t>(base)));
  if (bit == g_by_base.end()) return LK_ERR_INVALID_ARG;  // not a mapping made by lk_peer_open
  auto it = g_open.find(bit->second);
  if (--it->second.users > 0) return LK_OK;
  g_open.erase(it);
  g_by_base.erase(bit);
  return cuda_status(cudaIpcCloseMemHandle(base));
}
