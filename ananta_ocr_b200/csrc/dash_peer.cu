// dash_peer.cu -- device memory shared between the ranks of one node, for the
// prefill kernel's fused output gather (each rank stores its output rows
// straight into every rank's gathered output over NVLink).
//
// A rank exports a buffer as a CUDA IPC handle of the allocation that holds
// it plus the buffer's offset inside that allocation; the other ranks open the
// handle (once per allocation and process) and add the offset.  The handles
// travel between processes through the host (torch.distributed objects).
#include <cuda.h>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "dash_internal.h"

namespace {

struct Opened {
  void* base;
  int refs;
};
std::mutex g_mu;
std::map<std::string, Opened> g_open;                    // handle bytes -> mapping
std::map<void*, std::pair<std::string, int>> g_by_ptr;   // returned pointer -> (handle, imports)

// cuMemGetAddressRange through the runtime's driver entry point (the library
// does not link libcuda directly)
typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range() {
  static AddressRangeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  }
  return fn;
}

}  // namespace

extern "C" int dash_peer_export(const void* ptr, DashPeerHandle* out) {
  if (!ptr || !out) return dash::set_error(DASH_ERR_INVALID, "null pointer");
  AddressRangeFn range = address_range();
  if (!range) return dash::set_error(DASH_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range(&base, &size, (CUdeviceptr)ptr);
  if (r != CUDA_SUCCESS)
    return dash::set_error(DASH_ERR_CUDA, "cuMemGetAddressRange failed (%d): not device memory?", (int)r);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return dash::set_error(DASH_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == sizeof(out->handle), "IPC handle size");
  memcpy(out->handle, &h, sizeof(h));
  out->offset = (int64_t)((CUdeviceptr)ptr - base);
  out->alloc_bytes = (int64_t)size;
  return DASH_OK;
}

extern "C" int dash_peer_import(const DashPeerHandle* h, void** ptr) {
  if (!h || !ptr) return dash::set_error(DASH_ERR_INVALID, "null pointer");
  if (h->offset < 0 || h->offset >= h->alloc_bytes)
    return dash::set_error(DASH_ERR_INVALID, "offset outside the exported allocation");
  std::string key(h->handle, sizeof(h->handle));
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_open.find(key);
  if (it == g_open.end()) {
    cudaIpcMemHandle_t ih;
    memcpy(&ih, h->handle, sizeof(ih));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, ih, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess)
      return dash::set_error(DASH_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    it = g_open.emplace(key, Opened{base, 0}).first;
  }
  it->second.refs++;
  void* p = static_cast<char*>(it->second.base) + h->offset;
  auto& slot = g_by_ptr[p];
  slot.first = key;
  slot.second++;
  *ptr = p;
  return DASH_OK;
}

extern "C" int dash_peer_close(void* ptr) {
  std::lock_guard<std::mutex> lock(g_mu);
  auto it = g_by_ptr.find(ptr);
  if (it == g_by_ptr.end()) return dash::set_error(DASH_ERR_INVALID, "pointer was not imported");
  auto op = g_open.find(it->second.first);
  if (--it->second.second == 0) g_by_ptr.erase(it);
  if (op != g_open.end() && --op->second.refs == 0) {
    cudaError_t e = cudaIpcCloseMemHandle(op->second.base);
    g_open.erase(op);
    if (e != cudaSuccess)
      return dash::set_error(DASH_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  }
  return DASH_OK;
}
