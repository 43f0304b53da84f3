// dash_noalloc.cu -- decode attention that allocates nothing.
//
// dash_decode_attn() takes its split-KV scratch (partial outputs and the
// per-(row, head) arrival counters) from a caller-provided workspace.  Some
// callers cannot provide one: a host program whose device memory is owned by
// its own pool and that may not call cudaMalloc on the hot path, or a thin FFI
// consumer of this C ABI that has no allocator at all.  For them,
// dash_decode_attn_noalloc() runs the same kernel on a fixed scratch area that
// lives in this library's own device memory (a file-scope __device__ array).
#include <mutex>

#include "dash_internal.h"

namespace {

// Fixed scratch: 8 MiB per device, held from library load until process exit.
constexpr size_t kScratchBytes = DASH_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array for the current device.  The name of a
// __device__ array in host code is only a host-side stand-in, so the address
// is looked up once per device, with that device current.
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return dash::set_error(DASH_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return dash::set_error(DASH_ERR_UNSUPPORTED, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return dash::set_error(DASH_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DASH_OK;
}

}  // namespace

extern "C" size_t dash_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" int dash_decode_attn_noalloc(const DashDecodeArgs* args, dash_stream_t stream) {
  int splits = 0;
  const int rc0 = dash::validate_decode(args, &splits);
  if (rc0) return rc0;
  const size_t need = dash_decode_workspace_size(args);
  if (need > kScratchBytes)
    return dash::set_error(DASH_ERR_WORKSPACE,
                           "decode needs %zu bytes of split scratch; the allocation-free entry point "
                           "has a fixed %zu bytes (use fewer splits or rows, or dash_decode_attn with "
                           "a workspace)",
                           need, kScratchBytes);
  DashDecodeArgs a = *args;
  if (need > 0) {
    void* p = nullptr;
    int rc = scratch_address(&p);
    if (rc) return rc;
    a.workspace = p;
    a.workspace_bytes = kScratchBytes;
  }
  return dash_decode_attn(&a, stream);
}
