// m3b_layer_fwd_noalloc: the layer forward without any device allocation.
//
// Some callers cannot allocate device memory at the point where they run the
// layer: a plugin hosted inside another runtime that hands it only the input
// and output buffers (and owns the device allocator itself), or a hot path where
// allocation is forbidden because it would synchronise or fragment the heap.
// For them this entry point takes its workspace from one static device array
// of kNoallocScratchBytes, which every GPU that loads this library keeps until
// the process exits.  Problems whose workspace (m3b_layer_fwd_workspace) does
// not fit are rejected with M3B_ERR_WORKSPACE.
//
// Every call shares the array and it keeps the previous call's contents.  The
// forward writes every scratch word it later reads, so nothing has to be
// cleared between calls; two calls that overlap on the GPU (different streams,
// or different host threads on the same device) race on the array and must be
// serialised by the caller.
//
// The array's device address is looked up once per device, with that device
// current, on the first call made on it; make that first call before any
// stream capture begins.
#include <mutex>

#include "launch.h"

namespace {

constexpr size_t kNoallocScratchBytes = M3B_NOALLOC_SCRATCH_BYTES;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {nullptr};

// Device address of g_noalloc_scratch on the current device (host code may not
// use the symbol itself as a device pointer).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return m3b::fail(M3B_ERR_CUDA, "layer_fwd_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return m3b::fail(M3B_ERR_UNSUPPORTED, "layer_fwd_noalloc: device ordinal %d", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return m3b::fail(M3B_ERR_CUDA, "layer_fwd_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return M3B_OK;
}

}  // namespace

extern "C" int m3b_layer_fwd_noalloc(const m3b_layer_fwd_args* a, void* stream) {
  if (!a) return m3b::fail(M3B_ERR_INVALID_ARG, "layer_fwd_noalloc: null args");
  const size_t need = m3b::layer_fwd_workspace_min(a);
  if (need == 0) return m3b::layer_fwd(a, nullptr, 0, static_cast<cudaStream_t>(stream));  // reports why
  if (need > kNoallocScratchBytes)
    return m3b::fail(M3B_ERR_WORKSPACE,
                     "layer_fwd_noalloc: this problem needs %zu bytes of scratch; the static scratch holds %zu "
                     "(use m3b_layer_fwd with a caller-allocated workspace)",
                     need, kNoallocScratchBytes);
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != M3B_OK) return rc;
  return m3b::layer_fwd(a, scratch, kNoallocScratchBytes, static_cast<cudaStream_t>(stream));
}
