// noalloc.cu -- backward selective scan for callers that cannot allocate device memory.
//
// mb200_selective_scan_bwd needs a workspace that the caller allocates, and the *_f32 mirror
// allocates it itself with cudaMallocAsync. Some callers can do neither: for example a host
// framework or plugin interface that owns all device memory and forbids allocations inside its
// execute callbacks, or a latency-critical path that must not take an allocator's locks or its
// implicit synchronisation. mb200_selective_scan_bwd_noalloc serves them: its scratch is a
// file-scope static device array of kNoAllocScratchBytes that every GPU holds from the moment this
// library's device code is loaded on it until the process exits. Nothing is allocated per call.
//
// The host-side name of that array is only a stand-in for it, not a device address; the device
// address is obtained once per device with cudaGetSymbolAddress, on that device's first call.
// That first call therefore performs a runtime query and should be made before any stream
// capture on that device; if the query fails the call returns MB200_ERR_CUDA and the next call
// tries again. All calls on a device share the same array and it keeps the previous
// call's contents; the backward writes every scratch byte it later reads, so nothing has to be
// cleared between calls. Calls whose GPU work overlaps (different streams, or several host
// threads) race on the shared scratch and must be serialised by the caller.
#include <cuda_runtime.h>

#include <mutex>

#include "mamba_b200.h"

namespace {

constexpr size_t kNoAllocScratchBytes = MB200_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the static scratch on the current device. Only a successful lookup is kept:
// a lookup that failed (for example one attempted during stream capture) is retried by the next
// call instead of failing every later call on that device.
int current_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MB200_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();  // the failed query must not surface as a later call's launch error
      return MB200_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return MB200_OK;
}

}  // namespace

extern "C" {

MB200_API int mb200_selective_scan_bwd_noalloc(const mb200_scan_bwd_params* p, void* stream) {
  if (p == nullptr) return MB200_ERR_NULL_POINTER;
  const size_t need = mb200_selective_scan_bwd_workspace_size(p);
  if (need > kNoAllocScratchBytes) return MB200_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  if (need > 0) {
    const int st = current_scratch(&scratch);
    if (st != MB200_OK) return st;
  }
  // Argument validation (including requests whose workspace size is 0 because they are invalid)
  // happens in the regular entry point before anything is enqueued.
  return mb200_selective_scan_bwd(p, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
