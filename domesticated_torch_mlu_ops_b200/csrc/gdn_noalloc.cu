// gdn_chunk_fwd_noalloc: the chunked prefill for callers that cannot allocate
// device memory.
//
// gdn_chunk_fwd needs a caller-provided workspace (hundreds of MB for long
// prefills).  Some callers have no way to get one: plain C hosts that link
// this library without a device allocator of their own, and serving engines
// that hand all of the GPU's memory to their own pool at start-up (a
// cudaMalloc there fails, and a cudaMalloc/cudaFree pair in the request path
// would also synchronise the device).  This entry point serves them from a
// scratch array compiled into the library instead.  The array has a fixed
// size (kNoAllocScratchBytes, 32 MiB); every GPU that loads the library holds
// it until the process exits.  Requests whose workspace would not fit are
// rejected with GDN_ERR_WORKSPACE.
//
// The array's host-side name is only a stand-in for the symbol; its device
// address is fetched with cudaGetSymbolAddress once per device (on the first
// call made with that device current, so that first call should happen
// before any stream capture).  All calls share the one array: calls that
// overlap on the GPU (different streams, or different host threads on one
// device) race on it and must be serialised by the caller.  The error word
// at the start of the scratch is cleared on every call (and read back by
// gdn_chunk_noalloc_check_device_error); everything else is fully rewritten
// by the kernels before it is read.

#include <mutex>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 128;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up once per
// device).  Returns nullptr and sets the last error on failure.
void* scratch_on_current_device() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    gdn::set_last_error(GDN_ERR_CUDA, "gdn_chunk_fwd_noalloc: cudaGetDevice failed (%s)",
                        cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
      gdn::set_last_error(GDN_ERR_CUDA, "gdn_chunk_fwd_noalloc: cudaGetSymbolAddress failed (%s)",
                          cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_addr[dev] = ptr;
  }
  return g_scratch_addr[dev];
}

}  // namespace

extern "C" int gdn_chunk_fwd_noalloc(const gdn_chunk_args* args, void* stream) {
  const size_t need = gdn_chunk_workspace_size(args);
  if (need == 0) return GDN_ERR_INVALID;  // message set by gdn_chunk_workspace_size
  if (need > kNoAllocScratchBytes)
    return gdn::set_last_error(GDN_ERR_WORKSPACE,
                               "gdn_chunk_fwd_noalloc: this call needs %zu bytes of workspace; the "
                               "built-in scratch holds %zu (use gdn_chunk_fwd with a caller workspace)",
                               need, kNoAllocScratchBytes);
  void* scratch = scratch_on_current_device();
  if (!scratch) return GDN_ERR_CUDA;
  cudaError_t e = cudaMemsetAsync(scratch, 0, 16, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return gdn::set_last_error(GDN_ERR_CUDA, "gdn_chunk_fwd_noalloc: %s", cudaGetErrorString(e));
  gdn_chunk_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  return gdn_chunk_fwd(&a, stream);
}

// The device error word of the scratch on the current device (the word that
// gdn_chunk_check_device_error reads from a caller's workspace).
extern "C" int gdn_chunk_noalloc_check_device_error(void* stream) {
  void* scratch = scratch_on_current_device();
  if (!scratch) return GDN_ERR_CUDA;
  return gdn_chunk_check_device_error(scratch, stream);
}
