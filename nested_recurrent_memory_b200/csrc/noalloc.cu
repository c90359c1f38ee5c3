// Allocation-free variant of the forward: ngdn2_fwd_noalloc.
//
// Some callers cannot hand us a workspace: a plug-in running inside a host
// process that owns all device memory through its own pool, a serving loop
// that reserved its whole memory budget at start-up and may not allocate
// while requests are in flight, or code that must not take the device-wide
// synchronisation a cudaMalloc/cudaFree can imply. For them this entry point
// takes its scratch from one buffer that is part of the library image
// itself (a file-scope __device__ array), so neither the library nor the
// caller allocates anything per call; the caller still passes every input
// and output.
//
// Properties a caller must know:
//   * Capacity: NGDN2_NOALLOC_SCRATCH_BYTES (64 MiB). A call whose scratch
//     need (ngdn2_fwd_workspace_size) exceeds it is rejected with
//     NGDN2_ERR_WORKSPACE before anything is launched.
//   * Every GPU that loads the library holds this buffer until the process
//     exits.
//   * The buffer is shared by all calls on a device and keeps whatever the
//     last call left in it. Nothing in it needs to start at zero: every call
//     writes each scratch byte before it reads it. Two calls whose kernels
//     overlap on the GPU (for example on two streams) race on the buffer;
//     serialise them.
//   * The first call on each device looks up the buffer's device address
//     (cudaGetSymbolAddress) with that device current and caches it. Make
//     that first call before any stream capture. The cache lives as long as
//     the process: after cudaDeviceReset (or any teardown and re-creation of
//     the device's primary context) the cached address is stale, so a
//     process that resets a device must not call this entry point again.

#include <mutex>

#include "../../include/ngdn2.h"

#include <cuda_runtime.h>

namespace {

constexpr size_t kScratchBytes = NGDN2_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The fixed scratch. In host code this name only stands in for the symbol:
// its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_setup_mutex;

// Device address of the scratch on the current device, looked up once per
// device. Returns nullptr (and sets *err) when the lookup fails.
void* scratch_on_current_device(cudaError_t* err) {
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return nullptr;
  if (dev < 0 || dev >= kMaxDevices) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    *err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (*err != cudaSuccess || !ptr) return nullptr;
    g_scratch_ptr[dev] = ptr;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int ngdn2_fwd_noalloc(const ngdn2_fwd_args* args, void* stream) {
  if (!args) return NGDN2_ERR_NULL;
  size_t need = 0;
  const int rc = ngdn2_fwd_workspace_size(args, &need);
  if (rc != NGDN2_OK) return rc;
  if (need > kScratchBytes) return NGDN2_ERR_WORKSPACE;
  cudaError_t err = cudaSuccess;
  void* scratch = scratch_on_current_device(&err);
  if (!scratch) return NGDN2_ERR_CUDA;
  ngdn2_fwd_args local = *args;
  local.workspace = scratch;
  local.workspace_bytes = kScratchBytes;
  return ngdn2_fwd(&local, stream);
}
