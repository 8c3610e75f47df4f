// tfa_fwd_static_workspace: the paged attention forward for callers that cannot
// allocate device memory.
//
// Some hosts drive this library only through borrowed device pointers: a serving loop
// whose memory is carved up once at start-up and which must never call cudaMalloc in
// the middle of a step (cudaMalloc may implicitly synchronise the device and can fail
// under fragmentation), or a foreign-language host (cgo, JNI, N-API, ctypes without
// torch) that binds the C ABI but has no device allocator of its own to create the
// split-KV workspace tfa_fwd asks for. This entry point runs the same kernels with the
// workspace placed in a fixed-size array in the library's own device memory instead.
//
// Cost and limits:
//   * the array below is TFA_STATIC_WORKSPACE_BYTES (32 MiB) and exists on every GPU on
//     which the library's device code is loaded, until the process exits;
//   * a call whose workspace (tfa_workspace_size) exceeds it is rejected with
//     TFA_ERR_STATIC_WORKSPACE_LIMIT before anything is launched;
//   * every call on a device shares the one array and leaves its contents behind, so
//     calls that may overlap on the GPU (different streams without ordering between them)
//     race on it and must not be issued;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; that first call should come
//     before any stream capture on the calling thread.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/tfa.h"
#include "tfa_internal.h"

namespace tfa {
namespace {

constexpr int kMaxDevices = 128;

// Split-KV partial outputs / LSEs and the scheduler and error words of one call.
static __device__ __align__(256) unsigned char g_static_workspace[TFA_STATIC_WORKSPACE_BYTES];

// Device address of g_static_workspace per device, filled on the first call made
// with that device current. The host-side name g_static_workspace is only a stand-in
// for the symbol and must never be handed to a kernel.
void* g_workspace_addr[kMaxDevices] = {};
std::mutex g_workspace_mutex;

int static_workspace_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TFA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return TFA_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_workspace_mutex);
  if (!g_workspace_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_workspace) != cudaSuccess || !p) return TFA_ERR_CUDA;
    g_workspace_addr[dev] = p;
  }
  *out = g_workspace_addr[dev];
  return TFA_OK;
}

}  // namespace
}  // namespace tfa

extern "C" int tfa_fwd_static_workspace(const tfa_fwd_params* p, void* stream) {
  using namespace tfa;
  if (!p) return TFA_ERR_NULL_POINTER;
  if (p->batch == 0 || p->total_q == 0) return tfa_fwd(p, nullptr, 0, stream);  // validates, launches nothing
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TFA_ERR_CUDA;
  // Planned for the per-head decode kernel only: the page kernel's split partials can
  // exceed the fixed workspace. The scheduler counters, the error word and the decode
  // kernel's per-group split counters must start at zero; the split partials are fully
  // written before they are read, so only those leading ranges are cleared.
  size_t off[2], bytes[2], need = 0;
  if (workspace_zero_ranges(p, dev, off, bytes, false, &need) != TFA_OK)
    return tfa_fwd(p, nullptr, 0, stream);  // invalid arguments: same status as tfa_fwd
  if (need > (size_t)TFA_STATIC_WORKSPACE_BYTES) return TFA_ERR_STATIC_WORKSPACE_LIMIT;
  void* ws = nullptr;
  int rc = static_workspace_for_current_device(&ws);
  if (rc != TFA_OK) return rc;
  for (int i = 0; i < 2; ++i)
    if (bytes[i] && cudaMemsetAsync(static_cast<unsigned char*>(ws) + off[i], 0, bytes[i],
                                    reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
      return TFA_ERR_CUDA;
  return fwd_impl(p, ws, TFA_STATIC_WORKSPACE_BYTES, stream, nullptr, nullptr, false);
}

extern "C" int tfa_read_static_workspace_error(void* stream, int* err) {
  using namespace tfa;
  if (!err) return TFA_ERR_NULL_POINTER;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TFA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return TFA_ERR_DEVICE;
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_workspace_mutex);
    ws = g_workspace_addr[dev];
  }
  if (!ws) return TFA_ERR_CUDA;
  return tfa_read_device_error(ws, stream, err);
}
