// Allocation-free variant of the S+LR forward: slr_lrs_linear_forward_noalloc.
//
// Some callers cannot allocate device memory at all, not even once: a plugin
// running inside a host framework whose memory manager owns every allocation
// and forbids direct cudaMalloc, code that executes while someone else's
// stream capture is active (an allocation there would break the capture), or
// a latency-critical serving loop that must never enter the driver's
// allocator.  This entry point takes no workspace.  Its scratch — the
// low-rank intermediate H = x·Bᵀ — lives in one fixed array inside this
// library's device image, kScratchBytes per device.
//
// Behaviour a caller must know:
//  * Every GPU that loads this library holds the array until the process
//    exits.
//  * The first call on a device looks up the array's device address for that
//    device (cudaGetSymbolAddress, with the device current); make that first
//    call before any stream capture.
//  * All calls share the one array; calls that may run at the same time on
//    the GPU (different streams, or several devices' work aliased by the
//    caller) race on it.
//  * A call whose token count needs more scratch than the array holds is
//    rejected with SLR_ERR_WORKSPACE before anything is launched.
#include <mutex>

#include "internal.hpp"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kMaxDevices = 64;

// Host code must not take this name as a device pointer: it is a host-side
// stand-in.  The device address comes from scratch_address().
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  SLR_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return slr::fail(SLR_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return slr::cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return SLR_OK;
}

}  // namespace

extern "C" int slr_lrs_linear_forward_noalloc(const slr_layer* layer, const void* x, int64_t ldx, void* y,
                                              int64_t ldy, int64_t M, void* stream) {
  const size_t need = (layer != nullptr && M > 0) ? slr_lrs_linear_workspace_size(layer, M) : 0;
  if (need > kScratchBytes)
    return slr::fail(SLR_ERR_WORKSPACE,
                     "slr_lrs_linear_forward_noalloc: " + std::to_string(M) + " tokens need " +
                         std::to_string(need) + " bytes of scratch, above the built-in " +
                         std::to_string(kScratchBytes) +
                         " bytes; use fewer tokens per call or slr_lrs_linear_forward with a workspace");
  void* ws = nullptr;
  if (need > 0) {
    int rc = scratch_address(&ws);
    if (rc) return rc;
  }
  return slr_lrs_linear_forward(layer, x, ldx, y, ldy, M, ws, need > 0 ? kScratchBytes : 0, stream);
}
