// Multi-GPU plumbing of the fused all-gather: CUDA IPC mappings of the other
// ranks' buffers (so a kernel's epilogue can store its output tiles straight
// into every rank's y over NVLink) and the wait that ends a call.
//
// The reference runs on one device; this file has no reference counterpart.
// It replaces the NCCL all-gather of y (plus the column reassembly) that a
// block-row-sharded layer otherwise needs: each rank's tiles reach the peers
// while the kernel is still computing, and nothing is copied afterwards.
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "internal.hpp"

namespace slr {
namespace {

__device__ unsigned g_status_peer = 0;

// One thread: for a rank without rows of the layer, take part in the call
// (announce it, wait for the others, count an empty completion); then wait
// until every rank's stores into this rank's y are visible, check that no
// rank gave up during the call, and count the call.  Calls are numbered by
// this rank's own count (slot word kSigCalls).
__global__ void peer_wait_kernel(const PeerArgs p, int empty_shard) {
  if (threadIdx.x != 0) return;
  unsigned long long* me = p.my_sig;
  const unsigned long long call = *reinterpret_cast<volatile unsigned long long*>(me + kSigCalls) + 1;
  if (empty_shard) {
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < p.world) st_release_sys(p.sig[r] + kSigArrive + p.me, call);
    if (!wait_words(me + kSigArrive, p.world, call, p.wait_ns, true)) {
      atomicOr(&g_status_peer, SLR_TIMEOUT_BIT);
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < p.world) st_release_sys(p.sig[r] + kSigFail + p.me, call);
    }
    fence_sc_sys();
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < p.world) red_add_release_sys(p.sig[r] + kSigDone + p.me, kDonePerRank);
  }
  bool ok = wait_words(me + kSigDone, p.world, call * kDonePerRank, p.wait_ns, false);
  for (int q = 0; ok && q < p.world; ++q)
    if (ld_acquire_sys(me + kSigFail + q) == call) ok = false;
  if (!ok) atomicOr(&g_status_peer, SLR_TIMEOUT_BIT);
  *reinterpret_cast<volatile unsigned long long*>(me + kSigCalls) = call;
  __threadfence();
}

std::atomic<unsigned long long> g_wait_limit_ns{SLR_WAIT_LIMIT_NS};

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(p);
  });
  return fn;
}

// Imported allocations of this process: handle bytes -> (mapped base, users).
struct Mapping {
  void* base = nullptr;
  int users = 0;
};
std::mutex g_ipc_mu;
std::map<std::string, Mapping> g_ipc;

}  // namespace

unsigned long long peer_wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int launch_peer_wait(const PeerArgs& p, bool empty_shard, cudaStream_t s) {
  peer_wait_kernel<<<1, 32, 0, s>>>(p, empty_shard ? 1 : 0);
  SLR_CHECK_LAUNCH("peer_wait_kernel");
  return SLR_OK;
}

int read_and_clear_status_peer(unsigned* out) {
  unsigned v = 0, zero = 0;
  SLR_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status_peer, sizeof(v)));
  if (v) SLR_CHECK_CUDA(cudaMemcpyToSymbol(g_status_peer, &zero, sizeof(zero)));
  *out = v;
  return SLR_OK;
}

}  // namespace slr

using namespace slr;

extern "C" {

int slr_set_wait_limit_ns(uint64_t ns) {
  g_wait_limit_ns.store(ns > 0 ? ns : SLR_WAIT_LIMIT_NS, std::memory_order_relaxed);
  return SLR_OK;
}

int slr_ipc_export(const void* dev_ptr, void* handle, int64_t* offset) {
  if (!dev_ptr || !handle || !offset) return fail(SLR_ERR_INVALID_ARGUMENT, "slr_ipc_export: NULL argument");
  GetAddressRangeFn range = address_range_fn();
  if (!range) return fail(SLR_ERR_CUDA, "cuMemGetAddressRange unavailable from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  if (r != CUDA_SUCCESS)
    return fail(SLR_ERR_INVALID_ARGUMENT, "slr_ipc_export: not a device allocation (code " + std::to_string(int(r)) + ")");
  cudaIpcMemHandle_t h;
  SLR_CHECK_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(h) == SLR_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = int64_t(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return SLR_OK;
}

int slr_ipc_import(const void* handle, int64_t offset, void** dev_ptr) {
  if (!handle || !dev_ptr || offset < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "slr_ipc_import: bad argument");
  const std::string key(static_cast<const char*>(handle), SLR_IPC_HANDLE_BYTES);
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  Mapping& m = g_ipc[key];
  if (!m.base) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      g_ipc.erase(key);
      return cuda_fail(e, "cudaIpcOpenMemHandle");
    }
    m.base = base;
  }
  ++m.users;
  *dev_ptr = static_cast<char*>(m.base) + offset;
  return SLR_OK;
}

int slr_ipc_release(const void* handle) {
  if (!handle) return fail(SLR_ERR_INVALID_ARGUMENT, "slr_ipc_release: NULL handle");
  const std::string key(static_cast<const char*>(handle), SLR_IPC_HANDLE_BYTES);
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  auto it = g_ipc.find(key);
  if (it == g_ipc.end()) return fail(SLR_ERR_INVALID_ARGUMENT, "slr_ipc_release: handle not imported");
  if (--it->second.users > 0) return SLR_OK;
  void* base = it->second.base;
  g_ipc.erase(it);
  SLR_CHECK_CUDA(cudaIpcCloseMemHandle(base));
  return SLR_OK;
}

}  // extern "C"
