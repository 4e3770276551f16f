// Shared device/host helpers for libslr_b200: element types, error plumbing,
// PTX wrappers (mbarrier, TMA, ldmatrix, mma.sync, griddepcontrol) and the
// TMA tensor-map encoder.  sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/slr_b200.h"

namespace slr {

// ------------------------------------------------------------ errors ----

// Thread-local message for slr_last_error(); set by fail().
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define SLR_CHECK_CUDA(expr)                          \
  do {                                                \
    cudaError_t e__ = (expr);                         \
    if (e__ != cudaSuccess) return ::slr::cuda_fail(e__, #expr); \
  } while (0)

#define SLR_CHECK_LAUNCH(what)                        \
  do {                                                \
    cudaError_t e__ = cudaGetLastError();             \
    if (e__ != cudaSuccess) return ::slr::cuda_fail(e__, what); \
  } while (0)

// Device status word (one per translation unit that waits on the device);
// a bounded wait that gives up ORs SLR_TIMEOUT_BIT into it.
constexpr unsigned SLR_TIMEOUT_BIT = 1u;
// 2 s of %globaltimer: far above any legitimate wait inside one launch.
constexpr unsigned long long SLR_WAIT_LIMIT_NS = 2000000000ull;

// ------------------------------------------------------ element types ----

template <typename T> struct dtype_of;
template <> struct dtype_of<float> { static constexpr int value = SLR_F32; };
template <> struct dtype_of<__half> { static constexpr int value = SLR_F16; };
template <> struct dtype_of<__nv_bfloat16> { static constexpr int value = SLR_BF16; };

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

inline size_t dtype_size(int dtype) { return dtype == SLR_F32 ? 4 : 2; }

// ----------------------------------------------------------- PTX: misc ----

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and (in that kernel) wait for this one's memory to be visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ------------------------------------------------- PTX: cross-GPU signals ----
// Counters that other GPUs add to through CUDA IPC mappings over NVLink: the
// writer release-adds at system scope, the owner acquire-loads.

__device__ __forceinline__ void red_add_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }

// Barrier among `threads` threads (whole warps) of the CTA on hardware barrier `id` (1..15).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Spin until p[q] >= target (eq: == target) for every q < n (words of other
// ranks), at most limit_ns in all; false on timeout.
__device__ __forceinline__ bool wait_words(const unsigned long long* p, int n, unsigned long long target,
                                           unsigned long long limit_ns, bool eq) {
  const unsigned long long t0 = globaltimer_ns();
  for (int q = 0; q < n; ++q) {
    while (true) {
      const unsigned long long v = ld_acquire_sys(p + q);
      if (eq ? v == target : v >= target) break;
      if (globaltimer_ns() - t0 > limit_ns) return false;
      __nanosleep(100);
    }
  }
  return true;
}

// The k-th work item of worker p of P when the items, listed heaviest first,
// are dealt in snake order (0..P-1, then P-1..0, ...): every round hands each
// worker one item, and the worker that got the heaviest item of a round gets
// the lightest of the next, which evens out the persistent schedule's tail.
__device__ __forceinline__ int snake_item(int k, int p, int P) { return k * P + ((k & 1) ? P - 1 - p : p); }

// --------------------------------------------------------- PTX: mbarrier ----

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of the phase (about a third of try_wait's latency when
// the phase has already completed).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity` to complete.  Returns false after
// SLR_WAIT_LIMIT_NS; the caller then records SLR_TIMEOUT_BIT and unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_test_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > SLR_WAIT_LIMIT_NS) return false;
  }
}

// Warp-wide bounded wait (all 32 lanes call it): lane 0 polls, sleeping
// `sleep_ns` between polls when nonzero, so a waiting warp does not flood the
// shared-memory pipe with 32 polls per round; then every lane acquires the
// completed phase once.  Returns false after SLR_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, uint32_t sleep_ns) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) {
    ok = 0;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
      if (mbar_try_wait(bar, parity)) {
        ok = 1;
        break;
      }
      if (globaltimer_ns() - t0 > SLR_WAIT_LIMIT_NS) break;
      if (sleep_ns) __nanosleep(sleep_ns);
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok != 0;
}

// ------------------------------------------------------------- PTX: TMA ----

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// Pull one box of a 2-D tensor into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* tmap, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(c0), "r"(c1)
               : "memory");
}
// 2-D tiled load of one box into shared memory; completes `bytes` on `bar`.
// c0 is the innermost (contiguous) coordinate in elements.
// Tiled TMA store shared -> global (this GPU's memory or a peer's through a
// CUDA IPC mapping), tracked in the issuing thread's bulk groups.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The thread's bulk stores have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// The thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t c0,
                                            int32_t c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (both addresses 16-byte aligned, bytes a
// multiple of 16); completes `bytes` on `bar`.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------- PTX: ldmatrix / mma ----

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct mma16816;
template <> struct mma16816<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct mma16816<__half> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a shared tile whose
// rows are `row_bytes` (32, 64 or 128) long and that TMA filled with the
// matching swizzle (SWIZZLE_32B/64B/128B): the chunk index is XORed with
// address bits [7, 7+B) where row_bytes = 16 << B.  Tile base 1024-aligned.
__device__ __forceinline__ uint32_t swz_offset(int row, int chunk, int row_bytes) {
  const int B = row_bytes == 128 ? 3 : (row_bytes == 64 ? 2 : 1);
  const int x = (row >> (3 - B)) & ((1 << B) - 1);
  return static_cast<uint32_t>(row * row_bytes + ((chunk ^ x) << 4));
}

// ------------------------------------------------------- host: tensor maps ----

// Encodes a 2-D row-major tensor map: `inner` elements per row (contiguous),
// `outer` rows `row_stride_bytes` apart, box of box_inner x box_outer,
// swizzle chosen from the box row size (32/64/128 bytes) or none.
int make_tmap_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);

}  // namespace slr
