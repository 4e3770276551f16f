// Dense -> BSR conversion on the GPU, bit-exact with the reference's
// dense_to_bsr (ssalaad/efficient/artifact.py:20-37):
//   mask[i, j] = sum(|S block (i, j)|) > 0      (:27-29)
//   crow = [0, cumsum(row counts)] as int64     (:30-33)
//   col  = nonzero(mask)[:, 1], row-major order (:34-35)
//   values = blocks[mask], bits copied unchanged (:36)
// For IEEE values "sum of |s| > 0" equals "some element is nonzero and none
// is NaN" (a sum of non-negative terms is 0 only if all are 0; a NaN term
// makes the sum NaN, which compares false), so the mask is computed from the
// bit patterns and no summation order is involved.
//
// Also: the device-side BSR validity check used once at layer construction.
#include "internal.hpp"

namespace slr {
namespace {

// Per element: bit 0 = nonzero (not +-0, not NaN), bit 1 = NaN.
__device__ __forceinline__ unsigned classify(uint32_t bits, int dtype) {
  if (dtype == SLR_F32) {
    const uint32_t mag = bits & 0x7fffffffu;
    if (mag > 0x7f800000u) return 2u;
    return mag ? 1u : 0u;
  }
  const uint32_t mag = bits & 0x7fffu;
  const uint32_t inf = dtype == SLR_BF16 ? 0x7f80u : 0x7c00u;
  if (mag > inf) return 2u;
  return mag ? 1u : 0u;
}

__device__ __forceinline__ uint32_t load_bits(const void* S, int64_t idx, int dtype) {
  if (dtype == SLR_F32) return static_cast<const uint32_t*>(S)[idx];
  return static_cast<const uint16_t*>(S)[idx];
}

// One warp per block: classify its bp*bq elements.
__global__ void mask_kernel(const void* __restrict__ S, int64_t m, int64_t bp, int64_t bq,
                            int64_t rb, int64_t cb, int dtype, uint8_t* __restrict__ mask) {
  const int64_t wid = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= rb * cb) return;
  const int64_t i = wid / cb, j = wid % cb;
  unsigned f = 0;
  for (int64_t e = lane; e < bp * bq; e += 32) {
    const int64_t a = e / bq, b = e % bq;
    f |= classify(load_bits(S, (i * bp + a) * m + j * bq + b, dtype), dtype);
  }
  f = __reduce_or_sync(0xffffffffu, f);
  if (lane == 0) mask[wid] = (f == 1u) ? 1 : 0;
}

// Single CTA: counts per block-row and their exclusive scan -> crow (int64).
__global__ void crow_kernel(const uint8_t* __restrict__ mask, int64_t rb, int64_t cb,
                            int64_t* __restrict__ crow) {
  __shared__ int64_t carry;
  __shared__ int64_t warp_sums[32];
  if (threadIdx.x == 0) {
    carry = 0;
    crow[0] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < rb; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    int64_t c = 0;
    if (i < rb)
      for (int64_t j = 0; j < cb; ++j) c += mask[i * cb + j];
    // inclusive scan within the warp, then across warps
    int64_t v = c;
    for (int d = 1; d < 32; d <<= 1) {
      const int64_t o = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= d) v += o;
    }
    if (lane == 31) warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int64_t w = lane < int(blockDim.x >> 5) ? warp_sums[lane] : 0;
      for (int d = 1; d < 32; d <<= 1) {
        const int64_t o = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += o;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int64_t prefix = carry + (warp ? warp_sums[warp - 1] : 0) + v;
    if (i < rb) crow[i + 1] = prefix;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = prefix;
    __syncthreads();
  }
}

// One warp per block-row: compact the mask row into col[] in column order.
__global__ void col_kernel(const uint8_t* __restrict__ mask, int64_t rb, int64_t cb,
                           const int64_t* __restrict__ crow, int64_t* __restrict__ col) {
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= rb) return;
  int64_t pos = crow[i];
  for (int64_t j0 = 0; j0 < cb; j0 += 32) {
    const int64_t j = j0 + lane;
    const bool live = j < cb && mask[i * cb + j];
    const unsigned bal = __ballot_sync(0xffffffffu, live);
    if (live) col[pos + __popc(bal & ((1u << lane) - 1u))] = j;
    pos += __popc(bal);
  }
}

// One CTA per stored block: copy its bits, optionally transposed.
template <typename W>
__global__ void values_kernel(const W* __restrict__ S, int64_t m, int64_t bp, int64_t bq,
                              int64_t rb, const int64_t* __restrict__ crow,
                              const int64_t* __restrict__ col, W* __restrict__ values,
                              bool transpose) {
  const int64_t p = blockIdx.x;
  // block-row of entry p: last i with crow[i] <= p
  int64_t lo = 0, hi = rb;
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (crow[mid] <= p) lo = mid; else hi = mid;
  }
  const int64_t i = lo, j = col[p];
  W* dst = values + p * bp * bq;
  for (int64_t e = threadIdx.x; e < bp * bq; e += blockDim.x) {
    if (!transpose) {
      const int64_t a = e / bq, b = e % bq;  // dst [bp][bq]
      dst[e] = S[(i * bp + a) * m + j * bq + b];
    } else {
      const int64_t b = e / bp, a = e % bp;  // dst [bq][bp]
      dst[e] = S[(i * bp + a) * m + j * bq + b];
    }
  }
}

// BSR validity: flag |= 1 on any violation.
__global__ void validate_kernel(const int32_t* __restrict__ crow, int64_t NB,
                                const int32_t* __restrict__ col, int64_t nnz, int64_t nbk,
                                const int32_t* __restrict__ active, int64_t active_nb,
                                int* __restrict__ flag) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t == 0 && (crow[0] != 0 || crow[NB] != nnz)) atomicOr(flag, 1);
  for (int64_t i = t; i < NB; i += stride)
    if (crow[i + 1] < crow[i]) atomicOr(flag, 1);
  for (int64_t p = t; p < nnz; p += stride)
    if (col[p] < 0 || col[p] >= nbk) atomicOr(flag, 1);
  for (int64_t a = t; a < active_nb; a += stride) {
    const int32_t r = active[a];
    if (r < 0 || r >= NB || crow[r + 1] <= crow[r]) atomicOr(flag, 1);
  }
}

}  // namespace

int launch_bsr_mask(const void* S, int64_t n, int64_t m, int64_t bp, int64_t bq, int dtype,
                    uint8_t* mask, int64_t* crow, cudaStream_t s) {
  const int64_t rb = n / bp, cb = m / bq;
  const int64_t warps = rb * cb;
  if (warps > 0) {
    mask_kernel<<<unsigned(ceil_div(warps * 32, 256)), 256, 0, s>>>(S, m, bp, bq, rb, cb, dtype, mask);
    SLR_CHECK_LAUNCH("mask_kernel");
  }
  crow_kernel<<<1, 1024, 0, s>>>(mask, rb, cb, crow);
  SLR_CHECK_LAUNCH("crow_kernel");
  return SLR_OK;
}

int launch_bsr_fill(const void* S, int64_t n, int64_t m, int64_t bp, int64_t bq, int dtype,
                    const uint8_t* mask, const int64_t* crow, int64_t* col, void* values,
                    bool transpose, cudaStream_t s) {
  const int64_t rb = n / bp, cb = m / bq;
  if (rb == 0) return SLR_OK;
  col_kernel<<<unsigned(ceil_div(rb * 32, 256)), 256, 0, s>>>(mask, rb, cb, crow, col);
  SLR_CHECK_LAUNCH("col_kernel");
  // nnz is crow[rb]; read it here so the grid covers exactly the stored blocks.
  int64_t nnz = 0;
  SLR_CHECK_CUDA(cudaMemcpyAsync(&nnz, crow + rb, sizeof(nnz), cudaMemcpyDeviceToHost, s));
  SLR_CHECK_CUDA(cudaStreamSynchronize(s));
  if (nnz == 0) return SLR_OK;
  if (nnz > 0x7fffffffLL) return fail(SLR_ERR_UNSUPPORTED, "dense_to_bsr: more than 2^31 blocks");
  if (dtype == SLR_F32)
    values_kernel<uint32_t><<<unsigned(nnz), 256, 0, s>>>(static_cast<const uint32_t*>(S), m, bp, bq, rb,
                                                          crow, col, static_cast<uint32_t*>(values), transpose);
  else
    values_kernel<uint16_t><<<unsigned(nnz), 256, 0, s>>>(static_cast<const uint16_t*>(S), m, bp, bq, rb,
                                                          crow, col, static_cast<uint16_t*>(values), transpose);
  SLR_CHECK_LAUNCH("values_kernel");
  return SLR_OK;
}

int launch_validate_bsr(const int32_t* crow, int64_t NB, const int32_t* col, int64_t nnz,
                        int64_t nbk, const int32_t* active, int64_t active_nb, int* flag,
                        cudaStream_t s) {
  validate_kernel<<<148, 256, 0, s>>>(crow, NB, col, nnz, nbk, active, active_nb, flag);
  SLR_CHECK_LAUNCH("validate_kernel");
  return SLR_OK;
}

}  // namespace slr
