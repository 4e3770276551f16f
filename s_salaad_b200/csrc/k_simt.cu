// CUDA-core (FFMA) kernels.
//
// These carry the fp32 path, whose arithmetic restates the reference CPU layer
// (ssalaad/efficient/ls_linear.py:155-164 with the AVX2 kernel of
// ssalaad/cpu_sparse/bsr_addmm_avx2.cpp:67-140): the low-rank product in
// fp32, then per output element the chain of fused multiply-adds over the
// row's blocks in crow order and k ascending, starting from the low-rank value
// (or from `out` for the in-place operator), then the bias add.  They are also
// the generic fallback for 16-bit shapes the tensor-core kernels do not take
// (block sizes other than 16/32/64, odd ranks, unaligned pointers).
#include "internal.hpp"

namespace slr {
namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 8;  // k elements staged per step (block_q % 8 == 0)

// H[m, p] = sum_k x[m, k] * B[p, k] for p < r, 0 for r <= p < ldh.
template <typename TI, typename TH>
__global__ void __launch_bounds__(kThreads)
    simt_h_kernel(const TI* __restrict__ x, const TI* __restrict__ B, TH* __restrict__ H,
                  int64_t M, int64_t K, int64_t ldx, int64_t r, int64_t ldh) {
  __shared__ float xs[32][33];
  __shared__ float bs[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t m0 = int64_t(blockIdx.y) * 32, p0 = int64_t(blockIdx.x) * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t k0 = 0; k0 < K; k0 += 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = ty + 8 * i;
      const int64_t k = k0 + tx;
      xs[row][tx] = (m0 + row < M && k < K) ? to_f(x[(m0 + row) * ldx + k]) : 0.f;
      bs[row][tx] = (p0 + row < r && k < K) ? to_f(B[(p0 + row) * K + k]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float b = bs[tx][kk];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(xs[ty + 8 * i][kk], b, acc[i]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty + 8 * i, p = p0 + tx;
    if (m < M && p < ldh) H[m * ldh + p] = from_f<TH>(p < r ? acc[i] : 0.f);
  }
}

struct SimtArgs {
  const void* x;
  void* y;
  const void* H;
  int64_t ldh;
  const void* A;
  const void* bias;
  const int32_t* crow;
  const int32_t* col;
  const void* values;
  const int32_t* rows;
  int64_t M, K, N, r, ldx, ldy;
  int bp, bq, tm;
};

// One CTA = one block-row (bp output features) x tm tokens; <= 8 outputs per
// thread (tm * bp <= 2048).
template <typename TI, typename TH, int MODE>
__global__ void __launch_bounds__(kThreads) simt_rowblock_kernel(SimtArgs a) {
  extern __shared__ float sm[];
  const int tm = a.tm, bp = a.bp;
  float* xs = sm;                         // [tm][kChunk+1]
  float* ws = xs + tm * (kChunk + 1);     // [kChunk][bp]
  const int br = a.rows ? a.rows[blockIdx.x] : int(blockIdx.x);
  const int64_t m0 = int64_t(blockIdx.y) * tm;
  const TI* __restrict__ x = static_cast<const TI*>(a.x);
  TI* __restrict__ y = static_cast<TI*>(a.y);
  const int64_t col0 = int64_t(br) * bp;

  float acc[8];
  int om[8], on[8];
  bool ok[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int o = threadIdx.x + kThreads * i;
    om[i] = o / bp;
    on[i] = o - om[i] * bp;
    ok[i] = o < tm * bp && m0 + om[i] < a.M;
    acc[i] = 0.f;
    if (MODE == MODE_ADDMM && ok[i]) acc[i] = to_f(y[(m0 + om[i]) * a.ldy + col0 + on[i]]);
  }

  if (MODE == MODE_FUSED && a.r > 0) {
    // acc = sum_p H[m, p] * A[n, p], p ascending.
    const TH* __restrict__ H = static_cast<const TH*>(a.H);
    const TI* __restrict__ A = static_cast<const TI*>(a.A);
    float* hs = xs;                       // [tm][kChunk+1]
    float* as = ws;                       // [bp][kChunk+1]
    for (int64_t p0 = 0; p0 < a.r; p0 += kChunk) {
      for (int e = threadIdx.x; e < tm * kChunk; e += kThreads) {
        const int m = e / kChunk, kk = e % kChunk;
        hs[m * (kChunk + 1) + kk] =
            (m0 + m < a.M && p0 + kk < a.r) ? to_f(H[(m0 + m) * a.ldh + p0 + kk]) : 0.f;
      }
      for (int e = threadIdx.x; e < bp * kChunk; e += kThreads) {
        const int n = e / kChunk, kk = e % kChunk;
        as[n * (kChunk + 1) + kk] = (p0 + kk < a.r) ? to_f(A[(col0 + n) * a.r + p0 + kk]) : 0.f;
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (!ok[i]) continue;
        const float* hr = hs + om[i] * (kChunk + 1);
        const float* ar = as + on[i] * (kChunk + 1);
#pragma unroll
        for (int kk = 0; kk < kChunk; ++kk) acc[i] = fmaf(hr[kk], ar[kk], acc[i]);
      }
      __syncthreads();
    }
  }

  if (a.crow != nullptr) {
    // Sparse term in the reference's order: blocks in crow order, k ascending.
    const TI* __restrict__ vals = static_cast<const TI*>(a.values);
    const int j0 = a.crow[br], j1 = a.crow[br + 1];
    for (int ji = j0; ji < j1; ++ji) {
      const int64_t xc = int64_t(a.col[ji]) * a.bq;
      for (int k0 = 0; k0 < a.bq; k0 += kChunk) {
        for (int e = threadIdx.x; e < tm * kChunk; e += kThreads) {
          const int m = e / kChunk, kk = e % kChunk;
          xs[m * (kChunk + 1) + kk] = (m0 + m < a.M) ? to_f(x[(m0 + m) * a.ldx + xc + k0 + kk]) : 0.f;
        }
        const TI* vb = vals + (int64_t(ji) * a.bq + k0) * bp;
        for (int e = threadIdx.x; e < kChunk * bp; e += kThreads) ws[e] = to_f(vb[e]);
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (!ok[i]) continue;
          const float* xr = xs + om[i] * (kChunk + 1);
#pragma unroll
          for (int kk = 0; kk < kChunk; ++kk) acc[i] = fmaf(xr[kk], ws[kk * bp + on[i]], acc[i]);
        }
        __syncthreads();
      }
    }
  }

  const TI* __restrict__ bias = static_cast<const TI*>(a.bias);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (!ok[i]) continue;
    float v = acc[i];
    if (MODE == MODE_FUSED && bias != nullptr) v = v + to_f(bias[col0 + on[i]]);
    y[(m0 + om[i]) * a.ldy + col0 + on[i]] = from_f<TI>(v);
  }
}

template <typename TI, typename TH>
int launch_rowblock_t(const RowblockArgs& a, cudaStream_t s) {
  SimtArgs k{a.x, a.y, a.H, a.ldh, a.A, a.bias, a.crow, a.col, a.values, a.rows,
             a.M, a.K, a.N, a.r, a.ldx, a.ldy, a.bp, a.bq, 0};
  k.tm = int(std::max<int64_t>(1, std::min<int64_t>(32, 2048 / a.bp)));
  const size_t smem =
      sizeof(float) * (size_t(k.tm) * (kChunk + 1) + size_t(std::max(kChunk * a.bp, a.bp * (kChunk + 1))));
  const dim3 grid(unsigned(a.nrows), unsigned(ceil_div(a.M, k.tm)));
  if (grid.x == 0 || grid.y == 0) return SLR_OK;
  if (a.mode == MODE_ADDMM) {
    auto kern = simt_rowblock_kernel<TI, TH, MODE_ADDMM>;
    if (smem > 48 * 1024) SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    kern<<<grid, kThreads, smem, s>>>(k);
  } else {
    auto kern = simt_rowblock_kernel<TI, TH, MODE_FUSED>;
    if (smem > 48 * 1024) SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    kern<<<grid, kThreads, smem, s>>>(k);
  }
  SLR_CHECK_LAUNCH("simt_rowblock_kernel");
  return SLR_OK;
}

}  // namespace

int launch_simt_h(const void* x, int64_t ldx, const void* B, void* H, int64_t M, int64_t K, int64_t r,
                  int64_t ldh, int dtype, bool h_f32, cudaStream_t s) {
  const dim3 grid(unsigned(ceil_div(ldh, 32)), unsigned(ceil_div(M, 32)));
  if (grid.x == 0 || grid.y == 0) return SLR_OK;
  switch (dtype) {
    case SLR_F32:
      simt_h_kernel<float, float><<<grid, kThreads, 0, s>>>(
          static_cast<const float*>(x), static_cast<const float*>(B), static_cast<float*>(H), M, K, ldx, r, ldh);
      break;
    case SLR_F16:
      if (h_f32)
        simt_h_kernel<__half, float><<<grid, kThreads, 0, s>>>(
            static_cast<const __half*>(x), static_cast<const __half*>(B), static_cast<float*>(H), M, K, ldx, r, ldh);
      else
        simt_h_kernel<__half, __half><<<grid, kThreads, 0, s>>>(
            static_cast<const __half*>(x), static_cast<const __half*>(B), static_cast<__half*>(H), M, K, ldx, r, ldh);
      break;
    case SLR_BF16:
      if (h_f32)
        simt_h_kernel<__nv_bfloat16, float><<<grid, kThreads, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(B), static_cast<float*>(H), M, K, ldx, r, ldh);
      else
        simt_h_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, kThreads, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(B),
            static_cast<__nv_bfloat16*>(H), M, K, ldx, r, ldh);
      break;
    default:
      return fail(SLR_ERR_UNSUPPORTED_DTYPE, "simt_h: bad dtype");
  }
  SLR_CHECK_LAUNCH("simt_h_kernel");
  return SLR_OK;
}

int launch_simt_rowblock(const RowblockArgs& a, bool h_f32, cudaStream_t s) {
  if (a.bp <= 0 || a.bp > 2048) return fail(SLR_ERR_UNSUPPORTED, "simt path: block_p must be in [1, 2048]");
  switch (a.dtype) {
    case SLR_F32: return launch_rowblock_t<float, float>(a, s);
    case SLR_F16: return h_f32 ? launch_rowblock_t<__half, float>(a, s) : launch_rowblock_t<__half, __half>(a, s);
    case SLR_BF16:
      return h_f32 ? launch_rowblock_t<__nv_bfloat16, float>(a, s)
                   : launch_rowblock_t<__nv_bfloat16, __nv_bfloat16>(a, s);
    default: return fail(SLR_ERR_UNSUPPORTED_DTYPE, "simt_rowblock: bad dtype");
  }
}

}  // namespace slr
