// Small-token-batch path (decode-sized M), 16-bit dtypes, mma.sync tensor
// cores with tokens on the MMA's N side, so a batch of 1..8 tokens costs one
// n8 tile and the weights stream from HBM exactly once.
//
//   h_small_kernel      H[M, ldh] = x · Bᵀ (rounded to the I/O dtype): split-K
//                       over the CTAs, partial sums reduced deterministically
//                       by the last CTA of each 16-row tile (fixed order).
//   mma_rowblock_kernel one CTA per (block-row, <=64 tokens): a producer warp
//                       streams the block-row's BSR values (contiguous rows of
//                       the [nnz*bq, bp] view) and, for the fused layer, its
//                       rows of A through a 4-stage TMA/mbarrier ring; eight
//                       consumer warps take ldmatrix fragments and run
//                       m16n8k16 MMAs; the epilogue adds bias (fused) or the
//                       previous `out` (in-place operator) and stores once.
//
// Reference counterparts: the GPU kernel _bsr_body
// (ssalaad/tilelang_sparse/addmm_inplace.py:41-82: acc = out; acc += x_tile ·
// values[j] over the row's blocks) and the two F.linear calls plus bias of
// _LRSLinearLRBlockCUDA.forward (ssalaad/efficient/ls_linear.py:124-137).
#include <algorithm>

#include "internal.hpp"

namespace slr {
namespace {

__device__ unsigned g_status_mma = 0;

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr int kStageBytes = 16384;

struct MmaArgs {
  const void* x;
  void* y;
  const void* H;
  const void* bias;
  const int32_t* crow;
  const int32_t* col;
  const int32_t* rows;
  int64_t M, K, N, ldh, ldx, ldy;
  int r, bq, rb, kc;
};

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return *static_cast<const uint32_t*>(p);
}
__device__ __forceinline__ uint32_t ldg_u32(const void* p) {
  return __ldg(static_cast<const unsigned int*>(p));
}

template <int BP, int NT, typename TI, int MODE>
__global__ void __launch_bounds__(kThreads)
    mma_rowblock_kernel(const __grid_constant__ CUtensorMap tm_vals,
                        const __grid_constant__ CUtensorMap tm_A, const MmaArgs a) {
  constexpr int MT = BP / 16;              // 16-feature m-tiles
  constexpr int KG = kConsumerWarps / MT;  // k-groups splitting the k-steps
  constexpr int TT = 8 * NT;               // tokens per CTA
  constexpr int RWV = BP * 2;              // bytes per values row
  static_assert(MT >= 1 && KG >= 1 && KG * MT == kConsumerWarps, "BP must be 16, 32 or 64");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* red = reinterpret_cast<float*>(smem + kStages * kStageBytes);  // [KG][BP][TT]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + KG * BP * TT);
  uint64_t* empty = full + kStages;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int br = a.rows ? a.rows[blockIdx.x] : int(blockIdx.x);
  const int64_t t0 = int64_t(blockIdx.y) * TT;
  const int jb0 = a.crow ? a.crow[br] : 0;
  const int jb1 = a.crow ? a.crow[br + 1] : 0;
  const int rows_sp = (jb1 - jb0) * a.bq;
  const int n_sp = (rows_sp + a.rb - 1) / a.rb;
  const int n_lr = MODE == MODE_FUSED ? (a.r + a.kc - 1) / a.kc : 0;
  const int n_total = n_sp + n_lr;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (n_sp) tma_prefetch_desc(&tm_vals);
      if (n_lr) tma_prefetch_desc(&tm_A);
      for (int s = 0; s < n_total; ++s) {
        const int slot = s % kStages;
        if (!mbar_wait(&empty[slot], ((s / kStages) & 1) ^ 1)) {
          atomicOr(&g_status_mma, SLR_TIMEOUT_BIT);
          s_abort = 1;
          break;
        }
        uint8_t* dst = smem + slot * kStageBytes;
        if (s < n_sp) {
          mbar_arrive_expect_tx(&full[slot], uint32_t(a.rb * RWV));
          tma_load_2d(dst, &tm_vals, 0, jb0 * a.bq + s * a.rb, &full[slot]);
        } else {
          mbar_arrive_expect_tx(&full[slot], uint32_t(BP * a.kc * 2));
          tma_load_2d(dst, &tm_A, (s - n_sp) * a.kc, br * BP, &full[slot]);
        }
      }
    }
  } else {
    // ----------------------------------------------------------- consumers
    const int mt = warp % MT, kg = warp / MT;
    const int g = lane >> 2, tig = lane & 3;
    const int lj = lane >> 3, li = lane & 7;
    const TI* __restrict__ x = static_cast<const TI*>(a.x);
    const TI* H = static_cast<const TI*>(a.H);
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    bool waited_primary = false;

    for (int s = 0; s < n_total; ++s) {
      const int slot = s % kStages;
      if (!mbar_wait(&full[slot], (s / kStages) & 1)) {
        atomicOr(&g_status_mma, SLR_TIMEOUT_BIT);
        s_abort = 1;
        break;
      }
      const uint32_t base = smem_u32(smem + slot * kStageBytes);
      if (s < n_sp) {
        const int steps = min(a.rb, rows_sp - s * a.rb) >> 4;
        for (int kk = kg; kk < steps; kk += KG) {
          const int q = s * a.rb + 16 * kk;
          const int jb = q / a.bq;
          const int kin = q - jb * a.bq;
          const int64_t xk = int64_t(__ldg(a.col + jb0 + jb)) * a.bq + kin;
          uint32_t af[4];
          ldsm_x4_trans(base + swz_offset(16 * kk + (lj >> 1) * 8 + li, 2 * mt + (lj & 1), RWV),
                        af[0], af[1], af[2], af[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int64_t t = t0 + 8 * nt + g;
            uint32_t b0 = 0, b1 = 0;
            if (t < a.M) {
              const TI* xr = x + t * a.ldx + xk + 2 * tig;
              b0 = ldg_u32(xr);
              b1 = ldg_u32(xr + 8);
            }
            mma16816<TI>::run(acc[nt], af, b0, b1);
          }
        }
      } else {
        if (!waited_primary) {
          pdl_wait_primary();  // H is written by the preceding kernel
          waited_primary = true;
        }
        const int l = s - n_sp;
        const int steps = a.kc >> 4;
        for (int kk = kg; kk < steps; kk += KG) {
          const int rho = l * a.kc + 16 * kk;
          if (rho >= a.r) break;
          uint32_t af[4];
          ldsm_x4(base + swz_offset(16 * mt + (lj & 1) * 8 + li, 2 * kk + (lj >> 1), a.kc * 2),
                  af[0], af[1], af[2], af[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int64_t t = t0 + 8 * nt + g;
            uint32_t b0 = 0, b1 = 0;
            if (t < a.M) {
              const TI* hr = H + t * a.ldh + rho + 2 * tig;
              b0 = ld_u32(hr);
              b1 = ld_u32(hr + 8);
            }
            mma16816<TI>::run(acc[nt], af, b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // accumulators -> red[kg][feature][token]
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = 16 * mt + g + ((e & 2) ? 8 : 0);
        const int t = 8 * nt + 2 * tig + (e & 1);
        red[(kg * BP + m) * TT + t] = acc[nt][e];
      }
  }
  __syncthreads();
  if (s_abort) return;

  // ------------------------------------------------------------- epilogue
  TI* __restrict__ y = static_cast<TI*>(a.y);
  const TI* __restrict__ bias = static_cast<const TI*>(a.bias);
  for (int idx = threadIdx.x; idx < BP * TT; idx += kThreads) {
    const int n = idx % BP, t = idx / BP;
    const int64_t tok = t0 + t;
    if (tok >= a.M) continue;
    float v = 0.f;
#pragma unroll
    for (int k = 0; k < KG; ++k) v += red[(k * BP + n) * TT + t];
    const int64_t gi = tok * a.ldy + int64_t(br) * BP + n;
    if (MODE == MODE_ADDMM) {
      v = to_f(y[gi]) + v;
    } else if (bias != nullptr) {
      v = v + to_f(bias[int64_t(br) * BP + n]);
    }
    y[gi] = from_f<TI>(v);
  }
}

// ------------------------------------------------------------ h_small --

struct HArgs {
  const void* x;
  const void* B;
  void* H;
  float* part;
  unsigned* counters;
  int64_t M, K, ldx, kchunk;
  int r, ldh, ks, rt;
};

__device__ __forceinline__ uint4 ldg_u128(const void* p) {
  return __ldg(static_cast<const uint4*>(p));
}

// One CTA (4 warps) = 16 rows of B x one K-chunk x 8*NT tokens.  Each lane
// loads 16 contiguous bytes of a B row and of an x row per 32-wide k slice
// and feeds them to two m16n8k16 MMAs; both operands use the same k order
// inside the slice, which leaves the dot product unchanged.
template <int NT, typename TI>
__global__ void __launch_bounds__(128) h_small_kernel(const HArgs a) {
  pdl_launch_dependents();
  constexpr int TT = 8 * NT;
  __shared__ float red[4][16][TT];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int rt = blockIdx.x, ks = blockIdx.y, tc = blockIdx.z;
  const int rho0 = 16 * rt;
  const int64_t t0 = int64_t(tc) * TT;
  const int64_t kb = int64_t(ks) * a.kchunk;
  const int64_t ke = min(a.K, kb + a.kchunk);
  const TI* __restrict__ x = static_cast<const TI*>(a.x);
  const TI* __restrict__ B = static_cast<const TI*>(a.B);
  const bool v0 = rho0 + g < a.r, v1 = rho0 + g + 8 < a.r;
  const TI* B0 = B + int64_t(rho0 + g) * a.K;
  const TI* B1 = B + int64_t(rho0 + g + 8) * a.K;

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  for (int64_t k = kb + 32 * warp; k < ke; k += 128) {
    const int64_t kk = k + 8 * tig;
    const bool kin = kk < ke;
    const uint4 z = make_uint4(0, 0, 0, 0);
    const uint4 A0 = (v0 && kin) ? ldg_u128(B0 + kk) : z;
    const uint4 A1 = (v1 && kin) ? ldg_u128(B1 + kk) : z;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int64_t t = t0 + 8 * nt + g;
      const uint4 X = (t < a.M && kin) ? ldg_u128(x + t * a.ldx + kk) : z;
      const uint32_t s0[4] = {A0.x, A1.x, A0.y, A1.y};
      const uint32_t s1[4] = {A0.z, A1.z, A0.w, A1.w};
      mma16816<TI>::run(acc[nt], s0, X.x, X.y);
      mma16816<TI>::run(acc[nt], s1, X.z, X.w);
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      red[warp][g + ((e & 2) ? 8 : 0)][8 * nt + 2 * tig + (e & 1)] = acc[nt][e];
  __syncthreads();

  TI* __restrict__ H = static_cast<TI*>(a.H);
  if (a.ks == 1) {
    for (int idx = threadIdx.x; idx < 16 * TT; idx += 128) {
      const int m = idx % 16, t = idx / 16;
      const float v = ((red[0][m][t] + red[1][m][t]) + red[2][m][t]) + red[3][m][t];
      if (t0 + t < a.M) H[(t0 + t) * a.ldh + rho0 + m] = from_f<TI>(v);
    }
    return;
  }
  // Split-K: publish this CTA's partial, the last CTA of the tile reduces.
  const int tile = tc * a.rt + rt;
  float* part = a.part + size_t(tile) * a.ks * 16 * TT;
  for (int idx = threadIdx.x; idx < 16 * TT; idx += 128) {
    const int m = idx % 16, t = idx / 16;
    part[size_t(ks) * 16 * TT + idx] = ((red[0][m][t] + red[1][m][t]) + red[2][m][t]) + red[3][m][t];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[tile], 1u);
    s_last = prev == unsigned(a.ks - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < 16 * TT; idx += 128) {
    const int m = idx % 16, t = idx / 16;
    float v = 0.f;
    for (int k = 0; k < a.ks; ++k) v += __ldcg(part + size_t(k) * 16 * TT + idx);
    if (t0 + t < a.M) H[(t0 + t) * a.ldh + rho0 + m] = from_f<TI>(v);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;  // ready for the next call
}

template <typename TI>
int launch_h_small_t(const HArgs& a, int tt, dim3 grid, cudaStream_t s) {
  switch (tt) {
    case 8: h_small_kernel<1, TI><<<grid, 128, 0, s>>>(a); break;
    case 16: h_small_kernel<2, TI><<<grid, 128, 0, s>>>(a); break;
    case 32: h_small_kernel<4, TI><<<grid, 128, 0, s>>>(a); break;
    default: h_small_kernel<8, TI><<<grid, 128, 0, s>>>(a); break;
  }
  SLR_CHECK_LAUNCH("h_small_kernel");
  return SLR_OK;
}

int pick_tt(int64_t M) {
  if (M <= 8) return 8;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  return 64;
}

template <int BP, int NT, typename TI, int MODE>
int launch_rowblock_inst(const CUtensorMap& tv, const CUtensorMap& ta, const MmaArgs& k,
                         dim3 grid, bool pdl, cudaStream_t s) {
  constexpr int TT = 8 * NT;
  constexpr int KG = kConsumerWarps / (BP / 16);
  const size_t smem = 1024 + kStages * kStageBytes + sizeof(float) * KG * BP * TT + 2 * kStages * 8;
  auto kern = mma_rowblock_kernel<BP, NT, TI, MODE>;
  SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tv, ta, k));
  return SLR_OK;
}

template <int BP, typename TI, int MODE>
int launch_rowblock_nt(const CUtensorMap& tv, const CUtensorMap& ta, const MmaArgs& k,
                       int tt, unsigned nrows, bool pdl, cudaStream_t s) {
  const dim3 grid(nrows, unsigned(ceil_div(k.M, tt)));
  switch (tt) {
    case 8: return launch_rowblock_inst<BP, 1, TI, MODE>(tv, ta, k, grid, pdl, s);
    case 16: return launch_rowblock_inst<BP, 2, TI, MODE>(tv, ta, k, grid, pdl, s);
    case 32: return launch_rowblock_inst<BP, 4, TI, MODE>(tv, ta, k, grid, pdl, s);
    default: return launch_rowblock_inst<BP, 8, TI, MODE>(tv, ta, k, grid, pdl, s);
  }
}

template <typename TI, int MODE>
int launch_rowblock_bp(const CUtensorMap& tv, const CUtensorMap& ta, const MmaArgs& k, int bp,
                       int tt, unsigned nrows, bool pdl, cudaStream_t s) {
  switch (bp) {
    case 16: return launch_rowblock_nt<16, TI, MODE>(tv, ta, k, tt, nrows, pdl, s);
    case 32: return launch_rowblock_nt<32, TI, MODE>(tv, ta, k, tt, nrows, pdl, s);
    case 64: return launch_rowblock_nt<64, TI, MODE>(tv, ta, k, tt, nrows, pdl, s);
    default: return fail(SLR_ERR_UNSUPPORTED, "mma path: block_p must be 16, 32 or 64");
  }
}

}  // namespace

HSmallPlan plan_h_small(int64_t M, int64_t K, int64_t ldh) {
  HSmallPlan p;
  p.tt = pick_tt(M);
  p.rt = int(ldh / 16);
  p.tc = int(ceil_div(std::max<int64_t>(M, 1), p.tt));
  const int64_t base = int64_t(p.rt) * p.tc;
  const int64_t want = std::max<int64_t>(1, ceil_div(2 * 148, std::max<int64_t>(base, 1)));
  const int64_t max_split = std::max<int64_t>(1, ceil_div(K, 128));
  const int64_t ks = std::min(want, max_split);
  p.kchunk = round_up(ceil_div(K, ks), 128);
  p.ks = int(ceil_div(K, p.kchunk));
  if (p.ks < 1) p.ks = 1;
  p.part_floats = p.ks > 1 ? size_t(base) * p.ks * 16 * p.tt : 0;
  p.counters = p.ks > 1 ? size_t(base) : 0;
  return p;
}

int launch_h_small(const void* x, int64_t ldx, const void* B, void* H, float* part, unsigned* counters,
                   int64_t M, int64_t K, int64_t r, int64_t ldh, const HSmallPlan& plan,
                   int dtype, cudaStream_t s) {
  if (M <= 0 || ldh <= 0) return SLR_OK;
  HArgs a{x, B, H, part, counters, M, K, ldx, plan.kchunk, int(r), int(ldh), plan.ks, plan.rt};
  const dim3 grid(unsigned(plan.rt), unsigned(plan.ks), unsigned(plan.tc));
  if (dtype == SLR_BF16) return launch_h_small_t<__nv_bfloat16>(a, plan.tt, grid, s);
  if (dtype == SLR_F16) return launch_h_small_t<__half>(a, plan.tt, grid, s);
  return fail(SLR_ERR_UNSUPPORTED_DTYPE, "h_small: 16-bit dtypes only");
}

bool mma_rowblock_supported(int bp, int bq, int64_t K, int64_t r) {
  if (bp != 16 && bp != 32 && bp != 64) return false;
  if (bq % 16 != 0 || bq <= 0) return false;
  if (K % 8 != 0) return false;
  if (r != 0 && (r % 8 != 0 || r < 16)) return false;
  return true;
}

int launch_mma_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s) {
  if (a.nrows <= 0 || a.M <= 0) return SLR_OK;
  const int bp = a.bp;
  MmaArgs k{a.x, a.y, a.H, a.bias, a.crow, a.col, a.rows, a.M, a.K, a.N, a.ldh, a.ldx, a.ldy,
            int(a.r), a.bq, 0, 0};
  k.rb = std::min(256, kStageBytes / (bp * 2));
  k.kc = a.r >= 64 ? 64 : (a.r >= 32 ? 32 : 16);
  CUtensorMap tv{}, ta{};
  int rc;
  if (a.crow != nullptr && a.nnz > 0) {
    rc = make_tmap_2d(&tv, a.values, a.dtype, uint64_t(bp), uint64_t(a.nnz) * a.bq, uint64_t(bp) * 2,
                      uint32_t(bp), uint32_t(k.rb));
    if (rc) return rc;
  } else {
    k.crow = nullptr;
  }
  if (a.mode == MODE_FUSED && a.r > 0) {
    rc = make_tmap_2d(&ta, a.A, a.dtype, uint64_t(a.r), uint64_t(a.N), uint64_t(a.r) * 2,
                      uint32_t(k.kc), uint32_t(bp));
    if (rc) return rc;
  } else {
    k.r = 0;
  }
  const int tt = pick_tt(a.M);
  const unsigned nrows = unsigned(a.nrows);
  if (a.dtype == SLR_BF16) {
    return a.mode == MODE_ADDMM
               ? launch_rowblock_bp<__nv_bfloat16, MODE_ADDMM>(tv, ta, k, bp, tt, nrows, pdl, s)
               : launch_rowblock_bp<__nv_bfloat16, MODE_FUSED>(tv, ta, k, bp, tt, nrows, pdl, s);
  }
  if (a.dtype == SLR_F16) {
    return a.mode == MODE_ADDMM ? launch_rowblock_bp<__half, MODE_ADDMM>(tv, ta, k, bp, tt, nrows, pdl, s)
                                : launch_rowblock_bp<__half, MODE_FUSED>(tv, ta, k, bp, tt, nrows, pdl, s);
  }
  return fail(SLR_ERR_UNSUPPORTED_DTYPE, "mma path: 16-bit dtypes only");
}

int read_and_clear_status_mma(unsigned* out) {
  unsigned v = 0, zero = 0;
  SLR_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status_mma, sizeof(v)));
  if (v) SLR_CHECK_CUDA(cudaMemcpyToSymbol(g_status_mma, &zero, sizeof(zero)));
  *out = v;
  return SLR_OK;
}

}  // namespace slr
