// Small-token-batch path (decode-sized M), 16-bit dtypes, mma.sync tensor
// cores with tokens on the MMA's N side, so a batch of 1..8 tokens costs one
// n8 tile and the weights stream from HBM exactly once.
//
//   h_small_kernel      H[M, ldh] = x · Bᵀ (rounded to the I/O dtype): split-K
//                       over the CTAs, partial sums reduced deterministically
//                       by the last CTA of each 16-row tile (fixed order).
//   mma_rowblock_kernel one CTA per (16 output features of a block-row, <=64
//                       tokens): a producer warp streams the 16-column slice of
//                       the row's BSR values, the x tiles at those blocks'
//                       columns, and (fused layer) the row's A rows and H tiles
//                       through a 6-stage TMA/mbarrier ring; eight consumer
//                       warps run m16n8k16 MMAs from shared memory only; the
//                       epilogue adds bias (fused) or the previous `out`
//                       (in-place operator) and stores once.
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
constexpr int kStages = 6;
constexpr int kFT = 16;  // output features per CTA (one m16 tile)
// Low-rank stage layout: A rows (16 x kc, at most 2 KB) at 0, H tile at 2 KB
// (1024-aligned for its swizzle).
constexpr uint32_t kHOff = 2048;

struct MmaArgs {
  void* y;
  const void* bias;
  const int32_t* crow;
  const int32_t* col;
  const int32_t* rows;
  int64_t M, N, ldy;
  int bp, bq, r, kc;   // kc: rank chunk per low-rank stage
  int sb;              // value blocks per sparse stage
  int ft_per_row;      // bp / 16
  int nrows;
};

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return *static_cast<const uint32_t*>(p);
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// One CTA = 16 output features (a column slice of one block-row) x 8*NT
// tokens.  Warp 8 is the producer: per sparse stage it TMA-loads the 16-column
// slice of `sb` consecutive value blocks of the row (one box) and, for each of
// those blocks, the x tile [tokens x bq] at that block's column (lane j reads
// col[] of block j and issues its x tiles); per low-rank stage the 16 rows of
// A and the H tile [tokens x kc].  Warps 0-7 split each stage's k16 steps, take
// ldmatrix fragments from shared memory only, and run m16n8k16 MMAs (features
// on M, tokens on N); partial sums are reduced across warps in a fixed order.
//
// Launched as a programmatic dependent (PDL): before griddepcontrol.wait the
// CTA touches weights only -- the value and A boxes of the first kStages
// stages go to shared memory, those of later stages to L2, bias to shared
// memory -- so a decode step streams its weights while the previous kernel
// finishes.  x, H and y are read or written only after the wait.
template <int NT, int KX, typename TI, int MODE>
__global__ void __launch_bounds__(kThreads)
    mma_rowblock_kernel(const __grid_constant__ CUtensorMap tm_vals, const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_A, const __grid_constant__ CUtensorMap tm_h,
                        const MmaArgs a) {
  constexpr int TT = 8 * NT;                 // tokens per CTA
  constexpr int XB = TT * KX * 2;            // one x sub-tile (tokens x KX columns)
  constexpr int RWX = KX * 2;                // x tile row bytes (its TMA swizzle width)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nsub = a.bq / KX;                            // x sub-tiles per block
  const uint32_t v_bytes = uint32_t(a.sb * a.bq * kFT * 2);   // values box of a stage
  const uint32_t v_slot = (v_bytes + 1023) & ~1023u;
  const uint32_t x_region = uint32_t(a.sb * nsub * XB);
  const uint32_t lr_bytes = uint32_t(kFT * a.kc * 2 + TT * a.kc * 2);
  uint32_t stage_bytes = v_slot + x_region;
  if (stage_bytes < kHOff + TT * a.kc * 2) stage_bytes = kHOff + TT * a.kc * 2;
  stage_bytes = (stage_bytes + 1023) & ~1023u;
  float* red = reinterpret_cast<float*>(smem + kStages * stage_bytes);  // [8][16][TT]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + kConsumerWarps * kFT * TT);
  uint64_t* empty = full + kStages;
  __shared__ int s_abort;
  __shared__ float s_bias[kFT];

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ri = blockIdx.x / a.ft_per_row;
  const int f0 = (blockIdx.x - ri * a.ft_per_row) * kFT;  // feature offset inside the block
  const int br = a.rows ? a.rows[ri] : ri;
  const int64_t t0 = int64_t(blockIdx.y) * TT;
  const int jb0 = a.crow ? a.crow[br] : 0;
  const int nblk = a.crow ? a.crow[br + 1] - jb0 : 0;
  const int n_sp = (nblk + a.sb - 1) / a.sb;
  const int n_lr = MODE == MODE_FUSED ? (a.r + a.kc - 1) / a.kc : 0;
  const int n_total = n_sp + n_lr;
  const int64_t n0 = int64_t(br) * a.bp + f0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  if (threadIdx.x < kFT) {
    const TI* bias = static_cast<const TI*>(a.bias);
    s_bias[threadIdx.x] = (MODE == MODE_FUSED && bias != nullptr) ? to_f(bias[n0 + threadIdx.x]) : 0.f;
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (n_sp) {
        tma_prefetch_desc(&tm_vals);
        tma_prefetch_desc(&tm_x);
      }
      if (n_lr) {
        tma_prefetch_desc(&tm_A);
        tma_prefetch_desc(&tm_h);
      }
    }
    const int npre = min(n_total, kStages);
    // Weights of the first npre stages (fresh slots: no empty-barrier wait).
    int colr[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      colr[s] = 0;
      if (s < npre) {
        uint8_t* dst = smem + s * stage_bytes;
        if (s < n_sp) {
          const int j0 = s * a.sb;
          const int nb = min(a.sb, nblk - j0);
          if (lane < nb) colr[s] = __ldg(a.col + jb0 + j0 + lane);
          if (lane == 0) {
            mbar_arrive_expect_tx(&full[s], v_bytes + uint32_t(nb * nsub * XB));
            tma_load_2d(dst, &tm_vals, f0, (jb0 + j0) * a.bq, &full[s]);
          }
        } else if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], lr_bytes);
          tma_load_2d(dst, &tm_A, (s - n_sp) * a.kc, br * a.bp + f0, &full[s]);
        }
      }
    }
    // Weights of the later stages into L2.
    for (int s = npre + lane; s < n_total; s += 32) {
      if (s < n_sp)
        tma_prefetch_l2_2d(&tm_vals, f0, (jb0 + s * a.sb) * a.bq);
      else
        tma_prefetch_l2_2d(&tm_A, (s - n_sp) * a.kc, br * a.bp + f0);
    }
    pdl_wait_primary();  // x and H come from preceding kernels
    __syncwarp();
    // Activations of the pre-filled stages.
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      if (s < npre) {
        uint8_t* dst = smem + s * stage_bytes;
        if (s < n_sp) {
          const int nb = min(a.sb, nblk - s * a.sb);
          if (lane < nb)
            for (int h = 0; h < nsub; ++h)
              tma_load_2d(dst + v_slot + (lane * nsub + h) * XB, &tm_x, colr[s] * a.bq + h * KX, int(t0),
                          &full[s]);
        } else if (lane == 0) {
          tma_load_2d(dst + kHOff, &tm_h, (s - n_sp) * a.kc, int(t0), &full[s]);
        }
      }
    }
    // Remaining stages through the ring.
    for (int s = npre; s < n_total; ++s) {
      const int slot = s % kStages;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[slot], ((s / kStages) & 1) ^ 1) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) {
          atomicOr(&g_status_mma, SLR_TIMEOUT_BIT);
          s_abort = 1;
        }
        break;
      }
      uint8_t* dst = smem + slot * stage_bytes;
      if (s < n_sp) {
        const int j0 = s * a.sb;
        const int nb = min(a.sb, nblk - j0);
        const int c = lane < nb ? __ldg(a.col + jb0 + j0 + lane) : 0;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[slot], v_bytes + uint32_t(nb * nsub * XB));
          tma_load_2d(dst, &tm_vals, f0, (jb0 + j0) * a.bq, &full[slot]);
        }
        __syncwarp();
        if (lane < nb)
          for (int h = 0; h < nsub; ++h)
            tma_load_2d(dst + v_slot + (lane * nsub + h) * XB, &tm_x, c * a.bq + h * KX, int(t0), &full[slot]);
      } else if (lane == 0) {
        const int l = s - n_sp;
        mbar_arrive_expect_tx(&full[slot], lr_bytes);
        tma_load_2d(dst, &tm_A, l * a.kc, br * a.bp + f0, &full[slot]);
        tma_load_2d(dst + kHOff, &tm_h, l * a.kc, int(t0), &full[slot]);
      }
    }
  } else {
    // ----------------------------------------------------------- consumers
    const int lj = lane >> 3, li = lane & 7;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

    for (int s = 0; s < n_total; ++s) {
      const int slot = s % kStages;
      if (!mbar_wait(&full[slot], (s / kStages) & 1)) {
        atomicOr(&g_status_mma, SLR_TIMEOUT_BIT);
        s_abort = 1;
        break;
      }
      const uint32_t base = smem_u32(smem + slot * stage_bytes);
      if (s < n_sp) {
        const int nb = min(a.sb, nblk - s * a.sb);
        const int steps = nb * (a.bq >> 4);
        for (int kk = warp; kk < steps; kk += kConsumerWarps) {
          const int row = 16 * kk;              // k row inside the stage's value rows
          const int j = row / a.bq, kin = row - j * a.bq;
          uint32_t af[4];
          // values slice [k rows x 16 features], 32-byte rows (SWIZZLE_32B)
          ldsm_x4_trans(base + swz_offset(row + (lj >> 1) * 8 + li, lj & 1, 32), af[0], af[1], af[2], af[3]);
          const uint32_t xt = base + v_slot + uint32_t((j * nsub + kin / KX) * XB);
          const int kc16 = (kin % KX) >> 3;     // 16-byte chunk of the k16 step in the x row
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1;
            ldsm_x2(xt + swz_offset(8 * nt + li, kc16 + (lj & 1), RWX), b0, b1);
            mma16816<TI>::run(acc[nt], af, b0, b1);
          }
        }
      } else {
        const int steps = a.kc >> 4;
        const int l = s - n_sp;
        const int kcb = a.kc * 2;               // A / H tile row bytes
        for (int kk = warp; kk < steps; kk += kConsumerWarps) {
          if (l * a.kc + 16 * kk >= a.r) break;
          uint32_t af[4];
          ldsm_x4(base + swz_offset((lj & 1) * 8 + li, 2 * kk + (lj >> 1), kcb), af[0], af[1], af[2], af[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1;
            ldsm_x2(base + kHOff + swz_offset(8 * nt + li, 2 * kk + (lj & 1), kcb), b0, b1);
            mma16816<TI>::run(acc[nt], af, b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    const int g = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = g + ((e & 2) ? 8 : 0);
        const int t = 8 * nt + 2 * tig + (e & 1);
        red[(warp * kFT + m) * TT + t] = acc[nt][e];
      }
  }
  __syncthreads();
  if (s_abort) return;

  // ------------------------------------------------------------- epilogue
  pdl_wait_primary();  // y may be read (in-place operator) or written by preceding kernels
  TI* __restrict__ y = static_cast<TI*>(a.y);
  for (int idx = threadIdx.x; idx < kFT * TT; idx += kThreads) {
    const int n = idx % kFT, t = idx / kFT;
    const int64_t tok = t0 + t;
    if (tok >= a.M) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) v += red[(w * kFT + n) * TT + t];
    const int64_t gi = tok * a.ldy + n0 + n;
    if (MODE == MODE_ADDMM) {
      v = to_f(y[gi]) + v;
    } else if (a.bias != nullptr) {
      v = v + s_bias[n];
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

  const uint4 z = make_uint4(0, 0, 0, 0);
  auto step = [&](int64_t kk, bool kin, const uint4& A0, const uint4& A1) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int64_t t = t0 + 8 * nt + g;
      const uint4 X = (t < a.M && kin) ? ldg_u128(x + t * a.ldx + kk) : z;
      const uint32_t s0[4] = {A0.x, A1.x, A0.y, A1.y};
      const uint32_t s1[4] = {A0.z, A1.z, A0.w, A1.w};
      mma16816<TI>::run(acc[nt], s0, X.x, X.y);
      mma16816<TI>::run(acc[nt], s1, X.z, X.w);
    }
  };
  // B (a weight) for the first kPre slices is loaded before griddepcontrol.wait,
  // overlapping the preceding kernel; x only after it.
  constexpr int kPre = 4;
  uint4 pa0[kPre], pa1[kPre];
#pragma unroll
  for (int i = 0; i < kPre; ++i) {
    const int64_t k = kb + 32 * warp + 128 * i;
    const int64_t kk = k + 8 * tig;
    const bool kin = k < ke && kk < ke;
    pa0[i] = (v0 && kin) ? ldg_u128(B0 + kk) : z;
    pa1[i] = (v1 && kin) ? ldg_u128(B1 + kk) : z;
  }
  pdl_wait_primary();
#pragma unroll
  for (int i = 0; i < kPre; ++i) {
    const int64_t k = kb + 32 * warp + 128 * i;
    if (k < ke) step(k + 8 * tig, k + 8 * tig < ke, pa0[i], pa1[i]);
  }
  for (int64_t k = kb + 32 * warp + 128 * kPre; k < ke; k += 128) {
    const int64_t kk = k + 8 * tig;
    const bool kin = kk < ke;
    step(kk, kin, (v0 && kin) ? ldg_u128(B0 + kk) : z, (v1 && kin) ? ldg_u128(B1 + kk) : z);
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

template <int NT, typename TI>
int launch_h_small_inst(const HArgs& a, dim3 grid, bool pdl, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, h_small_kernel<NT, TI>, a));
  return SLR_OK;
}

template <typename TI>
int launch_h_small_t(const HArgs& a, int tt, dim3 grid, bool pdl, cudaStream_t s) {
  switch (tt) {
    case 8: return launch_h_small_inst<1, TI>(a, grid, pdl, s);
    case 16: return launch_h_small_inst<2, TI>(a, grid, pdl, s);
    case 32: return launch_h_small_inst<4, TI>(a, grid, pdl, s);
    default: return launch_h_small_inst<8, TI>(a, grid, pdl, s);
  }
}

int pick_tt(int64_t M) {
  if (M <= 8) return 8;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  return 64;
}

struct MmaShape {
  int sb, kc, kx;
  size_t smem;
};

MmaShape mma_shape(int bq, int r, int tt) {
  MmaShape m;
  m.kx = bq < 64 ? bq : 64;
  m.kc = r >= 64 ? 64 : (r >= 32 ? 32 : 16);
  // value rows per sparse stage: 128 (fewer for wide token tiles), at least one block
  const int rows = tt >= 64 ? 64 : (tt >= 32 ? 128 : 256);
  m.sb = std::max(1, rows / bq);
  const uint32_t v_bytes = uint32_t(m.sb * bq * kFT * 2);
  const uint32_t v_slot = (v_bytes + 1023) & ~1023u;
  const uint32_t x_region = uint32_t(m.sb * (bq / m.kx) * tt * m.kx * 2);
  uint32_t stage = v_slot + x_region;
  if (stage < kHOff + uint32_t(tt * m.kc * 2)) stage = kHOff + uint32_t(tt * m.kc * 2);
  stage = (stage + 1023) & ~1023u;
  m.smem = 1024 + size_t(kStages) * stage + sizeof(float) * kConsumerWarps * kFT * tt + 2 * kStages * 8;
  return m;
}

template <int NT, int KX, typename TI, int MODE>
int launch_inst(const CUtensorMap& tv, const CUtensorMap& tx, const CUtensorMap& ta, const CUtensorMap& th,
                const MmaArgs& k, size_t smem, dim3 grid, bool pdl, cudaStream_t s) {
  auto kern = mma_rowblock_kernel<NT, KX, TI, MODE>;
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
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tv, tx, ta, th, k));
  return SLR_OK;
}

template <int KX, typename TI, int MODE>
int launch_nt(int tt, const CUtensorMap& tv, const CUtensorMap& tx, const CUtensorMap& ta,
              const CUtensorMap& th, const MmaArgs& k, size_t smem, dim3 grid, bool pdl, cudaStream_t s) {
  switch (tt) {
    case 8: return launch_inst<1, KX, TI, MODE>(tv, tx, ta, th, k, smem, grid, pdl, s);
    case 16: return launch_inst<2, KX, TI, MODE>(tv, tx, ta, th, k, smem, grid, pdl, s);
    case 32: return launch_inst<4, KX, TI, MODE>(tv, tx, ta, th, k, smem, grid, pdl, s);
    default: return launch_inst<8, KX, TI, MODE>(tv, tx, ta, th, k, smem, grid, pdl, s);
  }
}

template <typename TI, int MODE>
int launch_kx(int kx, int tt, const CUtensorMap& tv, const CUtensorMap& tx, const CUtensorMap& ta,
              const CUtensorMap& th, const MmaArgs& k, size_t smem, dim3 grid, bool pdl, cudaStream_t s) {
  switch (kx) {
    case 16: return launch_nt<16, TI, MODE>(tt, tv, tx, ta, th, k, smem, grid, pdl, s);
    case 32: return launch_nt<32, TI, MODE>(tt, tv, tx, ta, th, k, smem, grid, pdl, s);
    default: return launch_nt<64, TI, MODE>(tt, tv, tx, ta, th, k, smem, grid, pdl, s);
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
                   int dtype, bool pdl, cudaStream_t s) {
  if (M <= 0 || ldh <= 0) return SLR_OK;
  HArgs a{x, B, H, part, counters, M, K, ldx, plan.kchunk, int(r), int(ldh), plan.ks, plan.rt};
  const dim3 grid(unsigned(plan.rt), unsigned(plan.ks), unsigned(plan.tc));
  if (dtype == SLR_BF16) return launch_h_small_t<__nv_bfloat16>(a, plan.tt, grid, pdl, s);
  if (dtype == SLR_F16) return launch_h_small_t<__half>(a, plan.tt, grid, pdl, s);
  return fail(SLR_ERR_UNSUPPORTED_DTYPE, "h_small: 16-bit dtypes only");
}

bool mma_rowblock_supported(int bp, int bq, int64_t K, int64_t r) {
  if (bp % 16 != 0 || bp <= 0) return false;
  if (bq <= 0 || (bq != 16 && bq != 32 && bq % 64 != 0) || bq > 256) return false;
  if (K % 8 != 0) return false;
  if (r != 0 && (r % 8 != 0 || r < 16)) return false;
  return true;
}

int launch_mma_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s) {
  if (a.nrows <= 0 || a.M <= 0) return SLR_OK;
  if (a.ldx % 8 != 0 || !aligned16(a.x)) return fail(SLR_ERR_UNSUPPORTED, "mma path: x must be 16-byte aligned");
  const int tt = pick_tt(a.M);
  const bool sparse = a.crow != nullptr && a.nnz > 0;
  const int bq = sparse ? a.bq : 16;
  const int r = a.mode == MODE_FUSED ? int(a.r) : 0;
  const MmaShape sh = mma_shape(bq, r, tt);
  MmaArgs k{a.y, a.bias, sparse ? a.crow : nullptr, a.col, a.rows, a.M, a.N, a.ldy,
            a.bp, bq, r, sh.kc, sh.sb, a.bp / kFT, int(a.nrows)};
  CUtensorMap tv{}, tx{}, ta{}, th{};
  int rc;
  if (sparse) {
    rc = make_tmap_2d(&tv, a.values, a.dtype, uint64_t(a.bp), uint64_t(a.nnz) * a.bq, uint64_t(a.bp) * 2,
                      uint32_t(kFT), uint32_t(sh.sb * a.bq));
    if (rc) return rc;
    rc = make_tmap_2d(&tx, a.x, a.dtype, uint64_t(a.K), uint64_t(a.M), uint64_t(a.ldx) * 2, uint32_t(sh.kx),
                      uint32_t(tt));
    if (rc) return rc;
  }
  if (r > 0) {
    rc = make_tmap_2d(&ta, a.A, a.dtype, uint64_t(a.r), uint64_t(a.N), uint64_t(a.r) * 2, uint32_t(sh.kc),
                      uint32_t(kFT));
    if (rc) return rc;
    rc = make_tmap_2d(&th, a.H, a.dtype, uint64_t(a.ldh), uint64_t(a.M), uint64_t(a.ldh) * 2, uint32_t(sh.kc),
                      uint32_t(tt));
    if (rc) return rc;
  }
  const dim3 grid(unsigned(a.nrows * (a.bp / kFT)), unsigned(ceil_div(a.M, tt)));
  if (a.dtype == SLR_BF16)
    return a.mode == MODE_ADDMM
               ? launch_kx<__nv_bfloat16, MODE_ADDMM>(sh.kx, tt, tv, tx, ta, th, k, sh.smem, grid, pdl, s)
               : launch_kx<__nv_bfloat16, MODE_FUSED>(sh.kx, tt, tv, tx, ta, th, k, sh.smem, grid, pdl, s);
  if (a.dtype == SLR_F16)
    return a.mode == MODE_ADDMM ? launch_kx<__half, MODE_ADDMM>(sh.kx, tt, tv, tx, ta, th, k, sh.smem, grid, pdl, s)
                                : launch_kx<__half, MODE_FUSED>(sh.kx, tt, tv, tx, ta, th, k, sh.smem, grid, pdl, s);
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
