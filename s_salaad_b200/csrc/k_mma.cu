// Small-token-batch path (decode-sized M), 16-bit dtypes, mma.sync tensor
// cores with tokens on the MMA's N side, so a batch of 1..8 tokens costs one
// n8 tile and the weights stream from HBM exactly once.
//
//   h_small_kernel      H[M, ldh] = x · Bᵀ (rounded to the I/O dtype): split-K
//                       over the CTAs of a cluster, partial sums reduced
//                       through distributed shared memory in a fixed order.
//   mma_rowblock_kernel one CTA per (16 output features of a block-row, <=64
//                       tokens): a producer warp streams the 16-column slice of
//                       the row's BSR values, the x tiles at those blocks'
//                       columns, and (fused layer) the row's A rows and H tiles
//                       through a 4- or 6-slot TMA/mbarrier ring; eight consumer
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
#include "tcgen05.cuh"

namespace slr {
namespace {

__device__ unsigned g_status_mma = 0;

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 6;  // ring slots at most (a launch uses 4..kStages)
constexpr int kFT = 16;  // output features per CTA (one m16 tile)
// Low-rank stage layout: A rows (16 x kc, at most 2 KB) at 0, H tile at 2 KB
// (1024-aligned for its swizzle).
constexpr uint32_t kHOff = 2048;

constexpr int kMaxLayers = kMaxLaunchLayers;  // layers per launch
constexpr int kMaxKSplit = 8;                 // h_small K-chunks per tile (one cluster)

// One layer of a launch; its CTAs are [cta0, cta0 + nrows * ft_per_row).
struct MmaLayer {
  void* y;
  const void* bias;
  const int32_t* crow;
  const int32_t* col;
  const int32_t* rows;
  int64_t N, ldy;
  int bp, bq, r, kc;   // kc: rank columns per chunk (one A box + one H box)
  int lrc;             // chunks per low-rank stage
  int sb;              // value blocks per sparse stage
  int ft_per_row;      // bp / 16
  int nrows;
  int cta0;
  int h_col0;          // first column of this layer's H in the shared H
};
struct MmaArgs {
  int64_t M;
  int n;
  int stages;   // ring slots of this launch (fewer slots -> more CTAs per SM)
  int x_early;  // x is complete at launch: read it before griddepcontrol.wait
  MmaLayer L[kMaxLayers];
};
// Tensor maps: H is shared by the layers of a launch (H column offsets per
// layer); x, values and A are per layer (layers of a group share one x).
struct MmaMaps {
  CUtensorMap h;
  CUtensorMap x[kMaxLayers], v[kMaxLayers], a[kMaxLayers];
};

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
// CTA touches weights only -- the value and A boxes of the first ring-full of
// stages go to shared memory, those of later stages to L2, bias to shared
// memory -- so a decode step streams its weights while the previous kernel
// finishes.  H and y are read or written only after the wait; x too, unless
// x_early says that x was complete when the kernel was launched (the
// preceding kernel is this call's h_small, which lets dependents start only
// after its own wait on the kernel before it): the sparse stages then run
// while h_small computes H, and the wait comes before the first H load.
//
// Several layers run in one launch (q/k/v or gate/up sharing one x, or
// independent projections each with its own x): the grid is the
// concatenation of their CTA ranges.
template <int NT, int KX, typename TI, int MODE>
__global__ void __launch_bounds__(kThreads)
    mma_rowblock_kernel(const __grid_constant__ MmaMaps maps, const __grid_constant__ MmaArgs ga) {
  int li = 0;
  while (li + 1 < ga.n && int(blockIdx.x) >= ga.L[li + 1].cta0) ++li;
  const MmaLayer& a = ga.L[li];
  const CUtensorMap& tm_vals = maps.v[li];
  const CUtensorMap& tm_A = maps.a[li];
  const CUtensorMap& tm_x = maps.x[li];
  const CUtensorMap& tm_h = maps.h;
  const int cta = int(blockIdx.x) - a.cta0;
  constexpr int TT = 8 * NT;                 // tokens per CTA
  constexpr int XB = TT * KX * 2;            // one x sub-tile (tokens x KX columns)
  constexpr int RWX = KX * 2;                // x tile row bytes (its TMA swizzle width)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nsub = a.bq / KX;                            // x sub-tiles per block
  const uint32_t v_bytes = uint32_t(a.sb * a.bq * kFT * 2);   // values box of a stage
  const uint32_t v_slot = (v_bytes + 1023) & ~1023u;
  const uint32_t x_region = uint32_t(a.sb * nsub * XB);
  const uint32_t chunk_bytes = uint32_t(kFT * a.kc * 2 + TT * a.kc * 2);  // A + H of one chunk
  const uint32_t cs = (kHOff + TT * a.kc * 2 + 1023) & ~1023u;            // chunk stride in a slot
  uint32_t stage_bytes = v_slot + x_region;
  if (stage_bytes < kHOff + TT * a.kc * 2) stage_bytes = kHOff + TT * a.kc * 2;
  stage_bytes = (stage_bytes + 1023) & ~1023u;
  const int S = ga.stages;
  float* red = reinterpret_cast<float*>(smem + S * stage_bytes);  // [8][16][TT]
  uint64_t* full = reinterpret_cast<uint64_t*>(red + kConsumerWarps * kFT * TT);
  uint64_t* empty = full + S;
  __shared__ int s_abort;
  __shared__ float s_bias[kFT];

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ri = cta / a.ft_per_row;
  const int f0 = (cta - ri * a.ft_per_row) * kFT;  // feature offset inside the block
  const int br = a.rows ? a.rows[ri] : ri;
  const int64_t t0 = int64_t(blockIdx.y) * TT;
  const int jb0 = a.crow ? a.crow[br] : 0;
  const int nblk = a.crow ? a.crow[br + 1] - jb0 : 0;
  const int n_sp = (nblk + a.sb - 1) / a.sb;
  // low-rank stages: lrc chunks of kc rank columns each (chunk c of the
  // stage at offset c * cs: A rows [16 x kc], then the H tile at kHOff)
  const int n_chunks = MODE == MODE_FUSED ? (a.r + a.kc - 1) / a.kc : 0;
  const int n_lr = (n_chunks + a.lrc - 1) / a.lrc;
  const int n_total = n_sp + n_lr;
  const int64_t n0 = int64_t(br) * a.bp + f0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
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
    const int npre = min(n_total, S);
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
          const int c0 = (s - n_sp) * a.lrc, nch = min(a.lrc, n_chunks - c0);
          mbar_arrive_expect_tx(&full[s], uint32_t(nch) * chunk_bytes);
          for (int c = 0; c < nch; ++c)
            tma_load_2d(dst + c * cs, &tm_A, (c0 + c) * a.kc, br * a.bp + f0, &full[s]);
        }
      }
    }
    // Weights of the later stages into L2.
    for (int s = npre + lane; s < n_total; s += 32) {
      if (s < n_sp)
        tma_prefetch_l2_2d(&tm_vals, f0, (jb0 + s * a.sb) * a.bq);
      else
        for (int c = (s - n_sp) * a.lrc; c < min(n_chunks, (s - n_sp + 1) * a.lrc); ++c)
          tma_prefetch_l2_2d(&tm_A, c * a.kc, br * a.bp + f0);
    }
    // x and H come from preceding kernels (x may already be complete, see x_early)
    bool waited = !ga.x_early;
    if (waited) pdl_wait_primary();
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
        } else {
          if (!waited) {
            pdl_wait_primary();  // H is written by the preceding kernel
            waited = true;
          }
          if (lane == 0) {
            const int c0 = (s - n_sp) * a.lrc, nch = min(a.lrc, n_chunks - c0);
            for (int c = 0; c < nch; ++c)
              tma_load_2d(dst + c * cs + kHOff, &tm_h, a.h_col0 + (c0 + c) * a.kc, int(t0), &full[s]);
          }
        }
      }
    }
    // Remaining stages through the ring.
    for (int s = npre; s < n_total; ++s) {
      const int slot = s % S;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&empty[slot], ((s / S) & 1) ^ 1) ? 1 : 0;
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
      } else {
        if (!waited) {
          pdl_wait_primary();  // H is written by the preceding kernel
          waited = true;
        }
        if (lane == 0) {
          const int c0 = (s - n_sp) * a.lrc, nch = min(a.lrc, n_chunks - c0);
          mbar_arrive_expect_tx(&full[slot], uint32_t(nch) * chunk_bytes);
          for (int c = 0; c < nch; ++c) {
            tma_load_2d(dst + c * cs, &tm_A, (c0 + c) * a.kc, br * a.bp + f0, &full[slot]);
            tma_load_2d(dst + c * cs + kHOff, &tm_h, a.h_col0 + (c0 + c) * a.kc, int(t0), &full[slot]);
          }
        }
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
      const int slot = s % S;
      if (!mbar_wait(&full[slot], (s / S) & 1)) {
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
        const int per = a.kc >> 4;              // k16 steps of a chunk
        const int c0 = (s - n_sp) * a.lrc;
        const int steps = min(a.lrc, n_chunks - c0) * per;
        const int kcb = a.kc * 2;               // A / H tile row bytes
        for (int kk = warp; kk < steps; kk += kConsumerWarps) {
          const int c = kk / per, k16 = kk - c * per;
          if ((c0 + c) * a.kc + 16 * k16 >= a.r) break;
          const uint32_t cb = base + uint32_t(c) * cs;
          uint32_t af[4];
          ldsm_x4(cb + swz_offset((lj & 1) * 8 + li, 2 * k16 + (lj >> 1), kcb), af[0], af[1], af[2], af[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1;
            ldsm_x2(cb + kHOff + swz_offset(8 * nt + li, 2 * k16 + (lj & 1), kcb), b0, b1);
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
    if (tok >= ga.M) continue;
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

// H[M, ldh] = x · [B_0; ...]ᵀ: row tiles [seg_rt[s], seg_rt[s+1]) of H come
// from the r_s rows of B_s (segments of one x, e.g. q/k/v).  Each segment
// keeps the K split (ks[s] chunks of kchunk[s]) it would get alone, so a
// grouped call computes every layer's H bit for bit as a call on that layer.
struct HArgs {
  const void* x[kMaxLayers];  // segment s reads x[s] [M, K[s]] (row stride ldx[s])
  const void* B[kMaxLayers];
  void* H;
  int64_t M;
  int64_t K[kMaxLayers], ldx[kMaxLayers];
  int64_t kchunk[kMaxLayers];
  int r[kMaxLayers];
  int ks[kMaxLayers];
  int seg_rt[kMaxLayers + 1];
  int nseg, ldh, ks_max, rt;
};

__device__ __forceinline__ uint4 ldg_u128(const void* p) {
  return __ldg(static_cast<const uint4*>(p));
}

// A float in another CTA's shared memory (shared::cluster address from mapa).
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// One CTA (4 warps) = 16 rows of B x one K-chunk x 8*NT tokens.  Each lane
// loads 16 contiguous bytes of a B row and of an x row per 32-wide k slice
// and feeds them to two m16n8k16 MMAs; both operands use the same k order
// inside the slice, which leaves the dot product unchanged.  The K-chunks of
// a tile are the CTAs of one cluster (gridDim.y = ks_max): each leaves its
// partial sum in shared memory and CTA 0 of the cluster adds them in chunk
// order through distributed shared memory and writes H.
//
// Launch order: a CTA loads its first B slices, waits for the preceding
// kernel (griddepcontrol.wait), and only then lets the next kernel start
// (griddepcontrol.launch_dependents).  So when the next kernel starts, every
// kernel before this one has completed: this call's combine may read x at
// once and need wait only for H.
template <int NT, typename TI>
__global__ void __launch_bounds__(128) h_small_kernel(const __grid_constant__ HArgs a) {
  constexpr int TT = 8 * NT;
  __shared__ float red[4][16][TT];
  __shared__ float part[16 * TT];  // this CTA's partial sum, [t][m]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int rt = blockIdx.x, ks = blockIdx.y, tc = blockIdx.z;  // ks = rank in the cluster
  int sg = 0;
  while (sg + 1 < a.nseg && rt >= a.seg_rt[sg + 1]) ++sg;
  const int nks = a.ks[sg];
  if (ks >= nks) {
    // past the segment's K split: only the launch order and the cluster barriers
    pdl_wait_primary();
    pdl_launch_dependents();
  } else {
    const int64_t t0 = int64_t(tc) * TT;
    const int64_t K = a.K[sg], ldx = a.ldx[sg];
    const int64_t kb = int64_t(ks) * a.kchunk[sg];
    const int64_t ke = min(K, kb + a.kchunk[sg]);
    const TI* __restrict__ x = static_cast<const TI*>(a.x[sg]);
    const TI* __restrict__ B = static_cast<const TI*>(a.B[sg]);
    const int lrow = 16 * (rt - a.seg_rt[sg]);  // first row of this tile within B_sg
    const bool v0 = lrow + g < a.r[sg], v1 = lrow + g + 8 < a.r[sg];
    const TI* B0 = B + int64_t(lrow + g) * K;
    const TI* B1 = B + int64_t(lrow + g + 8) * K;

    float acc[NT][4];
  #pragma unroll
    for (int nt = 0; nt < NT; ++nt)
  #pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

    const uint4 z = make_uint4(0, 0, 0, 0);
    // B (a weight) for the first kPre slices is loaded before griddepcontrol.wait,
    // overlapping the preceding kernel; x only after it.  Slice i of this warp
    // covers k = kw + 128 i.  The loads of kPre slices are issued together
    // before their MMAs (one memory round trip per batch, not per slice); the
    // MMAs run in slice order either way.
    constexpr int kPre = NT >= 4 ? 2 : 4;
    const int64_t kw = kb + 32 * warp;
    uint4 pa0[kPre], pa1[kPre];
  #pragma unroll
    for (int i = 0; i < kPre; ++i) {
      const int64_t k = kw + 128 * i;
      const int64_t kk = k + 8 * tig;
      const bool kin = k < ke && kk < ke;
      pa0[i] = (v0 && kin) ? ldg_u128(B0 + kk) : z;
      pa1[i] = (v1 && kin) ? ldg_u128(B1 + kk) : z;
    }
    pdl_wait_primary();
    pdl_launch_dependents();
    auto batch = [&](int64_t i0, bool preloaded) {
      uint4 X[kPre][NT], b0[kPre], b1[kPre];
  #pragma unroll
      for (int j = 0; j < kPre; ++j) {
        const int64_t k = kw + 128 * (i0 + j);
        const int64_t kk = k + 8 * tig;
        const bool kin = k < ke && kk < ke;
        if (preloaded) {
          b0[j] = pa0[j];
          b1[j] = pa1[j];
        } else {
          b0[j] = (v0 && kin) ? ldg_u128(B0 + kk) : z;
          b1[j] = (v1 && kin) ? ldg_u128(B1 + kk) : z;
        }
  #pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int64_t t = t0 + 8 * nt + g;
          X[j][nt] = (t < a.M && kin) ? ldg_u128(x + t * ldx + kk) : z;
        }
      }
  #pragma unroll
      for (int j = 0; j < kPre; ++j) {
        if (kw + 128 * (i0 + j) >= ke) break;
        const uint32_t s0[4] = {b0[j].x, b1[j].x, b0[j].y, b1[j].y};
        const uint32_t s1[4] = {b0[j].z, b1[j].z, b0[j].w, b1[j].w};
  #pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816<TI>::run(acc[nt], s0, X[j][nt].x, X[j][nt].y);
          mma16816<TI>::run(acc[nt], s1, X[j][nt].z, X[j][nt].w);
        }
      }
    };
    batch(0, true);
    for (int64_t i0 = kPre; kw + 128 * i0 < ke; i0 += kPre) batch(i0, false);
  #pragma unroll
    for (int nt = 0; nt < NT; ++nt)
  #pragma unroll
      for (int e = 0; e < 4; ++e)
        red[warp][g + ((e & 2) ? 8 : 0)][8 * nt + 2 * tig + (e & 1)] = acc[nt][e];
    __syncthreads();
    for (int idx = threadIdx.x; idx < 16 * TT; idx += 128) {
      const int m = idx % 16, t = idx / 16;
      part[idx] = ((red[0][m][t] + red[1][m][t]) + red[2][m][t]) + red[3][m][t];
    }
  }  // ks < nks
  tc::cluster_sync();  // every partial is in its CTA's shared memory
  if (ks == 0) {
    TI* __restrict__ H = static_cast<TI*>(a.H);
    const int64_t t0 = int64_t(tc) * TT;
    const int rho0 = 16 * rt;
    for (int idx = threadIdx.x; idx < 16 * TT; idx += 128) {
      const int m = idx % 16, t = idx / 16;
      float v = part[idx];
      for (int k = 1; k < nks; ++k) v += ld_shared_cluster_f32(tc::mapa(smem_u32(&part[idx]), uint32_t(k)));
      if (t0 + t < a.M) H[(t0 + t) * a.ldh + rho0 + m] = from_f<TI>(v);
    }
  }
  tc::cluster_sync();  // no CTA leaves while CTA 0 may still read its partial
}

template <int NT, typename TI>
int launch_h_small_inst(const HArgs& a, dim3 grid, bool pdl, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;  // the K-chunks of a tile
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = grid.y;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
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
  int lrc;         // rank chunks per low-rank stage
  uint32_t stage;  // bytes of one ring slot
};

// Dynamic shared memory of a launch with `stages` ring slots of `stage` bytes.
size_t mma_smem(uint32_t stage, int stages, int tt) {
  return 1024 + size_t(stages) * stage + sizeof(float) * kConsumerWarps * kFT * tt + 2 * size_t(stages) * 8;
}

int device_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 1;
  }
  return n;
}

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
  m.stage = (stage + 1023) & ~1023u;
  // As many rank chunks per low-rank stage as the slot holds (fewer ring
  // rounds per CTA at small token counts, where the slot is sized by the
  // sparse stages and one chunk fills a quarter of it).
  const uint32_t cs = (kHOff + uint32_t(tt * m.kc * 2) + 1023) & ~1023u;
  const int chunks = r > 0 ? (r + m.kc - 1) / m.kc : 1;
  m.lrc = std::max(1, std::min(chunks, int(m.stage / cs)));
  return m;
}

// Ring depth: the full kStages slots unless 4 slots fit enough more CTAs per
// SM to need fewer waves of the grid (decode grids of several hundred CTAs
// then run in one wave; a CTA needs a few stages only at small token counts).
template <int NT, int KX, typename TI, int MODE>
int launch_inst(const MmaMaps& maps, MmaArgs k, uint32_t stage, dim3 grid, bool pdl, cudaStream_t s) {
  auto kern = mma_rowblock_kernel<NT, KX, TI, MODE>;
  constexpr int TT = 8 * NT;
  const size_t smem_full = mma_smem(stage, kStages, TT), smem_low = mma_smem(stage, 4, TT);
  // CTAs per SM of this kernel instance at both depths, per slot size (the
  // layers of a model alternate between a few sizes; the queries and the
  // attribute are host calls worth avoiding on every launch)
  struct Occ {
    uint32_t stage;
    int full, low;
  };
  thread_local Occ cache[8] = {};
  thread_local int n_cached = 0;
  thread_local size_t max_smem_set = 0;
  if (smem_full > max_smem_set) {
    SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_full)));
    max_smem_set = smem_full;
  }
  int occ_full = -1, occ_low = -1;
  for (int i = 0; i < n_cached; ++i)
    if (cache[i].stage == stage) {
      occ_full = cache[i].full;
      occ_low = cache[i].low;
    }
  if (occ_full < 0) {
    SLR_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_full, kern, kThreads, smem_full));
    SLR_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_low, kern, kThreads, smem_low));
    cache[n_cached % 8] = Occ{stage, occ_full, occ_low};
    ++n_cached;
  }
  const int64_t ctas = int64_t(grid.x) * grid.y;
  const int64_t sms = device_sms();
  const int64_t waves_full = ceil_div(ctas, sms * std::max(occ_full, 1));
  const int64_t waves_low = ceil_div(ctas, sms * std::max(occ_low, 1));
  k.stages = waves_low < waves_full ? 4 : kStages;
  const size_t smem = k.stages == kStages ? smem_full : smem_low;
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
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, maps, k));
  return SLR_OK;
}

template <int KX, typename TI, int MODE>
int launch_nt(int tt, const MmaMaps& maps, const MmaArgs& k, uint32_t stage, dim3 grid, bool pdl, cudaStream_t s) {
  switch (tt) {
    case 8: return launch_inst<1, KX, TI, MODE>(maps, k, stage, grid, pdl, s);
    case 16: return launch_inst<2, KX, TI, MODE>(maps, k, stage, grid, pdl, s);
    case 32: return launch_inst<4, KX, TI, MODE>(maps, k, stage, grid, pdl, s);
    default: return launch_inst<8, KX, TI, MODE>(maps, k, stage, grid, pdl, s);
  }
}

template <typename TI, int MODE>
int launch_kx(int kx, int tt, const MmaMaps& maps, const MmaArgs& k, uint32_t stage, dim3 grid, bool pdl,
              cudaStream_t s) {
  switch (kx) {
    case 16: return launch_nt<16, TI, MODE>(tt, maps, k, stage, grid, pdl, s);
    case 32: return launch_nt<32, TI, MODE>(tt, maps, k, stage, grid, pdl, s);
    default: return launch_nt<64, TI, MODE>(tt, maps, k, stage, grid, pdl, s);
  }
}

bool is_sparse(const RowblockArgs& a) { return a.crow != nullptr && a.nnz > 0; }
int eff_bq(const RowblockArgs& a) { return is_sparse(a) ? a.bq : 16; }

// Layer `a` as entry li of a launch: its MmaLayer (CTAs from cta0) and its
// x / value / A tensor maps.  Returns the layer's ring slot bytes in *stage.
int fill_layer(const RowblockArgs& a, int tt, int cta0, int64_t h_col, MmaMaps& maps, MmaArgs& k, int li,
               uint32_t* stage) {
  const bool sparse = is_sparse(a);
  const int bq = eff_bq(a);
  const int r = a.mode == MODE_FUSED ? int(a.r) : 0;
  const MmaShape sh = mma_shape(bq, r, tt);
  MmaLayer& L = k.L[li];
  L = MmaLayer{a.y, a.bias, sparse ? a.crow : nullptr, a.col, a.rows, a.N, a.ldy,
               a.bp, bq, r, sh.kc, sh.lrc, sh.sb, a.bp / kFT, int(a.nrows), cta0, int(h_col)};
  *stage = sh.stage;
  int rc;
  if (sparse) {
    rc = make_tmap_2d(&maps.v[li], a.values, a.dtype, uint64_t(a.bp), uint64_t(a.nnz) * a.bq,
                      uint64_t(a.bp) * 2, uint32_t(kFT), uint32_t(sh.sb * a.bq));
    if (rc) return rc;
    // x box: tt tokens x kx columns
    rc = make_tmap_2d(&maps.x[li], a.x, a.dtype, uint64_t(a.K), uint64_t(a.M), uint64_t(a.ldx) * 2,
                      uint32_t(sh.kx), uint32_t(tt));
    if (rc) return rc;
  }
  if (r > 0) {
    rc = make_tmap_2d(&maps.a[li], a.A, a.dtype, uint64_t(a.r), uint64_t(a.N), uint64_t(a.r) * 2,
                      uint32_t(sh.kc), uint32_t(kFT));
    if (rc) return rc;
  }
  return SLR_OK;
}

// H map (box: tt x kc; kc is 16, 32 or 64 and the same box serves every
// layer of a launch only when their kc agree, which mma_group_compatible
// checks).
int fill_h_map(const RowblockArgs& a0, int tt, int kc, const void* H, int64_t ldh, MmaMaps& maps) {
  if (kc <= 0) return SLR_OK;
  return make_tmap_2d(&maps.h, H, a0.dtype, uint64_t(ldh), uint64_t(a0.M), uint64_t(ldh) * 2, uint32_t(kc),
                      uint32_t(tt));
}

int launch_maps(const RowblockArgs& a0, int kx, int tt, const MmaMaps& maps, const MmaArgs& k, uint32_t stage,
                int ctas, bool pdl, cudaStream_t s) {
  const dim3 grid(unsigned(ctas), unsigned(ceil_div(a0.M, tt)));
  if (a0.dtype == SLR_BF16)
    return a0.mode == MODE_ADDMM ? launch_kx<__nv_bfloat16, MODE_ADDMM>(kx, tt, maps, k, stage, grid, pdl, s)
                                 : launch_kx<__nv_bfloat16, MODE_FUSED>(kx, tt, maps, k, stage, grid, pdl, s);
  if (a0.dtype == SLR_F16)
    return a0.mode == MODE_ADDMM ? launch_kx<__half, MODE_ADDMM>(kx, tt, maps, k, stage, grid, pdl, s)
                                 : launch_kx<__half, MODE_FUSED>(kx, tt, maps, k, stage, grid, pdl, s);
  return fail(SLR_ERR_UNSUPPORTED_DTYPE, "mma path: 16-bit dtypes only");
}

}  // namespace

HSmallPlan plan_h_small(int64_t M, const int64_t* Ks, const int64_t* ldh, int nseg) {
  HSmallPlan p;
  p.tt = pick_tt(M);
  p.tc = int(ceil_div(std::max<int64_t>(M, 1), p.tt));
  p.nseg = nseg;
  for (int sg = 0; sg < nseg; ++sg) {
    const int64_t K = Ks[sg];
    // at most 8 K-chunks: they reduce within one (portable-size) cluster
    const int64_t max_split = std::min<int64_t>(kMaxKSplit, std::max<int64_t>(1, ceil_div(K, 128)));
    const int rt = int(ldh[sg] / 16);
    p.seg_rt[sg] = p.rt;
    p.rt += rt;
    // about two CTAs per SM for this segment alone
    const int64_t base = int64_t(rt) * p.tc;
    const int64_t want = std::max<int64_t>(1, ceil_div(2 * 148, std::max<int64_t>(base, 1)));
    const int64_t ks = std::min(want, max_split);
    p.kchunk[sg] = round_up(ceil_div(K, ks), 128);
    p.ks[sg] = std::max(1, int(ceil_div(K, p.kchunk[sg])));
    p.ks_max = std::max(p.ks_max, p.ks[sg]);
  }
  p.seg_rt[nseg] = p.rt;
  return p;
}

int launch_h_small(const void* const* x, const int64_t* ldx, const void* const* B, const int64_t* r, void* H,
                   int64_t M, const int64_t* K, int64_t ldh, const HSmallPlan& plan, int dtype, bool pdl,
                   cudaStream_t s) {
  if (M <= 0 || plan.rt <= 0) return SLR_OK;
  if (plan.nseg < 1 || plan.nseg > kMaxLayers || int64_t(plan.rt) * 16 > ldh)
    return fail(SLR_ERR_INVALID_ARGUMENT, "h_small: bad segment plan");
  HArgs a{};
  a.H = H;
  a.M = M;
  a.nseg = plan.nseg;
  a.ldh = int(ldh);
  a.ks_max = plan.ks_max;
  a.rt = plan.rt;
  for (int sg = 0; sg < plan.nseg; ++sg) {
    a.x[sg] = x[sg];
    a.ldx[sg] = ldx[sg];
    a.K[sg] = K[sg];
    a.B[sg] = B[sg];
    a.r[sg] = int(r[sg]);
    a.ks[sg] = plan.ks[sg];
    a.kchunk[sg] = plan.kchunk[sg];
    a.seg_rt[sg] = plan.seg_rt[sg];
  }
  a.seg_rt[plan.nseg] = plan.seg_rt[plan.nseg];
  const dim3 grid(unsigned(plan.rt), unsigned(plan.ks_max), unsigned(plan.tc));
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

int launch_mma_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s, bool x_early) {
  if (a.nrows <= 0 || a.M <= 0) return SLR_OK;
  if (a.ldx % 8 != 0 || !aligned16(a.x)) return fail(SLR_ERR_UNSUPPORTED, "mma path: x must be 16-byte aligned");
  const int tt = pick_tt(a.M);
  const int r = a.mode == MODE_FUSED ? int(a.r) : 0;
  const MmaShape sh = mma_shape(eff_bq(a), r, tt);
  MmaMaps maps{};
  MmaArgs k{};
  k.M = a.M;
  k.n = 1;
  k.x_early = x_early ? 1 : 0;
  uint32_t stage = 0;
  int rc = fill_layer(a, tt, 0, 0, maps, k, 0, &stage);
  if (rc) return rc;
  rc = fill_h_map(a, tt, r > 0 ? sh.kc : 0, a.H, a.ldh, maps);
  if (rc) return rc;
  return launch_maps(a, sh.kx, tt, maps, k, stage, int(a.nrows * (a.bp / kFT)), pdl, s);
}

bool mma_group_compatible(const RowblockArgs* a, int n, bool shared_x) {
  if (n < 1 || n > kMaxLayers) return false;
  const int tt = pick_tt(a[0].M);
  const MmaShape s0 = mma_shape(eff_bq(a[0]), a[0].mode == MODE_FUSED ? int(a[0].r) : 0, tt);
  for (int i = 0; i < n; ++i) {
    if (a[i].M != a[0].M || a[i].dtype != a[0].dtype || a[i].mode != MODE_FUSED || a[i].r <= 0)
      return false;
    if (shared_x && (a[i].x != a[0].x || a[i].ldx != a[0].ldx || a[i].K != a[0].K)) return false;
    if (a[i].ldx % 8 != 0 || !aligned16(a[i].x)) return false;
    const MmaShape si = mma_shape(eff_bq(a[i]), int(a[i].r), tt);
    if (si.kx != s0.kx || si.kc != s0.kc) return false;
  }
  return true;
}

int launch_mma_rowblock_group(const RowblockArgs* a, const int64_t* h_col, int n, const void* H, int64_t ldh,
                              bool pdl, cudaStream_t s, bool x_early) {
  if (!mma_group_compatible(a, n, false)) return fail(SLR_ERR_INVALID_ARGUMENT, "mma group: layers need one kernel shape");
  if (a[0].M <= 0) return SLR_OK;
  const int tt = pick_tt(a[0].M);
  const MmaShape sh = mma_shape(eff_bq(a[0]), int(a[0].r), tt);
  MmaMaps maps{};
  MmaArgs k{};
  k.M = a[0].M;
  k.n = n;
  k.x_early = x_early ? 1 : 0;
  uint32_t stage = 0;
  int ctas = 0;
  for (int i = 0; i < n; ++i) {
    uint32_t si = 0;
    int rc = fill_layer(a[i], tt, ctas, h_col[i], maps, k, i, &si);
    if (rc) return rc;
    stage = std::max(stage, si);
    ctas += int(a[i].nrows * (a[i].bp / kFT));
  }
  int rc = fill_h_map(a[0], tt, sh.kc, H, ldh, maps);
  if (rc) return rc;
  if (ctas == 0) return SLR_OK;
  return launch_maps(a[0], sh.kx, tt, maps, k, stage, ctas, pdl, s);
}

int read_and_clear_status_mma(unsigned* out) {
  unsigned v = 0, zero = 0;
  SLR_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status_mma, sizeof(v)));
  if (v) SLR_CHECK_CUDA(cudaMemcpyToSymbol(g_status_mma, &zero, sizeof(zero)));
  *out = v;
  return SLR_OK;
}

}  // namespace slr
