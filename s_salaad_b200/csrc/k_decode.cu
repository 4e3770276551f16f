// Single-launch decode path (1..32 tokens, 16-bit dtypes): x·Bᵀ and the
// combine (sparse term + H·Aᵀ + bias) of up to eight layers in ONE launch,
// so a decode step pays one kernel boundary instead of two.
//
// Every CTA takes one ticket from each of two counters in the control block
// when it starts, and does that H item (its consumer warps) and that Y item:
//   H items  (n_h of them): 16 rows of a layer's B x one 512-wide K chunk ->
//            x·Bᵀ for those 16 rank columns, all tokens.  When K takes
//            several chunks, each leaves fp32 partial sums in the workspace
//            and the CTA that completes a tile's last chunk adds them in
//            chunk order; the tile of H is written rounded to the I/O dtype
//            (the reference's first F.linear rounds it so) and the layer's
//            ready counter counts it.
//   Y items  (n_y of them): one block-row of a layer (bp output features; 64
//            features for a low-rank-only layer), layers with the heaviest
//            rows first and each layer's rows heaviest first: the producer
//            warp streams the row's value blocks (one 1-D bulk copy per stage)
//            and the x tiles at their columns, then the A rows, through a TMA
//            / mbarrier ring; four consumer warps run m16n8k16 MMAs (features
//            on M, tokens on N).  Before the first low-rank stage they wait
//            until the layer's H is complete (bounded spin) and copy it into
//            shared memory; the epilogue adds the bias and stores y.
// A CTA computes its H item before it waits for any H, and tickets are taken
// by running CTAs only, so every H item is in the hands of a CTA that gets to
// it: the waits for H end whatever the grid's residency.  The block scheduler
// evens out the items' different sizes.
//
// Results do not depend on the grid, on the other layers of the launch or on
// the token count (<= 32): the K chunks of H follow from K alone, and each
// warp takes the k steps of a block-row (and of the rank) whose index is its
// own modulo the warps per 16-feature tile, in index order, however the steps
// are packed into ring stages.
//
// Reference counterparts: the two F.linear calls, the sparse addmm and the
// bias of _LRSLinearLRBlockCUDA.forward (ssalaad/efficient/ls_linear.py:
// 124-137) and the TileLang kernel _bsr_body
// (ssalaad/tilelang_sparse/addmm_inplace.py:41-82).
#include <algorithm>
#include <cstring>

#include "internal.hpp"

namespace slr {
namespace {

__device__ unsigned g_status_dec = 0;

constexpr int kDW = 4;                      // consumer warps
constexpr int kProducer = kDW;              // warp that issues the ring stages
constexpr int kDThreads = (kDW + 1) * 32;
constexpr int kColCap = 512;                // block columns of a row held in shared memory
constexpr int kDMaxStages = 6;              // ring slots at most
constexpr int kDLayers = kMaxLaunchLayers;
constexpr int kHChunk = 512;                // K of one H item (4 warps x 4 slices of 32)
constexpr uint32_t kStageTarget = 12288;    // bytes a ring stage aims at

// Control block (uint32 words; zero before a launch, zero again after it).
constexpr int kCtlQueueH = 0;  // next H ticket
constexpr int kCtlExit = 1;    // CTAs finished
constexpr int kCtlQueueY = 2;  // next Y ticket
constexpr int kCtlReady = 8;   // + layer: 16-row tiles of H written
constexpr int kCtlTile = 16;   // + tile: K chunks of the tile done
constexpr int kCtlWords = SLR_DECODE_CTRL_BYTES / 4;

struct DLayer {
  const void* x;       // [M, K], row stride ldx
  const void* B;       // [r, K]
  const void* bias;    // [N] or null
  void* y;             // [M, N], row stride ldy
  const int32_t* crow; // null: no sparse term
  const int32_t* col;
  const int32_t* rows; // block-row order (null: 0, 1, ...)
  const void* values;  // [nnz, bq, bp]: a block-row's blocks are one contiguous run
  int64_t K, N, ldx, ldy;
  int bp, bq, r;
  int ft, mt;          // output features of a Y item (16 * mt)
  int sb;              // value blocks per full sparse stage
  int kc, lrc;         // rank columns per A chunk; chunks per low-rank stage
  int nkc;             // K chunks per 16-row tile of H
  int n_rt;            // 16-row tiles of H (r / 16)
  int h0, y0, ny;      // first H item, first Y item, Y items
  int hcol;            // first column of this layer in H
  int tile0;           // first tile counter (control word kCtlTile + tile0)
  int64_t p0;          // first float of this layer's partials
};

struct DArgs {
  int64_t M;
  int n, n_h, n_y;     // layers, H items, Y items
  int stages;
  uint32_t slot;       // bytes of one ring slot (1024-aligned)
  uint32_t hbuf;       // bytes of the shared-memory copy of one layer's H
  void* H;             // [M, ldh] x·Bᵀ of every layer, I/O dtype
  int64_t ldh;
  float* P;            // fp32 partials of x·Bᵀ: per layer [tile][chunk][M][16]
  unsigned* ctrl;
  unsigned long long wait_ns;  // limit of a wait for another CTA's H (below the in-kernel 2 s)
  DLayer L[kDLayers];
};

// x tiles (box bq x TT) and A chunks (box kc x ft) of each layer.  Value
// blocks are not tiled: a stage's blocks are one contiguous run of the
// row's values, copied with one 1-D bulk copy (rows of 32 or 64 bytes would
// make narrow TMA boxes).
struct DMaps {
  CUtensorMap x[kDLayers], a[kDLayers];
};

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Barrier of the consumer warps on an mbarrier (one arrival per warp),
// bounded like every other wait: false if it gave up.
__device__ __forceinline__ bool consumer_sync(uint64_t* bar, uint32_t& phase) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  return ok;
}

template <int NT, typename TI>
__global__ void __launch_bounds__(kDThreads, NT <= 2 ? 4 : 3)
    decode_kernel(const __grid_constant__ DMaps maps, const __grid_constant__ DArgs ga) {
  constexpr int TT = 8 * NT;  // token rows of every tile (rows >= M are zero)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = ga.stages;
  uint8_t* hbuf = smem + size_t(S) * ga.slot;                 // [ldh_l / 64][TT][64], 128B-swizzled
  float* red = reinterpret_cast<float*>(hbuf + ga.hbuf);     // 64 * TT floats
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 64 * TT);
  uint64_t* empty = full + kDMaxStages;
  uint64_t* cbar = empty + kDMaxStages;                       // consumer barrier
  uint64_t* mbar = cbar + 1;                                   // the Y item's row is known
  int* cols = reinterpret_cast<int*>(mbar + 1);               // [kColCap] block columns of the row
  __shared__ int s_th, s_ty, s_layer, s_br, s_jb0, s_nblk, s_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDW);
    }
    mbar_init(cbar, kDW);
    mbar_init(mbar, 1);
    fence_mbar_init();
  }
  pdl_launch_dependents();
  // x, the workspace and the control block belong to the preceding work
  pdl_wait_primary();
  if (threadIdx.x == 0) {
    s_th = int(atomicAdd(ga.ctrl + kCtlQueueH, 1u));
    s_ty = int(atomicAdd(ga.ctrl + kCtlQueueY, 1u));
  }
  __syncthreads();
  const int th = s_th, ty = s_ty;
  const int g = lane >> 2, tig = lane & 3;
  const int lj = lane >> 3, li = lane & 7;
  uint32_t cphase = 0;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  bool alive = true;
  if (th < ga.n_h && warp < kDW) {
    // ------------------------------------------------------------ H item
    // (the consumer warps, while the producer warp starts the Y item)
    const int ctid = threadIdx.x;
    int l = 0;
    while (l + 1 < ga.n && th >= ga.L[l + 1].h0) ++l;  // h0 grows with l
    const DLayer& L = ga.L[l];
    const int idx = th - L.h0;
    const int rt = idx / L.nkc, kc = idx - rt * L.nkc;
    const int64_t kb = int64_t(kc) * kHChunk, ke = min(L.K, kb + kHChunk);
    const TI* __restrict__ x = static_cast<const TI*>(L.x);
    const TI* __restrict__ B0 = static_cast<const TI*>(L.B) + int64_t(16 * rt + g) * L.K;
    const TI* __restrict__ B1 = B0 + 8 * L.K;
    constexpr int RB = NT <= 2 ? 4 : 2;  // 32-wide slices loaded together
    const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i0 = 0; i0 < 4; i0 += RB) {
      uint4 b0[RB], b1[RB], X[RB][NT];
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        const int64_t kk = kb + 32 * warp + 128 * (i0 + q) + 8 * tig;
        const bool kin = kk < ke;  // K % 8 == 0: the 8 elements are all in or all out
        b0[q] = kin ? __ldg(reinterpret_cast<const uint4*>(B0 + kk)) : z;
        b1[q] = kin ? __ldg(reinterpret_cast<const uint4*>(B1 + kk)) : z;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int64_t t = 8 * nt + g;
          X[q][nt] = (kin && t < ga.M) ? __ldg(reinterpret_cast<const uint4*>(x + t * L.ldx + kk)) : z;
        }
      }
#pragma unroll
      for (int q = 0; q < RB; ++q) {
        if (kb + 32 * warp + 128 * (i0 + q) >= ke) break;
        const uint32_t s0[4] = {b0[q].x, b1[q].x, b0[q].y, b1[q].y};
        const uint32_t s1[4] = {b0[q].z, b1[q].z, b0[q].w, b1[q].w};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816<TI>::run(acc[nt], s0, X[q][nt].x, X[q][nt].y);
          mma16816<TI>::run(acc[nt], s1, X[q][nt].z, X[q][nt].w);
        }
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        red[(warp * 16 + g + ((e & 2) ? 8 : 0)) * TT + 8 * nt + 2 * tig + (e & 1)] = acc[nt][e];
    alive = consumer_sync(cbar, cphase);
    TI* __restrict__ H = static_cast<TI*>(ga.H);
    float* __restrict__ P = ga.P + L.p0 + int64_t(rt) * L.nkc * 16 * ga.M;  // this tile's chunks
    bool publish = L.nkc == 1;
    if (alive) {
      // this chunk's sum, warps added in order: H itself, or a partial [M][16]
      for (int i = ctid; i < 16 * ga.M; i += kDW * 32) {
        const int m = i & 15, t = i >> 4;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kDW; ++w) v += red[(w * 16 + m) * TT + t];
        if (publish)
          H[int64_t(t) * ga.ldh + L.hcol + 16 * rt + m] = from_f<TI>(v);
        else
          __stcg(P + int64_t(kc) * 16 * ga.M + i, v);
      }
      // every thread's stores, then one thread fences at GPU scope and counts
      // (the CTA barrier orders the others' stores before its fence)
      alive = consumer_sync(cbar, cphase);
    }
    if (alive && !publish) {
      if (ctid == 0) {
        __threadfence();
        const unsigned done = atomicAdd(ga.ctrl + kCtlTile + L.tile0 + rt, 1u);
        s_flag = done == unsigned(L.nkc - 1);
        if (s_flag) __threadfence();  // the other chunks' partials are visible after it
      }
      alive = consumer_sync(cbar, cphase);
      publish = alive && s_flag != 0;
      if (publish) {
        // the tile's last chunk: add the partials in chunk order, eight
        // chunk loads in flight per element
        for (int i = ctid; i < 16 * ga.M; i += kDW * 32) {
          const int m = i & 15, t = i >> 4;
          float v = 0.f;
          for (int q0 = 0; q0 < L.nkc; q0 += 8) {
            float w[8];
#pragma unroll
            for (int qq = 0; qq < 8; ++qq)
              w[qq] = q0 + qq < L.nkc ? __ldcg(P + int64_t(q0 + qq) * 16 * ga.M + i) : 0.f;
#pragma unroll
            for (int qq = 0; qq < 8; ++qq)
              if (q0 + qq < L.nkc) v += w[qq];
          }
          H[int64_t(t) * ga.ldh + L.hcol + 16 * rt + m] = from_f<TI>(v);
        }
        alive = publish = consumer_sync(cbar, cphase);
      }
    }
    if (publish && ctid == 0) {
      __threadfence();
      atomicAdd(ga.ctrl + kCtlReady + l, 1u);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
  }

  if (ty < ga.n_y) {
    // ------------------------------------------------------------ Y item
    if (threadIdx.x == kProducer * 32) {
      int l = 0;
      for (; l + 1 < ga.n; ++l)
        if (ty >= ga.L[l].y0 && ty < ga.L[l].y0 + ga.L[l].ny) break;
      const DLayer& L = ga.L[l];
      const int j = ty - L.y0;
      const int br = L.rows ? __ldg(L.rows + j) : j;
      int jb0 = 0, nblk = 0;
      if (L.crow) {
        jb0 = __ldg(L.crow + br);
        nblk = __ldg(L.crow + br + 1) - jb0;
      }
      s_layer = l;
      s_br = br;
      s_jb0 = jb0;
      s_nblk = nblk;
      mbar_arrive(mbar);
    }
    // the row (consumers may still be on their H item)
    if (!mbar_wait(mbar, 0)) {
      atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);
      alive = false;
    }
    const int l = s_layer, br = s_br, jb0 = s_jb0, nblk = s_nblk;
    const DLayer& L = ga.L[l];
    const int n_sp = (nblk + L.sb - 1) / L.sb;
    const int n_ch = L.r / L.kc;
    const int n_lr = (n_ch + L.lrc - 1) / L.lrc;
    const int n_st = n_sp + n_lr;
    const uint32_t blk = uint32_t(L.bq * L.ft * 2);            // one value block
    const uint32_t vslot = (uint32_t(L.sb) * blk + 1023u) & ~1023u;
    const uint32_t xb = uint32_t(TT * L.bq * 2);               // one x tile
    const uint32_t cb = uint32_t(L.ft * L.kc * 2);             // one A chunk
    if (!alive) {
      // a wait gave up: no stage is issued, none is awaited
    } else if (warp == kProducer) {
      // ---------------------------------------------------------- producer
      if (lane == 0) {
        tma_prefetch_desc(&maps.x[l]);
        tma_prefetch_desc(&maps.a[l]);
      }
      for (int st = 0; st < n_st; ++st) {
        const int sl = st % S;
        int ok = 1;
        int j0 = 0, nb = 0, c0 = 0, nch = 0;
        uint32_t tx;
        if (st < n_sp) {
          j0 = st * L.sb;
          nb = min(L.sb, nblk - j0);
          tx = uint32_t(nb) * (blk + xb);
        } else {
          c0 = (st - n_sp) * L.lrc;
          nch = min(L.lrc, n_ch - c0);
          tx = uint32_t(nch) * cb;
        }
        if (lane == 0) {
          ok = mbar_wait(&empty[sl], ((st / S) & 1) ^ 1) ? 1 : 0;
          if (ok) mbar_arrive_expect_tx(&full[sl], tx);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);
          break;
        }
        uint8_t* dst = smem + size_t(sl) * ga.slot;
        if (st < n_sp) {
          if (lane == 0)
            bulk_load_1d(dst, static_cast<const uint8_t*>(L.values) + int64_t(jb0 + j0) * blk, uint32_t(nb) * blk,
                         &full[sl]);
          if (st == 0) {
            // the row's block columns, after the first values are on their way
            for (int i = lane; i < min(nblk, kColCap); i += 32) cols[i] = __ldg(L.col + jb0 + i);
            __syncwarp();
          }
          const int jj = j0 + lane;
          if (lane < nb) {
            const int c = jj < kColCap ? cols[jj] : __ldg(L.col + jb0 + jj);
            tma_load_2d(dst + vslot + lane * xb, &maps.x[l], c * L.bq, 0, &full[sl]);
          }
        } else if (lane < nch) {
          tma_load_2d(dst + lane * cb, &maps.a[l], (c0 + lane) * L.kc, br * L.ft, &full[sl]);
        }
      }
    } else {
      // --------------------------------------------------------- consumers
      const int ctid = threadIdx.x;
      const int mt = L.mt, wpm = kDW / mt, wm = warp % mt, wk = warp / mt;
      const uint32_t hb0 = smem_u32(hbuf);
      for (int st = 0; st < n_st && alive; ++st) {
        const int sl = st % S;
        if (!mbar_wait(&full[sl], (st / S) & 1)) {
          atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);
          alive = false;
          break;
        }
        const uint32_t base = smem_u32(smem + size_t(sl) * ga.slot);
        if (st < n_sp) {
          const int j0 = st * L.sb, nb = min(L.sb, nblk - j0);
          const int steps = nb * (L.bq >> 4);
          const int rb = L.ft * 2;  // value row bytes
          // k step u of the stage is step j0 * bq / 16 + u of the block-row: warp wk
          // takes the steps whose block-row index is wk modulo wpm, whatever the stages
          const int u0 = (wk - (j0 * (L.bq >> 4)) % wpm + wpm) % wpm;
          for (int u = u0; u < steps; u += wpm) {
            const int row = 16 * u;
            const int j = row / L.bq, kin = row - j * L.bq;
            uint32_t af[4];
            // values [k rows x ft features], plain row-major (bulk copy, no swizzle)
            ldsm_x4_trans(base + uint32_t((row + (lj >> 1) * 8 + li) * rb + ((2 * wm + (lj & 1)) << 4)), af[0],
                          af[1], af[2], af[3]);
            const uint32_t xt = base + vslot + uint32_t(j) * xb;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              uint32_t b0, b1;
              ldsm_x2(xt + swz_offset(8 * nt + li, (kin >> 3) + (lj & 1), L.bq * 2), b0, b1);
              mma16816<TI>::run(acc[nt], af, b0, b1);
            }
          }
        } else {
          const int c0 = (st - n_sp) * L.lrc, nch = min(L.lrc, n_ch - c0);
          if (st == n_sp) {
            // H of this layer: wait until all its tiles are written, then copy
            // it into shared memory (rows >= M zero)
            if (ctid == 0) {
              const unsigned long long t0 = globaltimer_ns();
              while (ld_acquire_gpu_u32(ga.ctrl + kCtlReady + l) < unsigned(L.n_rt)) {
                if (globaltimer_ns() - t0 > ga.wait_ns) {
                  atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);  // y of this layer is not valid
                  break;
                }
                __nanosleep(32);
              }
            }
            alive = consumer_sync(cbar, cphase);
            if (!alive) break;
            const TI* __restrict__ H = static_cast<const TI*>(ga.H);
            const int nc8 = L.r >> 3;  // 16-byte chunks of a row
            for (int i = ctid; i < TT * nc8; i += kDW * 32) {
              const int t = i / nc8, c8 = i - t * nc8;
              uint4 v = make_uint4(0, 0, 0, 0);
              if (t < ga.M) v = __ldcg(reinterpret_cast<const uint4*>(H + int64_t(t) * ga.ldh + L.hcol + 8 * c8));
              st_shared_v4(hb0 + uint32_t((c8 >> 3) * TT * 128) + swz_offset(t, c8 & 7, 128), v);
            }
            alive = consumer_sync(cbar, cphase);
            if (!alive) break;
          }
          const int per = L.kc >> 4;
          const int steps = nch * per;
          const int u0 = (wk - (c0 * per) % wpm + wpm) % wpm;  // by the step's index in the rank
          for (int u = u0; u < steps; u += wpm) {
            const int c = u / per, k16 = u - c * per;
            const int kg = (c0 + c) * L.kc + 16 * k16;  // rank column
            uint32_t af[4];
            ldsm_x4(base + uint32_t(c) * cb + swz_offset(16 * wm + (lj & 1) * 8 + li, 2 * k16 + (lj >> 1), L.kc * 2),
                    af[0], af[1], af[2], af[3]);
            const uint32_t hb = hb0 + uint32_t((kg >> 6) * TT * 128);
            const int ch = (kg & 63) >> 3;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              uint32_t b0, b1;
              ldsm_x2(hb + swz_offset(8 * nt + li, ch + (lj & 1), 128), b0, b1);
              mma16816<TI>::run(acc[nt], af, b0, b1);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[sl]);
      }
      if (alive) {
        // ---- epilogue: add the warps' partial sums (k-part order), bias, store
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            red[(wk * L.ft + 16 * wm + g + ((e & 2) ? 8 : 0)) * TT + 8 * nt + 2 * tig + (e & 1)] = acc[nt][e];
        if (consumer_sync(cbar, cphase)) {
          const int64_t n0 = int64_t(br) * L.ft;
          const TI* __restrict__ bias = static_cast<const TI*>(L.bias);
          TI* __restrict__ y = static_cast<TI*>(L.y);
          for (int i = ctid; i < L.ft * TT; i += kDW * 32) {
            const int n = i % L.ft, t = i / L.ft;
            if (t >= ga.M || n0 + n >= L.N) continue;
            float v = 0.f;
            for (int w = 0; w < wpm; ++w) v += red[(w * L.ft + n) * TT + t];
            if (bias) v += to_f(bias[n0 + n]);
            y[int64_t(t) * L.ldy + n0 + n] = from_f<TI>(v);
          }
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // The last CTA to finish leaves the control block zero for the next launch.
    __threadfence();
    const unsigned done = atomicAdd(ga.ctrl + kCtlExit, 1u);
    if (done == gridDim.x - 1) {
      __threadfence();
      ga.ctrl[kCtlQueueH] = 0;
      ga.ctrl[kCtlQueueY] = 0;
      for (int l = 0; l < ga.n; ++l) {
        ga.ctrl[kCtlReady + l] = 0;
        for (int t = 0; t < ga.L[l].n_rt; ++t) ga.ctrl[kCtlTile + ga.L[l].tile0 + t] = 0;
      }
      ga.ctrl[kCtlExit] = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------- host --

struct DecodePlan {
  DArgs a{};
  int tt = 8;
  size_t smem = 0;
  size_t h_bytes = 0, p_bytes = 0, total = 0;
};

size_t align256_(size_t v) { return (v + 255) & ~size_t(255); }

bool block_dim_ok(int64_t b) { return b == 16 || b == 32 || b == 64; }

size_t dec_smem(int stages, uint32_t slot, uint32_t hbuf, int tt) {
  return 1024 + size_t(stages) * slot + hbuf + size_t(64) * tt * 4 + (2 * kDMaxStages + 2) * 8 +
         kColCap * sizeof(int);
}

// Shape of layer i (everything that fixes its arithmetic order) and its share
// of the launch's items, control words and workspace.  Returns false if the
// layer is outside what the kernel handles.
bool plan_layer(const RowblockArgs& in, int tt, DecodePlan& p, int i, int& items_h, int& tiles, int64_t& pfl,
                int64_t& hcol, int64_t M) {
  DLayer& L = p.a.L[i];
  const bool sparse = in.crow != nullptr && in.nnz > 0;
  if (in.r < 0 || in.r % 16 || in.r > 512) return false;
  if (in.K <= 0 || in.K % 8 || in.ldx % 8 || !aligned16(in.x)) return false;
  if (in.r > 0 && (!aligned16(in.A) || !aligned16(in.B))) return false;
  if (sparse) {
    if (!block_dim_ok(in.bp) || !block_dim_ok(in.bq) || !aligned16(in.values)) return false;
    if (in.nnz * in.bq >= (int64_t(1) << 31)) return false;
  }
  L = DLayer{};
  L.x = in.x;
  L.B = in.B;
  L.bias = in.bias;
  L.y = in.y;
  L.crow = sparse ? in.crow : nullptr;
  L.col = in.col;
  L.rows = sparse ? in.rows : nullptr;
  L.values = sparse ? in.values : nullptr;
  L.K = in.K;
  L.N = in.N;
  L.ldx = in.ldx;
  L.ldy = in.ldy;
  L.bp = sparse ? in.bp : 64;
  L.bq = sparse ? in.bq : 16;
  L.r = int(in.r);
  L.ft = L.bp;
  L.mt = L.ft / 16;
  if (sparse) {
    const int per = int(kStageTarget / uint32_t(L.bq * (L.ft + tt) * 2));
    L.sb = std::max(1, std::min(per, 256 / L.bq));
  } else {
    L.sb = 1;
  }
  L.kc = L.r % 64 == 0 ? 64 : (L.r % 32 == 0 ? 32 : 16);
  const int n_ch = L.r > 0 ? L.r / L.kc : 0;
  L.lrc = std::max(1, std::min(std::max(n_ch, 1), int(kStageTarget / uint32_t(L.ft * L.kc * 2))));
  L.nkc = int(ceil_div(in.K, kHChunk));
  L.n_rt = L.r / 16;
  L.h0 = items_h;
  items_h += L.n_rt * L.nkc;
  L.ny = int(sparse ? in.N / in.bp : ceil_div(in.N, 64));
  L.tile0 = tiles;
  tiles += L.n_rt;
  L.hcol = int(hcol);
  hcol += round_up(L.r, 64);
  L.p0 = pfl;
  if (L.nkc > 1) pfl += int64_t(L.n_rt) * L.nkc * 16 * M;
  return true;
}

// Plans a launch of n layers (inputs bound or not).  false: not handled.
bool plan_decode(const RowblockArgs* layers, int n, int64_t M, DecodePlan& p) {
  if (n < 1 || n > kDLayers || M < 1 || M > SLR_DECODE_MAX_TOKENS) return false;
  const int dtype = layers[0].dtype;
  if (dtype != SLR_BF16 && dtype != SLR_F16) return false;
  p.tt = M <= 8 ? 8 : (M <= 16 ? 16 : 32);
  int items_h = 0, tiles = 0;
  int64_t pfl = 0, hcol = 0;
  for (int i = 0; i < n; ++i) {
    if (layers[i].dtype != dtype || layers[i].mode != MODE_FUSED) return false;
    if (!plan_layer(layers[i], p.tt, p, i, items_h, tiles, pfl, hcol, M)) return false;
  }
  if (kCtlTile + tiles > kCtlWords) return false;
  // Y items: the layers with the heaviest block-rows first (each layer's rows
  // heaviest first through its row order), so the longest items start first.
  int order[kDLayers];
  double avg[kDLayers];
  for (int i = 0; i < n; ++i) {
    const DLayer& L = p.a.L[i];
    const double blocks = L.crow ? double(layers[i].nnz) / std::max(L.ny, 1) : 0.0;
    avg[i] = blocks * L.bq * L.ft + double(L.ft) * L.r;
    order[i] = i;
  }
  std::stable_sort(order, order + n, [&](int a, int b) { return avg[a] > avg[b]; });
  int items = 0;
  for (int k = 0; k < n; ++k) {
    DLayer& L = p.a.L[order[k]];
    L.y0 = items;
    items += L.ny;
  }
  p.a.M = M;
  p.a.n = n;
  p.a.n_h = items_h;
  p.a.n_y = items;
  p.a.ldh = std::max<int64_t>(hcol, 8);
  uint32_t slot = 1024, hbuf = 0;
  for (int i = 0; i < n; ++i) {
    const DLayer& L = p.a.L[i];
    if (L.crow) {
      const uint32_t v = (uint32_t(L.sb * L.bq * L.ft * 2) + 1023u) & ~1023u;
      slot = std::max(slot, v + uint32_t(L.sb * p.tt * L.bq * 2));
    }
    if (L.r > 0) slot = std::max(slot, uint32_t(L.lrc * L.ft * L.kc * 2));
    hbuf = std::max(hbuf, uint32_t(p.tt * round_up(L.r, 64) * 2));
  }
  p.a.slot = (slot + 1023u) & ~1023u;
  p.a.hbuf = (hbuf + 1023u) & ~1023u;
  // ring depth: the most stages (3 at least) that let four CTAs share an SM
  // (three from 17 tokens on, whose instance has more registers)
  const int per_sm = p.tt <= 16 ? 4 : 3;
  const size_t budget = 228 * 1024 / per_sm - 2048;
  int stages = kDMaxStages;
  while (stages > 3 && dec_smem(stages, p.a.slot, p.a.hbuf, p.tt) > budget) --stages;
  p.a.stages = stages;
  p.smem = dec_smem(stages, p.a.slot, p.a.hbuf, p.tt);
  if (p.smem > 227 * 1024) return false;
  const size_t es = dtype_size(dtype);
  p.h_bytes = align256_(size_t(M) * size_t(p.a.ldh) * es);
  p.p_bytes = align256_(size_t(pfl) * 4);
  p.total = p.h_bytes + p.p_bytes;
  return true;
}

template <int NT, typename TI>
int launch_decode_inst(const DMaps& maps, const DecodePlan& p, bool pdl, cudaStream_t s) {
  auto kern = decode_kernel<NT, TI>;
  thread_local size_t c_smem = 0;
  if (c_smem != p.smem) {
    SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(p.smem)));
    c_smem = p.smem;
  }
  const int64_t ctas = std::max(p.a.n_h, p.a.n_y);  // an H item and a Y item per CTA
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(std::max<int64_t>(ctas, 1)));
  cfg.blockDim = dim3(kDThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, maps, p.a));
  return SLR_OK;
}

template <typename TI>
int launch_decode_t(const DMaps& maps, const DecodePlan& p, bool pdl, cudaStream_t s) {
  switch (p.tt) {
    case 8: return launch_decode_inst<1, TI>(maps, p, pdl, s);
    case 16: return launch_decode_inst<2, TI>(maps, p, pdl, s);
    default: return launch_decode_inst<4, TI>(maps, p, pdl, s);
  }
}

}  // namespace

bool decode_supported(const RowblockArgs* layers, int n, int64_t M) {
  DecodePlan p;
  return plan_decode(layers, n, M, p);
}

size_t decode_workspace_size(const RowblockArgs* layers, int n, int64_t M) {
  DecodePlan p;
  return plan_decode(layers, n, M, p) ? p.total : 0;
}

int launch_decode(const RowblockArgs* layers, int n, int64_t M, void* workspace, size_t workspace_bytes,
                  unsigned* ctrl, bool pdl, cudaStream_t s) {
  DecodePlan p;
  if (!plan_decode(layers, n, M, p)) return fail(SLR_ERR_UNSUPPORTED, "decode: layer set not supported");
  if (!ctrl || (reinterpret_cast<uintptr_t>(ctrl) & 15u))
    return fail(SLR_ERR_INVALID_ARGUMENT, "decode: control block must be a 16-byte aligned device pointer");
  if (workspace_bytes < p.total || (p.total > 0 && !workspace))
    return fail(SLR_ERR_WORKSPACE, "workspace too small: need " + std::to_string(p.total) + " bytes");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.a.H = ws;
  p.a.P = reinterpret_cast<float*>(ws + p.h_bytes);
  p.a.ctrl = ctrl;
  p.a.wait_ns = std::min(peer_wait_limit_ns(), SLR_WAIT_LIMIT_NS / 2);
  DMaps maps;
  memset(&maps, 0, sizeof(maps));
  const int dtype = layers[0].dtype;
  for (int i = 0; i < n; ++i) {
    const RowblockArgs& in = layers[i];
    const DLayer& L = p.a.L[i];
    int rc;
    if (L.crow) {
      rc = make_tmap_2d(&maps.x[i], in.x, dtype, uint64_t(in.K), uint64_t(M), uint64_t(in.ldx) * 2, uint32_t(L.bq),
                        uint32_t(p.tt));
      if (rc) return rc;
    }
    if (L.r > 0) {
      rc = make_tmap_2d(&maps.a[i], in.A, dtype, uint64_t(L.r), uint64_t(in.N), uint64_t(L.r) * 2, uint32_t(L.kc),
                        uint32_t(L.ft));
      if (rc) return rc;
    }
  }
  if (dtype == SLR_BF16) return launch_decode_t<__nv_bfloat16>(maps, p, pdl, s);
  return launch_decode_t<__half>(maps, p, pdl, s);
}

int read_and_clear_status_dec(unsigned* out) {
  unsigned v = 0, zero = 0;
  SLR_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status_dec, sizeof(v)));
  if (v) SLR_CHECK_CUDA(cudaMemcpyToSymbol(g_status_dec, &zero, sizeof(zero)));
  *out = v;
  return SLR_OK;
}

}  // namespace slr
