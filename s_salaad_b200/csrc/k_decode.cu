// Single-launch decode path (1..32 tokens, 16-bit dtypes): x·Bᵀ and the
// combine (sparse term + H·Aᵀ + bias) of up to eight layers in ONE persistent
// launch, so a decode step pays one kernel boundary instead of two and the
// combine runs as one wave of whole block-rows instead of several waves of
// 16-feature slices.
//
// Work items, handed out in order from a queue in the control block:
//   H items  (first): 16 rows of a layer's B x one 1024-wide K chunk ->
//            x·Bᵀ for those 16 rank columns, all tokens.  A layer whose K
//            needs several chunks leaves fp32 partials in the workspace; the
//            CTA that completes the last chunk of a 16-row tile adds them in
//            chunk order and writes H (rounded to the I/O dtype, as the
//            reference's first F.linear is).  Each finished tile of H adds 1
//            to the layer's ready counter.
//   Y items  (then): one block-row of a layer (bp output features; 64
//            features for a low-rank-only layer): its value blocks and the x
//            tiles at their columns, then the A rows, stream through a TMA /
//            mbarrier ring; eight consumer warps run m16n8k16 MMAs (features
//            on M, tokens on N) and the epilogue adds the bias and stores y.
//            The low-rank stages first wait until the layer's H is complete
//            (bounded spin on the ready counter) and copy H into shared
//            memory once per layer and CTA.
// Every CTA takes its items in increasing queue order and all H items come
// before all Y items, so an H item is always held by a running CTA that
// computes it before any of its own waits: the waits end whatever the grid
// size and residency.
//
// Results do not depend on the grid, on the other layers of the launch or on
// the token count (<= 32): the K chunks of H, the stages of a block-row and
// the k steps of each warp follow from the layer's own shape only.
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

constexpr int kDW = 8;                      // consumer warps
constexpr int kDThreads = (kDW + 1) * 32;   // + the producer warp
constexpr int kDMaxStages = 8;              // ring slots at most
constexpr int kDLayers = kMaxLaunchLayers;
constexpr int kHChunk = 1024;               // K of one H item (8 warps x 4 slices of 32)
constexpr uint32_t kStageTarget = 12288;    // bytes a ring stage aims at

// Control block (uint32 words; zero before a launch, zero again after it).
constexpr int kCtlQueue = 0;   // next work item
constexpr int kCtlExit = 1;    // CTAs finished
constexpr int kCtlReady = 8;   // + layer: 16-row tiles of H complete
constexpr int kCtlTile = 16;   // + tile: K chunks of the tile done
constexpr int kCtlWords = SLR_DECODE_CTRL_BYTES / 4;

enum : int { ST_END = 0, ST_H = 1, ST_SPARSE = 2, ST_LOWRANK = 3, ST_EMPTY = 4 };

struct DStage {
  int kind, layer, item;  // item: H item within the layer, or the feature tile of a Y item
  int a, b;               // sparse: first block of the stage, blocks; low-rank: first chunk, chunks
  int first, last;        // first / last stage of its Y item
};

struct DLayer {
  const void* x;       // [M, K], row stride ldx
  const void* B;       // [r, K]
  const void* bias;    // [N] or null
  void* y;             // [M, N], row stride ldy
  const int32_t* crow; // null: no sparse term
  const int32_t* col;
  const int32_t* rows; // block-row order (null: 0, 1, ...)
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
  int n, n_h, n_items;
  int64_t ldh;         // row stride of H
  int stages;
  uint32_t slot;       // bytes of one ring slot (1024-aligned)
  uint32_t hbuf;       // bytes of the shared-memory copy of one layer's H
  void* H;
  float* P;
  unsigned* ctrl;
  unsigned long long wait_ns;  // limit of a wait for another CTA's H (below the in-kernel 2 s)
  DLayer L[kDLayers];
};

// x tiles (box bq x TT), value boxes (sb blocks and one block) and A chunks
// (box kc x ft) of each layer.
struct DMaps {
  CUtensorMap x[kDLayers], v[kDLayers], v1[kDLayers], a[kDLayers];
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

// Barrier of the eight consumer warps on an mbarrier (one arrival per warp),
// bounded like every other wait: false if it gave up.
__device__ __forceinline__ bool consumer_sync(uint64_t* bar, uint32_t& phase) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  return ok;
}

template <int NT, typename TI>
__global__ void __launch_bounds__(kDThreads, NT <= 2 ? 2 : 1)
    decode_kernel(const __grid_constant__ DMaps maps, const __grid_constant__ DArgs ga) {
  constexpr int TT = 8 * NT;  // token rows of every tile (rows >= M are zero)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = ga.stages;
  uint8_t* hbuf = smem + size_t(S) * ga.slot;                 // [ldh_l / 64][TT][64], 128B-swizzled
  float* red = reinterpret_cast<float*>(hbuf + ga.hbuf);     // 128 * TT floats
  uint64_t* full = reinterpret_cast<uint64_t*>(red + 128 * TT);
  uint64_t* empty = full + kDMaxStages;
  uint64_t* cbar = empty + kDMaxStages;                       // consumer barrier
  DStage* recs = reinterpret_cast<DStage*>(cbar + 1);
  __shared__ int s_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDW);
    }
    mbar_init(cbar, kDW);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  // x, the workspace and the control block belong to the preceding work
  pdl_wait_primary();

  if (warp == kDW) {
    // ------------------------------------------------------------ producer
    if (lane == 0)
      for (int l = 0; l < ga.n; ++l) {
        tma_prefetch_desc(&maps.v[l]);
        tma_prefetch_desc(&maps.v1[l]);
        tma_prefetch_desc(&maps.x[l]);
        tma_prefetch_desc(&maps.a[l]);
      }
    int s = 0;  // stages issued
    bool ok = true;
    // Claims ring slot s for record r with `tx` bytes of TMA to come (0: the
    // record alone completes the slot).  Returns the slot, or -1 on timeout.
    auto claim = [&](const DStage& r, uint32_t tx) -> int {
      const int sl = s % S;
      int good = 1;
      if (lane == 0) {
        good = mbar_wait(&empty[sl], ((s / S) & 1) ^ 1) ? 1 : 0;
        if (good) {
          recs[sl] = r;
          if (tx)
            mbar_arrive_expect_tx(&full[sl], tx);
          else
            mbar_arrive(&full[sl]);
        }
      }
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) {
        if (lane == 0) atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);
        return -1;
      }
      ++s;
      return sl;
    };
    int item = 0;
    if (lane == 0) item = int(atomicAdd(ga.ctrl + kCtlQueue, 1u));
    item = __shfl_sync(0xffffffffu, item, 0);
    while (ok) {
      if (item >= ga.n_items) {
        ok = claim(DStage{ST_END, 0, 0, 0, 0, 1, 1}, 0) >= 0;
        break;
      }
      int next = 0;
      if (lane == 0) next = int(atomicAdd(ga.ctrl + kCtlQueue, 1u));  // taken ahead, used after this item
      if (item < ga.n_h) {
        int l = 0;
        while (l + 1 < ga.n && item >= ga.L[l + 1].h0) ++l;
        ok = claim(DStage{ST_H, l, item - ga.L[l].h0, 0, 0, 1, 1}, 0) >= 0;
      } else {
        int l = 0;
        while (l + 1 < ga.n && item >= ga.L[l + 1].y0) ++l;
        const DLayer& L = ga.L[l];
        const int j = item - L.y0;
        const int br = L.rows ? __ldg(L.rows + j) : j;
        int jb0 = 0, nblk = 0;
        if (L.crow) {
          jb0 = __ldg(L.crow + br);
          nblk = __ldg(L.crow + br + 1) - jb0;
        }
        const int n_sp = (nblk + L.sb - 1) / L.sb;
        const int n_ch = L.r / L.kc;
        const int n_lr = (n_ch + L.lrc - 1) / L.lrc;
        const int n_st = n_sp + n_lr;
        const uint32_t blk = uint32_t(L.bq * L.ft * 2);              // one value block
        const uint32_t vslot = (uint32_t(L.sb) * blk + 1023u) & ~1023u;
        const uint32_t xb = uint32_t(TT * L.bq * 2);                 // one x tile
        if (n_st == 0) ok = claim(DStage{ST_EMPTY, l, br, 0, 0, 1, 1}, 0) >= 0;
        for (int st = 0; ok && st < n_sp; ++st) {
          const int j0 = st * L.sb, nb = min(L.sb, nblk - j0);
          const int c = lane < nb ? __ldg(L.col + jb0 + j0 + lane) : 0;
          const int sl = claim(DStage{ST_SPARSE, l, br, j0, nb, st == 0, st == n_st - 1}, uint32_t(nb) * (blk + xb));
          if (sl < 0) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + size_t(sl) * ga.slot;
          const int row0 = (jb0 + j0) * L.bq;
          if (nb == L.sb) {
            if (lane == 0) tma_load_2d(dst, &maps.v[l], 0, row0, &full[sl]);
          } else if (lane < nb) {
            tma_load_2d(dst + lane * blk, &maps.v1[l], 0, row0 + lane * L.bq, &full[sl]);
          }
          if (lane < nb) tma_load_2d(dst + vslot + lane * xb, &maps.x[l], c * L.bq, 0, &full[sl]);
        }
        for (int st = 0; ok && st < n_lr; ++st) {
          const int c0 = st * L.lrc, nch = min(L.lrc, n_ch - c0);
          const uint32_t cb = uint32_t(L.ft * L.kc * 2);
          const int sl = claim(DStage{ST_LOWRANK, l, br, c0, nch, n_sp == 0 && st == 0, st == n_lr - 1},
                               uint32_t(nch) * cb);
          if (sl < 0) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + size_t(sl) * ga.slot;
          if (lane < nch) tma_load_2d(dst + lane * cb, &maps.a[l], (c0 + lane) * L.kc, br * L.ft, &full[sl]);
        }
      }
      item = __shfl_sync(0xffffffffu, next, 0);
    }
  } else {
    // ----------------------------------------------------------- consumers
    const int ctid = threadIdx.x;  // 0..255
    const int g = lane >> 2, tig = lane & 3;
    const int lj = lane >> 3, li = lane & 7;
    uint32_t cphase = 0;
    int cur_h = -1;
    bool alive = true;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
    const uint32_t hb0 = smem_u32(hbuf);

    for (int s = 0; alive; ++s) {
      const int sl = s % S;
      if (!mbar_wait(&full[sl], (s / S) & 1)) {
        atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);
        break;
      }
      const DStage rec = recs[sl];
      if (rec.kind == ST_END) break;
      const DLayer& L = ga.L[rec.layer];
      if (rec.kind == ST_H) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[sl]);  // the item carries no data in the slot
        // ---- 16 rank columns of x·Bᵀ over one K chunk, all tokens
        const int rt = rec.item / L.nkc, kc = rec.item - rt * L.nkc;
        const int64_t kb = int64_t(kc) * kHChunk, ke = min(L.K, kb + kHChunk);
        const TI* __restrict__ x = static_cast<const TI*>(L.x);
        const TI* __restrict__ B0 = static_cast<const TI*>(L.B) + int64_t(16 * rt + g) * L.K;
        const TI* __restrict__ B1 = B0 + 8 * L.K;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
        constexpr int RB = NT <= 2 ? 4 : 2;  // 32-wide slices loaded together
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i0 = 0; i0 < 4; i0 += RB) {
          uint4 b0[RB], b1[RB], X[RB][NT];
#pragma unroll
          for (int q = 0; q < RB; ++q) {
            const int64_t kk = kb + 32 * warp + 256 * (i0 + q) + 8 * tig;
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
            if (kb + 32 * warp + 256 * (i0 + q) >= ke) break;
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
        if (!alive) break;
        TI* __restrict__ H = static_cast<TI*>(ga.H);
        float* __restrict__ P = ga.P + L.p0 + int64_t(rt) * L.nkc * 16 * TT;
        for (int idx = ctid; idx < 16 * TT; idx += kDW * 32) {
          const int m = idx & 15, t = idx >> 4;
          float v = 0.f;
#pragma unroll
          for (int w = 0; w < kDW; ++w) v += red[(w * 16 + m) * TT + t];
          if (L.nkc == 1) {
            if (t < ga.M) H[int64_t(t) * ga.ldh + L.hcol + 16 * rt + m] = from_f<TI>(v);
          } else {
            __stcg(P + int64_t(kc) * 16 * TT + idx, v);
          }
        }
        bool publish = L.nkc == 1;
        if (!publish) {
          __threadfence();
          alive = consumer_sync(cbar, cphase);
          if (!alive) break;
          if (ctid == 0) {
            const unsigned done = atomicAdd(ga.ctrl + kCtlTile + L.tile0 + rt, 1u);
            s_flag = done == unsigned(L.nkc - 1);
            __threadfence();
          }
          alive = consumer_sync(cbar, cphase);
          if (!alive) break;
          publish = s_flag != 0;
          if (publish) {
            // the last chunk of this tile: add the partials in chunk order
            for (int idx = ctid; idx < 16 * TT; idx += kDW * 32) {
              const int m = idx & 15, t = idx >> 4;
              if (t >= ga.M) continue;
              float v = 0.f;
              for (int q = 0; q < L.nkc; ++q) v += __ldcg(P + int64_t(q) * 16 * TT + idx);
              H[int64_t(t) * ga.ldh + L.hcol + 16 * rt + m] = from_f<TI>(v);
            }
          }
        }
        if (publish) {
          __threadfence();
          alive = consumer_sync(cbar, cphase);
          if (!alive) break;
          if (ctid == 0) atomicAdd(ga.ctrl + kCtlReady + rec.layer, 1u);
        } else {
          alive = consumer_sync(cbar, cphase);  // red may be rewritten
          if (!alive) break;
        }
        continue;
      }

      // ---- a stage of a Y item
      const int mt = L.mt, wpm = kDW / mt, wm = warp % mt, wk = warp / mt;
      if (rec.first) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
      }
      const uint32_t base = smem_u32(smem + size_t(sl) * ga.slot);
      if (rec.kind == ST_SPARSE) {
        const int steps = rec.b * (L.bq >> 4);
        const int rb = L.ft * 2;  // value row bytes
        const uint32_t vslot = (uint32_t(L.sb * L.bq * L.ft * 2) + 1023u) & ~1023u;
        const uint32_t xb = uint32_t(TT * L.bq * 2);
        for (int u = wk; u < steps; u += wpm) {
          const int row = 16 * u;
          const int j = row / L.bq, kin = row - j * L.bq;
          uint32_t af[4];
          ldsm_x4_trans(base + swz_offset(row + (lj >> 1) * 8 + li, 2 * wm + (lj & 1), rb), af[0], af[1], af[2],
                        af[3]);
          const uint32_t xt = base + vslot + uint32_t(j) * xb;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            uint32_t b0, b1;
            ldsm_x2(xt + swz_offset(8 * nt + li, (kin >> 3) + (lj & 1), L.bq * 2), b0, b1);
            mma16816<TI>::run(acc[nt], af, b0, b1);
          }
        }
      } else if (rec.kind == ST_LOWRANK) {
        if (cur_h != rec.layer) {
          // H of this layer: wait until all its tiles are written, then copy
          if (ctid == 0) {
            const unsigned long long t0 = globaltimer_ns();
            while (ld_acquire_gpu_u32(ga.ctrl + kCtlReady + rec.layer) < unsigned(L.n_rt)) {
              if (globaltimer_ns() - t0 > ga.wait_ns) {
                atomicOr(&g_status_dec, SLR_TIMEOUT_BIT);  // y of this layer is not valid
                break;
              }
              __nanosleep(64);
            }
          }
          alive = consumer_sync(cbar, cphase);
          if (!alive) break;
          const TI* __restrict__ H = static_cast<const TI*>(ga.H);
          const int nch = L.r >> 3;  // 16-byte chunks of a row
          for (int idx = ctid; idx < TT * nch; idx += kDW * 32) {
            const int t = idx / nch, c8 = idx - t * nch;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (t < ga.M) v = __ldcg(reinterpret_cast<const uint4*>(H + int64_t(t) * ga.ldh + L.hcol + 8 * c8));
            st_shared_v4(hb0 + uint32_t((c8 >> 3) * TT * 128) + swz_offset(t, c8 & 7, 128), v);
          }
          alive = consumer_sync(cbar, cphase);
          if (!alive) break;
          cur_h = rec.layer;
        }
        const int per = L.kc >> 4;
        const int steps = rec.b * per;
        const uint32_t cb = uint32_t(L.ft * L.kc * 2);
        for (int u = wk; u < steps; u += wpm) {
          const int c = u / per, k16 = u - c * per;
          const int kg = (rec.a + c) * L.kc + 16 * k16;  // rank column
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
      if (rec.last) {
        // ---- epilogue: add the warps' partial sums (k-part order), bias, store
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            red[(wk * L.ft + 16 * wm + g + ((e & 2) ? 8 : 0)) * TT + 8 * nt + 2 * tig + (e & 1)] = acc[nt][e];
        alive = consumer_sync(cbar, cphase);
        if (!alive) break;
        const int64_t n0 = int64_t(rec.item) * L.ft;
        const TI* __restrict__ bias = static_cast<const TI*>(L.bias);
        TI* __restrict__ y = static_cast<TI*>(L.y);
        for (int idx = ctid; idx < L.ft * TT; idx += kDW * 32) {
          const int n = idx % L.ft, t = idx / L.ft;
          if (t >= ga.M || n0 + n >= L.N) continue;
          float v = 0.f;
          for (int w = 0; w < wpm; ++w) v += red[(w * L.ft + n) * TT + t];
          if (bias) v += to_f(bias[n0 + n]);
          y[int64_t(t) * L.ldy + n0 + n] = from_f<TI>(v);
        }
        alive = consumer_sync(cbar, cphase);
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
      ga.ctrl[kCtlQueue] = 0;
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
  return 1024 + size_t(stages) * slot + hbuf + size_t(128) * tt * 4 + (2 * kDMaxStages + 1) * 8 +
         kDMaxStages * sizeof(DStage);
}

int dec_device_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 1;
  }
  return n;
}

// Shape of layer i (everything that fixes its arithmetic order) and its share
// of the launch's items, control words and workspace.  Returns false if the
// layer is outside what the kernel handles.
bool plan_layer(const RowblockArgs& in, int tt, DecodePlan& p, int i, int& items_h, int& tiles, int64_t& pfl,
                int64_t& hcol) {
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
  L.hcol = int(hcol);
  hcol += round_up(L.r, 64);
  L.tile0 = tiles;
  tiles += L.n_rt;
  L.p0 = pfl;
  if (L.nkc > 1) pfl += int64_t(L.n_rt) * L.nkc * 16 * tt;
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
    if (!plan_layer(layers[i], p.tt, p, i, items_h, tiles, pfl, hcol)) return false;
  }
  if (kCtlTile + tiles > kCtlWords) return false;
  int items = items_h;
  for (int i = 0; i < n; ++i) {
    p.a.L[i].y0 = items;
    items += p.a.L[i].ny;
  }
  p.a.M = M;
  p.a.n = n;
  p.a.n_h = items_h;
  p.a.n_items = items;
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
  // two CTAs per SM when at least 4 slots fit in half of the shared memory, else one
  const size_t half = 112 * 1024;
  int stages = kDMaxStages;
  while (stages > 4 && dec_smem(stages, p.a.slot, p.a.hbuf, p.tt) > half) --stages;
  if (dec_smem(stages, p.a.slot, p.a.hbuf, p.tt) > half || p.tt > 16) {
    stages = kDMaxStages;
    while (stages > 3 && dec_smem(stages, p.a.slot, p.a.hbuf, p.tt) > 227 * 1024) --stages;
  }
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
  // CTAs per SM at this shared-memory size (cached per kernel instance)
  thread_local size_t c_smem = 0;
  thread_local int c_occ = 0;
  if (c_smem != p.smem) {
    SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(p.smem)));
    SLR_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c_occ, kern, kDThreads, p.smem));
    c_smem = p.smem;
  }
  const int occ = c_occ;
  const int64_t ctas = std::min<int64_t>(p.a.n_items, int64_t(dec_device_sms()) * std::max(occ, 1));
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
      rc = make_tmap_2d(&maps.v[i], in.values, dtype, uint64_t(L.bp), uint64_t(in.nnz) * L.bq, uint64_t(L.bp) * 2,
                        uint32_t(L.ft), uint32_t(L.sb * L.bq));
      if (rc) return rc;
      rc = make_tmap_2d(&maps.v1[i], in.values, dtype, uint64_t(L.bp), uint64_t(in.nnz) * L.bq,
                        uint64_t(L.bp) * 2, uint32_t(L.ft), uint32_t(L.bq));
      if (rc) return rc;
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
