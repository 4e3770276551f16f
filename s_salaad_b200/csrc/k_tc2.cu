// Large-token-batch path on CTA pairs: the fused S+LR kernel with 2-SM
// tcgen05 MMAs (cta_group::2, M = 256 tokens per pair).
//
// Same work decomposition as tc_rowblock_kernel (k_tc.cu): one work item =
// a token tile x a group of G = 256/bp consecutive block-rows of the row
// list, each distinct column of the group is one stage (taken from the
// layer's column schedule by three producer warps that each own two ring
// slots, or merged from col[] by one thread without a schedule), each run of
// consecutive present rows one MMA, then the low-rank chunks as N = 256
// MMAs, all into one fp32 TMEM accumulator.
// What changes on a pair of SMs:
//   * the token tile is 256: each CTA loads the x (and H) rows of its own 128
//     tokens and keeps those 128 accumulator rows in its own TMEM;
//   * the B operand is split by N halves between the two CTAs.  Value blocks
//     are therefore stored as two half-width N-atoms (bp/2 columns each); for
//     a run of `len` rows (2*len atoms) the leader loads the first len atoms
//     and the peer the last len, both into the same packed positions, and the
//     A rows of the low-rank step are split 128/128;
//   * only the leader issues MMAs; TMA loads of both CTAs complete on the
//     leader's barriers; MMA completions are multicast to both CTAs.
// Per stage each SM moves at most 32 KB (x or H tile 16 KB + its half of the
// B operand), and each MMA reads half as much B from each SM's shared memory.
//
// Reference counterparts: _bsr_body (ssalaad/tilelang_sparse/addmm_inplace.py:
// 41-82) and the F.linear pair + bias of _LRSLinearLRBlockCUDA.forward
// (ssalaad/efficient/ls_linear.py:124-137).
#include <algorithm>

#include "internal.hpp"
#include "tcgen05.cuh"

namespace slr {
namespace {
using namespace tc;

__device__ unsigned g_status_tc2 = 0;

constexpr int kThreads = 256;   // warps 0, 6, 7 load operands, 1 issues MMAs, 2-5 epilogue
constexpr int kProducers = 3;   // TMA warps working from a column schedule
constexpr int kStages = 6;      // ring slots (a multiple of kProducers)
constexpr uint32_t kMetaLR = 1u << 30;
constexpr uint32_t kMetaLast = 1u << 31;
// Layers with a low-rank term (fused mode): the present rows of a column
// form ONE MMA over the span from the first to the last of them (N up to 256),
// absent rows inside it zero atoms (a TMA box just past the values tensor,
// zero-filled).  An MMA with N <= 128 costs about the same whatever N, and
// the issuing thread's fixed span code replaces a data-dependent loop over
// runs: on B200, cfg4 (64-wide blocks) 0.752 -> 0.688 ms and cfg3-T2048
// (32-wide) 0.289 -> 0.227 ms per combine.  x * 0 adds exactly zero to a
// finite accumulator (a non-finite x already reaches every output through H).
constexpr uint32_t kMetaSpan = 1u << 29;
constexpr int kSpanRows = 8;  // rows per span window (8: one span per column; measured best)
constexpr uint32_t kSpanMask = (1u << kSpanRows) - 1u;

// Atoms of the window spans of an 8-row column mask.
__device__ __forceinline__ uint32_t span_atoms(uint32_t mask) {
  uint32_t n = 0;
#pragma unroll
  for (int w = 0; w < 8 / kSpanRows; ++w) {
    const uint32_t mw = (mask >> (kSpanRows * w)) & kSpanMask;
    if (mw) n += uint32_t((31 - __clz(mw)) - (__ffs(mw) - 1) + 1);
  }
  return n;
}
// Atoms of the spans of the windows before row w0's window.
__device__ __forceinline__ uint32_t span_atoms_below(uint32_t mask, int w0) {
  return span_atoms(mask & ((1u << w0) - 1u));
}
// After the ring: barriers and metadata, then (multi-GPU) the epilogue
// staging tiles of the 4 epilogue warps, 32 rows x block_p outputs each,
// laid out as the TMA store's swizzle (128B for block_p 64, 64B for 32).
constexpr uint32_t kEpiOff = 1024;
constexpr uint32_t epi_stage_bytes(int bp) { return 4u * 32u * uint32_t(bp) * 2u; }

struct Tc2Args {
  void* y;
  const void* bias;
  const int32_t* crow;
  const int32_t* col;
  const int32_t* rows;
  const uint32_t* plan;   // column schedule (slr_plan_stages) or null
  const int32_t* plan_start;
  int64_t M, ldy;
  int nrows, n_groups, n_mtiles, n_lr;
  PeerArgs peer;          // world > 1: tiles also go to the other ranks' y
  int xgrp;               // layers of a launch that read the same x share it
  int vrows;              // rows of the values tensor map (nnz * block_q); 0 = no window spans
};


// Several layers in one launch (same block shape, token count and mode):
// their work items are numbered one layer after the other, item0[l] being
// layer l's first, and dealt to the pairs as one list, so the launch has one
// persistent-schedule tail instead of one per layer.
constexpr int kTc2Layers = kMaxLaunchLayers;
// world > 1: TMA store maps of every rank's y at this rank's columns, per
// layer of the launch ([M, N] of the layer, box block_p x 32 rows); m[l][me]
// is layer l's local y.
struct YMaps {
  CUtensorMap m[kTc2Layers][kMaxRanks];
};
// Row groups of a launch that can be put in one heaviest-first order in
// shared memory at the start of the kernel.
constexpr int kOrderCap = 512;
struct Tc2Set {
  Tc2Args L[kTc2Layers];
  int n;
  int item0[kTc2Layers + 1];
};
// x tiles, value atoms, H tiles and A rows of each layer.
struct Tc2Maps {
  CUtensorMap x[kTc2Layers], v[kTc2Layers], h[kTc2Layers], a[kTc2Layers];
};

// Layer of work item `item` and the item's index within that layer.
__device__ __forceinline__ int tc2_layer_of(const Tc2Set& set, int item) {
  int l = 0;
  while (l + 1 < set.n && item >= set.item0[l + 1]) ++l;
  return l;
}

__device__ __forceinline__ void timeout2(volatile int* abort_flag) {
  atomicOr(&g_status_tc2, SLR_TIMEOUT_BIT);
  *abort_flag = 1;
}

template <int BP, int BQ, typename TI, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc2_rowblock_kernel(const __grid_constant__ Tc2Maps maps, const __grid_constant__ Tc2Set set,
                        const __grid_constant__ YMaps ym) {
  constexpr int G = 256 / BP;            // block-rows per item
  constexpr int KS = BQ < 64 ? BQ : 64;  // k per sparse stage
  constexpr int SUB = BQ / KS;
  constexpr int XW = KS * 2;             // x-tile row bytes
  constexpr int HW = BP;                 // row bytes of a half-block atom (bp/2 columns)
  constexpr uint32_t X_BYTES = 128 * XW;
  constexpr uint32_t POS = KS * HW;      // one half-block atom column
  constexpr uint32_t H_BYTES = 128 * 128;
  constexpr uint32_t AR_ROW = BP * 128;  // one block-row's A rows, 64 k
  constexpr uint32_t A_SLOT = 16384;
  constexpr uint32_t B_SLOT = (G * POS > (G / 2) * AR_ROW) ? G * POS : (G / 2) * AR_ROW;
  constexpr uint32_t STAGE = A_SLOT + B_SLOT;
  constexpr int STAGES = kStages;
  static_assert(STAGES * STAGE <= 200 * 1024 && STAGES % kProducers == 0, "ring size");
  constexpr uint32_t ACC = 256;
  constexpr uint32_t IDESC_SP = idesc_f16<TI>(256, 0, true);  // N set per run
  constexpr uint32_t IDESC_LR = idesc_f16<TI>(256, 256, false);
  static_assert(BP == 32 || BP == 64, "2-SM path: block_p 32 or 64");
  static_assert(STAGE % 1024 == 0 && POS % 256 == 0, "stage alignment");
  // Schedule columns per sparse stage: a 32-deep column fills half a stage,
  // so two of them share one (same MMAs in the same order, half the per-stage
  // barrier, TMA and issue overhead).
  constexpr int CPS = BQ == 32 ? 2 : 1;
  static_assert(CPS * X_BYTES <= A_SLOT && CPS * G * POS <= B_SLOT && G <= 8, "stage holds CPS columns");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* meta = reinterpret_cast<uint32_t*>(tempty + 2);
  uint32_t* tmem_slot = meta + STAGES;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_peer_fail;  // an epilogue warp gave up waiting for the other ranks

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // 4 epilogue warps in each CTA of the pair
    }
    fence_mbar_init();
    s_abort = 0;
    s_peer_fail = 0;
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, 2 * ACC);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // The next kernel of the stream (the next projection's combine or x*B^T,
  // launched as a programmatic dependent) may take SMs as this persistent
  // grid's CTAs leave; it reads what this grid writes only after its own
  // griddepcontrol.wait.
  pdl_launch_dependents();
  if (warp >= 2 && warp < 6) {
    const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;
    for (uint32_t c = 0; c < 2 * ACC; c += 16) tmem_st16_zero(tmem + lane_base + c);
    tmem_st_wait();
  }
  tc_fence_before();
  cluster_sync();  // both halves of every accumulator are zero before the first MMA
  tc_fence_after();

  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int n_items = set.item0[set.n];

  // Items of a multi-layer launch in one order: the layers that read one x
  // run together, the inputs whose heaviest row group is heaviest first, and
  // within an input the row groups go heaviest first by stages (schedule
  // columns + rank chunks; ties by layer, then group); item i is token tile
  // i % n_mtiles of the group ranked i / n_mtiles.  x, which every row group
  // of its layers re-reads, is then the L2 working set of one input at a
  // time: on B200 with LLaMA-7B-shaped layers at 4096 tokens the launch reads
  // 0.69 GB from DRAM (its operands once) where one heaviest-first order over
  // all layers read 2.0 GB, for 4 % more time.  Every CTA computes the same
  // order in shared memory, and an item's arithmetic does not depend on its
  // place.
  __shared__ uint32_t s_order[kOrderCap], s_key[kOrderCap];
  __shared__ uint32_t s_xmax[kTc2Layers];
  int n_groups_all = 0;
  for (int l = 0; l < set.n; ++l) n_groups_all += set.L[l].n_groups;
  // (one layer: its row groups are already planned heaviest first)
  const bool ordered = set.n > 1 && set.L[0].plan != nullptr && n_groups_all <= kOrderCap;
  if (ordered) {
    if (threadIdx.x < kTc2Layers) s_xmax[threadIdx.x] = 0u;
    __syncthreads();
    for (int gs = threadIdx.x; gs < n_groups_all; gs += blockDim.x) {
      int l = 0, gi = gs;
      while (gi >= set.L[l].n_groups) gi -= set.L[l++].n_groups;
      const uint32_t w = min(uint32_t(__ldg(set.L[l].plan_start + gi + 1) - __ldg(set.L[l].plan_start + gi) +
                                      set.L[l].n_lr), 0xFFFFFu);
      s_key[gs] = w;
      atomicMax(&s_xmax[set.L[l].xgrp], w);
    }
    __syncthreads();
    for (int gs = threadIdx.x; gs < n_groups_all; gs += blockDim.x) {
      int l = 0, gi = gs;
      while (gi >= set.L[l].n_groups) gi -= set.L[l++].n_groups;
      // the input's place: inputs with a heavier heaviest group first, ties by input
      const int xg = set.L[l].xgrp;
      int xr = 0;
      for (int q = 0; q < set.n; ++q) {
        const int xq = set.L[q].xgrp;
        bool first = true;  // q is the first layer of its input
        for (int u = 0; u < q; ++u) first = first && set.L[u].xgrp != xq;
        if (first && xq != xg && (s_xmax[xq] > s_xmax[xg] || (s_xmax[xq] == s_xmax[xg] && xq < xg))) ++xr;
      }
      s_order[gs] = (uint32_t(xr) << 20) | (0xFFFFFu - s_key[gs]);  // ascending = the order above
    }
    __syncthreads();
    for (int gs = threadIdx.x; gs < n_groups_all; gs += blockDim.x) s_key[gs] = s_order[gs];
    __syncthreads();
    for (int gs = threadIdx.x; gs < n_groups_all; gs += blockDim.x) {
      const uint32_t k = s_key[gs];
      int rk = 0;
      for (int j = 0; j < n_groups_all; ++j) {
        const uint32_t kj = s_key[j];
        rk += (kj < k || (kj == k && j < gs)) ? 1 : 0;
      }
      int l = 0, gi = gs;
      while (gi >= set.L[l].n_groups) gi -= set.L[l++].n_groups;
      s_order[rk] = (uint32_t(l) << 16) | uint32_t(gi);
    }
    __syncthreads();
  }
  // layer, row group and token tile of work item `item`
  auto decode_item = [&](int item, int& li, int& gi, int& mt) {
    if (ordered) {
      const int nm = set.L[0].n_mtiles;
      const int gs = item / nm;
      mt = item - gs * nm;
      const uint32_t e = s_order[gs];
      li = int(e >> 16);
      gi = int(e & 0xffffu);
    } else {
      li = tc2_layer_of(set, item);
      const int litem = item - set.item0[li];
      gi = litem / set.L[li].n_mtiles;
      mt = litem - gi * set.L[li].n_mtiles;
    }
  };

  if (warp == 0 || warp >= 6) {
    // ------------------------------------------------------- TMA producers
    if (lane == 0)
      for (int l = 0; l < set.n; ++l) {
        tma_prefetch_desc(&maps.x[l]);
        if (set.L[l].crow) tma_prefetch_desc(&maps.v[l]);
        if (set.L[l].n_lr) {
          tma_prefetch_desc(&maps.h[l]);
          tma_prefetch_desc(&maps.a[l]);
        }
      }
    if (set.L[0].plan) {
      // With the column schedule producer warp p (0, 6, 7 -> 0, 1, 2) fills
      // the stages g with g % 3 == p: always the same two ring slots, so its
      // waits on them stay in phase order.  Each CTA loads its own 128 token
      // rows and its half of the B operand; loads complete on the leader's
      // barrier.
      // A warp's stages pass through a three-deep software pipeline: before
      // it waits for the slot of stage k it requests the schedule records of
      // stage k+2 and the value-block indices of stage k+1 (which need k+1's
      // records, requested one step earlier); an item's row-group bounds and
      // row indices are requested one item ahead.  The latency of these
      // dependent global loads then overlaps the slot waits instead of
      // adding to every slot's round trip.
      const int pw = warp == 0 ? 0 : warp - 5;
      struct ItemCtx {
        int kr, li, gi, mt, p0, p1, rw;
        uint32_t g0;  // the item's first stage in the launch's stage sequence
        bool valid;
      };
      struct Stage {
        int li, mt, gcount, rw, n_sp, n_st, s, kb, nc;
        uint32_t gg;  // stage index in the launch's stage sequence
        uint32_t rec[CPS], firsts[CPS];
        int blk[CPS];
        bool valid;
      };
      auto load_ctx = [&](int kr) {
        ItemCtx c;
        const int item = snake_item(kr, pair, npairs);
        c.kr = kr;
        c.valid = item < n_items;
        c.g0 = 0;
        c.li = c.gi = c.mt = c.p0 = c.p1 = c.rw = 0;
        if (c.valid) {
          decode_item(item, c.li, c.gi, c.mt);
          const Tc2Args& a = set.L[c.li];
          c.p0 = __ldg(a.plan_start + c.gi);
          c.p1 = __ldg(a.plan_start + c.gi + 1);
          const int r0 = c.gi * G;
          c.rw = lane < min(G, a.nrows - r0) ? (a.rows ? __ldg(a.rows + r0 + lane) : r0 + lane) : 0;
        }
        return c;
      };
      auto n_sp_of = [&](const ItemCtx& c) { return ((c.p1 - c.p0 + CPS - 1) / CPS) * SUB; };
      auto n_st_of = [&](const ItemCtx& c) { return max(n_sp_of(c) + set.L[c.li].n_lr, 1); };
      // iterator over this warp's stages: stage s_it of item ci (cn: the next item)
      ItemCtx ci = load_ctx(0), cn = load_ctx(1);
      int s_it = pw;
      auto settle = [&]() {
        while (ci.valid && s_it >= n_st_of(ci)) {
          const int n = n_st_of(ci);
          s_it -= n;
          const uint32_t g0 = ci.g0 + uint32_t(n);
          ci = cn;
          ci.g0 = g0;
          cn = load_ctx(ci.kr + 1);
        }
      };
      // the iterator's stage; requests its schedule records
      auto make_stage = [&](Stage& st) {
        st.valid = ci.valid;
        st.li = ci.li;
        st.mt = ci.mt;
        st.rw = ci.rw;
        st.s = s_it;
        st.gg = ci.g0 + uint32_t(s_it);
        st.kb = st.nc = 0;
#pragma unroll
        for (int c = 0; c < CPS; ++c) {
          st.rec[c] = st.firsts[c] = 0u;
          st.blk[c] = 0;
        }
        if (!st.valid) return;
        const Tc2Args& a = set.L[ci.li];
        st.gcount = min(G, a.nrows - ci.gi * G);
        st.n_sp = n_sp_of(ci);
        st.n_st = n_st_of(ci);
        if (s_it < st.n_sp) {
          st.kb = ci.p0 + (s_it / SUB) * CPS;
          st.nc = min(CPS, ci.p1 - st.kb);
#pragma unroll
          for (int c = 0; c < CPS; ++c)
            if (c < st.nc) {
              st.rec[c] = __ldg(a.plan + 2 * (st.kb + c));
              st.firsts[c] = __ldg(a.plan + 2 * (st.kb + c) + 1);
            }
        }
      };
      // requests the value-block index of this lane's row in each column
      auto fetch_blocks = [&](Stage& st) {
        if (!st.valid || st.s >= st.n_sp) return;
        const uint32_t* plan = set.L[st.li].plan;
#pragma unroll
        for (int c = 0; c < CPS; ++c) {
          const uint32_t mask = st.rec[c] >> 16;
          if (c < st.nc && ((mask >> lane) & 1u))
            st.blk[c] = int(__ldg(plan + st.firsts[c] + __popc(mask & ((1u << lane) - 1u))));
        }
      };
      bool waited = false;
      // waits for the stage's slot and issues its loads; false on a timeout
      auto issue = [&](const Stage& st) -> bool {
        const Tc2Args& a = set.L[st.li];
        const CUtensorMap* tm_x = &maps.x[st.li];
        const CUtensorMap* tm_v = &maps.v[st.li];
        const CUtensorMap* tm_h = &maps.h[st.li];
        const CUtensorMap* tm_a = &maps.a[st.li];
        const int s = st.s;
        const uint32_t slot = st.gg % STAGES, ph = (st.gg / STAGES) & 1;
        int ok = lane == 0 ? int(mbar_wait(&empty[slot], ph ^ 1)) : 1;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) return false;
        const uint32_t fb = mapa(smem_u32(&full[slot]), 0);
        uint8_t* adst = smem + slot * STAGE;
        const bool last = s == st.n_st - 1;
        const int m0 = st.mt * 256 + int(rank) * 128;  // this CTA's tokens
        if (s < st.n_sp) {
          const int sub = s % SUB;
          const bool spans = (BP == 32 || BP == 64) && MODE == MODE_FUSED && a.n_lr > 0 && a.vrows > 0;
          uint32_t atoms = 0;
#pragma unroll
          for (int c = 0; c < CPS; ++c)
            atoms += spans ? span_atoms(st.rec[c] >> 16) : uint32_t(__popc(st.rec[c] >> 16));
          if (lane == 0) {
            if (leader) {
              uint32_t mm = st.rec[0] >> 16;
              if (CPS == 2) mm |= (st.rec[CPS - 1] >> 16) << 8;
              meta[slot] = mm | (last ? kMetaLast : 0u) | (spans ? kMetaSpan : 0u);
              mbar_arrive_expect_tx(&full[slot], 2 * (uint32_t(st.nc) * X_BYTES + atoms * POS));
            }
#pragma unroll
            for (int c = 0; c < CPS; ++c)
              if (c < st.nc) tma2_load_2d(adst + c * X_BYTES, tm_x, int(st.rec[c] & 0xffffu) * BQ + sub * KS, m0, fb);
          }
          uint32_t off = 0;  // this column's first atom in the stage's B slot
#pragma unroll
          for (int c = 0; c < CPS; ++c) {
            const uint32_t mask = st.rec[c] >> 16;
            if (spans) {
              // this row's span [f, l] (its window's first and last present rows):
              // its 2*len half-block atoms, the first len on the leader, the rest on
              // the peer; an absent row loads the box just past the values (zeros)
              const int w0 = lane & ~(kSpanRows - 1);
              const uint32_t mw = lane < 8 ? (mask >> w0) & kSpanMask : 0u;
              if (mw) {
                const int f = w0 + __ffs(mw) - 1, l = w0 + 31 - __clz(mw);
                if (lane >= f && lane <= l) {
                  const int len = l - f + 1;
                  const int p_run = int(off) + int(span_atoms_below(mask, w0));
                  const int brow = ((mask >> lane) & 1u) ? st.blk[c] * BQ + sub * KS : a.vrows;
#pragma unroll
                  for (int h = 0; h < 2; ++h) {
                    const int at = 2 * (lane - f) + h;
                    if (at / len == int(rank))
                      tma2_load_2d(adst + A_SLOT + (p_run + at - int(rank) * len) * POS, tm_v, h * (BP / 2), brow,
                                   fb);
                  }
                }
              }
              off += span_atoms(mask);
              continue;
            }
            if ((mask >> lane) & 1u) {
              // this row's run of consecutive present rows [j0, end): its 2*len
              // half-block atoms, the first len on the leader, the rest on the peer
              const uint32_t below = (1u << lane) - 1u, zeros = ~mask & below;
              const int j0 = zeros ? 32 - __clz(zeros) : 0;
              const int end = lane + __ffs(~(mask >> lane)) - 1;
              const int len = end - j0;
              const int p_run = int(off) + __popc(mask & ((1u << j0) - 1u));
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int at = 2 * (lane - j0) + h;
                if (at / len == int(rank))
                  tma2_load_2d(adst + A_SLOT + (p_run + at - int(rank) * len) * POS, tm_v, h * (BP / 2),
                               st.blk[c] * BQ + sub * KS, fb);
              }
            }
            off += uint32_t(__popc(mask));
          }
        } else if (s < st.n_sp + a.n_lr) {
          const int l = s - st.n_sp;
          if (!waited) {
            pdl_wait_primary();  // H comes from the preceding kernel
            waited = true;
          }
          if (lane == 0) {
            if (leader) {
              meta[slot] = kMetaLR | (last ? kMetaLast : 0u);
              mbar_arrive_expect_tx(&full[slot], 2 * H_BYTES + st.gcount * AR_ROW);
            }
            tma2_load_2d(adst, tm_h, l * 64, m0, fb);
          }
          const int jl = lane - int(rank) * (G / 2);
          if (jl >= 0 && jl < G / 2 && lane < st.gcount)
            tma2_load_2d(adst + A_SLOT + jl * AR_ROW, tm_a, l * 64, st.rw * BP, fb);
        } else if (lane == 0 && leader) {
          meta[slot] = kMetaLast;  // no block and no rank: the item still completes
          mbar_arrive(&full[slot]);
        }
        return true;
      };
      Stage d0, d1, d2;
      settle();
      make_stage(d0);
      s_it += kProducers;
      settle();
      make_stage(d1);
      fetch_blocks(d0);
      while (d0.valid) {
        s_it += kProducers;
        settle();
        make_stage(d2);   // records of stage k+2
        fetch_blocks(d1);  // block indices of stage k+1
        if (__shfl_sync(0xffffffffu, int(s_abort), 0)) break;  // another role gave up: unwind
        if (!issue(d0)) {
          if (lane == 0) timeout2(&s_abort);
          break;
        }
        d0 = d1;
        d1 = d2;
      }
    } else if (warp == 0 && lane == 0) {
      // (a launch without a schedule holds one layer)
      const Tc2Args& a = set.L[0];
      const CUtensorMap* tm_x = &maps.x[0];
      const CUtensorMap* tm_v = &maps.v[0];
      const CUtensorMap* tm_h = &maps.h[0];
      const CUtensorMap* tm_a = &maps.a[0];
      bool waited = false;
      uint32_t g = 0;
      for (int kr = 0, item = snake_item(0, pair, npairs); item < n_items && !s_abort; ++kr, item = snake_item(kr, pair, npairs)) {
        const int gi = item / a.n_mtiles, mt = item - gi * a.n_mtiles;
        const int r0 = gi * G;
        const int gcount = min(G, a.nrows - r0);
        const int m0 = mt * 256 + int(rank) * 128;  // this CTA's tokens
        int rw[G], ptr[G], end[G], cur[G];
#pragma unroll
        for (int j = 0; j < G; ++j) {
          rw[j] = j < gcount ? (a.rows ? a.rows[r0 + j] : r0 + j) : 0;
          ptr[j] = (a.crow && j < gcount) ? a.crow[rw[j]] : 0;
          end[j] = (a.crow && j < gcount) ? a.crow[rw[j] + 1] : 0;
          cur[j] = ptr[j] < end[j] ? __ldg(a.col + ptr[j]) : 0x7fffffff;
        }
        int c = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < G; ++j) c = min(c, cur[j]);
        bool published = false;
        while (c != 0x7fffffff && !s_abort) {
          uint32_t mask = 0;
          int blk[G];
#pragma unroll
          for (int j = 0; j < G; ++j) {
            blk[j] = ptr[j];
            if (cur[j] == c) {
              mask |= 1u << j;
              ++ptr[j];
              cur[j] = ptr[j] < end[j] ? __ldg(a.col + ptr[j]) : 0x7fffffff;
            }
          }
          int cn = 0x7fffffff;
#pragma unroll
          for (int j = 0; j < G; ++j) cn = min(cn, cur[j]);
          const uint32_t pc = __popc(mask);
          for (int sub = 0; sub < SUB; ++sub, ++g) {
            const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
            if (!mbar_wait(&empty[slot], ph ^ 1)) {
              timeout2(&s_abort);
              break;
            }
            const uint32_t fb = mapa(smem_u32(&full[slot]), 0);
            if (leader) {
              const bool last = cn == 0x7fffffff && a.n_lr == 0 && sub == SUB - 1;
              meta[slot] = mask | (last ? kMetaLast : 0u);
              mbar_arrive_expect_tx(&full[slot], 2 * (X_BYTES + pc * POS));
            }
            uint8_t* adst = smem + slot * STAGE;
            tma2_load_2d(adst, tm_x, c * BQ + sub * KS, m0, fb);
            // runs of consecutive rows: this CTA's len atoms of each run, packed
            uint32_t m = mask, p = 0;
            while (m) {
              const int j = __ffs(m) - 1;
              const int len = __ffs(~(m >> j)) - 1;
              m &= ~(((1u << len) - 1u) << j);
              for (int i = 0; i < len; ++i) {
                const int at = int(rank) * len + i;  // atom index within the run
                const int row = j + (at >> 1), half = at & 1;
                tma2_load_2d(adst + A_SLOT + (p + i) * POS, tm_v, half * (BP / 2), blk[row] * BQ + sub * KS, fb);
              }
              p += len;
            }
            published = true;
          }
          c = cn;
        }
        for (int l = 0; l < a.n_lr && !s_abort; ++l, ++g) {
          if (!waited) {
            pdl_wait_primary();  // H comes from the preceding kernel
            waited = true;
          }
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          if (!mbar_wait(&empty[slot], ph ^ 1)) {
            timeout2(&s_abort);
            break;
          }
          const uint32_t fb = mapa(smem_u32(&full[slot]), 0);
          if (leader) {
            meta[slot] = kMetaLR | (l == a.n_lr - 1 ? kMetaLast : 0u);
            mbar_arrive_expect_tx(&full[slot], 2 * H_BYTES + gcount * AR_ROW);
          }
          uint8_t* adst = smem + slot * STAGE;
          tma2_load_2d(adst, tm_h, l * 64, m0, fb);
          for (int j = int(rank) * (G / 2); j < (int(rank) + 1) * (G / 2) && j < gcount; ++j)
            tma2_load_2d(adst + A_SLOT + (j - int(rank) * (G / 2)) * AR_ROW, tm_a, l * 64, rw[j] * BP, fb);
          published = true;
        }
        if (!published && !s_abort) {
          // No block and no rank: a stage without loads so the item still completes.
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          if (!mbar_wait(&empty[slot], ph ^ 1)) {
            timeout2(&s_abort);
            break;
          }
          if (leader) {
            meta[slot] = kMetaLast;
            mbar_arrive(&full[slot]);
          }
          ++g;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      uint32_t g = 0, it = 0;
      for (int kr = 0, item = snake_item(0, pair, npairs); item < n_items && !s_abort; ++kr, item = snake_item(kr, pair, npairs), ++it) {
        const uint32_t buf = it & 1, tph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1)) {
          timeout2(&s_abort);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * ACC;
        while (true) {
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          if (!mbar_wait(&full[slot], ph)) {
            timeout2(&s_abort);
            break;
          }
          tc_fence_after();
          const uint32_t m = meta[slot];
          const uint32_t abase = smem_u32(smem + slot * STAGE);
          const uint32_t bbase = abase + A_SLOT;
          if (m & kMetaLR) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma2_f16(d, sdesc(abase + kk * 32, 16, 1024, 2), sdesc(bbase + kk * 32, 16, 1024, 2), IDESC_LR, 1u);
          } else if ((BP == 32 || BP == 64) && (m & kMetaSpan)) {
            // spans: one MMA per window (one column) with present rows
            uint32_t p = 0;
#pragma unroll
            for (int c = 0; c < CPS; ++c) {
              const uint32_t mask = (m >> (8 * c)) & 0xffu;
              const uint32_t xa = abase + uint32_t(c) * X_BYTES;
#pragma unroll
              for (int w = 0; w < 8 / kSpanRows; ++w) {
                const uint32_t mw = (mask >> (kSpanRows * w)) & kSpanMask;
                if (mw) {
                  const int f = kSpanRows * w + __ffs(mw) - 1;
                  const int len = kSpanRows * w + 31 - __clz(mw) - f + 1;
                  const uint32_t idesc = IDESC_SP | (uint32_t(len * BP) >> 3) << 17;
#pragma unroll
                  for (int kk = 0; kk < KS / 16; ++kk) {
                    const uint64_t ad = sdesc(xa + kk * 32, 16, 8 * XW, layout_for(XW));
                    const uint64_t bd = sdesc(bbase + p * POS + kk * 16 * HW, POS, 8 * HW, layout_for(HW));
                    umma2_f16(d + f * BP, ad, bd, idesc, 1u);
                  }
                  p += uint32_t(len);
                }
              }
            }
          } else {
            // up to CPS schedule columns: row masks in bits [0, 8) and [8, 16),
            // x tiles one after another in the A slot, atoms packed in the B slot
            uint32_t p = 0;
#pragma unroll
            for (int c = 0; c < CPS; ++c) {
              uint32_t mask = (m >> (8 * c)) & 0xffu;
              const uint32_t xa = abase + uint32_t(c) * X_BYTES;
              while (mask) {
                const int j = __ffs(mask) - 1;
                const int len = __ffs(~(mask >> j)) - 1;
                mask &= ~(((1u << len) - 1u) << j);
                const uint32_t idesc = IDESC_SP | (uint32_t(len * BP) >> 3) << 17;
#pragma unroll
                for (int kk = 0; kk < KS / 16; ++kk) {
                  const uint64_t ad = sdesc(xa + kk * 32, 16, 8 * XW, layout_for(XW));
                  const uint64_t bd = sdesc(bbase + p * POS + kk * 16 * HW, POS, 8 * HW, layout_for(HW));
                  umma2_f16(d + j * BP, ad, bd, idesc, 1u);
                }
                p += len;
              }
            }
          }
          umma2_commit_both(&empty[slot]);
          ++g;
          if (m & kMetaLast) break;
        }
        umma2_commit_both(&tfull[buf]);
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;
    const uint32_t lane_base = uint32_t(32 * q) << 16;
    const int row = 32 * q + lane;
    const Tc2Args& a0 = set.L[0];  // its peer args carry the launch's signal slots
    const uint32_t te0 = mapa(smem_u32(&tempty[0]), 0);
    constexpr int kCpr = BP / 8;  // 16-byte chunks of a row's BP outputs
    // 16-byte chunk c of staging row r, as TMA's 128B (BP 64) / 64B (BP 32) swizzle places it
    auto epi_swz = [](int r, int c) { return BP == 64 ? (c ^ (r & 7)) : (c ^ ((r >> 1) & 3)); };
    uint4* stage_w = reinterpret_cast<uint4*>(smem + STAGES * STAGE + kEpiOff) + (warp - 2) * 32 * kCpr;
    // Multi-GPU: this call's arrival at every rank, then (before the first
    // store into a peer) the wait for every rank's arrival.
    const int world = a0.peer.world;
    unsigned long long call_no = 0;  // this rank's call of the layer, 1-based
    bool peer_live = world > 1, arrived = false;
    if (world > 1) {
      pdl_wait_primary();  // the preceding wait of this rank has counted its calls
      call_no = *reinterpret_cast<volatile unsigned long long*>(a0.peer.my_sig + kSigCalls) + 1;
      if (blockIdx.x == 0 && warp == 2 && lane == 0) {
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
          if (p < world) st_release_sys(a0.peer.sig[p] + kSigArrive + a0.peer.me, call_no);
      }
    }
    auto wait_arrivals = [&]() {
      int ok = lane == 0 ? int(wait_words(a0.peer.my_sig + kSigArrive, world, call_no, a0.peer.wait_ns, true)) : 1;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0) {
          atomicOr(&g_status_tc2, SLR_TIMEOUT_BIT);
          s_peer_fail = 1;
        }
        peer_live = false;  // keep the local result, leave the peers alone
      }
      arrived = true;
    };
    uint32_t it = 0;
    for (int kr = 0, item = snake_item(0, pair, npairs); item < n_items; ++kr, item = snake_item(kr, pair, npairs), ++it) {
      int li, gi, mt;
      decode_item(item, li, gi, mt);
      const Tc2Args& a = set.L[li];
      TI* __restrict__ y = static_cast<TI*>(a.y);
      const TI* __restrict__ bias = static_cast<const TI*>(a.bias);
      const int r0 = gi * G;
      const int gcount = min(G, a.nrows - r0);
      const uint32_t buf = it & 1, tph = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[buf], tph, 256)) {
        if (lane == 0) timeout2(&s_abort);
        break;
      }
      tc_fence_after();
      if (peer_live && !arrived) wait_arrivals();
      const int64_t tok = int64_t(mt) * 256 + int64_t(rank) * 128 + row;
      const uint32_t acc = tmem + lane_base + buf * ACC;
      for (int j = 0; j < G; ++j) {
        if (j >= gcount) {
#pragma unroll
          for (int c0 = 0; c0 < BP; c0 += 16) tmem_st16_zero(acc + j * BP + c0);
          continue;
        }
        const int br = a.rows ? a.rows[r0 + j] : r0 + j;
        TI* yr = y + tok * a.ldy + int64_t(br) * BP;
        const TI* bb = bias ? bias + int64_t(br) * BP : nullptr;
        // Multi-GPU: the warp's 32 rows x BP features go to shared memory and
        // leave as one TMA store per destination (its own y and every peer's
        // y over NVLink); the TMA engine keeps the remote writes in flight
        // while the warps move on.
        const bool staged = world > 1;
        if (staged) {
          if (lane == 0) bulk_wait_read_all();  // the previous tile has left the stage
          __syncwarp();
        }
#pragma unroll
        for (int c0 = 0; c0 < BP; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(acc + j * BP + c0, r);
          tmem_ld_wait();
          tmem_st16_zero(acc + j * BP + c0);
          if (tok < a.M) {
            float v[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = __uint_as_float(r[e]);
            if (MODE == MODE_ADDMM || bb != nullptr) {
              const TI* src = MODE == MODE_ADDMM ? yr + c0 : bb + c0;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint4 o = MODE == MODE_ADDMM ? *reinterpret_cast<const uint4*>(src + 8 * h)
                                                   : __ldg(reinterpret_cast<const uint4*>(src + 8 * h));
                const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = unpack2(ow[e], (TI*)nullptr);
                  v[8 * h + 2 * e] = MODE == MODE_ADDMM ? f.x + v[8 * h + 2 * e] : v[8 * h + 2 * e] + f.x;
                  v[8 * h + 2 * e + 1] = MODE == MODE_ADDMM ? f.y + v[8 * h + 2 * e + 1] : v[8 * h + 2 * e + 1] + f.y;
                }
              }
            }
            uint4 o0, o1;
            o0.x = pack2(v[0], v[1], (TI*)nullptr);
            o0.y = pack2(v[2], v[3], (TI*)nullptr);
            o0.z = pack2(v[4], v[5], (TI*)nullptr);
            o0.w = pack2(v[6], v[7], (TI*)nullptr);
            o1.x = pack2(v[8], v[9], (TI*)nullptr);
            o1.y = pack2(v[10], v[11], (TI*)nullptr);
            o1.z = pack2(v[12], v[13], (TI*)nullptr);
            o1.w = pack2(v[14], v[15], (TI*)nullptr);
            if (staged) {
              const int c = c0 / 8;
              stage_w[lane * kCpr + epi_swz(lane, c + 0)] = o0;
              stage_w[lane * kCpr + epi_swz(lane, c + 1)] = o1;
            } else {
              reinterpret_cast<uint4*>(yr + c0)[0] = o0;
              reinterpret_cast<uint4*>(yr + c0)[1] = o1;
            }
          }
        }
        if (staged) {
          fence_proxy_async_smem();  // the stage's generic writes, before the TMA reads them
          __syncwarp();
          const int64_t tok0 = tok - lane;  // the warp's first row (rows >= M are clipped)
          if (lane == 0 && tok0 < a.M) {
#pragma unroll
            for (int p = 0; p < kMaxRanks; ++p)
              if (p < world && (p == a0.peer.me || peer_live))
                tma_store_2d(&ym.m[li][p], stage_w, br * BP, int(tok0));
            bulk_commit();
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(te0 + buf * 8);
    }
    if (world > 1) {
      // Completion: after every rank arrived (so the count belongs to this
      // call) and this CTA's stores are visible system-wide.  A CTA that gave
      // up on a wait first marks the call as failed at every rank, so their
      // waits report a timeout instead of passing on an incomplete y; it
      // still counts its completion, which keeps the counts in step.
      if (peer_live && !arrived) wait_arrivals();
      if (lane == 0) bulk_wait_all();
      __syncwarp();
      fence_proxy_async_global();
      fence_sc_sys();
      named_bar_sync(1, 128);
      if (warp == 2 && lane == 0) {
        if (s_abort || s_peer_fail) {
#pragma unroll
          for (int p = 0; p < kMaxRanks; ++p)
            if (p < world) st_release_sys(a0.peer.sig[p] + kSigFail + a0.peer.me, call_no);
        }
        const unsigned long long add = 1ull + (blockIdx.x == 0 ? kDonePerRank - gridDim.x : 0ull);
#pragma unroll
        for (int p = 0; p < kMaxRanks; ++p)
          if (p < world) red_add_release_sys(a0.peer.sig[p] + kSigDone + a0.peer.me, add);
      }
    }
  }

  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair may still touch its barriers or smem
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, 2 * ACC);
  }
}

int num_sms() { return sm_budget(); }

template <int BP, int BQ, typename TI, int MODE>
int launch_inst(const Tc2Maps& maps, const Tc2Set& set, const YMaps& ym, bool pdl, cudaStream_t s) {
  constexpr int G = 256 / BP;
  constexpr int KS = BQ < 64 ? BQ : 64;
  constexpr uint32_t POS = KS * BP, AR_ROW = BP * 128;
  constexpr uint32_t B_SLOT = (G * POS > (G / 2) * AR_ROW) ? G * POS : (G / 2) * AR_ROW;
  constexpr uint32_t STAGE = 16384 + B_SLOT;
  constexpr int STAGES = kStages;
  static_assert((2 * STAGES + 4) * 8 + STAGES * 4 + 16 <= kEpiOff, "barrier area");
  const size_t smem = 1024 + size_t(STAGES) * STAGE + kEpiOff + (set.L[0].peer.world > 1 ? epi_stage_bytes(BP) : 0);
  auto kern = tc2_rowblock_kernel<BP, BQ, TI, MODE>;
  SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int items = set.item0[set.n];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(2 * std::min(items, num_sms() / 2)));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, maps, set, ym));
  return SLR_OK;
}

template <int BP, typename TI, int MODE>
int dispatch_bq(int bq, const Tc2Maps& maps, const Tc2Set& set, const YMaps& ym, bool pdl, cudaStream_t s) {
  switch (bq) {
    case 16: return launch_inst<BP, 16, TI, MODE>(maps, set, ym, pdl, s);
    case 32: return launch_inst<BP, 32, TI, MODE>(maps, set, ym, pdl, s);
    case 64: return launch_inst<BP, 64, TI, MODE>(maps, set, ym, pdl, s);
    case 128: return launch_inst<BP, 128, TI, MODE>(maps, set, ym, pdl, s);
    default: return fail(SLR_ERR_UNSUPPORTED, "2-SM path: block_q must be 16, 32, 64 or 128");
  }
}

template <typename TI, int MODE>
int dispatch_bp(int bp, int bq, const Tc2Maps& maps, const Tc2Set& set, const YMaps& ym, bool pdl, cudaStream_t s) {
  if (bp == 32) return dispatch_bq<32, TI, MODE>(bq, maps, set, ym, pdl, s);
  if (bp == 64) return dispatch_bq<64, TI, MODE>(bq, maps, set, ym, pdl, s);
  return fail(SLR_ERR_UNSUPPORTED, "2-SM path: block_p must be 32 or 64");
}

// Layer `a` as entry li of a launch: its Tc2Args and tensor maps.
int fill_tc2_layer(const RowblockArgs& a, Tc2Maps& maps, Tc2Set& set, int li) {
  const bool sparse = a.crow != nullptr && a.nnz > 0;
  const int bq = sparse ? a.bq : 64;
  const int ks = bq < 64 ? bq : 64;
  int rc = make_tmap_2d(&maps.x[li], a.x, a.dtype, uint64_t(a.K), uint64_t(a.M), uint64_t(a.ldx) * 2, uint32_t(ks),
                        128u);
  if (rc) return rc;
  if (sparse) {
    rc = make_tmap_2d(&maps.v[li], a.values, a.dtype, uint64_t(a.bp), uint64_t(a.nnz) * a.bq, uint64_t(a.bp) * 2,
                      uint32_t(a.bp / 2), uint32_t(ks));
    if (rc) return rc;
  }
  const int G = 256 / a.bp;
  set.L[li] = Tc2Args{a.y, a.mode == MODE_FUSED ? a.bias : nullptr, sparse ? a.crow : nullptr, a.col, a.rows,
                      sparse ? a.stage_plan : nullptr, sparse ? a.stage_start : nullptr, a.M, a.ldy,
                      int(a.nrows), int(ceil_div(a.nrows, G)), int(ceil_div(a.M, 256)), 0};
  // window spans read absent rows as the box just past the values (zero-filled)
  set.L[li].vrows = (sparse && int64_t(a.nnz) * a.bq < (int64_t(1) << 30)) ? int(a.nnz * a.bq) : 0;
  if (a.mode == MODE_FUSED && a.r > 0) {
    set.L[li].n_lr = int(ceil_div(a.r, 64));
    rc = make_tmap_2d(&maps.h[li], a.H, a.dtype, uint64_t(a.ldh), uint64_t(a.M), uint64_t(a.ldh) * 2, 64u, 128u);
    if (rc) return rc;
    rc = make_tmap_2d(&maps.a[li], a.A, a.dtype, uint64_t(a.r), uint64_t(a.N), uint64_t(a.r) * 2, 64u, uint32_t(a.bp));
    if (rc) return rc;
  }
  return SLR_OK;
}

int dispatch_set(const RowblockArgs& a0, int bq, const Tc2Maps& maps, const Tc2Set& set, const YMaps& ym, bool pdl,
                 cudaStream_t s) {
  if (a0.dtype == SLR_BF16)
    return a0.mode == MODE_ADDMM ? dispatch_bp<__nv_bfloat16, MODE_ADDMM>(a0.bp, bq, maps, set, ym, pdl, s)
                                 : dispatch_bp<__nv_bfloat16, MODE_FUSED>(a0.bp, bq, maps, set, ym, pdl, s);
  return a0.mode == MODE_ADDMM ? dispatch_bp<__half, MODE_ADDMM>(a0.bp, bq, maps, set, ym, pdl, s)
                               : dispatch_bp<__half, MODE_FUSED>(a0.bp, bq, maps, set, ym, pdl, s);
}

}  // namespace

// Measured on B200 (LLaMA-7B-shaped layers, 64x64 blocks, 4096 tokens): with
// the column schedule the pair kernel takes 7-14% less time than the 1-SM
// kernel (half the B operand bytes per SM, half the MMA instructions per
// MAC); with the single-thread merge it was slower, so the dispatcher picks
// it only when a schedule is present (or SLR_FLAG_PAIR_MMA asks for it).
bool tc2_rowblock_supported(const RowblockArgs& a) {
  return (a.bp == 32 || a.bp == 64) && a.M >= 256 && tc_rowblock_supported(a);
}

int launch_tc2_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s, const PeerArgs* peers) {
  if (a.nrows <= 0 || a.M <= 0) return SLR_OK;
  const bool sparse = a.crow != nullptr && a.nnz > 0;
  Tc2Maps maps{};
  Tc2Set set{};
  int rc = fill_tc2_layer(a, maps, set, 0);
  if (rc) return rc;
  set.n = 1;
  set.item0[0] = 0;
  set.item0[1] = set.L[0].n_groups * set.L[0].n_mtiles;
  YMaps ym{};
  if (peers && peers->world > 1) {
    set.L[0].peer = *peers;
    // TMA store maps of every rank's y at this rank's columns: [M, N], box bp x 32 rows
    for (int p = 0; p < peers->world; ++p) {
      rc = make_tmap_2d(&ym.m[0][p], peers->y[p], a.dtype, uint64_t(a.N), uint64_t(a.M), uint64_t(a.ldy) * 2,
                        uint32_t(a.bp), 32u);
      if (rc) return rc;
    }
  }
  return dispatch_set(a, sparse ? a.bq : 64, maps, set, ym, pdl, s);
}

bool tc2_group_compatible(const RowblockArgs* as, int n) {
  if (n < 1 || n > kTc2Layers) return false;
  const RowblockArgs& a0 = as[0];
  for (int i = 0; i < n; ++i) {
    const RowblockArgs& a = as[i];
    const bool sparse = a.crow != nullptr && a.nnz > 0;
    if (!sparse || !a.stage_plan || !a.stage_start || !tc2_rowblock_supported(a)) return false;
    if (a.bp != a0.bp || a.bq != a0.bq || a.M != a0.M || a.dtype != a0.dtype || a.mode != a0.mode) return false;
  }
  return true;
}

int launch_tc2_rowblock_group(const RowblockArgs* as, int n, bool pdl, cudaStream_t s) {
  if (!tc2_group_compatible(as, n)) return fail(SLR_ERR_UNSUPPORTED, "2-SM path: layers cannot share one launch");
  if (as[0].M <= 0) return SLR_OK;
  Tc2Maps maps{};
  Tc2Set set{};
  set.n = n;
  set.item0[0] = 0;
  for (int i = 0; i < n; ++i) {
    int rc = fill_tc2_layer(as[i], maps, set, i);
    if (rc) return rc;
    set.item0[i + 1] = set.item0[i] + set.L[i].n_groups * set.L[i].n_mtiles;
    set.L[i].xgrp = i;
    for (int j = 0; j < i; ++j)
      if (as[j].x == as[i].x) {
        set.L[i].xgrp = set.L[j].xgrp;
        break;
      }
  }
  if (set.item0[n] == 0) return SLR_OK;
  const YMaps ym{};
  return dispatch_set(as[0], as[0].bq, maps, set, ym, pdl, s);
}

int launch_tc2_rowblock_group_peers(const RowblockArgs* as, int n, const PeerArgs* peers, const PeerArgs& sync,
                                    cudaStream_t s) {
  if (!tc2_group_compatible(as, n)) return fail(SLR_ERR_UNSUPPORTED, "2-SM path: layers cannot share one launch");
  if (sync.world < 2) return fail(SLR_ERR_INVALID_ARGUMENT, "peers: world must be >= 2");
  if (as[0].M <= 0) return SLR_OK;
  Tc2Maps maps{};
  Tc2Set set{};
  YMaps ym{};
  set.n = n;
  set.item0[0] = 0;
  for (int i = 0; i < n; ++i) {
    int rc = fill_tc2_layer(as[i], maps, set, i);
    if (rc) return rc;
    set.item0[i + 1] = set.item0[i] + set.L[i].n_groups * set.L[i].n_mtiles;
    set.L[i].xgrp = i;
    for (int j = 0; j < i; ++j)
      if (as[j].x == as[i].x) {
        set.L[i].xgrp = set.L[j].xgrp;
        break;
      }
    // the launch's signals are sync's; layer i's tiles go to every rank's y of layer i
    set.L[i].peer = sync;
    for (int p = 0; p < sync.world; ++p) {
      set.L[i].peer.y[p] = peers[i].y[p];
      rc = make_tmap_2d(&ym.m[i][p], peers[i].y[p], as[i].dtype, uint64_t(as[i].N), uint64_t(as[i].M),
                        uint64_t(as[i].ldy) * 2, uint32_t(as[i].bp), 32u);
      if (rc) return rc;
    }
  }
  if (set.item0[n] == 0)
    return fail(SLR_ERR_INVALID_ARGUMENT, "peers: no rows of these layers on this rank (end the call with the "
                                          "empty-shard wait instead)");
  return dispatch_set(as[0], as[0].bq, maps, set, ym, false, s);
}

int read_and_clear_status_tc2(unsigned* out) {
  unsigned v = 0, zero = 0;
  SLR_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status_tc2, sizeof(v)));
  if (v) SLR_CHECK_CUDA(cudaMemcpyToSymbol(g_status_tc2, &zero, sizeof(zero)));
  *out = v;
  return SLR_OK;
}

}  // namespace slr
