// Large-token-batch path (prefill), 16-bit dtypes, on the 5th-generation
// tensor cores: tcgen05.mma with the accumulator in tensor memory (TMEM),
// operands staged in shared memory by TMA, completion tracked by mbarriers.
//
//   tc_rowblock_kernel  persistent; one work item = (128-token tile, block-row
//                       of bp output features).  The K loop walks the row's
//                       BSR blocks (x tile 128 x bq gathered at col*bq, values
//                       block bq x bp, MN-major) and then, for the fused
//                       layer, rank chunks of 64 (H tile 128 x 64, rows of A
//                       64-wide, K-major) into ONE fp32 accumulator 128 x bp in
//                       TMEM.  The epilogue adds bias (fused layer) or the old
//                       `out` (in-place operator) and stores y once.
//   tc_dense_kernel     persistent dense GEMM H[M, ldh] = x · Bᵀ (tiles
//                       128 x 64), the rank-r down-projection, rounded to the
//                       I/O dtype like the reference's first F.linear.
//
// Warp roles: warp 1 lane 0 issues MMAs (warp 1 also owns the TMEM
// allocation), warps 2-5 drain TMEM (warp w reads TMEM lanes 32*(w%4) .. +31,
// i.e. tokens of that quarter).  TMA loads: warp 0 lane 0 in the dense kernel;
// in the fused kernel four warps (0, 6, 7, 8) each fill every fourth stage
// from the layer's precomputed column schedule, because one warp needs ~1000
// cycles of issue work per stage (waits, descriptors, ~60 cycles per TMA
// load) and the tensor core would otherwise wait on it.
// The accumulator is double-buffered in TMEM so the epilogue of one item
// overlaps the MMAs of the next.  Shared memory holds an 8-stage ring.
//
// Reference counterparts: _bsr_body (ssalaad/tilelang_sparse/addmm_inplace.py:
// 41-82) and the F.linear pair + bias of _LRSLinearLRBlockCUDA.forward
// (ssalaad/efficient/ls_linear.py:124-137).
#include <algorithm>
#include <type_traits>

#include "internal.hpp"
#include "tcgen05.cuh"

namespace slr {
namespace {
using namespace tc;

__device__ unsigned g_status_tc = 0;

constexpr int kThreads = 192;        // tc_dense_kernel
constexpr int kMaxSeg = kMaxLaunchLayers;  // weight matrices per x*B^T launch
constexpr int kRowThreads = 288;     // tc_rowblock_kernel: warps 0, 6, 7, 8 load operands
constexpr int kProd2 = 6;            // first of the extra TMA warps
constexpr int kProducers = 4;        // TMA warps working from a column schedule
constexpr int kTileM = 128;

struct TcArgs {
  void* y;
  const void* bias;
  const int32_t* crow;
  const int32_t* col;
  const int32_t* rows;
  const uint32_t* plan;   // stage records (column | row mask << 16) per row group, or null
  const int32_t* plan_start;
  int64_t M, ldy;
  int nrows, n_groups, n_mtiles, n_lr;
};

// Drain-and-exit after a bounded wait gave up: record the timeout.
__device__ __forceinline__ void tc_timeout(volatile int* abort_flag) {
  atomicOr(&g_status_tc, SLR_TIMEOUT_BIT);
  *abort_flag = 1;
}

// Operand staging of tc_rowblock_kernel.  Stages carry k-slices of up to 64
// (sparse: x tile 128 x 64 plus the group's value blocks; low-rank: H tile
// 128 x 64 plus A rows of the group; 48 KB).  Every stage costs the issuing
// threads a fixed ~1000 cycles of barrier waits and TMA / MMA issue, so
// fewer, fuller stages beat a deeper ring of small ones.
constexpr int kSparseK = 64;  // k per sparse stage
constexpr int kLrK = 64;      // rank columns per low-rank stage

template <int BP, int BQ>
struct RowCfg {
  static constexpr int G = 256 / BP;                     // block-rows per item
  static constexpr int KS = BQ < kSparseK ? BQ : kSparseK;
  static constexpr int SUB = BQ / KS;                    // sparse stages per block column
  static constexpr int XW = KS * 2, VW = BP * 2;         // x-tile / values row bytes
  static constexpr uint32_t X_BYTES = kTileM * XW, V_BYTES = KS * VW;
  static constexpr uint32_t H_BYTES = kTileM * kLrK * 2, AR_BYTES = BP * kLrK * 2;
  static constexpr uint32_t BOFF = X_BYTES > H_BYTES ? X_BYTES : H_BYTES;
  static constexpr uint32_t BREG = G * (V_BYTES > AR_BYTES ? V_BYTES : AR_BYTES);  // value blocks / A rows
  static constexpr uint32_t STAGE = (BOFF + BREG + 1023u) & ~1023u;
  static constexpr int STAGES = 4;  // a multiple of kProducers (each producer warp owns slots)
  static constexpr size_t SMEM = 1024 + size_t(STAGES) * STAGE + (3 * STAGES + 4) * 8 + STAGES * 4 + 16;
};

constexpr uint32_t kMetaLR = 1u << 30;    // stage holds an H tile + rows of A
constexpr uint32_t kMetaLast = 1u << 31;  // last stage of the work item

// Persistent fused kernel.  One work item = 128 tokens x a group of
// G = 256/BP block-rows, taken consecutively from the row list (heaviest
// first for the fused layer), so the item's accumulator is 128 x 256 fp32 in
// TMEM (double-buffered: all 512 columns).  The producers merge the G rows'
// sorted column lists: each distinct column is one stage holding the x tile
// once plus, in slot j, the value block of group row j if it has the column,
// so an x tile feeds up to G block-rows, and each run of consecutive rows
// present in a stage is one MMA with N = run length * BP.  The low-rank
// steps then add H[128 x 64] · A_rows[256 x 64]ᵀ with one N = 256 MMA per
// k16.  Every MMA accumulates: the epilogue re-zeroes each accumulator after
// draining it.
//
// Warps: 0 and 6-8 TMA producers, 1 MMA issuer, 2-5 epilogue.
template <int BP, int BQ, typename TI, int MODE>
__global__ void __launch_bounds__(kRowThreads, 1)
    tc_rowblock_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_a,
                       const TcArgs a) {
  using C = RowCfg<BP, BQ>;
  constexpr int G = C::G, KS = C::KS, SUB = C::SUB, XW = C::XW, VW = C::VW;
  constexpr uint32_t X_BYTES = C::X_BYTES, V_BYTES = C::V_BYTES, H_BYTES = C::H_BYTES, AR_BYTES = C::AR_BYTES;
  constexpr uint32_t STAGE = C::STAGE;
  constexpr int STAGES = C::STAGES;
  constexpr uint32_t BOFF = C::BOFF;     // slot offset of the value blocks / A rows
  constexpr int LRW = kLrK * 2;          // H / A row bytes
  constexpr uint32_t ACC = 256;          // accumulator columns
  constexpr uint32_t IDESC_SP = idesc_f16<TI>(kTileM, 0, true);  // N set per run of rows
  constexpr uint32_t IDESC_LR = idesc_f16<TI>(kTileM, 256, false);
  static_assert(X_BYTES % 1024 == 0 && H_BYTES % 1024 == 0 && AR_BYTES % 512 == 0, "tile alignment");
  static_assert(G * BP == 256 && G <= 16, "group must span 256 columns");
  static_assert(STAGES % kProducers == 0, "each producer warp owns whole ring slots");
  static_assert(STAGE % 1024 == 0 && V_BYTES % 256 == 0 && BOFF % 1024 == 0, "alignment of stages / value slots");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* meta = reinterpret_cast<uint32_t*>(tempty + 2);  // [STAGES]
  uint32_t* tmem_slot = meta + STAGES;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * ACC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp >= 2 && warp < 6) {  // both accumulators start at zero
    const uint32_t lane_base = uint32_t(32 * (warp & 3)) << 16;
    for (uint32_t c = 0; c < 2 * ACC; c += 16) tmem_st16_zero(tmem + lane_base + c);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int n_items = a.n_groups * a.n_mtiles;

  if (warp == 0 || warp >= kProd2) {
    // ------------------------------------------------------- TMA producers
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      if (a.crow) tma_prefetch_desc(&tm_v);
      if (a.n_lr) {
        tma_prefetch_desc(&tm_h);
        tma_prefetch_desc(&tm_a);
      }
    }
    if (a.plan) {
      // With the column schedule every stage is independent: producer warp p
      // (warps 0, 6, 7, 8) fills the stages g with g % 4 == p, i.e. always
      // the same ring slot, so its waits on that slot stay in phase order.
      const int pw = warp == 0 ? 0 : warp - kProd2 + 1;
      const uint32_t* blk_idx = a.plan;  // records' second words index into the plan
      uint32_t g = 0;
      bool waited = false, abort_now = false;
      for (int kr = 0, item = snake_item(0, blockIdx.x, gridDim.x); item < n_items && !abort_now; ++kr, item = snake_item(kr, blockIdx.x, gridDim.x)) {
        const int gi = item / a.n_mtiles, mt = item - gi * a.n_mtiles;
        const int r0 = gi * G;
        const int gcount = min(G, a.nrows - r0);
        const int m0 = mt * kTileM;
        const int p0 = __ldg(a.plan_start + gi), p1 = __ldg(a.plan_start + gi + 1);
        const int n_sp = (p1 - p0) * SUB;
        const int n_st = max(n_sp + a.n_lr, 1);  // a terminator stage when there is nothing
        const int rw = lane < gcount ? (a.rows ? a.rows[r0 + lane] : r0 + lane) : 0;
        for (int s = (pw - int(g % kProducers) + kProducers) % kProducers; s < n_st; s += kProducers) {
          const uint32_t gg = g + uint32_t(s);
          const uint32_t slot = gg % STAGES, ph = (gg / STAGES) & 1;
          int ok = lane == 0 ? int(mbar_wait(&empty[slot], ph ^ 1)) : 1;
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            if (lane == 0) tc_timeout(&s_abort);
            abort_now = true;
            break;
          }
          uint8_t* adst = smem + slot * STAGE;
          const bool last = s == n_st - 1;
          if (s < n_sp) {
            const int k = p0 + s / SUB, sub = s % SUB;
            const uint32_t rec = __ldg(a.plan + 2 * k), first = __ldg(a.plan + 2 * k + 1);
            const uint32_t c = rec & 0xffffu, mask = rec >> 16;
            if (lane == 0) {
              meta[slot] = mask | (last ? kMetaLast : 0u);
              mbar_arrive_expect_tx(&full[slot], X_BYTES + __popc(mask) * V_BYTES);
              tma_load_2d(adst, &tm_x, int(c) * BQ + sub * KS, m0, &full[slot]);
            }
            if ((mask >> lane) & 1u) {
              const int blk = int(__ldg(blk_idx + first + __popc(mask & ((1u << lane) - 1u))));
              tma_load_2d(adst + BOFF + lane * V_BYTES, &tm_v, 0, blk * BQ + sub * KS, &full[slot]);
            }
          } else if (s < n_sp + a.n_lr) {
            const int l = s - n_sp;
            if (!waited) {
              pdl_wait_primary();  // H comes from the preceding kernel
              waited = true;
            }
            if (lane == 0) {
              meta[slot] = kMetaLR | uint32_t(gcount) | (last ? kMetaLast : 0u);
              mbar_arrive_expect_tx(&full[slot], H_BYTES + gcount * AR_BYTES);
              tma_load_2d(adst, &tm_h, l * kLrK, m0, &full[slot]);
            }
            if (lane < gcount)
              tma_load_2d(adst + BOFF + lane * AR_BYTES, &tm_a, l * kLrK, rw * BP, &full[slot]);
          } else if (lane == 0) {
            meta[slot] = kMetaLast;  // no block and no rank: the item still completes
            mbar_arrive(&full[slot]);
          }
        }
        g += uint32_t(n_st);
      }
    } else if (warp == 0 || warp == kProd2) {
    // Without a schedule, warps 0 and 6 both walk the stage sequence.  Lane j
    // (< G) follows block-row j of the item's group: cur = column of the
    // row's next block, nxt = the one after (loaded a step ahead so no stage
    // waits on a col[] load); the next column is the warp minimum and its
    // rows a ballot.  Warp 0 publishes each stage (row mask, expected bytes),
    // warp 6 loads the x tile, the value blocks (and A rows) alternate.
    const int pw = warp == 0 ? 0 : 1;
    constexpr uint32_t kNone = 0x7fffffffu;
    bool waited = false;
    uint32_t g = 0;
    // warp-uniform view of the abort flag (the loops below use warp collectives)
    auto stop = [&]() { return __any_sync(0xffffffffu, s_abort != 0); };
    for (int kr = 0, item = snake_item(0, blockIdx.x, gridDim.x); item < n_items && !stop(); ++kr, item = snake_item(kr, blockIdx.x, gridDim.x)) {
      const int gi = item / a.n_mtiles, mt = item - gi * a.n_mtiles;
      const int r0 = gi * G;
      const int gcount = min(G, a.nrows - r0);
      const int m0 = mt * kTileM;
      int rw = 0, ptr = 0, end = 0;
      uint32_t cur = kNone, nxt = kNone;
      if (lane < gcount) {
        rw = a.rows ? a.rows[r0 + lane] : r0 + lane;
        if (a.crow) {
          ptr = a.crow[rw];
          end = a.crow[rw + 1];
        }
        if (ptr < end) cur = uint32_t(__ldg(a.col + ptr));
        if (ptr + 1 < end) nxt = uint32_t(__ldg(a.col + ptr + 1));
      }
      bool published = false;
      bool abort_now = false;
      uint32_t c = __reduce_min_sync(0xffffffffu, cur);
      // One stage per (column, sub-slice) of the union of the group's columns.
      while (c != kNone && !abort_now) {
        const bool mine = cur == c;
        const uint32_t mask = __ballot_sync(0xffffffffu, mine);
        const int blk = ptr;
        const uint32_t cidx = __popc(mask & ((1u << lane) - 1u));
        if (mine) {
          ++ptr;
          cur = nxt;
          nxt = ptr + 1 < end ? uint32_t(__ldg(a.col + ptr + 1)) : kNone;
        }
        const uint32_t cn = __reduce_min_sync(0xffffffffu, cur);
        for (int sub = 0; sub < SUB; ++sub, ++g) {
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          int ok = lane == 0 ? int(mbar_wait(&empty[slot], ph ^ 1)) : 1;
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) {
            if (lane == 0) tc_timeout(&s_abort);
            abort_now = true;
            break;
          }
          uint8_t* adst = smem + slot * STAGE;
          if (lane == 0) {
            if (pw == 0) {
              const bool last = cn == kNone && a.n_lr == 0 && sub == SUB - 1;
              meta[slot] = mask | (last ? kMetaLast : 0u);
              mbar_arrive_expect_tx(&full[slot], X_BYTES + __popc(mask) * V_BYTES);
            } else {
              tma_load_2d(adst, &tm_x, c * BQ + sub * KS, m0, &full[slot]);
            }
          }
          if (mine && int(cidx & 1u) == pw)
            tma_load_2d(adst + BOFF + lane * V_BYTES, &tm_v, 0, blk * BQ + sub * KS, &full[slot]);
          published = true;
        }
        c = cn;
      }
      for (int l = 0; l < a.n_lr && !abort_now; ++l, ++g) {
        if (!waited && pw == 0) {
          pdl_wait_primary();  // H comes from the preceding kernel
          waited = true;
        }
        const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
        int ok = lane == 0 ? int(mbar_wait(&empty[slot], ph ^ 1)) : 1;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) tc_timeout(&s_abort);
          abort_now = true;
          break;
        }
        uint8_t* adst = smem + slot * STAGE;
        if (pw == 0 && lane == 0) {
          meta[slot] = kMetaLR | uint32_t(gcount) | (l == a.n_lr - 1 ? kMetaLast : 0u);
          mbar_arrive_expect_tx(&full[slot], H_BYTES + gcount * AR_BYTES);
          tma_load_2d(adst, &tm_h, l * kLrK, m0, &full[slot]);
        }
        if (lane < gcount && (lane & 1) == pw)
          tma_load_2d(adst + BOFF + lane * AR_BYTES, &tm_a, l * kLrK, rw * BP, &full[slot]);
        published = true;
      }
      if (abort_now) break;
      if (!published) {
        // No block and no rank: a terminator stage so the item still completes.
        const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
        int ok = 1;
        if (pw == 0 && lane == 0) {
          ok = int(mbar_wait(&empty[slot], ph ^ 1));
          if (!ok) {
            tc_timeout(&s_abort);
          } else {
            meta[slot] = kMetaLast;
            mbar_arrive(&full[slot]);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ++g;
      }
    }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t g = 0, it = 0;
      for (int kr = 0, item = snake_item(0, blockIdx.x, gridDim.x); item < n_items && !s_abort; ++kr, item = snake_item(kr, blockIdx.x, gridDim.x), ++it) {
        const uint32_t buf = it & 1, tph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1)) {
          tc_timeout(&s_abort);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * ACC;
        while (true) {
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          if (!mbar_wait(&full[slot], ph)) {
            tc_timeout(&s_abort);
            break;
          }
          tc_fence_after();
          const uint32_t m = meta[slot];
          const uint32_t abase = smem_u32(smem + slot * STAGE);
          const uint32_t bbase = abase + BOFF;
          if (m & kMetaLR) {
#pragma unroll
            for (int kk = 0; kk < kLrK / 16; ++kk)
              umma_f16(d, sdesc(abase + kk * 32, 16, 8 * LRW, layout_for(LRW)),
                       sdesc(bbase + kk * 32, 16, 8 * LRW, layout_for(LRW)), IDESC_LR, 1u);
          } else {
            // One MMA per run of consecutive rows that have this column: their
            // value slots are adjacent N-atoms (LBO = slot stride), so the x
            // k-slice is read from shared memory once per run, not per row.
            uint32_t mask = m & 0xffffu;
            while (mask) {
              const int j = __ffs(mask) - 1;
              const int len = __ffs(~(mask >> j)) - 1;
              mask &= ~(((1u << len) - 1u) << j);
              const uint32_t idesc = IDESC_SP | (uint32_t(len * BP) >> 3) << 17;
#pragma unroll
              for (int kk = 0; kk < KS / 16; ++kk) {
                const uint64_t ad = sdesc(abase + kk * 32, 16, 8 * XW, layout_for(XW));
                const uint64_t bd = sdesc(bbase + j * V_BYTES + kk * 16 * VW, V_BYTES, 8 * VW, layout_for(VW));
                umma_f16(d + j * BP, ad, bd, idesc, 1u);
              }
            }
          }
          umma_commit(&empty[slot]);  // frees the stage once these MMAs finish
          ++g;
          if (m & kMetaLast) break;
        }
        umma_commit(&tfull[buf]);     // accumulator ready for the epilogue
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = uint32_t(32 * q) << 16;
    const int row = 32 * q + lane;
    TI* __restrict__ y = static_cast<TI*>(a.y);
    const TI* __restrict__ bias = static_cast<const TI*>(a.bias);
    uint32_t it = 0;
    for (int kr = 0, item = snake_item(0, blockIdx.x, gridDim.x); item < n_items; ++kr, item = snake_item(kr, blockIdx.x, gridDim.x), ++it) {
      const int gi = item / a.n_mtiles, mt = item - gi * a.n_mtiles;
      const int r0 = gi * G;
      const int gcount = min(G, a.nrows - r0);
      const uint32_t buf = it & 1, tph = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[buf], tph, 256)) {
        if (lane == 0) tc_timeout(&s_abort);
        break;
      }
      tc_fence_after();
      const int64_t tok = int64_t(mt) * kTileM + row;
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
                  // in-place operator: old + sum (the reference's acc = out; acc += ...)
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
            reinterpret_cast<uint4*>(yr + c0)[0] = o0;
            reinterpret_cast<uint4*>(yr + c0)[1] = o1;
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * ACC);
  }
}

// ---------------------------------------------------------- dense GEMM --

// H_s[M, ldh_s] = x_s · B_sᵀ for up to kMaxSeg segments in one launch: the
// weight matrices that share an x (the q/k/v or gate/up projections of a
// decoder layer) and the layers with their own x, each segment with its own
// K and H.  The N tiles of segment s are [seg_nt[s], seg_nt[s+1]); an H
// element is the same dot product in the same k order whatever the launch.
//
// Items (one 128-token x BN tile each) weigh their segment's k chunks, so a
// launch that mixes K = 11008 with K = 4096 segments is unbalanced under a
// round-robin deal.  The host deals them longest first to the least loaded
// CTA; CTA c runs deal_item[deal_off[c] .. deal_off[c+1]).  Larger launches
// than the tables hold (deal == 0) fall back to item = c + j * gridDim.x.
constexpr int kDealCtas = 160;
constexpr int kDealItems = 2048;
struct DenseArgs {
  int64_t M;
  int n_mtiles, n_ntiles;
  int n_seg;
  int deal;
  int seg_nt[kMaxSeg + 1];
  int seg_nk[kMaxSeg];     // 64-wide k chunks
  int seg_x[kMaxSeg];      // x map of the segment
  void* seg_H[kMaxSeg];    // the segment's first H column
  int64_t seg_ldh[kMaxSeg];
  uint16_t deal_off[kDealCtas + 1];
  uint16_t deal_item[kDealItems];
};
struct DenseMaps {
  CUtensorMap b[kMaxSeg];
  CUtensorMap x[kMaxSeg];
};

template <int BN, typename TI>
__global__ void __launch_bounds__(kThreads, 1)
    tc_dense_kernel(const __grid_constant__ DenseMaps maps, const __grid_constant__ DenseArgs a) {
  constexpr uint32_t A_BYTES = kTileM * 128, B_BYTES = BN * 128;
  constexpr uint32_t STAGE = A_BYTES + B_BYTES;
  constexpr int STAGES = (196 * 1024) / STAGE > 8 ? 8 : (196 * 1024) / STAGE;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_f16<TI>(kTileM, BN, false);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_items = a.n_mtiles * a.n_ntiles;
  // this CTA's items: the host's deal, or round-robin
  const int first = a.deal ? int(a.deal_off[blockIdx.x]) : int(blockIdx.x);
  const int n_mine = a.deal ? int(a.deal_off[blockIdx.x + 1]) - first
                            : (n_items - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
  auto item_at = [&](int j) -> int {
    return a.deal ? int(a.deal_item[first + j]) : first + j * int(gridDim.x);
  };
  // Launched as a programmatic dependent, this kernel waits here for the kernel
  // before it (x may be its output) and only then lets the next one start
  // (the combine, which reads x before its own wait and H after it).  So a
  // chain combine -> x*B^T -> combine never reads an unfinished x.
  pdl_wait_primary();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      for (int sg = 0; sg < a.n_seg; ++sg) {
        tma_prefetch_desc(&maps.b[sg]);
        tma_prefetch_desc(&maps.x[a.seg_x[sg]]);
      }

      uint32_t g = 0;
      for (int j = 0; j < n_mine && !s_abort; ++j) {
        const int item = item_at(j);
        const int mt = item % a.n_mtiles, nt = item / a.n_mtiles;
        int sg = 0;
        while (sg + 1 < a.n_seg && nt >= a.seg_nt[sg + 1]) ++sg;
        const CUtensorMap* tm_b = &maps.b[sg];
        const CUtensorMap* tm_x = &maps.x[a.seg_x[sg]];
        const int nl = nt - a.seg_nt[sg];
        for (int s = 0; s < a.seg_nk[sg]; ++s, ++g) {
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          if (!mbar_wait(&empty[slot], ph ^ 1)) {
            tc_timeout(&s_abort);
            break;
          }
          uint8_t* adst = smem + slot * STAGE;
          mbar_arrive_expect_tx(&full[slot], STAGE);
          tma_load_2d(adst, tm_x, s * 64, mt * kTileM, &full[slot]);
          // the whole BN x 64 tile of B as one box (one TMA issue instead of
          // BN / 64: this thread's per-box issue cost bounds the kernel)
          tma_load_2d(adst + A_BYTES, tm_b, s * 64, nl * BN, &full[slot]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t g = 0, it = 0;
      for (int j = 0; j < n_mine && !s_abort; ++j, ++it) {
        const int item = item_at(j);
        const uint32_t buf = it & 1, tph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[buf], tph ^ 1)) {
          tc_timeout(&s_abort);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        int sg = 0;
        while (sg + 1 < a.n_seg && item / a.n_mtiles >= a.seg_nt[sg + 1]) ++sg;
        uint32_t acc = 0;
        for (int s = 0; s < a.seg_nk[sg]; ++s, ++g) {
          const uint32_t slot = g % STAGES, ph = (g / STAGES) & 1;
          if (!mbar_wait(&full[slot], ph)) {
            tc_timeout(&s_abort);
            break;
          }
          tc_fence_after();
          const uint32_t abase = smem_u32(smem + slot * STAGE);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_f16(d, sdesc(abase + kk * 32, 16, 1024, 2), sdesc(abase + A_BYTES + kk * 32, 16, 1024, 2),
                     IDESC, acc);
            acc = 1;
          }
          umma_commit(&empty[slot]);
        }
        umma_commit(&tfull[buf]);
      }
    }
  } else {
    const int q = warp & 3;
    const int row = 32 * q + lane;
    uint32_t it = 0;
    for (int j = 0; j < n_mine; ++j, ++it) {
      const int item = item_at(j);
      const int mt = item % a.n_mtiles, nt = item / a.n_mtiles;
      int sg = 0;
      while (sg + 1 < a.n_seg && nt >= a.seg_nt[sg + 1]) ++sg;
      TI* __restrict__ H = static_cast<TI*>(a.seg_H[sg]);
      const int64_t ldh = a.seg_ldh[sg];
      const int nl = nt - a.seg_nt[sg];
      const uint32_t buf = it & 1, tph = (it >> 1) & 1;
      if (!mbar_wait_warp(&tfull[buf], tph, 256)) {
        if (lane == 0) tc_timeout(&s_abort);
        break;
      }
      tc_fence_after();
      const int64_t tok = int64_t(mt) * kTileM + row;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + (uint32_t(32 * q) << 16) + buf * BN + c0, r);
        tmem_ld_wait();
        uint32_t p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) p[j] = pack2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]), (TI*)nullptr);
        if (tok < a.M) {
          uint4* hr = reinterpret_cast<uint4*>(H + tok * ldh + int64_t(nl) * BN + c0);
          hr[0] = make_uint4(p[0], p[1], p[2], p[3]);
          hr[1] = make_uint4(p[4], p[5], p[6], p[7]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

int num_sms() { return sm_budget(); }

template <int BP, int BQ, typename TI, int MODE>
int launch_rowblock_inst(const CUtensorMap& tx, const CUtensorMap& tv, const CUtensorMap& th,
                         const CUtensorMap& ta, const TcArgs& k, bool pdl, cudaStream_t s) {
  const size_t smem = RowCfg<BP, BQ>::SMEM;
  auto kern = tc_rowblock_kernel<BP, BQ, TI, MODE>;
  SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int items = k.n_groups * k.n_mtiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(std::min(items, num_sms())));
  cfg.blockDim = dim3(kRowThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  SLR_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tx, tv, th, ta, k));
  return SLR_OK;
}

template <int BP, typename TI, int MODE>
int dispatch_bq(int bq, const CUtensorMap& tx, const CUtensorMap& tv, const CUtensorMap& th,
                const CUtensorMap& ta, const TcArgs& k, bool pdl, cudaStream_t s) {
  switch (bq) {
    case 16: return launch_rowblock_inst<BP, 16, TI, MODE>(tx, tv, th, ta, k, pdl, s);
    case 32: return launch_rowblock_inst<BP, 32, TI, MODE>(tx, tv, th, ta, k, pdl, s);
    case 64: return launch_rowblock_inst<BP, 64, TI, MODE>(tx, tv, th, ta, k, pdl, s);
    case 128: return launch_rowblock_inst<BP, 128, TI, MODE>(tx, tv, th, ta, k, pdl, s);
    default: return fail(SLR_ERR_UNSUPPORTED, "tcgen05 path: block_q must be 16, 32, 64 or 128");
  }
}

template <typename TI, int MODE>
int dispatch_bp(int bp, int bq, const CUtensorMap& tx, const CUtensorMap& tv, const CUtensorMap& th,
                const CUtensorMap& ta, const TcArgs& k, bool pdl, cudaStream_t s) {
  switch (bp) {
    case 16: return dispatch_bq<16, TI, MODE>(bq, tx, tv, th, ta, k, pdl, s);
    case 32: return dispatch_bq<32, TI, MODE>(bq, tx, tv, th, ta, k, pdl, s);
    case 64: return dispatch_bq<64, TI, MODE>(bq, tx, tv, th, ta, k, pdl, s);
    default: return fail(SLR_ERR_UNSUPPORTED, "tcgen05 path: block_p must be 16, 32 or 64");
  }
}

}  // namespace

bool tc_rowblock_supported(const RowblockArgs& a) {
  if (a.dtype == SLR_F32) return false;
  if (a.bp != 16 && a.bp != 32 && a.bp != 64) return false;
  if (a.crow != nullptr && a.bq != 16 && a.bq != 32 && a.bq != 64 && a.bq != 128) return false;
  if (a.mode == MODE_FUSED && a.r != 0 && (a.r < 64 || a.r % 8 != 0)) return false;
  if (a.ldx % 8 != 0 || a.ldy % 8 != 0 || a.K % 8 != 0 || a.K < 64 || a.M < kTileM) return false;
  if (!aligned16(a.x) || !aligned16(a.y)) return false;
  if (a.crow != nullptr && !aligned16(a.values)) return false;
  if (a.mode == MODE_FUSED && a.r != 0 && !aligned16(a.A)) return false;
  if (a.bias != nullptr && !aligned16(a.bias)) return false;
  return a.nrows <= (1 << 24) && ceil_div(a.M, kTileM) <= (1 << 20);
}

int launch_tc_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s) {
  if (a.nrows <= 0 || a.M <= 0) return SLR_OK;
  const bool sparse = a.crow != nullptr && a.nnz > 0;
  const int bq = sparse ? a.bq : 64;
  const int ks = bq < kSparseK ? bq : kSparseK;
  CUtensorMap tx{}, tv{}, th{}, ta{};
  int rc = make_tmap_2d(&tx, a.x, a.dtype, uint64_t(a.K), uint64_t(a.M), uint64_t(a.ldx) * 2, uint32_t(ks),
                        uint32_t(kTileM));
  if (rc) return rc;
  if (sparse) {
    rc = make_tmap_2d(&tv, a.values, a.dtype, uint64_t(a.bp), uint64_t(a.nnz) * a.bq, uint64_t(a.bp) * 2,
                      uint32_t(a.bp), uint32_t(ks));
    if (rc) return rc;
  }
  const int G = 256 / a.bp;
  TcArgs k{a.y, a.mode == MODE_FUSED ? a.bias : nullptr, sparse ? a.crow : nullptr, a.col, a.rows,
           sparse ? a.stage_plan : nullptr, sparse ? a.stage_start : nullptr, a.M, a.ldy,
           int(a.nrows), int(ceil_div(a.nrows, G)), int(ceil_div(a.M, kTileM)), 0};
  if (a.mode == MODE_FUSED && a.r > 0) {
    k.n_lr = int(ceil_div(a.r, kLrK));
    rc = make_tmap_2d(&th, a.H, a.dtype, uint64_t(a.ldh), uint64_t(a.M), uint64_t(a.ldh) * 2, uint32_t(kLrK),
                      uint32_t(kTileM));
    if (rc) return rc;
    rc = make_tmap_2d(&ta, a.A, a.dtype, uint64_t(a.r), uint64_t(a.N), uint64_t(a.r) * 2, uint32_t(kLrK),
                      uint32_t(a.bp));
    if (rc) return rc;
  }
  if (a.dtype == SLR_BF16)
    return a.mode == MODE_ADDMM ? dispatch_bp<__nv_bfloat16, MODE_ADDMM>(a.bp, bq, tx, tv, th, ta, k, pdl, s)
                                : dispatch_bp<__nv_bfloat16, MODE_FUSED>(a.bp, bq, tx, tv, th, ta, k, pdl, s);
  return a.mode == MODE_ADDMM ? dispatch_bp<__half, MODE_ADDMM>(a.bp, bq, tx, tv, th, ta, k, pdl, s)
                              : dispatch_bp<__half, MODE_FUSED>(a.bp, bq, tx, tv, th, ta, k, pdl, s);
}

bool tc_dense_supported(const void* x, int64_t ldx, const void* B, int64_t K, int64_t r, int dtype) {
  return dtype != SLR_F32 && r >= 64 && K >= 64 && K % 8 == 0 && ldx % 8 == 0 && aligned16(x) && aligned16(B);
}

// Longest-processing-time deal of a dense launch's items to `grid` CTAs.  The
// items of segment s are [seg_nt[s], seg_nt[s+1]) x n_mtiles, each weighing
// w[s]; the segments come heaviest first, so walking the items in index order
// takes them heaviest first, and each goes to the least loaded CTA (ties to the
// lowest index: equal weights deal round-robin).  off[c] .. off[c+1] indexes
// CTA c's items in `item`, in the order it runs them.
static void deal_longest_first(const int* seg_nt, const int* w, int n_seg, int n_mtiles, int grid,
                               uint16_t* off, uint16_t* item) {
  struct Bin {
    int64_t load;
    int cta;
  };
  auto before = [](const Bin& x, const Bin& y) { return x.load < y.load || (x.load == y.load && x.cta < y.cta); };
  Bin heap[kDealCtas];
  for (int c = 0; c < grid; ++c) heap[c] = Bin{0, c};  // ascending: already a min-heap
  uint8_t owner[kDealItems];
  int cnt[kDealCtas] = {};
  int i = 0;
  for (int sg = 0; sg < n_seg; ++sg) {
    const int end = seg_nt[sg + 1] * n_mtiles;
    for (; i < end; ++i) {
      owner[i] = uint8_t(heap[0].cta);
      ++cnt[heap[0].cta];
      heap[0].load += w[sg];
      for (int p = 0;;) {
        const int l = 2 * p + 1, r = l + 1;
        int m = p;
        if (l < grid && before(heap[l], heap[m])) m = l;
        if (r < grid && before(heap[r], heap[m])) m = r;
        if (m == p) break;
        std::swap(heap[p], heap[m]);
        p = m;
      }
    }
  }
  int pos[kDealCtas];
  off[0] = 0;
  for (int c = 0; c < grid; ++c) {
    pos[c] = off[c];
    off[c + 1] = uint16_t(off[c] + cnt[c]);
  }
  for (int j = 0; j < i; ++j) item[pos[owner[j]]++] = uint16_t(j);
}

int launch_tc_dense_multi(const DenseSeg* segs, int n, int64_t M, int dtype, cudaStream_t s, bool pdl) {
  if (M <= 0 || n <= 0) return SLR_OK;
  if (n > kMaxSeg) return fail(SLR_ERR_UNSUPPORTED, "tc_dense: too many weight matrices in one launch");
  // segments with the longest K first (the heaviest items lead the deal); an
  // H element does not depend on the order
  int ord[kMaxSeg];
  for (int i = 0; i < n; ++i) ord[i] = i;
  std::stable_sort(ord, ord + n, [&](int a, int b) { return segs[a].K > segs[b].K; });
  DenseMaps maps{};
  DenseArgs k{};
  k.M = M;
  k.n_mtiles = int(ceil_div(M, kTileM));
  k.n_seg = n;
  // each segment's columns: r_s rounded up to 64; the tile width must divide every one
  int64_t cols[kMaxSeg];
  int64_t total = 0;
  bool all256 = true, all128 = true;
  for (int i = 0; i < n; ++i) {
    const DenseSeg& g = segs[ord[i]];
    cols[i] = round_up(g.r, 64);
    total += cols[i];
    all256 = all256 && cols[i] % 256 == 0;
    all128 = all128 && cols[i] % 128 == 0;
    if (cols[i] > g.ldh) return fail(SLR_ERR_WORKSPACE, "tc_dense: H row narrower than the layer's columns");
  }
  // Widest tile that divides every segment and still gives the SMs work:
  // wide tiles move fewer operand bytes per MAC.
  int bn = 64;
  if (all256 && int64_t(k.n_mtiles) * (total / 256) * 2 >= num_sms()) bn = 256;
  else if (all128) bn = 128;
  int nx = 0;
  for (int i = 0; i < n; ++i) {
    const DenseSeg& g = segs[ord[i]];
    // one x map per distinct x (same pointer, stride and width)
    int xi = -1;
    for (int j = 0; j < i && xi < 0; ++j) {
      const DenseSeg& h = segs[ord[j]];
      if (h.x == g.x && h.ldx == g.ldx && h.K == g.K) xi = k.seg_x[j];
    }
    if (xi < 0) {
      xi = nx++;
      int rc = make_tmap_2d(&maps.x[xi], g.x, dtype, uint64_t(g.K), uint64_t(M), uint64_t(g.ldx) * 2, 64u,
                            uint32_t(kTileM));
      if (rc) return rc;
    }
    // B tiles of bn rows (rank columns of H) x 64 k, one box each; rows past r read as zeros
    int rc = make_tmap_2d(&maps.b[i], g.B, dtype, uint64_t(g.K), uint64_t(g.r), uint64_t(g.K) * 2, 64u,
                          uint32_t(bn));
    if (rc) return rc;
    k.seg_x[i] = xi;
    k.seg_nk[i] = int(ceil_div(g.K, 64));
    k.seg_H[i] = g.H;
    k.seg_ldh[i] = g.ldh;
    k.seg_nt[i + 1] = k.seg_nt[i] + int(cols[i] / bn);
  }
  k.n_ntiles = k.seg_nt[n];
  const int items = k.n_mtiles * k.n_ntiles;
  const int grid = std::min(items, num_sms());
  if (items <= kDealItems && grid <= kDealCtas) {
    // item i belongs to segment sg(i); its weight is the segment's k chunks
    // plus two for the tile's epilogue
    int w[kMaxSeg];
    for (int i = 0; i < n; ++i) w[i] = k.seg_nk[i] + 2;
    deal_longest_first(k.seg_nt, w, n, k.n_mtiles, grid, k.deal_off, k.deal_item);
    k.deal = 1;
  }
  auto launch = [&](auto kern, int BN) -> int {
    const uint32_t stage = kTileM * 128 + BN * 128;
    const int stages = std::min(8, int((196 * 1024) / stage));
    const size_t smem = 1024 + size_t(stages) * stage + (2 * stages + 4) * 8 + 16;
    SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid));
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
  };
  if (dtype == SLR_BF16) {
    if (bn == 256) return launch(tc_dense_kernel<256, __nv_bfloat16>, 256);
    if (bn == 128) return launch(tc_dense_kernel<128, __nv_bfloat16>, 128);
    return launch(tc_dense_kernel<64, __nv_bfloat16>, 64);
  }
  if (bn == 256) return launch(tc_dense_kernel<256, __half>, 256);
  if (bn == 128) return launch(tc_dense_kernel<128, __half>, 128);
  return launch(tc_dense_kernel<64, __half>, 64);
}

int launch_tc_dense_group(const void* x, int64_t ldx, const void* const* Bs, const int64_t* rs, int n,
                          void* H, int64_t M, int64_t K, int64_t ldh, int dtype, cudaStream_t s, bool pdl) {
  if (M <= 0 || n <= 0) return SLR_OK;
  if (n > kMaxSeg) return fail(SLR_ERR_UNSUPPORTED, "tc_dense: too many weight matrices in one group");
  DenseSeg segs[kMaxSeg];
  int64_t col = 0;
  for (int i = 0; i < n; ++i) {
    segs[i] = DenseSeg{x, ldx, K, Bs[i], rs[i], static_cast<uint8_t*>(H) + col * dtype_size(dtype), ldh};
    col += round_up(rs[i], 64);
  }
  if (col > ldh) return fail(SLR_ERR_WORKSPACE, "tc_dense: H row narrower than the group's columns");
  return launch_tc_dense_multi(segs, n, M, dtype, s, pdl);
}

int launch_tc_dense(const void* x, int64_t ldx, const void* B, void* H, int64_t M, int64_t K, int64_t r,
                    int64_t ldh, int dtype, cudaStream_t s, bool pdl) {
  if (M <= 0 || r <= 0) return SLR_OK;
  return launch_tc_dense_group(x, ldx, &B, &r, 1, H, M, K, ldh, dtype, s, pdl);
}

int read_and_clear_status_tc(unsigned* out) {
  unsigned v = 0, zero = 0;
  SLR_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_status_tc, sizeof(v)));
  if (v) SLR_CHECK_CUDA(cudaMemcpyToSymbol(g_status_tc, &zero, sizeof(zero)));
  *out = v;
  return SLR_OK;
}

}  // namespace slr
