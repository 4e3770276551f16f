// Internal launcher interface of libslr_b200 (not part of the C ABI).
#pragma once

#include "common.cuh"

namespace slr {

enum RowMode : int {
  MODE_FUSED = 0,  // y = sparse + H·Aᵀ + bias, y written
  MODE_ADDMM = 1,  // y += sparse, y read and written (active rows only)
};

// One launch over a list of block-rows x token tiles.
struct RowblockArgs {
  const void* x = nullptr;      // [M, K]
  void* y = nullptr;            // [M, N]
  const void* H = nullptr;      // [M, ldh] low-rank intermediate x·Bᵀ (FUSED)
  int64_t ldh = 0;
  const void* A = nullptr;      // [N, r]
  const void* B = nullptr;      // [r, K] (read by the single-launch decode kernel)
  const void* bias = nullptr;   // [N] or null
  const int32_t* crow = nullptr;  // [NB+1] or null (no sparse term)
  const int32_t* col = nullptr;
  const void* values = nullptr;   // [nnz, bq, bp]
  const int32_t* rows = nullptr;  // block-row list (null = 0..nrows-1)
  const uint32_t* stage_plan = nullptr;  // column schedule of each 256-feature row group
  const int32_t* stage_start = nullptr;  // (from slr_plan_stages), or null
  int64_t nrows = 0;
  int64_t route_nrows = 0;  // block-rows of the whole layer for kernel choice (0 = nrows)
  int64_t M = 0, K = 0, N = 0, r = 0, nnz = 0;
  int64_t ldx = 0, ldy = 0;  // row strides of x and y (elements)
  int bp = 0, bq = 0;
  int dtype = SLR_F32;
  int mode = MODE_FUSED;
};

// ---- SIMT (CUDA-core FFMA) kernels: fp32 parity path and generic fallback.
// H element type is float when h_f32, else the I/O dtype.
int launch_simt_h(const void* x, int64_t ldx, const void* B, void* H, int64_t M, int64_t K, int64_t r,
                  int64_t ldh, int dtype, bool h_f32, cudaStream_t s);
int launch_simt_rowblock(const RowblockArgs& a, bool h_f32, cudaStream_t s);

// ---- mma.sync + TMA kernels (16-bit dtypes): small token batches.
// Layers sharing one x that a grouped call runs as one launch.
constexpr int kMaxGroupLayers = 4;
// Layers (each with its own x, or groups sharing one) in one small-batch launch.
constexpr int kMaxLaunchLayers = 8;

// x·Bᵀ for 1..kMaxLaunchLayers weight segments (one layer each) into one H
// [M, ldh]: segment s reads its own x (segments of a group share one), owns
// the 16-row tiles [seg_rt[s], seg_rt[s + 1]) of H's columns and splits K as
// it would alone.
struct HSmallPlan {
  int tt = 8;        // tokens per CTA (8 * NT)
  int tc = 0;        // token chunks
  int nseg = 0;
  int rt = 0;        // 16-column tiles of H over all segments (ldh / 16)
  int ks_max = 1;    // largest K split of a segment
  int seg_rt[kMaxLaunchLayers + 1] = {};
  int ks[kMaxLaunchLayers] = {};
  int64_t kchunk[kMaxLaunchLayers] = {};
};
// K[s]: input width of segment s; ldh[s]: columns of H owned by segment s (a
// multiple of 16, >= r_s).
HSmallPlan plan_h_small(int64_t M, const int64_t* K, const int64_t* ldh, int nseg);
// pdl: may start while the preceding kernel runs (B loads only before the
// wait).  Either way the next kernel can start only after this one's wait,
// so it may read anything the kernels before this one wrote (x_early below).
int launch_h_small(const void* const* x, const int64_t* ldx, const void* const* B, const int64_t* r, void* H,
                   int64_t M, const int64_t* K, int64_t ldh, const HSmallPlan& plan, int dtype, bool pdl,
                   cudaStream_t s);
bool mma_rowblock_supported(int bp, int bq, int64_t K, int64_t r);
// x_early: the kernel issued just before is this call's h_small, so x is
// complete at launch and the combine reads it before griddepcontrol.wait.
int launch_mma_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s, bool x_early = false);
// Layers that read one H [M, ldh] (layer i's columns from h_col[i]), each its
// own x (or one shared x), in one launch; false from mma_group_compatible
// when their shapes need different kernel instances (or, with shared_x, when
// they do not read one x).
bool mma_group_compatible(const RowblockArgs* a, int n, bool shared_x);
int launch_mma_rowblock_group(const RowblockArgs* a, const int64_t* h_col, int n, const void* H, int64_t ldh,
                              bool pdl, cudaStream_t s, bool x_early = false);

// ---- single-launch decode: x·Bᵀ and the combine of up to kMaxLaunchLayers
// layers (16-bit, 1..SLR_DECODE_MAX_TOKENS tokens, MODE_FUSED) in one
// persistent kernel; ctrl is the caller's zeroed control block.
bool decode_supported(const RowblockArgs* layers, int n, int64_t M);
size_t decode_workspace_size(const RowblockArgs* layers, int n, int64_t M);
int launch_decode(const RowblockArgs* layers, int n, int64_t M, void* workspace, size_t workspace_bytes,
                  unsigned* ctrl, bool pdl, cudaStream_t s);
int read_and_clear_status_dec(unsigned* out);

// ---- peer memory: a rank's output tiles stored straight into every rank's y.
// Signal slot of one layer on each rank (SLR_SIGNAL_WORDS x u64, zero at start).
// Every rank numbers the calls of a layer by its own count (1, 2, ...), so
// words written for one call never satisfy the wait of another:
//   [kSigArrive + p] rank p stores its call number (release) when the call
//                    starts;
//   [kSigDone + p]   rank p adds kDonePerRank per call once its stores are
//                    visible (its CTAs add 1 each, CTA 0 adds
//                    kDonePerRank - gridDim.x on top);
//   [kSigFail + p]   rank p stores the number of a call in which one of its
//                    CTAs gave up a wait (its tiles for that call may be
//                    missing), before adding its completion;
//   [kSigCalls]      calls of the layer completed on this rank (written by its
//                    own wait).
// Call c of a rank may store into peers only once every [kSigArrive + q] ==
// c (so a peer's y is no longer read by that rank's previous call; a rank
// that skipped a call, or is a call ahead, never matches and the wait times
// out); y is complete on rank p after call c when every [kSigDone + q] >=
// kDonePerRank * c and no [kSigFail + q] == c.
constexpr int kMaxRanks = SLR_MAX_RANKS;
constexpr int kSigArrive = 0;
constexpr int kSigDone = kMaxRanks;
constexpr int kSigFail = 2 * kMaxRanks;
constexpr int kSigCalls = 3 * kMaxRanks;
static_assert(kSigCalls < SLR_SIGNAL_WORDS, "signal slot layout");
constexpr unsigned long long kDonePerRank = 1ull << 32;
struct PeerArgs {
  void* y[kMaxRanks];                   // rank p's y at this rank's columns (y[me] = local)
  unsigned long long* sig[kMaxRanks];   // rank p's signal slot of this layer
  unsigned long long* my_sig;           // sig[me]
  unsigned long long wait_ns = 0;       // limit of each wait on other ranks
  int world = 0, me = 0;
};
// Limit of the waits on other ranks (slr_set_wait_limit_ns), in ns.
unsigned long long peer_wait_limit_ns();
// The wait that ends a call (and, for a rank with no rows of the layer, its
// arrival and completion signals).
int launch_peer_wait(const PeerArgs& p, bool empty_shard, cudaStream_t s);
int read_and_clear_status_peer(unsigned* out);

// ---- tcgen05 / TMEM kernels (16-bit dtypes): large token batches.
// SMs the persistent kernels may fill: the device's count, or fewer after
// slr_set_sm_limit (to leave SMs to collectives running alongside).
int sm_budget();

constexpr int64_t kTcMinTokens = 128;  // below this the mma.sync path is used
constexpr int64_t kTileTokens = 128;   // token rows per tensor-core work item
bool tc_rowblock_supported(const RowblockArgs& a);
int launch_tc_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s);
bool tc2_rowblock_supported(const RowblockArgs& a);  // 2-SM pairs, M >= 256, bp 32/64
// peers: also store every output tile into the other ranks' y (null = local only).
int launch_tc2_rowblock(const RowblockArgs& a, bool pdl, cudaStream_t s, const PeerArgs* peers = nullptr);
// The combines of n layers in one launch, every output tile also stored into
// every rank's y: layer i's into peers[i].y[p]; the launch's arrival and
// completion signals are sync's.
int launch_tc2_rowblock_group_peers(const RowblockArgs* as, int n, const PeerArgs* peers, const PeerArgs& sync,
                                    cudaStream_t s);
// Up to kMaxLaunchLayers layers in one launch of the pair kernel (one
// persistent schedule, one tail): every layer sparse with a column schedule,
// one block shape, token count, dtype and mode; local y only.
bool tc2_group_compatible(const RowblockArgs* a, int n);
int launch_tc2_rowblock_group(const RowblockArgs* a, int n, bool pdl, cudaStream_t s);
bool tc_dense_supported(const void* x, int64_t ldx, const void* B, int64_t K, int64_t r, int dtype);
// pdl: may start while the preceding kernel runs (it waits for that kernel
// before its first load).
int launch_tc_dense(const void* x, int64_t ldx, const void* B, void* H, int64_t M, int64_t K, int64_t r,
                    int64_t ldh, int dtype, cudaStream_t s, bool pdl = false);
// x · [B_0; ...; B_{n-1}]ᵀ (n <= 8, same K) into H [M, ldh]: segment i takes
// columns [sum_{j<i} round_up(r_j, 64), + round_up(r_i, 64)).
int launch_tc_dense_group(const void* x, int64_t ldx, const void* const* Bs, const int64_t* rs, int n,
                          void* H, int64_t M, int64_t K, int64_t ldh, int dtype, cudaStream_t s, bool pdl = false);
// One x·Bᵀ product of a launch: H [M, ldh] (its first round_up(r, 64) columns)
// = x [M, K] · B [r, K]ᵀ.
struct DenseSeg {
  const void* x;
  int64_t ldx, K;
  const void* B;
  int64_t r;
  void* H;
  int64_t ldh;
};
// Up to kMaxLaunchLayers products (several inputs, each its own K and H) in
// one launch; each H element is the one launch_tc_dense computes.
int launch_tc_dense_multi(const DenseSeg* segs, int n, int64_t M, int dtype, cudaStream_t s, bool pdl = false);

// ---- N:M 2:4 + low-rank layer (16-bit): packer and fused combine (mma.sp).
int launch_nm_pack(const void* S, int64_t N, int64_t K, int dtype, void* values, uint32_t* meta, int* bad,
                   cudaStream_t s);
int launch_nm_combine(const void* x, int64_t ldx, void* y, int64_t ldy, const void* values, const uint32_t* meta,
                      const void* A, const void* H, int64_t ldh, const void* bias, int64_t M, int64_t N, int64_t K,
                      int64_t r, int dtype, cudaStream_t s);
// Prefill form of the layer: S unpacked into all (N/64) x (K/64) blocks of 64
// x 64 in the combine's value layout ([k][n] per block, row-major block
// order), with the row pointers, column indices and column schedule
// (slr_plan_stages layout, natural row order, block_p 64) of that structure.
int64_t nm_dense_plan_words(int64_t N, int64_t K);
int launch_nm_dense_blocks(const void* values, const uint32_t* meta, int64_t N, int64_t K, int dtype, void* blocks,
                           uint32_t* plan, int32_t* stage_start, int32_t* crow, int32_t* col, cudaStream_t s);

// ---- dense -> BSR conversion.
int launch_bsr_mask(const void* S, int64_t n, int64_t m, int64_t bp, int64_t bq, int dtype,
                    uint8_t* mask, int64_t* crow, cudaStream_t s);
int launch_bsr_fill(const void* S, int64_t n, int64_t m, int64_t bp, int64_t bq, int dtype,
                    const uint8_t* mask, const int64_t* crow, int64_t* col, void* values,
                    bool transpose, cudaStream_t s);
int launch_validate_bsr(const int32_t* crow, int64_t NB, const int32_t* col, int64_t nnz,
                        int64_t nbk, const int32_t* active, int64_t active_nb, int* flag,
                        cudaStream_t s);

// Device status words (bounded-wait timeouts) of each translation unit.
int read_and_clear_status_mma(unsigned* out);
int read_and_clear_status_tc(unsigned* out);
int read_and_clear_status_tc2(unsigned* out);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace slr
