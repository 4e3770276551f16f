// C ABI of libslr_b200.so (declared in include/slr_b200.h): argument
// validation with the reference's error classes, path dispatch, workspace
// layout, TMA tensor-map encoding and host-side planning.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <numeric>
#include <string>
#include <vector>

#include "internal.hpp"

namespace slr {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }
int fail(int status, const std::string& msg) {
  t_last_error = msg;
  return status;
}
int cuda_fail(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return SLR_ERR_CUDA;
}

// ------------------------------------------------------------ tensor maps --

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return fail(SLR_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  const size_t es = dtype_size(dtype);
  const size_t box_bytes = box_inner * es;
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (box_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  else if (box_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  else if (box_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUtensorMapDataType dt = dtype == SLR_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == SLR_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SLR_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (code " + std::to_string(int(r)) +
                                              "): base/stride must be 16-byte aligned");
  return SLR_OK;
}

namespace {
std::atomic<int> g_sm_limit{0};
}  // namespace

int sm_budget() {
  static int n = 0;
  if (n == 0) {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n = v > 0 ? v : 148;
  }
  const int lim = g_sm_limit.load(std::memory_order_relaxed);
  return (lim > 0 && lim < n) ? std::max(lim, 2) : n;
}

}  // namespace slr

using namespace slr;

namespace {

// slr_layer.flags bit that selects the 2-SM pair kernel for the combine phase.
constexpr int32_t kFlagPairMma = SLR_FLAG_PAIR_MMA;
// slr_layer.flags bit that turns off programmatic dependent launch.
constexpr int32_t kFlagStrict = SLR_FLAG_STRICT_ORDER;

bool valid_dtype(int d) { return d == SLR_F32 || d == SLR_F16 || d == SLR_BF16; }

// Workspace layout of slr_lrs_linear_forward for a given (layer, M).
struct FwdPlan {
  int path = 0;          // 0 = simt, 1 = mma (small M)
  int64_t ldh = 0;       // row stride of H
  size_t h_bytes = 0;
  size_t total = 0;
  int row_bp = 0;        // block-row height used by the kernels
  HSmallPlan hs;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

int effective_bp(const slr_layer& L) {
  if (L.nnz > 0) return int(L.block_p);
  // Low-rank only: any row blocking works; prefer the tensor-core sizes.
  for (int b : {64, 32, 16, 8, 4, 2, 1})
    if (L.out_features % b == 0) return b;
  return 1;
}

bool layer_aligned16(const slr_layer& L) {
  return aligned16(L.A) && aligned16(L.B) && (L.nnz == 0 || aligned16(L.values));
}

FwdPlan plan_forward(const slr_layer& L, int64_t M, const void* x) {
  FwdPlan p;
  p.row_bp = effective_bp(L);
  const bool is16 = L.dtype != SLR_F32;
  const int bq = L.nnz > 0 ? int(L.block_q) : 16;
  if (is16 && mma_rowblock_supported(p.row_bp, bq, L.in_features, L.rank) && layer_aligned16(L) &&
      (x == nullptr || aligned16(x)))
    p.path = 1;
  p.ldh = L.rank > 0 ? round_up(L.rank, 64) : 0;
  const size_t hes = (p.path == 0 && !is16) ? 4 : dtype_size(L.dtype);
  p.h_bytes = align256(size_t(std::max<int64_t>(M, 0)) * p.ldh * hes);
  if (p.path == 1 && L.rank > 0) p.hs = plan_h_small(M, &L.in_features, &p.ldh, 1);
  p.total = p.h_bytes;
  return p;
}

// The tensor-core kernels take one 128-token tile x 256 features per SM at a
// time; with fewer than 16 such items (few tokens and few output features,
// e.g. 128 tokens of a 2048-wide projection) the small-batch kernel, which
// spreads 16 features x 64 tokens per CTA over all SMs, is faster.
// A block-row shard decides as its whole layer would (route_nrows).
bool tc_worthwhile(const RowblockArgs& a) {
  if (a.M < kTcMinTokens || a.bp <= 0) return false;
  const int64_t G = a.bp <= 256 ? 256 / a.bp : 1;
  const int64_t rows = a.route_nrows > 0 ? a.route_nrows : a.nrows;
  return ceil_div(rows, G) * ceil_div(a.M, kTileTokens) >= 16;
}

int check_layer(const slr_layer* L) {
  if (!L) return fail(SLR_ERR_INVALID_ARGUMENT, "layer is NULL");
  if (!valid_dtype(L->dtype))
    return fail(SLR_ERR_UNSUPPORTED_DTYPE, "dtype must be SLR_F32, SLR_F16 or SLR_BF16");
  if ((L->flags & ~(kFlagPairMma | kFlagStrict)) != 0) return fail(SLR_ERR_INVALID_ARGUMENT, "unknown flags");
  if (L->in_features <= 0 || L->out_features <= 0 || L->rank < 0)
    return fail(SLR_ERR_INVALID_ARGUMENT, "in_features/out_features must be > 0 and rank >= 0");
  if (L->rank > 0 && (!L->A || !L->B)) return fail(SLR_ERR_INVALID_ARGUMENT, "A and B are required when rank > 0");
  if (L->nnz < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "nnz must be >= 0");
  if (L->route_out_features != 0 && L->route_out_features < L->out_features)
    return fail(SLR_ERR_INVALID_ARGUMENT, "route_out_features must be 0 or >= out_features");
  if (L->nnz > 0) {
    if (!L->crow || !L->col || !L->values) return fail(SLR_ERR_INVALID_ARGUMENT, "crow/col/values are required when nnz > 0");
    if (L->block_p <= 0 || L->block_q <= 0) return fail(SLR_ERR_INVALID_ARGUMENT, "block_p/block_q must be > 0");
    if (L->out_features % L->block_p || L->in_features % L->block_q)
      return fail(SLR_ERR_INVALID_ARGUMENT, "S shape must be divisible by the block shape");
    const int mult = L->dtype == SLR_F32 ? 8 : 16;
    if (L->block_p % mult || L->block_q % mult)
      return fail(SLR_ERR_UNSUPPORTED, std::string("block dimensions must be divisible by ") + std::to_string(mult));
    if (L->nnz > int64_t(L->out_features / L->block_p) * (L->in_features / L->block_q))
      return fail(SLR_ERR_INVALID_ARGUMENT, "nnz exceeds the number of blocks");
  }
  return SLR_OK;
}

}  // namespace

extern "C" {

int slr_abi_version(void) { return SLR_ABI_VERSION; }

int slr_set_sm_limit(int n) {
  g_sm_limit.store(n > 0 ? n : 0, std::memory_order_relaxed);
  return SLR_OK;
}

const char* slr_status_string(int status) {
  switch (status) {
    case SLR_OK: return "SLR_OK";
    case SLR_ERR_INVALID_ARGUMENT: return "SLR_ERR_INVALID_ARGUMENT";
    case SLR_ERR_UNSUPPORTED_DTYPE: return "SLR_ERR_UNSUPPORTED_DTYPE";
    case SLR_ERR_UNSUPPORTED: return "SLR_ERR_UNSUPPORTED";
    case SLR_ERR_CUDA: return "SLR_ERR_CUDA";
    case SLR_ERR_WORKSPACE: return "SLR_ERR_WORKSPACE";
    case SLR_ERR_BAD_INDEX: return "SLR_ERR_BAD_INDEX";
    case SLR_ERR_TIMEOUT: return "SLR_ERR_TIMEOUT";
    default: return "SLR_ERR_UNKNOWN";
  }
}

const char* slr_last_error(void) { return t_last_error.c_str(); }

int slr_device_status(int* status_out) {
  if (!status_out) return fail(SLR_ERR_INVALID_ARGUMENT, "status_out is NULL");
  SLR_CHECK_CUDA(cudaDeviceSynchronize());
  unsigned v = 0, w = 0;
  int rc = read_and_clear_status_mma(&v);
  if (rc) return rc;
  rc = read_and_clear_status_tc(&w);
  if (rc) return rc;
  v |= w;
  rc = read_and_clear_status_tc2(&w);
  if (rc) return rc;
  v |= w;
  rc = read_and_clear_status_peer(&w);
  if (rc) return rc;
  v |= w;
  rc = read_and_clear_status_dec(&w);
  if (rc) return rc;
  v |= w;
  *status_out = (v & SLR_TIMEOUT_BIT) ? SLR_ERR_TIMEOUT : SLR_OK;
  return SLR_OK;
}

int slr_bsr_addmm_inplace(void* out, const void* x, int64_t M, int64_t K, const int32_t* crow,
                          int64_t NB, const int32_t* col, const void* values, int64_t nnz,
                          int64_t block_p, int64_t block_q, const int32_t* active_rows,
                          int64_t active_nb, int dtype, void* stream) {
  if (!valid_dtype(dtype))
    return fail(SLR_ERR_UNSUPPORTED_DTYPE, "BSR kernel supports float32/float16/bfloat16");
  if (M < 0 || K < 0 || NB < 0 || nnz < 0 || active_nb < 0)
    return fail(SLR_ERR_INVALID_ARGUMENT, "sizes must be non-negative");
  if (block_p <= 0 || block_q <= 0) return fail(SLR_ERR_INVALID_ARGUMENT, "block_p/block_q must be > 0");
  const int mult = dtype == SLR_F32 ? 8 : 16;
  if (block_p % mult || block_q % mult)
    return fail(SLR_ERR_UNSUPPORTED, "block dimensions must be divisible by " + std::to_string(mult));
  if (K % block_q) return fail(SLR_ERR_INVALID_ARGUMENT, "x K must be divisible by block_q");
  if (M == 0 || active_nb == 0 || NB == 0) return SLR_OK;
  if (!out || !x || !crow || !active_rows || (nnz > 0 && (!col || !values)))
    return fail(SLR_ERR_INVALID_ARGUMENT, "null tensor pointer");
  RowblockArgs a;
  a.x = x;
  a.y = out;
  a.crow = crow;
  a.col = col;
  a.values = values;
  a.rows = active_rows;
  a.nrows = active_nb;
  a.M = M;
  a.K = K;
  a.N = NB * block_p;
  a.ldx = K;
  a.ldy = NB * block_p;
  a.nnz = nnz;
  a.bp = int(block_p);
  a.bq = int(block_q);
  a.dtype = dtype;
  a.mode = MODE_ADDMM;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype != SLR_F32 && nnz > 0 && tc_worthwhile(a) && tc_rowblock_supported(a))
    return launch_tc_rowblock(a, false, s);
  if (dtype != SLR_F32 && nnz > 0 && mma_rowblock_supported(a.bp, a.bq, K, 0) && aligned16(values) &&
      aligned16(x) && aligned16(out))
    return launch_mma_rowblock(a, false, s);
  return launch_simt_rowblock(a, true, s);
}

int slr_validate_bsr(const int32_t* crow, int64_t NB, const int32_t* col, int64_t nnz, int64_t nbk,
                     const int32_t* active_rows, int64_t active_nb, void* stream) {
  if (NB < 0 || nnz < 0 || nbk < 0 || active_nb < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if (!crow || (nnz > 0 && !col) || (active_nb > 0 && !active_rows))
    return fail(SLR_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* flag = nullptr;
  // The flag lives in pinned host memory mapped into the device: no device allocation.
  SLR_CHECK_CUDA(cudaHostAlloc(&flag, sizeof(int), cudaHostAllocMapped));
  *flag = 0;
  int* dflag = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(&dflag, flag, 0);
  int rc = SLR_OK;
  if (e != cudaSuccess) rc = cuda_fail(e, "cudaHostGetDevicePointer");
  if (!rc) rc = launch_validate_bsr(crow, NB, col, nnz, nbk, active_rows, active_nb, dflag, s);
  if (!rc) {
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) rc = cuda_fail(e, "validate_bsr sync");
  }
  const int bad = *flag;
  cudaFreeHost(flag);
  if (rc) return rc;
  if (bad) return fail(SLR_ERR_BAD_INDEX, "BSR structure invalid: crow not monotone / crow[0]!=0 / crow[NB]!=nnz, "
                                          "col out of [0, K/block_q), or a bad active row");
  return SLR_OK;
}

size_t slr_lrs_linear_workspace_size(const slr_layer* layer, int64_t M) {
  if (check_layer(layer) != SLR_OK || M < 0) return 0;
  return plan_forward(*layer, M, nullptr).total;
}

}  // extern "C"

namespace {

// Shared argument checks and argument packing of the three forward entry points.
struct FwdCall {
  FwdPlan p;
  RowblockArgs a;
  uint8_t* ws = nullptr;
};

int prepare_forward(const slr_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                    void* workspace, size_t workspace_bytes, bool need_y, FwdCall& c, bool check_ws = true) {
  int rc = check_layer(layer);
  if (rc) return rc;
  const slr_layer& L = *layer;
  if (M < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "M must be >= 0");
  if (ldx == 0) ldx = L.in_features;
  if (ldy == 0) ldy = L.out_features;
  if (ldx < L.in_features || ldy < L.out_features)
    return fail(SLR_ERR_INVALID_ARGUMENT, "ldx/ldy must be >= in_features/out_features");
  if (M > 0 && (!x || (need_y && !y))) return fail(SLR_ERR_INVALID_ARGUMENT, "x/y is NULL");
  // Every 16-bit path keeps H as [M, ldh] in the I/O dtype, so the two phases
  // may pick different kernels; the path only depends on x, never on y.
  c.p = plan_forward(L, M, (ldx % 8 == 0) ? x : reinterpret_cast<const void*>(uintptr_t(1)));
  if (check_ws && c.p.total > 0 && M > 0) {
    if (!workspace) return fail(SLR_ERR_WORKSPACE, "workspace is NULL");
    if (workspace_bytes < c.p.total)
      return fail(SLR_ERR_WORKSPACE, "workspace too small: need " + std::to_string(c.p.total) + " bytes");
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(SLR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  c.ws = static_cast<uint8_t*>(workspace);
  RowblockArgs& a = c.a;
  a.x = x;
  a.y = y;
  a.H = L.rank > 0 ? c.ws : nullptr;
  a.ldh = c.p.ldh;
  a.A = L.A;
  a.B = L.B;
  a.bias = L.bias;
  a.crow = L.nnz > 0 ? L.crow : nullptr;
  a.col = L.col;
  a.values = L.values;
  a.rows = L.nnz > 0 ? L.row_order : nullptr;
  a.stage_plan = (L.nnz > 0 && L.stage_start) ? L.stage_plan : nullptr;
  a.stage_start = a.stage_plan ? L.stage_start : nullptr;
  a.nrows = L.out_features / c.p.row_bp;
  a.route_nrows = L.route_out_features > 0 ? ceil_div(L.route_out_features, c.p.row_bp) : 0;
  a.M = M;
  a.K = L.in_features;
  a.N = L.out_features;
  a.ldx = ldx;
  a.ldy = ldy;
  a.r = L.rank;
  a.nnz = L.nnz;
  a.bp = c.p.row_bp;
  a.bq = L.nnz > 0 ? int(L.block_q) : 16;
  a.dtype = L.dtype;
  a.mode = MODE_FUSED;
  return SLR_OK;
}

// True when the combine phase runs on the small-batch kernel (mma_rowblock).
// That kernel and h_small read x and H only after griddepcontrol.wait, so
// both may be launched as programmatic dependents of the preceding kernel.
// The 2-SM pair kernel runs the combine phase when the layer carries a column
// schedule (it then beats the 1-SM kernel on B200) or when the caller asks
// for it; it needs block_p 32 or 64 and M >= 256.
bool use_pair(const slr_layer& L, const FwdCall& c) {
  return c.p.path == 1 && tc_worthwhile(c.a) && ((L.flags & kFlagPairMma) || c.a.stage_plan != nullptr) &&
         tc2_rowblock_supported(c.a);
}

bool small_batch_path(const slr_layer& L, const FwdCall& c) {
  if (c.p.path != 1) return false;
  if (use_pair(L, c)) return false;
  if (tc_worthwhile(c.a) && tc_rowblock_supported(c.a)) return false;
  return true;
}

bool early_start(const slr_layer& L) { return (L.flags & kFlagStrict) == 0; }

int run_lowrank(const slr_layer& L, const FwdCall& c, cudaStream_t s) {
  if (L.rank == 0 || c.a.M == 0) return SLR_OK;
  // x*B^T on the tensor cores from 128 tokens on, whatever kernel the combine
  // phase takes: the choice depends only on M, so a token slice (>= 128
  // tokens) or a block-row shard of the layer computes H bit for bit as the
  // whole layer does (the small-batch kernel splits K by M).
  if (c.p.path == 1 && c.a.M >= kTcMinTokens &&
      tc_dense_supported(c.a.x, c.a.ldx, L.B, L.in_features, L.rank, L.dtype))
    return launch_tc_dense(c.a.x, c.a.ldx, L.B, c.ws, c.a.M, L.in_features, L.rank, c.p.ldh, L.dtype, s,
                           early_start(L));
  if (c.p.path == 1) {
    const void* B = L.B;
    const void* x = c.a.x;
    const int64_t r = L.rank, ldx = c.a.ldx, K = L.in_features;
    return launch_h_small(&x, &ldx, &B, &r, c.ws, c.a.M, &K, c.p.ldh, c.p.hs, L.dtype,
                          early_start(L) && small_batch_path(L, c), s);
  }
  return launch_simt_h(c.a.x, c.a.ldx, L.B, c.ws, c.a.M, L.in_features, L.rank, c.p.ldh, L.dtype,
                       L.dtype == SLR_F32, s);
}

// True when run_lowrank launches h_small for this call: every kernel after it
// in the call then starts with x complete (h_small lets dependents start only
// after its own wait on the kernel before it).
bool lowrank_is_h_small(const slr_layer& L, const FwdCall& c) {
  return L.rank > 0 && c.a.M > 0 && c.p.path == 1 &&
         !(c.a.M >= kTcMinTokens && tc_dense_supported(c.a.x, c.a.ldx, L.B, L.in_features, L.rank, L.dtype));
}

// pdl: the tensor-core combine may overlap the x*B^T kernel issued just
// before it by this library (it reads H only after griddepcontrol.wait).
// x_early: an h_small of this call precedes the combine (lowrank_is_h_small).
int run_combine(const slr_layer& L, const FwdCall& c, bool pdl, cudaStream_t s, bool x_early = false) {
  if (c.a.M == 0) return SLR_OK;
  if (use_pair(L, c)) return launch_tc2_rowblock(c.a, pdl && L.rank > 0 && early_start(L), s);
  if (c.p.path == 1 && tc_worthwhile(c.a) && tc_rowblock_supported(c.a))
    return launch_tc_rowblock(c.a, pdl && L.rank > 0 && early_start(L), s);
  if (c.p.path == 1) return launch_mma_rowblock(c.a, early_start(L), s, x_early);
  return launch_simt_rowblock(c.a, L.dtype == SLR_F32, s);
}

}  // namespace

extern "C" {

int slr_lrs_linear_forward(const slr_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* stream) {
  FwdCall c;
  int rc = prepare_forward(layer, x, ldx, y, ldy, M, workspace, workspace_bytes, true, c);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = run_lowrank(*layer, c, s);
  if (rc) return rc;
  return run_combine(*layer, c, true, s, lowrank_is_h_small(*layer, c));
}

int slr_lrs_linear_lowrank(const slr_layer* layer, const void* x, int64_t ldx, int64_t M, void* workspace,
                           size_t workspace_bytes, void* stream) {
  FwdCall c;
  int rc = prepare_forward(layer, x, ldx, nullptr, 0, M, workspace, workspace_bytes, false, c);
  if (rc) return rc;
  return run_lowrank(*layer, c, static_cast<cudaStream_t>(stream));
}

int slr_lrs_linear_combine(const slr_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* stream) {
  FwdCall c;
  int rc = prepare_forward(layer, x, ldx, y, ldy, M, workspace, workspace_bytes, true, c);
  if (rc) return rc;
  return run_combine(*layer, c, false, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {

constexpr int kMaxGroup = kMaxGroupLayers;  // layers per grouped call

// Workspace of slr_lrs_linear_forward_group, in one of three layouts chosen
// by M (and the layers' paths):
//   TC    (M >= 128): the group's H [M, ldh_all] (layer i owns columns
//         [col[i], col[i] + round_up(r_i, 64))), written by one tensor-core GEMM;
//   SMALL (M < 128): the same H, written by one grouped small-batch x*B^T;
//   EACH: each layer's own workspace one after another (one forward per layer).
struct GroupPlan {
  int64_t ldh_all = 0;
  int64_t col[kMaxGroup] = {};
  size_t h_bytes = 0;
  HSmallPlan hs;                  // SMALL: all layers as segments of one x*B^T
  size_t off[kMaxGroup] = {}, bytes[kMaxGroup] = {};
  size_t total = 0;
};

int plan_group(const slr_layer* layers, int n, int64_t M, GroupPlan& g) {
  if (!layers || n <= 0 || n > kMaxGroup)
    return fail(SLR_ERR_INVALID_ARGUMENT, "a group holds 1 to " + std::to_string(kMaxGroup) + " layers");
  for (int i = 0; i < n; ++i) {
    int rc = check_layer(&layers[i]);
    if (rc) return rc;
    if (layers[i].in_features != layers[0].in_features || layers[i].dtype != layers[0].dtype)
      return fail(SLR_ERR_INVALID_ARGUMENT, "grouped layers must share in_features and dtype (they read one x)");
  }
  if (M <= 0) return SLR_OK;
  int64_t ldh[kMaxGroup];
  for (int i = 0; i < n; ++i) {
    ldh[i] = round_up(layers[i].rank, 64);
    g.col[i] = g.ldh_all;
    g.ldh_all += ldh[i];
  }
  g.h_bytes = align256(size_t(M) * size_t(g.ldh_all) * dtype_size(layers[0].dtype));
  if (M < kTcMinTokens && layers[0].dtype != SLR_F32) {
    int64_t Ks[kMaxGroup];
    for (int i = 0; i < n; ++i) Ks[i] = layers[i].in_features;
    g.hs = plan_h_small(M, Ks, ldh, n);
  }
  size_t off = 0;
  for (int i = 0; i < n; ++i) {
    g.off[i] = off;
    g.bytes[i] = plan_forward(layers[i], M, nullptr).total;
    off += align256(g.bytes[i]);
  }
  g.total = std::max(g.h_bytes, off);
  return SLR_OK;
}

}  // namespace

extern "C" {

size_t slr_lrs_linear_group_workspace_size(const slr_layer* layers, int n, int64_t M) {
  GroupPlan g;
  if (M < 0 || plan_group(layers, n, M, g) != SLR_OK) return 0;
  return g.total;
}

}  // extern "C"

namespace {

// Argument checks, per-layer packing and the layout decision of the group
// entry points.  y may be NULL (x*B^T phase only).
enum GroupMode { GROUP_EACH = 0, GROUP_TC = 1, GROUP_SMALL = 2 };

struct GroupCall {
  GroupPlan g;
  FwdCall c[kMaxGroup];
  int mode = GROUP_EACH;
  uint8_t* ws = nullptr;
};

int prepare_group(const slr_layer* layers, int n, const void* x, int64_t ldx, void* const* y, const int64_t* ldy,
                  int64_t M, void* workspace, size_t workspace_bytes, GroupCall& gc) {
  int rc = plan_group(layers, n, M, gc.g);
  if (rc) return rc;
  if (M < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "M must be >= 0");
  if (M == 0) return SLR_OK;
  // One x*B^T launch for the whole group (a single layer included) whenever
  // every layer has a rank and takes the 16-bit path: the tensor-core GEMM
  // from 128 tokens on, the small-batch kernel below.  The layout depends on
  // M only, so a call on a slice of the tokens writes its rows of the same H
  // as a call on all of them, and every combine kernel reads H through a
  // pointer and row stride.
  int mode = M >= kTcMinTokens ? GROUP_TC : GROUP_SMALL;
  for (int i = 0; mode != GROUP_EACH && i < n; ++i) {
    const slr_layer& L = layers[i];
    const int64_t lx = ldx ? ldx : L.in_features;
    const bool p16 = plan_forward(L, M, (lx % 8 == 0) ? x : reinterpret_cast<const void*>(uintptr_t(1))).path == 1;
    if (!p16 || L.rank <= 0 ||
        (mode == GROUP_TC && !tc_dense_supported(x, lx, L.B, L.in_features, L.rank, L.dtype)))
      mode = GROUP_EACH;
  }
  const size_t need = mode == GROUP_TC ? gc.g.h_bytes : gc.g.total;
  if (need > 0) {
    if (!workspace) return fail(SLR_ERR_WORKSPACE, "workspace is NULL");
    if (workspace_bytes < need)
      return fail(SLR_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(SLR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  gc.ws = static_cast<uint8_t*>(workspace);
  for (int i = 0; i < n; ++i) {
    // shared-H layouts: the layers' own workspaces are not used (the combine reads the group H)
    rc = prepare_forward(&layers[i], x, ldx, y ? y[i] : nullptr, ldy ? ldy[i] : 0, M, gc.ws + gc.g.off[i],
                         gc.g.bytes[i], y != nullptr, gc.c[i], mode == GROUP_EACH);
    if (rc) return rc;
  }
  gc.mode = mode;
  if (mode != GROUP_EACH)
    for (int i = 0; i < n; ++i) {
      gc.c[i].a.H = gc.ws + size_t(gc.g.col[i]) * dtype_size(layers[i].dtype);
      gc.c[i].a.ldh = gc.g.ldh_all;
    }
  return SLR_OK;
}

bool group_early_start(const slr_layer* layers, int n) {
  for (int i = 0; i < n; ++i)
    if (!early_start(layers[i])) return false;
  return true;
}

int group_lowrank(const slr_layer* layers, int n, const GroupCall& gc, cudaStream_t s) {
  if (gc.mode == GROUP_EACH) {
    for (int i = 0; i < n; ++i) {
      int rc = run_lowrank(layers[i], gc.c[i], s);
      if (rc) return rc;
    }
    return SLR_OK;
  }
  const void* Bs[kMaxGroup];
  int64_t rs[kMaxGroup];
  for (int i = 0; i < n; ++i) {
    Bs[i] = layers[i].B;
    rs[i] = layers[i].rank;
  }
  const RowblockArgs& a0 = gc.c[0].a;
  if (gc.mode == GROUP_TC)
    return launch_tc_dense_group(a0.x, a0.ldx, Bs, rs, n, gc.ws, a0.M, layers[0].in_features, gc.g.ldh_all,
                                 layers[0].dtype, s, group_early_start(layers, n));
  const void* xs[kMaxGroup];
  int64_t ldxs[kMaxGroup], Ks[kMaxGroup];
  for (int i = 0; i < n; ++i) {
    xs[i] = a0.x;
    ldxs[i] = a0.ldx;
    Ks[i] = layers[0].in_features;
  }
  return launch_h_small(xs, ldxs, Bs, rs, gc.ws, a0.M, Ks, gc.g.ldh_all, gc.g.hs, layers[0].dtype,
                        group_early_start(layers, n), s);
}

// Combine phase of every layer: one small-batch launch over all of them when
// their kernel shapes agree, else one launch per layer.  x_early: this call's
// h_small was launched just before (GROUP_SMALL after group_lowrank).
int group_combine_all(const slr_layer* layers, int n, const GroupCall& gc, cudaStream_t s, bool x_early) {
  if (gc.mode == GROUP_TC && n > 1) {
    // every layer on the pair kernel: one launch for all (one schedule tail)
    RowblockArgs as[kMaxGroup];
    bool all_pair = true, pdl = true;
    for (int i = 0; i < n; ++i) {
      as[i] = gc.c[i].a;
      all_pair = all_pair && use_pair(layers[i], gc.c[i]);
      pdl = pdl && layers[i].rank > 0 && early_start(layers[i]);
    }
    if (all_pair && tc2_group_compatible(as, n)) return launch_tc2_rowblock_group(as, n, pdl, s);
  }
  if (gc.mode == GROUP_SMALL) {
    RowblockArgs as[kMaxGroup];
    for (int i = 0; i < n; ++i) as[i] = gc.c[i].a;
    if (mma_group_compatible(as, n, true))
      return launch_mma_rowblock_group(as, gc.g.col, n, gc.ws, gc.g.ldh_all, group_early_start(layers, n), s,
                                       x_early);
  }
  for (int i = 0; i < n; ++i) {
    int rc = run_combine(layers[i], gc.c[i], true, s, x_early);
    if (rc) return rc;
  }
  return SLR_OK;
}

}  // namespace

extern "C" {

int slr_lrs_linear_forward_group(const slr_layer* layers, int n, const void* x, int64_t ldx, void* const* y,
                                 const int64_t* ldy, int64_t M, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  if (!y) return fail(SLR_ERR_INVALID_ARGUMENT, "y is NULL");
  GroupCall gc;
  int rc = prepare_group(layers, n, x, ldx, y, ldy, M, workspace, workspace_bytes, gc);
  if (rc || M == 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gc.mode == GROUP_EACH) {
    for (int i = 0; i < n; ++i) {
      rc = run_lowrank(layers[i], gc.c[i], s);
      if (rc) return rc;
      rc = run_combine(layers[i], gc.c[i], true, s, lowrank_is_h_small(layers[i], gc.c[i]));
      if (rc) return rc;
    }
    return SLR_OK;
  }
  rc = group_lowrank(layers, n, gc, s);
  if (rc) return rc;
  return group_combine_all(layers, n, gc, s, gc.mode == GROUP_SMALL);
}

int slr_lrs_linear_group_lowrank(const slr_layer* layers, int n, const void* x, int64_t ldx, int64_t M,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  GroupCall gc;
  int rc = prepare_group(layers, n, x, ldx, nullptr, nullptr, M, workspace, workspace_bytes, gc);
  if (rc || M == 0) return rc;
  return group_lowrank(layers, n, gc, static_cast<cudaStream_t>(stream));
}

int slr_lrs_linear_group_combine(const slr_layer* layers, int n, int i, const void* x, int64_t ldx, void* y,
                                 int64_t ldy, int64_t M, void* workspace, size_t workspace_bytes, void* stream) {
  if (i < 0 || i >= n) return fail(SLR_ERR_INVALID_ARGUMENT, "layer index out of range");
  if (!y) return fail(SLR_ERR_INVALID_ARGUMENT, "y is NULL");
  GroupCall gc;
  int rc = prepare_group(layers, n, x, ldx, nullptr, nullptr, M, workspace, workspace_bytes, gc);
  if (rc || M == 0) return rc;
  FwdCall c = gc.c[i];
  rc = prepare_forward(&layers[i], x, ldx, y, ldy, M, gc.ws + gc.g.off[i], gc.g.bytes[i], true, c,
                       gc.mode == GROUP_EACH);
  if (rc) return rc;
  c.a.H = gc.c[i].a.H;
  c.a.ldh = gc.c[i].a.ldh;
  return run_combine(layers[i], c, false, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {

// The low-rank half of an N:M layer as an S+LR layer without S: its x·Bᵀ
// runs on the same kernels (h_small / tc_dense) into the same H layout.
slr_layer nm_lowrank_layer(const slr_nm_layer& L) {
  slr_layer lr{};
  lr.in_features = L.in_features;
  lr.out_features = L.out_features;
  lr.rank = L.rank;
  lr.A = L.A;
  lr.B = L.B;
  lr.bias = L.bias;
  lr.dtype = L.dtype;
  lr.flags = L.flags & kFlagStrict;
  return lr;
}

// Prefill route of the N:M layer (M >= kNmDenseTokens): S unpacked per call
// into full-density 64 x 64 blocks in the workspace and the layer run as a
// block-sparse S+LR layer on the 2-SM tensor-core combine, whose 256-wide
// MMAs keep the tensor cores busy where the mma.sp kernel's 16-feature tiles
// re-read S for every 64 tokens.  Same arithmetic: x·Sᵀ, H·Aᵀ and the bias
// accumulated in fp32, y rounded once.
constexpr int64_t kNmDenseTokens = 256;

struct NmDenseLayout {
  size_t blocks = 0, plan = 0, start = 0, crow = 0, col = 0, total = 0;
};

bool nm_dense_route(const slr_nm_layer& L, int64_t M) {
  return M >= kNmDenseTokens && L.out_features % 64 == 0 && L.in_features % 64 == 0 && L.rank % 64 == 0 &&
         (L.flags & kFlagStrict) == 0;
}

// Offsets of the route's buffers after the first `base` bytes of the workspace.
NmDenseLayout nm_dense_layout(const slr_nm_layer& L, size_t base) {
  const int64_t NB = L.out_features / 64, KB = L.in_features / 64, groups = (NB + 3) / 4;
  NmDenseLayout d;
  size_t o = align256(base);
  d.blocks = o;
  o = align256(o + size_t(L.out_features) * size_t(L.in_features) * dtype_size(L.dtype));
  d.plan = o;
  o = align256(o + 4 * size_t(nm_dense_plan_words(L.out_features, L.in_features)));
  d.start = o;
  o = align256(o + 4 * size_t(groups + 1));
  d.crow = o;
  o = align256(o + 4 * size_t(NB + 1));
  d.col = o;
  o = align256(o + 4 * size_t(NB * KB));
  d.total = o;
  return d;
}

int check_nm_layer(const slr_nm_layer* L) {
  if (!L) return fail(SLR_ERR_INVALID_ARGUMENT, "layer is NULL");
  if (L->dtype != SLR_F16 && L->dtype != SLR_BF16)
    return fail(SLR_ERR_UNSUPPORTED_DTYPE, "N:M layer: dtype must be SLR_F16 or SLR_BF16");
  if (L->in_features <= 0 || L->out_features <= 0 || L->in_features % 32 || L->out_features % 16)
    return fail(SLR_ERR_INVALID_ARGUMENT, "N:M layer: in_features % 32 == 0 and out_features % 16 == 0 required");
  if (L->rank < 16 || L->rank % 8) return fail(SLR_ERR_UNSUPPORTED, "N:M layer: rank must be a multiple of 8, >= 16");
  if (!L->values || !L->meta || !L->A || !L->B) return fail(SLR_ERR_INVALID_ARGUMENT, "N:M layer: NULL tensor");
  if ((L->flags & ~kFlagStrict) != 0) return fail(SLR_ERR_INVALID_ARGUMENT, "unknown flags");
  if (!aligned16(L->values) || !aligned16(L->A) || !aligned16(L->B))
    return fail(SLR_ERR_UNSUPPORTED, "N:M layer: values, A and B must be 16-byte aligned");
  return SLR_OK;
}

}  // namespace

extern "C" {

int slr_nm_compress(const void* S, int64_t N, int64_t K, int dtype, void* values, uint32_t* meta, void* stream) {
  if (dtype != SLR_F16 && dtype != SLR_BF16) return fail(SLR_ERR_UNSUPPORTED_DTYPE, "N:M: 16-bit dtypes only");
  if (N <= 0 || K <= 0 || K % 32) return fail(SLR_ERR_INVALID_ARGUMENT, "N:M: K must be a positive multiple of 32");
  if (!S || !values || !meta) return fail(SLR_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* flag = nullptr;
  SLR_CHECK_CUDA(cudaHostAlloc(&flag, sizeof(int), cudaHostAllocMapped));
  *flag = 0;
  int* dflag = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(&dflag, flag, 0);
  int rc = e == cudaSuccess ? SLR_OK : cuda_fail(e, "cudaHostGetDevicePointer");
  if (!rc) rc = launch_nm_pack(S, N, K, dtype, values, meta, dflag, s);
  if (!rc) {
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) rc = cuda_fail(e, "nm_compress sync");
  }
  const int bad = *flag;
  cudaFreeHost(flag);
  if (rc) return rc;
  if (bad) return fail(SLR_ERR_BAD_INDEX, "S is not 2:4 sparse: a group of 4 input features holds more than 2 entries");
  return SLR_OK;
}

size_t slr_nm_linear_workspace_size(const slr_nm_layer* layer, int64_t M) {
  if (check_nm_layer(layer) != SLR_OK || M < 0) return 0;
  const slr_layer lr = nm_lowrank_layer(*layer);
  const size_t base = slr_lrs_linear_workspace_size(&lr, M);
  return nm_dense_route(*layer, M) ? nm_dense_layout(*layer, base).total : base;
}

int slr_nm_linear_forward(const slr_nm_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                          void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_nm_layer(layer);
  if (rc) return rc;
  const slr_nm_layer& L = *layer;
  if (ldx == 0) ldx = L.in_features;
  if (ldy == 0) ldy = L.out_features;
  if (M < 0 || ldx < L.in_features || ldy < L.out_features)
    return fail(SLR_ERR_INVALID_ARGUMENT, "bad M or row strides");
  if (M == 0) return SLR_OK;
  if (!x || !y) return fail(SLR_ERR_INVALID_ARGUMENT, "x/y is NULL");
  if (ldx % 8 || !aligned16(x)) return fail(SLR_ERR_UNSUPPORTED, "N:M layer: x rows must be 16-byte aligned");
  const slr_layer lr = nm_lowrank_layer(L);
  FwdCall c;
  rc = prepare_forward(&lr, x, ldx, y, ldy, M, workspace, workspace_bytes, true, c);
  if (rc) return rc;
  if (c.p.path != 1) return fail(SLR_ERR_UNSUPPORTED, "N:M layer: shapes outside the 16-bit kernels");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (nm_dense_route(L, M)) {
    const NmDenseLayout d = nm_dense_layout(L, slr_lrs_linear_workspace_size(&lr, M));
    uint8_t* w = static_cast<uint8_t*>(workspace);
    RowblockArgs a;
    a.x = x;
    a.y = y;
    a.H = c.ws;
    a.ldh = c.p.ldh;
    a.A = L.A;
    a.B = L.B;
    a.bias = L.bias;
    a.crow = reinterpret_cast<const int32_t*>(w + d.crow);
    a.col = reinterpret_cast<const int32_t*>(w + d.col);
    a.values = w + d.blocks;
    a.stage_plan = reinterpret_cast<const uint32_t*>(w + d.plan);
    a.stage_start = reinterpret_cast<const int32_t*>(w + d.start);
    a.nrows = L.out_features / 64;
    a.M = M;
    a.K = L.in_features;
    a.N = L.out_features;
    a.r = L.rank;
    a.nnz = a.nrows * (L.in_features / 64);
    a.ldx = ldx;
    a.ldy = ldy;
    a.bp = a.bq = 64;
    a.dtype = L.dtype;
    a.mode = MODE_FUSED;
    if (workspace_bytes >= d.total && tc2_rowblock_supported(a)) {
      rc = launch_nm_dense_blocks(L.values, L.meta, L.out_features, L.in_features, L.dtype, w + d.blocks,
                                  reinterpret_cast<uint32_t*>(w + d.plan), reinterpret_cast<int32_t*>(w + d.start),
                                  reinterpret_cast<int32_t*>(w + d.crow), reinterpret_cast<int32_t*>(w + d.col), s);
      if (!rc) rc = run_lowrank(lr, c, s);
      if (!rc) rc = launch_tc2_rowblock(a, false, s);
      return rc;
    }
  }
  rc = run_lowrank(lr, c, s);
  if (rc) return rc;
  return launch_nm_combine(x, ldx, y, ldy, L.values, L.meta, L.A, c.ws, c.p.ldh, L.bias, M, L.out_features,
                           L.in_features, L.rank, L.dtype, s);
}

}  // extern "C"

namespace {

constexpr int kMaxMulti = kMaxLaunchLayers;  // layers per multi-input call

// Workspace of slr_lrs_linear_forward_multi: below 128 tokens with every
// layer on the 16-bit small-batch path with a rank, one H [M, sum of
// round_up(r_i, 64)] (layer i's columns from col[i]) filled by one h_small
// launch; otherwise each layer's own forward workspace, one after another.
struct MultiPlan {
  bool small = false;
  int64_t ldh_all = 0;
  int64_t col[kMaxMulti] = {};
  size_t h_bytes = 0;
  HSmallPlan hs;
  size_t off[kMaxMulti] = {}, bytes[kMaxMulti] = {};
  size_t total = 0;
};

int plan_multi(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx, int64_t M,
               MultiPlan& m) {
  if (!layers || n <= 0 || n > kMaxMulti)
    return fail(SLR_ERR_INVALID_ARGUMENT, "a multi-input call holds 1 to " + std::to_string(kMaxMulti) + " layers");
  for (int i = 0; i < n; ++i) {
    int rc = check_layer(&layers[i]);
    if (rc) return rc;
    if (layers[i].dtype != layers[0].dtype)
      return fail(SLR_ERR_INVALID_ARGUMENT, "the layers of a multi-input call must share one dtype");
  }
  if (M < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "M must be >= 0");
  size_t off = 0;
  m.small = M > 0 && M < kTcMinTokens && layers[0].dtype != SLR_F32;
  int64_t ldh[kMaxMulti], Ks[kMaxMulti];
  for (int i = 0; i < n; ++i) {
    const slr_layer& L = layers[i];
    const void* xi = x ? x[i] : nullptr;
    const int64_t lx = (ldx && ldx[i]) ? ldx[i] : L.in_features;
    m.off[i] = off;
    m.bytes[i] = plan_forward(L, M, nullptr).total;
    off += align256(m.bytes[i]);
    if (x && plan_forward(L, M, (lx % 8 == 0) ? xi : reinterpret_cast<const void*>(uintptr_t(1))).path != 1)
      m.small = false;
    if (L.rank <= 0) m.small = false;
    ldh[i] = round_up(std::max<int64_t>(L.rank, 0), 64);
    Ks[i] = L.in_features;
    m.col[i] = m.ldh_all;
    m.ldh_all += ldh[i];
  }
  m.h_bytes = align256(size_t(std::max<int64_t>(M, 0)) * size_t(m.ldh_all) * dtype_size(layers[0].dtype));
  if (m.small) m.hs = plan_h_small(M, Ks, ldh, n);
  // sized for either layout, so the size query needs no inputs
  m.total = std::max(m.h_bytes, off);
  return SLR_OK;
}

// One multi-input call, checked and packed once: every layer's forward
// arguments; below 128 tokens their H share one buffer (one h_small launch),
// from 128 tokens on each layer keeps its own (layers on one input share
// their run's), and pair_group says whether all combines run as one launch of
// the pair kernel.
struct MultiCall {
  MultiPlan m;
  FwdCall c[kMaxMulti];
  bool pair_group = false;
  bool pdl = true;
  // From 128 tokens: runs of consecutive layers that read one x (same
  // pointer, stride and width) whose x*B^T is one grouped tensor-core GEMM
  // into one H (the run's own workspace regions, taken together).
  int n_runs = 0;
  int run0[kMaxMulti + 1] = {};
  bool grouped[kMaxMulti] = {};
  GroupCall gc[kMaxMulti];
};

int prepare_multi(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx, void* const* y,
                  const int64_t* ldy, int64_t M, void* workspace, size_t workspace_bytes, bool need_y,
                  MultiCall& mc) {
  if (!x || (need_y && !y)) return fail(SLR_ERR_INVALID_ARGUMENT, "x/y is NULL");
  int rc = plan_multi(layers, n, x, ldx, M, mc.m);
  if (rc || M == 0) return rc;
  const MultiPlan& m = mc.m;
  if (m.total > 0) {
    if (!workspace) return fail(SLR_ERR_WORKSPACE, "workspace is NULL");
    if (workspace_bytes < m.total)
      return fail(SLR_ERR_WORKSPACE, "workspace too small: need " + std::to_string(m.total) + " bytes");
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return fail(SLR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  for (int i = 0; i < n; ++i) {
    rc = prepare_forward(&layers[i], x[i], ldx ? ldx[i] : 0, need_y ? y[i] : nullptr, ldy ? ldy[i] : 0, M,
                         ws + m.off[i], m.bytes[i], need_y, mc.c[i], !m.small);
    if (rc) return rc;
  }
  if (m.small) {
    for (int i = 0; i < n; ++i) {
      mc.c[i].a.H = ws + size_t(m.col[i]) * dtype_size(layers[i].dtype);
      mc.c[i].a.ldh = m.ldh_all;
      mc.pdl = mc.pdl && early_start(layers[i]);
    }
  } else {
    // runs of layers on one input: one grouped x*B^T each
    for (int i = 0; i < n;) {
      const int64_t lx = (ldx && ldx[i]) ? ldx[i] : layers[i].in_features;
      int j = i + 1;
      while (j < n && j - i < kMaxGroup && x[j] == x[i] && layers[j].in_features == layers[i].in_features &&
             ((ldx && ldx[j]) ? ldx[j] : layers[j].in_features) == lx)
        ++j;
      const int r = mc.n_runs++;
      mc.run0[r] = i;
      mc.run0[r + 1] = j;
      if (j - i > 1 && M >= kTcMinTokens) {
        size_t bytes = 0;
        for (int k = i; k < j; ++k) bytes += align256(m.bytes[k]);
        GroupCall& gc = mc.gc[r];
        rc = prepare_group(&layers[i], j - i, x[i], lx, need_y ? y + i : nullptr, ldy ? ldy + i : nullptr, M,
                           ws + m.off[i], bytes, gc);
        if (rc) return rc;
        if (gc.mode == GROUP_TC) {
          mc.grouped[r] = true;
          for (int k = i; k < j; ++k) mc.c[k] = gc.c[k - i];
        }
      }
      i = j;
    }
    RowblockArgs as[kMaxMulti];
    bool all_pair = M >= kTcMinTokens && n > 1;
    for (int i = 0; i < n && all_pair; ++i) {
      as[i] = mc.c[i].a;
      all_pair = use_pair(layers[i], mc.c[i]);
      mc.pdl = mc.pdl && layers[i].rank > 0 && early_start(layers[i]);
    }
    mc.pair_group = all_pair && tc2_group_compatible(as, n);
  }
  return SLR_OK;
}

// x*B^T of every layer: one h_small launch below 128 tokens (each layer keeps
// the K split it would get alone, so H is the one of slr_lrs_linear_forward
// bit for bit), else each layer's own.
int multi_lowrank(const slr_layer* layers, int n, const MultiCall& mc, void* workspace, cudaStream_t s) {
  if (!mc.m.small) {
    // From 128 tokens: every layer's x*B^T (one segment per layer, the
    // grouped runs' layers into their shared H) in ONE tensor-core launch,
    // the layers with the longest K first, when every layer takes that kernel;
    // H is bit for bit the per-run launches'.
    DenseSeg segs[kMaxMulti];
    int ns = 0;
    bool all_tc = true, pdl = true;
    for (int r = 0; r < mc.n_runs && all_tc; ++r) {
      const int i0 = mc.run0[r], i1 = mc.run0[r + 1];
      for (int i = i0; i < i1 && all_tc; ++i) {
        const slr_layer& L = layers[i];
        const FwdCall& c = mc.c[i];
        if (L.rank == 0 || c.a.M == 0) continue;
        all_tc = L.dtype == layers[0].dtype;
        if (mc.grouped[r]) {
          const GroupCall& gc = mc.gc[r];
          segs[ns++] = DenseSeg{c.a.x, c.a.ldx, L.in_features, L.B, L.rank,
                                gc.ws + size_t(gc.g.col[i - i0]) * dtype_size(L.dtype), gc.g.ldh_all};
          pdl = pdl && group_early_start(&layers[i0], i1 - i0);
        } else {
          all_tc = all_tc && c.p.path == 1 && c.a.M >= kTcMinTokens &&
                   tc_dense_supported(c.a.x, c.a.ldx, L.B, L.in_features, L.rank, L.dtype);
          segs[ns++] = DenseSeg{c.a.x, c.a.ldx, L.in_features, L.B, L.rank, c.ws, c.p.ldh};
          pdl = pdl && early_start(L);
        }
      }
    }
    if (all_tc && ns > 1) return launch_tc_dense_multi(segs, ns, mc.c[0].a.M, layers[0].dtype, s, pdl);
    for (int r = 0; r < mc.n_runs; ++r) {
      const int i0 = mc.run0[r], i1 = mc.run0[r + 1];
      if (mc.grouped[r]) {
        int rc = group_lowrank(&layers[i0], i1 - i0, mc.gc[r], s);
        if (rc) return rc;
        continue;
      }
      for (int i = i0; i < i1; ++i) {
        int rc = run_lowrank(layers[i], mc.c[i], s);
        if (rc) return rc;
      }
    }
    return SLR_OK;
  }
  const void* xs[kMaxMulti];
  const void* Bs[kMaxMulti];
  int64_t ldxs[kMaxMulti], rs[kMaxMulti], Ks[kMaxMulti];
  for (int i = 0; i < n; ++i) {
    xs[i] = mc.c[i].a.x;
    ldxs[i] = mc.c[i].a.ldx;
    Bs[i] = layers[i].B;
    rs[i] = layers[i].rank;
    Ks[i] = layers[i].in_features;
  }
  return launch_h_small(xs, ldxs, Bs, rs, workspace, mc.c[0].a.M, Ks, mc.m.ldh_all, mc.m.hs, layers[0].dtype, mc.pdl,
                        s);
}

// The combines: one launch when the kernel shapes agree (the pair kernel from
// 128 tokens on, the small-batch kernel below), else one per layer.  x_early:
// this call's h_small was launched just before.
int multi_combine(const slr_layer* layers, int n, const MultiCall& mc, void* workspace, cudaStream_t s,
                  bool x_early) {
  RowblockArgs as[kMaxMulti];
  for (int i = 0; i < n; ++i) as[i] = mc.c[i].a;
  if (!mc.m.small) {
    if (mc.pair_group) return launch_tc2_rowblock_group(as, n, mc.pdl, s);
    for (int i = 0; i < n; ++i) {
      int rc = run_combine(layers[i], mc.c[i], true, s, false);
      if (rc) return rc;
    }
    return SLR_OK;
  }
  if (mma_group_compatible(as, n, false))
    return launch_mma_rowblock_group(as, mc.m.col, n, workspace, mc.m.ldh_all, mc.pdl, s, x_early);
  for (int i = 0; i < n; ++i) {
    int rc = run_combine(layers[i], mc.c[i], true, s, x_early);
    if (rc) return rc;
  }
  return SLR_OK;
}

}  // namespace

extern "C" {

size_t slr_lrs_linear_multi_workspace_size(const slr_layer* layers, int n, int64_t M) {
  MultiPlan m;
  if (plan_multi(layers, n, nullptr, nullptr, M, m) != SLR_OK) return 0;
  return m.total;
}

int slr_lrs_linear_forward_multi(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx,
                                 void* const* y, const int64_t* ldy, int64_t M, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  MultiCall mc;
  int rc = prepare_multi(layers, n, x, ldx, y, ldy, M, workspace, workspace_bytes, true, mc);
  if (rc || M == 0) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool any_grouped = false;
  for (int r = 0; r < mc.n_runs; ++r) any_grouped = any_grouped || mc.grouped[r];
  if (!mc.m.small && !mc.pair_group && !any_grouped) {
    // each layer's forward in turn
    for (int i = 0; i < n; ++i) {
      rc = run_lowrank(layers[i], mc.c[i], s);
      if (rc) return rc;
      rc = run_combine(layers[i], mc.c[i], true, s, lowrank_is_h_small(layers[i], mc.c[i]));
      if (rc) return rc;
    }
    return SLR_OK;
  }
  rc = multi_lowrank(layers, n, mc, workspace, s);
  if (rc) return rc;
  return multi_combine(layers, n, mc, workspace, s, mc.m.small);
}

int slr_lrs_linear_multi_lowrank(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx,
                                 int64_t M, void* workspace, size_t workspace_bytes, void* stream) {
  MultiCall mc;
  int rc = prepare_multi(layers, n, x, ldx, nullptr, nullptr, M, workspace, workspace_bytes, false, mc);
  if (rc || M == 0) return rc;
  return multi_lowrank(layers, n, mc, workspace, static_cast<cudaStream_t>(stream));
}

int slr_lrs_linear_multi_h(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx, int64_t M,
                           void* workspace, size_t workspace_bytes, void** H, int64_t* ldh) {
  if (!H || !ldh) return fail(SLR_ERR_INVALID_ARGUMENT, "H/ldh is NULL");
  MultiCall mc;
  int rc = prepare_multi(layers, n, x, ldx, nullptr, nullptr, M, workspace, workspace_bytes, false, mc);
  if (rc) return rc;
  for (int i = 0; i < n; ++i) {
    H[i] = M > 0 && layers[i].rank > 0 ? const_cast<void*>(mc.c[i].a.H) : nullptr;
    ldh[i] = M > 0 && layers[i].rank > 0 ? mc.c[i].a.ldh : 0;
  }
  return SLR_OK;
}

int slr_lrs_linear_multi_combine(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx,
                                 void* const* y, const int64_t* ldy, int64_t M, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  MultiCall mc;
  int rc = prepare_multi(layers, n, x, ldx, y, ldy, M, workspace, workspace_bytes, true, mc);
  if (rc || M == 0) return rc;
  return multi_combine(layers, n, mc, workspace, static_cast<cudaStream_t>(stream), false);
}

}  // extern "C"

namespace {

int to_peer_args(const slr_peers* P, PeerArgs& pa) {
  if (!P) return fail(SLR_ERR_INVALID_ARGUMENT, "peers is NULL");
  if (P->world < 2 || P->world > kMaxRanks || P->rank < 0 || P->rank >= P->world)
    return fail(SLR_ERR_INVALID_ARGUMENT, "peers: world must be 2.." + std::to_string(kMaxRanks) +
                                              " and rank in [0, world)");
  pa = PeerArgs{};
  pa.world = P->world;
  pa.me = P->rank;
  for (int p = 0; p < P->world; ++p) {
    if (!P->y[p] || !P->signal[p]) return fail(SLR_ERR_INVALID_ARGUMENT, "peers: NULL y or signal");
    if (!aligned16(P->y[p]) || (reinterpret_cast<uintptr_t>(P->signal[p]) & 7u))
      return fail(SLR_ERR_INVALID_ARGUMENT, "peers: y must be 16-byte and signal 8-byte aligned");
    pa.y[p] = P->y[p];
    pa.sig[p] = reinterpret_cast<unsigned long long*>(P->signal[p]);
  }
  pa.my_sig = pa.sig[pa.me];
  pa.wait_ns = peer_wait_limit_ns();
  return SLR_OK;
}

int check_peer_call(const slr_layer& L, const FwdCall& c, int64_t ldy, int64_t M) {
  if (M <= 0) return fail(SLR_ERR_INVALID_ARGUMENT, "peers: M must be > 0");
  if ((ldy * int64_t(dtype_size(L.dtype))) % 16)
    return fail(SLR_ERR_INVALID_ARGUMENT, "peers: y rows must be 16-byte multiples");
  if (!use_pair(L, c))
    return fail(SLR_ERR_UNSUPPORTED, "peers: this layer's combine does not run on the 2-SM tensor-core kernel");
  return SLR_OK;
}

}  // namespace

extern "C" {

int slr_lrs_linear_peers_supported(const slr_layer* layer, const void* x, int64_t ldx, int64_t M) {
  FwdCall c;
  if (M <= 0 || prepare_forward(layer, x, ldx, nullptr, 0, M, nullptr, 0, false, c, false) != SLR_OK) return 0;
  return use_pair(*layer, c) ? 1 : 0;
}

int slr_lrs_linear_combine_peers(const slr_layer* layer, const void* x, int64_t ldx, int64_t ldy, int64_t M,
                                 void* workspace, size_t workspace_bytes, const slr_peers* peers, void* stream) {
  PeerArgs pa;
  int rc = to_peer_args(peers, pa);
  if (rc) return rc;
  FwdCall c;
  rc = prepare_forward(layer, x, ldx, pa.y[pa.me], ldy, M, workspace, workspace_bytes, true, c);
  if (rc) return rc;
  rc = check_peer_call(*layer, c, c.a.ldy, M);
  if (rc) return rc;
  return launch_tc2_rowblock(c.a, false, static_cast<cudaStream_t>(stream), &pa);
}

int slr_lrs_linear_group_combine_peers(const slr_layer* layers, int n, int i, const void* x, int64_t ldx,
                                       int64_t ldy, int64_t M, void* workspace, size_t workspace_bytes,
                                       const slr_peers* peers, void* stream) {
  if (i < 0 || i >= n) return fail(SLR_ERR_INVALID_ARGUMENT, "layer index out of range");
  PeerArgs pa;
  int rc = to_peer_args(peers, pa);
  if (rc) return rc;
  GroupCall gc;
  rc = prepare_group(layers, n, x, ldx, nullptr, nullptr, M, workspace, workspace_bytes, gc);
  if (rc) return rc;
  FwdCall c = gc.c[i];
  rc = prepare_forward(&layers[i], x, ldx, pa.y[pa.me], ldy, M, gc.ws + gc.g.off[i], gc.g.bytes[i], true, c,
                       gc.mode == GROUP_EACH);
  if (rc) return rc;
  c.a.H = gc.c[i].a.H;
  c.a.ldh = gc.c[i].a.ldh;
  rc = check_peer_call(layers[i], c, c.a.ldy, M);
  if (rc) return rc;
  return launch_tc2_rowblock(c.a, false, static_cast<cudaStream_t>(stream), &pa);
}

int slr_lrs_linear_multi_combine_peers(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx,
                                       const void* const* H, const int64_t* ldh, const int64_t* ldy, int64_t M,
                                       const slr_peers* peers, const slr_peers* sync, void* stream) {
  if (!layers || !x || !peers || !sync || n < 1 || n > kMaxLaunchLayers)
    return fail(SLR_ERR_INVALID_ARGUMENT, "bad arguments (1.." + std::to_string(kMaxLaunchLayers) + " layers)");
  PeerArgs ps;
  int rc = to_peer_args(sync, ps);
  if (rc) return rc;
  PeerArgs pa[kMaxLaunchLayers];
  RowblockArgs as[kMaxLaunchLayers];
  for (int i = 0; i < n; ++i) {
    rc = to_peer_args(&peers[i], pa[i]);
    if (rc) return rc;
    if (pa[i].world != ps.world || pa[i].me != ps.me)
      return fail(SLR_ERR_INVALID_ARGUMENT, "peers: world or rank differs between the layers and sync");
    const int64_t lx = (ldx && ldx[i]) ? ldx[i] : layers[i].in_features;
    const int64_t ly = (ldy && ldy[i]) ? ldy[i] : layers[i].out_features;
    FwdCall c;
    rc = prepare_forward(&layers[i], x[i], lx, pa[i].y[pa[i].me], ly, M, nullptr, 0, true, c, false);
    if (rc) return rc;
    if (layers[i].rank > 0) {
      const int64_t lh = (ldh && ldh[i]) ? ldh[i] : round_up(layers[i].rank, 64);
      if (!H || !H[i] || !aligned16(H[i]) || lh < layers[i].rank || lh % 8)
        return fail(SLR_ERR_INVALID_ARGUMENT, "H of layer " + std::to_string(i) +
                                                  ": NULL, not 16-byte aligned, or ldh < rank / not a multiple of 8");
      c.a.H = H[i];
      c.a.ldh = lh;
    }
    rc = check_peer_call(layers[i], c, c.a.ldy, M);
    if (rc) return rc;
    as[i] = c.a;
  }
  return launch_tc2_rowblock_group_peers(as, n, pa, ps, static_cast<cudaStream_t>(stream));
}

int slr_peers_wait(const slr_peers* peers, int empty_shard, void* stream) {
  PeerArgs pa;
  int rc = to_peer_args(peers, pa);
  if (rc) return rc;
  return launch_peer_wait(pa, empty_shard != 0, static_cast<cudaStream_t>(stream));
}

int slr_dense_to_bsr_mask(const void* S, int64_t n, int64_t m, int64_t block_p, int64_t block_q,
                          int dtype, uint8_t* mask, int64_t* crow, void* stream) {
  if (!valid_dtype(dtype)) return fail(SLR_ERR_UNSUPPORTED_DTYPE, "dense_to_bsr: dtype must be f32/f16/bf16");
  if (block_p <= 0 || block_q <= 0 || n < 0 || m < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "bad sizes");
  if (n % block_p || m % block_q)
    return fail(SLR_ERR_INVALID_ARGUMENT, "shape (" + std::to_string(n) + ", " + std::to_string(m) +
                                              ") not divisible by block (" + std::to_string(block_p) + ", " +
                                              std::to_string(block_q) + ")");
  if (!crow || ((n / block_p) * (m / block_q) > 0 && (!S || !mask)))
    return fail(SLR_ERR_INVALID_ARGUMENT, "null pointer");
  return launch_bsr_mask(S, n, m, block_p, block_q, dtype, mask, crow, static_cast<cudaStream_t>(stream));
}

int slr_dense_to_bsr_fill(const void* S, int64_t n, int64_t m, int64_t block_p, int64_t block_q, int dtype,
                          const uint8_t* mask, const int64_t* crow, int64_t* col, void* values,
                          int transpose, void* stream) {
  if (!valid_dtype(dtype)) return fail(SLR_ERR_UNSUPPORTED_DTYPE, "dense_to_bsr: dtype must be f32/f16/bf16");
  if (block_p <= 0 || block_q <= 0 || n < 0 || m < 0 || n % block_p || m % block_q)
    return fail(SLR_ERR_INVALID_ARGUMENT, "bad sizes");
  if (!crow) return fail(SLR_ERR_INVALID_ARGUMENT, "null pointer");
  return launch_bsr_fill(S, n, m, block_p, block_q, dtype, mask, crow, col, values, transpose != 0,
                         static_cast<cudaStream_t>(stream));
}

int slr_plan_stages(const int32_t* crow, const int32_t* col, int64_t NB, const int32_t* order, int64_t block_p,
                    uint32_t* plan, int32_t* stage_start, int64_t capacity, int64_t* n_words) {
  if (!n_words || NB < 0 || (NB > 0 && (!crow || (crow[NB] > 0 && !col))))
    return fail(SLR_ERR_INVALID_ARGUMENT, "bad arguments");
  if (block_p != 16 && block_p != 32 && block_p != 64)
    return fail(SLR_ERR_UNSUPPORTED, "stage schedules exist for block_p 16, 32 or 64 only");
  const int G = int(256 / block_p);
  const int64_t groups = (NB + G - 1) / G;
  if (plan && !stage_start) return fail(SLR_ERR_INVALID_ARGUMENT, "stage_start is NULL");
  // Pass 1 counts stages (records) and blocks; pass 2 writes records
  // [0, 2 * stages) and the block indices after them.  The merge is the
  // kernel's: the next column is the smallest head among the group's rows;
  // every row whose head equals it advances.
  int64_t n_st = 0, n_blk = 0;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1 && !plan) break;
    if (pass == 1 && 2 * n_st + n_blk > capacity) return fail(SLR_ERR_INVALID_ARGUMENT, "plan capacity too small");
    int64_t st = 0, bk = 2 * n_st;
    for (int64_t gi = 0; gi < groups; ++gi) {
      if (pass == 1) stage_start[gi] = int32_t(st);
      const int cnt = int(std::min<int64_t>(G, NB - gi * G));
      int64_t ptr[16], end[16];
      for (int j = 0; j < cnt; ++j) {
        const int64_t r = order ? order[gi * G + j] : gi * G + j;
        if (r < 0 || r >= NB) return fail(SLR_ERR_INVALID_ARGUMENT, "row_order entry out of range");
        ptr[j] = crow[r];
        end[j] = crow[r + 1];
      }
      while (true) {
        int64_t c = INT64_MAX;
        for (int j = 0; j < cnt; ++j)
          if (ptr[j] < end[j]) c = std::min<int64_t>(c, col[ptr[j]]);
        if (c == INT64_MAX) break;
        if (c < 0 || c > 0xffff) return fail(SLR_ERR_UNSUPPORTED, "column index outside [0, 65535]");
        uint32_t mask = 0;
        const int64_t first = bk;
        for (int j = 0; j < cnt; ++j)
          if (ptr[j] < end[j] && col[ptr[j]] == c) {
            mask |= 1u << j;
            if (pass == 1) plan[bk] = uint32_t(ptr[j]);
            ++bk;
            ++ptr[j];
          }
        if (pass == 1) {
          plan[2 * st] = uint32_t(c) | (mask << 16);
          plan[2 * st + 1] = uint32_t(first);
        }
        ++st;
      }
    }
    if (pass == 0) {
      n_st = st;
      n_blk = bk;
    } else {
      stage_start[groups] = int32_t(st);
    }
  }
  if (2 * n_st + n_blk > INT32_MAX) return fail(SLR_ERR_UNSUPPORTED, "plan larger than 2^31 words");
  *n_words = 2 * n_st + n_blk;
  return SLR_OK;
}

int slr_plan_row_order(const int32_t* crow_host, int64_t NB, int32_t* order) {
  if (NB < 0 || (NB > 0 && (!crow_host || !order))) return fail(SLR_ERR_INVALID_ARGUMENT, "bad arguments");
  std::vector<int32_t> idx(static_cast<size_t>(NB));
  std::iota(idx.begin(), idx.end(), 0);
  std::stable_sort(idx.begin(), idx.end(), [&](int32_t a, int32_t b) {
    return (crow_host[a + 1] - crow_host[a]) > (crow_host[b + 1] - crow_host[b]);
  });
  std::memcpy(order, idx.data(), sizeof(int32_t) * size_t(NB));
  return SLR_OK;
}

int slr_plan_shards(const int32_t* crow_host, int64_t NB, int64_t block_p, int64_t block_q, int64_t rank,
                    int world, int64_t* bounds) {
  if (world <= 0 || NB < 0 || !bounds || (NB > 0 && !crow_host))
    return fail(SLR_ERR_INVALID_ARGUMENT, "bad arguments");
  // Prefix sums of per-row cost; boundary p sits where the prefix first
  // reaches p/world of the total (ties resolve to the earlier row).
  std::vector<double> pre(static_cast<size_t>(NB) + 1, 0.0);
  for (int64_t i = 0; i < NB; ++i)
    pre[size_t(i) + 1] = pre[size_t(i)] + double(crow_host[i + 1] - crow_host[i]) * double(block_p * block_q) +
                         double(block_p) * double(rank);
  const double total = pre[size_t(NB)];
  bounds[0] = 0;
  for (int p = 1; p < world; ++p) {
    const double target = total * p / world;
    int64_t b = std::lower_bound(pre.begin(), pre.end(), target) - pre.begin();
    // pick the closer of b-1 and b
    if (b > 0 && (target - pre[size_t(b - 1)]) <= (pre[size_t(std::min(b, NB))] - target)) b -= 1;
    b = std::max<int64_t>(b, bounds[p - 1]);
    bounds[p] = std::min<int64_t>(b, NB);
  }
  bounds[world] = NB;
  return SLR_OK;
}

}  // extern "C"

namespace {

// Checks and argument packing of the single-launch decode call (inputs
// optional for the size and support queries).
int prepare_decode(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx, void* const* y,
                   const int64_t* ldy, int64_t M, RowblockArgs* as) {
  if (!layers || n <= 0 || n > kMaxLaunchLayers)
    return fail(SLR_ERR_INVALID_ARGUMENT, "a decode call holds 1 to " + std::to_string(kMaxLaunchLayers) + " layers");
  if (M < 0) return fail(SLR_ERR_INVALID_ARGUMENT, "M must be >= 0");
  for (int i = 0; i < n; ++i) {
    if (layers[i].dtype != layers[0].dtype)
      return fail(SLR_ERR_INVALID_ARGUMENT, "the layers of a decode call must share one dtype");
    FwdCall c;
    const void* xi = x ? x[i] : nullptr;
    void* yi = y ? y[i] : nullptr;
    int rc = prepare_forward(&layers[i], xi, ldx ? ldx[i] : 0, yi, ldy ? ldy[i] : 0, x ? M : 0, nullptr, 0, y != nullptr,
                             c, false);
    if (rc) return rc;
    as[i] = c.a;
    as[i].M = M;
  }
  return SLR_OK;
}

}  // namespace

extern "C" {

int slr_lrs_linear_decode_supported(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx,
                                    int64_t M) {
  RowblockArgs as[kMaxLaunchLayers];
  if (prepare_decode(layers, n, x, ldx, nullptr, nullptr, M, as) != SLR_OK) return 0;
  return decode_supported(as, n, M) ? 1 : 0;
}

size_t slr_lrs_linear_decode_workspace_size(const slr_layer* layers, int n, int64_t M) {
  RowblockArgs as[kMaxLaunchLayers];
  if (prepare_decode(layers, n, nullptr, nullptr, nullptr, nullptr, M, as) != SLR_OK) return 0;
  return decode_workspace_size(as, n, M);
}

int slr_lrs_linear_decode(const slr_layer* layers, int n, const void* const* x, const int64_t* ldx, void* const* y,
                          const int64_t* ldy, int64_t M, void* workspace, size_t workspace_bytes, void* ctrl,
                          void* stream) {
  if (!x || !y) return fail(SLR_ERR_INVALID_ARGUMENT, "x/y is NULL");
  RowblockArgs as[kMaxLaunchLayers];
  int rc = prepare_decode(layers, n, x, ldx, y, ldy, M, as);
  if (rc || M == 0) return rc;
  if (!decode_supported(as, n, M))
    return fail(SLR_ERR_UNSUPPORTED, "decode: layer set outside the single-launch path "
                                     "(16-bit, rank % 16 == 0 and <= 512, blocks 16/32/64, M <= 32, aligned inputs)");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(SLR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  bool pdl = true;
  for (int i = 0; i < n; ++i) pdl = pdl && early_start(layers[i]);
  return launch_decode(as, n, M, workspace, workspace_bytes, static_cast<unsigned*>(ctrl), pdl,
                       static_cast<cudaStream_t>(stream));
}

}  // extern "C"
