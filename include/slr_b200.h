/*
 * slr_b200.h — C ABI of libslr_b200.so, the B200 (sm_100a) implementation of
 * S-SALAAD's sparse-plus-low-rank (S+LR) linear forward
 *
 *     y = x · Sᵀ + (x · Bᵀ) · Aᵀ + bias
 *
 * with S block-sparse in BSR form.  Names follow the reference: the weight is
 * W ≈ A·B + S with A [out, r] and B [r, in] (ssalaad/efficient/ls_linear.py:
 * 20-27), BSR indices are int32 crow/col, BSR values are stored per block
 * TRANSPOSED as [nnz, block_q, block_p] (ls_linear.py:92-94), and
 * active_rows lists the block-rows that hold at least one block
 * (ls_linear.py:95-97).  Paths in citations are within the S-SALAAD project.
 *
 * Conventions shared by every entry point:
 *   - Plain pointers and sizes; no framework types.  Device pointers refer to
 *     memory on the CUDA device that is current on the calling thread.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Work is enqueued on it; nothing synchronises the host unless
 *     the entry point's comment says so.
 *   - The return value is an slr_status; 0 means success.  Nothing calls
 *     exit() or abort().  slr_last_error() returns a message for the last
 *     failing call on the calling thread.
 *   - The library allocates no device memory inside these calls.  Scratch
 *     memory is the caller's "workspace" (size from the matching *_size
 *     query).
 *   - dtype is an slr_dtype: every floating-point tensor of one call has the
 *     same element type, as in the reference (addmm_inplace.py:100-104).
 */
#ifndef SLR_B200_H_
#define SLR_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SLR_ABI_VERSION 8

#if defined(__GNUC__)
#define SLR_API __attribute__((visibility("default")))
#else
#define SLR_API
#endif

typedef enum slr_status {
  SLR_OK = 0,
  SLR_ERR_INVALID_ARGUMENT = 1, /* bad shape / size / null pointer (Python: ValueError) */
  SLR_ERR_UNSUPPORTED_DTYPE = 2, /* element type not supported (Python: TypeError) */
  SLR_ERR_UNSUPPORTED = 3,       /* valid but unsupported configuration (Python: RuntimeError) */
  SLR_ERR_CUDA = 4,              /* a CUDA runtime call or launch failed */
  SLR_ERR_WORKSPACE = 5,         /* workspace missing, too small or misaligned */
  SLR_ERR_BAD_INDEX = 6,         /* slr_validate_bsr found an index out of range */
  SLR_ERR_TIMEOUT = 7            /* a bounded device-side wait gave up */
} slr_status;

/* slr_layer.flags: run the combine phase of large batches (M >= 256, block_p
 * 32 or 64) on SM pairs with 2-SM MMAs (M = 256 per MMA) even when the layer
 * has no column schedule.  With a schedule (slr_layer.stage_plan) the pair
 * kernel is the default for those shapes. */
#define SLR_FLAG_PAIR_MMA 1
/* slr_layer.flags: launch every kernel of a call only after all earlier work
 * on the stream has finished.  Without it, the small-batch kernels (M < 128)
 * of slr_lrs_linear_forward / _lowrank / _combine / _forward_noalloc start
 * while the kernel issued before them is still running (programmatic
 * dependent launch) and load the layer's weights (values, col, crow,
 * row_order, A, B, bias) meanwhile; x, y and the workspace are touched only
 * after that kernel has completed.  Set it when the kernel issued just before
 * the call may still be writing this layer's weights and signals early
 * completion itself (griddepcontrol.launch_dependents). */
#define SLR_FLAG_STRICT_ORDER 2

typedef enum slr_dtype {
  SLR_F32 = 0,
  SLR_F16 = 1,
  SLR_BF16 = 2
} slr_dtype;

/* ------------------------------------------------------------ library -- */

SLR_API int slr_abi_version(void);
SLR_API const char* slr_status_string(int status);
/* Message of the last failing call on this thread ("" if none). */
SLR_API const char* slr_last_error(void);
/* Caps the SMs that the persistent tensor-core kernels fill (n <= 0: all),
 * process-wide, e.g. to leave SMs to NCCL kernels that run alongside in a
 * multi-GPU step.  No reference counterpart. */
SLR_API int slr_set_sm_limit(int n);
/* Reads and clears the device-side status word that bounded waits set when
 * they time out (SLR_OK or SLR_ERR_TIMEOUT).  Synchronises the device. */
SLR_API int slr_device_status(int* status_out);

/* ------------------------------------------------- in-place BSR addmm -- */

/*
 * out[M, NB*block_p] += x[M, K] · Sᵀ, in place, for the block-rows listed in
 * active_rows (others untouched); fp32 accumulation, one rounding to dtype.
 *
 * Replaces the torch operator
 *   ssalaad::tilelang_bsr_addmm_inplace_dense_(Tensor(a!) out_inplace,
 *       Tensor x, Tensor crow_indices, Tensor col_indices, Tensor values,
 *       Tensor active_rows) -> ()
 * defined at ssalaad/tilelang_sparse/addmm_inplace.py:130-141, whose
 * implementation is _tilelang_bsr_addmm_inplace_dense_impl (:88-127) and
 * kernel _bsr_body (:41-82); and, for dtype SLR_F32, the CPU operator
 * bsr_addmm_avx2_ (ssalaad/cpu_sparse/bsr_addmm_avx2.cpp:144-178).
 *
 *   out          device, [M, NB*block_p] row-major, dtype
 *   x            device, [M, K] row-major, dtype; K % block_q == 0
 *   crow         device int32 [NB+1]
 *   col          device int32 [nnz], each in [0, K/block_q)
 *   values       device, [nnz, block_q, block_p], dtype
 *   active_rows  device int32 [active_nb], each in [0, NB)
 *   block_p, block_q: multiples of 16 for SLR_F16/SLR_BF16 (the reference
 *     CUDA kernel's rule, ls_linear.py:114-117), multiples of 8 for SLR_F32.
 * Unlike the reference CUDA operator, M needs no padding to a tile multiple.
 * For SLR_F32 each output element is accumulated in exactly the reference
 * AVX2 kernel's order (fused multiply-adds over blocks in crow order, then k
 * ascending), so the result is bit-identical to bsr_addmm_avx2_.
 */
SLR_API int slr_bsr_addmm_inplace(void* out, const void* x, int64_t M, int64_t K,
                          const int32_t* crow, int64_t NB, const int32_t* col,
                          const void* values, int64_t nnz, int64_t block_p,
                          int64_t block_q, const int32_t* active_rows,
                          int64_t active_nb, int dtype, void* stream);

/*
 * Checks a BSR structure on the device: crow[0] == 0, crow non-decreasing,
 * crow[NB] == nnz, every col in [0, nbk), every active row in [0, NB) with a
 * nonempty block-row.  The reference checks none of this on the GPU (its
 * kernel only assumes col in range, addmm_inplace.py:76-77); the layer
 * classes call this once at construction.  Synchronises `stream`.
 * Returns SLR_OK or SLR_ERR_BAD_INDEX.
 */
SLR_API int slr_validate_bsr(const int32_t* crow, int64_t NB, const int32_t* col,
                     int64_t nnz, int64_t nbk, const int32_t* active_rows,
                     int64_t active_nb, void* stream);

/* ------------------------------------------------------ S+LR forward -- */

/* One S+LR linear layer: the buffers of _LRSLinearLRBlockBase
 * (ls_linear.py:57-97) plus an optional block-row schedule. */
typedef struct slr_layer {
  int64_t in_features;    /* K */
  int64_t out_features;   /* N */
  int64_t rank;           /* r (A.shape[1] == B.shape[0]); may be 0 */
  int64_t block_p;        /* rows of a block (output features); 0 if nnz == 0 */
  int64_t block_q;        /* cols of a block (input features);  0 if nnz == 0 */
  int64_t nnz;            /* number of stored blocks; 0 = low-rank only */
  const int32_t* crow;    /* device int32 [N/block_p + 1] (ignored if nnz == 0) */
  const int32_t* col;     /* device int32 [nnz] */
  const void* values;     /* device [nnz, block_q, block_p] */
  const int32_t* row_order; /* device int32 [N/block_p] permutation of the
                               block-rows, heaviest first, from
                               slr_plan_row_order; NULL = natural order */
  const void* A;          /* device [N, r] */
  const void* B;          /* device [r, K] */
  const void* bias;       /* device [N] or NULL */
  int32_t dtype;          /* slr_dtype of x, y, values, A, B, bias */
  int32_t flags;          /* 0, or SLR_FLAG_PAIR_MMA | SLR_FLAG_STRICT_ORDER */
  const uint32_t* stage_plan;  /* device: column schedule of the tensor-core
                                  path from slr_plan_stages for these crow, col,
                                  row_order and block_p; NULL = computed on
                                  the fly by the kernel (same result) */
  const int32_t* stage_start;  /* device int32 [groups + 1] from slr_plan_stages */
  int64_t route_out_features;  /* 0, or (for a block-row shard of a wider layer)
                                  the whole layer's out_features: kernels are
                                  then chosen as for the whole layer, so the
                                  shard's outputs equal the whole layer's bit
                                  for bit */
} slr_layer;

/*
 * Workspace bytes that slr_lrs_linear_forward needs for M tokens (it holds
 * H = x·Bᵀ between the two phases).  The workspace must be 256-byte aligned
 * and not shared by calls that may overlap on the GPU; it needs no
 * initialisation.
 */
SLR_API size_t slr_lrs_linear_workspace_size(const slr_layer* layer, int64_t M);

/*
 * y[M, N] = x[M, K] · Sᵀ + (x · Bᵀ) · Aᵀ + bias.
 *
 * Replaces the forward of the compressed layer on CUDA,
 * _LRSLinearLRBlockCUDA.forward (ls_linear.py:124-137: pad, two F.linear
 * calls, the in-place sparse operator, the bias add, slice), and with
 * nnz == 0 the low-rank-only layer _LRSLinearLR.forward (ls_linear.py:47-51).
 * For SLR_F32 it computes the CPU layer's arithmetic
 * (_LRSLinearLRBlockCPU.forward, ls_linear.py:155-164): the low-rank
 * product in fp32, then the sparse term accumulated in the reference
 * kernel's order, then the bias.  For 16-bit dtypes x·Bᵀ is rounded to the
 * dtype (as the reference's first F.linear does) and everything after it is
 * accumulated in fp32 and rounded once.
 *   ldx  row stride of x in elements (0 = K); ldy row stride of y (0 = N).
 * y must not overlap x.  No M padding is needed.  Equivalent to
 * slr_lrs_linear_lowrank followed by slr_lrs_linear_combine, with the second
 * launch allowed to start its sparse part while the first finishes.
 */
SLR_API int slr_lrs_linear_forward(const slr_layer* layer, const void* x, int64_t ldx,
                           void* y, int64_t ldy, int64_t M, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * Phase 1 alone: H = x · Bᵀ into the workspace (the reference's first
 * F.linear, ls_linear.py:131).  A no-op when rank == 0.
 */
SLR_API int slr_lrs_linear_lowrank(const slr_layer* layer, const void* x, int64_t ldx,
                           int64_t M, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Phase 2 alone: y = x · Sᵀ + H · Aᵀ + bias with H read from a workspace that
 * slr_lrs_linear_lowrank filled for the same layer, x and M (the reference's
 * second F.linear, sparse operator and bias, ls_linear.py:131-137).
 */
SLR_API int slr_lrs_linear_combine(const slr_layer* layer, const void* x, int64_t ldx,
                           void* y, int64_t ldy, int64_t M, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * slr_lrs_linear_forward without a workspace argument, for callers that
 * cannot allocate device memory (a plugin inside a framework that owns all
 * allocations, code running under someone else's stream capture, a serving
 * loop that must not enter the allocator).  No counterpart in the reference.
 * Scratch comes from a fixed 16 MiB array in this library's device image
 * (held by every GPU that loads the library until exit); a token count that
 * needs more is rejected with SLR_ERR_WORKSPACE before any launch.  The first
 * call on a device looks up the array's address for that device: make it
 * before any stream capture.  The address is kept for the life of the
 * process, so a cudaDeviceReset after the first call is not supported.  The
 * scratch needs no initialisation: each call overwrites what it reads.  All
 * calls share the array; calls that overlap on the GPU race on it.
 */
SLR_API int slr_lrs_linear_forward_noalloc(const slr_layer* layer, const void* x,
                           int64_t ldx, void* y, int64_t ldy, int64_t M,
                           void* stream);

/*
 * n (1..4) layers that read the same x — the q/k/v or gate/up projections of
 * a decoder layer, each an _LRSLinearLRBlockCUDA (ls_linear.py:124-137)
 * called on one input by the reference: y[i] = x · S_iᵀ + (x · B_iᵀ) · A_iᵀ
 * + bias_i, the results of slr_lrs_linear_forward on each layer, bit for
 * bit.  When every layer has a rank and takes a 16-bit path, the x · B_iᵀ
 * products are one launch over the stacked B_i into H [M, sum of
 * round_up(r_i, 64)] at the start of the workspace: a tensor-core GEMM from
 * M >= 128 on (x is read once, the GEMM has n times the tiles), the
 * small-batch kernel below (each B_i keeps its own K split, so H is the same
 * bit for bit), where the combine of all layers is one launch too when their
 * block and rank chunk shapes agree.  The M >= 128 layout depends on M only,
 * so _group_lowrank on tokens [t0, t0 + m) (m >= 128) with the workspace
 * advanced by t0 H rows fills exactly those rows of the H of all M tokens (a
 * multi-GPU caller can split the tokens and all-gather H).
 * Layers must share in_features and dtype; ldy may be NULL (packed rows).
 * The workspace rules are those of slr_lrs_linear_forward.
 */
SLR_API size_t slr_lrs_linear_group_workspace_size(const slr_layer* layers, int n, int64_t M);
SLR_API int slr_lrs_linear_forward_group(const slr_layer* layers, int n, const void* x,
                           int64_t ldx, void* const* y, const int64_t* ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* stream);
/* The two phases of slr_lrs_linear_forward_group, like _lowrank / _combine
 * for one layer: the group's x · B_iᵀ, then layer i's combine (any order of
 * i, same x, M and workspace).  Within slr_lrs_linear_forward_group, from
 * 128 tokens on, the combines of layers that all take the 2-SM pair kernel
 * with one block shape are one launch. */
SLR_API int slr_lrs_linear_group_lowrank(const slr_layer* layers, int n, const void* x,
                           int64_t ldx, int64_t M, void* workspace,
                           size_t workspace_bytes, void* stream);
SLR_API int slr_lrs_linear_group_combine(const slr_layer* layers, int n, int i,
                           const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* stream);

/*
 * n (1..8) layers, each with its own input: y[i] = x[i] · S_iᵀ +
 * (x[i] · B_iᵀ) · A_iᵀ + bias_i for i < n, the result of
 * slr_lrs_linear_forward on each layer bit for bit.  It serves a step that
 * runs independent projections side by side (a layer set whose inputs are
 * all ready, or the same projection of several models); layers may also
 * share an input (pass the same pointer).  Below 128 tokens, when every layer
 * takes the 16-bit small-batch path and has a rank, all x[i] · B_iᵀ products
 * are one launch and the combine phases of all layers one more launch (when
 * their block and rank-chunk shapes agree; else one per layer), instead of
 * two launches per layer.  From 128 tokens on the layers run one forward
 * each.  Layers share the dtype; ldx / ldy may be NULL (packed rows).  The
 * workspace rules are those of slr_lrs_linear_forward.  No reference
 * counterpart (the reference calls its layers one by one,
 * ssalaad/efficient/ls_linear.py:124-137).
 */
SLR_API size_t slr_lrs_linear_multi_workspace_size(const slr_layer* layers, int n, int64_t M);
SLR_API int slr_lrs_linear_forward_multi(const slr_layer* layers, int n, const void* const* x,
                           const int64_t* ldx, void* const* y, const int64_t* ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* stream);
/* Where slr_lrs_linear_multi_lowrank leaves each layer's H = x·Bᵀ for this
 * call (same arguments): H[i] its first element, ldh[i] its row stride in
 * elements (NULL / 0 for a layer without rank).  For callers that read H
 * themselves, e.g. slr_lrs_linear_multi_combine_peers.  No reference
 * counterpart. */
SLR_API int slr_lrs_linear_multi_h(const slr_layer* layers, int n, const void* const* x,
                                   const int64_t* ldx, int64_t M, void* workspace,
                                   size_t workspace_bytes, void** H, int64_t* ldh);
/* The two phases of slr_lrs_linear_forward_multi (same layers, inputs, M and
 * workspace in both calls): every layer's x[i] · B_iᵀ, then the combines.
 * From 128 tokens on, when every layer takes the 2-SM pair kernel with one
 * block shape (layers with a column schedule), the combines of all layers
 * are ONE launch whose work items are dealt as one list, so the set pays
 * one persistent-schedule tail; results equal per-layer calls bit for bit. */
SLR_API int slr_lrs_linear_multi_lowrank(const slr_layer* layers, int n, const void* const* x,
                           const int64_t* ldx, int64_t M, void* workspace, size_t workspace_bytes,
                           void* stream);
SLR_API int slr_lrs_linear_multi_combine(const slr_layer* layers, int n, const void* const* x,
                           const int64_t* ldx, void* const* y, const int64_t* ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------- single-launch decode -- */

/* Bytes of the control block of slr_lrs_linear_decode. */
#define SLR_DECODE_CTRL_BYTES 4096
/* Largest token count of slr_lrs_linear_decode. */
#define SLR_DECODE_MAX_TOKENS 32

/*
 * n (1..8) layers, each with its own input (or a shared one), and 1 ..
 * SLR_DECODE_MAX_TOKENS tokens in ONE kernel launch: x[i] · B_iᵀ and the
 * combine phase of every layer run in one kernel (each CTA computes a tile
 * of some layer's H and one block-row of some layer's y; a block-row waits
 * inside the kernel until its layer's H is written), so a decode step pays
 * one kernel boundary.  An alternative to the two-launch small-batch path
 * of slr_lrs_linear_forward / _forward_multi, not a replacement: measured on
 * B200 it is faster only for large layer sets (seven LLaMA-1B-shaped
 * projections at one token: 36 µs against 38 µs) and slower for single
 * layers and small layer sets.  y[i] = x[i] · S_iᵀ + (x[i] · B_iᵀ) · A_iᵀ +
 * bias_i, x · Bᵀ rounded to the dtype and the rest accumulated in fp32 and
 * rounded once, as in slr_lrs_linear_forward.  The arithmetic of a layer
 * depends on its own shape only: the result is the same bit for bit whatever
 * the other layers of the call and whatever M <= SLR_DECODE_MAX_TOKENS for the
 * same token rows (it is not bit-identical to the two-launch path of
 * slr_lrs_linear_forward, which splits K differently).
 *
 * Handled (slr_lrs_linear_decode_supported): 16-bit dtypes, one dtype for all
 * layers; rank a multiple of 16 up to 512; in_features and ldx multiples of
 * 8; block_p and block_q 16, 32 or 64; x, A, B and values 16-byte aligned.
 * ctrl: SLR_DECODE_CTRL_BYTES of device memory, 16-byte aligned, all zero
 * before the first call that uses it; every call leaves it zero again (also
 * a call that reports SLR_ERR_TIMEOUT).  Calls that may run at the same time
 * on the GPU need separate control blocks.  The workspace (size from
 * slr_lrs_linear_decode_workspace_size) needs no initialisation.  ldx / ldy
 * may be NULL (packed rows).  No reference counterpart (the reference runs
 * two F.linear calls, the sparse operator and the bias add per layer,
 * ssalaad/efficient/ls_linear.py:124-137).
 */
SLR_API int slr_lrs_linear_decode_supported(const slr_layer* layers, int n, const void* const* x,
                           const int64_t* ldx, int64_t M);
SLR_API size_t slr_lrs_linear_decode_workspace_size(const slr_layer* layers, int n, int64_t M);
SLR_API int slr_lrs_linear_decode(const slr_layer* layers, int n, const void* const* x,
                           const int64_t* ldx, void* const* y, const int64_t* ldy, int64_t M,
                           void* workspace, size_t workspace_bytes, void* ctrl, void* stream);

/* ------------------------------------------- N:M 2:4 + low-rank layer -- */

/*
 * The other compressed-layer kind of the reference: y = x · Sᵀ + (x · Bᵀ) ·
 * Aᵀ + bias with S 2:4 sparse along K (at most 2 nonzeros in every aligned
 * group of 4 input features of a row), _LRSLinearLRNM (ssalaad/efficient/
 * ls_linear.py:167-224), whose forward (:210-221) runs S on torch's
 * semi-structured (cuSPARSELt) tensor.  Here S is kept as
 *   values [N, K/2]  (dtype) the two kept entries of every group of 4, in
 *                    K order (zeros at the lowest unused positions of a group
 *                    with fewer nonzeros);
 *   meta   [N, K/32] uint32: word w of row n covers K [32w, 32w + 32), bits
 *                    [4i, 4i + 4) group i: low 2 bits the position of the
 *                    first kept entry, high 2 bits the second (first < second).
 * 16-bit dtypes; N % 16 == 0, K % 32 == 0, rank % 8 == 0 (rank >= 16).
 */
typedef struct slr_nm_layer {
  int64_t in_features;    /* K */
  int64_t out_features;   /* N */
  int64_t rank;           /* r */
  const void* values;     /* device [N, K/2] */
  const uint32_t* meta;   /* device [N, K/32] */
  const void* A;          /* device [N, r] */
  const void* B;          /* device [r, K] */
  const void* bias;       /* device [N] or NULL */
  int32_t dtype;          /* SLR_F16 or SLR_BF16 */
  int32_t flags;          /* 0 or SLR_FLAG_STRICT_ORDER */
} slr_nm_layer;

/*
 * Dense S [N, K] (row-major, dtype) -> values and meta above.  Entries that
 * are nonzero (or NaN) are kept; SLR_ERR_BAD_INDEX if a group of 4 holds more
 * than two of them (S is not 2:4 sparse).  Synchronises `stream`.  No
 * reference counterpart: the reference packs with
 * torch.sparse.to_sparse_semi_structured (ssalaad/efficient/artifact.py:44-61).
 */
SLR_API int slr_nm_compress(const void* S, int64_t N, int64_t K, int dtype, void* values, uint32_t* meta,
                            void* stream);
/* Workspace bytes of slr_nm_linear_forward for M tokens (holds H = x · Bᵀ). */
SLR_API size_t slr_nm_linear_workspace_size(const slr_nm_layer* layer, int64_t M);
/*
 * y[M, N] = x[M, K] · Sᵀ + (x · Bᵀ) · Aᵀ + bias: x · Bᵀ rounded to the dtype
 * (the reference's latent), then the 2:4 sparse product on the sparse tensor
 * cores, H · Aᵀ and the bias accumulated in fp32 and rounded once (the
 * reference rounds the sparse product, the addmm and the bias add each).
 * ldx / ldy: row strides in elements (0 = K / N).
 */
SLR_API int slr_nm_linear_forward(const slr_nm_layer* layer, const void* x, int64_t ldx, void* y, int64_t ldy,
                                  int64_t M, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------- dense -> BSR -- */

/*
 * Block mask and crow of dense S[n, m] (row-major, dtype) cut into
 * block_p x block_q blocks — steps 1-3 of dense_to_bsr
 * (ssalaad/efficient/artifact.py:20-33): a block is kept iff the sum of |s|
 * over it is > 0, i.e. it holds a nonzero and no NaN.
 *   mask  device uint8 [(n/block_p) * (m/block_q)]  (1 = kept)
 *   crow  device int64 [n/block_p + 1]              (crow[0] = 0)
 * nnz = crow[n/block_p] (the caller reads it back to size the outputs).
 */
SLR_API int slr_dense_to_bsr_mask(const void* S, int64_t n, int64_t m, int64_t block_p,
                          int64_t block_q, int dtype, uint8_t* mask,
                          int64_t* crow, void* stream);

/*
 * Steps 4-5 of dense_to_bsr (artifact.py:34-37): col indices of the kept
 * blocks in row-major order (torch.nonzero order) and their values, copied
 * bit for bit.
 *   col     device int64 [nnz]
 *   values  device, dtype: [nnz, block_p, block_q] if transpose == 0 (the
 *           artifact / torch.sparse_bsr_tensor layout), or [nnz, block_q,
 *           block_p] if transpose == 1 (the layer layout, ls_linear.py:92-94)
 */
SLR_API int slr_dense_to_bsr_fill(const void* S, int64_t n, int64_t m, int64_t block_p,
                          int64_t block_q, int dtype, const uint8_t* mask,
                          const int64_t* crow, int64_t* col, void* values,
                          int transpose, void* stream);

/* -------------------------------------------------- planning (host) -- */

/*
 * Host-only.  Writes the block-rows in the order a persistent schedule should
 * take them: descending work (nnz of the row), ties by row index.  The
 * reference launches one CTA per active row in index order
 * (addmm_inplace.py:65); this order feeds heavy (skewed) rows first.
 */
/*
 * Column schedule of the tensor-core path (M >= 128), built once per layer on
 * the host.  The kernel processes block-rows in groups of G = 256 / block_p
 * (block_p 16, 32 or 64) taken consecutively from row_order (NULL = natural
 * order); for each group it visits the union of the rows' columns, one stage
 * per distinct column.  slr_plan_stages writes `plan` (uint32 words): for
 * every stage a record {column | (mask of the group rows that have it) << 16,
 * index of its first block index}, i.e. words [2s, 2s+1], then, after all
 * records, the value-block index of each present row of each stage.
 * stage_start[group] is the group's first stage (groups + 1 entries, the
 * last = total stages).  The kernel's producers then take stages
 * independently instead of merging col[] lists.  With plan == NULL only
 * *n_words is set.  SLR_ERR_UNSUPPORTED if block_p is not 16, 32 or 64 or a
 * column index exceeds 65535.  No reference counterpart (the reference kernel
 * walks one row per CTA, addmm_inplace.py:67-80).
 */
SLR_API int slr_plan_stages(const int32_t* crow_host, const int32_t* col_host, int64_t NB,
                            const int32_t* row_order_host, int64_t block_p, uint32_t* plan,
                            int32_t* stage_start, int64_t capacity, int64_t* n_words);

SLR_API int slr_plan_row_order(const int32_t* crow_host, int64_t NB, int32_t* order);

/*
 * Host-only.  Splits NB block-rows into `world` contiguous ranges of nearly
 * equal cost c_i = nnz_i*block_p*block_q + block_p*rank (the multiply-adds a
 * row costs per token).  bounds[world+1]: rank p owns block-rows
 * [bounds[p], bounds[p+1]).  No reference counterpart: the reference runs on
 * one device.
 */
SLR_API int slr_plan_shards(const int32_t* crow_host, int64_t NB, int64_t block_p,
                    int64_t block_q, int64_t rank, int world, int64_t* bounds);

/* ------------------------------- multi-GPU: y assembled in peer memory -- */

/*
 * A block-row-sharded layer on `world` GPUs (one process each) whose combine
 * kernel stores every output tile into its own y AND into the y of every
 * other rank over NVLink (CUDA IPC mappings), instead of a local slot plus an
 * NCCL all-gather and a column reassembly.  No reference counterpart: the
 * reference runs on one device.
 *
 * Each rank owns a full y [M, N] (same ldy on every rank) and, per layer, a
 * signal slot of SLR_SIGNAL_WORDS uint64 words that is zero before the first
 * call.  y[p] is rank p's y advanced to THIS rank's first output column;
 * signal[p] is rank p's slot of the layer.  A call is
 * slr_lrs_linear_combine_peers (or the group form; ranks without rows of the
 * layer call slr_peers_wait with empty_shard = 1 instead) followed by
 * slr_peers_wait on the same stream; after the wait, y on this rank holds
 * every rank's columns.  Every rank must make the calls of a layer in the
 * same order.  Each rank numbers the calls by its own count and writes its
 * number into one word per rank of every slot, so words left by an older
 * call never satisfy a newer call's wait.
 *
 * Waits on other ranks are bounded (slr_set_wait_limit_ns, 2 s by default)
 * and report SLR_ERR_TIMEOUT through slr_device_status.  A rank that gives up
 * a wait marks the call as failed in every rank's slot, so every rank's wait
 * for that call reports the timeout and the y of that call must not be used.
 * If every rank still makes every call, the next calls are synchronised again
 * by their numbers.  A rank that skips (or repeats) a call makes every later
 * wait of the layer time out on all ranks, until all ranks meet on the host
 * and zero their slots.
 */
#define SLR_MAX_RANKS 8
#define SLR_IPC_HANDLE_BYTES 64
#define SLR_SIGNAL_WORDS 32

/* Limit, in ns, of every later wait on other ranks (the peer epilogue and
 * slr_peers_wait) and of the decode kernel's wait for H written by its other
 * CTAs (there at most 1 s), process-wide; 0 restores the default of 2 s.
 * Waits inside one CTA (its own pipeline) keep their fixed 2 s limit.  No
 * reference counterpart. */
SLR_API int slr_set_wait_limit_ns(uint64_t ns);

typedef struct slr_peers {
  int32_t world;                    /* ranks, 2..SLR_MAX_RANKS */
  int32_t rank;                     /* this rank */
  void* y[SLR_MAX_RANKS];           /* rank p's y at this rank's first column */
  uint64_t* signal[SLR_MAX_RANKS];  /* rank p's signal slot of this layer */
} slr_peers;

/* The IPC handle (SLR_IPC_HANDLE_BYTES) of the device allocation holding
 * dev_ptr and dev_ptr's offset in it; slr_ipc_import on another process maps
 * it (once per handle and process; counted) and returns the same address
 * there; slr_ipc_release drops one import. */
SLR_API int slr_ipc_export(const void* dev_ptr, void* handle, int64_t* offset);
SLR_API int slr_ipc_import(const void* handle, int64_t offset, void** dev_ptr);
SLR_API int slr_ipc_release(const void* handle);

/* 1 when the combine of `layer` on M tokens (x row stride ldx) runs on the
 * kernel that stores into peers (the 2-SM tensor-core kernel), else 0. */
SLR_API int slr_lrs_linear_peers_supported(const slr_layer* layer, const void* x, int64_t ldx,
                                           int64_t M);
/* slr_lrs_linear_combine (after _lowrank on the same workspace) with the
 * output written to peers->y[p] for every rank p. */
SLR_API int slr_lrs_linear_combine_peers(const slr_layer* layer, const void* x, int64_t ldx,
                                         int64_t ldy, int64_t M, void* workspace,
                                         size_t workspace_bytes, const slr_peers* peers,
                                         void* stream);
/* slr_lrs_linear_group_combine (after _group_lowrank) into peers->y[p]. */
SLR_API int slr_lrs_linear_group_combine_peers(const slr_layer* layers, int n, int i,
                                               const void* x, int64_t ldx, int64_t ldy, int64_t M,
                                               void* workspace, size_t workspace_bytes,
                                               const slr_peers* peers, void* stream);
/* The combines of n (<= 8) layers in ONE launch of the 2-SM kernel, every
 * output tile stored into every rank's y: layer i's into peers[i].y[p].  H[i]
 * is layer i's H = x·Bᵀ [M, ldh[i]] (0 = round_up(rank, 64)) from its low-rank
 * phase, wherever the caller keeps it (a layer's or a group's workspace, rows
 * gathered from other ranks).  The launch's arrival and completion signals
 * use sync's signal slots (sync.y is not read); end the call with
 * slr_peers_wait(sync, 0, stream).  A rank with no rows in any of the layers
 * calls slr_peers_wait(sync, 1, stream) instead (SLR_ERR_INVALID_ARGUMENT
 * here).  SLR_ERR_UNSUPPORTED when the layers cannot share one launch (each
 * on the 2-SM kernel with a column schedule, one block shape, M and dtype).
 * Every rank must make the calls with the same sync slot in the same order.
 * No reference counterpart. */
SLR_API int slr_lrs_linear_multi_combine_peers(const slr_layer* layers, int n, const void* const* x,
                                               const int64_t* ldx, const void* const* H, const int64_t* ldh,
                                               const int64_t* ldy, int64_t M, const slr_peers* peers,
                                               const slr_peers* sync, void* stream);
/* Ends a call: returns (on the stream) once every rank's stores into this
 * rank's y are visible. */
SLR_API int slr_peers_wait(const slr_peers* peers, int empty_shard, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SLR_B200_H_ */
