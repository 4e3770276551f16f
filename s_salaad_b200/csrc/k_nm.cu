// The N:M 2:4 + low-rank layer:  y = x · Sᵀ + (x · Bᵀ) · Aᵀ + bias with S
// 2:4 sparse along K (at most 2 nonzeros in every aligned group of 4 input
// features of a row).
//
// Reference counterpart: _LRSLinearLRNM.forward
// (ssalaad/efficient/ls_linear.py:210-221): latent = F.linear(x, B), y =
// F.linear(x, S_semi) on torch's semi-structured (cuSPARSELt) tensor,
// y.addmm_(latent, A.t()), bias.  Here the sparse product runs on the sparse
// tensor cores (mma.sp, m16n8k32) in a hand-written kernel, accumulated in
// fp32 together with H·Aᵀ (H = x·Bᵀ rounded to the I/O dtype, as the
// reference's latent) and the bias, and y is rounded once.
//
// Storage (built once by nm_pack_kernel from a dense S):
//   values [N, K/2]   the two kept entries of every group of 4, in K order
//                     (a group with fewer nonzeros keeps zeros at its
//                     lowest unused positions);
//   meta   [N, K/32]  uint32: word w of row n covers K [32w, 32w + 32); bits
//                     [4i, 4i + 4) describe group i (K 32w + 4i .. + 3): low
//                     2 bits the position of the first kept entry, high 2
//                     bits the second (first < second).
// mma.sp (m16n8k32, 16-bit, sparsity selector 0) takes the metadata of a 16 x
// 32 A tile from lanes 4g and 4g + 1 of each quad g: lane 4g holds groups 0-3
// of rows g (bits 0-15) and g + 8 (bits 16-31), lane 4g + 1 groups 4-7 of the
// same rows (checked on a B200 with an exact small-integer product); the
// kernel builds those registers from the two rows' words.
#include <algorithm>

#include "internal.hpp"

namespace slr {
namespace {

__device__ unsigned g_status_nm = 0;

// ---------------------------------------------------------------- packing --

// One thread per (row, 32-wide K word): 8 groups of 4 -> 16 values + 1 word.
// bad gets 1 if a group holds more than 2 nonzeros (not 2:4 sparse).
template <typename TI>
__global__ void nm_pack_kernel(const TI* __restrict__ S, int64_t N, int64_t K, TI* __restrict__ values,
                               uint32_t* __restrict__ meta, int* bad) {
  const int64_t words = K / 32;
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= N * words) return;
  const int64_t n = idx / words, w = idx - n * words;
  const TI* row = S + n * K + w * 32;
  TI* out = values + n * (K / 2) + w * 16;
  uint32_t word = 0;
  for (int i = 0; i < 8; ++i) {
    int pos[2] = {-1, -1}, cnt = 0;
    for (int j = 0; j < 4; ++j) {
      const float v = to_f(row[4 * i + j]);
      if (v != 0.f || v != v) {  // kept: nonzero or NaN
        if (cnt < 2) pos[cnt] = j;
        ++cnt;
      }
    }
    if (cnt > 2) atomicOr(bad, 1);
    // fill missing slots with the lowest unused positions, keeping order
    for (int c = 0; c < 2; ++c) {
      if (pos[c] >= 0) continue;
      for (int j = 0; j < 4; ++j)
        if (j != pos[0] && j != pos[1]) {
          pos[c] = j;
          break;
        }
    }
    if (pos[0] > pos[1]) {
      const int t = pos[0];
      pos[0] = pos[1];
      pos[1] = t;
    }
    out[2 * i] = row[4 * i + pos[0]];
    out[2 * i + 1] = row[4 * i + pos[1]];
    word |= uint32_t(pos[0] | (pos[1] << 2)) << (4 * i);
  }
  meta[n * words + w] = word;
}

// --------------------------------------------------------- the fused layer --

struct NmArgs {
  const void* x;       // [M, ldx]
  void* y;             // [M, ldy]
  const void* values;  // [N, K/2]
  const uint32_t* meta;  // [N, K/32]
  const void* A;       // [N, r]
  const void* H;       // [M, ldh] = x·Bᵀ (I/O dtype) or null when r == 0
  const void* bias;    // [N] or null
  int64_t M, N, K, r, ldx, ldy, ldh;
};

constexpr int kNmWarps = 4;
constexpr int kNmDepth = 4;  // k-steps in flight per warp

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T> struct mma_sp16832;
template <> struct mma_sp16832<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, const uint32_t* b, uint32_t e) {
    asm volatile(
        "mma.sp::ordered_metadata.sync.aligned.m16n8k32.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9,%10,%11}, {%0,%1,%2,%3}, %12, 0x0;"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(b[2]), "r"(b[3]), "r"(e));
  }
};
template <> struct mma_sp16832<__half> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, const uint32_t* b, uint32_t e) {
    asm volatile(
        "mma.sp::ordered_metadata.sync.aligned.m16n8k32.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9,%10,%11}, {%0,%1,%2,%3}, %12, 0x0;"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]), "r"(b[2]), "r"(b[3]), "r"(e));
  }
};

// One CTA = 16 output features x 8*NT tokens.  Its 4 warps split the K steps
// (32 input features each: warp w takes steps w, w + 4, ...) and then the
// 16-wide rank chunks of the low-rank term the same way; each warp streams its
// own tiles through a private ring of kNmDepth slots with cp.async (the
// compressed 16 x 16 value tile, 512 B, and the x tile, 8*NT tokens x 32
// features), with mma.sp for the sparse steps and mma.sync for H·Aᵀ.  The 4
// partial sums are added in warp order, then the bias, and y is written once.
// The smem rows are XOR-swizzled by 16-byte chunk so ldmatrix reads them
// without bank conflicts.
template <int NT, typename TI>
__global__ void __launch_bounds__(kNmWarps * 32) nm_combine_kernel(const NmArgs a) {
  constexpr int TT = 8 * NT;
  constexpr uint32_t A_TILE = 16 * 32;    // 16 rows x 32 bytes
  constexpr uint32_t X_TILE = TT * 64;    // TT rows x 32 features x 2 bytes
  constexpr uint32_t SLOT = A_TILE + X_TILE;
  extern __shared__ __align__(128) uint8_t smem[];
  float* red = reinterpret_cast<float*>(smem + kNmWarps * kNmDepth * SLOT);  // [4][16][TT]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int64_t f0 = int64_t(blockIdx.x) * 16, t0 = int64_t(blockIdx.y) * TT;
  const uint32_t ring = smem_u32(smem + warp * kNmDepth * SLOT);
  const TI* __restrict__ x = static_cast<const TI*>(a.x);
  const TI* __restrict__ vals = static_cast<const TI*>(a.values);
  const TI* __restrict__ Aw = static_cast<const TI*>(a.A);
  const TI* __restrict__ H = static_cast<const TI*>(a.H);

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  // ---- sparse steps: 32 input features each
  const int n_sp = int(a.K / 32);
  const int my_sp = n_sp > warp ? (n_sp - warp + kNmWarps - 1) / kNmWarps : 0;
  // ---- low-rank steps: 16 rank columns each
  const int n_lr = a.H ? int((a.r + 15) / 16) : 0;
  const int my_lr = n_lr > warp ? (n_lr - warp + kNmWarps - 1) / kNmWarps : 0;
  const int my_total = my_sp + my_lr;

  // Issue the loads of this warp's i-th step into slot i % kNmDepth.
  uint32_t metas[kNmDepth];
  auto issue = [&](int i) {
    const uint32_t slot = ring + uint32_t(i % kNmDepth) * SLOT;
    if (i < my_sp) {
      const int s = warp + kNmWarps * i;
      // values: 16 rows x 32 bytes, lane -> (row, 16-byte half)
      const int row = lane >> 1, hf = lane & 1;
      cp_async16(slot + row * 32 + ((hf ^ ((row >> 2) & 1)) << 4),
                 vals + (f0 + row) * (a.K / 2) + int64_t(s) * 16 + hf * 8, 16);
      // x: TT rows x 64 bytes (4 chunks); tokens past M are zero-filled
#pragma unroll
      for (int j = 0; j < TT / 8; ++j) {
        const int q = lane + 32 * j, xr = q >> 2, c = q & 3;
        const int64_t tok = t0 + xr;
        const TI* src = x + (tok < a.M ? tok : 0) * a.ldx + int64_t(s) * 32 + c * 8;
        cp_async16(slot + A_TILE + xr * 64 + ((c ^ ((xr >> 1) & 3)) << 4), src, tok < a.M ? 16u : 0u);
      }
      // metadata: lane 4g takes groups 0-3 of rows g and g + 8, lane 4g + 1 groups 4-7
      uint32_t m = 0;
      if (tq < 2) {
        const uint32_t w0 = __ldg(a.meta + (f0 + g) * (a.K / 32) + s);
        const uint32_t w1 = __ldg(a.meta + (f0 + g + 8) * (a.K / 32) + s);
        m = tq == 0 ? ((w0 & 0xffffu) | (w1 << 16)) : ((w0 >> 16) | (w1 & 0xffff0000u));
      }
      metas[i % kNmDepth] = m;
    } else {
      const int l = warp + kNmWarps * (i - my_sp);  // rank chunk of 16
      // A rows: 16 rows x 16 rank columns (32 bytes)
      const int row = lane >> 1, hf = lane & 1;
      const int64_t col = int64_t(l) * 16 + hf * 8;
      cp_async16(slot + row * 32 + ((hf ^ ((row >> 2) & 1)) << 4), Aw + (f0 + row) * a.r + (col < a.r ? col : 0),
                 col < a.r ? 16u : 0u);
      // H: TT rows x 16 rank columns (32 bytes, 2 chunks)
#pragma unroll
      for (int j = 0; j < (TT * 2 + 31) / 32; ++j) {
        const int q = lane + 32 * j;
        if (q < TT * 2) {
          const int hr = q >> 1, c = q & 1;
          const int64_t tok = t0 + hr;
          const int64_t hc = int64_t(l) * 16 + c * 8;
          const bool ok = tok < a.M && hc < a.r;
          cp_async16(slot + A_TILE + hr * 32 + ((c ^ ((hr >> 2) & 1)) << 4),
                     H + (ok ? tok * a.ldh + hc : 0), ok ? 16u : 0u);
        }
      }
    }
    cp_async_commit();
  };

#pragma unroll
  for (int i = 0; i < kNmDepth; ++i) {
    if (i < my_total) issue(i);
    else cp_async_commit();  // empty groups keep the wait count uniform
  }
  const int lr = lane & 7, lm = lane >> 3;
  for (int i = 0; i < my_total; ++i) {
    cp_async_wait<kNmDepth - 1>();
    __syncwarp();
    const uint32_t slot = ring + uint32_t(i % kNmDepth) * SLOT;
    if (i < my_sp) {
      // compressed A fragment: matrices (rows 0-7 | 8-15) x (16-byte chunk 0 | 1)
      const int arow = lr + ((lm & 1) << 3), ach = lm >> 1;
      uint32_t af[4];
      ldsm_x4(slot + arow * 32 + ((ach ^ ((arow >> 2) & 1)) << 4), af[0], af[1], af[2], af[3]);
      const uint32_t e = metas[i % kNmDepth];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        // x fragment: token rows 8nt..8nt+7, chunks 0..3 (features 0-7, 8-15, 16-23, 24-31)
        const int xr = 8 * nt + lr;
        uint32_t bf[4];
        ldsm_x4(slot + A_TILE + xr * 64 + ((lm ^ ((xr >> 1) & 3)) << 4), bf[0], bf[1], bf[2], bf[3]);
        mma_sp16832<TI>::run(acc[nt], af, bf, e);
      }
    } else {
      const int arow = lr + ((lm & 1) << 3), ach = lm >> 1;
      uint32_t af[4];
      ldsm_x4(slot + arow * 32 + ((ach ^ ((arow >> 2) & 1)) << 4), af[0], af[1], af[2], af[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int hr = 8 * nt + lr, hch = lm & 1;
        uint32_t b0, b1;
        asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                     : "=r"(b0), "=r"(b1)
                     : "r"(slot + A_TILE + hr * 32 + ((hch ^ ((hr >> 2) & 1)) << 4)));
        mma16816<TI>::run(acc[nt], af, b0, b1);
      }
    }
    __syncwarp();
    if (i + kNmDepth < my_total) issue(i + kNmDepth);
    else cp_async_commit();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int m = g + ((e & 2) ? 8 : 0);
      const int t = 8 * nt + 2 * tq + (e & 1);
      red[(warp * 16 + m) * TT + t] = acc[nt][e];
    }
  __syncthreads();
  TI* __restrict__ y = static_cast<TI*>(a.y);
  const TI* __restrict__ bias = static_cast<const TI*>(a.bias);
  for (int idx = threadIdx.x; idx < 16 * TT; idx += kNmWarps * 32) {
    const int n = idx % 16, t = idx / 16;
    const int64_t tok = t0 + t;
    if (tok >= a.M) continue;
    float v = ((red[(0 * 16 + n) * TT + t] + red[(1 * 16 + n) * TT + t]) + red[(2 * 16 + n) * TT + t]) +
              red[(3 * 16 + n) * TT + t];
    if (bias) v += to_f(bias[f0 + n]);
    y[tok * a.ldy + f0 + n] = from_f<TI>(v);
  }
}

int nm_pick_tt(int64_t M) { return M <= 8 ? 8 : M <= 16 ? 16 : M <= 32 ? 32 : 64; }

// ------------------------------------------------ prefill: dense 64 x 64 blocks --
//
// From 256 tokens the layer runs as a full-density block-sparse layer on the
// 2-SM tensor-core combine: S is unpacked per call into every 64 x 64 block
// in the combine's value layout, block (i, j) at index i * (K/64) + j holding
// S[64i + n][64j + k] at [k][n], and a column schedule of the full structure
// is written beside it.  One CTA per block: each thread expands 4 groups of 4
// (16 K entries) of one row into a shared tile, transposed, then the tile
// leaves as 16-byte stores.
constexpr int kUnpackPad = 72;  // tile row (64 n + 8): 16-byte aligned, fewer bank conflicts

template <typename TI>
__global__ void __launch_bounds__(256) nm_unpack_blocks_kernel(const TI* __restrict__ values,
                                                               const uint32_t* __restrict__ meta, int64_t K,
                                                               int64_t KB, TI* __restrict__ blocks) {
  __shared__ __align__(16) TI tile[64 * kUnpackPad];  // [k][n]
  const int64_t bi = blockIdx.x / KB, bj = blockIdx.x - bi * KB;
  const int n = threadIdx.x >> 2, q = threadIdx.x & 3;  // row n of the block, K entries [16q, 16q + 16)
  const int64_t row = bi * 64 + n, k0 = bj * 64 + q * 16;
  const uint4 v = *reinterpret_cast<const uint4*>(values + row * (K / 2) + k0 / 2);  // 8 kept entries
  const uint32_t word = __ldg(meta + row * (K / 32) + k0 / 32) >> (16 * (q & 1));  // their 4 groups
  const TI* kept = reinterpret_cast<const TI*>(&v);
  const TI zero = from_f<TI>(0.f);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const uint32_t nib = (word >> (4 * g)) & 0xfu;
    const int p0 = int(nib & 3u), p1 = int(nib >> 2);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      tile[(q * 16 + 4 * g + e) * kUnpackPad + n] = e == p0 ? kept[2 * g] : (e == p1 ? kept[2 * g + 1] : zero);
  }
  __syncthreads();
  // the block's 64 x 64 entries, [k][n]: thread t writes k = t / 4, n = 16 (t % 4) .. + 16
  const int k = threadIdx.x >> 2, c = (threadIdx.x & 3) * 16;
  uint4* out = reinterpret_cast<uint4*>(blocks + blockIdx.x * int64_t(64 * 64) + k * 64 + c);
  const uint4* src = reinterpret_cast<const uint4*>(tile + k * kUnpackPad + c);
  out[0] = src[0];
  out[1] = src[1];
}

// Row pointers, column indices and the column schedule (the layout
// slr_plan_stages writes) of NB x KB present blocks, natural row order, groups
// of G = 4 block-rows (block_p 64): group gi has one stage per column s, all
// its rows present; the block indices follow the 2 * groups * KB records.
__global__ void dense_plan_kernel(int64_t NB, int64_t KB, uint32_t* __restrict__ plan, int32_t* __restrict__ stage_start,
                                  int32_t* __restrict__ crow, int32_t* __restrict__ col) {
  constexpr int G = 4;
  const int64_t groups = (NB + G - 1) / G, n_st = groups * KB;
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx < n_st) {
    const int64_t gi = idx / KB, s = idx - gi * KB;
    const int cnt = int(NB - gi * G < G ? NB - gi * G : G);
    // blocks of the groups before: gi * G * KB (only the last group is short)
    const int64_t first = 2 * n_st + gi * G * KB + s * cnt;
    plan[2 * idx] = uint32_t(s) | (((1u << cnt) - 1u) << 16);
    plan[2 * idx + 1] = uint32_t(first);
    for (int j = 0; j < cnt; ++j) plan[first + j] = uint32_t((gi * G + j) * KB + s);
  }
  if (idx <= groups) stage_start[idx] = int32_t(idx * KB);
  if (idx <= NB) crow[idx] = int32_t(idx * KB);
  if (idx < NB * KB) col[idx] = int32_t(idx % KB);
}

template <int NT, typename TI>
int launch_nm_inst(const NmArgs& a, cudaStream_t s) {
  constexpr int TT = 8 * NT;
  const size_t smem = size_t(kNmWarps) * kNmDepth * (16 * 32 + TT * 64) + sizeof(float) * kNmWarps * 16 * TT;
  auto kern = nm_combine_kernel<NT, TI>;
  SLR_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const dim3 grid(unsigned(a.N / 16), unsigned(ceil_div(a.M, TT)));
  kern<<<grid, kNmWarps * 32, smem, s>>>(a);
  SLR_CHECK_LAUNCH("nm_combine_kernel");
  return SLR_OK;
}

template <typename TI>
int launch_nm_t(const NmArgs& a, cudaStream_t s) {
  switch (nm_pick_tt(a.M)) {
    case 8: return launch_nm_inst<1, TI>(a, s);
    case 16: return launch_nm_inst<2, TI>(a, s);
    case 32: return launch_nm_inst<4, TI>(a, s);
    default: return launch_nm_inst<8, TI>(a, s);
  }
}

}  // namespace

int launch_nm_pack(const void* S, int64_t N, int64_t K, int dtype, void* values, uint32_t* meta, int* bad,
                   cudaStream_t s) {
  const int64_t work = N * (K / 32);
  if (work <= 0) return SLR_OK;
  const unsigned blocks = unsigned(ceil_div(work, 256));
  if (dtype == SLR_BF16)
    nm_pack_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(S), N, K,
                                                          static_cast<__nv_bfloat16*>(values), meta, bad);
  else if (dtype == SLR_F16)
    nm_pack_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(S), N, K, static_cast<__half*>(values),
                                                   meta, bad);
  else
    return fail(SLR_ERR_UNSUPPORTED_DTYPE, "N:M layer: 16-bit dtypes only");
  SLR_CHECK_LAUNCH("nm_pack_kernel");
  return SLR_OK;
}

int launch_nm_combine(const void* x, int64_t ldx, void* y, int64_t ldy, const void* values, const uint32_t* meta,
                      const void* A, const void* H, int64_t ldh, const void* bias, int64_t M, int64_t N, int64_t K,
                      int64_t r, int dtype, cudaStream_t s) {
  if (M <= 0) return SLR_OK;
  NmArgs a{x, y, values, meta, A, H, bias, M, N, K, r, ldx, ldy, ldh};
  if (dtype == SLR_BF16) return launch_nm_t<__nv_bfloat16>(a, s);
  if (dtype == SLR_F16) return launch_nm_t<__half>(a, s);
  return fail(SLR_ERR_UNSUPPORTED_DTYPE, "N:M layer: 16-bit dtypes only");
}

int64_t nm_dense_plan_words(int64_t N, int64_t K) {
  const int64_t NB = N / 64, KB = K / 64, groups = (NB + 3) / 4;
  return 2 * groups * KB + NB * KB;
}

int launch_nm_dense_blocks(const void* values, const uint32_t* meta, int64_t N, int64_t K, int dtype, void* blocks,
                           uint32_t* plan, int32_t* stage_start, int32_t* crow, int32_t* col, cudaStream_t s) {
  const int64_t NB = N / 64, KB = K / 64;
  if (NB <= 0 || KB <= 0) return SLR_OK;
  if (N % 64 || K % 64) return fail(SLR_ERR_UNSUPPORTED, "N:M dense blocks: N and K must be multiples of 64");
  if (nm_dense_plan_words(N, K) > INT32_MAX) return fail(SLR_ERR_UNSUPPORTED, "N:M dense blocks: schedule too large");
  const unsigned nblk = unsigned(NB * KB);
  if (dtype == SLR_BF16)
    nm_unpack_blocks_kernel<__nv_bfloat16><<<nblk, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(values), meta, K,
                                                                 KB, static_cast<__nv_bfloat16*>(blocks));
  else if (dtype == SLR_F16)
    nm_unpack_blocks_kernel<__half><<<nblk, 256, 0, s>>>(static_cast<const __half*>(values), meta, K, KB,
                                                          static_cast<__half*>(blocks));
  else
    return fail(SLR_ERR_UNSUPPORTED_DTYPE, "N:M layer: 16-bit dtypes only");
  SLR_CHECK_LAUNCH("nm_unpack_blocks_kernel");
  const int64_t groups = (NB + 3) / 4;
  const int64_t work = std::max(std::max(NB * KB, NB + 1), std::max(groups * KB, groups + 1));
  dense_plan_kernel<<<unsigned(ceil_div(work, 256)), 256, 0, s>>>(NB, KB, plan, stage_start, crow, col);
  SLR_CHECK_LAUNCH("dense_plan_kernel");
  return SLR_OK;
}

}  // namespace slr
