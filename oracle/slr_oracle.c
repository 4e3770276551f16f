/*
 * TEST INFRASTRUCTURE — CPU oracle for the sparse-plus-low-rank (S+LR) linear.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker or as the timed CPU baseline.
 * The product path (s_salaad_b200, libslr_b200.so) never calls it.
 *
 * What it restates (paths are within the S-SALAAD project):
 *
 *   oracle_bsr_addmm_f32
 *     ssalaad/cpu_sparse/bsr_addmm_avx2.cpp:67-140 (run_block) and :144-174.
 *     out[m, by*bp + n] += sum over the nonzero blocks ji of block-row `by`
 *     (crow order) and k in [0, bq) of x[m, col[ji]*bq + k] * values[ji, k, n].
 *     The accumulation order per output element is the reference's: the
 *     accumulator starts at the current `out` value, then one fused
 *     multiply-add per (ji, k) in ascending ji, then ascending k.  Because
 *     each AVX2 lane performs exactly that chain of correctly rounded FMAs,
 *     a scalar fmaf() chain in the same order reproduces the reference bit
 *     for bit (tests/test_oracle.py checks this against the golden vectors).
 *     Only block-rows listed in active_rows are touched (:86-89), so empty
 *     block-rows of `out` keep their contents.
 *     The reference kernel accepts square 8/16/32/64 blocks only (:46-51);
 *     this restatement also accepts rectangular bq x bp blocks, matching the
 *     index arithmetic of the CUDA operator (ssalaad/tilelang_sparse/
 *     addmm_inplace.py:74-80: x column = col_j * block_q).
 *
 *   oracle_block_mask
 *     ssalaad/efficient/artifact.py:26-29.  A block is live iff the sum of
 *     |s| over the block compares greater than zero.  For IEEE values that
 *     is "no NaN in the block and at least one nonzero element": a sum of
 *     non-negative terms is zero only if every term is zero, and any NaN
 *     makes the sum NaN, which compares false.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, fmaf from libm).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_EINVAL 1

int oracle_bsr_addmm_f32(float* out, const float* x, const int32_t* crow,
                         const int32_t* col, const float* values,
                         const int32_t* active_rows, int64_t M, int64_t K,
                         int64_t NB, int64_t nnz, int64_t active_nb,
                         int64_t bp, int64_t bq) {
  if (bp <= 0 || bq <= 0 || M < 0 || K % bq != 0) return ORACLE_EINVAL;
  const int64_t N = NB * bp;
  const int64_t nbk = K / bq;
  for (int64_t ai = 0; ai < active_nb; ++ai) {
    const int64_t by = active_rows[ai];
    if (by < 0 || by >= NB) return ORACLE_EINVAL;
    const int32_t r0 = crow[by], r1 = crow[by + 1];
    if (r0 < 0 || r1 < r0 || r1 > nnz) return ORACLE_EINVAL;
    for (int32_t ji = r0; ji < r1; ++ji)
      if (col[ji] < 0 || col[ji] >= nbk) return ORACLE_EINVAL;
  }
  for (int64_t m = 0; m < M; ++m) {
    const float* xm = x + m * K;
    float* om = out + m * N;
    for (int64_t ai = 0; ai < active_nb; ++ai) {
      const int64_t by = active_rows[ai];
      const int32_t r0 = crow[by], r1 = crow[by + 1];
      for (int64_t n = 0; n < bp; ++n) {
        float acc = om[by * bp + n];
        for (int32_t ji = r0; ji < r1; ++ji) {
          const float* xk = xm + (int64_t)col[ji] * bq;
          const float* w = values + (int64_t)ji * bq * bp + n;
          for (int64_t k = 0; k < bq; ++k) acc = fmaf(xk[k], w[k * bp], acc);
        }
        om[by * bp + n] = acc;
      }
    }
  }
  return ORACLE_OK;
}

/* Block liveness mask of a dense fp32 matrix S[n, m] (row-major) cut into
 * bp x bq blocks; mask is [n/bp, m/bq] bytes, 1 = live. */
int oracle_block_mask_f32(const float* S, int64_t n, int64_t m, int64_t bp,
                          int64_t bq, uint8_t* mask) {
  if (bp <= 0 || bq <= 0 || n % bp || m % bq) return ORACLE_EINVAL;
  const int64_t rb = n / bp, cb = m / bq;
  for (int64_t i = 0; i < rb; ++i)
    for (int64_t j = 0; j < cb; ++j) {
      int any_nonzero = 0, any_nan = 0;
      for (int64_t a = 0; a < bp; ++a)
        for (int64_t b = 0; b < bq; ++b) {
          const float v = S[(i * bp + a) * m + j * bq + b];
          if (v != v) any_nan = 1;
          else if (v != 0.0f) any_nonzero = 1;
        }
      mask[i * cb + j] = (uint8_t)(any_nonzero && !any_nan);
    }
  return ORACLE_OK;
}

/* Same for 16-bit storage (bf16 or fp16 bit patterns): zero is +-0 and NaN
 * is an all-ones exponent with a nonzero mantissa.  exp_bits/man_bits pick
 * the format (bf16: 8/7, fp16: 5/10). */
int oracle_block_mask_u16(const uint16_t* S, int64_t n, int64_t m, int64_t bp,
                          int64_t bq, int exp_bits, int man_bits,
                          uint8_t* mask) {
  if (bp <= 0 || bq <= 0 || n % bp || m % bq) return ORACLE_EINVAL;
  const uint16_t man_mask = (uint16_t)((1u << man_bits) - 1u);
  const uint16_t exp_mask = (uint16_t)(((1u << exp_bits) - 1u) << man_bits);
  const int64_t rb = n / bp, cb = m / bq;
  for (int64_t i = 0; i < rb; ++i)
    for (int64_t j = 0; j < cb; ++j) {
      int any_nonzero = 0, any_nan = 0;
      for (int64_t a = 0; a < bp; ++a)
        for (int64_t b = 0; b < bq; ++b) {
          const uint16_t v = S[(i * bp + a) * m + j * bq + b];
          if ((v & exp_mask) == exp_mask && (v & man_mask)) any_nan = 1;
          else if (v & 0x7fffu) any_nonzero = 1;
        }
      mask[i * cb + j] = (uint8_t)(any_nonzero && !any_nan);
    }
  return ORACLE_OK;
}
