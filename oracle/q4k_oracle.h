/*
 * q4k_oracle.h -- CPU restatement of the Q4_K x q8_1 GEMV path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load this library,
 * and only as the checker or as the timed CPU baseline.  The product path
 * (the CUDA library) never calls it.
 *
 * Pinning: the integer and scale semantics are checked against the
 * reference's own vec_dot_q4_K_q8_1 (kernels/vecdotq.cuh:775-819), compiled
 * on the host by oracle/Makefile into oracle/_ref/, and against the
 * committed golden fixtures under tests/golden/ that the same build
 * produced.  The Q4_K byte layout is cross-checked against the independent
 * gguf-py dequantizer at test time.
 */
#ifndef Q4K_ORACLE_H
#define Q4K_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 <-> binary32 (round-to-nearest-even), as CUDA's
 * __float2half / __half2float behave. */
float    or_h2f(uint16_t h);
uint16_t or_f2h(float f);

/* q8_1 quantization of ncols columns of length K into ggml block_q8_1
 * (36 bytes per 32 values: half d, half sum, int8 qs[32]).  Positions
 * K <= i < Kpad are zero padding.  Kpad is a multiple of 32 and >= K.
 * Column j of x starts at x + j*stride_col_x; column j of the output starts
 * at out + j*(Kpad/32)*36. */
void or_quantize_q8_1(const float *x, int64_t K, int64_t stride_col_x,
                      int64_t Kpad, int ncols, uint8_t *out);

/* Per-sub-block integer sums for one super-block and one q8_1 column:
 * S[s] = sum_{32} nibble*q8 and T[s] = sum_{32} q8 for s = 0..7. */
void or_subblock_sums_sb(const uint8_t *sb144, const uint8_t *q8_8blocks,
                         int32_t S[8], int32_t T[8]);

/* 6-bit scale/min of sub-block s (0..7) from the 12 packed bytes. */
void or_scale_min(const uint8_t *scales12, int s, int *sc, int *m);

/* GEMV over pre-quantized q8_1 activations:
 * dst[j*stride_col_dst + r] = sum_k W[r,k] * y_j[k], computed from the exact
 * integer sub-block sums with every product and sum taken in double and
 * rounded to float once at the end.
 * W row r starts at W + r*stride_row_blocks*144.
 * Column j of y starts at block j*stride_col_y_blocks (36-byte blocks). */
void or_gemv_q4k_q8_1(const uint8_t *W, int64_t nrows, int64_t K,
                      int64_t stride_row_blocks, const uint8_t *y_q8_1,
                      int64_t stride_col_y_blocks, int ncols, float *dst,
                      int64_t stride_col_dst, int nthreads);

/* fp32 activations in, quantize (Kpad = K rounded up to 512) then GEMV. */
void or_gemv_q4k_f32(const uint8_t *W, int64_t nrows, int64_t K,
                     int64_t stride_row_blocks, const float *x,
                     int64_t stride_col_x, int ncols, float *dst,
                     int64_t stride_col_dst, int nthreads);

/* Dump S and T for every (row, sub-block, column):
 * S_out[((j*nrows + r)*(K/32)) + b], same for T_out. */
void or_subblock_sums(const uint8_t *W, int64_t nrows, int64_t K,
                      int64_t stride_row_blocks, const uint8_t *y_q8_1,
                      int64_t stride_col_y_blocks, int ncols,
                      int32_t *S_out, int32_t *T_out);

/* Number of OpenMP threads the oracle would use with nthreads <= 0. */
int or_max_threads(void);

/* Q6_K: dequantized rows and the exact GEMV against q8_1 columns
 * (kernels/vecdotq.cuh:576-601, :867-890). */
void or_dequant_q6k(const uint8_t *W, int64_t nrows, int64_t K, int64_t stride_row_blocks, float *out);
void or_gemv_q6k_q8_1(const uint8_t *W, int64_t nrows, int64_t K, int64_t stride_row_blocks,
                      const uint8_t *y_q8_1, int64_t stride_col_y_blocks, int ncols, float *dst,
                      int64_t stride_col_dst, int nthreads);

/* RMSNorm in the library's reduction order: y (ncols x K, dense) from x. */
float or_rmsnorm_scale(const float *x, int64_t K, float eps);
void or_rmsnorm(const float *x, int64_t K, int64_t stride_col_x, int ncols, const float *w, float eps,
                float *y);

#ifdef __cplusplus
}
#endif
#endif
