/*
 * q4k_oracle.c -- scalar CPU restatement of the reference's Q4_K x q8_1 GEMV.
 *
 * TEST INFRASTRUCTURE ONLY (see q4k_oracle.h).  This file is the checker the
 * tests compare the CUDA library against, and the timed CPU baseline.  It is
 * never linked into, loaded by or called from the product library.
 *
 * Every function cites the reference file:line it restates.  Paths are
 * relative to the reference project root (vijay-kodamalla/gemv-q4_k-optimization).
 *
 * Build: oracle/Makefile (gcc -O3 -march=native -fopenmp, no -ffast-math: the
 * q8_1 quantizer relies on IEEE float division and roundf).
 */
#include "q4k_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QK_K 256      /* weights per Q4_K super-block */
#define QK8_1 32      /* activations per q8_1 block */
#define Q4K_BYTES 144 /* sizeof(block_q4_K), pinned by kernels/w_tile.cu:6 */
#define Q81_BYTES 36  /* sizeof(block_q8_1), pinned by kernels/w_tile.cu:7 */

/* ------------------------------------------------------------------------ */
/* binary16 conversions (IEEE 754, round to nearest even)                    */
/* ------------------------------------------------------------------------ */

float or_h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t mant = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do {
                mant <<= 1;
                ++e;
            } while ((mant & 0x400u) == 0);
            mant &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (mant << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t or_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t hm = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) ++hm;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)h;
}

/* ------------------------------------------------------------------------ */
/* q8_1 quantization                                                          */
/* ------------------------------------------------------------------------ */

/*
 * Restates the q8_1 quantizer the reference calls at kernels/mmvq.cu:734
 * (upstream quantize_row_q8_1_cuda, not vendored in the reference; its
 * semantics are this project's specification):
 *   per 32-value block: amax = max|x|, d = amax/127 (IEEE float division),
 *   q = amax == 0 ? 0 : roundf(x/d) (round half away from zero),
 *   ds = half2(d, sum) with sum taken in the order of a 32-lane xor-butterfly
 *   (offsets 16, 8, 4, 2, 1), the warp reduction upstream uses.
 * Padding to Kpad (kernels/mmvq.cu:728, MATRIX_ROW_PADDING) is zeros.
 * The Q4_K dot reads only half(d) (kernels/vecdotq.cuh:811).
 */
static void quantize_block(const float v[32], uint8_t *blk) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) {
        float a = fabsf(v[i]);
        amax = a > amax ? a : amax;
    }
    float t[32], n[32];
    memcpy(t, v, sizeof(t));
    for (int off = 16; off >= 1; off >>= 1) {
        for (int i = 0; i < 32; ++i) n[i] = t[i] + t[i ^ off];
        memcpy(t, n, sizeof(t));
    }
    const float sum = t[0];
    const float d = amax / 127.0f;
    uint16_t hd = or_f2h(d), hs = or_f2h(sum);
    memcpy(blk + 0, &hd, 2);
    memcpy(blk + 2, &hs, 2);
    int8_t *qs = (int8_t *)(blk + 4);
    for (int i = 0; i < 32; ++i) {
        qs[i] = amax == 0.0f ? (int8_t)0 : (int8_t)roundf(v[i] / d);
    }
}

void or_quantize_q8_1(const float *x, int64_t K, int64_t stride_col_x,
                      int64_t Kpad, int ncols, uint8_t *out) {
    const int64_t nblk = Kpad / QK8_1;
    for (int j = 0; j < ncols; ++j) {
        const float *xc = x + (int64_t)j * stride_col_x;
        uint8_t *oc = out + (int64_t)j * nblk * Q81_BYTES;
        for (int64_t b = 0; b < nblk; ++b) {
            float v[32];
            for (int i = 0; i < 32; ++i) {
                int64_t idx = b * 32 + i;
                v[i] = idx < K ? xc[idx] : 0.0f;
            }
            quantize_block(v, oc + b * Q81_BYTES);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q6_K (the other k-quant of Q4_K_M checkpoints: output head, some layers)  */
/* ------------------------------------------------------------------------ */

#define Q6K_BYTES 210 /* ql[128], qh[64], int8 scales[16], fp16 d */

/*
 * Signed 6-bit value of weight w (0..255) of a Q6_K super-block: low 4 bits
 * from ql, high 2 bits from qh, minus 32.  With w = 128n + 32j + l (n = 0,1,
 * j = 0..3, l = 0..31): low nibble (j >> 1) of ql[64n + 32(j & 1) + l], bits
 * 2j..2j+1 of qh[32n + l]; its 16-weight sub-block is s = w / 16 with scale
 * scales[s].  This is the indexing of kernels/vecdotq.cuh:867-890 (vl from
 * ql at iqs, vh from qh shifted by vh_shift, scales at scale_offset) spelled
 * out per weight.
 */
static int q6_value(const uint8_t *sb, int w) {
    const int n = w >> 7, j = (w >> 5) & 3, l = w & 31;
    const int lo = (sb[64 * n + 32 * (j & 1) + l] >> (4 * (j >> 1))) & 0xF;
    const int hi = (sb[128 + 32 * n + l] >> (2 * j)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* Dequantized weights of Q6_K rows (for cross-checks): (nrows, K) floats. */
void or_dequant_q6k(const uint8_t *W, int64_t nrows, int64_t K, int64_t stride_row_blocks, float *out) {
    const int64_t nb = K / QK_K;
    for (int64_t r = 0; r < nrows; ++r)
        for (int64_t kb = 0; kb < nb; ++kb) {
            const uint8_t *sb = W + (r * stride_row_blocks + kb) * Q6K_BYTES;
            const float d = or_h2f((uint16_t)(sb[208] | (sb[209] << 8)));
            for (int w = 0; w < QK_K; ++w)
                out[r * K + kb * QK_K + w] = d * (float)(int8_t)sb[192 + w / 16] * (float)q6_value(sb, w);
        }
}

/*
 * y[col][row] = sum over super-blocks of d * sum_k d8_k * (sc[2k] * S[2k] +
 * sc[2k+1] * S[2k+1]), S[s] = sum over sub-block s (16 weights) of (q6 - 32)
 * * q8 -- vec_dot_q6_K_q8_1_impl_mmvq (kernels/vecdotq.cuh:576-601): integer
 * dot per 4 weights, times the int8 scale, times d8 of the q8_1 block, the
 * total times d.  Exact sums in fp64.
 */
void or_gemv_q6k_q8_1(const uint8_t *W, int64_t nrows, int64_t K, int64_t stride_row_blocks,
                      const uint8_t *y_q8_1, int64_t stride_col_y_blocks, int ncols, float *dst,
                      int64_t stride_col_dst, int nthreads) {
    const int64_t nb = K / QK_K;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t r = 0; r < nrows; ++r) {
        for (int j = 0; j < ncols; ++j) {
            const uint8_t *yc = y_q8_1 + (int64_t)j * stride_col_y_blocks * Q81_BYTES;
            double acc = 0.0;
            for (int64_t kb = 0; kb < nb; ++kb) {
                const uint8_t *sb = W + (r * stride_row_blocks + kb) * Q6K_BYTES;
                const double d = or_h2f((uint16_t)(sb[208] | (sb[209] << 8)));
                double sbsum = 0.0;
                for (int k = 0; k < 8; ++k) {
                    const uint8_t *blk = yc + (kb * 8 + k) * Q81_BYTES;
                    const double d8 = or_h2f((uint16_t)(blk[0] | (blk[1] << 8)));
                    long isum = 0;
                    for (int h = 0; h < 2; ++h) {
                        long S = 0;
                        for (int i = 0; i < 16; ++i) {
                            const int w = 32 * k + 16 * h + i;
                            S += (long)q6_value(sb, w) * (int8_t)blk[4 + 16 * h + i];
                        }
                        isum += (long)(int8_t)sb[192 + 2 * k + h] * S;
                    }
                    sbsum += d8 * (double)isum;
                }
                acc += d * sbsum;
            }
            dst[(int64_t)j * stride_col_dst + r] = (float)acc;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* RMSNorm ahead of the quantizer                                            */
/* ------------------------------------------------------------------------ */

/*
 * y = x / sqrt(mean(x^2) + eps) (* w), the step before quantize_q8_1 in the
 * reference's decode trace (rms_norm_f32 -> quantize_q8_1 -> mul_mat_vec_q;
 * upstream ggml, not vendored: restated from the published definition).
 * The sum of squares is formed in the library's fixed order so the scale is
 * bit-identical: 256 partial sums s_t = fma(x_i, x_i, s_t) over
 * i = t, t+256, ... (ascending), an xor-butterfly sum (offsets 16..1) inside
 * each group of 32, then the same butterfly over the 8 group sums (lanes 8..31
 * adding zeros).  scale = 1 / sqrtf(sum / K + eps) (IEEE division and square
 * root), y_i = (x_i * scale) * w_i.
 */
static void butterfly32(float *v) {
    for (int off = 16; off > 0; off >>= 1) {
        float n[32];
        for (int l = 0; l < 32; ++l) n[l] = v[l] + v[l ^ off];
        memcpy(v, n, sizeof(n));
    }
}

float or_rmsnorm_scale(const float *x, int64_t K, float eps) {
    float part[256];
    for (int t = 0; t < 256; ++t) {
        float s = 0.0f;
        for (int64_t i = t; i < K; i += 256) s = fmaf(x[i], x[i], s);
        part[t] = s;
    }
    float lanes[32];
    float warp_tot[8];
    for (int w = 0; w < 8; ++w) {
        memcpy(lanes, part + 32 * w, sizeof(lanes));
        butterfly32(lanes);
        warp_tot[w] = lanes[0];
    }
    for (int l = 0; l < 32; ++l) lanes[l] = l < 8 ? warp_tot[l] : 0.0f;
    butterfly32(lanes);
    const float mean = lanes[0] / (float)K;
    return 1.0f / sqrtf(mean + eps);
}

void or_rmsnorm(const float *x, int64_t K, int64_t stride_col_x, int ncols, const float *w, float eps,
                float *y) {
    for (int j = 0; j < ncols; ++j) {
        const float *xc = x + (int64_t)j * stride_col_x;
        float *yc = y + (int64_t)j * K;
        const float scale = or_rmsnorm_scale(xc, K, eps);
        for (int64_t i = 0; i < K; ++i) {
            const float v = xc[i] * scale;
            yc[i] = w ? v * w[i] : v;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Q4_K super-block decode and integer sub-block sums                        */
/* ------------------------------------------------------------------------ */

/*
 * 6-bit scale and min of sub-block s.  Byte-wise form of the uint16-pair
 * unpacking at kernels/vecdotq.cuh:796-807:
 *   s < 4 : sc = b[s] & 63,                      m = b[s+4] & 63
 *   s >= 4: sc = (b[s+4] & 15) | ((b[s-4] >> 6) << 4),
 *           m  = (b[s+4] >> 4) | ((b[s]   >> 6) << 4)
 */
void or_scale_min(const uint8_t *b, int s, int *sc, int *m) {
    if (s < 4) {
        *sc = b[s] & 63;
        *m = b[s + 4] & 63;
    } else {
        *sc = (b[s + 4] & 0x0f) | ((b[s - 4] >> 6) << 4);
        *m = (b[s + 4] >> 4) | ((b[s] >> 6) << 4);
    }
}

/*
 * S[s] = sum over the 32 weights of sub-block s of nibble * q8, and
 * T[s] = sum of the 32 q8 values of the matching q8_1 block.
 * Weight byte qs[32c + l] holds sub-block 2c in its low nibble and sub-block
 * 2c+1 in its high nibble, each paired with byte l of q8_1 block 2c (resp.
 * 2c+1): kernels/vecdotq.cuh:784-794 (q4 offsets), :809-816 (q8 offsets),
 * :470-474 (nibble shift 4*i, dp4a pairing, dp4a with 0x01010101 for T).
 */
void or_subblock_sums_sb(const uint8_t *sb, const uint8_t *q8, int32_t S[8],
                         int32_t T[8]) {
    const uint8_t *qs = sb + 16;
    for (int s = 0; s < 8; ++s) {
        const int c = s >> 1, h = s & 1;
        const int8_t *u = (const int8_t *)(q8 + s * Q81_BYTES + 4);
        int32_t acc = 0, sum = 0;
        for (int l = 0; l < 32; ++l) {
            const int nib = (qs[32 * c + l] >> (4 * h)) & 0x0f;
            acc += nib * (int32_t)u[l];
            sum += (int32_t)u[l];
        }
        S[s] = acc;
        T[s] = sum;
    }
}

static inline float h2f_at(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return or_h2f(h);
}

/*
 * One super-block times one q8_1 column, in double:
 *   d * sum_s d8_s*sc_s*S_s - dmin * sum_s d8_s*m_s*T_s
 * (combine formula of kernels/vecdotq.cuh:461-483 with d/dmin = half2 dm at
 * :818 and d8 = low half of the q8_1 ds at :811).
 */
static double sb_dot(const uint8_t *sb, const uint8_t *q8) {
    int32_t S[8], T[8];
    or_subblock_sums_sb(sb, q8, S, T);
    const double d = h2f_at(sb + 0), dmin = h2f_at(sb + 2);
    double sd = 0.0, sm = 0.0;
    for (int s = 0; s < 8; ++s) {
        int sc, m;
        or_scale_min(sb + 4, s, &sc, &m);
        const double d8 = h2f_at(q8 + s * Q81_BYTES);
        sd += d8 * (double)sc * (double)S[s];
        sm += d8 * (double)m * (double)T[s];
    }
    return d * sd - dmin * sm;
}

int or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/*
 * Row/column loop with the strides of kernels/mmvq.cu:233-247 (W row r at
 * block r*stride_row_x, y column j at block j*stride_col_y, super-block kbx
 * paired with q8_1 blocks kby = 8*kbx) and the output indexing of
 * kernels/mmvq.cu:285, :337 (dst[j*stride_col_dst + row]).
 */
void or_gemv_q4k_q8_1(const uint8_t *W, int64_t nrows, int64_t K,
                      int64_t stride_row_blocks, const uint8_t *y_q8_1,
                      int64_t stride_col_y_blocks, int ncols, float *dst,
                      int64_t stride_col_dst, int nthreads) {
    const int64_t nb = K / QK_K;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t r = 0; r < nrows; ++r) {
        const uint8_t *wr = W + r * stride_row_blocks * Q4K_BYTES;
        for (int j = 0; j < ncols; ++j) {
            const uint8_t *yc = y_q8_1 + (int64_t)j * stride_col_y_blocks * Q81_BYTES;
            double acc = 0.0;
            for (int64_t kb = 0; kb < nb; ++kb) {
                acc += sb_dot(wr + kb * Q4K_BYTES, yc + kb * 8 * Q81_BYTES);
            }
            dst[(int64_t)j * stride_col_dst + r] = (float)acc;
        }
    }
    (void)nthreads;
}

void or_gemv_q4k_f32(const uint8_t *W, int64_t nrows, int64_t K,
                     int64_t stride_row_blocks, const float *x,
                     int64_t stride_col_x, int ncols, float *dst,
                     int64_t stride_col_dst, int nthreads) {
    const int64_t Kpad = (K + 511) / 512 * 512;
    const int64_t nblk = Kpad / QK8_1;
    uint8_t *q = (uint8_t *)malloc((size_t)ncols * (size_t)nblk * Q81_BYTES);
    if (!q) return;
    or_quantize_q8_1(x, K, stride_col_x, Kpad, ncols, q);
    or_gemv_q4k_q8_1(W, nrows, K, stride_row_blocks, q, nblk, ncols, dst,
                     stride_col_dst, nthreads);
    free(q);
}

void or_subblock_sums(const uint8_t *W, int64_t nrows, int64_t K,
                      int64_t stride_row_blocks, const uint8_t *y_q8_1,
                      int64_t stride_col_y_blocks, int ncols,
                      int32_t *S_out, int32_t *T_out) {
    const int64_t nb = K / QK_K;
    const int64_t nsub = K / QK8_1;
    for (int j = 0; j < ncols; ++j) {
        const uint8_t *yc = y_q8_1 + (int64_t)j * stride_col_y_blocks * Q81_BYTES;
        for (int64_t r = 0; r < nrows; ++r) {
            const uint8_t *wr = W + r * stride_row_blocks * Q4K_BYTES;
            for (int64_t kb = 0; kb < nb; ++kb) {
                int32_t S[8], T[8];
                or_subblock_sums_sb(wr + kb * Q4K_BYTES, yc + kb * 8 * Q81_BYTES, S, T);
                for (int s = 0; s < 8; ++s) {
                    const int64_t o = ((int64_t)j * nrows + r) * nsub + kb * 8 + s;
                    S_out[o] = S[s];
                    T_out[o] = T[s];
                }
            }
        }
    }
}
