// ref_harness.cpp -- runs the REFERENCE's own Q4_K x q8_1 and Q6_K x q8_1 dot
// products on the CPU.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile together with the
// reference's unmodified kernels/vecdotq.cuh (included from where it lies in
// the reference checkout) and the host shim oracle/ref_shim/common.cuh, into
// oracle/_ref/libq4k_ref.so.  Used to pin oracle/q4k_oracle.c, to produce the
// golden fixtures under tests/golden/, and as the timed reference CPU arm of
// bench.py.  Never linked into the product library.
#include "vecdotq.cuh"  // reference: kernels/vecdotq.cuh

#include <cstdint>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// kernels/vecdotq.cuh:775-819, called exactly as the MMVQ kernel calls it.
float ref_vec_dot_q4_K_q8_1(const void *vbq, const void *bq8_1, int kbx, int iqs) {
    return vec_dot_q4_K_q8_1(vbq, (const block_q8_1 *)bq8_1, kbx, iqs);
}

// kernels/vecdotq.cuh:867-890, called exactly as the MMVQ kernel calls it.
float ref_vec_dot_q6_K_q8_1(const void *vbq, const void *bq8_1, int kbx, int iqs) {
    return vec_dot_q6_K_q8_1(vbq, (const block_q8_1 *)bq8_1, kbx, iqs);
}

// One output value the way upstream mul_mat_vec_q<type, ncols_dst, false>
// forms it (kernels/mmvq.cu:150-338): nwarps*32 threads; with qi the ints of
// quants per super-block and vdr the ints one call consumes, thread tid
// visits super-blocks kbx = tid/(qi/vdr), + blocks_per_iter, ... (mmvq.cu:236)
// with blocks_per_iter = vdr*nwarps*32/qi (mmvq.cu:172) and
// kqs = vdr*(tid%(qi/vdr)) (mmvq.cu:240), accumulates tmp += vec_dot in
// float (mmvq.cu:246), warps 1..nwarps-1 are added into warp 0 in order
// (mmvq.cu:293-294), then a 32-lane xor-butterfly (mmvq.cu:301).
// nwarps = 4 for ncols_dst <= 4 and 2 for 5..8 (mmvq.cu:95-110).
// Q4_K: qi = QI4_K = 32, vdr = VDR_Q4_K_Q8_1_MMVQ = 2; Q6_K: qi = QI6_K = 32,
// vdr = VDR_Q6_K_Q8_1_MMVQ = 1 (vecdotq.cuh:576); both 8 q8_1 blocks per
// super-block (kby = 8*kbx, mmvq.cu:237).
typedef float (*VecDot)(const void *, const block_q8_1 *, const int &, const int &);

static float mmvq_value(VecDot dot, int vdr, const void *row, const block_q8_1 *ycol, int nb, int nwarps) {
    const int qi = 32;
    const int nthreads = nwarps * 32;
    const int tpb = qi / vdr;                         // threads per super-block
    const int blocks_per_iter = vdr * nwarps * 32 / qi;
    float tmp[8 * 32];
    for (int tid = 0; tid < nthreads; ++tid) {
        float t = 0.0f;
        const int kqs = vdr * (tid % tpb);
        for (int kbx = tid / tpb; kbx < nb; kbx += blocks_per_iter) {
            t += dot(row, &ycol[kbx * 8], kbx, kqs);
        }
        tmp[tid] = t;
    }
    float lane[32];
    for (int l = 0; l < 32; ++l) {
        float v = tmp[l];
        for (int w = 1; w < nwarps; ++w) v += tmp[w * 32 + l];
        lane[l] = v;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float n[32];
        for (int l = 0; l < 32; ++l) n[l] = lane[l] + lane[l ^ off];
        for (int l = 0; l < 32; ++l) lane[l] = n[l];
    }
    return lane[0];
}

static void mmvq_gemv(VecDot dot, int vdr, size_t sb_bytes, const void *W, int64_t nrows, int64_t K,
                      int64_t stride_row_blocks, const void *y_q8_1, int64_t stride_col_y_blocks, int ncols,
                      float *dst, int64_t stride_col_dst, int nthreads) {
    const int nb = (int)(K / QK_K);
    const int nwarps = ncols <= 4 ? 4 : 2;
    const uint8_t *w = (const uint8_t *)W;
    const block_q8_1 *y = (const block_q8_1 *)y_q8_1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t r = 0; r < nrows; ++r) {
        for (int j = 0; j < ncols; ++j) {
            dst[(int64_t)j * stride_col_dst + r] = mmvq_value(dot, vdr, w + r * stride_row_blocks * sb_bytes,
                                                              y + (int64_t)j * stride_col_y_blocks, nb, nwarps);
        }
    }
    (void)nthreads;
}

// GEMV over ggml q8_1 activations with the strides of kernels/mmvq.cu:233-247,
// :285, :337.  ncols in 1..8.
void ref_gemv_q4k_q8_1(const void *W, int64_t nrows, int64_t K, int64_t stride_row_blocks,
                       const void *y_q8_1, int64_t stride_col_y_blocks, int ncols,
                       float *dst, int64_t stride_col_dst, int nthreads) {
    mmvq_gemv(vec_dot_q4_K_q8_1, VDR_Q4_K_Q8_1_MMVQ, sizeof(block_q4_K), W, nrows, K, stride_row_blocks, y_q8_1,
              stride_col_y_blocks, ncols, dst, stride_col_dst, nthreads);
}

// The same for Q6_K rows (mul_mat_vec_q<GGML_TYPE_Q6_K, ...>).
void ref_gemv_q6k_q8_1(const void *W, int64_t nrows, int64_t K, int64_t stride_row_blocks,
                       const void *y_q8_1, int64_t stride_col_y_blocks, int ncols,
                       float *dst, int64_t stride_col_dst, int nthreads) {
    mmvq_gemv(vec_dot_q6_K_q8_1, VDR_Q6_K_Q8_1_MMVQ, sizeof(block_q6_K), W, nrows, K, stride_row_blocks, y_q8_1,
              stride_col_y_blocks, ncols, dst, stride_col_dst, nthreads);
}

int ref_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

}  // extern "C"
