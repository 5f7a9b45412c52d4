// Host-side stand-in for upstream ggml's common.cuh / ggml-common.h, which the
// reference's kernels/vecdotq.cuh includes (vecdotq.cuh:3) but does not ship.
// Written for this project so that the reference's own dot-product code can
// be compiled with g++ and run on the CPU as the pin for oracle/q4k_oracle.c.
//
// Only block_q4_K, block_q6_K and block_q8_1 are exercised; their layouts are
// the format contract (144, 210 and 36 bytes, asserted below; the reference
// asserts the first and last at kernels/w_tile.cu:6-7).  Every other block type, table and constant exists
// only so that the header's other (never called) functions compile; their
// member lists follow the member names the header uses and their values are
// placeholders.
#pragma once
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <vector_types.h>
#include <vector_functions.h>

// ---- constants the Q4_K path uses -----------------------------------------
#define QK_K 256
#define QK8_1 32
#define QR8_1 1
#define QI8_1 (QK8_1 / (4 * QR8_1))  // 8 ints per q8_1 block
#define QR4_K 2
#define QI4_K (QK_K / (4 * QR4_K))   // 32 ints of nibbles per super-block

// ---- constants only the unused functions reference ------------------------
#define QI4_0 4
#define QR4_1 2
#define QI4_1 4
#define QI5_0 4
#define QI5_1 4
#define QI8_0 8
#define QR2_K 4
#define QR3_K 4
#define QI3_K 16
#define QR5_K 2
#define QR6_K 2
#define QI6_K 32
#define IQ1S_DELTA 0.125f
#define IQ1M_DELTA 0.125f

// ---- the two layouts this project depends on ------------------------------
struct block_q4_K {
    half2 dm;             // d (super-block scale), dmin (super-block min scale)
    uint8_t scales[12];   // 8 six-bit scales + 8 six-bit mins, packed
    uint8_t qs[QK_K / 2]; // 256 nibbles
};
struct block_q8_1 {
    half2 ds;             // d (block scale), s (sum of the unquantized block)
    int8_t qs[QK8_1];
};
static_assert(sizeof(block_q4_K) == 144, "block_q4_K size mismatch");
static_assert(sizeof(block_q8_1) == 36, "block_q8_1 size mismatch");

// ---- compile-only stand-ins -------------------------------------------------
struct block_q4_0 { half d; uint8_t qs[16]; };
struct block_q4_1 { half2 dm; uint8_t qs[16]; };
struct block_q5_0 { half d; uint8_t qh[4]; uint8_t qs[16]; };
struct block_q5_1 { half2 dm; uint8_t qh[4]; uint8_t qs[16]; };
struct block_q8_0 { half d; int8_t qs[32]; };
struct block_mxfp4 { uint8_t e; uint8_t qs[16]; };
struct block_q2_K { uint8_t scales[16]; uint8_t qs[64]; half2 dm; };
struct block_q3_K { uint8_t hmask[32]; uint8_t qs[64]; uint8_t scales[12]; half d; };
struct block_q5_K { half2 dm; uint8_t scales[12]; uint8_t qh[32]; uint8_t qs[128]; };
// Q6_K: ql[128] low nibbles, qh[64] high 2 bits, 16 int8 scales, fp16 d.
struct block_q6_K { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; half d; };
static_assert(sizeof(block_q6_K) == 210, "block_q6_K size mismatch");
struct block_iq2_xxs { half d; uint16_t qs[32]; };
struct block_iq2_xs { half d; uint16_t qs[32]; uint8_t scales[8]; };
struct block_iq2_s { half d; uint8_t qs[64]; uint8_t qh[8]; uint8_t scales[8]; };
struct block_iq3_xxs { half d; uint8_t qs[96]; };
struct block_iq3_s { half d; uint8_t qs[64]; uint8_t qh[8]; uint8_t signs[32]; uint8_t scales[4]; };
struct block_iq1_s { half d; uint8_t qs[32]; uint16_t qh[8]; };
struct block_iq1_m { uint8_t qs[32]; uint8_t qh[16]; uint8_t scales[8]; };
struct block_iq4_nl { half d; uint8_t qs[16]; };
struct block_iq4_xs { half d; uint16_t scales_h; uint8_t scales_l[4]; uint8_t qs[128]; };
union iq1m_scale_t { half f16; uint16_t u16; };

extern const uint64_t iq2xxs_grid[256];
extern const uint64_t iq2xs_grid[512];
extern const uint64_t iq2s_grid[1024];
extern const uint32_t iq3xxs_grid[256];
extern const uint32_t iq3s_grid[512];
extern const uint32_t iq1s_grid_gpu[2048];
extern const uint8_t ksigns_iq2xs[128];
extern const uint64_t ksigns64[128];
extern const int8_t kvalues_iq4nl[16];
extern const int8_t kvalues_mxfp4[16];
float ggml_cuda_e8m0_to_fp32(uint8_t x);

// ---- host versions of the integer SIMD helpers ------------------------------
// dp4a: c + sum of the four signed-byte products of a and b (sm_61 DP4A).
static inline int ggml_cuda_dp4a(const int a, const int b, int c) {
    const int8_t *a8 = (const int8_t *)&a;
    const int8_t *b8 = (const int8_t *)&b;
    return c + a8[0] * b8[0] + a8[1] * b8[1] + a8[2] * b8[2] + a8[3] * b8[3];
}
static inline unsigned int __byte_perm(unsigned int x, unsigned int y, unsigned int s) {
    uint8_t b[8];
    std::memcpy(b, &x, 4);
    std::memcpy(b + 4, &y, 4);
    unsigned int r = 0;
    for (int i = 0; i < 4; ++i) r |= (unsigned int)b[(s >> (4 * i)) & 7] << (8 * i);
    return r;
}
static inline int __vsub4(int a, int b) {
    int r = 0;
    for (int i = 0; i < 4; ++i) {
        uint8_t x = (uint8_t)(a >> (8 * i)), y = (uint8_t)(b >> (8 * i));
        r |= (int)(uint8_t)(x - y) << (8 * i);
    }
    return r;
}
static inline int __vsubss4(int a, int b) {
    int r = 0;
    for (int i = 0; i < 4; ++i) {
        int x = (int8_t)(a >> (8 * i)), y = (int8_t)(b >> (8 * i));
        int d = x - y;
        d = d > 127 ? 127 : (d < -128 ? -128 : d);
        r |= (int)(uint8_t)d << (8 * i);
    }
    return r;
}
static inline unsigned int __vcmpne4(unsigned int a, unsigned int b) {
    unsigned int r = 0;
    for (int i = 0; i < 4; ++i)
        if (((a >> (8 * i)) & 0xff) != ((b >> (8 * i)) & 0xff)) r |= 0xffu << (8 * i);
    return r;
}
