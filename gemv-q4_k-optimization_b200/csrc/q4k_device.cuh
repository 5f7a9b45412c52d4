// q4k_device.cuh -- device-side building blocks for the sm_100a Q4_K GEMV.
//
// Formats (ggml, unchanged):
//   Q4_K super-block (144 B / 256 weights): [0,2) half d, [2,4) half dmin,
//     [4,16) 12 packed scale/min bytes, [16,144) 128 bytes of nibbles.
//     Byte qs[32c+l] holds weight 64c+l (sub-block 2c) in its low nibble and
//     weight 64c+32+l (sub-block 2c+1) in its high nibble.
//   q8_1 block (36 B / 32 activations): half d, half sum, int8 qs[32].
//
// Internal activation pack ("q8a"), one 320-byte record per super-block and
// column, produced once per call by the prep kernel and read by every warp:
//   [0,256)   int8 quants in natural order (q8_1 block s at [32s, 32s+32))
//   [256,320) four float4, one per sub-block pair c = 0..3:
//             { f(2c), f(2c+1), a(2c), a(2c+1) }
//             f(s) = d8(s) for even s, d8(s)/16 for odd s (the high-nibble dot
//             is taken on the unshifted byte, i.e. 16x the nibble dot),
//             a(s) = d8(s) * T(s), T(s) = sum of the 32 quants (exact in fp32),
//             d8(s) = float(half(d)) as the reference reads it
//             (kernels/vecdotq.cuh:811).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "q4k_internal.h"

namespace q4k {

// dp4a chains start from this bias so that the int32 result, read as a
// float, is 1.5*2^23 + S exactly for |S| < 2^22; subtracting kMagicF gives
// float(S) with one full-rate FADD instead of a conversion.
constexpr int kMagicI = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

// ---- addresses, loads ----------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// Read-only, L1-cached 16-byte load (activation records shared by all warps).
__device__ __forceinline__ uint4 ldg_nc128(const void *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}
// L2-coherent load (partials written by other SMs during this launch).
__device__ __forceinline__ float ldcg_f32(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// ---- integer dot products -------------------------------------------------
// c + sum_i a.byte[i] * b.byte[i], a bytes unsigned, b bytes signed.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// 32-bit shared-memory load (4-byte aligned address).
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// float(byte k of w) + 2^23, as bits: 0x4B0000bb.
__device__ __forceinline__ float byte_magic(uint32_t w, int k) {
    return __uint_as_float(prmt(w, 0x4B000000u, 0x7540u | static_cast<uint32_t>(k)));
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic) ---------------------------
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0,%1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// ---- mbarrier + bulk asynchronous copy (TMA, non-tensor, no multicast) ------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// fp32 shared-memory load / store (ordered with the other shared-memory asm).
__device__ __forceinline__ float lds32f(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void sts32f(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
// Shared-memory words for hand-offs between the warps of a CTA.
__device__ __forceinline__ int ld_acquire_cta_s32(uint32_t a) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_s32(uint32_t a) {
    int v;
    asm volatile("ld.volatile.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta_s32(uint32_t a, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void st_volatile_s32(uint32_t a, int v) {
    asm volatile("st.volatile.shared::cta.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Global -> this CTA's shared memory, completion counted on bar (bytes).
// Requires 16-byte aligned addresses and a size that is a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
// 2D tensor-map tile load (no multicast): box at element coordinates (x, y).
// x * element size must be a multiple of 16 bytes.
// L2 policy for data read once (the weight stream): evicted first, so the
// activations, their q8a records and the outputs stay resident.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(tm), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(tm), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// Non-binding L2 prefetch of the line holding p, kept in L2 ahead of streamed data.
__device__ __forceinline__ void prefetch_l2(const void *p) {
    asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}
// L2 evict-last policy (data read again soon: activations among the weight stream).
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Non-binding bulk L2 prefetch of [p, p + bytes) (16-byte aligned, bytes a
// multiple of 16), kept with the evict-last policy.
__device__ __forceinline__ void bulk_prefetch_l2(const void *p, uint32_t bytes, uint64_t policy) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p), "r"(bytes), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- release/acquire counters (split-group completion) ------------------------
// Device-scope fetch-add with acquire-release semantics.
__device__ __forceinline__ int atom_add_acqrel_gpu(int *p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// Device-scope fetch-add without ordering: a ticket.  No memory clobber, so the
// warp runs on until it reads the result.
__device__ __forceinline__ int atom_add_relaxed_gpu(int *p, int v) {
    int old;
    asm volatile("atom.relaxed.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v));
    return old;
}
__device__ __forceinline__ void st_relaxed_gpu(int *p, int v) {
    asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_add_release_gpu_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Acquire-release fence at system scope (orders peer stores over NVLink).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// System-scope release store / acquire load (peer flags over NVLink).
__device__ __forceinline__ void st_release_sys_u32(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- programmatic dependent launch -------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- warp reductions ------------------------------------------------------------
__device__ __forceinline__ float warp_max_f32(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
// Xor-butterfly sum; every lane ends with the same value, formed in the
// order offsets 16, 8, 4, 2, 1 (the order the q8_1 block sum is specified in).
__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
__device__ __forceinline__ int warp_sum_i32(int v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

}  // namespace q4k
