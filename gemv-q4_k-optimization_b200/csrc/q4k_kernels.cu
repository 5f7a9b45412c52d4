// q4k_kernels.cu -- sm_100a kernels of the Q4_K x q8_1 decode GEMV.
//
//   k_prep  : fp32 -> q8_1 quantization (and/or ggml q8_1 -> q8a repack) of
//             every activation column of the call, one warp per 32-value
//             block; also clears the GEMV's split counters.  It triggers the
//             dependent GEMV launch immediately, so the GEMV's weight stream
//             starts while the activations are being quantized.
//   k_gemv  : persistent GEMV over a list of matrices ("tasks").  Each warp
//             owns an equal share of the flattened weight stream and pulls it
//             into shared memory with bulk asynchronous copies (one per row
//             segment, issued by the 32 lanes at once), then lane r computes
//             row r of its 32-row group.  Row groups split between warps are
//             completed by whichever contributor finishes last (atomic
//             counter, fixed summation order, no waiting).
//
// Semantics restated from the reference (paths relative to the reference
// project):
//   q8_1 quantization: the call at kernels/mmvq.cu:734 (upstream
//     quantize_q8_1, not vendored: d = amax/127, q = roundf(x/d)).
//   super-block dot: kernels/vecdotq.cuh:775-819 (nibble/q8 pairing, 6-bit
//     scale/min unpacking) and :461-483 (d*sum d8*sc*S - dmin*sum d8*m*T).
//   row/column strides and output layout: kernels/mmvq.cu:233-247, :285, :337.
#include "q4k_device.cuh"
#include "q4k_gemv.h"  // Q4K_TIMELINE_* record geometry
#include "q4k_internal.h"

#include <mutex>

namespace q4k {

// ============================================================================
// q8_1 quantization of one 32-value block (one warp, lane = value)
// ============================================================================
// d = amax/127 (IEEE division), q = amax == 0 ? 0 : roundf(x/d): the semantics
// of the quantizer the reference calls at kernels/mmvq.cu:734.
__device__ __forceinline__ void quantize_value(float x, int &q, __half &dh) {
    const float amax = warp_max_f32(fabsf(x));
    const float d = amax / 127.0f;  // IEEE division (no fast-math in this build)
    q = amax == 0.0f ? 0 : static_cast<int>(roundf(x / d));
    dh = __float2half_rn(d);
}

// Write block b's quants and metadata into its q8a record (column base act_col).
__device__ __forceinline__ void write_q8a(uint8_t *act_col, int b, int lane, int q, __half dh, int32_t *dump_T) {
    const int T = warp_sum_i32(q);
    uint8_t *rec = act_col + static_cast<int64_t>(b >> 3) * kActSBBytes;
    const int s = b & 7;
    rec[s * 32 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
    if (lane == 0) {
        const float d8 = __half2float(dh);
        float *meta = reinterpret_cast<float *>(rec + kActMetaOff + 16 * (s >> 1));
        meta[s & 1] = (s & 1) ? d8 * 0.0625f : d8;
        meta[2 + (s & 1)] = d8 * static_cast<float>(T);
        if (dump_T != nullptr) *dump_T = T;
    }
}

// ============================================================================
// prep: quantize / repack activations, clear counters
// ============================================================================
// RMSNorm of one column, then its q8a / q8_1 blocks (a whole CTA of 256
// threads).  y = x / sqrt(mean(x^2) + eps) (* w): the step the reference's
// decode trace runs before quantize_q8_1 (rms_norm_f32, upstream ggml).  The
// sum of squares has a fixed order (per-thread fma over i = tid, tid+256, ...;
// xor butterflies inside and across the 8 warps) and the scale is
// 1 / sqrtf(mean + eps) with IEEE division and square root, so the CPU
// checker reproduces it bit for bit (upstream uses rsqrtf).
__device__ __forceinline__ void prep_norm_column(const PrepJob &J, int col) {
    __shared__ float red[8];
    __shared__ float scale_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *xc = static_cast<const float *>(J.src) + col * J.src_col_stride;
    float s = 0.0f;
    for (int i = tid; i < J.K; i += 256) s = fmaf(xc[i], xc[i], s);
    s = warp_sum_f32(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float t = lane < 8 ? red[lane] : 0.0f;
        t = warp_sum_f32(t);
        if (lane == 0) scale_s = 1.0f / sqrtf(t / static_cast<float>(J.K) + J.norm_eps);
    }
    __syncthreads();
    const float scale = scale_s;
    for (int b = warp; b < J.nblk; b += 8) {
        const int pos = b * 32 + lane;
        float y = 0.0f;
        if (pos < J.K) {
            y = xc[pos] * scale;
            if (J.norm_w != nullptr) y = y * J.norm_w[pos];
        }
        int q;
        __half dh;
        quantize_value(y, q, dh);
        if (J.q81_out != nullptr) {
            const float sum = warp_sum_f32(y);
            uint8_t *blk = J.q81_out + (col * J.q81_col_stride + b) * kQ81Bytes;
            blk[4 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
            if (lane == 0) *reinterpret_cast<__half2 *>(blk) = __halves2half2(dh, __float2half_rn(sum));
        }
        if (J.act != nullptr && b * 32 < J.K) write_q8a(J.act + col * J.act_col_stride, b, lane, q, dh, nullptr);
    }
}

// Consumer side of the fused all-gather: one thread waits (bounded) until
// every peer's flag word in this rank's flags has reached this rank's epoch,
// i.e. every peer's rows of the last gathering launch on this stream are in
// this rank's buffer; acquire loads at system scope.  Returns false (and sets
// the status word) when the wait gives up.
__device__ __forceinline__ bool gather_wait_flags(const GatherWait &G) {
    const uint32_t e = *reinterpret_cast<const volatile uint32_t *>(G.epoch);
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < G.world; ++q) {
        if (q == G.rank) continue;
        for (uint32_t it = 0;; ++it) {
            if (static_cast<int32_t>(ld_acquire_sys_u32(G.flags + q) - e) >= 0) break;
            if ((it & 63u) == 0 && globaltimer_ns() - t0 > kPeerWaitLimitNs) {
                if (G.status != nullptr) atomicExch(G.status, kStatusTimeout);
                return false;
            }
        }
    }
    return true;
}

// q4k_gather_wait: one CTA, one waiting thread.
__global__ void __launch_bounds__(32) k_gather_wait(const __grid_constant__ GatherWait G) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) gather_wait_flags(G);
}

__global__ void __launch_bounds__(256) k_prep(const __grid_constant__ PrepParams P) {
#if Q4K_TIMELINE
    const uint64_t tl_start = globaltimer_ns();
#endif
    // Let the dependent GEMV grid launch now: it only issues weight copies
    // before its griddepcontrol.wait, which returns after this grid completes.
    pdl_launch_dependents();
    const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
    // While the previous grid runs, ask L2 for this CTA's activation lines.  A
    // prefetch binds no value: if the previous grid writes x, the reads after
    // the wait still see its stores (L2 is the point of coherence).
    if (static_cast<int>(blockIdx.x) < P.norm_ctas) {
        int j = 0;
        while (!(P.job[j].norm && static_cast<int>(blockIdx.x) < P.job[j].cta_base + P.job[j].ncols)) ++j;
        const PrepJob &J = P.job[j];
        const float *xc = static_cast<const float *>(J.src) +
                          (static_cast<int>(blockIdx.x) - J.cta_base) * J.src_col_stride;
        for (int i = static_cast<int>(threadIdx.x) * 32; i < J.K; i += 256 * 32) prefetch_l2(xc + i);
    } else if ((threadIdx.x & 31) == 0) {
        const int64_t w0 = (tid - static_cast<int64_t>(P.norm_ctas) * blockDim.x) >> 5;
        const int64_t nw0 = (nthr - static_cast<int64_t>(P.norm_ctas) * blockDim.x) >> 5;
        for (int64_t item = w0; item < P.nitems; item += nw0) {
            int j = 0;
            while (j + 1 < P.njobs && item >= P.job[j + 1].item_base) ++j;
            const PrepJob &J = P.job[j];
            const int64_t local = item - J.item_base;
            const int col = static_cast<int>(local / J.nblk);
            const int b = static_cast<int>(local - static_cast<int64_t>(col) * J.nblk);
            if (J.kind == kPrepF32) {
                if (b * 32 < J.K) prefetch_l2(static_cast<const float *>(J.src) + col * J.src_col_stride + b * 32);
            } else {
                prefetch_l2(static_cast<const uint8_t *>(J.src) + (col * J.src_col_stride + b) * kQ81Bytes);
            }
        }
    }
    // This grid may itself be a programmatic dependent of the previous GEMV
    // launch (which shares the workspace): wait for it before writing.
    pdl_wait();
#if Q4K_TIMELINE
    const uint64_t tl_wait = globaltimer_ns();
#endif

    for (int64_t i = tid; i < P.zero_count; i += nthr) P.zero_ptr[i] = 0;
    // A gathering call reads activations that may come from the previous
    // gathering call's full output: wait for the peers' rows first.
    if (P.gwait.world > 1) {
        if (threadIdx.x == 0) gather_wait_flags(P.gwait);
        __syncthreads();
    }

    if (static_cast<int>(blockIdx.x) < P.norm_ctas) {
        int j = 0;
        while (!(P.job[j].norm && static_cast<int>(blockIdx.x) < P.job[j].cta_base + P.job[j].ncols)) ++j;
        prep_norm_column(P.job[j], static_cast<int>(blockIdx.x) - P.job[j].cta_base);
        return;
    }
    const int lane = threadIdx.x & 31;
    // warp items of the other jobs, over the CTAs after the normalizing ones
    const int64_t ftid = tid - static_cast<int64_t>(P.norm_ctas) * blockDim.x;
    const int64_t wid = ftid >> 5, nw = (nthr - static_cast<int64_t>(P.norm_ctas) * blockDim.x) >> 5;
    for (int64_t item = wid; item < P.nitems; item += nw) {
        // (a normalizing job owns no items: its item_base equals the next job's)
        int j = 0;
        while (j + 1 < P.njobs && item >= P.job[j + 1].item_base) ++j;
        const PrepJob &J = P.job[j];
        const int64_t local = item - J.item_base;
        const int col = static_cast<int>(local / J.nblk);
        const int b = static_cast<int>(local - static_cast<int64_t>(col) * J.nblk);
        const int pos = b * 32 + lane;

        int q;
        __half dh;
        if (J.kind == kPrepF32) {
            const float *xc = static_cast<const float *>(J.src) + col * J.src_col_stride;
            const float x = pos < J.K ? xc[pos] : 0.0f;
            quantize_value(x, q, dh);
            if (J.q81_out != nullptr) {
                const float sum = warp_sum_f32(x);
                uint8_t *blk = J.q81_out + (col * J.q81_col_stride + b) * kQ81Bytes;
                blk[4 + lane] = static_cast<uint8_t>(static_cast<int8_t>(q));
                if (lane == 0) {
                    *reinterpret_cast<__half2 *>(blk) = __halves2half2(dh, __float2half_rn(sum));
                }
            }
        } else {
            const uint8_t *blk = static_cast<const uint8_t *>(J.src) +
                                 (col * J.src_col_stride + b) * kQ81Bytes;
            q = static_cast<int8_t>(blk[4 + lane]);
            dh = *reinterpret_cast<const __half *>(blk);
        }

        if (J.act != nullptr && b * 32 < J.K) {
            int32_t *dT = J.dump_T != nullptr ? J.dump_T + static_cast<int64_t>(col) * (J.K / 32) + b : nullptr;
            write_q8a(J.act + col * J.act_col_stride, b, lane, q, dh, dT);
        }
    }
#if Q4K_TIMELINE
    // (the normalizing CTAs returned above: block-uniform, so the barrier is safe)
    __syncthreads();
    if (threadIdx.x == 0 && P.tl != nullptr && blockIdx.x < Q4K_TIMELINE_PREP_CTAS) {
        unsigned long long *o = P.tl + (static_cast<int64_t>(P.tl_slot) * Q4K_TIMELINE_PREP_CTAS + blockIdx.x) * 4;
        o[0] = tl_start;
        o[1] = tl_wait;
        o[2] = globaltimer_ns();
        o[3] = 1;
    }
#endif
}

// ============================================================================
// GEMV
// ============================================================================
// Position of an atom: task t, row group g of the task, atom kp of the group.
// Workers walk their contiguous atom range with an incremental cursor.
struct AtomCursor {
    int t;
    int g;
    int kp;
};

__device__ __forceinline__ AtomCursor locate_atom(const GemvParams &P, int64_t a) {
    int t = 0;
    while (t + 1 < P.ntasks && a >= P.task[t + 1].atom_base) ++t;
    const int local = static_cast<int>(a - P.task[t].atom_base);
    const int apr = P.task[t].apr;
    AtomCursor c;
    c.t = t;
    c.g = local / apr;
    c.kp = local - c.g * apr;
    return c;
}

// The same, searching from task t (a task near atom a: the previous one of a
// monotonic walk).
__device__ __forceinline__ AtomCursor locate_atom_from(const GemvParams &P, int64_t a, int t) {
    while (t + 1 < P.ntasks && a >= P.task[t + 1].atom_base) ++t;
    while (t > 0 && a < P.task[t].atom_base) --t;
    const int local = static_cast<int>(a - P.task[t].atom_base);
    const int apr = P.task[t].apr;
    AtomCursor c;
    c.t = t;
    c.g = local / apr;
    c.kp = local - c.g * apr;
    return c;
}

__device__ __forceinline__ void advance(const GemvParams &P, AtomCursor &c) {
    if (++c.kp == P.task[c.t].apr) {
        c.kp = 0;
        if (++c.g == P.task[c.t].ngroups) {
            c.g = 0;
            ++c.t;
        }
    }
}

// The atom before c (never called on atom 0).
__device__ __forceinline__ void retreat(const GemvParams &P, AtomCursor &c) {
    if (c.kp > 0) {
        --c.kp;
        return;
    }
    if (c.g > 0) {
        --c.g;
    } else {
        --c.t;
        c.g = P.task[c.t].ngroups - 1;
    }
    c.kp = P.task[c.t].apr - 1;
}

// Odd workers walk their atom range backwards, so that both sides of every
// worker boundary read it at about the same time (both first or both last):
// the tensor-map copies promote each 144-byte row piece to whole 256-byte L2
// lines, and a line shared by two workers' ranges is then read from DRAM once
// instead of twice (the second reader used to come a whole range later, long
// after the line had been evicted).
#ifndef Q4K_ALTERNATE_WALK
#define Q4K_ALTERNATE_WALK 1
#endif
__device__ __forceinline__ bool walks_back(int64_t worker) { return Q4K_ALTERNATE_WALK && (worker & 1) != 0; }
__device__ __forceinline__ void step(const GemvParams &P, AtomCursor &c, bool back) {
    if (back)
        retreat(P, c);
    else
        advance(P, c);
}

// First atom of worker w under the uniform partition of natoms over nworkers.
__device__ __forceinline__ int64_t worker_begin(const GemvParams &P, int64_t w) {
    return P.natoms * w / P.nworkers;
}
// Worker whose range holds atom a.
__device__ __forceinline__ int64_t worker_of(const GemvParams &P, int64_t a) {
    return ((a + 1) * P.nworkers - 1) / P.natoms;
}

// Stage layout: [kKS boxes of 32 rows x 144 B][NC columns x kKS activation
// records]; Q6_K: [8 rows x 1680 B][NC columns x 8 records at a 336-byte pitch].
template <int NC, int MODE = kModePlain>
struct Stage {
    static constexpr int kActOff = MODE == kModeQ6 ? kQ6BoxBytes : kWStageBytes;
    static constexpr int kBytes = stage_bytes_m(NC, MODE);
    // tensor-map boxes land 128-byte aligned: every stage, box and record
    // region starts on a multiple of 128 bytes from the ring base
    static_assert(kBoxBytes % 128 == 0 && kActOff % 128 == 0 && kBytes % 128 == 0, "stage alignment");
};
static_assert(sizeof(GemvParams) <= 32764, "kernel parameters exceed the 32 KB launch limit");

// Announce the atom's bytes and copy its weights: one tensor-map box (32 rows
// x 144 bytes) per super-block, issued by lane 0.  Rows past the matrix end
// are zero-filled by the copy and still counted in its byte total.
template <int NC, int MODE>
__device__ __forceinline__ void issue_weights(const GemvParams &P, const AtomCursor &c, uint32_t stage,
                                              uint32_t bar, int lane) {
    const TaskDesc &T = P.task[c.t];
    if (lane == 0) {
#if Q4K_WEIGHT_EVICT_FIRST
        const uint64_t pol = l2_evict_first_policy();
#define Q4K_TMA(dst, tm, x, y, b) tma_load_2d_hint(dst, tm, x, y, b, pol)
#else
#define Q4K_TMA(dst, tm, x, y, b) tma_load_2d(dst, tm, x, y, b)
#endif
        if (MODE == kModeQ6) {
            // 8 rows x 8 super-blocks: one box of 210 uint64 x 8 rows
            mbar_expect_tx(bar, static_cast<uint32_t>(kQ6BoxBytes + NC * kQ6AtomSB * kActSBBytes));
            Q4K_TMA(stage, &P.tmap[c.t], c.kp * (kQ6RowBytes / 8), c.g * kQ6Rows, bar);
        } else if (MODE == kModeR2) {
            // one super-block of 64 rows: two boxes of 32 rows
            mbar_expect_tx(bar, static_cast<uint32_t>(2 * kBoxBytes + NC * kActSBBytes));
            Q4K_TMA(stage, &P.tmap[c.t], c.kp * 36, c.g * 64, bar);
            Q4K_TMA(stage + kBoxBytes, &P.tmap[c.t], c.kp * 36, c.g * 64 + 32, bar);
        } else {
            // a gated task's second half of atoms reads the gate matrix
            const bool second = MODE == kModeGated && T.has_gate && c.kp >= T.half;
            const CUtensorMap *tm = second ? &P.tmap_gate[T.gate_map] : &P.tmap[c.t];
            const int kb0 = (second ? c.kp - T.half : c.kp) * kKS;
            const int nsb = min(kKS, T.nb - kb0);
            // (the single-launch mode's stages carry weights only)
            mbar_expect_tx(bar, static_cast<uint32_t>(nsb * (kBoxBytes + (MODE == kModeActSmem ? 0 : NC * kActSBBytes))));
#pragma unroll
            for (int i = 0; i < kKS; ++i)
                if (i < nsb) Q4K_TMA(stage + i * kBoxBytes, tm, (kb0 + i) * 36, c.g * 32, bar);
        }
#undef Q4K_TMA
    }
    __syncwarp();
}

// Copy the atom's activation records (one copy per column, lanes 0..NC-1).
// Only after griddepcontrol.wait: the prep kernel writes them.
template <int NC, int MODE>
__device__ __forceinline__ void issue_acts(const GemvParams &P, const AtomCursor &c, uint32_t stage,
                                           uint32_t bar, int lane) {
    if constexpr (MODE == kModeActSmem) return;  // records already in shared memory
    const TaskDesc &T = P.task[c.t];
    if constexpr (MODE == kModeQ6) {
        // the 8 records of the atom's super-blocks, per column, at a 336-byte pitch
        for (int i = lane; i < NC * kQ6AtomSB; i += 32) {
            const int j = i / kQ6AtomSB, sbi = i % kQ6AtomSB;
            const uint8_t *src =
                T.act + j * T.act_col_stride + static_cast<int64_t>(c.kp * kQ6AtomSB + sbi) * kActSBBytes;
            bulk_g2s(stage + Stage<NC, MODE>::kActOff + j * (kQ6AtomSB * kQ6RecPitch) + sbi * kQ6RecPitch, src,
                     static_cast<uint32_t>(kActSBBytes), bar);
        }
        return;
    }
    // a two-row atom is one super-block (one record); a gated task's second
    // half of atoms reads the same records as its first
    const int kq = (MODE == kModeGated && T.has_gate && c.kp >= T.half) ? c.kp - T.half : c.kp;
    const int kb0 = MODE == kModeR2 ? kq : kq * kKS;
    const int nsb = MODE == kModeR2 ? 1 : min(kKS, T.nb - kb0);
    if (lane < NC) {
        const uint8_t *src = T.act + lane * T.act_col_stride + static_cast<int64_t>(kb0) * kActSBBytes;
        bulk_g2s(stage + Stage<NC, MODE>::kActOff + lane * q_col_pitch(MODE), src,
                 static_cast<uint32_t>(nsb * kActSBBytes), bar);
    }
}

// Bounded wait on an mbarrier phase.  false after `limit_ns` without completion.
__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// Bounded wait until the shared-memory word at a reaches want (written by
// another warp of the CTA); backs off with nanosleep.  false after kWaitLimitNs.
__device__ __forceinline__ bool wait_word_geq(uint32_t a, int want) {
    if (ld_volatile_s32(a) >= want) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        __nanosleep(it < 16 ? 32 : 128);
        if (ld_volatile_s32(a) >= want) return true;
        if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// Sub-block pair c (sub-blocks 2c, 2c+1) of one super-block of one row
// (weights at p) against NC activation records (act, column stride acs).
// acc[j] holds a packed pair of partial sums for column j.
template <int NC, bool DUMP>
__device__ __forceinline__ void pair_dot(uint32_t p, uint32_t act, uint32_t acs, int c, float d, float nd23,
                                         float dmin, float pm23, uint32_t scw, uint32_t mw, uint64_t (&acc)[NC],
                                         int32_t *dumpS, int64_t dump_col_stride) {
    const int b0 = (c & 1) * 2;
    // d*sc and -dmin*m of sub-blocks 2c, 2c+1: (byte + 2^23)*x - 2^23*x == byte*x, one rounding
    const uint64_t dsc = f2_pack(fmaf(byte_magic(scw, b0), d, nd23), fmaf(byte_magic(scw, b0 + 1), d, nd23));
    const uint64_t ndm =
        f2_pack(fmaf(byte_magic(mw, b0), -dmin, pm23), fmaf(byte_magic(mw, b0 + 1), -dmin, pm23));
    const uint4 wa = lds128(p + 16 + 32 * c);
    const uint4 wb = lds128(p + 32 + 32 * c);
    const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    uint32_t lo[8], hi[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        lo[k] = w[k] & 0x0F0F0F0Fu;
        hi[k] = w[k] & 0xF0F0F0F0u;  // 16 x nibble, unsigned bytes
    }
    const uint64_t magic2 = f2_pack(-kMagicF, -kMagicF);
#pragma unroll
    for (int j = 0; j < NC; ++j) {
        const uint32_t aj = act + j * acs;
        const uint4 qe0 = lds128(aj + 64 * c);
        const uint4 qe1 = lds128(aj + 64 * c + 16);
        const uint4 qo0 = lds128(aj + 64 * c + 32);
        const uint4 qo1 = lds128(aj + 64 * c + 48);
        const uint4 meta = lds128(aj + kActMetaOff + 16 * c);
        const uint32_t qe[8] = {qe0.x, qe0.y, qe0.z, qe0.w, qe1.x, qe1.y, qe1.z, qe1.w};
        const uint32_t qo[8] = {qo0.x, qo0.y, qo0.z, qo0.w, qo1.x, qo1.y, qo1.z, qo1.w};
        int se = kMagicI, so = kMagicI;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            se = dp4a_us(lo[k], qe[k], se);
            so = dp4a_us(hi[k], qo[k], so);
        }
        if constexpr (DUMP) {
            // exact sub-block sums (the odd one was formed on 16 x nibble)
            dumpS[j * dump_col_stride + 2 * c] = se - kMagicI;
            dumpS[j * dump_col_stride + 2 * c + 1] = (so - kMagicI) >> 4;
        }
        const uint64_t sf = f2_add(f2_pack(__int_as_float(se), __int_as_float(so)), magic2);
        const uint64_t g = f2_mul(sf, f2_pack(__uint_as_float(meta.x), __uint_as_float(meta.y)));
        acc[j] = f2_fma(g, dsc, acc[j]);
        acc[j] = f2_fma(f2_pack(__uint_as_float(meta.z), __uint_as_float(meta.w)), ndm, acc[j]);
    }
}

// One super-block of one row: weights at p, the activation records of its
// NC columns at act, acs bytes apart.  Semantics of kernels/vecdotq.cuh:461-483,
// :775-819.
template <int NC, bool DUMP>
__device__ __forceinline__ void sb_dot(uint32_t p, uint32_t act, uint32_t acs, uint64_t (&acc)[NC],
                                       int32_t *dumpS, int64_t dump_col_stride) {
    const uint4 h = lds128(p);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
    const float d = dm.x, dmin = dm.y;
    // 6-bit scales sc0..7 and mins m0..7, four per word (vecdotq.cuh:796-807).
    const uint32_t sc03 = h.y & 0x3F3F3F3Fu;
    const uint32_t m03 = h.z & 0x3F3F3F3Fu;
    const uint32_t sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    const float nd23 = -8388608.0f * d;
    const float pm23 = 8388608.0f * dmin;
    if constexpr (NC <= 2) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
            pair_dot<NC, DUMP>(p, act, acs, c, d, nd23, dmin, pm23, c < 2 ? sc03 : sc47, c < 2 ? m03 : m47,
                               acc, dumpS, dump_col_stride);
    } else {
#pragma unroll 1
        for (int c = 0; c < 4; ++c)
            pair_dot<NC, DUMP>(p, act, acs, c, d, nd23, dmin, pm23, c < 2 ? sc03 : sc47, c < 2 ? m03 : m47,
                               acc, dumpS, dump_col_stride);
    }
}

// Columns [j0, j0 + NCW) of one atom (all NC columns unless two warps split
// them) against its ring stage.
// A row's running sums, one per column.  Each super-block is summed in fp32
// from zero (16 products per column) and added here with Kahan compensation:
// the running sum of a row can grow far beyond its final value, and plain
// fp32 accumulation across super-blocks loses ~1e-4 absolute on rows that
// cancel (outside the 1e-4 + 1e-5 relative bar for K >= 14336).
template <int NCW>
struct RowAcc {
    float sum[NCW];
    float comp[NCW];  // low-order part lost by sum, negated
    __device__ __forceinline__ void clear() {
#pragma unroll
        for (int j = 0; j < NCW; ++j) sum[j] = comp[j] = 0.0f;
    }
    __device__ __forceinline__ void add(int j, float v) {
        const float y = v - comp[j];
        const float t = sum[j] + y;
        comp[j] = (t - sum[j]) - y;
        sum[j] = t;
    }
    __device__ __forceinline__ float value(int j) const { return sum[j] - comp[j]; }
};

// Q6_K rows: super-block terms reach ~1e5 (int8 scales times 6-bit values)
// while rows cancel to ~1, and a row's super-blocks are spread over four
// lanes, so the sums run in fp64 (one rounding at the end).
template <int NCW>
struct RowAccD {
    double s[NCW];
    __device__ __forceinline__ void clear() {
#pragma unroll
        for (int j = 0; j < NCW; ++j) s[j] = 0.0;
    }
    __device__ __forceinline__ void add(int j, double v) { s[j] += v; }
};

// Per-row constants of one super-block: d, dmin and the 6-bit scales/mins.
struct SbHead {
    float d, dmin, nd23, pm23;
    uint32_t sc03, m03, sc47, m47;
};
__device__ __forceinline__ SbHead sb_head(uint32_t p) {
    const uint4 h = lds128(p);
    const float2 dm = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
    SbHead H;
    H.d = dm.x;
    H.dmin = dm.y;
    H.sc03 = h.y & 0x3F3F3F3Fu;
    H.m03 = h.z & 0x3F3F3F3Fu;
    H.sc47 = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    H.m47 = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    H.nd23 = -8388608.0f * H.d;
    H.pm23 = 8388608.0f * H.dmin;
    return H;
}

// Sub-block pair c of one super-block for two rows (weights at pA, pB) that
// share every activation load: the arithmetic of pair_dot, once per row.
template <int NC>
__device__ __forceinline__ void pair_dot2(uint32_t pA, uint32_t pB, uint32_t act, int c, const SbHead &A,
                                          const SbHead &B, uint64_t (&accA)[NC], uint64_t (&accB)[NC]) {
    const int b0 = (c & 1) * 2;
    const uint32_t scA = c < 2 ? A.sc03 : A.sc47, mA = c < 2 ? A.m03 : A.m47;
    const uint32_t scB = c < 2 ? B.sc03 : B.sc47, mB = c < 2 ? B.m03 : B.m47;
    const uint64_t dscA = f2_pack(fmaf(byte_magic(scA, b0), A.d, A.nd23), fmaf(byte_magic(scA, b0 + 1), A.d, A.nd23));
    const uint64_t ndmA =
        f2_pack(fmaf(byte_magic(mA, b0), -A.dmin, A.pm23), fmaf(byte_magic(mA, b0 + 1), -A.dmin, A.pm23));
    const uint64_t dscB = f2_pack(fmaf(byte_magic(scB, b0), B.d, B.nd23), fmaf(byte_magic(scB, b0 + 1), B.d, B.nd23));
    const uint64_t ndmB =
        f2_pack(fmaf(byte_magic(mB, b0), -B.dmin, B.pm23), fmaf(byte_magic(mB, b0 + 1), -B.dmin, B.pm23));
    uint32_t loA[8], hiA[8], loB[8], hiB[8];
    {
        const uint4 wa = lds128(pA + 16 + 32 * c), wb = lds128(pA + 32 + 32 * c);
        const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            loA[k] = w[k] & 0x0F0F0F0Fu;
            hiA[k] = w[k] & 0xF0F0F0F0u;
        }
    }
    {
        const uint4 wa = lds128(pB + 16 + 32 * c), wb = lds128(pB + 32 + 32 * c);
        const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            loB[k] = w[k] & 0x0F0F0F0Fu;
            hiB[k] = w[k] & 0xF0F0F0F0u;
        }
    }
    const uint64_t magic2 = f2_pack(-kMagicF, -kMagicF);
#pragma unroll
    for (int j = 0; j < NC; ++j) {
        const uint32_t aj = act + j * q_col_pitch(kModeR2);
        const uint4 qe0 = lds128(aj + 64 * c);
        const uint4 qe1 = lds128(aj + 64 * c + 16);
        const uint4 qo0 = lds128(aj + 64 * c + 32);
        const uint4 qo1 = lds128(aj + 64 * c + 48);
        const uint4 meta = lds128(aj + kActMetaOff + 16 * c);
        const uint32_t qe[8] = {qe0.x, qe0.y, qe0.z, qe0.w, qe1.x, qe1.y, qe1.z, qe1.w};
        const uint32_t qo[8] = {qo0.x, qo0.y, qo0.z, qo0.w, qo1.x, qo1.y, qo1.z, qo1.w};
        int seA = kMagicI, soA = kMagicI, seB = kMagicI, soB = kMagicI;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            seA = dp4a_us(loA[k], qe[k], seA);
            soA = dp4a_us(hiA[k], qo[k], soA);
            seB = dp4a_us(loB[k], qe[k], seB);
            soB = dp4a_us(hiB[k], qo[k], soB);
        }
        const uint64_t f = f2_pack(__uint_as_float(meta.x), __uint_as_float(meta.y));
        const uint64_t a = f2_pack(__uint_as_float(meta.z), __uint_as_float(meta.w));
        const uint64_t gA = f2_mul(f2_add(f2_pack(__int_as_float(seA), __int_as_float(soA)), magic2), f);
        const uint64_t gB = f2_mul(f2_add(f2_pack(__int_as_float(seB), __int_as_float(soB)), magic2), f);
        accA[j] = f2_fma(a, ndmA, f2_fma(gA, dscA, accA[j]));
        accB[j] = f2_fma(a, ndmB, f2_fma(gB, dscB, accB[j]));
    }
}

#if Q4K_R2_MMA
// ---- two-row atoms on the tensor cores (ncols >= kR2MmaMin) ------------------
// The integer sub-block sums of a 64-row atom come from int8 MMAs instead of
// dp4a: per sub-block pair c, for each 16-row tile of the atom,
// D(16 x 8) = nibbles(16 x 32, u8) x q8(32 x 8 columns, s8), once for the
// even sub-block (low nibbles) and once for the odd one (high nibbles).
// Fragments (mma.m16n8k32, g = lane / 4, t = lane % 4): A words = 4 weight
// bytes of rows g and g + 8 at k = 4t and 16 + 4t (the row's 32 qs bytes of
// the pair); B words = 4 q8 values of column g at the same k; D = rows g and
// g + 8, columns 2t and 2t + 1.  The exact integer sums go through a
// per-warp scratch [2 sub-blocks][64 rows][8 columns] (int32, 16-byte
// halves of a row swapped on rows 4-7 mod 8 so that neither the stores nor
// the row reads conflict) and come back lane = row, where the float
// combination is pair_dot2's, operation for operation (bit-identical sums).
__device__ __forceinline__ void mma_u8s8(uint32_t (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void sts64u(uint32_t a, uint32_t x, uint32_t y) {
    asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
constexpr int kR2ScrBytes = 2 * 64 * 8 * 4;  // per warp
static_assert(r2_scr_bytes(8, kModeR2) == kMaxWarps * kR2ScrBytes, "two-row scratch size");
// byte address of (sub-block e, row r, column col) in a warp's scratch
__device__ __forceinline__ uint32_t r2_scr(uint32_t scr, int e, int r, int col) {
    return scr + static_cast<uint32_t>(((e * 64 + r) * 8 + (col ^ (((r >> 2) & 1) * 4))) * 4);
}

// The 8 MMAs of sub-block pair c: d[e][i] = sums of sub-block 2c + e, tile i.
template <int NC>
__device__ __forceinline__ void pair_mma(uint32_t box, uint32_t act, int lane, int c, uint32_t (&d)[2][4][4]) {
    const int g = lane >> 2, t = lane & 3;
    uint32_t bE0 = 0u, bE1 = 0u, bO0 = 0u, bO1 = 0u;  // columns >= NC stay zero
    if (g < NC) {
        const uint32_t aj = act + static_cast<uint32_t>(g * q_col_pitch(kModeR2) + 64 * c + 4 * t);
        bE0 = lds32(aj);
        bE1 = lds32(aj + 16);
        bO0 = lds32(aj + 32);
        bO1 = lds32(aj + 48);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t p = box + static_cast<uint32_t>((i >> 1) * kBoxBytes + (16 * (i & 1) + g) * kPitch + 16 +
                                                       32 * c + 4 * t);
        const uint32_t w0 = lds32(p), w1 = lds32(p + 8 * kPitch), w2 = lds32(p + 16), w3 = lds32(p + 8 * kPitch + 16);
        const uint32_t aE[4] = {w0 & 0x0F0F0F0Fu, w1 & 0x0F0F0F0Fu, w2 & 0x0F0F0F0Fu, w3 & 0x0F0F0F0Fu};
        const uint32_t aO[4] = {(w0 >> 4) & 0x0F0F0F0Fu, (w1 >> 4) & 0x0F0F0F0Fu, (w2 >> 4) & 0x0F0F0F0Fu,
                                (w3 >> 4) & 0x0F0F0F0Fu};
        mma_u8s8(d[0][i], aE, bE0, bE1);
        mma_u8s8(d[1][i], aO, bO0, bO1);
    }
}

// Pair c's sums into the warp's scratch (every lane's reads of the previous
// pair are done: the caller's __syncwarp).
__device__ __forceinline__ void pair_store(uint32_t scr, int lane, const uint32_t (&d)[2][4][4]) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = 16 * i + g;
            sts64u(r2_scr(scr, e, r, 2 * t), d[e][i][0], d[e][i][1]);
            sts64u(r2_scr(scr, e, r + 8, 2 * t), d[e][i][2], d[e][i][3]);
        }
    }
}

// Pair c's sums back lane = row (rows lane and 32 + lane), combined as
// pair_dot2 combines them.
template <int NC>
__device__ __forceinline__ void pair_combine(uint32_t act, uint32_t scr, int lane, int c, const SbHead &A,
                                             const SbHead &B, uint64_t (&accA)[NC], uint64_t (&accB)[NC]) {
    int eA[8], oA[8], eB[8], oB[8];
#pragma unroll
    for (int h = 0; h < (NC + 3) / 4; ++h) {
        const uint4 v0 = lds128(r2_scr(scr, 0, lane, 4 * h)), v1 = lds128(r2_scr(scr, 1, lane, 4 * h));
        const uint4 v2 = lds128(r2_scr(scr, 0, 32 + lane, 4 * h)), v3 = lds128(r2_scr(scr, 1, 32 + lane, 4 * h));
        eA[4 * h] = v0.x; eA[4 * h + 1] = v0.y; eA[4 * h + 2] = v0.z; eA[4 * h + 3] = v0.w;
        oA[4 * h] = v1.x; oA[4 * h + 1] = v1.y; oA[4 * h + 2] = v1.z; oA[4 * h + 3] = v1.w;
        eB[4 * h] = v2.x; eB[4 * h + 1] = v2.y; eB[4 * h + 2] = v2.z; eB[4 * h + 3] = v2.w;
        oB[4 * h] = v3.x; oB[4 * h + 1] = v3.y; oB[4 * h + 2] = v3.z; oB[4 * h + 3] = v3.w;
    }
    const int b0 = (c & 1) * 2;
    const uint32_t scA = c < 2 ? A.sc03 : A.sc47, mA = c < 2 ? A.m03 : A.m47;
    const uint32_t scB = c < 2 ? B.sc03 : B.sc47, mB = c < 2 ? B.m03 : B.m47;
    const uint64_t dscA = f2_pack(fmaf(byte_magic(scA, b0), A.d, A.nd23), fmaf(byte_magic(scA, b0 + 1), A.d, A.nd23));
    const uint64_t ndmA =
        f2_pack(fmaf(byte_magic(mA, b0), -A.dmin, A.pm23), fmaf(byte_magic(mA, b0 + 1), -A.dmin, A.pm23));
    const uint64_t dscB = f2_pack(fmaf(byte_magic(scB, b0), B.d, B.nd23), fmaf(byte_magic(scB, b0 + 1), B.d, B.nd23));
    const uint64_t ndmB =
        f2_pack(fmaf(byte_magic(mB, b0), -B.dmin, B.pm23), fmaf(byte_magic(mB, b0 + 1), -B.dmin, B.pm23));
#pragma unroll
    for (int j = 0; j < NC; ++j) {
        const uint4 meta = lds128(act + j * q_col_pitch(kModeR2) + kActMetaOff + 16 * c);
        const uint64_t f = f2_pack(__uint_as_float(meta.x), __uint_as_float(meta.y));
        const uint64_t a = f2_pack(__uint_as_float(meta.z), __uint_as_float(meta.w));
        // the odd sum as pair_dot2 forms it (on 16 x nibble): exact in fp32
        const uint64_t gA = f2_mul(f2_pack(static_cast<float>(eA[j]), static_cast<float>(oA[j] * 16)), f);
        const uint64_t gB = f2_mul(f2_pack(static_cast<float>(eB[j]), static_cast<float>(oB[j] * 16)), f);
        accA[j] = f2_fma(a, ndmA, f2_fma(gA, dscA, accA[j]));
        accB[j] = f2_fma(a, ndmB, f2_fma(gB, dscB, accB[j]));
    }
}

// The 4 pairs of a super-block, software-pipelined: pair c + 1's loads and
// MMAs are issued before pair c's scratch round trip and float combination.
template <int NC>
__device__ __forceinline__ void sb_dot2_mma(uint32_t box, uint32_t act, uint32_t scr, int lane,
                                            uint64_t (&accA)[NC], uint64_t (&accB)[NC]) {
    const SbHead A = sb_head(box + lane * kPitch), B = sb_head(box + kBoxBytes + lane * kPitch);
    uint32_t d0[2][4][4], d1[2][4][4];
    pair_mma<NC>(box, act, lane, 0, d0);
    // (unrolled: rolled, it measured 4 % slower at 8 columns)
#pragma unroll
    for (int c = 0; c < 4; c += 2) {
        __syncwarp();  // the previous pair's scratch reads are done
        pair_store(scr, lane, d0);
        pair_mma<NC>(box, act, lane, c + 1, d1);
        __syncwarp();
        pair_combine<NC>(act, scr, lane, c, A, B, accA, accB);
        __syncwarp();
        pair_store(scr, lane, d1);
        if (c + 2 < 4) pair_mma<NC>(box, act, lane, c + 2, d0);
        __syncwarp();
        pair_combine<NC>(act, scr, lane, c + 1, A, B, accA, accB);
    }
}
#endif

// One super-block of two rows (weights at pA and pB) against NC activation
// records: sb_dot for both, with the activation loads shared.
template <int NC>
__device__ __forceinline__ void sb_dot2(uint32_t pA, uint32_t pB, uint32_t act, uint64_t (&accA)[NC],
                                        uint64_t (&accB)[NC]) {
    const SbHead A = sb_head(pA), B = sb_head(pB);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) pair_dot2<NC>(pA, pB, act, c, A, B, accA, accB);
}

// ---- Q6_K --------------------------------------------------------------------
// Word i (4 bytes) of the super-block at smem byte address a; MIS: a is 2 mod 4
// (odd super-blocks of a 1680-byte row), read as two aligned words and a
// funnel shift.
template <bool MIS>
__device__ __forceinline__ uint32_t q6_word(uint32_t a, int i) {
    if constexpr (!MIS) {
        return lds32(a + 4 * i);
    } else {
        return __funnelshift_r(lds32(a - 2 + 4 * i), lds32(a + 2 + 4 * i), 16);
    }
}

// Signed 6-bit values minus 32, four per word: v - 32 for v in 0..63 is v ^ 0x20
// with bit 5 of the result copied into bits 6 and 7 (sign extension).
__device__ __forceinline__ uint32_t q6_signed(uint32_t v) {
    const uint32_t t = v ^ 0x20202020u;
    const uint32_t m = t & 0x20202020u;
    return t | (m << 1) | (m << 2);
}

// One Q6_K super-block of one row (at smem a) against NC activation records
// (act, column pitch 8 * 336): per q8_1 block k, S = sum over each 16-weight
// half of (q6 - 32) * q8 (signed dp4a), isum = sc[2k] S0 + sc[2k+1] S1, times
// d8; the super-block total times d (kernels/vecdotq.cuh:576-601, :867-890).
template <int NC, bool MIS>
__device__ __forceinline__ void q6_sb(uint32_t a, uint32_t act, RowAccD<NC> &acc) {
    const uint32_t dw = MIS ? lds32(a + 206) : lds32(a + 208);
    const double d = __half2float(__ushort_as_half(static_cast<unsigned short>(MIS ? dw >> 16 : dw & 0xFFFFu)));
    uint32_t scw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) scw[i] = q6_word<MIS>(a + 192, i);
    double s[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) s[c] = 0.0;
#pragma unroll 1
    for (int n = 0; n < 2; ++n) {
        uint32_t ql[16], qh[8];
#pragma unroll
        for (int i = 0; i < 16; ++i) ql[i] = q6_word<MIS>(a + 64 * n, i);
#pragma unroll
        for (int i = 0; i < 8; ++i) qh[i] = q6_word<MIS>(a + 128 + 32 * n, i);
        // Up to two columns: unsigned 6-bit values (dp4a.u32.s32) and the
        // 16-value activation sums T0, T1 (dp4a with 0x01010101) for the -32
        // offset: fewer operations per weight than the bytewise subtraction,
        // which pays off while the per-row work is shared by few columns.
        constexpr bool kUnsigned = NC <= Q4K_Q6_UNSIGNED_MAX;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int k = 4 * n + jj;
            uint32_t vi[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t lo = (ql[8 * (jj & 1) + i] >> (4 * (jj >> 1))) & 0x0F0F0F0Fu;
                const uint32_t hi = (jj < 2 ? (qh[i] << (4 - 2 * jj)) : (qh[i] >> (2 * jj - 4))) & 0x30303030u;
                vi[i] = kUnsigned ? (lo | hi) : q6_signed(lo | hi);
            }
            const uint32_t sw = scw[k >> 1];
            const int sc0 = static_cast<int32_t>(sw << (24 - 16 * (k & 1))) >> 24;
            const int sc1 = static_cast<int32_t>(sw << (16 - 16 * (k & 1))) >> 24;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const uint32_t ac = act + c * (kQ6AtomSB * kQ6RecPitch);
                const uint4 q0 = lds128(ac + 32 * k), q1 = lds128(ac + 32 * k + 16);
                int S0, S1;
                if constexpr (kUnsigned) {
                    S0 = dp4a_us(vi[0], q0.x, 0);
                    S0 = dp4a_us(vi[1], q0.y, S0);
                    S0 = dp4a_us(vi[2], q0.z, S0);
                    S0 = dp4a_us(vi[3], q0.w, S0);
                    S1 = dp4a_us(vi[4], q1.x, 0);
                    S1 = dp4a_us(vi[5], q1.y, S1);
                    S1 = dp4a_us(vi[6], q1.z, S1);
                    S1 = dp4a_us(vi[7], q1.w, S1);
                    int T0 = dp4a_us(0x01010101u, q0.x, 0);
                    T0 = dp4a_us(0x01010101u, q0.y, T0);
                    T0 = dp4a_us(0x01010101u, q0.z, T0);
                    T0 = dp4a_us(0x01010101u, q0.w, T0);
                    int T1 = dp4a_us(0x01010101u, q1.x, 0);
                    T1 = dp4a_us(0x01010101u, q1.y, T1);
                    T1 = dp4a_us(0x01010101u, q1.z, T1);
                    T1 = dp4a_us(0x01010101u, q1.w, T1);
                    S0 -= 32 * T0;
                    S1 -= 32 * T1;
                } else {
                    S0 = dp4a_ss(vi[0], q0.x, 0);
                    S0 = dp4a_ss(vi[1], q0.y, S0);
                    S0 = dp4a_ss(vi[2], q0.z, S0);
                    S0 = dp4a_ss(vi[3], q0.w, S0);
                    S1 = dp4a_ss(vi[4], q1.x, 0);
                    S1 = dp4a_ss(vi[5], q1.y, S1);
                    S1 = dp4a_ss(vi[6], q1.z, S1);
                    S1 = dp4a_ss(vi[7], q1.w, S1);
                }
                // d8 of block k: the record keeps d8 for even k and d8/16 for odd k
                const float f = __uint_as_float(lds32(ac + kActMetaOff + 16 * (k >> 1) + 4 * (k & 1)));
                const double d8 = (k & 1) ? f * 16.0f : f;  // exact (power-of-two factor)
                s[c] = fma(d8, static_cast<double>(sc0 * S0 + sc1 * S1), s[c]);  // products exact in fp64
            }
        }
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) acc.add(c, s[c] * d);
}

template <int NCW>
__device__ __forceinline__ void add_sb(RowAcc<NCW> &acc, const uint64_t (&sb)[NCW]) {
#pragma unroll
    for (int j = 0; j < NCW; ++j) {
        const float2 v = f2_unpack(sb[j]);
        acc.add(j, v.x + v.y);
    }
}

// Where the single-launch mode keeps a CTA's activation records: the base of
// the shared-memory region after the rings and, per task, its byte offset
// there (column j of super-block kb at base + off + j * nb * 320 + kb * 320).
struct ActView {
    uint32_t base;
    const int *task_off;
};

// One atom of the per-warp and dynamically scheduled kernels, added into the
// lane's running row sums: Q6_K into dacc; two-row atoms row 64g + lane into
// acc and 64g + 32 + lane into gacc; else per super-block into acc, or gacc
// for a gated task's second half of atoms (the gate matrix).  Columns
// [j0, j0 + NCW).
template <int NCW, int NC, int MODE>
__device__ __forceinline__ void compute_atom(const GemvParams &P, const AtomCursor &c, uint32_t stage, int lane,
                                             int j0, RowAcc<NCW> &acc, RowAcc<NCW> &gacc, RowAccD<NCW> &dacc,
                                             const ActView &AV) {
    const TaskDesc &T = P.task[c.t];
    if constexpr (MODE == kModeQ6) {
        // row lane & 7 of the group, super-blocks 2q and 2q+1 (q = lane >> 3)
        const int r = lane & 7, q = lane >> 3;
        const uint32_t rowa = stage + r * kQ6RowBytes;
        const uint32_t acts = stage + Stage<NC, MODE>::kActOff;
        q6_sb<NCW, false>(rowa + (2 * q) * kQ6Bytes, acts + (2 * q) * kQ6RecPitch, dacc);
        q6_sb<NCW, true>(rowa + (2 * q + 1) * kQ6Bytes, acts + (2 * q + 1) * kQ6RecPitch, dacc);
        return;
    } else if constexpr (MODE == kModeR2) {
        // 64-row group: lane holds rows 64g + lane (box 0) and 64g + 32 + lane
        // (box 1) of super-block c.kp, summed into acc and gacc; rows past
        // the end are zero-filled by the copy
        uint64_t sbA[NCW], sbB[NCW];
#pragma unroll
        for (int j = 0; j < NCW; ++j) sbA[j] = sbB[j] = 0ull;
#if Q4K_R2_MMA
        if constexpr (NC >= kR2MmaMin) {
            // (the warp's scratch follows the rings: one per ring, ring = warp)
            sb_dot2_mma<NCW>(stage, stage + Stage<NC, MODE>::kActOff,
                             AV.base + static_cast<uint32_t>((threadIdx.x >> 5) * kR2ScrBytes), lane, sbA, sbB);
        } else
#endif
        {
            sb_dot2<NCW>(stage + lane * kPitch, stage + kBoxBytes + lane * kPitch, stage + Stage<NC, MODE>::kActOff,
                         sbA, sbB);
        }
        add_sb(acc, sbA);
        add_sb(gacc, sbB);
    } else {
        constexpr bool DUMP = MODE == kModeDump;
        constexpr bool ASM = MODE == kModeActSmem;
        if constexpr (ASM) {
            // the CTA's activation table must hold this task's activation (the
            // host's bits follow the kernel's partition): never read at offset -1
            if (AV.task_off[c.t] < 0) {
                if (lane == 0) atomicExch(P.status, kStatusBadPlan);
                return;
            }
        }
        const int rows = min(32, T.nrows - c.g * 32);
        if (lane >= rows) return;
        // a gated task's second half of atoms (the dynamic kernel's launches
        // with a fused task): the gate matrix, summed into gacc
        const bool second = MODE == kModeGated && T.has_gate && c.kp >= T.half;
        const int kb0 = (second ? c.kp - T.half : c.kp) * kKS;
        // records of the atom's super-blocks: in the ring stage (copied per
        // atom), or in the CTA's activation table (single-launch mode)
        const uint32_t acs = ASM ? static_cast<uint32_t>(T.nb) * kActSBBytes : q_col_pitch(MODE);
        const uint32_t act = ASM ? AV.base + static_cast<uint32_t>(AV.task_off[c.t]) + j0 * acs +
                                       static_cast<uint32_t>(kb0) * kActSBBytes
                                 : stage + Stage<NC, MODE>::kActOff + j0 * acs;
        const int nsb = min(kKS, T.nb - kb0);
        const int row = c.g * 32 + lane;
#pragma unroll
        for (int i = 0; i < kKS; ++i) {
            if (i < nsb) {
                int32_t *dS = nullptr;
                int64_t dcs = 0;
                if constexpr (DUMP) {
                    dcs = static_cast<int64_t>(T.nrows) * T.nb * 8;
                    dS = P.dump_S + j0 * dcs + static_cast<int64_t>(row) * T.nb * 8 + (kb0 + i) * 8;
                }
                uint64_t sb[NCW];
#pragma unroll
                for (int j = 0; j < NCW; ++j) sb[j] = 0ull;
                sb_dot<NCW, DUMP>(stage + i * kBoxBytes + lane * kPitch, act + i * kActSBBytes, acs, sb, dS, dcs);
                if (second)
                    add_sb(gacc, sb);
                else
                    add_sb(acc, sb);
            }
        }
    }
}

// A task's output fields, read from the parameters once per row group.
struct OutDesc {
    float *dst;
    int64_t dcs;             // floats between output columns
    const float *xb, *gb;    // biases (or nullptr)
    int64_t bcs;             // floats between bias columns
    int has_gate, glu;
    int gworld;
};
__device__ __forceinline__ OutDesc out_desc(const GemvParams &P, const TaskDesc &T) {
    return OutDesc{T.dst, T.dst_col_stride, T.x_bias, T.gate_bias, T.bias_col_stride, T.has_gate, T.glu_op, P.gworld};
}

// Store one output value; with a fused all-gather also into every peer's
// full output buffer (same offset, plain stores over NVLink).
__device__ __forceinline__ void store_out(const GemvParams &P, const OutDesc &O, int j, int row, float v) {
    float *p = O.dst + j * O.dcs + row;
    *p = v;
    if (O.gworld > 1) {
        const int64_t off = p - P.gout_local;
        for (int q = 0; q < O.gworld; ++q)
            if (q != P.grank) P.gout_peer[q][off] = v;
    }
}

// Output of a fused row (kernels/mmvq.cu:309-338): the main result plus its
// bias, combined with the gate result plus its bias.  SWIGLU: times
// silu(g) = g / (1 + e^-g); GEGLU: times the tanh approximation of gelu(g);
// SWIGLU_OAI: the clamped variant (alpha 1.702, limit 7) with the roles of
// the reference's call (gate first); MUL: times g.
// Kept out of line: the GLU arithmetic (expf, tanhf) runs once per output
// row of a gated task, and inlined into every kernel variant it grew the
// code around the hot loops (measured: the two-row kernel 8 % slower).
__device__ __noinline__ float glu_out(int op, float v, float g) {
    switch (op) {
        case kGluSwiglu:
            return v * (g / (1.0f + expf(-g)));
        case kGluGeglu:
            return v * (0.5f * g * (1.0f + tanhf(0.79788456080286535588f * g * (1.0f + 0.044715f * g * g))));
        case kGluSwigluOai: {
            const float a = fminf(g, 7.0f);
            const float b = fmaxf(fminf(v, 7.0f), -7.0f);
            return a / (1.0f + expf(-a * 1.702f)) * (1.0f + b);
        }
        case kGluMul:
            return v * g;
        default:
            return v;
    }
}

// Final value of output (row, column j): v = W.x, g = Wg.x (a task with a
// gate), with the task's biases and gate epilogue applied (EPI: the kernel
// variants of launches with a fused task; the others store v as it is and
// carry no epilogue code).
template <bool EPI>
__device__ __forceinline__ void store_final(const GemvParams &P, const OutDesc &O, int j, int row, float v,
                                            float g) {
    if constexpr (!EPI) {
        store_out(P, O, j, row, v);
        return;
    }
    if (O.xb != nullptr) v += O.xb[j * O.bcs + row];
    if (O.has_gate) {
        if (O.gb != nullptr) g += O.gb[j * O.bcs + row];
        v = glu_out(O.glu, v, g);
    }
    store_out(P, O, j, row, v);
}

// Finish a row group this warp worked on: write it out directly if the
// worker covered all of its atoms, otherwise deposit the partial sums and let
// the last of the contributing warps add them up (always in worker order, so
// the result is deterministic) and write.  With a column split both warps of
// a worker deposit their columns and count as arrivals.  Contributors that all
// belong to this CTA count arrivals in shared memory under block-scope
// ordering; otherwise a device-scope acquire-release counter in the workspace
// is used.
// Row groups split with another CTA (plain and single-launch kernels): the
// device-scope arrival (and, for the last contributor, the sum) stalls the
// warp ~1-2 us, so a compute warp hands them to the CTA's boundary warp
// instead.  A worker has at most two split groups (the one it began inside,
// slot 0, and the one it ends inside, slot 1): one entry each per compute
// warp -- the NC main sums per lane in shared memory, the group's task and
// row group -- announced by the arrival of all 32 lanes on the entry's
// mbarrier (block-scope release).  The boundary warp knows from the workers'
// atom ranges which entries will come and waits for each on its mbarrier.
struct XHelp {
    uint32_t vals;  // [kR][2][NC][32] floats
    uint32_t bar;   // uint64 [kR][2]: one mbarrier per entry (32 arrivals)
    uint32_t tg;    // int [kR][2][2]: task, row group
    int w;          // this compute warp's ring
};

template <int NCW, int NC, int MODE>
__device__ __forceinline__ void flush_values(const GemvParams &P, const AtomCursor &cur, const float (&v)[NCW],
                                             const float (&gv)[NCW], int64_t worker, int64_t a0, int64_t a1, int lane,
                                             int j0, int64_t cta_w0, int64_t cta_w1, int *cta_cnt,
                                             const XHelp *xh = nullptr) {
    constexpr int kSplit = split_for(NC);
    constexpr bool DUMP = MODE == kModeDump;
    constexpr bool R2 = MODE == kModeR2;
    constexpr bool Q6 = MODE == kModeQ6;
    constexpr bool EPI = MODE == kModeGated;  // launches with a fused task
    const TaskDesc &T = P.task[cur.t];
    // second set of sums: the gate (gated task) or row 64g + 32 + lane (two-row launch)
    const bool gated = R2 || (EPI && T.has_gate);
    const int64_t sg = T.atom_base + static_cast<int64_t>(cur.g) * T.apr;
    const int64_t eg = sg + T.apr;
    const int row = cur.g * (R2 ? 64 : Q6 ? kQ6Rows : 32) + lane;
    const bool valid = row < T.nrows && (!Q6 || lane < kQ6Rows);
    const bool valid2 = R2 && row + 32 < T.nrows;
    const OutDesc O = out_desc(P, T);
    if (sg >= a0 && eg <= a1) {
        if (!DUMP && valid) {
#pragma unroll
            for (int j = 0; j < NCW; ++j) store_final<EPI>(P, O, j0 + j, row, v[j], gv[j]);
        }
        if (valid2) {
#pragma unroll
            for (int j = 0; j < NCW; ++j) store_out(P, O, j0 + j, row + 32, gv[j]);
        }
        return;
    }
    // Partial slot: [pcols][32] floats, the main sums of the NC columns and,
    // for a gated task, the gate sums after them (two-row launch: the second
    // row's sums).  pcols: 2 * NC in launches with a gate or two rows per lane.
    const int slot = (a0 > sg) ? 0 : 1;  // 0: group began before this worker, 1: it covers the start
    const int64_t w1 = worker_of(P, sg), w2 = worker_of(P, eg - 1);
    const bool local = P.packed && w1 >= cta_w0 && w2 <= cta_w1;
    if (xh != nullptr && !local) {
        // to the boundary warp (it deposits, arrives and, if last, adds up)
        const uint32_t dst = xh->vals + static_cast<uint32_t>(((xh->w * 2 + slot) * NCW) * 128 + lane * 4);
#pragma unroll
        for (int j = 0; j < NCW; ++j) sts32f(dst + j * 128, v[j]);
        if (lane == 0) {
            st_volatile_s32(xh->tg + static_cast<uint32_t>((xh->w * 2 + slot) * 8), cur.t);
            st_volatile_s32(xh->tg + static_cast<uint32_t>((xh->w * 2 + slot) * 8 + 4), cur.g);
        }
        __syncwarp();
        mbar_arrive(xh->bar + static_cast<uint32_t>((xh->w * 2 + slot) * 8));
        return;
    }
    const int64_t pc = P.pcols;
    float *mine = P.partials + ((worker * 2 + slot) * pc + j0) * 32;
#pragma unroll
    for (int j = 0; j < NCW; ++j) mine[j * 32 + lane] = v[j];
    if (gated) {
#pragma unroll
        for (int j = 0; j < NCW; ++j) mine[(NC + j) * 32 + lane] = gv[j];
    }
    const int last = kSplit * static_cast<int>(w2 - w1 + 1) - 1;
    int old = 0;
    if (local) {
        __threadfence_block();
        __syncwarp();
        if (lane == 0) old = atomicAdd(&cta_cnt[w1 - cta_w0], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != last) return;  // not the last contributor
        __threadfence_block();
    } else {
        __syncwarp();
        if (lane == 0) old = atom_add_acqrel_gpu(&P.counters[T.rg_base + cur.g], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != last) return;
        __syncwarp();
    }
    float tot[NC], gtot[NC];
#pragma unroll
    for (int j = 0; j < NC; ++j) tot[j] = gtot[j] = 0.0f;
    for (int64_t w = w1; w <= w2; ++w) {
        const float *src = P.partials + ((w * 2 + (w == w1 ? 1 : 0)) * pc) * 32;
#pragma unroll
        for (int j = 0; j < NC; ++j) tot[j] += ldcg_f32(src + j * 32 + lane);
        if (gated) {
#pragma unroll
            for (int j = 0; j < NC; ++j) gtot[j] += ldcg_f32(src + (NC + j) * 32 + lane);
        }
    }
    if (!DUMP && valid) {
#pragma unroll
        for (int j = 0; j < NC; ++j) store_final<EPI>(P, O, j, row, tot[j], gtot[j]);
    }
    if (valid2) {
#pragma unroll
        for (int j = 0; j < NC; ++j) store_out(P, O, j, row + 32, gtot[j]);
    }
    if (lane == 0) {
        if (local)
            cta_cnt[w1 - cta_w0] = 0;
        else
            st_relaxed_gpu(&P.counters[T.rg_base + cur.g], 0);
    }
}

// The same from a warp's running sums (Q6_K: fp64, the four lanes of a row
// -- lane & 7 -- holding two super-blocks each).
template <int NCW, int NC, int MODE>
__device__ __forceinline__ void flush_group(const GemvParams &P, const AtomCursor &cur, const RowAcc<NCW> &acc,
                                            const RowAcc<NCW> &gacc, const RowAccD<NCW> &dacc, int64_t worker,
                                            int64_t a0, int64_t a1,
                                            int lane, int j0, int64_t cta_w0, int64_t cta_w1, int *cta_cnt,
                                            const XHelp *xh = nullptr) {
    constexpr bool Q6 = MODE == kModeQ6;
    float v[NCW], gv[NCW];
#pragma unroll
    for (int j = 0; j < NCW; ++j) {
        v[j] = acc.value(j);
        gv[j] = Q6 ? 0.0f : gacc.value(j);
        if constexpr (Q6) {
            double t = dacc.s[j];
            t += __shfl_xor_sync(0xffffffffu, t, 8);
            t += __shfl_xor_sync(0xffffffffu, t, 16);
            v[j] = static_cast<float>(t);
        }
    }
    flush_values<NCW, NC, MODE>(P, cur, v, gv, worker, a0, a1, lane, j0, cta_w0, cta_w1, cta_cnt, xh);
}

// Per-warp pipeline state of one worker.
struct WorkerPipe {
    int64_t a0, a1;
    int n;
    bool back;                  // walks its range from a1 - 1 down to a0
    uint32_t ring;
    AtomCursor icur;            // next atom to issue
    AtomCursor pro[kStages];    // the prologue atoms
};

// Issue the weight copies of the first kStages atoms (they do not depend on
// any earlier grid: the weights are read-only).
// (A column-split partner only follows the cursors: issue == false.)
template <int NC, int MODE>
// In the single-launch mode only the first stage is issued here; the others
// follow once the CTA's activation loads are in flight (issue_rest_prologue),
// so that a CTA starting after the previous grid has completed does not queue
// its activations behind a whole ring of weights.
__device__ __forceinline__ void worker_prologue(const GemvParams &P, WorkerPipe &W, int lane,
                                                const uint32_t (&bar)[kStages], bool issue) {
    constexpr int kSB = Stage<NC, MODE>::kBytes;
    constexpr int kNow = MODE == kModeActSmem ? 1 : kStages;
    W.icur = locate_atom(P, W.back ? W.a1 - 1 : W.a0);
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
        W.pro[s] = W.icur;
        if (s < W.n) {
            if (issue && s < kNow) issue_weights<NC, MODE>(P, W.icur, W.ring + s * kSB, bar[s], lane);
            if (s + 1 < W.n) step(P, W.icur, W.back);
        }
    }
}

template <int NC, int MODE>
__device__ __forceinline__ void issue_rest_prologue(const GemvParams &P, const WorkerPipe &W, int lane,
                                                    const uint32_t (&bar)[kStages]) {
    constexpr int kSB = Stage<NC, MODE>::kBytes;
#pragma unroll
    for (int s = 1; s < kStages; ++s)
        if (s < W.n) issue_weights<NC, MODE>(P, W.pro[s], W.ring + s * kSB, bar[s], lane);
}

// Start-up: touch every kernel-parameter line the prologue and the plan read
// (one thread per task, in parallel), and ask for the tasks' tensor maps, so
// that the walk over the task table that follows does not take one
// constant-cache miss after another.
__device__ __forceinline__ void warm_params(const GemvParams &P) {
    const int t = threadIdx.x;
    uint64_t v = 0;
    if (t < P.ntasks) {
        const TaskDesc &T = P.task[t];
        v = reinterpret_cast<uint64_t>(T.W) ^ static_cast<uint64_t>(T.atom_base) ^
            static_cast<uint64_t>(T.bias_col_stride) ^ static_cast<uint64_t>(T.apr);
        asm volatile("prefetch.tensormap [%0];" ::"l"(&P.tmap[t]) : "memory");
        if (T.has_gate) asm volatile("prefetch.tensormap [%0];" ::"l"(&P.tmap_gate[T.gate_map]) : "memory");
    } else if (t == 32) {
        v = static_cast<uint64_t>(P.natoms) ^ static_cast<uint64_t>(P.nworkers) ^
            static_cast<uint64_t>(P.act_nb[0]) ^ static_cast<uint64_t>(P.cta_act_mask[blockIdx.x % kMaxPlanCtas]);
    }
    asm volatile("" ::"l"(v));  // keep the loads
}

// The rest of one worker's range, once the activations are ready: stream its
// atoms through the ring and flush its row groups.  The issuer warp (the only
// one unless the columns are split) owns the copies; with a split it refills
// a stage only after both warps have released it (empty barrier, two
// arrivals).  Returns (never exits the kernel) so that the CTA-wide epilogues
// can still run.
template <int NC, int NCW, int MODE>
__device__ __forceinline__ void worker_main(const GemvParams &P, WorkerPipe &W, int64_t worker, int lane, int j0,
                                            bool issuer, const uint32_t (&full)[kStages],
                                            const uint32_t (&empty)[kStages], int64_t cta_w0, int64_t cta_w1,
                                            int *cta_cnt, const ActView &AV, const XHelp *xh) {
    constexpr int kSB = Stage<NC, MODE>::kBytes;
    constexpr bool kShared = split_for(NC) > 1;
    const int n = W.n;
    const uint32_t ring = W.ring;
    AtomCursor icur = W.icur;
    if (issuer) {
#pragma unroll
        for (int s = 0; s < kStages; ++s)
            if (s < n) issue_acts<NC, MODE>(P, W.pro[s], ring + s * kSB, full[s], lane);
    }

    // Sums of the open row group: main and gate (gated launches), or rows
    // 64g + lane and 64g + 32 + lane (two-row launches).
    RowAcc<NCW> acc, gacc;
    RowAccD<NCW> dacc;  // Q6_K launches
    acc.clear();
    if constexpr (MODE != kModeQ6) gacc.clear();
    if constexpr (MODE == kModeQ6) dacc.clear();
    AtomCursor cur = W.pro[0];
    int open_t = -1, open_g = -1;

    for (int i = 0; i < n; ++i) {
        const int s = i % kStages;
        const uint32_t parity = static_cast<uint32_t>((i / kStages) & 1);
        if (cur.t != open_t || cur.g != open_g) {
            if (open_t >= 0) {
                AtomCursor o{open_t, open_g, 0};
                flush_group<NCW, NC, MODE>(P, o, acc, gacc, dacc, worker, W.a0, W.a1, lane, j0, cta_w0, cta_w1,
                                           cta_cnt, xh);
            }
            open_t = cur.t;
            open_g = cur.g;
            acc.clear();
            if constexpr (MODE != kModeQ6) gacc.clear();
            if constexpr (MODE == kModeQ6) dacc.clear();
        }
        bool ok = wait_phase(full[s], parity, kWaitLimitNs);
        if (ok) {
            compute_atom<NCW, NC, MODE>(P, cur, ring + s * kSB, lane, j0, acc, gacc, dacc, AV);
            __syncwarp();
            if constexpr (kShared) {
                if (lane == 0) mbar_arrive(empty[s]);
            }
            if (issuer && i + kStages < n) {
                if constexpr (kShared) ok = wait_phase(empty[s], parity, kWaitLimitNs);
                if (ok) {
                    fence_proxy_async_smem();
                    issue_weights<NC, MODE>(P, icur, ring + s * kSB, full[s], lane);
                    issue_acts<NC, MODE>(P, icur, ring + s * kSB, full[s], lane);
                    if (i + kStages + 1 < n) step(P, icur, W.back);
                }
            }
        }
        if (!ok) {
            if (lane == 0) atomicExch(P.status, kStatusTimeout);
            // The issuer lets its other copies in flight land (bounded) before leaving.
            if (issuer) {
                for (int k = 1; k < kStages; ++k) {
                    const int ii = i + k;
                    if (ii < n)
                        wait_phase(full[ii % kStages], static_cast<uint32_t>((ii / kStages) & 1), kDrainLimitNs);
                }
            }
            return;
        }
        if (i + 1 < n) step(P, cur, W.back);
    }
    if (open_t >= 0) {
        // the last group: this warp is done, so it does its own hand-off
        // (handing it over would only serialise it behind the boundary warp)
        AtomCursor o{open_t, open_g, 0};
        flush_group<NCW, NC, MODE>(P, o, acc, gacc, dacc, worker, W.a0, W.a1, lane, j0, cta_w0, cta_w1,
                                   cta_cnt, nullptr);
    }
}

// ---- single-launch mode: activations quantized into shared memory ----------
// Which distinct activations a CTA's atoms read, and where their q8a records
// go in its shared memory.  The host sizes the region with the same rule
// (act_smem_need in the C ABI), so both agree on every CTA's need.
struct ActPlan {
    int n;                     // activations this CTA needs
    int act[kMaxTasks];        // their ids, increasing
    int off[kMaxTasks];        // byte offset of each in the region
    int blk0[kMaxTasks + 1];   // prefix sums of their q8_1 blocks (ncols * nb * 8 each)
    int task_off[kMaxTasks];   // per task: offset of its activation (-1: not needed)
    int bytes;                 // region bytes used
};

// Task holding global atom a (a < natoms).
__device__ __forceinline__ int task_of_atom(const GemvParams &P, int64_t a) {
    int t = 0;
    while (t + 1 < P.ntasks && a >= P.task[t + 1].atom_base) ++t;
    return t;
}

// Laid out by lane 0 of one warp from the host's tables: the CTA's bit set of
// activations (cta_act_mask, the same rule as act_smem_need in the C ABI:
// the tasks its workers' atom ranges span), their super-block counts and the
// tasks' activation ids -- a few parameter lines, read once.
template <int NC>
__device__ void act_plan_cta(const GemvParams &P, ActPlan &A) {
    const uint32_t mask = P.cta_act_mask[blockIdx.x];
    int nb[kMaxTasks], ta[kMaxTasks];
#pragma unroll
    for (int a = 0; a < kMaxTasks; ++a) {
        nb[a] = P.act_nb[a];
        ta[a] = P.task_act[a];
    }
    int off = 0, n = 0, blk = 0;
    int off_of[kMaxTasks];
    A.blk0[0] = 0;
#pragma unroll
    for (int a = 0; a < kMaxTasks; ++a) {
        off_of[a] = -1;
        if (!((mask >> a) & 1u)) continue;
        A.act[n] = a;
        A.off[n] = off;
        off_of[a] = off;
        off += NC * nb[a] * kActSBBytes;
        blk += NC * nb[a] * 8;
        A.blk0[++n] = blk;
    }
    A.n = n;
    A.bytes = off;
#pragma unroll
    for (int t = 0; t < kMaxTasks; ++t) A.task_off[t] = ta[t] >= 0 ? off_of[ta[t]] : -1;
}

__device__ __forceinline__ float rcp_approx_ftz(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// 32 bytes (one L2 sector) from a 32-byte aligned address, cached in L2 only.
__device__ __forceinline__ void ldg_cg_f8(const float *p, float (&v)[8]) {
    asm volatile("ld.global.cg.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
                 : "l"(p));
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// One half of a q8_1 block per lane: lanes 2i and 2i+1 take values [0, 16)
// and [16, 32) of a block (32-byte aligned: each lane reads two whole L2
// sectors, so every sector is requested once per CTA) and write them into its q8a
// record slot (sub-block s of the record at rec).  Semantics of
// quantize_value / write_q8a, bit for bit: d = amax/127 (IEEE division),
// q = amax == 0 ? 0 : roundf(x/d), d8 = float(half(d)), T = sum of q.
// The quotient x/d is formed as t = x * r with r ~ 1/d (approximate
// reciprocal plus one Newton step, so |t - x/d| < 2^-15 for |x/d| <= 127.x):
// where t is not within 2^-14 of a half-integer, x/d rounded to nearest lies
// on the same side of every half-integer as t, so roundf(x/d) = rint(t),
// formed with the 1.5 * 2^23 addition (the integer lands in the low mantissa
// bits; its low byte is the int8 quant).  The loop over the values has no
// branch (so their chains interleave); values near a half-integer (about 1
// in 8000), or whose scale is zero or subnormal, are marked and recomputed
// with the IEEE division afterwards.  Both lanes of a pair must execute this
// (the amax and T exchanges); store = false computes without writing.
template <typename F>
__device__ __forceinline__ void quantize_half_block(const float *src, uint32_t rec, int s, int half, bool store,
                                                    bool first, F &&after_loads) {
    float v[16], v1[8];
    ldg_cg_f8(src, reinterpret_cast<float(&)[8]>(v[0]));
    ldg_cg_f8(src + 8, v1);
    if (first) after_loads();
#pragma unroll
    for (int i = 0; i < 8; ++i) v[8 + i] = v1[i];
    float m8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m8[i] = fmaxf(fabsf(v[i]), fabsf(v[i + 8]));
#pragma unroll
    for (int i = 0; i < 4; ++i) m8[i] = fmaxf(m8[i], m8[i + 4]);
    float amax = fmaxf(fmaxf(m8[0], m8[2]), fmaxf(m8[1], m8[3]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    const float d = amax / 127.0f;  // IEEE division (no fast-math in this build)
    const __half dh = __float2half_rn(d);
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    int T = 0;
    if (amax != 0.0f) {
        float r = rcp_approx_ftz(d);
        r = __fmaf_rn(__fmaf_rn(-d, r, 1.0f), r, r);
        constexpr float kMagic = 12582912.0f;               // 1.5 * 2^23
        constexpr float kNearTie = 0.5f - 6.103515625e-05f;  // 0.5 - 2^-14
        uint32_t qb[16];
        uint32_t redo = 0u;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float t = __fmul_rn(v[i], r);
            const float m = __fadd_rn(t, kMagic);
            const float rt = __fsub_rn(m, kMagic);
            qb[i] = __float_as_uint(m);  // low byte: rint(t) as int8
            redo |= (fabsf(__fsub_rn(t, rt)) < kNearTie ? 0u : 1u) << i;
        }
        if (redo != 0u) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if ((redo >> i) & 1u) qb[i] = static_cast<uint32_t>(static_cast<int>(roundf(v[i] / d)));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            w[k] = __byte_perm(__byte_perm(qb[4 * k], qb[4 * k + 1], 0x0040u),
                               __byte_perm(qb[4 * k + 2], qb[4 * k + 3], 0x0040u), 0x5410u);
            T = dp4a_ss(w[k], 0x01010101u, T);
        }
    }
    T += __shfl_xor_sync(0xffffffffu, T, 1);
    if (!store) return;
    sts128(rec + 32 * s + 16 * half, w[0], w[1], w[2], w[3]);
    if (half == 0) {
        const float d8 = __half2float(dh);
        const uint32_t meta = rec + kActMetaOff + 16 * (s >> 1) + 4 * (s & 1);
        sts32f(meta, (s & 1) ? d8 * 0.0625f : d8);
        sts32f(meta + 8, d8 * static_cast<float>(T));
    }
}

// All q8_1 blocks of the CTA's activations, half a block per lane, every
// warp of the CTA: lane l of warp w takes half-block (w + k * warps) * 32 + l.
// after_loads() runs once per warp, right after the warp's first loads are
// issued (or at once if it has none).
template <int NC, typename F>
__device__ __forceinline__ void quantize_acts_smem(const GemvParams &P, const ActPlan &A, uint32_t base,
                                                   F &&after_loads) {
    const int lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int total = 2 * A.blk0[A.n];  // half-blocks (even)
    bool pending = true;
    for (int chunk = threadIdx.x >> 5; chunk * 32 < total; chunk += nwarps) {
        const int gh0 = chunk * 32 + lane;
        const bool store = gh0 < total;
        const int gh = store ? gh0 : total - 2 + (lane & 1);  // pairs stay pairs
        const int gb = gh >> 1;
        int i = 0;
        while (gb >= A.blk0[i + 1]) ++i;
        const int a = A.act[i];
        const int nb = P.act_nb[a];
        const int nbl = nb * 8;
        const int rem = gb - A.blk0[i];
        const int j = rem / nbl;
        const int b = rem - j * nbl;
        const uint32_t rec = base + static_cast<uint32_t>(A.off[i] + (j * nb + (b >> 3)) * kActSBBytes);
        quantize_half_block(P.act_x[a] + j * P.act_xcs[a] + b * 32 + 16 * (gh & 1), rec, b & 7, gh & 1, store,
                            pending, after_loads);
        pending = false;
    }
    if (pending) after_loads();
}

// Fused all-gather epilogue (producer side): after every CTA of this grid has
// stored its outputs (locally and into the peers' buffers), the last CTA to
// finish publishes epoch+1 in each peer's flag word for this rank and exits;
// it does not wait for the peers.  A consumer of the gathered buffer waits
// for every peer's flag to reach this rank's epoch (gather_wait_flags: the
// next gathering call's quantization step, or q4k_gather_wait).  The epoch
// word persists across calls, so replays of a captured sequence keep counting.
// Ordering: each CTA's peer stores -> block barrier -> release fence (system
// scope) -> arrival count; the last CTA's acquire fence -> per-peer release
// stores of the flag (one lane per peer) -> the consumer's acquire loads.
// The last CTA also returns the arrival count to 0 for the next launch.
__device__ __forceinline__ void gather_epilogue(const GemvParams &P) {
    __shared__ int last_cta;
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();
        last_cta = atomicAdd(P.gdone, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last_cta || threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    if (lane == 0) fence_acq_rel_sys();
    __syncwarp();
    const uint32_t e = *reinterpret_cast<volatile uint32_t *>(P.gepoch) + 1u;
    if (lane < P.gworld && lane != P.grank) st_release_sys_u32(P.gflags_peer[lane] + P.grank, e);
    if (lane == 0) {
        *reinterpret_cast<volatile uint32_t *>(P.gepoch) = e;
        *reinterpret_cast<volatile uint32_t *>(P.gdone) = 0u;  // ready for the next launch
    }
}

// Per-warp static partition (every launch without a fused task): worker w
// (one warp) owns atoms [natoms * w / nworkers, natoms * (w + 1) / nworkers)
// and streams them through its own ring; a row group split between workers
// is added up by its last contributor (flush_group).
template <int NC, int MODE>
__device__ __forceinline__ void gemv_per_warp(const GemvParams &P) {
    constexpr bool DUMP = MODE == kModeDump;
    constexpr int kR = rings_m(NC, MODE);
    constexpr int kSplit = split_for(NC);
    constexpr int kNC0 = (NC + kSplit - 1) / kSplit;  // columns of the issuer warp
    constexpr int kSB = Stage<NC, MODE>::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bars[kR][kStages];
    __shared__ __align__(8) uint64_t empty_bars[kR][kStages];
    __shared__ int cta_cnt[kR];  // arrivals at row groups split between this CTA's workers
    constexpr bool ASM = MODE == kModeActSmem;
    __shared__ ActPlan act_plan[1];  // single-launch mode only
    __shared__ int plan_ok;
    // plain and single-launch kernels: warp kR is the boundary warp (row
    // groups split with another CTA, XHelp); its entries' values follow the
    // rings in dynamic shared memory
    constexpr bool XH = has_xhelp(MODE);
    static_assert(!XH || kSplit == 1, "boundary-warp entries are per ring: one warp per ring");
    constexpr int kXH = XH ? kR : 1;
    __shared__ int xh_tg[kXH][2][2];
    __shared__ __align__(8) uint64_t xh_bar[kXH][2];

#if Q4K_TIMELINE
    const uint64_t tl_start = globaltimer_ns();
#endif
    // The next launch on the stream may start now; it waits for this grid's
    // completion before it touches the workspace.
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int rid = warp / kSplit;           // ring = worker slot in this CTA
    if constexpr (MODE == kModeActSmem) warm_params(P);
    const int half = warp - rid * kSplit;    // 0: issuer, columns [0, kNC0); 1: columns [kNC0, NC)
    if (threadIdx.x < kR) {
        cta_cnt[threadIdx.x] = 0;
        if constexpr (XH) {
            mbar_init(smem_addr(&xh_bar[threadIdx.x][0]), 32);
            mbar_init(smem_addr(&xh_bar[threadIdx.x][1]), 32);
        }
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_addr(&full_bars[threadIdx.x][s]), 1);
            mbar_init(smem_addr(&empty_bars[threadIdx.x][s]), kSplit);
        }
        mbar_fence_init();
    }
    __syncthreads();
    // Large problems: CTA-contiguous worker ranges (most split row groups stay
    // inside a CTA).  Small ones: consecutive workers on different SMs.
    const int64_t worker = P.packed ? static_cast<int64_t>(blockIdx.x) * kR + rid
                                    : static_cast<int64_t>(rid) * gridDim.x + blockIdx.x;
    const int64_t cta_w0 = static_cast<int64_t>(blockIdx.x) * kR;
    const int64_t cta_w1 = cta_w0 + kR - 1;
    const bool active = rid < kR && worker < P.nworkers;  // (warp kR: the boundary warp)
    const bool issuer = half == 0;
    uint32_t full[kStages], empty[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
        full[s] = smem_addr(&full_bars[rid < kR ? rid : 0][s]);
        empty[s] = smem_addr(&empty_bars[rid < kR ? rid : 0][s]);
    }
    WorkerPipe W;
    if (active) {
        W.a0 = worker_begin(P, worker);
        W.a1 = worker_begin(P, worker + 1);
        W.n = static_cast<int>(W.a1 - W.a0);
        W.back = walks_back(worker);
        W.ring = smem_addr(smem) + static_cast<uint32_t>(rid * kStages * kSB);
    }
    // Weights stream while the previous grid on the stream (the prep launch,
    // or the previous single-launch GEMV) finishes; griddepcontrol.wait
    // returns once it has completed.
    if (active) worker_prologue<NC, MODE>(P, W, lane, full, issuer);
    if constexpr (ASM) {
        // this CTA's activation table (after the weight copies are out); a
        // plan the region cannot hold (the host sizes it with the same rule)
        // is refused, never overrun
        if (threadIdx.x == 0) {
            act_plan_cta<NC>(P, act_plan[0]);
            plan_ok = blockIdx.x < kMaxPlanCtas && act_plan[0].bytes <= P.act_smem_bytes;
            // Ask L2 for the activation columns while the previous grid runs: a
            // prefetch binds no value (if that grid writes x, the loads after
            // the wait still see its stores; L2 is the point of coherence).
            const uint64_t pol = l2_evict_last_policy();
            const ActPlan &A = act_plan[0];
            for (int i = 0; i < A.n; ++i) {
                const int a = A.act[i];
                for (int j = 0; j < NC; ++j)
                    bulk_prefetch_l2(P.act_x[a] + j * P.act_xcs[a], static_cast<uint32_t>(P.act_nb[a]) * kQK * 4u,
                                     pol);
            }
        }
    }
#if Q4K_TIMELINE
    const uint64_t tl_plan = globaltimer_ns();
#endif
    pdl_wait();
#if Q4K_TIMELINE
    const uint64_t tl_wait = globaltimer_ns();
#endif
    const uint32_t xh_vals = smem_addr(smem) + static_cast<uint32_t>(kR * kStages * kSB);
    // (the single-launch activation table follows the boundary warp's entries)
    const ActView AV{xh_vals + static_cast<uint32_t>(xh_bytes(NC, MODE)), ASM ? act_plan[0].task_off : nullptr};
#if Q4K_TIMELINE
    uint64_t tl_d[3] = {0, 0, 0};  // single-launch mode: after the plan barrier, before / after quantizing
#endif
    if constexpr (ASM) {
        // Single launch: the activations are read after the previous grid on
        // the stream has completed (it may have written them), quantized by
        // every warp of the CTA into its activation table, then used by all.
        __syncthreads();  // the plan
#if Q4K_TIMELINE
        tl_d[0] = globaltimer_ns();
#endif
        if (!plan_ok) {
            if (threadIdx.x == 0) atomicExch(P.status, kStatusBadPlan);
            // let this warp's weight copy (the first stage only, so far) land
            // (bounded) before leaving
            if (active && issuer && W.n > 0) wait_phase(full[0], 0u, kDrainLimitNs);
            return;
        }
        if (threadIdx.x == 0 && blockIdx.x == 0) *P.status = kStatusOk;
        if (P.gworld > 1) {
            if (threadIdx.x == 0) gather_wait_flags(P.gwait);  // x may be a gathered output
            __syncthreads();
        }
#if Q4K_TIMELINE
        tl_d[1] = globaltimer_ns();
#endif
        quantize_acts_smem<NC>(P, act_plan[0], AV.base, [&]() {
            if (active && issuer) issue_rest_prologue<NC, MODE>(P, W, lane, full);
        });
#if Q4K_TIMELINE
        tl_d[2] = globaltimer_ns();
#endif
        __syncthreads();
    }
#if Q4K_TIMELINE
    const uint64_t tl_quant = globaltimer_ns();
#endif
    const XHelp xh{xh_vals, smem_addr(&xh_bar[0][0]), smem_addr(&xh_tg[0][0][0]), rid};
    if (active) {
        if (issuer) {
            worker_main<NC, kNC0, MODE>(P, W, worker, lane, 0, true, full, empty, cta_w0, cta_w1, cta_cnt, AV,
                                        XH ? &xh : nullptr);
        } else if constexpr (kSplit > 1) {
            worker_main<NC, NC - kNC0, MODE>(P, W, worker, lane, kNC0, false, full, empty, cta_w0, cta_w1,
                                             cta_cnt, AV, XH ? &xh : nullptr);
        }
    }
    if constexpr (XH) {
        static_assert(2 * kR <= 32, "one lane of the boundary warp per entry");
        if (rid == kR) {
            // The boundary warp.  Lane L < 2 kR stands for entry (ring L / 2,
            // slot L % 2): whether that compute warp hands over a split group
            // in that slot (from its atom range, as flush_values decides), and
            // after how many of its atoms it does so (the order to wait in).
            bool expect = false;
            int key = 0;
            if (lane < 2 * kR) {
                const int w = lane >> 1, e = lane & 1;
                const int64_t wk = P.packed ? static_cast<int64_t>(blockIdx.x) * kR + w
                                            : static_cast<int64_t>(w) * gridDim.x + blockIdx.x;
                const int64_t a0 = wk < P.nworkers ? worker_begin(P, wk) : 0;
                const int64_t a1 = wk < P.nworkers ? worker_begin(P, wk + 1) : 0;
                if (a1 > a0) {
                    const bool back = walks_back(wk);
                    // slot 0: the group holding a0, if it began before a0;
                    // slot 1: the group holding a1 - 1, if it begins at or
                    // after a0 and ends after a1
                    const AtomCursor c = locate_atom(P, e == 0 ? a0 : a1 - 1);
                    const TaskDesc &T = P.task[c.t];
                    const int64_t sg = T.atom_base + static_cast<int64_t>(c.g) * T.apr, eg = sg + T.apr;
                    const bool split = e == 0 ? sg < a0 : (sg >= a0 && eg > a1);
                    // handed over only before the warp's last atom (its last
                    // group it flushes itself)
                    const int64_t at = e == 0 ? (back ? a1 - a0 : (eg < a1 ? eg : a1) - a0)
                                              : (back ? a1 - sg : a1 - a0);
                    if (split && at < a1 - a0) {
                        const int64_t w1 = worker_of(P, sg), w2 = worker_of(P, eg - 1);
                        expect = !(P.packed && w1 >= cta_w0 && w2 <= cta_w1);
                        key = static_cast<int>(at);
                    }
                }
            }
            uint32_t pend = __ballot_sync(0xffffffffu, expect);
            bool ok = true;
            while (pend != 0u) {
                const bool mine = (pend >> lane) & 1u;
                const int kmin = static_cast<int>(__reduce_min_sync(0xffffffffu, mine ? static_cast<unsigned>(key)
                                                                                      : 0x7fffffffu));
                const int b = __ffs(static_cast<int>(__ballot_sync(0xffffffffu, mine && key == kmin))) - 1;
                pend &= ~(1u << b);
                const int w = b >> 1, e = b & 1;
                if (!wait_phase(smem_addr(&xh_bar[w][e]), 0u, kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                float v[NC], gv[NC];
#pragma unroll
                for (int j = 0; j < NC; ++j) {
                    v[j] = lds32f(xh_vals + static_cast<uint32_t>(((w * 2 + e) * NC + j) * 128 + lane * 4));
                    gv[j] = 0.0f;
                }
                const AtomCursor cur{ld_volatile_s32(smem_addr(&xh_tg[w][e][0])),
                                     ld_volatile_s32(smem_addr(&xh_tg[w][e][1])), 0};
                const int64_t wk = P.packed ? static_cast<int64_t>(blockIdx.x) * kR + w
                                            : static_cast<int64_t>(w) * gridDim.x + blockIdx.x;
                flush_values<NC, NC, MODE>(P, cur, v, gv, wk, worker_begin(P, wk), worker_begin(P, wk + 1), lane, 0,
                                           cta_w0, cta_w1, cta_cnt);
            }
            if (!ok && lane == 0) atomicExch(P.status, kStatusTimeout);
        }
    }
#if Q4K_TIMELINE
    // (the boundary warp: record 14, word 3 = 0)
    const int rec = rid < kR ? warp : 14;
    if (lane == 0 && P.tl != nullptr && blockIdx.x < Q4K_TIMELINE_CTAS && warp < 16) {
        unsigned long long *o =
            P.tl + ((static_cast<int64_t>(P.tl_slot) * Q4K_TIMELINE_CTAS + blockIdx.x) * 16 + rec) * 8;
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        o[0] = tl_start;
        o[1] = tl_wait;
        o[2] = globaltimer_ns();
        o[3] = active ? static_cast<unsigned long long>(W.n) : 0ull;
        o[4] = smid;
        o[5] = static_cast<unsigned long long>(worker);
        // single-launch mode: when the activation table was planned and when
        // its quantization ended; else the worker's atom range
        o[6] = ASM ? tl_quant : active ? static_cast<unsigned long long>(W.a0) : 0ull;
        o[7] = ASM ? tl_plan : active ? static_cast<unsigned long long>(W.a1) : 0ull;
        if (ASM && warp < 6) {
            // the phases of the quantization, in the record of warp + 8 (word 3
            // stays 0: not a worker record; records 14 and 15 stay free)
            unsigned long long *d = o + 8 * 8;
            d[0] = tl_d[0];
            d[1] = tl_d[1];
            d[2] = tl_d[2];
            d[3] = 0;
        }
    }
#endif
    if (!DUMP && P.gworld > 1) gather_epilogue(P);
}

// ---- launches with a fused task: per-CTA atom queue, fold and flush warps ----
// kModeGated (a task with a bias or a fused gate; a gated task's row group
// runs over its main matrix, then its gate matrix).  CTA c of G owns the
// contiguous atom range [natoms*c/G, natoms*(c+1)/G) (walk order below).  Its
// R compute warps take the range's atoms one at a time, in walk order, from
// a shared-memory counter, each streaming them through its own kStages-deep
// ring, so the warps of a CTA finish within about one atom of each other.  A
// compute warp leaves the sums of the k-th atom of the walk (NC floats per
// lane) in result slot k % S (S = q_slots); warp R folds the slots in walk
// order into the row groups' compensated sums (the gate's apart) and hands
// each completed group to warp R + 1, which applies the biases and the gate
// epilogue and writes the rows, or deposits the CTA's share of a group that
// spans CTAs (added up by the last CTA to arrive, in CTA order).  The result
// does not depend on which warp computed which atom, and the epilogue code
// stays out of the compute warps' instruction stream (inlined into the
// per-warp kernel it measured 2-8 % slower on every launch).
//
// Slot hand-off through shared-memory words (cheaper than mbarrier phases
// here, where every atom takes one each way): tag[s] = k + 1 once slot s
// holds atom k (stored with release by lane 0 of the writing warp, after the
// warp's stores and a warp barrier; the folding warp reads the tags of up to
// 32 slots at once with acquire loads), and fold_done = the atoms folded so
// far (published by the folding warp once it has used the values it loaded).
// Atom k is written once atom k - S has been folded; the warp that holds the
// lowest atom not yet folded can always write it, so the fold always
// advances.  Every wait is bounded (Q4K_ETIMEOUT in the status word) and
// backs off with nanosleep, so that waiting warps leave the issue slots to
// the others.

// Sums of one atom per lane: NC floats (the lane's row, the atom's
// super-blocks added in fp32).  Rows past the matrix end give 0.
template <int NC, int MODE>
__device__ __forceinline__ void atom_sums(const GemvParams &P, const AtomCursor &c, uint32_t stage, int lane,
                                          float (&r)[NC]) {
#pragma unroll
    for (int q = 0; q < NC; ++q) r[q] = 0.0f;
    const TaskDesc &T = P.task[c.t];
    const int rows = min(32, T.nrows - c.g * 32);
    if (lane >= rows) return;
    // a gated task's second half of atoms: the gate matrix (folded apart)
    const bool second = T.has_gate && c.kp >= T.half;
    const int kb0 = (second ? c.kp - T.half : c.kp) * kKS;
    const uint32_t act = stage + Stage<NC, MODE>::kActOff;
    const int nsb = min(kKS, T.nb - kb0);
#pragma unroll
    for (int i = 0; i < kKS; ++i) {
        if (i < nsb) {
            uint64_t sb[NC];
#pragma unroll
            for (int j = 0; j < NC; ++j) sb[j] = 0ull;
            sb_dot<NC, false>(stage + i * kBoxBytes + lane * kPitch, act + i * kActSBBytes, q_col_pitch(MODE), sb,
                              nullptr, 0);
#pragma unroll
            for (int j = 0; j < NC; ++j) {
                const float2 v = f2_unpack(sb[j]);
                r[j] += v.x + v.y;
            }
        }
    }
}


template <int NC, int MODE>
__device__ __forceinline__ void gemv_queue(const GemvParams &P) {
    static_assert(MODE == kModeGated, "the queue kernel serves the launches with a fused task");
    constexpr int kR = rings_m(NC, MODE);  // compute warps; warp kR folds, warp kR + 1 flushes
    constexpr int kSB = Stage<NC, MODE>::kBytes;
    constexpr int kQ = NC;  // floats per lane and atom
    constexpr int kSlotB = q_slot_bytes(NC, MODE);
    constexpr int kS = q_slots(NC, MODE);
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bars[kR][kStages];
    __shared__ int slot_tag[kS];
    __shared__ int fold_done;
    __shared__ int claim_next;
    // group ring (fold -> flush): entry e % kGroupRing holds the e-th group
    // of the walk once gr_tag == e + 1; gr_taken: groups flushed; gr_total:
    // groups sent in all (-1 until the fold ends)
    __shared__ int gr_tag[kGroupRing], gr_t[kGroupRing], gr_g[kGroupRing];
    __shared__ int gr_taken, gr_total;

#if Q4K_TIMELINE
    const uint64_t tl_start = globaltimer_ns();
#endif
    // The next launch on the stream may start now; it waits for this grid's
    // completion before it touches the workspace.
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const bool folder = warp == kR;
    const bool flusher = warp == kR + 1;
    const bool computes = warp < kR;
    if (threadIdx.x < kR) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) mbar_init(smem_addr(&full_bars[threadIdx.x][s]), 1);
        mbar_fence_init();
    } else if (folder) {
        for (int i = lane; i < kS; i += 32) slot_tag[i] = 0;
        if (lane < kGroupRing) gr_tag[lane] = 0;
    }
    if (threadIdx.x == 0) {
        claim_next = 0;
        fold_done = 0;
        gr_taken = 0;
        gr_total = -1;
    }
    __syncthreads();
    // (CTAs past nworkers have no atoms: nworkers <= natoms keeps every
    // unit of the partition non-empty)
    const bool active = blockIdx.x < P.nworkers;
    const int64_t A0 = active ? worker_begin(P, blockIdx.x) : 0;
    const int64_t A1 = active ? worker_begin(P, blockIdx.x + 1) : 0;
    const int n = static_cast<int>(A1 - A0);
    // The walk, in three pieces: [A0, e1), the range's part of a row group
    // that began in the previous CTA's range; [s2, A1), its part of a group
    // that continues into the next CTA's range; then [e1, s2), the groups
    // of its own.  Both contributors of a group shared by two CTAs reach it
    // among their first atoms, so its cross-CTA hand-off overlaps the rest
    // of the work (and both read the L2 lines they share at about the same
    // time), and the walk ends on a group of its own where it has one.
    int64_t e1 = A0, s2 = A1;
    if (n > 0) {
        const AtomCursor b = locate_atom(P, A0);
        if (b.kp > 0) e1 = min(A1, A0 - b.kp + P.task[b.t].apr);
        const AtomCursor e = locate_atom(P, A1 - 1);
        const int64_t gs = A1 - 1 - e.kp;
        if (e.kp + 1 < P.task[e.t].apr && gs >= e1) s2 = gs;
    }
    const int len1 = static_cast<int>(e1 - A0), len2 = static_cast<int>(A1 - s2);
    const uint32_t ring = smem_addr(smem) + static_cast<uint32_t>((computes ? warp : 0) * kStages * kSB);
    const uint32_t slots = smem_addr(smem) + static_cast<uint32_t>(kR * kStages * kSB);
    const uint32_t fullb = smem_addr(&full_bars[computes ? warp : 0][0]);  // stage s: fullb + 8 s
    // The k-th atom of this CTA's walk, and the next claim (-1: none left).
    auto atom_of = [&](int k) -> int64_t {
        return k < len1 ? A0 + k : k < len1 + len2 ? s2 + (k - len1) : e1 + (k - len1 - len2);
    };
    auto claim = [&]() -> int {
        int k = 0;
        if (lane == 0) k = atomicAdd(&claim_next, 1);
        k = __shfl_sync(0xffffffffu, k, 0);
        return k < n ? k : -1;
    };
    // Compute warps: the ring's stages in the order they are consumed
    // (st[0] next); each holds an atom (k: its place in the walk, -1: none),
    // its position, the parity of the stage's next copy and the stage index.
    // Rotated after every atom, so the loop stays rolled and the state in
    // registers.
    struct StageSt {
        int k;
        AtomCursor c;
        uint32_t par;
        int s;
    };
    StageSt st[kStages];
#pragma unroll
    for (int j = 0; j < kStages; ++j) st[j] = StageSt{-1, AtomCursor{0, 0, 0}, 0u, j};
    if (computes) {
        // weights stream while the previous grid on the stream finishes
#pragma unroll
        for (int j = 0; j < kStages; ++j) {
            st[j].k = claim();
            if (st[j].k >= 0) {
                st[j].c = locate_atom_from(P, atom_of(st[j].k), j > 0 ? st[j - 1].c.t : 0);
                issue_weights<NC, MODE>(P, st[j].c, ring + j * kSB, fullb + 8 * j, lane);
            }
        }
    }
    pdl_wait();
#if Q4K_TIMELINE
    const uint64_t tl_wait = globaltimer_ns();
#endif
    if (computes) {
        // activation records of the prologue atoms (written by the previous grid)
#pragma unroll
        for (int j = 0; j < kStages; ++j)
            if (st[j].k >= 0) issue_acts<NC, MODE>(P, st[j].c, ring + j * kSB, fullb + 8 * j, lane);
    }

    // (wait results are made warp-uniform: the warp stays converged for its
    // shuffles and its 32 arrivals)
    bool ok = true;
    int count = 0;  // atoms computed (compute warps) or folded (warp kR)
#if Q4K_TIMELINE
    // SM cycles: compute warps waiting for a free slot / for their copies;
    // the folding warp waiting for a filled slot / writing row groups
    long long tl_cy[2] = {0, 0};
#endif
    if (computes) {
        // claims are monotonic: the first stage without an atom ends the walk
        while (st[0].k >= 0) {
            const int k = st[0].k;
            const uint32_t stage = ring + static_cast<uint32_t>(st[0].s * kSB);
            const uint32_t bar = fullb + 8u * static_cast<uint32_t>(st[0].s);
#if Q4K_TIMELINE
            const long long tw0 = clock64();
#endif
            ok = __all_sync(0xffffffffu, wait_phase(bar, st[0].par, kWaitLimitNs));
#if Q4K_TIMELINE
            tl_cy[1] += clock64() - tw0;
#endif
            if (!ok) break;
            st[0].par ^= 1u;
            float r[kQ];
            atom_sums<NC, MODE>(P, st[0].c, stage, lane, r);
            __syncwarp();
            // refill the stage with the next atom of the walk
            st[0].k = claim();
            if (st[0].k >= 0) {
                st[0].c = locate_atom_from(P, atom_of(st[0].k), st[kStages - 1].c.t);
                fence_proxy_async_smem();
                issue_weights<NC, MODE>(P, st[0].c, stage, bar, lane);
                issue_acts<NC, MODE>(P, st[0].c, stage, bar, lane);
            }
            // hand the sums over: slot k % kS, once atom k - kS is folded
            const int sl = k % kS;
#if Q4K_TIMELINE
            const long long tf0 = clock64();
#endif
            if (k >= kS) ok = __all_sync(0xffffffffu, wait_word_geq(smem_addr(&fold_done), k - kS + 1));
#if Q4K_TIMELINE
            tl_cy[0] += clock64() - tf0;
#endif
            if (!ok) break;
            const uint32_t dst = slots + static_cast<uint32_t>(sl * kSlotB + lane * 4);
#pragma unroll
            for (int q = 0; q < kQ; ++q) sts32f(dst + q * 128, r[q]);
            __syncwarp();
            if (lane == 0) st_release_cta_s32(smem_addr(&slot_tag[sl]), k + 1);  // orders the warp's stores
            ++count;
            // the refilled stage is consumed after the others
            const StageSt t = st[0];
#pragma unroll
            for (int j = 0; j + 1 < kStages; ++j) st[j] = st[j + 1];
            st[kStages - 1] = t;
        }
        if (!ok) {
            if (lane == 0) atomicExch(P.status, kStatusTimeout);
            // let this warp's copies in flight land (bounded) before leaving
#pragma unroll
            for (int j = 0; j < kStages; ++j)
                if (st[j].k >= 0) wait_phase(fullb + 8u * static_cast<uint32_t>(st[j].s), st[j].par, kDrainLimitNs);
        }
    } else if (folder && n > 0) {
        // Fold in walk order, a row group at a time: the group's atoms of this
        // walk as their slots fill -- every filled slot in a row from the next
        // one (the tags of up to 32 slots read at once), their loads issued
        // kBatch at a time, their sums still added atom by atom in walk order
        // -- then the group is written out, or its share deposited.
        constexpr int kBatch = kQ >= 16 ? 2 : kQ >= 4 ? 4 : 8;
        constexpr int kLook = kS < 32 ? kS : 32;
        RowAcc<NC> acc, gacc;
        RowAccD<NC> dacc;  // (Q6_K only)
        acc.clear();
        gacc.clear();
        const uint32_t tag0 = smem_addr(&slot_tag[0]);
        const uint32_t grv = slots + static_cast<uint32_t>(kS * kSlotB);  // group ring values
        int sent = 0;  // groups handed to the flushing warp
        int k = 0;
        uint64_t t0 = 0;
        uint32_t idle = 0;
        // the walk's pieces: [A0, e1), [s2, A1), [e1, s2) (empty ones skipped)
        const int64_t pa[3] = {A0, s2, e1}, pb[3] = {e1, A1, s2};
        int piece = 0;
        while (piece < 2 && pa[piece] == pb[piece]) ++piece;
        int64_t a = pa[piece], pend = pb[piece];
        AtomCursor c = locate_atom(P, a);
        while (k < n) {
            if (a == pend) {
                // the next non-empty piece
                do {
                    ++piece;
                } while (piece < 2 && pa[piece] == pb[piece]);
                a = pa[piece];
                pend = pb[piece];
                c = locate_atom(P, a);
            }
            const TaskDesc &T = P.task[c.t];
            const int m = static_cast<int>(min(static_cast<int64_t>(T.apr - c.kp), pend - a));  // in this group
            const int gate_from = T.has_gate ? T.half : 0x7fffffff;  // kp of the first gate atom
            for (int i = 0; i < m;) {
                const int k0 = k + i;
                // how many slots from k0 on are filled, in a row
#if Q4K_TIMELINE
                const long long tw0 = clock64();
#endif
                int b = 0;
                for (;;) {
                    const int want = min(kLook, m - i);
                    const bool rd = lane < want &&
                                    ld_acquire_cta_s32(tag0 + 4u * static_cast<uint32_t>((k0 + lane) % kS)) == k0 + lane + 1;
                    const uint32_t ball = __ballot_sync(0xffffffffu, rd);
                    b = ball == 0xffffffffu ? 32 : __ffs(~ball) - 1;
                    if (b > 0) break;
                    if (idle == 0) t0 = globaltimer_ns();
                    ++idle;
                    __nanosleep(idle < 16 ? 32 : 128);
                    if ((idle & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
                        ok = false;
                        break;
                    }
                }
#if Q4K_TIMELINE
                tl_cy[0] += clock64() - tw0;
#endif
                if (!ok) break;
                idle = 0;
                // every lane's loads below come after every lane's acquire above
                __syncwarp();
                for (int i0 = 0; i0 < b; i0 += kBatch) {
                    const int bb = min(kBatch, b - i0);
                    float v[kBatch][kQ];
#pragma unroll
                    for (int bi = 0; bi < kBatch; ++bi) {
                        if (bi < bb) {
                            const uint32_t src =
                                slots + static_cast<uint32_t>(((k0 + i0 + bi) % kS) * kSlotB + lane * 4);
#pragma unroll
                            for (int q = 0; q < kQ; ++q) v[bi][q] = lds32f(src + q * 128);
                        }
                    }
#pragma unroll
                    for (int bi = 0; bi < kBatch; ++bi) {
                        if (bi < bb) {
                            const int kp = c.kp + (i + i0 + bi);
                            if (kp >= gate_from) {
#pragma unroll
                                for (int j = 0; j < NC; ++j) gacc.add(j, v[bi][j]);
                            } else {
#pragma unroll
                                for (int j = 0; j < NC; ++j) acc.add(j, v[bi][j]);
                            }
                        }
                    }
                }
                // The values are in registers and used (every lane's loads
                // have returned): the slots may be rewritten.
                __syncwarp();
                if (lane == 0) st_volatile_s32(smem_addr(&fold_done), k0 + b);
                i += b;
                count += b;
            }
            if (!ok) break;
            // hand the group to the flushing warp (entry sent % kGroupRing,
            // once group sent - kGroupRing has been flushed)
#if Q4K_TIMELINE
            const long long tg0 = clock64();
#endif
            if (sent >= kGroupRing)
                ok = __all_sync(0xffffffffu, wait_word_geq(smem_addr(&gr_taken), sent - kGroupRing + 1));
#if Q4K_TIMELINE
            tl_cy[1] += clock64() - tg0;
#endif
            if (!ok) break;
            {
                const int e = sent % kGroupRing;
                const uint32_t dst = grv + static_cast<uint32_t>(e * 2 * NC * 128 + lane * 4);
#pragma unroll
                for (int j = 0; j < NC; ++j) {
                    sts32f(dst + j * 128, acc.value(j));
                    sts32f(dst + (NC + j) * 128, gacc.value(j));
                }
                if (lane == 0) {
                    gr_t[e] = c.t;
                    gr_g[e] = c.g;
                }
                __syncwarp();
                if (lane == 0) st_release_cta_s32(smem_addr(&gr_tag[e]), sent + 1);
                ++sent;
            }
            (void)dacc;
            acc.clear();
            gacc.clear();
            k += m;
            a += m;
            if (a < pend) {
                // the first atom of the next group of the piece
                c.kp = T.apr - 1;
                advance(P, c);
            }
        }
        if (!ok && lane == 0) atomicExch(P.status, kStatusTimeout);
        __syncwarp();
        if (lane == 0) st_release_cta_s32(smem_addr(&gr_total), sent);  // (also after a timeout)
    } else if (folder) {
        if (lane == 0) gr_total = 0;  // no atoms: no groups
    } else if (flusher && n > 0) {
        // Write out the groups in the order the fold sends them: stores of
        // the rows (with biases and the gate epilogue), or this CTA's share
        // of a group that spans CTAs (the last CTA to arrive adds the shares
        // in CTA order, flush_values).
        const uint32_t grv = slots + static_cast<uint32_t>(kS * kSlotB);
        uint64_t t0 = 0;
        uint32_t idle = 0;
        for (int e = 0;; ++e) {
            const int x = e % kGroupRing;
#if Q4K_TIMELINE
            const long long tw0 = clock64();
#endif
            bool have = false, done = false;
            for (;;) {
                have = __all_sync(0xffffffffu, ld_acquire_cta_s32(smem_addr(&gr_tag[x])) == e + 1);
                if (have) break;
                const int tot = ld_volatile_s32(smem_addr(&gr_total));
                if (tot >= 0 && e >= tot) {
                    done = true;
                    break;
                }
                if (idle == 0) t0 = globaltimer_ns();
                ++idle;
                __nanosleep(idle < 16 ? 32 : 128);
                if ((idle & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
                    ok = false;
                    break;
                }
            }
#if Q4K_TIMELINE
            tl_cy[0] += clock64() - tw0;
#endif
            if (!ok) {
                if (lane == 0) atomicExch(P.status, kStatusTimeout);
                break;
            }
            if (done) break;
            idle = 0;
            __syncwarp();
            const uint32_t src = grv + static_cast<uint32_t>(x * 2 * NC * 128 + lane * 4);
            float v[NC], gv[NC];
#pragma unroll
            for (int j = 0; j < NC; ++j) {
                v[j] = lds32f(src + j * 128);
                gv[j] = lds32f(src + (NC + j) * 128);
            }
            const AtomCursor cur{ld_volatile_s32(smem_addr(&gr_t[x])), ld_volatile_s32(smem_addr(&gr_g[x])), 0};
            // the entry is in registers: it may be rewritten
            __syncwarp();
            if (lane == 0) st_volatile_s32(smem_addr(&gr_taken), e + 1);
#if Q4K_TIMELINE
            const long long tg0 = clock64();
#endif
            flush_values<NC, NC, MODE>(P, cur, v, gv, blockIdx.x, A0, A1, lane, 0, blockIdx.x, blockIdx.x, nullptr);
#if Q4K_TIMELINE
            tl_cy[1] += clock64() - tg0;
#endif
            ++count;
        }
    }
#if Q4K_TIMELINE
    // records 0..kR-1: compute warps (word 3: atoms computed); record 15: the
    // folding warp, record 14: the flushing warp (word 3 stays 0: not worker
    // records; word 5: atoms folded / groups written)
    const int rec = folder ? 15 : flusher ? 14 : warp;
    if (lane == 0 && P.tl != nullptr && blockIdx.x < Q4K_TIMELINE_CTAS) {
        unsigned long long *o =
            P.tl + ((static_cast<int64_t>(P.tl_slot) * Q4K_TIMELINE_CTAS + blockIdx.x) * 16 + rec) * 8;
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        o[0] = tl_start;
        o[1] = tl_wait;
        o[2] = globaltimer_ns();
        o[3] = computes ? static_cast<unsigned long long>(count) : 0ull;
        o[4] = smid;
        o[5] = computes ? static_cast<unsigned long long>(blockIdx.x) * 16 + static_cast<unsigned long long>(warp)
                        : static_cast<unsigned long long>(count);
        // the wait / hand-off / write cycles above
        o[6] = static_cast<unsigned long long>(tl_cy[0]);
        o[7] = static_cast<unsigned long long>(tl_cy[1]);
    }
#endif
    if (P.gworld > 1) gather_epilogue(P);
}

// Registers per thread: the two-row MMA variants are capped so that the next
// launch's quantization CTA (256 threads x 32 registers) fits on the SM
// beside a GEMV CTA and runs during its tail (216 x 256 + 8192 <= 65536).
__host__ __device__ constexpr int max_regs_m(int ncols, int mode) {
    return (Q4K_R2_MMA && mode == kModeR2 && ncols >= kR2MmaMin) ? Q4K_R2_MMA_MAXREG : 255;
}
template <int NC, int MODE>
__global__ void __launch_bounds__(warps_m(NC, MODE) * 32, 1) __maxnreg__(max_regs_m(NC, MODE))
    k_gemv(const __grid_constant__ GemvParams P) {
    if constexpr (is_queue(MODE))
        gemv_queue<NC, MODE>(P);
    else
        gemv_per_warp<NC, MODE>(P);
}

// ============================================================================
// Dynamically scheduled GEMV (kModeDynPlain / kModeDynGated)
// ============================================================================
// The unit of work is a whole row group (32 rows x all super-blocks of a
// task).  Every warp of a CTA takes a fixed share of each group's atoms (warp
// w: atoms [w*apr/R, (w+1)*apr/R)) through its own ring, and the CTA adds the
// R warp sums of each row in warp order in shared memory, so a row's result
// does not depend on which CTA computed it.  CTAs take groups from a global
// ticket counter (a workspace header word, cleared by the quantization
// launch): groups blockIdx.x + k * gridDim.x for its first kDynAhead
// entries (their weight copies can start before griddepcontrol.wait), then
// claims, published two groups ahead so that the weight copies never wait for
// a claim.  The host orders the tasks by decreasing K, so the last groups
// handed out are the shortest (longest-first).  Row groups
// are never split between CTAs: no device-scope counters, no partials in
// global memory.
//
// Queue of claimed groups: entry k (the CTA's k-th group) sits in slot
// k % kDynQ; lane 0 of warp 0 fills it and arrives on q_bar[slot], the warps
// wait for phase k / kDynQ.  The filler is at most kDynAhead entries ahead of
// its own group, and no warp is more than two groups behind another (a
// warp's sums for group k + 2 wait until group k's have been added up), so a
// slot is rewritten only after every warp has read it.

__device__ __forceinline__ void dyn_locate(const GemvParams &P, int gi, int &t, int &g) {
    t = 0;
    while (t + 1 < P.ntasks && gi >= P.task[t + 1].rg_base) ++t;
    g = gi - P.task[t].rg_base;
}

// One warp's walk over its atoms of the CTA's groups.  A cursor that has
// passed its last atom of a group reads the next queue entry only when it is
// used (need): the filler publishes entry k + 2 as it starts group k, which is
// exactly as far as a warp's copies run ahead of its sums.
struct DynCursor {
    int k;      // queue entry (the CTA's k-th group)
    int gi;     // global row group (-1: no more work)
    AtomCursor c;
    int s1;     // end of this warp's atoms in the group
    bool need;  // the atoms of entry k are done; entry k + 1 is next
};

template <int R>
__device__ __forceinline__ void dyn_enter(const GemvParams &P, DynCursor &d, int k, int gi, int warp) {
    d.k = k;
    d.gi = gi;
    d.need = false;
    if (gi < 0) return;
    int t, g;
    dyn_locate(P, gi, t, g);
    const int apr = P.task[t].apr;
    d.c = AtomCursor{t, g, warp * apr / R};
    d.s1 = (warp + 1) * apr / R;
}

// Entry k of the queue (waits until it is filled).  Entries below kDynAhead
// are static: group blockIdx.x + k * gridDim.x.
__device__ __forceinline__ int dyn_entry(const int *q_group, const uint64_t *q_bar, int k, int G, bool &ok) {
    if (k < kDynAhead) {
        const int gi = static_cast<int>(blockIdx.x + k * gridDim.x);
        return gi < G ? gi : -1;
    }
    const int slot = k % kDynQ;
    ok = ok && wait_phase(smem_addr(&q_bar[slot]), static_cast<uint32_t>((k / kDynQ) & 1), kWaitLimitNs);
    return ok ? q_group[slot] : -1;
}

// Step past the current atom; at the end of the warp's share mark the cursor.
__device__ __forceinline__ void dyn_step(DynCursor &d) {
    if (++d.c.kp == d.s1) d.need = true;
}

// Move a marked cursor to the next entry (waiting for it to be filled).
template <int R>
__device__ __forceinline__ void dyn_resolve(const GemvParams &P, DynCursor &d, const int *q_group,
                                            const uint64_t *q_bar, int warp, bool &ok) {
    if (!d.need || d.gi < 0) return;
    const int gi = dyn_entry(q_group, q_bar, d.k + 1, P.dyn_groups, ok);
    dyn_enter<R>(P, d, d.k + 1, gi, warp);
}

template <int NC, int BASE>
__global__ void __launch_bounds__(rings_dyn(NC, BASE == kModeGated) * 32, 1)
    k_gemv_dyn(const __grid_constant__ GemvParams P) {
    constexpr bool GATED = BASE == kModeGated;
    constexpr int R = rings_dyn(NC, GATED);
    constexpr int kPC = dyn_pcols(NC, GATED);
    constexpr int kSB = Stage<NC, BASE>::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bars[R][kStages];
    __shared__ __align__(8) uint64_t q_bar[kDynQ];
    __shared__ __align__(8) uint64_t free_bar[2];
    __shared__ int q_group[kDynQ];
    __shared__ int red_cnt[2];
    __shared__ float part[2][R][kPC][32];

#if Q4K_TIMELINE
    const uint64_t tl_start = globaltimer_ns();
#endif
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int r = 0; r < R; ++r)
            for (int s = 0; s < kStages; ++s) mbar_init(smem_addr(&full_bars[r][s]), 1);
        for (int q = 0; q < kDynQ; ++q) mbar_init(smem_addr(&q_bar[q]), 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_addr(&free_bar[b]), 1);
            red_cnt[b] = 0;
        }
        mbar_fence_init();
    }
    __syncthreads();
    uint32_t full[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) full[s] = smem_addr(&full_bars[warp][s]);
    const uint32_t ring = smem_addr(smem) + static_cast<uint32_t>(warp * kStages * kSB);
    const int G = P.dyn_groups;
    const bool producer = warp == 0 && lane == 0;
    if (producer) {
        // the static entries also complete their slots' first phases, so that
        // entry k always completes phase k / kDynQ of slot k % kDynQ
        for (int e = 0; e < kDynAhead; ++e) {
            bool unused = true;
            q_group[e] = dyn_entry(q_group, q_bar, e, G, unused);
            mbar_arrive(smem_addr(&q_bar[e]));
        }
    }

    // Prologue: this warp's first atoms of the static groups (read-only weights).
    bool ok = true;
    DynCursor ic, cc;
    dyn_enter<R>(P, ic, 0, dyn_entry(q_group, q_bar, 0, G, ok), warp);
    cc = ic;
    int issued = 0;
    AtomCursor pro[kStages];
    while (issued < kStages) {
        if (ic.need && ic.k + 1 >= kDynAhead) break;      // a claimed entry: after the wait
        dyn_resolve<R>(P, ic, q_group, q_bar, warp, ok);  // static entries: no wait
        if (ic.gi < 0 || ic.k >= kDynAhead) break;
        pro[issued] = ic.c;
        issue_weights<NC, BASE>(P, ic.c, ring + (issued % kStages) * kSB, full[issued % kStages], lane);
        ++issued;
        dyn_step(ic);
    }
    pdl_wait();
#if Q4K_TIMELINE
    const uint64_t tl_wait = globaltimer_ns();
#endif
    int pend = 0;
    int filled = kDynAhead;       // producer: entries published so far
    bool claiming = producer && dyn_entry(q_group, q_bar, kDynAhead - 1, G, ok) >= 0;
    // activation records of the prologue atoms (written by the previous grid)
    for (int i = 0; i < issued; ++i)
        issue_acts<NC, BASE>(P, pro[i], ring + (i % kStages) * kSB, full[i % kStages], lane);
    // the rest of the ring (when the first group holds fewer atoms than stages)
    while (ok && issued < kStages) {
        dyn_resolve<R>(P, ic, q_group, q_bar, warp, ok);
        if (!ok || ic.gi < 0) break;
        const int s = issued % kStages;
        issue_weights<NC, BASE>(P, ic.c, ring + s * kSB, full[s], lane);
        issue_acts<NC, BASE>(P, ic.c, ring + s * kSB, full[s], lane);
        ++issued;
        dyn_step(ic);
    }

    RowAcc<NC> acc, gacc;
    RowAccD<NC> dacc;  // unused (Q6_K is statically scheduled)
    acc.clear();
    gacc.clear();
    int done = 0;
    int group_k = -1;  // producer: last group whose claim duties ran
    while (ok && cc.gi >= 0) {
        if (producer && cc.k != group_k) {
            group_k = cc.k;
            // publish the ticket drawn one group ago, draw the next one
            if (claiming && cc.k >= 1) {
                const int gi = static_cast<int>(gridDim.x) * kDynAhead + pend;
                const int e = filled++;
                q_group[e % kDynQ] = gi < G ? gi : -1;
                mbar_arrive(smem_addr(&q_bar[e % kDynQ]));
                claiming = gi < G;
            }
            if (claiming) pend = atom_add_relaxed_gpu(P.dyn_claim, 1);
        }
        const int s = done % kStages;
        ok = wait_phase(full[s], static_cast<uint32_t>((done / kStages) & 1), kWaitLimitNs);
        if (!ok) break;
        compute_atom<NC, NC, BASE>(P, cc.c, ring + s * kSB, lane, 0, acc, gacc, dacc, ActView{0u, nullptr});
        __syncwarp();
        dyn_resolve<R>(P, ic, q_group, q_bar, warp, ok);
        if (!ok) break;
        if (ic.gi >= 0) {
            fence_proxy_async_smem();
            issue_weights<NC, BASE>(P, ic.c, ring + s * kSB, full[s], lane);
            issue_acts<NC, BASE>(P, ic.c, ring + s * kSB, full[s], lane);
            ++issued;
            dyn_step(ic);
        }
        ++done;
        if (++cc.c.kp < cc.s1) continue;
        // This warp's share of group cc.gi is summed: deposit it, and the last
        // warp to arrive adds the R shares (warp order) and writes the rows.
        const int b = cc.k & 1;
        const int use = cc.k >> 1;
        if (use >= 1) {
            ok = wait_phase(smem_addr(&free_bar[b]), static_cast<uint32_t>((use - 1) & 1), kWaitLimitNs);
            if (!ok) break;
        }
#pragma unroll
        for (int j = 0; j < NC; ++j) {
            part[b][warp][j][lane] = acc.value(j);
            if constexpr (GATED) part[b][warp][NC + j][lane] = gacc.value(j);
        }
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&red_cnt[b], 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == R - 1) {
            __threadfence_block();
            __syncwarp();
            const TaskDesc &T = P.task[cc.c.t];
            const OutDesc O = out_desc(P, T);
            const int row = cc.c.g * 32 + lane;
#pragma unroll
            for (int j = 0; j < NC; ++j) {
                float tot = 0.0f, gtot = 0.0f;
#pragma unroll
                for (int w = 0; w < R; ++w) {
                    tot += part[b][w][j][lane];
                    if constexpr (GATED) gtot += part[b][w][NC + j][lane];
                }
                if (row < T.nrows) store_final<GATED>(P, O, j, row, tot, gtot);
            }
            __syncwarp();
            if (lane == 0) {
                red_cnt[b] = 0;
                mbar_arrive(smem_addr(&free_bar[b]));
            }
        }
        acc.clear();
        gacc.clear();
        const int gi = dyn_entry(q_group, q_bar, cc.k + 1, G, ok);
        dyn_enter<R>(P, cc, cc.k + 1, gi, warp);
    }
    if (!ok) {
        if (lane == 0) atomicExch(P.status, kStatusTimeout);
        // let this warp's copies in flight land (bounded) before leaving
        for (int i = done; i < issued; ++i)
            wait_phase(full[i % kStages], static_cast<uint32_t>((i / kStages) & 1), kDrainLimitNs);
    }
#if Q4K_TIMELINE
    if (lane == 0 && P.tl != nullptr && blockIdx.x < Q4K_TIMELINE_CTAS && warp < 16) {
        unsigned long long *o =
            P.tl + ((static_cast<int64_t>(P.tl_slot) * Q4K_TIMELINE_CTAS + blockIdx.x) * 16 + warp) * 8;
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        o[0] = tl_start;
        o[1] = tl_wait;
        o[2] = globaltimer_ns();
        o[3] = static_cast<unsigned long long>(done > 0 ? done : 1);
        o[4] = smid;
        o[5] = static_cast<unsigned long long>(blockIdx.x * R + warp);
        o[6] = 0;
        o[7] = static_cast<unsigned long long>(cc.k);
    }
#endif
}

// ============================================================================
// host-side launchers
// ============================================================================
namespace {
std::mutex g_setup_mu;
struct DevState {
    bool ready = false;
    int num_sms = 0;
};
DevState g_dev[64];

template <int NC, int MODE>
cudaError_t set_attrs() {
    return cudaFuncSetAttribute(k_gemv<NC, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_m(NC, MODE));
}

template <int MODE>
cudaError_t set_attrs_all() {
    cudaError_t e;
    if ((e = set_attrs<1, MODE>()) != cudaSuccess) return e;
    if ((e = set_attrs<2, MODE>()) != cudaSuccess) return e;
    if ((e = set_attrs<3, MODE>()) != cudaSuccess) return e;
    if ((e = set_attrs<4, MODE>()) != cudaSuccess) return e;
    if ((e = set_attrs<5, MODE>()) != cudaSuccess) return e;
    if ((e = set_attrs<6, MODE>()) != cudaSuccess) return e;
    if ((e = set_attrs<7, MODE>()) != cudaSuccess) return e;
    return set_attrs<8, MODE>();
}

template <int NC, int BASE>
cudaError_t set_attrs_dyn1() {
    return cudaFuncSetAttribute(k_gemv_dyn<NC, BASE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem_m(NC, BASE == kModeGated ? kModeDynGated : kModeDynPlain));
}

template <int BASE>
cudaError_t set_attrs_dyn() {
    cudaError_t e;
    if ((e = set_attrs_dyn1<1, BASE>()) != cudaSuccess) return e;
    if ((e = set_attrs_dyn1<2, BASE>()) != cudaSuccess) return e;
    if ((e = set_attrs_dyn1<3, BASE>()) != cudaSuccess) return e;
    if ((e = set_attrs_dyn1<4, BASE>()) != cudaSuccess) return e;
    if ((e = set_attrs_dyn1<5, BASE>()) != cudaSuccess) return e;
    if ((e = set_attrs_dyn1<6, BASE>()) != cudaSuccess) return e;
    if ((e = set_attrs_dyn1<7, BASE>()) != cudaSuccess) return e;
    return set_attrs_dyn1<8, BASE>();
}

template <int BASE>
void *gemv_fn_dyn(int ncols) {
    switch (ncols) {
        case 1: return reinterpret_cast<void *>(k_gemv_dyn<1, BASE>);
        case 2: return reinterpret_cast<void *>(k_gemv_dyn<2, BASE>);
        case 3: return reinterpret_cast<void *>(k_gemv_dyn<3, BASE>);
        case 4: return reinterpret_cast<void *>(k_gemv_dyn<4, BASE>);
        case 5: return reinterpret_cast<void *>(k_gemv_dyn<5, BASE>);
        case 6: return reinterpret_cast<void *>(k_gemv_dyn<6, BASE>);
        case 7: return reinterpret_cast<void *>(k_gemv_dyn<7, BASE>);
        case 8: return reinterpret_cast<void *>(k_gemv_dyn<8, BASE>);
        default: return nullptr;
    }
}

// The single-launch variant exists for ncols <= kActSmemMaxCols only.
cudaError_t set_attrs_asm() {
    cudaError_t e;
    static_assert(kActSmemMaxCols == 2, "instantiate the single-launch variant for every width");
    constexpr int kMax = kSmemLimit - kActSmemStatic;
    if ((e = cudaFuncSetAttribute(k_gemv<1, kModeActSmem>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax)) !=
        cudaSuccess)
        return e;
    return cudaFuncSetAttribute(k_gemv<2, kModeActSmem>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMax);
}

void *gemv_fn_asm(int ncols) {
    switch (ncols) {
        case 1: return reinterpret_cast<void *>(k_gemv<1, kModeActSmem>);
        case 2: return reinterpret_cast<void *>(k_gemv<2, kModeActSmem>);
        default: return nullptr;
    }
}

// The two-row variant exists for ncols >= kR2Min only.
cudaError_t set_attrs_r2() {
    cudaError_t e;
    if ((e = set_attrs<3, kModeR2>()) != cudaSuccess) return e;
    if ((e = set_attrs<4, kModeR2>()) != cudaSuccess) return e;
    if ((e = set_attrs<5, kModeR2>()) != cudaSuccess) return e;
    if ((e = set_attrs<6, kModeR2>()) != cudaSuccess) return e;
    if ((e = set_attrs<7, kModeR2>()) != cudaSuccess) return e;
    return set_attrs<8, kModeR2>();
}

void *gemv_fn_r2(int ncols) {
    switch (ncols) {
        case 3: return reinterpret_cast<void *>(k_gemv<3, kModeR2>);
        case 4: return reinterpret_cast<void *>(k_gemv<4, kModeR2>);
        case 5: return reinterpret_cast<void *>(k_gemv<5, kModeR2>);
        case 6: return reinterpret_cast<void *>(k_gemv<6, kModeR2>);
        case 7: return reinterpret_cast<void *>(k_gemv<7, kModeR2>);
        case 8: return reinterpret_cast<void *>(k_gemv<8, kModeR2>);
        default: return nullptr;
    }
}

template <int MODE>
void *gemv_fn(int ncols) {
    switch (ncols) {
        case 1: return reinterpret_cast<void *>(k_gemv<1, MODE>);
        case 2: return reinterpret_cast<void *>(k_gemv<2, MODE>);
        case 3: return reinterpret_cast<void *>(k_gemv<3, MODE>);
        case 4: return reinterpret_cast<void *>(k_gemv<4, MODE>);
        case 5: return reinterpret_cast<void *>(k_gemv<5, MODE>);
        case 6: return reinterpret_cast<void *>(k_gemv<6, MODE>);
        case 7: return reinterpret_cast<void *>(k_gemv<7, MODE>);
        case 8: return reinterpret_cast<void *>(k_gemv<8, MODE>);
        default: return nullptr;
    }
}
}  // namespace

cudaError_t device_setup(int *num_sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_setup_mu);
    DevState &st = g_dev[dev];
    if (!st.ready) {
        if ((e = cudaDeviceGetAttribute(&st.num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        if ((e = set_attrs_all<kModePlain>()) != cudaSuccess) return e;
        if ((e = set_attrs_all<kModeDump>()) != cudaSuccess) return e;
        if ((e = set_attrs_all<kModeGated>()) != cudaSuccess) return e;
        if ((e = set_attrs_r2()) != cudaSuccess) return e;
        if ((e = set_attrs_all<kModeQ6>()) != cudaSuccess) return e;
        if ((e = set_attrs_dyn<kModePlain>()) != cudaSuccess) return e;
        if ((e = set_attrs_dyn<kModeGated>()) != cudaSuccess) return e;
        if ((e = set_attrs_asm()) != cudaSuccess) return e;
        st.ready = true;
    }
    *num_sms = st.num_sms;
    return cudaSuccess;
}

cudaError_t launch_prep(const PrepParams &p, cudaStream_t s) {
    int64_t blocks = (p.nitems * 32 + 255) / 256;
    const int64_t zb = (p.zero_count + 255) / 256;
    if (zb > blocks) blocks = zb;
    if (blocks < 1) blocks = 1;
    if (blocks > 4096) blocks = 4096;
    blocks += p.norm_ctas;  // the normalizing CTAs come first
    // Programmatic dependent of whatever precedes it on the stream: it can be
    // resident before the previous GEMV ends and waits for it on the device.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_prep, p);
}

cudaError_t launch_gather_wait(const GatherWait &g, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_gather_wait, g);
}

cudaError_t launch_gemv(const GemvParams &p, int ncols, int mode, int grid, cudaStream_t s) {
    void *fn = mode == kModeDump    ? gemv_fn<kModeDump>(ncols)
               : mode == kModeGated ? gemv_fn<kModeGated>(ncols)
               : mode == kModeR2    ? gemv_fn_r2(ncols)
               : mode == kModeQ6    ? gemv_fn<kModeQ6>(ncols)
               : mode == kModeDynPlain ? gemv_fn_dyn<kModePlain>(ncols)
               : mode == kModeDynGated ? gemv_fn_dyn<kModeGated>(ncols)
               : mode == kModeActSmem  ? gemv_fn_asm(ncols)
                                    : gemv_fn<kModePlain>(ncols);
    if (fn == nullptr) return cudaErrorInvalidValue;
    if (mode == kModeActSmem && (p.act_smem_bytes < 0 || p.act_smem_bytes > kActSmemCap))
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(warps_m(ncols, mode) * 32);
    cfg.dynamicSmemBytes = smem_m(ncols, mode) + (mode == kModeActSmem ? p.act_smem_bytes : 0);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {const_cast<GemvParams *>(&p)};
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace q4k
