// q4k_internal.h -- launch parameters shared by the host runtime and the kernels.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>  // CUtensorMap (type only; the encoder is fetched at run time)
#include <cuda_runtime.h>

namespace q4k {

constexpr int kQK = 256;          // weights per super-block
constexpr int kSBBytes = 144;     // bytes per super-block
constexpr int kQ81Bytes = 36;     // bytes per q8_1 block
constexpr int kActSBBytes = 320;  // q8a bytes per super-block and column
constexpr int kActMetaOff = 256;  // q8a: offset of the per-pair float4 metadata
constexpr int kMaxCols = 8;
constexpr int kMaxTasks = 16;
constexpr int kMaxGated = 4;  // tasks with a fused gate per launch (their tensor maps are kernel parameters)
constexpr int kMaxJobs = 16;
constexpr int kMaxPeers = 8;

// GEMV geometry.  A "worker" is one warp; it owns a contiguous range of
// "atoms" (32 weight rows x kKS super-blocks, plus the kKS activation records
// of every column) of the flattened work of all tasks, streamed through a
// private kStages-deep ring of shared-memory stages by bulk asynchronous
// copies.  Lane = weight row.
#ifndef Q4K_MAX_WARPS
#define Q4K_MAX_WARPS 8
#endif
#ifndef Q4K_STAGES
#define Q4K_STAGES 2
#endif
#ifndef Q4K_KS
#define Q4K_KS 2
#endif
// Launch timeline stamps (diagnostic builds only; q4k_timeline_* in the C-ABI).
#ifndef Q4K_TIMELINE
#define Q4K_TIMELINE 0
#endif
// Weight boxes are copied with an L2 evict-first policy (read once).
#ifndef Q4K_WEIGHT_EVICT_FIRST
#define Q4K_WEIGHT_EVICT_FIRST 1
#endif
constexpr int kMaxWarps = Q4K_MAX_WARPS;
constexpr int kStages = Q4K_STAGES;
constexpr int kKS = Q4K_KS;  // super-blocks per atom and row
// Weights of one super-block for 32 rows: one 2D tensor-map box of 32 rows x
// 144 bytes, landing densely at a 144-byte row pitch -- an odd number of
// 16-byte units, so the 8 lanes of a quarter-warp (8 consecutive rows) hit
// 8 different bank groups.
constexpr int kPitch = 144;
constexpr int kBoxBytes = 32 * kPitch;
constexpr int kWStageBytes = kKS * kBoxBytes;
constexpr int kSmemLimit = 227 * 1024;

// One ring stage: weights (32 rows) then the activation records of ncols columns.
__host__ __device__ constexpr int stage_bytes(int ncols) { return kWStageBytes + ncols * kKS * 320; }
// Warps that share one ring, each computing a share of the columns: from
// Q4K_SPLIT_MIN columns on, two.  The split doubles the warps per SM without
// more shared memory, but repeats the per-row work in both warps; on B200 it
// measured no faster at 8 columns and slower at 3-5 (the dp4a/f32x2 pipe and
// the shared-memory wavefronts, not latency, bound those), so the default
// (9) leaves it off.
#ifndef Q4K_SPLIT_MIN
#define Q4K_SPLIT_MIN 9
#endif
__host__ __device__ constexpr int split_for(int ncols) { return ncols >= Q4K_SPLIT_MIN ? 2 : 1; }
// Rings (= workers) per CTA for ncols columns: as many as fit (one CTA per SM).
__host__ __device__ constexpr int rings_for(int ncols) {
    return kSmemLimit / (kStages * stage_bytes(ncols)) < kMaxWarps ? kSmemLimit / (kStages * stage_bytes(ncols))
                                                                   : kMaxWarps;
}
__host__ __device__ constexpr int warps_for(int ncols) { return rings_for(ncols) * split_for(ncols); }
__host__ __device__ constexpr int smem_bytes(int ncols) { return rings_for(ncols) * kStages * stage_bytes(ncols); }
static_assert(rings_for(8) >= 4, "ring too large for 8 columns");
static_assert(warps_for(8) * 32 <= 1024, "block too large");

// Kernel variants: plain, debug dump of the sub-block sums; kModeGated:
// launches with a fused task (a bias or a gate: the epilogue code lives only
// in this variant and kModeDynGated).  kModeR2: plain Q4_K tasks at ncols >=
// kR2Min, 64-row groups with two rows per lane (one activation load serves
// both rows).  kModeQ6: Q6_K weights.  kModeDynPlain / kModeDynGated: the
// dynamically scheduled kernel (k_gemv_dyn: whole row groups per CTA),
// without / with a fused task.
// kModeActSmem: the plain arithmetic and partition in one launch: every CTA
// quantizes the activations its atoms need straight into shared memory
// (no separate quantization launch), ring stages carry weights only.
enum GemvMode : int {
    kModePlain = 0,
    kModeDump = 1,
    kModeGated = 2,
    kModeR2 = 3,
    kModeQ6 = 4,
    kModeDynPlain = 5,
    kModeDynGated = 6,
    kModeActSmem = 7
};
#ifndef Q4K_R2_MIN
#define Q4K_R2_MIN 3
#endif
constexpr int kR2Min = Q4K_R2_MIN;
// Two-row atoms of Q4K_R2_MMA_MIN or more columns take their integer sums
// from int8 tensor-core MMAs (fewer columns: dp4a); each warp then needs a
// 4 KB scratch after the rings.  Measured on B200 (Mistral-7B layer launch,
// us): ncols 3 33.3 dp4a / 35.1 MMA, 4 37.2 / 35.3, 5 43.9 / 39.2, 8 58.9 /
// 45.4 (the MMA always computes 8 columns, padding included).
#ifndef Q4K_R2_MMA
#define Q4K_R2_MMA 1
#endif
#ifndef Q4K_R2_MMA_MIN
#define Q4K_R2_MMA_MIN 4
#endif
constexpr int kR2MmaMin = Q4K_R2_MMA_MIN;
// Register cap of the two-row MMA variants (k_gemv's max_regs_m): measured
// on B200, 14336x4096 chain ncols 4 18.7 -> 16.2 us, ncols 8 21.3 -> 19.2 us
// (the next quantization launch runs beside the GEMV's tail); the Mistral
// layer chain 2 % slower at ncols 4 and 8.
#ifndef Q4K_R2_MMA_MAXREG
#define Q4K_R2_MMA_MAXREG 216
#endif
__host__ __device__ constexpr int r2_scr_bytes(int ncols, int mode) {
    return (Q4K_R2_MMA && mode == kModeR2 && ncols >= kR2MmaMin) ? kMaxWarps * 2 * 64 * 8 * 4 : 0;
}

// Q6_K (210-byte super-blocks: ql[128], qh[64], int8 scales[16], fp16 d).  A
// 210-byte row chunk is never a multiple of 16 bytes, 8 super-blocks (1680 B)
// are: an atom is 8 rows x 8 super-blocks, one tensor-map box of 210 uint64
// x 8 rows, landing at a 1680-byte row pitch.  Lane (r = lane & 7,
// q = lane >> 3) takes super-blocks 2q and 2q+1 of row r.  The activation
// records of the 8 super-blocks sit at a 336-byte pitch (lanes with different
// q read different banks).
constexpr int kQ6Bytes = 210;
constexpr int kQ6AtomSB = 8;
constexpr int kQ6Rows = 8;
constexpr int kQ6RowBytes = kQ6AtomSB * kQ6Bytes;  // 1680
constexpr int kQ6BoxBytes = kQ6Rows * kQ6RowBytes;  // 13440
constexpr int kQ6RecPitch = 336;
// Up to this many columns the Q6_K path takes the -32 offset out of the sums
// (unsigned dp4a and activation sums) instead of out of the bytes.
#ifndef Q4K_Q6_UNSIGNED_MAX
#define Q4K_Q6_UNSIGNED_MAX 2
#endif
__host__ __device__ constexpr int q6_stage_bytes(int ncols) { return kQ6BoxBytes + ncols * kQ6AtomSB * kQ6RecPitch; }
__host__ __device__ constexpr int rings_q6(int ncols) {
    return kSmemLimit / (kStages * q6_stage_bytes(ncols)) < kMaxWarps ? kSmemLimit / (kStages * q6_stage_bytes(ncols))
                                                                      : kMaxWarps;
}
static_assert(rings_q6(8) >= 2, "Q6_K ring too large for 8 columns");
// Dynamically scheduled launches: one warp per ring, each warp holds a
// fixed share of every row group's atoms, and the CTA adds the warps' sums in
// double-buffered shared memory (2 x rings x pcols x 32 floats beside the
// rings; pcols = 2 * ncols with a gate).
__host__ __device__ constexpr int dyn_pcols(int ncols, bool gated) { return gated ? 2 * ncols : ncols; }
__host__ __device__ constexpr int rings_dyn(int ncols, bool gated) {
    int r = kMaxWarps;
    while (r > 1 && r * kStages * stage_bytes(ncols) + 2 * r * dyn_pcols(ncols, gated) * 128 > kSmemLimit - 2048) --r;
    return r;
}
static_assert(rings_dyn(8, true) >= 4, "dynamic ring too small for 8 gated columns");
// Queue of a CTA's row groups: kDynQ slots; entries 0 .. kDynAhead-1 are
// static (blockIdx.x + k * gridDim.x), later ones claimed kDynAhead - 1
// groups ahead.
constexpr int kDynQ = 16;
constexpr int kDynAhead = 3;
// Geometry by kernel variant.
__host__ __device__ constexpr bool is_dyn(int mode) {
    return mode == kModeDynPlain || mode == kModeDynGated;
}
// ---- balanced partition (k_gemv, launches with a fused task) -----------------
// CTA c of G owns the contiguous atom range [natoms*c/G, natoms*(c+1)/G).  Its
// R compute warps take the range's atoms in order from a shared-memory
// counter, each through its own kStages-deep ring, and leave every atom's
// sums (ncols floats per lane) in one of q_slots result slots; one more warp
// folds the slots in atom order into the row groups' sums, and another
// applies the epilogue and writes the rows.  Shared memory: the rings, the
// slots, the group ring.
constexpr int kQueueStatic = 2048;  // reserve for the kernel's static shared memory
// (launches with a fused task; the others keep per-warp ranges: measured
// faster in a chain of launches, where the next launch's CTAs already start
// on the SMs that finish early)
__host__ __device__ constexpr bool is_queue(int mode) { return mode == kModeGated; }
__host__ __device__ constexpr int q_slot_bytes(int ncols, int /*mode*/) { return 32 * 4 * ncols; }
// Result slots: as many as fit well (the fold may fall behind the compute
// warps for a while without stalling them), at least two per compute warp.
__host__ __device__ constexpr int q_slots(int ncols, int mode) {
    return q_slot_bytes(ncols, mode) <= 128   ? 128
           : q_slot_bytes(ncols, mode) <= 256 ? 64
           : q_slot_bytes(ncols, mode) <= 512 ? 32
                                              : 16;
}
// Row groups handed from the folding warp to the flushing warp (which
// writes them out, or does the cross-CTA hand-off of a group shared with a
// neighbouring CTA): a ring of kGroupRing entries of 2 * ncols floats per
// lane (the main and the second sums).
constexpr int kGroupRing = 4;
__host__ __device__ constexpr int q_group_bytes(int ncols) { return kGroupRing * 2 * ncols * 128; }
__host__ __device__ constexpr int q_aux_bytes(int ncols, int mode) {
    return q_slots(ncols, mode) * q_slot_bytes(ncols, mode) + q_group_bytes(ncols);
}
// activation records per column in a ring stage: a two-row atom covers one
// super-block, the others kKS (ring geometry of the static kernel's variants)
// (two-row atoms: 336, an odd number of 16-byte units, so the MMA operand
// loads of 8 columns at the same offset hit 8 different bank groups)
__host__ __device__ constexpr int q_col_pitch(int mode) { return mode == kModeR2 ? kActSBBytes + 16 : kKS * kActSBBytes; }
__host__ __device__ constexpr int round128(int b) { return (b + 127) / 128 * 128; }
__host__ __device__ constexpr int q_stage_bytes(int ncols, int mode) {
    return mode == kModeActSmem ? kWStageBytes : round128(kWStageBytes + ncols * q_col_pitch(mode));
}
// Plain and single-launch kernels: one more warp, the boundary warp, takes
// the row groups a compute warp shares with another CTA (at most two per
// warp: ncols floats per lane each, placed after the rings).
__host__ __device__ constexpr bool has_xhelp(int mode) { return mode == kModePlain || mode == kModeActSmem; }
__host__ __device__ constexpr int xh_bytes(int ncols, int mode) {
    return has_xhelp(mode) ? kMaxWarps * 2 * ncols * 128 : 0;
}
__host__ __device__ constexpr int q_rings(int ncols, int mode) {
    int r = kMaxWarps;
    while (r > 1 && r * kStages * q_stage_bytes(ncols, mode) + (is_queue(mode) ? q_aux_bytes(ncols, mode) : 0) +
                            xh_bytes(ncols, mode) + r2_scr_bytes(ncols, mode) >
                        kSmemLimit - kQueueStatic)
        --r;
    return r;
}
static_assert(q_rings(8, kModeR2) == kMaxWarps && q_rings(2, kModePlain) == kMaxWarps, "rings per CTA");
static_assert(q_rings(8, kModeGated) >= 6, "epilogue variant: ring too small for 8 columns");
// Single-launch mode: up to kActSmemMaxCols columns; shared memory beyond the
// rings (8 warps x kStages x one weight stage) and the boundary warp's
// entries holds the CTA's activation records, at most kActSmemCap bytes (the
// rest of the 227 KB, less a reserve for the kernel's static shared memory).
constexpr int kActSmemMaxCols = 2;
constexpr int kActSmemRings = kMaxWarps;
constexpr int kActSmemStatic = 2048;
constexpr int kActSmemCap =
    kSmemLimit - kActSmemRings * kStages * kWStageBytes - xh_bytes(kActSmemMaxCols, kModeActSmem) - kActSmemStatic;
constexpr int kMaxPlanCtas = 256;  // launches of more CTAs (SMs) run the two-launch sequence
static_assert(kActSmemCap > 0, "no room for activations beside the rings");
__host__ __device__ constexpr int stage_bytes_m(int ncols, int mode) {
    return mode == kModeQ6 ? q6_stage_bytes(ncols) : is_dyn(mode) ? stage_bytes(ncols) : q_stage_bytes(ncols, mode);
}
__host__ __device__ constexpr int rings_m(int ncols, int mode) {
    return mode == kModeQ6         ? rings_q6(ncols)
           : is_dyn(mode)          ? rings_dyn(ncols, mode == kModeDynGated)
           : mode == kModeActSmem  ? kActSmemRings
                                   : q_rings(ncols, mode);
}
// threads per CTA / 32: the epilogue variant adds the folding and the
// flushing warp, the plain and single-launch kernels the boundary warp
__host__ __device__ constexpr int warps_m(int ncols, int mode) {
    return rings_m(ncols, mode) + (is_queue(mode) ? 2 : has_xhelp(mode) ? 1 : 0);
}
// The single-launch mode keeps the plain kernel's partition (same rings per
// CTA), so both paths give bit-identical results.
static_assert(q_rings(1, kModePlain) == kActSmemRings && q_rings(2, kModePlain) == kActSmemRings &&
                  split_for(2) == 1,
              "single-launch partition differs from the two-launch one");
__host__ __device__ constexpr int smem_m(int ncols, int mode) {
    return rings_m(ncols, mode) * kStages * stage_bytes_m(ncols, mode) +
           (is_queue(mode) ? q_aux_bytes(ncols, mode) : 0) + xh_bytes(ncols, mode) + r2_scr_bytes(ncols, mode);
}

// Device status codes (match q4k_status).
constexpr int kStatusOk = 0;
constexpr int kStatusBadPlan = 1;  // a launch plan the kernel refused (Q4K_EINVAL)
constexpr int kStatusTimeout = 3;
// Bounded waits: a bulk copy that has not landed after this long is an error.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s
constexpr unsigned long long kDrainLimitNs = 20000000ull;   // 20 ms
constexpr unsigned long long kPeerWaitLimitNs = 2000000000ull;  // 2 s for the peers' epoch

// Consumer wait of the fused all-gather: this rank's flag words (one per
// sender), its epoch word, and where to report a wait that gave up.
struct GatherWait {
    const uint32_t *flags;
    const uint32_t *epoch;
    int32_t *status;
    int32_t world;   // <= 1: no wait
    int32_t rank;
};

struct TaskDesc {
    const uint8_t *W;        // weight row 0 (16-byte aligned)
    const uint8_t *act;      // q8a column 0
    float *dst;              // output column 0
    int64_t row_stride;      // bytes between weight rows
    int64_t act_col_stride;  // bytes between q8a columns
    int64_t dst_col_stride;  // floats between output columns
    int64_t atom_base;       // first global atom of this task
    int32_t nrows;
    int32_t nb;              // super-blocks per row
    int32_t apr;             // atoms per row group: ceil(nb / kKS), twice that with a gate
    int32_t rg_base;         // global row-group index of row group 0
    int32_t ngroups;         // row groups = ceil(nrows / 32)
    int32_t act_id;          // index of this task's distinct activation
    // single-launch path: the fp32 activation this task's q8a records come from
    const float *x;
    int64_t x_col_stride;    // floats between activation columns
    // Fused epilogue (kernels/mmvq.cu:182-227, :309-338): with a gate matrix
    // (tensor map tmap_gate[gate_map]) a row group runs over both matrices in
    // turn: its first `half` atoms are the main matrix's, the next `half` the
    // gate's (apr = 2 * half, half = ceil(nb / kKS)), summed apart, and the
    // output is glu(W.x + x_bias, Wg.x + gate_bias).  Atoms stay the plain
    // ones (32 rows x kKS super-blocks of one matrix), with the plain
    // arithmetic.
    int32_t has_gate;
    int32_t glu_op;          // GluOp
    int32_t gate_map;
    int32_t half;            // atoms per row group of each matrix (0 without a gate)
    const float *x_bias;     // per output row, or nullptr
    const float *gate_bias;  // per output row, or nullptr (only with a gate)
    int64_t bias_col_stride; // floats between bias columns (0: one column for all)
};

// Epilogue ops (values of q4k_gemv.h's Q4K_GLU_*).
enum GluOp : int32_t { kGluNone = 0, kGluSwiglu = 1, kGluGeglu = 2, kGluSwigluOai = 3, kGluMul = 4 };

struct GemvParams {
    CUtensorMap tmap[kMaxTasks];        // per task: uint32 view {nb*36, nrows}, box {36, 32}
    CUtensorMap tmap_gate[kMaxGated];   // gate matrices of the tasks with a fused gate
    TaskDesc task[kMaxTasks];
    int32_t ntasks;
    int32_t nworkers;        // partition units, each with >= 1 atom (<= natoms): CTAs
                             // (<= gridDim.x, balanced partition) or warps (<= gridDim.x * rings)
    int32_t packed;          // warps: 1: worker = cta * rings + ring (CTA-contiguous ranges);
                             // 0: worker = ring * gridDim.x + cta (small problems spread over SMs)
    int32_t pad0_;
    int64_t natoms;
    int32_t *counters;       // one per global row group, zero at kernel start
    float *partials;         // [nworkers][2][pcols][32]
    int32_t pcols;           // columns per partial slot: ncols, or 2*ncols (a task with a gate, two-row launches)
    int32_t dyn_groups;      // dynamically scheduled launches: row groups of all tasks
    int32_t *status;
    int32_t *dump_S;         // debug: sub-block sums (nullptr in the product path)
    // Fused all-gather over peer memory (gworld > 1): every output value is
    // also stored at the same offset from gout_peer[q] for each peer q, and
    // the grid's last CTA exchanges an epoch with every peer before exiting.
    int32_t gworld;
    int32_t grank;
    float *gout_local;               // this rank's full output buffer
    float *gout_peer[kMaxPeers];     // every rank's full output buffer, mapped here
    uint32_t *gflags_peer[kMaxPeers];// every rank's flag words (one per sender), mapped here
    uint32_t *gepoch;                // this rank's epoch word (persists across calls)
    uint32_t *gdone;                 // CTAs finished (workspace; zero at kernel start)
    GatherWait gwait;                // single-launch path: wait for the previous gather before reading x
    // Single-launch path: the distinct activations (a task that reads each,
    // its fp32 columns, column stride and super-blocks), which of them each
    // CTA's atoms read (a bit per activation, computed on the host), each
    // task's activation, and the shared-memory bytes every CTA has for the
    // q8a records.  Flat tables, so that a CTA's plan reads few parameter lines.
    int32_t n_act;
    int32_t act_smem_bytes;
    int32_t act_task[kMaxTasks];
    const float *act_x[kMaxTasks];
    int64_t act_xcs[kMaxTasks];
    int32_t act_nb[kMaxTasks];
    int8_t task_act[kMaxTasks];
    uint16_t cta_act_mask[kMaxPlanCtas];
    int32_t *dyn_claim;              // dynamically scheduled launches: group tickets (zero at kernel start)
    unsigned long long *tl;          // launch timeline records (Q4K_TIMELINE builds; else nullptr)
    int32_t tl_slot;
    int32_t tl_pad_;
};

enum PrepKind : int32_t { kPrepF32 = 0, kPrepQ81 = 1 };

struct PrepJob {
    const void *src;         // fp32 columns or ggml q8_1 columns
    uint8_t *act;            // q8a output (nullptr: none)
    uint8_t *q81_out;        // ggml q8_1 output (nullptr: none)
    int32_t *dump_T;         // debug: T per (column, block) (nullptr: none)
    int64_t src_col_stride;  // floats (fp32) or blocks (q8_1)
    int64_t act_col_stride;  // bytes
    int64_t q81_col_stride;  // blocks
    int64_t item_base;       // first global warp item of this job
    int32_t K;               // valid activations per column
    int32_t nblk;            // q8 blocks per column to produce
    int32_t ncols;
    int32_t kind;
    // RMSNorm ahead of the quantizer (fp32 jobs): one CTA per column, CTAs
    // [cta_base, cta_base + ncols) of the launch; the job has no warp items.
    int32_t norm;
    float norm_eps;
    const float *norm_w;     // per-element weight, or nullptr
    int32_t cta_base;
    int32_t pad_;
};

struct PrepParams {
    PrepJob job[kMaxJobs];
    GatherWait gwait;        // gathering calls: wait for the previous gather before reading x
    int32_t njobs;
    int32_t zero_count;      // int32 words to clear at zero_ptr (counters, status)
    int64_t nitems;
    int32_t *zero_ptr;
    int32_t norm_ctas;       // leading CTAs that normalize whole columns (RMSNorm jobs)
    int32_t pad_;
    unsigned long long *tl;  // launch timeline records (Q4K_TIMELINE builds; else nullptr)
    int32_t tl_slot;
    int32_t tl_pad_;
};

// Launchers (q4k_kernels.cu).  Return cudaSuccess or the launch error.
cudaError_t launch_prep(const PrepParams &p, cudaStream_t s);
cudaError_t launch_gemv(const GemvParams &p, int ncols, int mode, int grid, cudaStream_t s);
cudaError_t launch_gather_wait(const GatherWait &g, cudaStream_t s);
// Per-device setup (SM count, shared-memory opt-in); thread-safe, idempotent.
cudaError_t device_setup(int *num_sms);

}  // namespace q4k
