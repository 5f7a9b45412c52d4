// q4k_capi.cu -- host runtime and C ABI of libq4k_gemv.so (declared in
// include/q4k_gemv.h).
//
// Responsibilities: argument validation (status codes instead of the
// reference's aborts), workspace layout, de-duplication of shared
// activations, the flattened work schedule (atoms and row groups) and the
// two-launch sequence prep -> GEMV (the GEMV is a programmatic dependent
// launch, so its weight stream overlaps the activation quantization).
#include "q4k_gemv.h"
#include "q4k_internal.h"

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

using namespace q4k;

namespace {

thread_local std::string g_last_error;

int fail(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(Q4K_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

constexpr size_t kAlign = 256;
size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Upper bound on workers when no device can be queried.
constexpr int kFallbackSMs = 256;

int num_sms_or_bound() {
    int n = 0;
    if (device_setup(&n) == cudaSuccess && n > 0) return n;
    cudaGetLastError();
    return kFallbackSMs;
}

// Workspace layout: [status word | pad][counters][partials][activations];
// header bytes 4 (gather), 64 (dynamic tickets) and 128 (grid barrier) hold sync words.
struct Layout {
    size_t counters_off = 0, partials_off = 0, act_off = 0, total = 0;
};

Layout make_layout(int64_t n_rowgroups, int ncols, size_t act_bytes, int64_t partial_slots) {
    Layout L;
    L.counters_off = kAlign;
    L.partials_off = L.counters_off + round_up(static_cast<size_t>(n_rowgroups) * 4, kAlign);
    L.act_off = L.partials_off + round_up(static_cast<size_t>(partial_slots) * ncols * 32 * sizeof(float), kAlign);
    L.total = L.act_off + round_up(act_bytes, kAlign);
    return L;
}

// One matrix as the runtime sees it: activations are fp32 or ggml q8_1.
struct Job {
    const void *W;
    const void *src;
    float *dst;
    int64_t nrows, K, stride_row_x, src_col_stride, stride_col_dst;
    int kind;  // kPrepF32 / kPrepQ81
    // fused epilogue (kernels/mmvq.cu:182-227, :309-338)
    const void *gate = nullptr;      // gate matrix: same shape and row stride as W
    const float *x_bias = nullptr;
    const float *gate_bias = nullptr;
    int64_t bias_col_stride = 0;
    int glu_op = Q4K_GLU_NONE;
    // RMSNorm of x ahead of the quantizer (fp32 jobs)
    int norm = 0;
    float norm_eps = 0.0f;
    const float *norm_w = nullptr;
    int q6 = 0;  // W holds Q6_K super-blocks (210 bytes) instead of Q4_K
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cuTensorMapEncodeTiled, fetched through the runtime (no link against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tensor_map_encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// Weight matrix as a 2D uint32 tensor {nb*36 words, nrows}, row stride in
// bytes, box {36 words = one super-block, 32 rows}.
// Encoded tensor maps of recent calls: a pure function of (matrix, shape,
// stride, format), so calls that reuse their weights (every decode step)
// skip the driver's encoder.  Per host thread, bounded.
struct MapKey {
    const void *W;
    int64_t nrows, nb, stride;
    int q6;
    bool operator==(const MapKey &o) const {
        return W == o.W && nrows == o.nrows && nb == o.nb && stride == o.stride && q6 == o.q6;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        uint64_t h = reinterpret_cast<uintptr_t>(k.W) * 0x9E3779B97F4A7C15ull;
        h ^= static_cast<uint64_t>(k.nrows) + 0x7F4A7C15ull + (h << 6) + (h >> 2);
        h ^= static_cast<uint64_t>(k.nb * 131 + k.stride) + (h << 6) + (h >> 2);
        return static_cast<size_t>(h ^ static_cast<uint64_t>(k.q6));
    }
};
constexpr size_t kMapCacheMax = 4096;
thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_map_cache;

bool cached_map(const MapKey &k, CUtensorMap *tm) {
    auto it = g_map_cache.find(k);
    if (it == g_map_cache.end()) return false;
    *tm = it->second;
    return true;
}
void remember_map(const MapKey &k, const CUtensorMap &tm) {
    if (g_map_cache.size() >= kMapCacheMax) g_map_cache.clear();
    g_map_cache.emplace(k, tm);
}

int encode_weight_map(CUtensorMap *tm, const void *W, int64_t nrows, int64_t nb, int64_t row_stride_bytes) {
    const MapKey key{W, nrows, nb, row_stride_bytes, 0};
    if (cached_map(key, tm)) return Q4K_OK;
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return fail(Q4K_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(nb * 36), static_cast<cuuint64_t>(nrows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_bytes)};
    const cuuint32_t box[2] = {36, 32};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void *>(W), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(Q4K_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    remember_map(key, *tm);
    return Q4K_OK;
}

// Q6_K rows as uint64 elements: a box of 210 elements (8 super-blocks,
// 1680 bytes) x 8 rows.  Needs nb % 8 == 0 and a row stride that is a
// multiple of 16 bytes (stride_row_x % 8 == 0).
int encode_q6_map(CUtensorMap *tm, const void *W, int64_t nrows, int64_t nb, int64_t row_stride_bytes) {
    const MapKey key{W, nrows, nb, row_stride_bytes, 1};
    if (cached_map(key, tm)) return Q4K_OK;
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return fail(Q4K_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(nb * kQ6Bytes / 8), static_cast<cuuint64_t>(nrows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride_bytes)};
    const cuuint32_t box[2] = {kQ6RowBytes / 8, kQ6Rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(W), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(Q4K_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    remember_map(key, *tm);
    return Q4K_OK;
}

int validate_job(const Job &j, int ncols, int idx) {
    if (ncols < 1 || ncols > Q4K_MAX_NCOLS)
        return fail(Q4K_EINVAL, "ncols=%d outside 1..%d", ncols, Q4K_MAX_NCOLS);
    if (j.nrows < 0) return fail(Q4K_EINVAL, "task %d: nrows=%lld < 0", idx, (long long)j.nrows);
    if (j.K < 0 || j.K % Q4K_QK_K != 0)
        return fail(Q4K_EINVAL, "task %d: K=%lld is not a non-negative multiple of 256", idx, (long long)j.K);
    if (j.K > (int64_t(1) << 30)) return fail(Q4K_EINVAL, "task %d: K=%lld too large", idx, (long long)j.K);
    if (j.nrows > (int64_t(1) << 30)) return fail(Q4K_EINVAL, "task %d: nrows too large", idx);
    if (j.nrows == 0) return Q4K_OK;
    if (!j.dst) return fail(Q4K_EINVAL, "task %d: null dst", idx);
    if (ncols > 1 && j.stride_col_dst < j.nrows)
        return fail(Q4K_EINVAL, "task %d: stride_col_dst=%lld < nrows", idx, (long long)j.stride_col_dst);
    if (j.q6) {
        if (j.K % (Q4K_QK_K * kQ6AtomSB) != 0)
            return fail(Q4K_EINVAL, "task %d: Q6_K needs K %% 2048 == 0 (K=%lld)", idx, (long long)j.K);
        if (j.stride_row_x % kQ6AtomSB != 0)
            return fail(Q4K_EINVAL, "task %d: Q6_K needs stride_row_x %% 8 == 0 (rows 16-byte aligned)", idx);
        if (j.gate || j.x_bias || j.gate_bias || j.glu_op != Q4K_GLU_NONE)
            return fail(Q4K_EINVAL, "task %d: no fused epilogue with Q6_K weights", idx);
    }
    const bool fused = j.gate || j.x_bias || j.gate_bias || j.glu_op != Q4K_GLU_NONE;
    if (fused) {
        if (j.gate ? (j.glu_op < Q4K_GLU_SWIGLU || j.glu_op > Q4K_GLU_MUL) : j.glu_op != Q4K_GLU_NONE)
            return fail(Q4K_EINVAL, "task %d: glu_op=%d does not match the gate (%s)", idx, j.glu_op,
                        j.gate ? "given" : "absent");
        if (j.gate_bias && !j.gate) return fail(Q4K_EINVAL, "task %d: gate_bias without a gate", idx);
        if (j.gate && !aligned16(j.gate)) return fail(Q4K_EINVAL, "task %d: gate is not 16-byte aligned", idx);
        if (ncols > 1 && (j.x_bias || j.gate_bias) && j.bias_col_stride != 0 && j.bias_col_stride < j.nrows)
            return fail(Q4K_EINVAL, "task %d: stride_col_bias=%lld < nrows", idx, (long long)j.bias_col_stride);
        if (j.bias_col_stride < 0) return fail(Q4K_EINVAL, "task %d: stride_col_bias < 0", idx);
        if (j.K == 0) return fail(Q4K_EINVAL, "task %d: a fused epilogue needs K > 0", idx);
    }
    if (j.norm) {
        if (j.kind != kPrepF32) return fail(Q4K_EINVAL, "task %d: RMSNorm needs fp32 activations", idx);
        if (!(j.norm_eps >= 0.0f) || j.norm_eps > 1.0f)
            return fail(Q4K_EINVAL, "task %d: norm_eps=%g outside [0, 1]", idx, static_cast<double>(j.norm_eps));
    }
    if (j.K == 0) return Q4K_OK;  // empty sums: dst is zeroed
    if (!j.W || !j.src) return fail(Q4K_EINVAL, "task %d: null pointer", idx);
    if (!aligned16(j.W)) return fail(Q4K_EINVAL, "task %d: W is not 16-byte aligned", idx);
    if (j.stride_row_x < j.K / Q4K_QK_K)
        return fail(Q4K_EINVAL, "task %d: stride_row_x=%lld < K/256", idx, (long long)j.stride_row_x);
    if (j.kind == kPrepF32) {
        if (ncols > 1 && j.src_col_stride < j.K)
            return fail(Q4K_EINVAL, "task %d: stride_col_x=%lld < K", idx, (long long)j.src_col_stride);
    } else {
        if (ncols > 1 && j.src_col_stride < j.K / Q4K_QK8_1)
            return fail(Q4K_EINVAL, "task %d: stride_col_y=%lld < K/32", idx, (long long)j.src_col_stride);
    }
    return Q4K_OK;
}

struct Plan {
    PrepParams prep{};
    GemvParams gemv{};
    Layout layout{};
    int64_t n_rowgroups = 0;
    size_t act_bytes = 0;
    int act_of_job[kMaxTasks] = {};
    int n_act = 0;
    bool any_work = false;
    bool any_fused = false;  // a task with a gate or a bias: the epilogue kernel variant
    bool r2 = false;         // the two-rows-per-lane variant (64-row groups)
    bool q6 = false;         // Q6_K weights
    int mode = kModePlain;   // kernel variant
};

// Build the schedule (no device memory touched).  ws may be null (sizing).
// Kernel choice: the measured one, unless the library was built with
// Q4K_SCHED_FORCE (measurement builds only, see the Makefile's variants):
// 1 keeps every launch on the statically partitioned kernel, 2 uses the
// dynamically scheduled one wherever it can run.
#ifndef Q4K_SCHED_FORCE
#define Q4K_SCHED_FORCE 0
#endif
constexpr int kSchedForce = Q4K_SCHED_FORCE;

// ---- single-launch mode (activations quantized into each CTA's shared memory)
// Plain Q4_K tasks with fp32 activations whose blocks can be read in 32-byte
// pieces (32-byte aligned columns), at most kActSmemMaxCols columns.
bool asm_eligible(const Job *jobs, int njobs, int ncols, const Plan &P, bool dump) {
    if (dump || P.q6 || P.any_fused || P.mode != kModePlain || ncols > kActSmemMaxCols) return false;
    for (int i = 0; i < njobs; ++i) {
        const Job &j = jobs[i];
        if (P.act_of_job[i] < 0) continue;
        if (j.kind != kPrepF32 || j.norm || j.gate || j.x_bias || j.q6) return false;
        if ((reinterpret_cast<uintptr_t>(j.src) & 31u) != 0 || (ncols > 1 && j.src_col_stride % 8 != 0)) return false;
    }
    return true;
}

int task_of_atom_host(const GemvParams &G, int64_t a) {
    int t = 0;
    while (t + 1 < G.ntasks && a >= G.task[t + 1].atom_base) ++t;
    return t;
}

// Which activations each CTA's atoms read (the tasks its workers' atom ranges
// span; a bit per activation, into G.cta_act_mask) and the largest table any
// CTA needs (bytes).  The kernel lays its table out from these bits.
int64_t act_smem_need(GemvParams &G, int grid, int ncols) {
    // (worker_begin of the kernel)
    auto wbegin = [&](int64_t w) -> int64_t { return G.natoms * w / G.nworkers; };
    const int R = kActSmemRings;
    auto bytes_of = [&](uint32_t mask) {
        int64_t b = 0;
        for (int a = 0; a < G.n_act; ++a)
            if ((mask >> a) & 1u) b += static_cast<int64_t>(ncols) * G.task[G.act_task[a]].nb * kActSBBytes;
        return b;
    };
    int64_t worst = 0;
    auto begin = wbegin;
    for (int c = 0; c < grid; ++c) {
        uint32_t mask = 0;
        auto add_range = [&](int64_t a0, int64_t a1) {
            if (a1 <= a0) return;
            const int t1 = task_of_atom_host(G, a1 - 1);
            for (int t = task_of_atom_host(G, a0); t <= t1; ++t) mask |= 1u << G.task[t].act_id;
        };
        if (G.packed) {
            // the CTA's workers are consecutive: one contiguous atom range
            const int64_t w0 = static_cast<int64_t>(c) * R;
            const int64_t w1 = w0 + R < G.nworkers ? w0 + R : G.nworkers;
            if (w0 < w1) add_range(begin(w0), begin(w1));
        } else {
            for (int r = 0; r < R; ++r) {
                const int64_t w = static_cast<int64_t>(r) * grid + c;
                if (w < G.nworkers) add_range(begin(w), begin(w + 1));
            }
        }
        G.cta_act_mask[c] = static_cast<uint16_t>(mask);
        const int64_t b = bytes_of(mask);
        if (b > worst) worst = b;
    }
    return worst;
}

// want_dyn: use the dynamically scheduled kernel when the launch qualifies
// (plain or gated Q4_K tasks whose row groups give every warp of a CTA at
// least one atom, and at least two row groups per SM); its tasks are ordered
// by decreasing K.
int make_plan(const Job *jobs, int njobs, int ncols, uint8_t *ws, int num_sms, Plan &P,
              int32_t *dump_T = nullptr, bool dump = false, size_t ws_bytes = 0, bool want_dyn = false,
              bool want_asm = false) {
    if (njobs < 1 || njobs > kMaxTasks) return fail(Q4K_EINVAL, "ntasks=%d outside 1..%d", njobs, kMaxTasks);
    for (int i = 0; i < njobs; ++i) {
        int st = validate_job(jobs[i], ncols, i);
        if (st != Q4K_OK) return st;
    }
    // distinct activations
    struct Act {
        const void *src;
        int64_t K, stride;
        int kind;
        size_t off;
        int norm;
        float eps;
        const float *w;
    };
    Act acts[kMaxTasks];
    P.n_act = 0;
    P.act_bytes = 0;
    for (int i = 0; i < njobs; ++i) {
        const Job &j = jobs[i];
        P.act_of_job[i] = -1;
        if (j.nrows == 0 || j.K == 0) continue;
        int found = -1;
        for (int a = 0; a < P.n_act; ++a)
            if (acts[a].src == j.src && acts[a].K == j.K && acts[a].stride == j.src_col_stride &&
                acts[a].kind == j.kind && acts[a].norm == j.norm &&
                (!j.norm || (acts[a].eps == j.norm_eps && acts[a].w == j.norm_w)))
                found = a;
        if (found < 0) {
            found = P.n_act++;
            acts[found] = {j.src, j.K, j.src_col_stride, j.kind, P.act_bytes, j.norm, j.norm_eps, j.norm_w};
            P.act_bytes += round_up(static_cast<size_t>(ncols) * (j.K / Q4K_QK_K) * kActSBBytes, kAlign);
        }
        P.act_of_job[i] = found;
    }
    // kernel variant: the epilogue one for a gate or bias (a gated task's row
    // groups run over its main matrix, then its gate matrix); else, from
    // kR2Min columns on, 64-row groups with two rows per lane
    P.any_fused = false;
    for (int i = 0; i < njobs; ++i)
        if (P.act_of_job[i] >= 0 && (jobs[i].gate || jobs[i].x_bias)) P.any_fused = true;
    // Q6_K: every task of the launch (one kernel variant per launch)
    P.q6 = jobs[0].q6 != 0;
    for (int i = 1; i < njobs; ++i)
        if ((jobs[i].q6 != 0) != P.q6) return fail(Q4K_EINVAL, "Q4_K and Q6_K tasks in one launch");
    if (P.q6 && dump) return fail(Q4K_EINVAL, "no sub-block dump for Q6_K");
    P.r2 = !P.q6 && !dump && !P.any_fused && ncols >= kR2Min && split_for(ncols) == 1;
    P.mode = dump ? kModeDump : P.any_fused ? kModeGated : P.q6 ? kModeQ6 : P.r2 ? kModeR2 : kModePlain;
    if (want_dyn && !dump && !P.q6) {
        const bool gated = P.any_fused;
        const int R = rings_dyn(ncols, gated);
        int64_t G = 0, natoms = 0;
        bool fits = true;
        for (int i = 0; i < njobs; ++i) {
            if (P.act_of_job[i] < 0) continue;
            const int64_t nb = jobs[i].K / Q4K_QK_K;
            const int64_t apr = (jobs[i].gate ? 2 : 1) * ((nb + kKS - 1) / kKS);
            if (apr < R) fits = false;
            G += (jobs[i].nrows + 31) / 32;
            natoms += (jobs[i].nrows + 31) / 32 * apr;
        }
        // Measured on B200 (chained launches of one 14336 x 4096 matrix, us):
        // ncols 1 11.8 -> 10.8, 2 13.5 -> 12.5, 4 17.2 -> 17.1, 8 24.5 -> 34.8;
        // whole Mistral / Llama-3 layers and the 128256-row head 7-12 % slower
        // (their per-warp streams cut into shares of one or two atoms per
        // group).  So: one or two columns, and only where the static kernel
        // spreads fewer than four atoms per worker over the SMs.
        const bool spread = natoms < 4 * static_cast<int64_t>(num_sms) * rings_for(ncols);
        const bool measured_win = spread && ncols <= 2;
        if (fits && (measured_win || kSchedForce == 2) && G >= kDynAhead * static_cast<int64_t>(num_sms) &&
            G < (int64_t{1} << 30)) {
            P.r2 = false;
            P.mode = gated ? kModeDynGated : kModeDynPlain;
        }
    }
    const bool dyn = is_dyn(P.mode);
    const int64_t group_rows = P.r2 ? 64 : P.q6 ? kQ6Rows : 32;
    // task order: as given, or by decreasing K (stable) for the dynamic kernel
    int ord[kMaxTasks];
    for (int i = 0; i < njobs; ++i) ord[i] = i;
    if (dyn) {
        for (int a = 1; a < njobs; ++a)
            for (int b = a; b > 0 && jobs[ord[b]].K > jobs[ord[b - 1]].K; --b) {
                const int tmp = ord[b];
                ord[b] = ord[b - 1];
                ord[b - 1] = tmp;
            }
    }
    // row groups and atoms
    int64_t atoms = 0, rgs = 0;
    int nt = 0;
    int ngated = 0;
    for (int ii = 0; ii < njobs; ++ii) {
        const int i = ord[ii];
        const Job &j = jobs[i];
        if (P.act_of_job[i] < 0) continue;
        const int64_t groups = (j.nrows + group_rows - 1) / group_rows;
        const int64_t nb = j.K / Q4K_QK_K;
        // a two-row atom is one super-block of 64 rows, a plain one kKS
        // super-blocks of 32 rows (a gated task: those of both matrices)
        const int64_t half = (nb + kKS - 1) / kKS;
        const int64_t apr = P.q6 ? nb / kQ6AtomSB : P.r2 ? nb : j.gate ? 2 * half : half;
        TaskDesc &T = P.gemv.task[nt++];
        T.W = static_cast<const uint8_t *>(j.W);
        T.dst = j.dst;
        T.row_stride = j.stride_row_x * (P.q6 ? kQ6Bytes : Q4K_BLOCK_BYTES);
        T.act_col_stride = nb * kActSBBytes;
        T.dst_col_stride = j.stride_col_dst;
        T.atom_base = atoms;
        T.nrows = static_cast<int32_t>(j.nrows);
        T.nb = static_cast<int32_t>(nb);
        T.apr = static_cast<int32_t>(apr);
        T.rg_base = static_cast<int32_t>(rgs);
        T.ngroups = static_cast<int32_t>(groups);
        T.act_id = P.act_of_job[i];
        T.x = j.kind == kPrepF32 ? static_cast<const float *>(j.src) : nullptr;
        T.x_col_stride = j.src_col_stride;
        T.has_gate = j.gate ? 1 : 0;
        T.gate_map = j.gate ? ngated : -1;
        T.half = j.gate ? static_cast<int32_t>(half) : 0;
        if (j.gate && ++ngated > kMaxGated)
            return fail(Q4K_EINVAL, "more than %d tasks with a fused gate in one launch", kMaxGated);
        T.glu_op = j.glu_op;
        T.x_bias = j.x_bias;
        T.gate_bias = j.gate_bias;
        T.bias_col_stride = j.bias_col_stride;
        atoms += groups * apr;
        rgs += groups;
    }
    P.n_rowgroups = rgs;
    P.any_work = atoms > 0;
    P.gemv.ntasks = nt;
    P.gemv.natoms = atoms;
    // Partition units: the CTAs (one per SM) in the balanced partition of
    // the epilogue variant; single warps otherwise (CTA-contiguous ranges for
    // large problems, consecutive workers on different SMs for small ones).
    // The dynamic kernel hands out row groups instead.
    // Every unit holds at least one atom (the count of a split row group's
    // contributors is the span of their units); CTAs past nworkers idle.
    const bool queue = is_queue(P.mode);
    const int64_t max_workers = static_cast<int64_t>(num_sms) * (queue ? 1 : rings_m(ncols, P.mode));
    const int64_t nw = atoms < max_workers ? atoms : max_workers;
    P.gemv.nworkers = static_cast<int32_t>(nw);
    P.gemv.packed = !queue && atoms >= 4 * max_workers ? 1 : 0;
    P.gemv.pad0_ = 0;
    // partial slots hold the gate sums beside the main ones (a launch with a
    // gate), or the second row's (two-row launches)
    P.gemv.pcols = (P.any_fused || P.r2) ? 2 * ncols : ncols;
    P.gemv.dyn_groups = dyn ? static_cast<int32_t>(rgs) : 0;
    // two partial slots per unit; the dynamic kernel keeps its row groups
    // inside one CTA and needs none (so the sizing plan, made for the static
    // kernel with an upper bound on the SMs, covers whichever kernel runs)
    P.layout = make_layout(rgs, P.gemv.pcols, P.act_bytes, dyn ? 0 : 2 * nw);
    // distinct activations: a task that reads each
    P.gemv.n_act = P.n_act;
    for (int a = 0; a < kMaxTasks; ++a) P.gemv.act_task[a] = -1;
    for (int t = 0; t < nt; ++t)
        if (P.gemv.act_task[P.gemv.task[t].act_id] < 0) P.gemv.act_task[P.gemv.task[t].act_id] = t;
    P.gemv.act_smem_bytes = 0;
    if (want_asm && num_sms <= kMaxPlanCtas && asm_eligible(jobs, njobs, ncols, P, dump)) {
        for (int a = 0; a < kMaxTasks; ++a) {
            const int t = P.gemv.act_task[a];
            P.gemv.act_x[a] = t >= 0 ? P.gemv.task[t].x : nullptr;
            P.gemv.act_xcs[a] = t >= 0 ? P.gemv.task[t].x_col_stride : 0;
            P.gemv.act_nb[a] = t >= 0 ? P.gemv.task[t].nb : 0;
            P.gemv.task_act[a] = static_cast<int8_t>(a < nt ? P.gemv.task[a].act_id : -1);
        }
        const int64_t need = act_smem_need(P.gemv, num_sms, ncols);
        if (need <= kActSmemCap) {
            P.mode = kModeActSmem;
            P.gemv.act_smem_bytes = static_cast<int32_t>(round_up(static_cast<size_t>(need), 128));
        }
    }
    if (ws == nullptr) return Q4K_OK;
    if (ws_bytes < P.layout.total)
        return fail(Q4K_EWORKSPACE, "workspace of %zu bytes < %zu required", ws_bytes, P.layout.total);

    // pointers into the workspace
    P.gemv.status = reinterpret_cast<int32_t *>(ws);
    P.gemv.counters = reinterpret_cast<int32_t *>(ws + P.layout.counters_off);
    // header word 16 (bytes 64..67): the dynamic kernel's ticket counter,
    // cleared with the header by every quantization launch
    P.gemv.dyn_claim = reinterpret_cast<int32_t *>(ws + 64);
    P.gemv.partials = reinterpret_cast<float *>(ws + P.layout.partials_off);
    P.gemv.dump_S = nullptr;
    nt = 0;
    for (int ii = 0; ii < njobs; ++ii) {
        const int i = ord[ii];
        if (P.act_of_job[i] < 0) continue;
        const Job &j = jobs[i];
        int st = j.q6 ? encode_q6_map(&P.gemv.tmap[nt], j.W, j.nrows, j.K / Q4K_QK_K, j.stride_row_x * kQ6Bytes)
                      : encode_weight_map(&P.gemv.tmap[nt], j.W, j.nrows, j.K / Q4K_QK_K,
                                          j.stride_row_x * Q4K_BLOCK_BYTES);
        if (st != Q4K_OK) return st;
        if (j.gate) {
            const int gm = P.gemv.task[nt].gate_map;
            st = encode_weight_map(&P.gemv.tmap_gate[gm], j.gate, j.nrows, j.K / Q4K_QK_K,
                                   j.stride_row_x * Q4K_BLOCK_BYTES);
            if (st != Q4K_OK) return st;
        }
        P.gemv.task[nt++].act = ws + P.layout.act_off + acts[P.act_of_job[i]].off;
    }
    // prep jobs: one per distinct activation
    int64_t items = 0;
    int32_t norm_ctas = 0;
    for (int a = 0; a < P.n_act; ++a) {
        PrepJob &J = P.prep.job[a];
        J.src = acts[a].src;
        J.act = ws + P.layout.act_off + acts[a].off;
        J.q81_out = nullptr;
        J.dump_T = dump_T;
        J.src_col_stride = acts[a].stride;
        J.act_col_stride = (acts[a].K / Q4K_QK_K) * kActSBBytes;
        J.q81_col_stride = 0;
        J.item_base = items;
        J.K = static_cast<int32_t>(acts[a].K);
        J.nblk = static_cast<int32_t>(acts[a].K / Q4K_QK8_1);
        J.ncols = ncols;
        J.kind = acts[a].kind;
        J.norm = acts[a].norm;
        J.norm_eps = acts[a].eps;
        J.norm_w = acts[a].w;
        J.pad_ = 0;
        if (J.norm) {
            J.cta_base = norm_ctas;  // one CTA per column; no warp items
            norm_ctas += ncols;
        } else {
            J.cta_base = 0;
            items += static_cast<int64_t>(ncols) * J.nblk;
        }
    }
    P.prep.njobs = P.n_act;
    P.prep.nitems = items;
    P.prep.norm_ctas = norm_ctas;
    P.prep.pad_ = 0;
    P.prep.zero_ptr = reinterpret_cast<int32_t *>(ws);
    P.prep.zero_count = static_cast<int32_t>((P.layout.counters_off + rgs * 4) / 4);
    return Q4K_OK;
}

// Zero the outputs of empty-K tasks (an empty sum).
int zero_outputs(const Job *jobs, int njobs, int ncols, cudaStream_t s) {
    for (int i = 0; i < njobs; ++i) {
        const Job &j = jobs[i];
        if (j.K != 0 || j.nrows == 0) continue;
        for (int c = 0; c < ncols; ++c) {
            cudaError_t e = cudaMemsetAsync(j.dst + c * j.stride_col_dst, 0, j.nrows * sizeof(float), s);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
        }
    }
    return Q4K_OK;
}

int validate_gather(const q4k_gather *g) {
    if (!g) return fail(Q4K_EINVAL, "gather descriptor is null");
    if (g->world < 1 || g->world > Q4K_MAX_PEERS) return fail(Q4K_EINVAL, "gather world=%d outside 1..8", g->world);
    if (g->rank < 0 || g->rank >= g->world) return fail(Q4K_EINVAL, "gather rank=%d outside 0..world-1", g->rank);
    if (!g->out_local || !g->epoch) return fail(Q4K_EINVAL, "gather out_local/epoch is null");
    for (int q = 0; q < g->world; ++q)
        if (!g->out_peer[q] || !g->flags_peer[q]) return fail(Q4K_EINVAL, "gather peer %d pointers are null", q);
    if (g->out_peer[g->rank] != g->out_local) return fail(Q4K_EINVAL, "gather out_peer[rank] != out_local");
    if (g->out_elems < 0) return fail(Q4K_EINVAL, "gather out_elems < 0");
    return Q4K_OK;
}

// Every output of a gathering call is also stored at the same offset in every
// peer's buffer, so each task's dst columns must lie inside the full buffer:
// [dst, dst + (ncols-1)*stride_col_dst + nrows) within [out_local, out_local + out_elems).
int validate_gather_tasks(const q4k_gather *g, const q4k_task *tasks, int ntasks, int ncols) {
    const intptr_t base = reinterpret_cast<intptr_t>(g->out_local);
    for (int i = 0; i < ntasks; ++i) {
        const q4k_task &t = tasks[i];
        if (t.nrows <= 0) continue;
        const intptr_t d = reinterpret_cast<intptr_t>(t.dst);
        if (d < base || (d - base) % static_cast<intptr_t>(sizeof(float)) != 0)
            return fail(Q4K_EINVAL, "task %d: dst is not a float inside the gather buffer out_local", i);
        const int64_t off = static_cast<int64_t>((d - base) / static_cast<intptr_t>(sizeof(float)));
        if (ncols > 1 && t.stride_col_dst < t.nrows)
            return fail(Q4K_EINVAL, "task %d: stride_col_dst=%lld < nrows", i, (long long)t.stride_col_dst);
        const int64_t end = off + static_cast<int64_t>(ncols - 1) * (ncols > 1 ? t.stride_col_dst : 0) + t.nrows;
        if (end > g->out_elems)
            return fail(Q4K_EINVAL, "task %d: outputs [%lld, %lld) reach past the gather buffer's %lld floats", i,
                        (long long)off, (long long)end, (long long)g->out_elems);
    }
    return Q4K_OK;
}

GatherWait gather_wait_of(const q4k_gather *g, void *workspace) {
    GatherWait w{};
    if (g == nullptr || g->world <= 1) return w;
    w.flags = g->flags_peer[g->rank];
    w.epoch = g->epoch;
    w.status = static_cast<int32_t *>(workspace);
    w.world = g->world;
    w.rank = g->rank;
    return w;
}

#if Q4K_TIMELINE
// Launch timeline records: one buffer per device, allocated by the first call
// on that device (a diagnostic build; the release library has none of this).
std::mutex g_tl_mu;
constexpr int kTlDevices = 64;
unsigned long long *g_tl[kTlDevices] = {};
int g_tl_calls[kTlDevices] = {};
constexpr size_t kTlGemvWords = static_cast<size_t>(Q4K_TIMELINE_SLOTS) * Q4K_TIMELINE_CTAS * 16 * 8;
constexpr size_t kTlPrepWords = static_cast<size_t>(Q4K_TIMELINE_SLOTS) * Q4K_TIMELINE_PREP_CTAS * 4;
constexpr size_t kTlBytes = (kTlGemvWords + kTlPrepWords) * sizeof(unsigned long long);

int tl_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= kTlDevices) return fail(Q4K_EINVAL, "device %d beyond the timeline table", *dev);
    return Q4K_OK;
}

// Points the launch parameters at the next ring slot of the current device's
// buffer.  The first call on a device allocates and clears the buffer
// (synchronously: not inside a graph capture).
int timeline_attach(Plan &P) {
    int dev = 0;
    int st = tl_device(&dev);
    if (st != Q4K_OK) return st;
    std::lock_guard<std::mutex> lk(g_tl_mu);
    if (g_tl[dev] == nullptr) {
        cudaError_t e = cudaMalloc(&g_tl[dev], kTlBytes);
        if (e == cudaSuccess) e = cudaMemset(g_tl[dev], 0, kTlBytes);
        if (e != cudaSuccess) return cuda_fail(e, "timeline buffer");
    }
    const int slot = g_tl_calls[dev]++ % Q4K_TIMELINE_SLOTS;
    P.gemv.tl = g_tl[dev];
    P.gemv.tl_slot = slot;
    P.prep.tl = g_tl[dev] + kTlGemvWords;
    P.prep.tl_slot = slot;
    return Q4K_OK;
}
#endif


// fused: run the batch as one launch that quantizes the activations itself
// (kModeActSmem) where the tasks allow it, else as the two-launch sequence;
// the workspace's status word, gather count and split counters must be zero
// on entry, which every completed call leaves them.
int run(const Job *jobs, int njobs, int ncols, void *workspace, size_t ws_bytes, cudaStream_t s,
        int32_t *dump_S = nullptr, int32_t *dump_T = nullptr, const q4k_gather *gather = nullptr,
        bool fused = false) {
    Plan P;
    // Arguments are validated before the device is touched.
    const bool dump = dump_S != nullptr;
    int st = make_plan(jobs, njobs, ncols, nullptr, kFallbackSMs, P, nullptr, dump);
    if (st != Q4K_OK) return st;
    int num_sms = 0;
    cudaError_t e = device_setup(&num_sms);
    if (e != cudaSuccess) return cuda_fail(e, "device setup");
    st = zero_outputs(jobs, njobs, ncols, s);
    if (st != Q4K_OK) return st;
    // With a fused all-gather the launch happens even without local rows: the
    // peers wait for this rank's epoch flag.
    const bool gathering = gather && gather->world > 1;
    if (!P.any_work && !gathering) return Q4K_OK;
    if (workspace == nullptr) return fail(Q4K_EWORKSPACE, "workspace is null");
    if (!aligned16(workspace)) return fail(Q4K_EWORKSPACE, "workspace is not 16-byte aligned");
    // The device's plan (its SM count fixes the workers and the layout); the
    // workspace size is checked before any pointer into it is formed.
    st = make_plan(jobs, njobs, ncols, static_cast<uint8_t *>(workspace), num_sms, P, dump_T, dump, ws_bytes,
                   !fused && !gathering && kSchedForce != 1, fused);
    if (st != Q4K_OK) return st;
    P.gemv.dump_S = dump_S;
    P.gemv.gworld = 1;
    if (gather && gather->world > 1) {
        P.gemv.gworld = gather->world;
        P.gemv.grank = gather->rank;
        P.gemv.gout_local = gather->out_local;
        for (int q = 0; q < gather->world; ++q) {
            P.gemv.gout_peer[q] = gather->out_peer[q];
            P.gemv.gflags_peer[q] = gather->flags_peer[q];
        }
        P.gemv.gepoch = gather->epoch;
        P.gemv.gdone = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(workspace) + 4);
        P.prep.gwait = gather_wait_of(gather, workspace);
        P.gemv.gwait = P.prep.gwait;
    }
#if Q4K_TIMELINE
    if ((st = timeline_attach(P)) != Q4K_OK) return st;
#endif
    if (P.mode != kModeActSmem && (e = launch_prep(P.prep, s)) != cudaSuccess) return cuda_fail(e, "prep launch");
    const int mode = P.mode;
    if ((e = launch_gemv(P.gemv, ncols, mode, num_sms, s)) != cudaSuccess)
        return cuda_fail(e, "gemv launch");
    return Q4K_OK;
}

Job job_of(const q4k_task_ex &t) {
    Job j{t.t.W, t.t.x, t.t.dst, t.t.nrows, t.t.K, t.t.stride_row_x, t.t.stride_col_x, t.t.stride_col_dst, kPrepF32};
    j.gate = t.W_gate;
    j.x_bias = t.x_bias;
    j.gate_bias = t.gate_bias;
    j.bias_col_stride = t.stride_col_bias;
    j.glu_op = t.glu_op;
    j.norm = t.rms_norm;
    j.norm_eps = t.norm_eps;
    j.norm_w = t.norm_weight;
    return j;
}

size_t plan_bytes(const Job *jobs, int njobs, int ncols) {
    Plan P;
    if (make_plan(jobs, njobs, ncols, nullptr, num_sms_or_bound(), P) != Q4K_OK) return 0;
    return P.layout.total;
}

}  // namespace

namespace q4k {
// Lets other translation units of the library report through q4k_last_error().
void set_last_error_message(const char *msg) { g_last_error = msg; }
}  // namespace q4k

extern "C" {

const char *q4k_status_string(int status) {
    switch (status) {
        case Q4K_OK: return "Q4K_OK";
        case Q4K_EINVAL: return "Q4K_EINVAL";
        case Q4K_ECUDA: return "Q4K_ECUDA";
        case Q4K_ETIMEOUT: return "Q4K_ETIMEOUT";
        case Q4K_ENCCL: return "Q4K_ENCCL";
        case Q4K_EWORKSPACE: return "Q4K_EWORKSPACE";
        default: return "Q4K_UNKNOWN";
    }
}

const char *q4k_last_error(void) { return g_last_error.c_str(); }

int q4k_version(void) { return 100; }

int q4k_device_supported(void) {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return 0; }
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return major == 10 && minor == 0;
}

size_t q4k_row_bytes(int64_t K) {
    if (K < 0 || K % Q4K_QK_K) return 0;
    return static_cast<size_t>(K / Q4K_QK_K) * Q4K_BLOCK_BYTES;
}

size_t q4k_q8_1_bytes(int64_t Kpad, int ncols) {
    if (Kpad < 0 || Kpad % Q4K_QK8_1 || ncols < 0) return 0;
    return static_cast<size_t>(Kpad / Q4K_QK8_1) * Q8_1_BLOCK_BYTES * ncols;
}

size_t q4k_gemv_workspace_bytes(int64_t nrows, int64_t K, int ncols) {
    static const float dummy = 0.0f;
    static float dummy_out = 0.0f;
    Job j{reinterpret_cast<const void *>(uintptr_t(256)), &dummy, &dummy_out, nrows, K, K / Q4K_QK_K,
          K, nrows, kPrepF32};
    return plan_bytes(&j, 1, ncols);
}

size_t q4k_batch_workspace_bytes(const q4k_task *tasks, int ntasks, int ncols) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return 0;
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i)
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
    return plan_bytes(jobs, ntasks, ncols);
}

int q4k_quantize_q8_1(const float *x, int64_t K, int64_t stride_col_x, int64_t Kpad, int ncols,
                      void *y_q8_1, q4k_stream_t stream) {
    if (ncols < 1 || ncols > Q4K_MAX_NCOLS) return fail(Q4K_EINVAL, "ncols=%d outside 1..8", ncols);
    if (K < 0 || Kpad < K || Kpad % Q4K_QK8_1 || Kpad > (int64_t(1) << 30))
        return fail(Q4K_EINVAL, "need 0 <= K <= Kpad, Kpad %% 32 == 0 (K=%lld Kpad=%lld)", (long long)K,
                    (long long)Kpad);
    if (Kpad == 0) return Q4K_OK;
    if (!y_q8_1 || (K > 0 && !x)) return fail(Q4K_EINVAL, "null pointer");
    if (ncols > 1 && stride_col_x < K) return fail(Q4K_EINVAL, "stride_col_x < K");
    int num_sms = 0;
    cudaError_t e = device_setup(&num_sms);
    if (e != cudaSuccess) return cuda_fail(e, "device setup");
    PrepParams p{};
    PrepJob &J = p.job[0];
    J.src = x;
    J.act = nullptr;
    J.q81_out = static_cast<uint8_t *>(y_q8_1);
    J.dump_T = nullptr;
    J.src_col_stride = stride_col_x;
    J.q81_col_stride = Kpad / Q4K_QK8_1;
    J.item_base = 0;
    J.K = static_cast<int32_t>(K);
    J.nblk = static_cast<int32_t>(Kpad / Q4K_QK8_1);
    J.ncols = ncols;
    J.kind = kPrepF32;
    p.njobs = 1;
    p.nitems = static_cast<int64_t>(ncols) * J.nblk;
    p.zero_ptr = nullptr;
    p.zero_count = 0;
    if ((e = launch_prep(p, reinterpret_cast<cudaStream_t>(stream))) != cudaSuccess)
        return cuda_fail(e, "quantize launch");
    return Q4K_OK;
}

int q4k_rms_norm_quantize_q8_1(const float *x, int64_t K, int64_t stride_col_x, int64_t Kpad, int ncols,
                               const float *norm_weight, float eps, void *y_q8_1, q4k_stream_t stream) {
    if (ncols < 1 || ncols > Q4K_MAX_NCOLS) return fail(Q4K_EINVAL, "ncols=%d outside 1..8", ncols);
    if (K < 1 || Kpad < K || Kpad % Q4K_QK8_1 || Kpad > (int64_t(1) << 30))
        return fail(Q4K_EINVAL, "need 0 < K <= Kpad, Kpad %% 32 == 0 (K=%lld Kpad=%lld)", (long long)K,
                    (long long)Kpad);
    if (!x || !y_q8_1) return fail(Q4K_EINVAL, "null pointer");
    if (ncols > 1 && stride_col_x < K) return fail(Q4K_EINVAL, "stride_col_x < K");
    if (!(eps >= 0.0f) || eps > 1.0f) return fail(Q4K_EINVAL, "eps=%g outside [0, 1]", static_cast<double>(eps));
    int num_sms = 0;
    cudaError_t e = device_setup(&num_sms);
    if (e != cudaSuccess) return cuda_fail(e, "device setup");
    PrepParams p{};
    PrepJob &J = p.job[0];
    J.src = x;
    J.act = nullptr;
    J.q81_out = static_cast<uint8_t *>(y_q8_1);
    J.dump_T = nullptr;
    J.src_col_stride = stride_col_x;
    J.q81_col_stride = Kpad / Q4K_QK8_1;
    J.item_base = 0;
    J.K = static_cast<int32_t>(K);
    J.nblk = static_cast<int32_t>(Kpad / Q4K_QK8_1);
    J.ncols = ncols;
    J.kind = kPrepF32;
    J.norm = 1;
    J.norm_eps = eps;
    J.norm_w = norm_weight;
    J.cta_base = 0;
    p.njobs = 1;
    p.nitems = 0;
    p.norm_ctas = ncols;
    p.zero_ptr = nullptr;
    p.zero_count = 0;
    if ((e = launch_prep(p, reinterpret_cast<cudaStream_t>(stream))) != cudaSuccess)
        return cuda_fail(e, "rms-norm quantize launch");
    return Q4K_OK;
}

int q4k_mul_mat_vec_q8_1(const void *W, const void *y_q8_1, float *dst, int64_t K, int64_t nrows, int ncols,
                         int64_t stride_row_x, int64_t stride_col_y, int64_t stride_col_dst, void *workspace,
                         size_t workspace_bytes, q4k_stream_t stream) {
    Job j{W, y_q8_1, dst, nrows, K, stride_row_x, stride_col_y, stride_col_dst, kPrepQ81};
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int q4k_mul_mat_vec(const void *W, const float *x, float *dst, int64_t K, int64_t nrows, int ncols,
                    int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst, void *workspace,
                    size_t workspace_bytes, q4k_stream_t stream) {
    Job j{W, x, dst, nrows, K, stride_row_x, stride_col_x, stride_col_dst, kPrepF32};
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int q4k_op_mul_mat_vec_q(const void *W_slice, int64_t K, const void *y_q8_1, float *dst_slice, int64_t row_low,
                         int64_t row_high, int64_t src1_ncols, int64_t src1_padded_row_size, int64_t nrows_dst,
                         void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    if (row_high < row_low) return fail(Q4K_EINVAL, "row_high < row_low");
    if (src1_padded_row_size < K || src1_padded_row_size % Q4K_QK8_1)
        return fail(Q4K_EINVAL, "src1_padded_row_size must be >= K and a multiple of 32");
    if (src1_ncols < 1 || src1_ncols > Q4K_MAX_NCOLS)
        return fail(Q4K_EINVAL, "src1_ncols=%lld outside 1..8", (long long)src1_ncols);
    const int64_t rows = row_high - row_low;
    if (nrows_dst < rows) return fail(Q4K_EINVAL, "nrows_dst < row_high - row_low");
    Job j{W_slice, y_q8_1, dst_slice, rows, K, K / Q4K_QK_K, src1_padded_row_size / Q4K_QK8_1, nrows_dst,
          kPrepQ81};
    return run(&j, 1, static_cast<int>(src1_ncols), workspace, workspace_bytes,
               reinterpret_cast<cudaStream_t>(stream));
}

int q4k_custom_q4k_gemv(const void *vx, const void *vy, float *dst, int num_blocks_total, int stride_col_y_blocks,
                        int stride_col_dst, int ncols_dst, void *workspace, size_t workspace_bytes,
                        q4k_stream_t stream) {
    if (num_blocks_total < 0) return fail(Q4K_EINVAL, "num_blocks_total < 0");
    Job j{vx, vy, dst, stride_col_dst, static_cast<int64_t>(num_blocks_total) * Q4K_QK_K, num_blocks_total,
          stride_col_y_blocks, stride_col_dst, kPrepQ81};
    return run(&j, 1, ncols_dst, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int q4k_gemv_batch(const q4k_task *tasks, int ntasks, int ncols, void *workspace, size_t workspace_bytes,
                   q4k_stream_t stream) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i)
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
    return run(jobs, ntasks, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

// Kernel id of a plan: its variant, told apart for two-row launches by
// where their integer sums run.
static int kernel_id(int mode, int ncols) {
    return (mode == kModeR2 && Q4K_R2_MMA && ncols >= kR2MmaMin) ? Q4K_KERNEL_STATIC_TWO_ROW_MMA : mode;
}

int q4k_batch_ex_kernel(const q4k_task_ex *tasks, int ntasks, int ncols, int num_sms) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) {
        fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
        return -1;
    }
    if (num_sms < 1 || num_sms > 4096) {
        fail(Q4K_EINVAL, "num_sms=%d outside 1..4096", num_sms);
        return -1;
    }
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) jobs[i] = job_of(tasks[i]);
    Plan P;
    // the decision run() makes for a plain (not single-launch, not gathering) call
    if (make_plan(jobs, ntasks, ncols, nullptr, num_sms, P, nullptr, false, 0, kSchedForce != 1) != Q4K_OK)
        return -1;
    static_assert(Q4K_KERNEL_STATIC == kModePlain && Q4K_KERNEL_STATIC_GATED == kModeGated &&
                      Q4K_KERNEL_STATIC_TWO_ROW == kModeR2 && Q4K_KERNEL_DYNAMIC == kModeDynPlain &&
                      Q4K_KERNEL_DYNAMIC_GATED == kModeDynGated,
                  "kernel ids");
    return kernel_id(P.mode, ncols);
}

int q4k_batch_persistent_kernel(const q4k_task *tasks, int ntasks, int ncols, int num_sms) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) {
        fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
        return -1;
    }
    if (num_sms < 1 || num_sms > 4096) {
        fail(Q4K_EINVAL, "num_sms=%d outside 1..4096", num_sms);
        return -1;
    }
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i)
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
    Plan P;
    // the decision run() makes for q4k_gemv_batch_persistent
    if (make_plan(jobs, ntasks, ncols, nullptr, num_sms, P, nullptr, false, 0, false, true) != Q4K_OK) return -1;
    static_assert(Q4K_KERNEL_SINGLE_LAUNCH == kModeActSmem, "kernel ids");
    return kernel_id(P.mode, ncols);
}

size_t q4k_batch_ex_workspace_bytes(const q4k_task_ex *tasks, int ntasks, int ncols) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return 0;
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) jobs[i] = job_of(tasks[i]);
    return plan_bytes(jobs, ntasks, ncols);
}

int q4k_gemv_batch_ex(const q4k_task_ex *tasks, int ntasks, int ncols, void *workspace, size_t workspace_bytes,
                      q4k_stream_t stream) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) jobs[i] = job_of(tasks[i]);
    return run(jobs, ntasks, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t q4k_gemv_fused_workspace_bytes(int64_t nrows, int64_t K, int ncols) {
    static const float dummy = 0.0f;
    static float dummy_out = 0.0f;
    Job j{reinterpret_cast<const void *>(uintptr_t(256)), &dummy, &dummy_out, nrows, K, K / Q4K_QK_K,
          K, nrows, kPrepF32};
    j.gate = reinterpret_cast<const void *>(uintptr_t(256));
    j.glu_op = Q4K_GLU_SWIGLU;
    return plan_bytes(&j, 1, ncols);
}

int q4k_mul_mat_vec_q8_1_fused(const void *W, const void *W_gate, const void *y_q8_1, float *dst, int64_t K,
                               int64_t nrows, int ncols, int64_t stride_row_x, int64_t stride_col_y,
                               int64_t stride_col_dst, const float *x_bias, const float *gate_bias, int glu_op,
                               void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    Job j{W, y_q8_1, dst, nrows, K, stride_row_x, stride_col_y, stride_col_dst, kPrepQ81};
    j.gate = W_gate;
    j.x_bias = x_bias;
    j.gate_bias = gate_bias;
    j.bias_col_stride = stride_col_dst;  // x_bias[j*stride_col_dst + row], kernels/mmvq.cu:211
    j.glu_op = glu_op;
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int q4k_mul_mat_vec_fused(const void *W, const void *W_gate, const float *x, float *dst, int64_t K, int64_t nrows,
                          int ncols, int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst,
                          const float *x_bias, const float *gate_bias, int glu_op, void *workspace,
                          size_t workspace_bytes, q4k_stream_t stream) {
    Job j{W, x, dst, nrows, K, stride_row_x, stride_col_x, stride_col_dst, kPrepF32};
    j.gate = W_gate;
    j.x_bias = x_bias;
    j.gate_bias = gate_bias;
    j.bias_col_stride = stride_col_dst;
    j.glu_op = glu_op;
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t q4k_q6_k_workspace_bytes(int64_t nrows, int64_t K, int ncols) {
    static const float dummy = 0.0f;
    static float dummy_out = 0.0f;
    Job j{reinterpret_cast<const void *>(uintptr_t(256)), &dummy, &dummy_out, nrows, K, K / Q4K_QK_K,
          K, nrows, kPrepF32};
    j.q6 = 1;
    return plan_bytes(&j, 1, ncols);
}

int q4k_mul_mat_vec_q6_k(const void *W, const float *x, float *dst, int64_t K, int64_t nrows, int ncols,
                         int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst, void *workspace,
                         size_t workspace_bytes, q4k_stream_t stream) {
    Job j{W, x, dst, nrows, K, stride_row_x, stride_col_x, stride_col_dst, kPrepF32};
    j.q6 = 1;
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int q4k_mul_mat_vec_q6_k_q8_1(const void *W, const void *y_q8_1, float *dst, int64_t K, int64_t nrows, int ncols,
                              int64_t stride_row_x, int64_t stride_col_y, int64_t stride_col_dst, void *workspace,
                              size_t workspace_bytes, q4k_stream_t stream) {
    Job j{W, y_q8_1, dst, nrows, K, stride_row_x, stride_col_y, stride_col_dst, kPrepQ81};
    j.q6 = 1;
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t q4k_batch_q6_k_workspace_bytes(const q4k_task *tasks, int ntasks, int ncols) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return 0;
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) {
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
        jobs[i].q6 = 1;
    }
    return plan_bytes(jobs, ntasks, ncols);
}

int q4k_gemv_batch_q6_k(const q4k_task *tasks, int ntasks, int ncols, void *workspace, size_t workspace_bytes,
                        q4k_stream_t stream) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) {
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
        jobs[i].q6 = 1;
    }
    return run(jobs, ntasks, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int q4k_gemv_batch_allgather(const q4k_task *tasks, int ntasks, int ncols, const q4k_gather *gather,
                             void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
    int st = validate_gather(gather);
    if (st == Q4K_OK) st = validate_gather_tasks(gather, tasks, ntasks, ncols);
    if (st != Q4K_OK) return st;
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) {
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
        if (tasks[i].nrows > 0 && tasks[i].K == 0)
            return fail(Q4K_EINVAL, "task %d: K = 0 is not supported with a fused all-gather", i);
    }
    return run(jobs, ntasks, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr,
               nullptr, gather);
}

int q4k_gather_wait(const q4k_gather *gather, void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    int st = validate_gather(gather);
    if (st != Q4K_OK) return st;
    if (workspace == nullptr || workspace_bytes < 4) return fail(Q4K_EWORKSPACE, "workspace is null or too small");
    if (!aligned16(workspace)) return fail(Q4K_EWORKSPACE, "workspace is not 16-byte aligned");
    if (gather->world <= 1) return Q4K_OK;
    cudaError_t e = launch_gather_wait(gather_wait_of(gather, workspace), reinterpret_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? Q4K_OK : cuda_fail(e, "gather wait launch");
}

int q4k_workspace_init(void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    if (workspace == nullptr || workspace_bytes == 0) return fail(Q4K_EWORKSPACE, "workspace is null or empty");
    if (!aligned16(workspace)) return fail(Q4K_EWORKSPACE, "workspace is not 16-byte aligned");
    cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    return Q4K_OK;
}

int q4k_gemv_batch_persistent(const q4k_task *tasks, int ntasks, int ncols, const q4k_gather *gather,
                              void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    if (!tasks || ntasks < 1 || ntasks > kMaxTasks) return fail(Q4K_EINVAL, "ntasks=%d outside 1..16", ntasks);
    if (gather) {
        int st = validate_gather(gather);
        if (st == Q4K_OK) st = validate_gather_tasks(gather, tasks, ntasks, ncols);
        if (st != Q4K_OK) return st;
    }
    Job jobs[kMaxTasks];
    for (int i = 0; i < ntasks; ++i) {
        jobs[i] = {tasks[i].W, tasks[i].x, tasks[i].dst, tasks[i].nrows, tasks[i].K,
                   tasks[i].stride_row_x, tasks[i].stride_col_x, tasks[i].stride_col_dst, kPrepF32};
        if (gather && gather->world > 1 && tasks[i].nrows > 0 && tasks[i].K == 0)
            return fail(Q4K_EINVAL, "task %d: K = 0 is not supported with a fused all-gather", i);
    }
    return run(jobs, ntasks, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr,
               nullptr, gather, /*fused=*/true);
}

int q4k_ipc_alloc(size_t bytes, void **ptr) {
    if (!ptr || bytes == 0) return fail(Q4K_EINVAL, "q4k_ipc_alloc: null pointer or zero size");
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "q4k_ipc_alloc");
    return Q4K_OK;
}

int q4k_ipc_free(void *ptr) {
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? Q4K_OK : cuda_fail(e, "q4k_ipc_free");
}

int q4k_ipc_handle(const void *ptr, void *handle64) {
    if (!ptr || !handle64) return fail(Q4K_EINVAL, "q4k_ipc_handle: null pointer");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(ptr));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    memcpy(handle64, &h, sizeof(h));
    return Q4K_OK;
}

int q4k_ipc_open(const void *handle64, void **ptr) {
    if (!ptr || !handle64) return fail(Q4K_EINVAL, "q4k_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    return Q4K_OK;
}

int q4k_ipc_close(void *ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? Q4K_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int q4k_debug_subblock_sums(const void *W, const void *y_q8_1, int64_t K, int64_t nrows, int ncols,
                            int64_t stride_row_x, int64_t stride_col_y, int32_t *S_out, int32_t *T_out,
                            void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    if (!S_out || !T_out) return fail(Q4K_EINVAL, "null S_out/T_out");
    float *dummy_dst = reinterpret_cast<float *>(S_out);  // never written in dump mode
    Job j{W, y_q8_1, dummy_dst, nrows, K, stride_row_x, stride_col_y, nrows, kPrepQ81};
    if (K == 0 || nrows == 0) return validate_job(j, ncols, 0);
    return run(&j, 1, ncols, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), S_out, T_out);
}

int q4k_workspace_status(const void *workspace, int *device_status, q4k_stream_t stream) {
    if (!workspace || !device_status) return fail(Q4K_EINVAL, "null pointer");
    int32_t v = 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "status read");
    *device_status = v;
    return Q4K_OK;
}

size_t q4k_timeline_bytes(void) {
#if Q4K_TIMELINE
    return kTlBytes;
#else
    return 0;
#endif
}

int q4k_timeline_read(void *host, size_t bytes, int *ncalls) {
#if Q4K_TIMELINE
    if (host == nullptr || bytes > kTlBytes)
        return fail(Q4K_EINVAL, "timeline read of %zu bytes (at most %zu)", bytes, kTlBytes);
    int dev = 0;
    int st = tl_device(&dev);
    if (st != Q4K_OK) return st;
    std::lock_guard<std::mutex> lk(g_tl_mu);
    if (ncalls) *ncalls = g_tl_calls[dev];
    if (g_tl[dev] == nullptr) {
        std::memset(host, 0, bytes);
        return Q4K_OK;
    }
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(host, g_tl[dev], bytes, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? Q4K_OK : cuda_fail(e, "timeline read");
#else
    (void)host;
    (void)bytes;
    (void)ncalls;
    return fail(Q4K_EINVAL, "library built without Q4K_TIMELINE");
#endif
}

int q4k_timeline_reset(void) {
#if Q4K_TIMELINE
    int dev = 0;
    int st = tl_device(&dev);
    if (st != Q4K_OK) return st;
    std::lock_guard<std::mutex> lk(g_tl_mu);
    g_tl_calls[dev] = 0;
    if (g_tl[dev] == nullptr) return Q4K_OK;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemset(g_tl[dev], 0, kTlBytes);
    return e == cudaSuccess ? Q4K_OK : cuda_fail(e, "timeline reset");
#else
    return fail(Q4K_EINVAL, "library built without Q4K_TIMELINE");
#endif
}

}  // extern "C"
