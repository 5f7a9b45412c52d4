// q4k_sharded.cu -- q4k_gemv_sharded: a row-sharded GEMV whose output rows
// are gathered with NCCL, for runtimes that already hold one NCCL
// communicator per device.
//
// The reference's multi-GPU mode is ggml's row split: every device computes
// the rows [row_low, row_high) of its weight slice (ggml_cuda_op_mul_mat_vec_q,
// kernels/mmvq.cu:764-793) and upstream ggml copies the slices together.  Here
// each rank owns the contiguous ceil-split row range [rank * S, rank * S + S)
// (S = ceil(nrows / world), the last ranks possibly short or empty), runs the
// single-GEMV launch sequence on its slice into a staging area of the
// workspace, all-gathers the staging areas in place with ncclAllGather on the
// caller's stream, and a small kernel places the rows into y at the caller's
// column stride.  All three steps are stream-ordered; nothing synchronises
// the host.
//
// NCCL is not linked: the library uses the NCCL already loaded in the process
// (the one that created the communicator; a communicator only works with the
// library instance that made it) and loads libnccl.so.2 from the loader path
// only if none is loaded.  The NCCL header supplies the types.
#include "q4k_gemv.h"
#include "q4k_internal.h"

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

namespace q4k {
void set_last_error_message(const char *msg);  // q4k_capi.cu
}

namespace {

int fail(int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    q4k::set_last_error_message(buf);
    return status;
}

// ---- the NCCL entry points ---------------------------------------------------
struct NcclApi {
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int *) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int *) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    char why[200] = {0};
};

// Resolved on first use; a failed lookup is retried on the next call (the
// process may load NCCL later), a successful one is kept.
const NcclApi &nccl_api() {
    static NcclApi api;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (api.ok) return api;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own NCCL
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (h == nullptr) {
        const char *why = dlerror();
        snprintf(api.why, sizeof(api.why), "libnccl.so.2 not loadable: %s", why ? why : "unknown");
        return api;
    }
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_count = reinterpret_cast<decltype(api.comm_count)>(dlsym(h, "ncclCommCount"));
    api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(dlsym(h, "ncclCommUserRank"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.all_gather && api.comm_count && api.comm_user_rank && api.error_string;
    if (!api.ok) snprintf(api.why, sizeof(api.why), "libnccl.so.2 lacks ncclAllGather / ncclCommCount");
    return api;
}

constexpr size_t kAlign = 256;
size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
int64_t shard_rows(int64_t nrows, int world) { return (nrows + world - 1) / world; }

// Staging area after the GEMV workspace: world blocks of ncols x S floats
// (block r = rank r's rows, column stride S).
struct ShardLayout {
    int64_t S = 0;
    size_t gemv_bytes = 0, stage_off = 0, total = 0;
};

ShardLayout shard_layout(int64_t nrows, int64_t K, int ncols, int world) {
    ShardLayout L;
    L.S = shard_rows(nrows, world);
    L.gemv_bytes = q4k_gemv_workspace_bytes(L.S, K, ncols);
    if (L.gemv_bytes == 0) return L;
    L.stage_off = round_up(L.gemv_bytes, kAlign);
    L.total = L.stage_off + static_cast<size_t>(world) * ncols * L.S * sizeof(float);
    return L;
}

// y[j * ldy + row] = stage[(row / S * ncols + j) * S + row % S], rows < nrows.
__global__ void k_shard_place(const float *__restrict__ stage, float *__restrict__ y, int64_t nrows, int64_t S,
                              int ncols, int64_t ldy) {
    const int64_t n = nrows * ncols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t j = i / nrows, row = i - j * nrows;
        const int64_t r = row / S;
        y[j * ldy + row] = stage[(r * ncols + j) * S + (row - r * S)];
    }
}

}  // namespace

extern "C" {

size_t q4k_sharded_workspace_bytes(int64_t nrows, int64_t K, int ncols, int world) {
    if (nrows < 1 || world < 1 || world > Q4K_MAX_SHARD_RANKS) return 0;
    return shard_layout(nrows, K, ncols, world).total;
}

int q4k_gemv_sharded(const void *W_shard, const float *x, float *y, int64_t K, int64_t nrows, int ncols,
                     int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_y, void *nccl_comm, int rank,
                     int world, void *workspace, size_t workspace_bytes, q4k_stream_t stream) {
    if (world < 1 || world > Q4K_MAX_SHARD_RANKS)
        return fail(Q4K_EINVAL, "world=%d outside 1..%d", world, Q4K_MAX_SHARD_RANKS);
    if (rank < 0 || rank >= world) return fail(Q4K_EINVAL, "rank=%d outside 0..%d", rank, world - 1);
    if (nccl_comm == nullptr) return fail(Q4K_EINVAL, "null NCCL communicator");
    if (ncols < 1 || ncols > Q4K_MAX_NCOLS) return fail(Q4K_EINVAL, "ncols=%d outside 1..8", ncols);
    if (nrows < 1) return fail(Q4K_EINVAL, "nrows=%lld < 1", (long long)nrows);
    if (y == nullptr || x == nullptr) return fail(Q4K_EINVAL, "null pointer");
    if (ncols > 1 && stride_col_y < nrows)
        return fail(Q4K_EINVAL, "stride_col_y=%lld < nrows=%lld", (long long)stride_col_y, (long long)nrows);
    const ShardLayout L = shard_layout(nrows, K, ncols, world);
    if (L.total == 0)
        return fail(Q4K_EINVAL, "invalid shape (K=%lld must be a positive multiple of 256)", (long long)K);
    if (workspace == nullptr || workspace_bytes < L.total || reinterpret_cast<uintptr_t>(workspace) % kAlign)
        return fail(Q4K_EWORKSPACE, "workspace %p of %zu bytes; need %zu bytes, 256-byte aligned", workspace,
                    workspace_bytes, L.total);
    const NcclApi &api = nccl_api();
    if (!api.ok) return fail(Q4K_ENCCL, "%s", api.why);
    ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    int n = 0, r = -1;
    ncclResult_t nr = api.comm_count(comm, &n);
    if (nr == ncclSuccess) nr = api.comm_user_rank(comm, &r);
    if (nr != ncclSuccess) return fail(Q4K_ENCCL, "NCCL communicator query: %s", api.error_string(nr));
    if (n != world || r != rank)
        return fail(Q4K_EINVAL, "communicator has %d ranks, this is rank %d; the call says world=%d rank=%d", n, r,
                    world, rank);

    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    float *stage = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + L.stage_off);
    const int64_t lo = static_cast<int64_t>(rank) * L.S;
    const int64_t mine = nrows - lo < L.S ? (nrows - lo > 0 ? nrows - lo : 0) : L.S;
    float *my_stage = stage + static_cast<int64_t>(rank) * ncols * L.S;
    if (mine > 0) {
        if (W_shard == nullptr) return fail(Q4K_EINVAL, "null W_shard for %lld local rows", (long long)mine);
        const int st = q4k_mul_mat_vec(W_shard, x, my_stage, K, mine, ncols, stride_row_x, stride_col_x, L.S,
                                       workspace, L.gemv_bytes, stream);
        if (st != Q4K_OK) return st;  // (its message stays the last error)
    }
    nr = api.all_gather(my_stage, stage, static_cast<size_t>(ncols) * L.S, ncclFloat32, comm, s);
    if (nr != ncclSuccess) return fail(Q4K_ENCCL, "ncclAllGather: %s", api.error_string(nr));
    const int64_t total = nrows * ncols;
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    const int blocks = static_cast<int>(want < 1184 ? want : 1184);
    k_shard_place<<<blocks, threads, 0, s>>>(stage, y, nrows, L.S, ncols, ncols > 1 ? stride_col_y : nrows);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(Q4K_ECUDA, "row placement launch: %s", cudaGetErrorString(e));
    return Q4K_OK;
}

}  // extern "C"
