// q4k_noalloc.cu -- q4k_mul_mat_vec_noalloc: the fp32-activation GEMV for
// callers that cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc at all: inference
// runtimes that plan every device buffer ahead of time and forbid allocation
// on the decode path (cudaMalloc can implicitly synchronise the device and
// stall the pipeline), and host applications that own the GPU memory budget
// and hand plugins only the tensors they work on.  Such a caller has W, x and
// dst but no scratch buffer to pass as the workspace of q4k_mul_mat_vec.
//
// This entry point brings its own scratch: a file-scope device array of
// kScratchBytes (4 MiB), which every GPU that loads the library holds until
// the process exits.  It is one array per device, shared by every call of
// this entry point on that device; each call starts by clearing the parts
// that must start at zero (status word and split counters, done by the prep
// kernel), so leftovers of the previous call do no harm, but two calls that
// can overlap on the GPU (e.g. issued on two streams) race on it.
#include "q4k_gemv.h"
#include "q4k_internal.h"

#include <cuda_runtime.h>

#include <cstdio>

namespace {

constexpr size_t kScratchBytes = size_t(4) << 20;  // 4 MiB per device

// In host code this name is only a host-side stand-in for the device array;
// kernels get its device address from cudaGetSymbolAddress (below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Device address of the scratch array on the current device.  Looked up on
// every call (the lookup allocates nothing and is cheap), so the address
// stays right if the device's context is reset and the module reloaded
// somewhere else.  The first lookup on a device can load the module; make
// that first call before any stream capture.
cudaError_t scratch_address(void **out) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    *out = p;
    return cudaSuccess;
}

}  // namespace

namespace q4k {
void set_last_error_message(const char *msg);  // q4k_capi.cu
}

extern "C" {

size_t q4k_noalloc_scratch_bytes(void) { return kScratchBytes; }

int q4k_mul_mat_vec_noalloc(const void *W, const float *x, float *dst, int64_t K, int64_t nrows, int ncols,
                            int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst,
                            q4k_stream_t stream) {
    // Size check first, on the host: everything the call needs must fit the
    // fixed array (the workspace layout of q4k_mul_mat_vec).
    const size_t need = q4k_gemv_workspace_bytes(nrows, K, ncols);
    if (need == 0) {
        // invalid shape: let the regular entry point report the precise reason
        return q4k_mul_mat_vec(W, x, dst, K, nrows, ncols, stride_row_x, stride_col_x, stride_col_dst, nullptr, 0,
                               stream);
    }
    if (need > kScratchBytes) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "q4k_mul_mat_vec_noalloc: this call needs %zu bytes of scratch, more than the %zu-byte "
                 "built-in array (nrows=%lld K=%lld ncols=%d); use q4k_mul_mat_vec with a caller workspace",
                 need, kScratchBytes, (long long)nrows, (long long)K, ncols);
        q4k::set_last_error_message(msg);
        return Q4K_EINVAL;
    }
    void *scratch = nullptr;
    const cudaError_t e = scratch_address(&scratch);
    if (e != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof(msg), "q4k_mul_mat_vec_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
        q4k::set_last_error_message(msg);
        return Q4K_ECUDA;
    }
    return q4k_mul_mat_vec(W, x, dst, K, nrows, ncols, stride_row_x, stride_col_x, stride_col_dst, scratch,
                           kScratchBytes, stream);
}

}  // extern "C"
