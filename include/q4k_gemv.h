/*
 * q4k_gemv.h -- C ABI of the B200 (sm_100a) Q4_K x q8_1 decode GEMV library
 * (libq4k_gemv.so).
 *
 * Drop-in boundary for the Q4_K branch of llama.cpp's ggml-cuda mul_mat_vec_q
 * dispatch as the reference wires it.  Reference interfaces replaced
 * (paths relative to the reference project, vijay-kodamalla/gemv-q4_k-optimization):
 *
 *   kernels/mmvq.cu:479-486, :536-593  mul_mat_vec_q_switch_type, Q4_K case
 *                                      -> q4k_mul_mat_vec_q8_1()
 *   kernels/mmvq.cu:10-18, :563-584    custom_q4k_gemv<...> launch (6 args)
 *                                      -> q4k_custom_q4k_gemv()
 *   kernels/mmvq.cu:666-762            ggml_cuda_mul_mat_vec_q (fp32 src1:
 *                                      quantize, then GEMV)  -> q4k_mul_mat_vec()
 *   kernels/mmvq.cu:734                quantize_row_q8_1_cuda call
 *                                      -> q4k_quantize_q8_1()
 *   kernels/mmvq.cu:764-793            ggml_cuda_op_mul_mat_vec_q (row-split
 *                                      slice per device) -> q4k_op_mul_mat_vec_q()
 *                                      (with the slices gathered over an NCCL
 *                                      communicator) -> q4k_gemv_sharded()
 *
 * Data formats (unchanged from ggml, so tensors pass through untouched):
 *   Q4_K super-block, 144 bytes per 256 weights: half d, half dmin,
 *     uint8 scales[12] (8 six-bit scales + 8 six-bit mins), uint8 qs[128].
 *   q8_1 block, 36 bytes per 32 activations: half d, half sum, int8 qs[32].
 * Weight row r of a matrix starts at W + r*stride_row_x*144 bytes; W must be
 * 16-byte aligned (rows are streamed with bulk asynchronous copies).
 * Column j of an fp32 activation starts at x + j*stride_col_x, of a q8_1
 * activation at block j*stride_col_y, and of the output at
 * dst + j*stride_col_dst (the column-major ggml dst layout, mmvq.cu:337).
 *
 * Conventions (differences from the reference, on purpose):
 *   - every entry point returns a q4k_status instead of aborting the process
 *     (the reference asserts: mmvq.cu:375, :393-394, :472-474, :669-686);
 *   - all work is asynchronous on the caller's stream; the library never
 *     synchronises and never allocates on the call path;
 *   - the caller owns all memory, including the scratch "workspace" (it may
 *     come from a pool and need not be initialised); one workspace must not
 *     be used by two calls that can overlap on the GPU (e.g. two streams).
 */
#ifndef Q4K_GEMV_H
#define Q4K_GEMV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define Q4K_API __attribute__((visibility("default")))
#else
#define Q4K_API
#endif

/* cudaStream_t without including the CUDA headers. */
typedef struct CUstream_st *q4k_stream_t;

#define Q4K_QK_K 256          /* weights per super-block */
#define Q4K_BLOCK_BYTES 144   /* sizeof(block_q4_K)  (kernels/w_tile.cu:6) */
#define Q4K_QK8_1 32          /* activations per q8_1 block */
#define Q8_1_BLOCK_BYTES 36   /* sizeof(block_q8_1)  (kernels/w_tile.cu:7) */
#define Q4K_ROW_PADDING 512   /* q8_1 row padding, MATRIX_ROW_PADDING (mmvq.cu:728) */
#define Q4K_MAX_NCOLS 8       /* MMVQ_MAX_BATCH_SIZE (mmvq.cu:394) */
#define Q4K_MAX_TASKS 16      /* matrices per q4k_gemv_batch launch */

typedef enum q4k_status {
    Q4K_OK = 0,
    Q4K_EINVAL = 1,     /* bad shape, stride, alignment, ncols outside 1..8, K % 256 != 0 */
    Q4K_ECUDA = 2,      /* a CUDA runtime call or launch failed (message via q4k_last_error) */
    Q4K_ETIMEOUT = 3,   /* a bounded device-side wait expired (status word) */
    Q4K_ENCCL = 4,      /* a collective failed */
    Q4K_EWORKSPACE = 5  /* workspace missing, too small or misaligned */
} q4k_status;

/* Human-readable name of a status; detail of the last failure on this thread. */
Q4K_API const char *q4k_status_string(int status);
Q4K_API const char *q4k_last_error(void);

/* Library version, and whether the CUDA device of the calling thread is
 * supported (compute capability 10.0: the library is built for sm_100a only). */
Q4K_API int q4k_version(void);
Q4K_API int q4k_device_supported(void);

/* ---- sizes ---------------------------------------------------------------- */

/* Bytes of one Q4_K row of length K (K % 256 == 0). */
Q4K_API size_t q4k_row_bytes(int64_t K);
/* Bytes of ncols q8_1 activation columns of padded length Kpad (Kpad % 32 == 0). */
Q4K_API size_t q4k_q8_1_bytes(int64_t Kpad, int ncols);
/* Workspace bytes for one GEMV of nrows x K with ncols activation columns. */
Q4K_API size_t q4k_gemv_workspace_bytes(int64_t nrows, int64_t K, int ncols);

/* ---- q8_1 quantization ------------------------------------------------------ */

/* fp32 -> ggml q8_1 blocks (the src1 quantization of mmvq.cu:728-735).
 * Output column j starts at block j*(Kpad/32); positions K <= i < Kpad are
 * zero padding.  Per block: d = amax/127, q = roundf(x/d), ds = (half d,
 * half of the sum of x in xor-butterfly order). */
Q4K_API int q4k_quantize_q8_1(const float *x, int64_t K, int64_t stride_col_x, int64_t Kpad,
                      int ncols, void *y_q8_1, q4k_stream_t stream);

/* ---- single GEMV ------------------------------------------------------------ */

/* dst[j*stride_col_dst + r] = sum_k W[r,k] * q8_1 column j, r < nrows, j < ncols.
 * Same arguments as the Q4_K case of mul_mat_vec_q_switch_type
 * (mmvq.cu:479-486: vx, vy, dst, ncols_x = K, nrows_x, ncols_dst,
 * stride_row_x, stride_col_y, stride_col_dst) plus the workspace. */
Q4K_API int q4k_mul_mat_vec_q8_1(const void *W, const void *y_q8_1, float *dst,
                         int64_t K, int64_t nrows, int ncols,
                         int64_t stride_row_x, int64_t stride_col_y, int64_t stride_col_dst,
                         void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* fp32 activations: the q8_1 quantization is fused into the GEMV launch
 * sequence (ggml_cuda_mul_mat_vec_q, mmvq.cu:666-762, without ids/fusion). */
Q4K_API int q4k_mul_mat_vec(const void *W, const float *x, float *dst,
                    int64_t K, int64_t nrows, int ncols,
                    int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst,
                    void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* Row-split slice on one device (ggml_cuda_op_mul_mat_vec_q, mmvq.cu:764-793):
 * W_slice holds rows [row_low, row_high) of a K-column Q4_K matrix, y_q8_1 is
 * the already quantized src1 (src1_ncols columns, src1_padded_row_size
 * values per column), dst_slice receives the slice with column stride
 * nrows_dst. */
Q4K_API int q4k_op_mul_mat_vec_q(const void *W_slice, int64_t K, const void *y_q8_1,
                         float *dst_slice, int64_t row_low, int64_t row_high,
                         int64_t src1_ncols, int64_t src1_padded_row_size, int64_t nrows_dst,
                         void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* The custom kernel hook's launch contract (mmvq.cu:10-18, :548-584):
 * num_blocks_total = super-blocks per row (the reference passes stride_row_x,
 * mmvq.cu:548), stride_col_dst doubles as the row count (2rowCTA.cu:62),
 * ncols_dst in 1..8 (the reference's hook stops at 4, mmvq.cu:541). */
Q4K_API int q4k_custom_q4k_gemv(const void *vx, const void *vy, float *dst, int num_blocks_total,
                        int stride_col_y_blocks, int stride_col_dst, int ncols_dst,
                        void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* ---- persistent multi-matrix launch ----------------------------------------- */

/* One matrix of a batched launch.  Tasks that name the same x (same pointer,
 * K and stride) share one quantization. */
typedef struct q4k_task {
    const void *W;          /* nrows x K Q4_K, 16-byte aligned */
    const float *x;         /* K x ncols fp32, column stride stride_col_x */
    float *dst;             /* nrows x ncols fp32, column stride stride_col_dst */
    int64_t nrows;
    int64_t K;
    int64_t stride_row_x;   /* super-blocks between rows (>= K/256) */
    int64_t stride_col_x;   /* floats between activation columns (>= K) */
    int64_t stride_col_dst; /* floats between output columns (>= nrows) */
} q4k_task;

/* Workspace bytes for q4k_gemv_batch over these tasks. */
Q4K_API size_t q4k_batch_workspace_bytes(const q4k_task *tasks, int ntasks, int ncols);

/* Every task's GEMV in one launch sequence: one quantization launch for all
 * distinct activations, then one persistent GEMV launch whose warps stream the
 * weight bytes of all tasks, balanced across the SMs. */
Q4K_API int q4k_gemv_batch(const q4k_task *tasks, int ntasks, int ncols,
                   void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* ---- fused epilogue: bias and gated linear unit (kernels/mmvq.cu:182-227, :309-338) */

/* The reference's fused MMVQ (ggml_cuda_mul_mat_vec_q with fusion args,
 * mmvq.cu:666-762; device part mmvq.cu:182-227 and :309-338) computes, per
 * output, r = W.x (+ x_bias) and, with a gate matrix, g = Wg.x (+ gate_bias),
 * and stores op(r, g).  Here both matrices stream in the same launch: an
 * atom holds one super-block of each for 32 rows, and the epilogue runs on
 * the final sums.  Ops (the reference's switch at mmvq.cu:318-333):
 *   SWIGLU      r * g / (1 + exp(-g))
 *   GEGLU       r * 0.5 g (1 + tanh(sqrt(2/pi) g (1 + 0.044715 g^2)))
 *   SWIGLU_OAI  a / (1 + exp(-1.702 a)) * (1 + b), a = min(g, 7), b = clamp(r, -7, 7)
 *   MUL         r * g (the reference's default branch)
 * Bias element (row, column j) is x_bias[j*stride_col_bias + row]. */
#define Q4K_GLU_NONE 0       /* no gate (a bias alone is allowed) */
#define Q4K_GLU_SWIGLU 1
#define Q4K_GLU_GEGLU 2
#define Q4K_GLU_SWIGLU_OAI 3
#define Q4K_GLU_MUL 4

typedef struct q4k_task_ex {
    q4k_task t;               /* t.W: the main matrix (the reference's vx, the "up" projection) */
    const void *W_gate;       /* gate matrix (fusion.gate): same shape and row stride as t.W, or NULL */
    const float *x_bias;      /* added to the main result (fusion.x_bias), or NULL */
    const float *gate_bias;   /* added to the gate result (fusion.gate_bias), or NULL; needs W_gate */
    int64_t stride_col_bias;  /* floats between bias columns (0: one column for all) */
    int glu_op;               /* Q4K_GLU_*: SWIGLU..MUL with W_gate, NONE without */
    int rms_norm;             /* 1: quantize RMSNorm(x) * norm_weight instead of x (see below) */
    float norm_eps;           /* RMSNorm epsilon */
    const float *norm_weight; /* K per-element weights, or NULL (no multiply) */
} q4k_task_ex;

/* ---- RMSNorm fused into the quantization launch ---------------------------------
 * The reference's decode trace runs rms_norm_f32 -> quantize_q8_1 ->
 * mul_mat_vec_q (upstream ggml; no source in the reference).  With
 * rms_norm = 1 the quantization launch normalizes each column first:
 * y = x / sqrt(mean(x^2) + eps) * w, one CTA per column, the sum of squares
 * in a fixed order (per-thread fma over a stride of 256, xor butterflies) and
 * scale = 1 / sqrtf(mean + eps) (upstream: rsqrtf, within 2 ulp).  Tasks that
 * name the same x with the same norm share one normalized quantization. */
Q4K_API int q4k_rms_norm_quantize_q8_1(const float *x, int64_t K, int64_t stride_col_x, int64_t Kpad, int ncols,
                                       const float *norm_weight, float eps, void *y_q8_1, q4k_stream_t stream);

/* Workspace bytes / batched launch for tasks with optional fused epilogues
 * (q4k_gemv_batch otherwise).  K = 0 is rejected for a fused task; at most
 * Q4K_MAX_GATED tasks of one launch may have a gate. */
#define Q4K_MAX_GATED 4
Q4K_API size_t q4k_batch_ex_workspace_bytes(const q4k_task_ex *tasks, int ntasks, int ncols);
Q4K_API int q4k_gemv_batch_ex(const q4k_task_ex *tasks, int ntasks, int ncols, void *workspace,
                              size_t workspace_bytes, q4k_stream_t stream);

/* One fused GEMV: the reference's fused Q4_K call with q8_1 input
 * (mul_mat_vec_q_switch_type with fusion, mmvq.cu:479-593) and its fp32-input
 * form (ggml_cuda_mul_mat_vec_q with fusion, mmvq.cu:666-762).  The bias
 * column stride is stride_col_dst, as in the reference (mmvq.cu:211).
 * Workspace: q4k_gemv_fused_workspace_bytes. */
Q4K_API size_t q4k_gemv_fused_workspace_bytes(int64_t nrows, int64_t K, int ncols);
Q4K_API int q4k_mul_mat_vec_q8_1_fused(const void *W, const void *W_gate, const void *y_q8_1, float *dst,
                                       int64_t K, int64_t nrows, int ncols, int64_t stride_row_x,
                                       int64_t stride_col_y, int64_t stride_col_dst, const float *x_bias,
                                       const float *gate_bias, int glu_op, void *workspace,
                                       size_t workspace_bytes, q4k_stream_t stream);
Q4K_API int q4k_mul_mat_vec_fused(const void *W, const void *W_gate, const float *x, float *dst, int64_t K,
                                  int64_t nrows, int ncols, int64_t stride_row_x, int64_t stride_col_x,
                                  int64_t stride_col_dst, const float *x_bias, const float *gate_bias, int glu_op,
                                  void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* ---- Q6_K weights -----------------------------------------------------------------
 * The reference's MMVQ also serves Q6_K (mul_mat_vec_q<GGML_TYPE_Q6_K>; dot
 * product kernels/vecdotq.cuh:576-601, :867-890): the output head and some
 * layers of Q4_K_M checkpoints.  block_q6_K is 210 bytes per 256 weights
 * (ql[128] low 4 bits, qh[64] high 2 bits, int8 scales[16] per 16 weights,
 * fp16 d); weight = d * scale * (q6 - 32).  Same activations (fp32 or q8_1),
 * same output layout and strides (stride_row_x in super-blocks) as the Q4_K
 * entries.  Needs K % 2048 == 0 and stride_row_x % 8 == 0 (each row starts on
 * a 16-byte boundary); Q4_K and Q6_K tasks do not share a launch. */
Q4K_API size_t q4k_q6_k_workspace_bytes(int64_t nrows, int64_t K, int ncols);
Q4K_API int q4k_mul_mat_vec_q6_k(const void *W, const float *x, float *dst, int64_t K, int64_t nrows, int ncols,
                                 int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst,
                                 void *workspace, size_t workspace_bytes, q4k_stream_t stream);
Q4K_API int q4k_mul_mat_vec_q6_k_q8_1(const void *W, const void *y_q8_1, float *dst, int64_t K, int64_t nrows,
                                      int ncols, int64_t stride_row_x, int64_t stride_col_y, int64_t stride_col_dst,
                                      void *workspace, size_t workspace_bytes, q4k_stream_t stream);
Q4K_API size_t q4k_batch_q6_k_workspace_bytes(const q4k_task *tasks, int ntasks, int ncols);
Q4K_API int q4k_gemv_batch_q6_k(const q4k_task *tasks, int ntasks, int ncols, void *workspace,
                                size_t workspace_bytes, q4k_stream_t stream);

/* ---- row-sharded multi-GPU: GEMV fused with the output all-gather ------------- */

/* Row-split across GPUs is the reference's multi-GPU mode (mmvq.cu:764-793,
 * the main device then collects the slices).  Here every rank computes its
 * rows and, in the same kernel, stores them straight into every rank's full
 * output buffer over NVLink (peer memory); its last CTA then raises this
 * rank's epoch flag in every peer and the launch ends without waiting for
 * the peers.  The peers' rows of a call are in this rank's buffer once every
 * peer's flag has reached this rank's epoch, which two things wait for
 * (bounded, 2 s, then Q4K_ETIMEOUT in the workspace status word):
 *   - the next gathering call on the stream, before it reads its activations
 *     (so a chain whose activations come from gathered outputs is safe), and
 *   - q4k_gather_wait, which the caller issues before anything else on the
 *     stream reads the gathered buffer (e.g. before copying it to the host).
 * Every rank must make the same sequence of calls. */
#define Q4K_MAX_PEERS 8

typedef struct q4k_gather {
    int world;                        /* ranks, 1..Q4K_MAX_PEERS */
    int rank;                         /* this rank */
    float *out_local;                 /* this rank's full output buffer */
    float *out_peer[Q4K_MAX_PEERS];   /* each rank's full output buffer, mapped in this process
                                         (out_peer[rank] == out_local) */
    uint32_t *flags_peer[Q4K_MAX_PEERS]; /* each rank's flag words (world of them), mapped here */
    uint32_t *epoch;                  /* this rank's epoch word, zero before the first call */
    int64_t out_elems;                /* floats in every rank's full output buffer; every
                                         task's dst columns must lie inside it */
} q4k_gather;

/* q4k_gemv_batch over this rank's row shards, gathered into every rank's
 * buffer.  Each task's dst must point into out_local at this rank's first
 * row of that matrix (all ranks use the same layout of the full buffer);
 * a task whose columns reach outside [out_local, out_local + out_elems) is
 * rejected with Q4K_EINVAL before anything is launched.
 * A rank stores into its peers' buffers as soon as its launch runs: a region
 * of the full buffer may be rewritten only once every rank is done reading
 * it (use different regions for consecutive calls, e.g. one per layer, or
 * synchronise the ranks before reuse). */
Q4K_API int q4k_gemv_batch_allgather(const q4k_task *tasks, int ntasks, int ncols, const q4k_gather *gather,
                                     void *workspace, size_t workspace_bytes, q4k_stream_t stream);
/* Stream-ordered wait until every peer's rows of the last gathering call on
 * this rank are in out_local (one small launch).  A wait that gives up after
 * 2 s writes Q4K_ETIMEOUT into the workspace status word (workspace: the one
 * the gathering calls use, at least 4 bytes). */
Q4K_API int q4k_gather_wait(const q4k_gather *gather, void *workspace, size_t workspace_bytes,
                            q4k_stream_t stream);

/* ---- single-launch path (no reference counterpart) --------------------------- */

/* The calls above issue two launches (activation quantization, then the
 * GEMV) and accept a workspace with arbitrary contents, as ggml's pool hands
 * it out.  A caller that keeps one workspace per stream can save the first
 * launch: q4k_gemv_batch_persistent runs the batch as ONE launch in which
 * every CTA quantizes the activations its rows need straight into its shared
 * memory (the same q8_1 semantics, bit for bit) and reads them from there;
 * the weights start streaming before the previous launch on the stream has
 * finished.  It applies to plain Q4_K tasks with fp32 activations whose
 * columns start 32-byte aligned, ncols <= 2, and launches where no CTA needs
 * more than 81 KB of activation records (e.g. a whole Mistral-7B or
 * Llama-3-70B decoder layer at ncols 1); other calls run the two-launch
 * sequence.  Results are identical to q4k_gemv_batch's static kernel.  It
 * needs the same workspace size (q4k_batch_workspace_bytes) and its control
 * words in a known state on entry: zero the workspace once with
 * q4k_workspace_init before the first call; every call that completes leaves
 * them valid again (the two-launch calls may use the same workspace in
 * between).  After a call reports Q4K_ETIMEOUT (q4k_workspace_status) call
 * q4k_workspace_init again.  gather may be NULL (no all-gather) or a
 * descriptor as for q4k_gemv_batch_allgather; the launch then waits for the
 * previous gathering call's rows before it reads its activations. */
Q4K_API int q4k_workspace_init(void *workspace, size_t workspace_bytes, q4k_stream_t stream);
Q4K_API int q4k_gemv_batch_persistent(const q4k_task *tasks, int ntasks, int ncols, const q4k_gather *gather,
                                      void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* Set-up helpers for the buffers above (not on the call path): device memory
 * that other processes can map (zero-filled), its 64-byte IPC handle, and
 * mapping / unmapping a peer's buffer from its handle. */
Q4K_API int q4k_ipc_alloc(size_t bytes, void **ptr);
Q4K_API int q4k_ipc_free(void *ptr);
Q4K_API int q4k_ipc_handle(const void *ptr, void *handle64);
Q4K_API int q4k_ipc_open(const void *handle64, void **ptr);
Q4K_API int q4k_ipc_close(void *ptr);

/* ---- row-sharded GEMV over an NCCL communicator ------------------------------ */

/* Replaces the row-split call ggml_cuda_op_mul_mat_vec_q (mmvq.cu:764-793)
 * plus upstream ggml's copy of the slices into one tensor, for a runtime
 * that holds one NCCL communicator per device (nccl_comm: its ncclComm_t).
 * Rank r owns rows [r*S, min(r*S + S, nrows)) of the nrows x K matrix,
 * S = ceil(nrows / world) (the last ranks may own fewer rows, or none);
 * W_shard holds those rows (stride_row_x super-blocks apart; unused when the
 * rank owns none).  Every rank passes the same fp32 activations x (ncols
 * columns, stride_col_x apart) and receives all nrows rows of every column
 * in y (stride_col_y apart).  Stream-ordered: the rank's GEMV, one
 * ncclAllGather on the caller's stream, and one small kernel that places the
 * rows; every rank of the communicator must make the same calls in the same
 * order.  The communicator's size and rank must equal world and rank
 * (Q4K_EINVAL otherwise); an NCCL failure returns Q4K_ENCCL.  The library
 * uses the NCCL already loaded in the process (the one that created the
 * communicator), else loads libnccl.so.2. */
#define Q4K_MAX_SHARD_RANKS 1024
Q4K_API size_t q4k_sharded_workspace_bytes(int64_t nrows, int64_t K, int ncols, int world);
Q4K_API int q4k_gemv_sharded(const void *W_shard, const float *x, float *y, int64_t K, int64_t nrows, int ncols,
                             int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_y, void *nccl_comm,
                             int rank, int world, void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* ---- callers that cannot allocate --------------------------------------------- */

/* q4k_mul_mat_vec without a caller workspace.  No counterpart in the reference.
 * For callers that may not allocate device memory at all (runtimes that plan
 * every buffer ahead and forbid cudaMalloc on the decode path, host
 * applications that own the GPU memory budget): the scratch comes from a
 * 4 MiB array built into the library, held on every GPU that loads it until
 * the process exits.  Calls that need more (q4k_gemv_workspace_bytes(nrows, K,
 * ncols) > q4k_noalloc_scratch_bytes()) return Q4K_EINVAL with a message.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture.  All calls on a device share the
 * array: calls that can overlap on the GPU (e.g. on two streams) race. */
Q4K_API int q4k_mul_mat_vec_noalloc(const void *W, const float *x, float *dst,
                                    int64_t K, int64_t nrows, int ncols,
                                    int64_t stride_row_x, int64_t stride_col_x, int64_t stride_col_dst,
                                    q4k_stream_t stream);
/* Size of that built-in scratch array in bytes. */
Q4K_API size_t q4k_noalloc_scratch_bytes(void);

/* ---- diagnostics ------------------------------------------------------------- */

/* Which GEMV kernel q4k_gemv_batch_ex (or q4k_gemv_batch) would run for these
 * tasks on a device with num_sms SMs (the library's measured choice; builds
 * made with -DQ4K_SCHED_FORCE for measurements force one kernel).
 * Touches no device.  Returns a Q4K_KERNEL_* value, or -1 (reason in
 * q4k_last_error()) for tasks the call would reject.  No counterpart in the
 * reference, which has one kernel per ncols. */
#define Q4K_KERNEL_STATIC 0          /* statically partitioned atom stream */
#define Q4K_KERNEL_STATIC_GATED 2    /* launches with a bias / GLU epilogue: per-CTA atom queue */
#define Q4K_KERNEL_STATIC_TWO_ROW 3  /* the static kernel, two rows per lane (ncols >= 3) */
#define Q4K_KERNEL_DYNAMIC 5         /* whole row groups per CTA from a ticket queue */
#define Q4K_KERNEL_DYNAMIC_GATED 6   /* the same with the bias / GLU epilogue */
#define Q4K_KERNEL_SINGLE_LAUNCH 7   /* static partition, activations quantized in the GEMV launch */
#define Q4K_KERNEL_STATIC_TWO_ROW_MMA 8 /* two rows per lane, integer sums on int8 tensor-core MMAs (ncols >= 4) */
Q4K_API int q4k_batch_ex_kernel(const q4k_task_ex *tasks, int ntasks, int ncols, int num_sms);
/* The same question for q4k_gemv_batch_persistent: Q4K_KERNEL_SINGLE_LAUNCH
 * when the tasks run as one launch, else the kernel of its two-launch
 * fallback (its gather argument does not change the answer). */
Q4K_API int q4k_batch_persistent_kernel(const q4k_task *tasks, int ntasks, int ncols, int num_sms);

/* Per-sub-block integer sums as the kernels form them, for bit-exact parity
 * checks (the GEMV kernel runs in a dump mode and writes no dst):
 *   S_out[(j*nrows + r)*(K/32) + b] = sum over sub-block b of row r of
 *                                     nibble * q8 (column j),
 *   T_out[j*(K/32) + b]             = sum of the 32 quants of q8_1 block b
 *                                     of column j (the min-term sum). */
Q4K_API int q4k_debug_subblock_sums(const void *W, const void *y_q8_1, int64_t K, int64_t nrows,
                            int ncols, int64_t stride_row_x, int64_t stride_col_y,
                            int32_t *S_out, int32_t *T_out,
                            void *workspace, size_t workspace_bytes, q4k_stream_t stream);

/* Device status word of the last call that used this workspace (0 = OK,
 * otherwise a q4k_status such as Q4K_ETIMEOUT).  Synchronises the stream. */
Q4K_API int q4k_workspace_status(const void *workspace, int *device_status, q4k_stream_t stream);

/* Launch timeline (diagnostics).  A library built with -DQ4K_TIMELINE=1
 * (make timeline: libq4k_gemv_timeline.so) stamps the device clock
 * (%globaltimer, ns) in every GEMV launch, per CTA and warp, at three points:
 * the warp starts, its griddepcontrol.wait returns, it has flushed its last
 * row group; and in every quantization launch, per CTA: start, wait return,
 * end.  Records go to a ring of Q4K_TIMELINE_SLOTS launches in a device
 * buffer of the current device (allocated at the first call), slot = call
 * index modulo the ring, reset by q4k_timeline_reset:
 *   GEMV  u64[slot][Q4K_TIMELINE_CTAS][16 warps][8] =
 *         {start, wait return, end, atoms of the worker (0: idle), SM id,
 *          worker index, first atom, end atom}; the dynamically scheduled
 *          kernel records atoms done in word 3, 0 in word 6 and its last
 *          queue entry in word 7; the single-launch mode records in words 6
 *          and 7 when its activations were quantized and when the CTA had
 *          planned its activation table
 *   prep  u64[slot][Q4K_TIMELINE_PREP_CTAS][4] = {start, wait return, end, 1}
 * q4k_timeline_bytes() is the size of both regions (GEMV first); it returns 0
 * and the other two Q4K_EINVAL in a library built without the option.  Each
 * device keeps its own buffer; read and reset act on the current device's.
 * The timeline build allocates that buffer at its first call on a device, so
 * in that build q4k_mul_mat_vec_noalloc does allocate (once per device). */
#define Q4K_TIMELINE_SLOTS 64
#define Q4K_TIMELINE_CTAS 256
#define Q4K_TIMELINE_PREP_CTAS 4096
Q4K_API size_t q4k_timeline_bytes(void);
/* Copies the records (bytes <= q4k_timeline_bytes()) after a device
 * synchronisation; *ncalls = calls recorded since the last reset. */
Q4K_API int q4k_timeline_read(void *host, size_t bytes, int *ncalls);
Q4K_API int q4k_timeline_reset(void);

#ifdef __cplusplus
}
#endif
#endif /* Q4K_GEMV_H */
