/*
 * pfrt_cuda.h -- C ABI of the B200 (sm_100a) backend for PyFlameRT's
 * MatMul / Gemm / QuantizedMatMul / sparse-weight MatMul hot path.
 *
 * Plain C: pointers, sizes and status codes, no C++ or torch types, so the
 * library can be bound from C++ (the PyFlameRT CudaBackend), ctypes, cgo or
 * JNI alike.  Device pointers are CUDA device addresses of the context's
 * device; "host" pointers are ordinary host memory.  Every function returns
 * PFRT_OK (0) or an error code; pfrt_last_error() gives the message of the
 * last failure on the calling thread.  There is no CPU fallback: on a machine
 * without a usable sm_100 GPU, pfrt_ctx_create fails with PFRT_ERR_NO_DEVICE.
 *
 * Layouts are dense row-major, as in the reference Tensor
 * (include/pyflame_rt/tensor.hpp:12-90).  Each entry point names the
 * reference routine whose result it reproduces.
 *
 * Kernels are enqueued asynchronously on the given stream (NULL = the
 * context's own stream, (pfrt_stream)1 = CUDA's legacy default stream).  Device-side failures (a bounded wait that gave up,
 * an out-of-range CSR index) are recorded in the context and reported by
 * pfrt_ctx_check().  A context and its scratch memory serve one stream at a
 * time; use one context per thread for concurrent calls.
 */
#ifndef PFRT_CUDA_H
#define PFRT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PFRT_API __attribute__((visibility("default")))
#else
#define PFRT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum pfrt_status {
    PFRT_OK = 0,
    PFRT_ERR_INVALID_ARGUMENT = 1, /* shape / dtype / attribute error (the reference throws std::invalid_argument) */
    PFRT_ERR_BAD_CSR = 2,          /* malformed CSR structure or index out of range */
    PFRT_ERR_CUDA = 3,             /* CUDA runtime or launch failure */
    PFRT_ERR_OUT_OF_MEMORY = 4,
    PFRT_ERR_UNSUPPORTED = 5,      /* a size or mode this backend does not implement */
    PFRT_ERR_DEVICE_TIMEOUT = 6,   /* a bounded device-side wait gave up */
    PFRT_ERR_NO_DEVICE = 7         /* no usable sm_100 device */
} pfrt_status;

/* Output element types of the quantized path. */
typedef enum pfrt_out_mode {
    PFRT_OUT_F32 = 0, /* dequantized fp32 (quant_ops.cpp:464) */
    PFRT_OUT_S8 = 1,  /* requantized int8 (quantize_tensor, quant_ops.cpp:42-47) */
    PFRT_OUT_U8 = 2   /* requantized uint8 (quant_ops.cpp:49-54) */
} pfrt_out_mode;

typedef struct pfrt_ctx pfrt_ctx;
typedef struct pfrt_qweight pfrt_qweight;
typedef struct pfrt_fweight pfrt_fweight;
typedef struct pfrt_csr pfrt_csr;
/* A cudaStream_t.  NULL selects the context's own stream; CUDA's legacy
 * default stream is (pfrt_stream)1 (cudaStreamLegacy). */
typedef void* pfrt_stream;

/* ------------------------------------------------------------ context
 * Replaces the CPUExecutor construction in InferenceSession::select_backend
 * (src/session.cpp:90-94): one context per device. */
PFRT_API const char* pfrt_version(void);
PFRT_API const char* pfrt_last_error(void);
PFRT_API pfrt_status pfrt_device_count(int* count);
PFRT_API pfrt_status pfrt_ctx_create(int device, pfrt_ctx** out);
PFRT_API pfrt_status pfrt_ctx_destroy(pfrt_ctx* ctx);
PFRT_API pfrt_status pfrt_ctx_stream(pfrt_ctx* ctx, pfrt_stream* out);
PFRT_API pfrt_status pfrt_ctx_num_sms(pfrt_ctx* ctx, int* out);
/* Synchronizes `stream` and reports device-side failures recorded since the
 * last check (PFRT_ERR_DEVICE_TIMEOUT, PFRT_ERR_BAD_CSR); clears them. */
PFRT_API pfrt_status pfrt_ctx_check(pfrt_ctx* ctx, pfrt_stream stream);

/* ------------------------------------------------------------ memory
 * Device and pinned host buffers, so that C callers need no CUDA headers.
 * Copies are asynchronous on `stream` (pinned host memory for overlap). */
PFRT_API pfrt_status pfrt_malloc(pfrt_ctx* ctx, size_t bytes, void** dptr);
PFRT_API pfrt_status pfrt_free(pfrt_ctx* ctx, void* dptr);
PFRT_API pfrt_status pfrt_host_alloc(pfrt_ctx* ctx, size_t bytes, void** hptr);
PFRT_API pfrt_status pfrt_host_free(pfrt_ctx* ctx, void* hptr);
PFRT_API pfrt_status pfrt_memcpy_h2d(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream stream);
PFRT_API pfrt_status pfrt_memcpy_d2h(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream stream);
PFRT_API pfrt_status pfrt_memcpy_d2d(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream stream);
PFRT_API pfrt_status pfrt_memset(pfrt_ctx* ctx, void* dst, int value, size_t bytes, pfrt_stream stream);
/* Copies between PAGEABLE host memory (a host Tensor of the reference
 * runtime, src/tensor.cpp) and the device.  They replace the per-run host
 * copies of graph inputs and outputs that CPUExecutor::execute makes
 * (src/backends/cpu/executor.cpp:65-74).  The bytes go through the context's
 * ring of pinned buffers (8 x 256 KiB, allocated by the first call): several
 * host threads copy one chunk while the DMA of the previous chunk runs.
 * pfrt_memcpy_h2d_staged returns once src has been read (its DMAs complete
 * in order on `stream`); pfrt_memcpy_d2h_staged returns once dst holds the
 * bytes (it waits for the work queued before it on `stream`). */
PFRT_API pfrt_status pfrt_memcpy_h2d_staged(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes,
                                            pfrt_stream stream);
PFRT_API pfrt_status pfrt_memcpy_d2h_staged(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes,
                                            pfrt_stream stream);

/* ------------------------------------------------------------ fp32 Gemm / MatMul
 * Replaces cpu_gemm (src/backends/cpu/ops/math.cpp:377-438) and the 2-D path
 * of cpu_matmul (math.cpp:326-336):
 *     Y[M,N] = alpha * op(A) * op(B) + beta * C[(m*N + n) % c_len]
 * computed on tcgen05 tensor cores with the 3xTF32 split (hi*hi + hi*lo +
 * lo*hi), which keeps the result within ~1e-6 relative of fp32.
 *
 * pfrt_fweight_create uploads and prepares a constant B operand (a graph
 * initializer) once: B is [K,N] (trans_b = 0) or [N,K] (trans_b = 1) in HOST
 * memory.  pfrt_gemm_f32 then takes device A ([M,K], or [K,M] if trans_a),
 * optional device C of c_len elements (c_len = 0 or C = NULL: no bias), and
 * writes device Y [M,N]. */
PFRT_API pfrt_status pfrt_fweight_create(pfrt_ctx* ctx, int64_t K, int64_t N, int trans_b,
                                const float* b_host, pfrt_fweight** out);
PFRT_API pfrt_status pfrt_fweight_destroy(pfrt_fweight* w);
PFRT_API pfrt_status pfrt_gemm_f32(pfrt_ctx* ctx, int64_t M, int trans_a, float alpha, const float* a,
                          const pfrt_fweight* b, float beta, const float* c, int64_t c_len,
                          float* y, pfrt_stream stream);
/* No counterpart in the reference: an allocation-free form of pfrt_gemm_f32
 * for callers that cannot allocate device memory while they run (for example
 * a host program whose device memory is all handed out by its own pool, or a
 * latency-bound loop that must not pay cudaMalloc's device synchronization).
 * Same arguments as pfrt_gemm_f32; the per-call split of A uses a fixed
 * 16 MiB device array built into the library instead of the context's
 * scratch memory.  Limit: M * Kpad <= 2097152 (Kpad = K rounded up to 32),
 * else PFRT_ERR_UNSUPPORTED.  No split-K (no room for partial sums;
 * PFRT_GEMM_SPLITS is ignored): the result agrees with pfrt_gemm_f32 within
 * fp32 tolerance, and shapes whose tiles leave SMs idle may run slower.  The
 * first call on each device does a one-time set-up (it looks up the array's
 * device address), so make that first call before any stream capture.  All
 * calls share the array and it keeps the last call's contents: calls that
 * overlap on the GPU race on it. */
PFRT_API pfrt_status pfrt_gemm_f32_noalloc(pfrt_ctx* ctx, int64_t M, int trans_a, float alpha,
                                           const float* a, const pfrt_fweight* b, float beta,
                                           const float* c, int64_t c_len, float* y,
                                           pfrt_stream stream);
/* Same with B a device matrix given per call (a graph input rather than an
 * initializer); B is prepared into the context's scratch memory each call. */
PFRT_API pfrt_status pfrt_gemm_f32_dense(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t K, int trans_a,
                                int trans_b, float alpha, const float* a, const float* b,
                                float beta, const float* c, int64_t c_len, float* y,
                                pfrt_stream stream);

/* ------------------------------------------------------------ quantized MatMul
 * Replaces quantization::quantized_matmul + quantize_tensor
 * (src/quantization/quant_ops.cpp:387-506, 15-127) and, fused, the Add (bias)
 * and Relu that follow it (math.cpp:222-226, activation.cpp:45-60), with
 * per-output-channel weight scales:
 *     acc[m,n] = sum_k (a[m,k] - a_zp) * (w[k,n] - w_zp)       (exact int)
 *     y        = (float)acc * (a_scale * w_scale[n])  [+ bias[n]]  [max(0,.)]
 *     out      = y (PFRT_OUT_F32) or clamp(round(y / y_scale) + y_zp)
 * Results are bit-identical to the reference CPU arithmetic.
 *
 * pfrt_qweight_create uploads int8 weights w [K,N] (the reference's B
 * layout, HOST memory) once, with w_zp and n_scales = N per-channel scales
 * (or 1 per-tensor scale).  K must be <= 65536 (the s32 tensor-core
 * accumulator is exact up to there).
 *
 * pfrt_qlinear: a is device [M,K] uint8 (a_is_u8 = 1) or int8 with row
 * stride lda elements (lda >= K); bias is device fp32 [N] or NULL; y is device
 * [M,N] with row stride ldy elements, fp32 or int8/uint8 per out_mode;
 * acc_out (device int32 [M,N], nullable) receives the exact accumulators. */
PFRT_API pfrt_status pfrt_qweight_create(pfrt_ctx* ctx, int64_t K, int64_t N, const int8_t* w_host,
                                int32_t w_zp, const float* w_scale_host, int64_t n_scales,
                                pfrt_qweight** out);
PFRT_API pfrt_status pfrt_qweight_destroy(pfrt_qweight* w);
PFRT_API pfrt_status pfrt_qlinear(pfrt_ctx* ctx, const pfrt_qweight* w, int64_t M, const void* a,
                         int64_t lda, int a_is_u8, float a_scale, int32_t a_zp,
                         const float* bias, int relu, int out_mode, float y_scale, int32_t y_zp,
                         void* y, int64_t ldy, int32_t* acc_out, pfrt_stream stream);
/* pfrt_qlinear with HOST activations and output: the layer as
 * InferenceSession::run presents it (src/session.cpp:97-120, host tensors in
 * and out).  Copies a_host [M rows, stride lda bytes] to the device, runs
 * pfrt_qlinear, and copies the result to y_host [M rows, stride ldy
 * elements]; bytes between rows are not touched.  Asynchronous on `stream`
 * (all three steps in order): with pinned host buffers (pfrt_host_alloc) the
 * copies overlap other streams' work, and y_host is valid once the stream is
 * synchronized (pfrt_ctx_check).  The device copies are the context's own,
 * so a context serves one such stream at a time.  bias stays a device
 * pointer (a parameter prepared once, like the weight). */
PFRT_API pfrt_status pfrt_qlinear_host(pfrt_ctx* ctx, const pfrt_qweight* w, int64_t M, const void* a_host,
                                       int64_t lda, int a_is_u8, float a_scale, int32_t a_zp,
                                       const float* bias, int relu, int out_mode, float y_scale,
                                       int32_t y_zp, void* y_host, int64_t ldy, pfrt_stream stream);

/* ------------------------------------------------------------ CSR SpMM
 * Replaces pruning::sparse_matmul (src/pruning/sparse_tensor.cpp:473-519) in
 * the pruned-Linear orientation used by the SparseMatMul graph op:
 *     Y[M,N] = X[M,K] * W^T,   W [N,K] in CSR (one CSR row per output channel)
 * i.e. Y = transpose(sparse_matmul(W, X^T)).
 *
 * pfrt_csr_create validates and uploads a HOST CSR once: indptr [N+1] and
 * indices [nnz] of int32 (index_bits = 32) or int64 (index_bits = 64), values
 * fp32 [nnz].  It checks what SparseTensor::from_csr (:170-197) does not:
 * indptr[0] = 0, indptr non-decreasing, indptr[N] = nnz, 0 <= index < K
 * (PFRT_ERR_BAD_CSR otherwise).  The device copy uses int32 indices.
 *
 * pfrt_spmm: X device [M,K] (row stride ldx), Y device [M,N] (row stride ldy).
 * The first call with a given M class builds state kept with the CSR (for
 * M = 3..8 a row partition; for M > 8 row groups, a dense copy of W, W's
 * compressed form, or its structured-sparse form: for M >= 16 the first call
 * counts the entries past the second of every group of four columns, and
 * the first call that chooses the structured-sparse tensor cores builds W's
 * 2:4 part, as images or, for large sparse weights, as a compressed form the
 * kernel expands on chip, and its remainder; each allocates device memory
 * and synchronizes):
 * make one call of each batch size class before capturing calls in a CUDA
 * graph, and do not use one CSR from several threads or contexts at once.
 * pfrt_spmm_csr_f32: same on a caller-owned device CSR (int32); the kernel
 * bounds-checks every index, skips out-of-range entries and reports
 * PFRT_ERR_BAD_CSR through pfrt_ctx_check(). */
PFRT_API pfrt_status pfrt_csr_create(pfrt_ctx* ctx, int64_t N, int64_t K, int64_t nnz,
                            const void* indptr_host, const void* indices_host, int index_bits,
                            const float* values_host, pfrt_csr** out);
PFRT_API pfrt_status pfrt_csr_destroy(pfrt_csr* w);
/* The host-side structure check of pfrt_csr_create on its own (no device
 * needed): returns PFRT_OK or PFRT_ERR_BAD_CSR / PFRT_ERR_INVALID_ARGUMENT. */
PFRT_API pfrt_status pfrt_csr_validate_host(int64_t N, int64_t K, int64_t nnz,
                                            const void* indptr_host, const void* indices_host,
                                            int index_bits);
PFRT_API pfrt_status pfrt_csr_info(const pfrt_csr* w, int64_t* n, int64_t* k, int64_t* nnz);
PFRT_API pfrt_status pfrt_spmm(pfrt_ctx* ctx, const pfrt_csr* w, int64_t M, const float* x, int64_t ldx,
                      float* y, int64_t ldy, pfrt_stream stream);
PFRT_API pfrt_status pfrt_spmm_csr_f32(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t K, int64_t nnz,
                              const int32_t* indptr, const int32_t* indices,
                              const float* values, const float* x, int64_t ldx, float* y,
                              int64_t ldy, pfrt_stream stream);

/* Magnitude pruning of a dense fp32 weight straight into a CSR weight (the
 * "pruning -> CSR" step that feeds SparseMatMul).  Reproduces
 * pruning::MagnitudePruning::compute_mask (src/pruning/magnitude_pruning.cpp:
 * 22-102) followed by pruning::to_sparse of W * mask with threshold 0
 * (src/pruning/sparse_tensor.cpp:560-587): the threshold is the
 * floor(n*sparsity)-th smallest |w|, weights above it are kept, ties at it
 * are kept in index order while more than (size_t)((float)n * sparsity)
 * weights would be pruned, and the CSR holds the kept nonzeros row by row.
 * w_dev: device W [N, K] (one CSR row per row of W).  The threshold search,
 * the tie ranking and the compaction run on the GPU; the CSR is then prepared
 * as by pfrt_csr_create.  mask_dev (optional, device [N*K] floats) receives
 * compute_mask's 0/1 mask.  NaN weights: PFRT_ERR_INVALID_ARGUMENT (the
 * reference's sort is undefined for them); N*K = 0 with 0 < sparsity < 1:
 * PFRT_ERR_INVALID_ARGUMENT "Cannot prune empty weight tensor", as the
 * reference throws. */
PFRT_API pfrt_status pfrt_csr_from_magnitude_pruning(pfrt_ctx* ctx, int64_t N, int64_t K, const float* w_dev,
                                                     float sparsity, float* mask_dev, pfrt_csr** out);

/* Replaces pruning::NMSparsityPruning(n, m).compute_mask (src/pruning/
 * nm_sparsity.cpp:45-126) followed by to_sparse(W * mask) (sparse_tensor.cpp:
 * 560-587) for a device weight W [N, K]: in every m consecutive weights of W
 * in row-major order (a group may span rows; the last may be shorter) the n
 * largest |w| are kept, equal ones chosen as the reference's
 * std::partial_sort (libstdc++) chooses them.  mask_dev (nullable, N*K
 * floats) receives the 0/1 mask.  Errors as the reference's constructor:
 * n > m "N must be <= M in N:M sparsity", n or m 0 "N and M must be > 0";
 * m above 32 is PFRT_ERR_UNSUPPORTED. */
PFRT_API pfrt_status pfrt_csr_from_nm_pruning(pfrt_ctx* ctx, int64_t N, int64_t K, const float* w_dev, int32_t n,
                                              int32_t m, float* mask_dev, pfrt_csr** out);

/* ------------------------------------------------------------ peer memory
 * No counterpart in the reference: it has no communication backend (its
 * partitioner, src/partition/graph_partitioner.cpp:111-200, only plans
 * CommOps).  These entry points let the ranks of one node (one process per
 * GPU) map each other's device buffers over NVLink.
 *
 * pfrt_ipc_get_handle: a process-shareable handle (64 opaque bytes) of a
 * buffer from pfrt_malloc; pfrt_ipc_open maps a handle made by another
 * process into this context; pfrt_ipc_close unmaps it. */
typedef struct pfrt_ipc_handle {
    unsigned char bytes[64];
} pfrt_ipc_handle;
PFRT_API pfrt_status pfrt_ipc_get_handle(pfrt_ctx* ctx, const void* dev_ptr, pfrt_ipc_handle* out);
PFRT_API pfrt_status pfrt_ipc_open(pfrt_ctx* ctx, const pfrt_ipc_handle* handle, void** dev_ptr);
PFRT_API pfrt_status pfrt_ipc_close(pfrt_ctx* ctx, void* dev_ptr);

/* Output-channel-sharded SpMM fused with the all-gather of its output.
 * Replaces pruning::sparse_matmul (src/pruning/sparse_tensor.cpp:473-519) for
 * a W too large to replicate: rank r holds rows [r*ns, r*ns + ns) of W as its
 * CSR w_shard (ns = w_shard's N) and the whole X [M, K], and every rank ends
 * with the whole Y [M, world*ns] in its own y (row stride world*ns).  The
 * reference has no communication backend; the exchange is the all-gather its
 * partitioner plans (src/partition/graph_partitioner.cpp:111-200).
 *
 * M = 1: the kernel sends every output value straight to every other rank as
 * it is computed, together with the call's number in one 8-byte store over
 * NVLink (no fences), and each rank's blocks unpack the values that arrive
 * into its own y.
 * M > 1: the rank computes its column block of Y into its own y (the kernel
 * pfrt_spmm would pick for the shard) and the block reaches every other
 * rank's y over NVLink: by a copy kernel after the SpMM, or (PFRT_PEER_FUSE=1,
 * dense path only) stored by the shard GEMM's epilogue as each tile is
 * computed.  Nothing is written into another rank's y before that
 * rank has declared it free for this call (a rank declares it when its
 * stream reaches the call, i.e. after everything it ran on the previous
 * output); the call ends once every other rank has reported its block
 * written.
 *
 * The call number lives on the device (the call can sit in a CUDA graph).  A
 * rank can run at most one call ahead of another without overwriting data
 * not yet read.  Every rank must make the same sequence of calls with the
 * same M; consumers of y must run on the call's stream (or after it).
 *
 *   y          this rank's gathered output [max_m][world*ns] floats (device);
 *   recv[p]    rank p's M = 1 receive buffer [2][world*ns] uint64, mapped
 *              into this process (pfrt_ipc_open; recv[rank] is this rank's
 *              own);
 *   state      this rank's private [4] uint32;
 *   ns, max_m  the shard height and the rows of y (M <= max_m);
 *   y_peer[p]  rank p's y mapped into this process (y_peer[rank] = y);
 *   sig[p]     rank p's signal words [PFRT_PEER_SIG_WORDS] uint32, mapped
 *              into this process (sig[rank] is this rank's own).
 * recv, state and sig are zeroed once before the first call.  y_peer and sig
 * are needed for M > 1 only.
 *
 * Waits on other ranks give up after about 2 s (PFRT_PEER_WAIT_MS overrides
 * the limit): the call then reports PFRT_ERR_DEVICE_TIMEOUT through
 * pfrt_ctx_check, and later calls report it at once until every rank has
 * called pfrt_peer_reset (and the ranks have synchronized on the host).
 * M > max_m or missing M > 1 buffers: PFRT_ERR_INVALID_ARGUMENT. */
#define PFRT_MAX_PEERS 8
#define PFRT_PEER_SIG_WORDS 16
typedef struct pfrt_peer_set {
    int32_t rank;
    int32_t world;
    float* y;
    uint64_t* recv[PFRT_MAX_PEERS];
    uint32_t* state;
    int64_t ns;
    int64_t max_m;
    float* y_peer[PFRT_MAX_PEERS];
    uint32_t* sig[PFRT_MAX_PEERS];
} pfrt_peer_set;
PFRT_API pfrt_status pfrt_spmm_allgather(pfrt_ctx* ctx, const pfrt_csr* w_shard, int64_t M, const float* x,
                                         int64_t ldx, const pfrt_peer_set* peers, pfrt_stream stream);
/* The all-gather alone, for an output whose column blocks the ranks have
 * computed themselves: rank r has written columns [r*ns, r*ns + ns) of the
 * first M rows of its own y (row stride world*ns); the call stores that block
 * into every other rank's y and returns once every other rank's block has
 * arrived.  Same protocol, call numbering and rules as pfrt_spmm_allgather
 * with M > 1 (the two share one call sequence).  The C-ABI form of the NCCL
 * all-gather of column blocks that the reference's partitioner plans as a
 * CommOp (src/partition/graph_partitioner.cpp:111-200). */
PFRT_API pfrt_status pfrt_peer_allgather(pfrt_ctx* ctx, int64_t M, const pfrt_peer_set* peers, pfrt_stream stream);
/* No counterpart in the reference.  Zeroes this rank's state, its M = 1
 * receive buffer and its signal words (asynchronously on `stream`), which
 * clears a timeout recorded by pfrt_spmm_allgather.  Every rank of the set
 * calls it, and the ranks synchronize their streams and each other on the
 * host, before the next pfrt_spmm_allgather. */
PFRT_API pfrt_status pfrt_peer_reset(pfrt_ctx* ctx, const pfrt_peer_set* peers, pfrt_stream stream);

/* ------------------------------------------------------------ elementwise
 * Standalone forms of the ops the backend normally fuses into epilogues:
 * quantize_tensor per-tensor (quant_ops.cpp:33-55), bias Add broadcast over
 * rows (math.cpp:222-226 for a [N] operand) and Relu (activation.cpp:45-60). */
PFRT_API pfrt_status pfrt_quantize_f32(pfrt_ctx* ctx, int64_t n, const float* x, float scale, int32_t zp,
                              int out_is_u8, void* q, pfrt_stream stream);
PFRT_API pfrt_status pfrt_add_rowvec_f32(pfrt_ctx* ctx, int64_t rows, int64_t cols, const float* x,
                                const float* b, float* y, pfrt_stream stream);
PFRT_API pfrt_status pfrt_relu_f32(pfrt_ctx* ctx, int64_t n, const float* x, float* y,
                          pfrt_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* PFRT_CUDA_H */
