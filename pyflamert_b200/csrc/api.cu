// api.cu -- context, memory and error entry points of the C ABI, and the
// shared host plumbing (scratch arena, TMA descriptor encoding).
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.hpp"

namespace pfrt {

namespace {
thread_local std::string g_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
}  // namespace

pfrt_status fail(pfrt_status st, const std::string& msg) {
    g_last_error = msg;
    return st;
}

pfrt_status cuda_fail(cudaError_t e, const char* what) {
    cudaGetLastError();  // clear a sticky-free error so later calls are not misattributed
    const pfrt_status st =
        (e == cudaErrorMemoryAllocation) ? PFRT_ERR_OUT_OF_MEMORY : PFRT_ERR_CUDA;
    return fail(st, std::string(what) + ": " + cudaGetErrorString(e));
}

pfrt_status enter(pfrt_ctx* ctx) {
    if (ctx == nullptr) return fail(PFRT_ERR_INVALID_ARGUMENT, "null context");
    PFRT_CUDA_TRY(cudaSetDevice(ctx->device));
    return PFRT_OK;
}

cudaStream_t pick_stream(pfrt_ctx* ctx, pfrt_stream s) {
    return s ? static_cast<cudaStream_t>(s) : ctx->stream;
}

pfrt_status scratch(pfrt_ctx* ctx, size_t bytes, void** out) {
    if (bytes == 0) bytes = 256;
    if (bytes > ctx->scratch_cap) {
        const size_t cap = align_up(bytes + bytes / 4, 1 << 20);
        PFRT_CUDA_TRY(cudaDeviceSynchronize());
        if (ctx->scratch) PFRT_CUDA_TRY(cudaFree(ctx->scratch));
        ctx->scratch = nullptr;
        ctx->scratch_cap = 0;
        PFRT_CUDA_TRY(cudaMalloc(&ctx->scratch, cap));
        ctx->scratch_cap = cap;
    }
    *out = ctx->scratch;
    return PFRT_OK;
}

pfrt_status io_buffer(pfrt_ctx* ctx, size_t bytes, void** out) {
    if (bytes == 0) bytes = 256;
    if (bytes > ctx->io_cap) {
        const size_t cap = align_up(bytes + bytes / 4, 1 << 20);
        PFRT_CUDA_TRY(cudaDeviceSynchronize());
        if (ctx->io) PFRT_CUDA_TRY(cudaFree(ctx->io));
        ctx->io = nullptr;
        ctx->io_cap = 0;
        PFRT_CUDA_TRY(cudaMalloc(&ctx->io, cap));
        ctx->io_cap = cap;
    }
    *out = ctx->io;
    return PFRT_OK;
}

pfrt_status make_tmap_2d(CUtensorMap* tm, const void* base, CUtensorMapDataType dt, int elem_bytes,
                         uint64_t cols, uint64_t rows, uint64_t ld_bytes, uint32_t box_cols,
                         uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return fail(PFRT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "TMA base address must be 16-byte aligned");
    if (ld_bytes % 16 != 0)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "TMA row stride must be a multiple of 16 bytes");
    if (static_cast<uint64_t>(box_cols) * elem_bytes != 128)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "TMA box inner extent must be 128 bytes");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(PFRT_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string(r) + ")");
    return PFRT_OK;
}

pfrt_status make_tmap_2d_plain(CUtensorMap* tm, const void* base, CUtensorMapDataType dt,
                               int elem_bytes, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                               uint32_t box_cols, uint32_t box_rows) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return fail(PFRT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || ld_bytes % 16 != 0 ||
        (static_cast<uint64_t>(box_cols) * elem_bytes) % 16 != 0 || box_cols > 256 || box_rows > 256)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "TMA tensor map: alignment or box size");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(PFRT_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string(r) + ")");
    return PFRT_OK;
}

}  // namespace pfrt

using namespace pfrt;

extern "C" {

const char* pfrt_version(void) { return "pfrt-b200 0.1.0 (sm_100a)"; }

const char* pfrt_last_error(void) { return g_last_error.c_str(); }

pfrt_status pfrt_device_count(int* count) {
    if (!count) return fail(PFRT_ERR_INVALID_ARGUMENT, "null count");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
        return fail(PFRT_ERR_NO_DEVICE, std::string("no CUDA device: ") + cudaGetErrorString(e));
    }
    *count = n;
    return PFRT_OK;
}

pfrt_status pfrt_ctx_create(int device, pfrt_ctx** out) {
    if (!out) return fail(PFRT_ERR_INVALID_ARGUMENT, "null output");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(PFRT_ERR_NO_DEVICE, "no CUDA device visible");
    }
    if (device < 0 || device >= n)
        return fail(PFRT_ERR_NO_DEVICE, "device ordinal " + std::to_string(device) +
                                            " out of range (" + std::to_string(n) + " visible)");
    cudaDeviceProp prop{};
    PFRT_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(PFRT_ERR_NO_DEVICE, std::string("device ") + prop.name + " is sm_" +
                                            std::to_string(prop.major) + std::to_string(prop.minor) +
                                            "; this library is built for sm_100a only");
    auto* ctx = new pfrt_ctx();
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    ctx->cc_major = prop.major;
    ctx->cc_minor = prop.minor;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(int));
    if (e != cudaSuccess) {
        pfrt_ctx_destroy(ctx);
        return cuda_fail(e, "pfrt_ctx_create");
    }
    *out = ctx;
    return PFRT_OK;
}

pfrt_status pfrt_ctx_destroy(pfrt_ctx* ctx) {
    if (!ctx) return PFRT_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    staging_release(ctx);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->io) cudaFree(ctx->io);
    if (ctx->d_err) cudaFree(ctx->d_err);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return PFRT_OK;
}

pfrt_status pfrt_ctx_stream(pfrt_ctx* ctx, pfrt_stream* out) {
    if (!ctx || !out) return fail(PFRT_ERR_INVALID_ARGUMENT, "null argument");
    *out = ctx->stream;
    return PFRT_OK;
}

pfrt_status pfrt_ctx_num_sms(pfrt_ctx* ctx, int* out) {
    if (!ctx || !out) return fail(PFRT_ERR_INVALID_ARGUMENT, "null argument");
    *out = ctx->num_sms;
    return PFRT_OK;
}

pfrt_status pfrt_ctx_check(pfrt_ctx* ctx, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    cudaStream_t s = pick_stream(ctx, stream);
    PFRT_CUDA_TRY(cudaStreamSynchronize(s));
    int h = 0;
    PFRT_CUDA_TRY(cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h == 0) return PFRT_OK;
    PFRT_CUDA_TRY(cudaMemset(ctx->d_err, 0, sizeof(int)));
    if (h == 1)
        return fail(PFRT_ERR_DEVICE_TIMEOUT,
                    "a kernel's bounded wait gave up; its output is not valid");
    if (h == 2)
        return fail(PFRT_ERR_BAD_CSR, "CSR index out of range: the entry was skipped");
    return fail(PFRT_ERR_CUDA, "device error code " + std::to_string(h));
}

pfrt_status pfrt_ipc_get_handle(pfrt_ctx* ctx, const void* dev_ptr, pfrt_ipc_handle* out) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!dev_ptr || !out) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_ipc_get_handle: null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(pfrt_ipc_handle), "IPC handle size");
    cudaIpcMemHandle_t h;
    PFRT_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
    std::memset(out, 0, sizeof(*out));
    std::memcpy(out->bytes, &h, sizeof(h));
    return PFRT_OK;
}

pfrt_status pfrt_ipc_open(pfrt_ctx* ctx, const pfrt_ipc_handle* handle, void** dev_ptr) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!handle || !dev_ptr) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_ipc_open: null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    PFRT_CUDA_TRY(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return PFRT_OK;
}

pfrt_status pfrt_ipc_close(pfrt_ctx* ctx, void* dev_ptr) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!dev_ptr) return PFRT_OK;
    PFRT_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
    return PFRT_OK;
}

pfrt_status pfrt_malloc(pfrt_ctx* ctx, size_t bytes, void** dptr) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!dptr) return fail(PFRT_ERR_INVALID_ARGUMENT, "null output");
    PFRT_CUDA_TRY(cudaMalloc(dptr, bytes ? bytes : 1));
    return PFRT_OK;
}

pfrt_status pfrt_free(pfrt_ctx* ctx, void* dptr) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (dptr) PFRT_CUDA_TRY(cudaFree(dptr));
    return PFRT_OK;
}

pfrt_status pfrt_host_alloc(pfrt_ctx* ctx, size_t bytes, void** hptr) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!hptr) return fail(PFRT_ERR_INVALID_ARGUMENT, "null output");
    PFRT_CUDA_TRY(cudaMallocHost(hptr, bytes ? bytes : 1));
    return PFRT_OK;
}

pfrt_status pfrt_host_free(pfrt_ctx* ctx, void* hptr) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (hptr) PFRT_CUDA_TRY(cudaFreeHost(hptr));
    return PFRT_OK;
}

static pfrt_status copy(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream s,
                        cudaMemcpyKind kind) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (bytes == 0) return PFRT_OK;
    if (!dst || !src) return fail(PFRT_ERR_INVALID_ARGUMENT, "null pointer");
    PFRT_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, kind, pick_stream(ctx, s)));
    return PFRT_OK;
}

pfrt_status pfrt_memcpy_h2d(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream s) {
    return copy(ctx, dst, src, bytes, s, cudaMemcpyHostToDevice);
}
pfrt_status pfrt_memcpy_d2h(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream s) {
    return copy(ctx, dst, src, bytes, s, cudaMemcpyDeviceToHost);
}
pfrt_status pfrt_memcpy_d2d(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream s) {
    return copy(ctx, dst, src, bytes, s, cudaMemcpyDeviceToDevice);
}

pfrt_status pfrt_memset(pfrt_ctx* ctx, void* dst, int value, size_t bytes, pfrt_stream s) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (bytes == 0) return PFRT_OK;
    PFRT_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, pick_stream(ctx, s)));
    return PFRT_OK;
}

}  // extern "C"
