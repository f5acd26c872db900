// internal.hpp -- host-side plumbing shared by the C-ABI translation units:
// the context object, error reporting, scratch memory and TMA descriptors.
#pragma once

#include <cstdlib>
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "pfrt_cuda.h"

namespace pfrt {
struct StagingRing;  // pinned host chunks for pageable copies (staging.cu)
}

struct pfrt_ctx {
    int device = 0;
    int num_sms = 0;
    int cc_major = 0, cc_minor = 0;
    cudaStream_t stream = nullptr;
    int* d_err = nullptr;       // device error word (pfrt::DeviceError)
    void* scratch = nullptr;    // grow-only scratch arena
    size_t scratch_cap = 0;
    void* io = nullptr;         // grow-only device copies of host-buffer calls' inputs and outputs
    size_t io_cap = 0;
    pfrt::StagingRing* staging = nullptr;  // created by the first staged copy
};

namespace pfrt {

// Records `msg` as this thread's last error and returns `st`.
pfrt_status fail(pfrt_status st, const std::string& msg);
// Maps a CUDA error to PFRT_ERR_CUDA / PFRT_ERR_OUT_OF_MEMORY with context.
pfrt_status cuda_fail(cudaError_t e, const char* what);

#define PFRT_CUDA_TRY(expr)                                 \
    do {                                                    \
        cudaError_t e__ = (expr);                           \
        if (e__ != cudaSuccess) return ::pfrt::cuda_fail(e__, #expr); \
    } while (0)

#define PFRT_CHECK_LAUNCH(what)                             \
    do {                                                    \
        cudaError_t e__ = cudaGetLastError();               \
        if (e__ != cudaSuccess) return ::pfrt::cuda_fail(e__, what); \
    } while (0)

// Frees the context's pinned staging ring (staging.cu), after its copies.
void staging_release(pfrt_ctx* ctx);

// Makes the context's device current for the calling thread.
pfrt_status enter(pfrt_ctx* ctx);
cudaStream_t pick_stream(pfrt_ctx* ctx, pfrt_stream s);

// Returns a pointer to at least `bytes` of scratch device memory owned by the
// context.  Growing it synchronizes the device.  The memory is shared by all
// calls on the context.
pfrt_status scratch(pfrt_ctx* ctx, size_t bytes, void** out);
// The same for the device copies of a host-buffer call (pfrt_qlinear_host);
// separate from the scratch arena, which the call's kernels use.
pfrt_status io_buffer(pfrt_ctx* ctx, size_t bytes, void** out);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// 2-D K-major tensor map with 128-byte swizzle:
// global [rows, cols] with row stride `ld_bytes`, box [box_rows, 128 bytes].
pfrt_status make_tmap_2d(CUtensorMap* tm, const void* base, CUtensorMapDataType dt, int elem_bytes,
                         uint64_t cols, uint64_t rows, uint64_t ld_bytes, uint32_t box_cols,
                         uint32_t box_rows);

// 2-D tensor map without swizzle: global [rows, cols] with row stride
// `ld_bytes`, box [box_rows, box_cols]; box_cols * elem_bytes a multiple of 16.
pfrt_status make_tmap_2d_plain(CUtensorMap* tm, const void* base, CUtensorMapDataType dt,
                               int elem_bytes, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                               uint32_t box_cols, uint32_t box_rows);

// Wraps device buffers hi/lo [N][Kpad] (K-major, tf32 split, zero padded,
// Kpad = K rounded up to 32) as a prepared fp32 weight.  The weight takes
// ownership of both buffers.
pfrt_status fweight_from_device_split(pfrt_ctx* ctx, int64_t N, int64_t K, float* hi, float* lo,
                                      pfrt_fweight** out);

// Y[M, N] = A[M, K] * B^T on a prepared weight (alpha 1, beta 0, no C), with
// row strides lda (>= K) and ldy (>= N); the context's device is current and
// `s` the stream.  Used by the SpMM's dense path, which may write a column
// block of a wider output.  The epilogue also stores every output value into
// the n_peer_y (at most 7) further outputs peer_y[i], same offsets and row
// stride (other GPUs' outputs mapped into this process).
pfrt_status gemm_f32_strided(pfrt_ctx* ctx, int64_t M, const float* a, int64_t lda, const pfrt_fweight* b,
                             float* y, int64_t ldy, cudaStream_t s, float* const* peer_y = nullptr,
                             int n_peer_y = 0);

// hi[r, k] = tf32(src[r*ld + k]), lo = src - hi for k < K, zeros for
// K <= k < Kpad: the K-major 3xTF32 split of a row-major operand.
pfrt_status split_tf32_kmajor(const float* src, int64_t rows, int64_t K, int64_t ld, float* hi, float* lo,
                              int64_t Kpad, cudaStream_t s);

// Fills `a` with the programmatic-stream-serialization launch attribute
// (the kernel may start while the previous kernel on the stream finishes;
// it calls pdl_wait before touching that kernel's data) and returns 1, or
// returns 0 when PFRT_PDL=0.
inline int pdl_attr(cudaLaunchAttribute* a) {
    static const bool on = [] {
        const char* v = std::getenv("PFRT_PDL");
        return !(v && *v == '0');
    }();
    if (!on) return 0;
    a->id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a->val.programmaticStreamSerializationAllowed = 1;
    return 1;
}

}  // namespace pfrt
