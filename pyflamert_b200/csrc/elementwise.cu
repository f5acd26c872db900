// elementwise.cu -- standalone forms of the ops the backend normally fuses
// into GEMM epilogues: per-tensor requantization, bias Add broadcast over
// rows, and Relu.  Used when a graph has them without a producing GEMM to
// fuse into.  Memory-bound; grid-stride loops over a persistent grid.
#include <algorithm>
#include <cmath>
#include <string>

#include "epilogues.cuh"
#include "internal.hpp"

namespace pfrt {

// quantize_tensor per-tensor branch (src/quantization/quant_ops.cpp:33-55).
__global__ void quantize_kernel(int64_t n, const float* __restrict__ x, float inv_scale, int32_t zp,
                                int u8, uint8_t* __restrict__ q) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        q[i] = static_cast<uint8_t>(requant_rn(x[i], inv_scale, zp, u8 != 0) & 0xFF);
}

// binary_elementwise Add with a [cols] operand broadcast over rows
// (src/backends/cpu/ops/math.cpp:141-226).
__global__ void add_rowvec_kernel(int64_t rows, int64_t cols, const float* __restrict__ x,
                                  const float* __restrict__ b, float* __restrict__ y) {
    const int64_t n = rows * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = __fadd_rn(x[i], b[i % cols]);
}

// cpu_relu (src/backends/cpu/ops/activation.cpp:45-60): std::max(0.0f, x).
__global__ void relu_kernel(int64_t n, const float* __restrict__ x, float* __restrict__ y) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = x[i];
        y[i] = (0.0f < v) ? v : 0.0f;
    }
}

namespace {
int blocks_for(pfrt_ctx* ctx, int64_t n) {
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), ctx->num_sms * 16)));
}
}  // namespace

}  // namespace pfrt

using namespace pfrt;

extern "C" {

pfrt_status pfrt_quantize_f32(pfrt_ctx* ctx, int64_t n, const float* x, float scale, int32_t zp,
                              int out_is_u8, void* q, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (n < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "quantize: negative size");
    if (!(scale > 0.0f) || !std::isfinite(scale))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "quantize_tensor: invalid scale " + std::to_string(scale));
    if (n == 0) return PFRT_OK;
    if (!x || !q) return fail(PFRT_ERR_INVALID_ARGUMENT, "quantize: null pointer");
    quantize_kernel<<<blocks_for(ctx, n), 256, 0, pick_stream(ctx, stream)>>>(
        n, x, 1.0f / scale, zp, out_is_u8, static_cast<uint8_t*>(q));
    PFRT_CHECK_LAUNCH("quantize_kernel");
    return PFRT_OK;
}

pfrt_status pfrt_add_rowvec_f32(pfrt_ctx* ctx, int64_t rows, int64_t cols, const float* x,
                                const float* b, float* y, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (rows < 0 || cols < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "Add: negative size");
    if (rows == 0 || cols == 0) return PFRT_OK;
    if (!x || !b || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "Add: null pointer");
    add_rowvec_kernel<<<blocks_for(ctx, rows * cols), 256, 0, pick_stream(ctx, stream)>>>(rows, cols, x, b, y);
    PFRT_CHECK_LAUNCH("add_rowvec_kernel");
    return PFRT_OK;
}

pfrt_status pfrt_relu_f32(pfrt_ctx* ctx, int64_t n, const float* x, float* y, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (n < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "Relu: negative size");
    if (n == 0) return PFRT_OK;
    if (!x || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "Relu: null pointer");
    relu_kernel<<<blocks_for(ctx, n), 256, 0, pick_stream(ctx, stream)>>>(n, x, y);
    PFRT_CHECK_LAUNCH("relu_kernel");
    return PFRT_OK;
}

}  // extern "C"
