// qgemm.cu -- quantized (uint8/int8 x int8) linear layer on tcgen05 kind::i8.
//
// Replaces quantization::quantized_matmul + quantize_tensor
// (src/quantization/quant_ops.cpp:387-506, 15-127) with per-output-channel
// weight scales and the Add(bias)/Relu tail fused into the epilogue.
//
// Weight preparation (once per initializer): the reference stores the weight
// as B [K,N] row-major; the tensor cores want it K-major, so it is transposed
// to Wt [N, Kpad] (Kpad = K rounded up to 16 bytes, zero padded) and its
// column sums colsum[n] = sum_k W[k,n] are kept for the zero-point
// correction of the activations.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <string>
#include <vector>

#include "epilogues.cuh"
#include "internal.hpp"
#include "umma_gemm.cuh"
#include "umma_gemm2.cuh"
#include "umma_gemm_sk.cuh"

struct pfrt_qweight {
    pfrt_ctx* ctx = nullptr;
    int64_t K = 0, N = 0, Kpad = 0, Npad = 0;
    int32_t w_zp = 0;
    int8_t* wt = nullptr;        // [N, Kpad]
    int32_t* colsum = nullptr;   // [Npad]
    float* w_scale = nullptr;    // [Npad]
    CUtensorMap tm_b128{};       // box [128 rows, 128 bytes]
    CUtensorMap tm_b256{};       // box [256 rows, 128 bytes]
    CUtensorMap tm_b64{};        // box [64 rows, 128 bytes] (the pair kernel's B half at BN = 128)
};

namespace pfrt {

// Wt[n, k] = W[k, n] for k < K, zero for K <= k < Kpad.  32x32 tiles through
// shared memory so that both the read of W and the write of Wt are coalesced.
__global__ void q_transpose_kernel(const int8_t* __restrict__ w, int64_t K, int64_t N,
                                   int8_t* __restrict__ wt, int64_t Kpad) {
    __shared__ int8_t tile[32][33];
    const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t k = k0 + i, n = n0 + threadIdx.x;
        tile[i][threadIdx.x] = (k < K && n < N) ? w[k * N + n] : int8_t(0);
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t n = n0 + i, k = k0 + threadIdx.x;
        if (n < N && k < Kpad) wt[n * Kpad + k] = tile[threadIdx.x][i];
    }
}

// colsum[n] = sum_k Wt[n, k]; one warp per row of Wt.  Rows n >= N are zero.
__global__ void q_colsum_kernel(const int8_t* __restrict__ wt, int64_t N, int64_t Kpad, int64_t Npad,
                                int32_t* __restrict__ colsum) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (n >= Npad) return;
    int32_t s = 0;
    if (n < N)
        for (int64_t k = lane; k < Kpad; k += 32) s += wt[n * Kpad + k];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) colsum[n] = s;
}

// rowsum[m] = sum_k A[m, k] (uint8 or int8), needed only when w_zp != 0.
__global__ void q_rowsum_kernel(const uint8_t* __restrict__ a, int64_t M, int64_t K, int64_t lda,
                                int a_is_u8, int32_t* __restrict__ rowsum) {
    const int64_t m = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (m >= M) return;
    int32_t s = 0;
    for (int64_t k = lane; k < K; k += 32) {
        const uint8_t v = a[m * lda + k];
        s += a_is_u8 ? static_cast<int32_t>(v) : static_cast<int32_t>(static_cast<int8_t>(v));
    }
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) rowsum[m] = s;
}

// Copies A [M, K] (row stride lda) into a 16-byte aligned [M, Kpad] buffer,
// zero padding columns K..Kpad.
__global__ void q_pad_rows_kernel(const uint8_t* __restrict__ a, int64_t M, int64_t K, int64_t lda,
                                  uint8_t* __restrict__ out, int64_t Kpad) {
    const int64_t total = M * Kpad;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t m = i / Kpad, k = i % Kpad;
        out[i] = (k < K) ? a[m * lda + k] : uint8_t(0);
    }
}

// Thread per (row, 4 columns): partial sums added in split order (exact in
// int64), then the single-pass epilogue's finalisation.
__global__ void q_splitk_reduce_kernel(const QEpi e, int splits) {
    const int quads = (e.N + 3) / 4;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(e.M) * quads) return;
    const int row = static_cast<int>(idx / quads);
    const int col0 = static_cast<int>(idx % quads) * 4;
    const int32_t rs = (e.w_zp != 0) ? e.rowsum[row] : 0;
    int64_t raw[4] = {0, 0, 0, 0};
    const bool vec = (e.N % 4) == 0;
    for (int s = 0; s < splits; ++s) {
        const int32_t* p = e.partial + (static_cast<int64_t>(s) * e.M + row) * e.N + col0;
        if (vec) {
            const int4 v = *reinterpret_cast<const int4*>(p);
            raw[0] += v.x; raw[1] += v.y; raw[2] += v.z; raw[3] += v.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (col0 + j < e.N) raw[j] += p[j];
        }
    }
    int32_t at[4];
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) y[j] = e.finalize(row, col0 + j, raw[j], rs, at[j]);
    e.emit<4>(row, col0, at, y);
}

namespace {

int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

// tmB: B with a BN-row box; tmBn: B with a BN/2-row box, for the half-width
// units of a narrow tail (passed in the kernel's second-part B slot, which
// the int8 kernel does not otherwise use).
template <int BN, int STAGES>
pfrt_status launch_q(pfrt_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmBn,
                     const GemmSched& s, const QEpi& e, cudaStream_t st) {
    using Cfg = GemmCfg<KIND_I8, BN, STAGES>;
    auto kern = umma_gemm_kernel<KIND_I8, BN, STAGES, QEpi>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg::SMEM_BYTES));
    const int grid = std::min(s.num_units, ctx->num_sms);
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = st;
    cfg.numAttrs = pdl_attr(attr);
    cfg.attrs = attr;
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmA, tmBn, s, e, ctx->d_err));
    return PFRT_OK;
}

// The CTA-pair kernel (umma_gemm2.cuh): clusters of two, as many clusters as
// can be resident at once, each looping over 256 x BN pair tiles.
template <int BN, int STAGES>
pfrt_status launch_q2(pfrt_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmBh, const GemmSched& s,
                      const QEpi& e, cudaStream_t st) {
    using Cfg = Gemm2Cfg<BN, STAGES>;
    auto kern = umma_gemm2_kernel<BN, STAGES, QEpi>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(ctx->num_sms & ~1));
    int clusters = 0;
    PFRT_CUDA_TRY(cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg));
    if (clusters < 1) return fail(PFRT_ERR_UNSUPPORTED, "int8 GEMM: no CTA pair fits on this device");
    const int pairs = std::min(s.num_units, clusters);
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.numAttrs = 1 + pdl_attr(attr + 1);
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmA, tmBh, s, e, ctx->d_err));
    return PFRT_OK;
}

// The split-K cluster kernel (umma_gemm_sk.cuh): one 128 x BN tile per
// cluster of two CTAs, each taking about half of K (tmBh: the weight's map
// with a BN/2-row box; tail: the k-blocks in which each CTA accumulates only
// its own half of the columns, umma_gemm_sk.cuh).
template <int BN, int STAGES>
pfrt_status launch_qsk2(pfrt_ctx* ctx, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmBh,
                        const GemmSched& s, int tail, const QEpi& e, uint4* xchg, cudaStream_t st) {
    using Cfg = GemmSkCfg<BN, STAGES>;
    auto kern = umma_gemm_sk2_kernel<BN, STAGES, QEpi>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * s.num_units));
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1 + pdl_attr(attr + 1);
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmBh, s, tail, e, xchg, ctx->d_err));
    return PFRT_OK;
}

}  // namespace
}  // namespace pfrt

using namespace pfrt;

extern "C" {

pfrt_status pfrt_qweight_create(pfrt_ctx* ctx, int64_t K, int64_t N, const int8_t* w_host,
                                int32_t w_zp, const float* w_scale_host, int64_t n_scales,
                                pfrt_qweight** out) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!out || !w_host || !w_scale_host)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qweight_create: null argument");
    *out = nullptr;
    if (K <= 0 || N <= 0)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qweight_create: K and N must be positive");
    if (K > 65536)
        return fail(PFRT_ERR_UNSUPPORTED,
                    "pfrt_qweight_create: K > 65536 could overflow the s32 tensor-core accumulator");
    if (n_scales != 1 && n_scales != N)
        return fail(PFRT_ERR_INVALID_ARGUMENT,
                    "pfrt_qweight_create: need 1 or N weight scales (quantize_tensor: scale count mismatch)");
    for (int64_t i = 0; i < n_scales; ++i)
        if (!(w_scale_host[i] > 0.0f) || !std::isfinite(w_scale_host[i]))
            return fail(PFRT_ERR_INVALID_ARGUMENT,
                        "pfrt_qweight_create: weight scale " + std::to_string(i) +
                            " must be positive and finite");

    auto* w = new pfrt_qweight();
    w->ctx = ctx;
    w->K = K;
    w->N = N;
    w->Kpad = static_cast<int64_t>(align_up(K, 16));
    w->Npad = static_cast<int64_t>(align_up(N, 256));
    w->w_zp = w_zp;
    int8_t* staging = nullptr;
    std::vector<float> scales(static_cast<size_t>(w->Npad), 0.0f);
    for (int64_t n = 0; n < N; ++n) scales[n] = w_scale_host[n_scales == 1 ? 0 : n];

    auto cleanup = [&](pfrt_status s) {
        if (staging) cudaFree(staging);
        if (s != PFRT_OK) pfrt_qweight_destroy(w);
        return s;
    };
    cudaError_t e = cudaMalloc(&w->wt, static_cast<size_t>(N * w->Kpad));
    if (e == cudaSuccess) e = cudaMalloc(&w->colsum, sizeof(int32_t) * w->Npad);
    if (e == cudaSuccess) e = cudaMalloc(&w->w_scale, sizeof(float) * w->Npad);
    if (e == cudaSuccess) e = cudaMalloc(&staging, static_cast<size_t>(K * N));
    // On the context stream, ordered before the kernels below (a pageable
    // cudaMemcpy may return before its DMA lands, and the context stream does
    // not wait for the legacy stream); the stream is synchronized below.
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(staging, w_host, static_cast<size_t>(K * N), cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(w->w_scale, scales.data(), sizeof(float) * w->Npad, cudaMemcpyHostToDevice,
                            ctx->stream);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "pfrt_qweight_create"));

    dim3 tb(32, 8);
    dim3 tg(static_cast<unsigned>(ceil_div(N, 32)), static_cast<unsigned>(ceil_div(w->Kpad, 32)));
    q_transpose_kernel<<<tg, tb, 0, ctx->stream>>>(staging, K, N, w->wt, w->Kpad);
    q_colsum_kernel<<<static_cast<unsigned>(ceil_div(w->Npad, 8)), 256, 0, ctx->stream>>>(
        w->wt, N, w->Kpad, w->Npad, w->colsum);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "pfrt_qweight_create kernels"));

    st = make_tmap_2d(&w->tm_b128, w->wt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->Kpad, N, w->Kpad,
                      128, 128);
    if (st == PFRT_OK)
        st = make_tmap_2d(&w->tm_b256, w->wt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->Kpad, N,
                          w->Kpad, 128, 256);
    if (st == PFRT_OK)
        st = make_tmap_2d(&w->tm_b64, w->wt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w->Kpad, N, w->Kpad,
                          128, 64);
    if (st != PFRT_OK) return cleanup(st);
    *out = w;
    return cleanup(PFRT_OK);
}

pfrt_status pfrt_qweight_destroy(pfrt_qweight* w) {
    if (!w) return PFRT_OK;
    if (w->ctx) cudaSetDevice(w->ctx->device);
    if (w->wt) cudaFree(w->wt);
    if (w->colsum) cudaFree(w->colsum);
    if (w->w_scale) cudaFree(w->w_scale);
    delete w;
    return PFRT_OK;
}

pfrt_status pfrt_qlinear(pfrt_ctx* ctx, const pfrt_qweight* w, int64_t M, const void* a,
                         int64_t lda, int a_is_u8, float a_scale, int32_t a_zp,
                         const float* bias, int relu, int out_mode, float y_scale, int32_t y_zp,
                         void* y, int64_t ldy, int32_t* acc_out, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!w) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: null weight");
    if (w->ctx != ctx) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: weight belongs to another context");
    if (M < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: negative M");
    if (M == 0) return PFRT_OK;
    if (M > (int64_t{1} << 31) - 256)
        return fail(PFRT_ERR_UNSUPPORTED, "pfrt_qlinear: M too large");
    if (!a || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: null input or output");
    if (lda < w->K) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: lda < K");
    if (ldy < w->N) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: ldy < N");
    if (out_mode < PFRT_OUT_F32 || out_mode > PFRT_OUT_U8)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: bad out_mode");
    if (!(a_scale > 0.0f) || !std::isfinite(a_scale))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: a_scale must be positive and finite");
    if (out_mode != PFRT_OUT_F32 && (!(y_scale > 0.0f) || !std::isfinite(y_scale)))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "quantize_tensor: invalid scale " + std::to_string(y_scale));
    cudaStream_t s = pick_stream(ctx, stream);
    const int64_t K = w->K, N = w->N;

    // Scratch layout: [padded A][rowsum][split-K partials]
    const bool need_pad = (lda % 16 != 0) || (reinterpret_cast<uintptr_t>(a) & 15u) != 0;
    const size_t pad_bytes = need_pad ? align_up(static_cast<size_t>(M * w->Kpad), 256) : 0;
    const size_t rs_bytes = (w->w_zp != 0) ? align_up(sizeof(int32_t) * M, 256) : 0;

    // Tile shape and split-K.
    const int64_t mblk = ceil_div(M, 128);
    const int64_t t256 = mblk * ceil_div(N, 256), t128 = mblk * ceil_div(N, 128);
    // Tile width from the waves each choice takes on the persistent grid,
    // in units of one 128x256 tile's time; a 128x128 tile costs ~0.7 of that
    // (measured on B200: per MAC it moves more bytes from L2).  With 256-wide
    // tiles, a last wave that fills at most half the SMs runs as 128-wide
    // halves (the narrow tail of umma_gemm_kernel).
    const int64_t G = ctx->num_sms;
    const int64_t wfull = t256 / G, rem = t256 % G;
    const bool tail_narrow = rem > 0 && 2 * rem <= G;
    const double cost256 = static_cast<double>(wfull) + (rem == 0 ? 0.0 : (tail_narrow ? 0.7 : 1.0));
    const double cost128 = 0.7 * static_cast<double>(ceil_div(t128, G));
    int bn = (cost256 < cost128) ? 256 : 128;
    bn = env_int("PFRT_QGEMM_BN", bn);
    if (bn != 128 && bn != 256) bn = 128;
    const int64_t tiles = (bn == 256) ? t256 : t128;
    const int kb_total = static_cast<int>(ceil_div(w->Kpad, 128));
    (void)tiles;
    // Split-K (partial accumulators + a reduction pass) is available but off
    // by default: measured slower than one pass at every benchmark shape.
    int splits = env_int("PFRT_QGEMM_SPLITS", 1);
    splits = std::max(1, std::min(splits, kb_total));
    const int kb_per = static_cast<int>(ceil_div(kb_total, splits));
    splits = static_cast<int>(ceil_div(kb_total, kb_per));
    const size_t part_bytes = (splits > 1) ? align_up(sizeof(int32_t) * splits * M * N, 256) : 0;
    // K split over CTA pairs (umma_gemm_sk.cuh): 128 x 256 tiles, one per
    // cluster of two CTAs, where those clusters fit on the GPU at once.  It
    // pulls a quarter fewer bytes through L2 per SM than 128 x 128 tiles but
    // pays ~2 us more per call for the exchange of partial sums, so it is
    // chosen from 28 k-blocks (K >= 3457) on (measured on B200 at M = 512,
    // N = 4096: 4.7 % faster at K = 4096, 2 % slower at K = 3072, 24 % faster
    // at K = 16384).  PFRT_QGEMM_SK2 = 0|1 overrides.
    const int64_t tiles256 = mblk * ceil_div(N, 256);
    const bool sk2_fits = splits == 1 && kb_total >= 2 && 2 * tiles256 <= G;
    const int sk2_env = env_int("PFRT_QGEMM_SK2", -1);
    // An explicit tile width or pair choice (PFRT_QGEMM_BN / _PAIR) selects
    // those kernels instead.
    const bool forced = env_int("PFRT_QGEMM_BN", 0) != 0 || env_int("PFRT_QGEMM_PAIR", -1) >= 0;
    const bool use_sk2 = sk2_fits && (sk2_env >= 0 ? sk2_env != 0 : (kb_total >= 28 && !forced));
    const size_t xchg_bytes = use_sk2 ? align_up(gemm_sk_xchg_bytes<256>(tiles256), 256) : 0;

    void* scr = nullptr;
    st = scratch(ctx, pad_bytes + rs_bytes + part_bytes + xchg_bytes, &scr);
    if (st) return st;
    uint8_t* base = static_cast<uint8_t*>(scr);
    const uint8_t* a_use = static_cast<const uint8_t*>(a);
    int64_t lda_use = lda;
    if (need_pad) {
        uint8_t* ap = base;
        const int64_t total = M * w->Kpad;
        const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(total, 256), 4096));
        q_pad_rows_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint8_t*>(a), M, K, lda, ap, w->Kpad);
        PFRT_CHECK_LAUNCH("q_pad_rows_kernel");
        a_use = ap;
        lda_use = w->Kpad;
    }
    int32_t* rowsum = nullptr;
    if (rs_bytes) {
        rowsum = reinterpret_cast<int32_t*>(base + pad_bytes);
        q_rowsum_kernel<<<static_cast<unsigned>(ceil_div(M, 8)), 256, 0, s>>>(a_use, M, K, lda_use, a_is_u8,
                                                                            rowsum);
        PFRT_CHECK_LAUNCH("q_rowsum_kernel");
    }

    CUtensorMap tmA;
    st = make_tmap_2d(&tmA, a_use, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, static_cast<uint64_t>(w->Kpad),
                      static_cast<uint64_t>(M), static_cast<uint64_t>(lda_use), 128, 128);
    if (st) return st;

    QEpi e{};
    e.idesc = idesc_make(2, a_is_u8 ? 0u : 1u, 1u, 128, static_cast<uint32_t>(bn));
    e.M = static_cast<int>(M);
    e.N = static_cast<int>(N);
    e.K = static_cast<int>(K);
    e.a_zp = a_zp;
    e.w_zp = w->w_zp;
    e.a_scale = a_scale;
    e.colsum = w->colsum;
    e.rowsum = rowsum;
    e.w_scale = w->w_scale;
    e.bias = bias;
    e.relu = relu ? 1 : 0;
    e.out_mode = out_mode;
    e.inv_y_scale = (out_mode == PFRT_OUT_F32) ? 1.0f : 1.0f / y_scale;  // quant_ops.cpp:41
    e.y_zp = y_zp;
    e.out = y;
    e.ldo = ldy;
    e.acc_out = acc_out;
    const int esz = (out_mode == PFRT_OUT_F32) ? 4 : 1;
    e.vec_ok = ((reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (ldy * esz) % 16 == 0) ? 1 : 0;
    e.acc_vec_ok = ((reinterpret_cast<uintptr_t>(acc_out) & 15u) == 0 && (N % 4) == 0) ? 1 : 0;
    {
        // Largest magnitude any intermediate of raw - a_zp*colsum - w_zp*rowsum
        // + K*a_zp*w_zp can reach; below 2^31 the epilogue runs in int32.
        const double k = static_cast<double>(K);
        const double bound = k * 255.0 * 128.0 + std::fabs(static_cast<double>(a_zp)) * k * 128.0 +
                             std::fabs(static_cast<double>(w->w_zp)) * k * 255.0 +
                             k * std::fabs(static_cast<double>(a_zp) * w->w_zp);
        e.fast32 = (bound < 2147483647.0) ? 1 : 0;
    }

    GemmSched sched{};
    sched.num_m_blk = static_cast<int>(mblk);
    sched.num_n_blk = static_cast<int>(ceil_div(N, bn));
    sched.splits = splits;
    sched.kb_total = kb_total;
    sched.kb_per_split = kb_per;
    sched.num_units = sched.num_m_blk * sched.num_n_blk * splits;
    sched.wide_units = sched.num_units;
    if (bn == 256 && splits == 1 && tail_narrow && env_int("PFRT_QGEMM_NARROW", 1) != 0) {
        sched.wide_units = static_cast<int>(wfull * G);
        sched.num_units = sched.wide_units + static_cast<int>(2 * rem);
    }

    QEpi eg = e;
    if (splits > 1) {
        eg.out_mode = kOutPartial;
        eg.partial = reinterpret_cast<int32_t*>(base + pad_bytes + rs_bytes);
        eg.acc_out = nullptr;
        e.partial = eg.partial;
    }
    if (use_sk2) {
        GemmSched ks2 = sched;
        ks2.num_n_blk = static_cast<int>(ceil_div(N, 256));
        ks2.num_units = static_cast<int>(tiles256);
        ks2.wide_units = ks2.num_units;
        ks2.kb_per_split = kb_total;
        QEpi ek = eg;
        ek.idesc = idesc_make(2, a_is_u8 ? 0u : 1u, 1u, 128, 256);
        // Early exchange: each CTA's last `tail` k-blocks cover only its own
        // half of the columns, so the peer's half is exchanged while they run
        // (umma_gemm_sk.cuh).  PFRT_QGEMM_SK2_TAIL overrides.
        int tail = env_int("PFRT_QGEMM_SK2_TAIL", kb_total / 8);
        tail = std::max(0, std::min(tail, kb_total - 2));
        st = launch_qsk2<256, 4>(ctx, tmA, w->tm_b256, w->tm_b128, ks2, tail, ek,
                                 reinterpret_cast<uint4*>(base + pad_bytes + rs_bytes + part_bytes), s);
        if (st) return st;
        PFRT_CHECK_LAUNCH("umma_gemm_sk2_kernel<i8>");
        return PFRT_OK;
    }
    // CTA pairs (256-row tiles over two SMs) where the tile width is 256:
    // measured 5-7 % faster than one CTA per tile at M = 1024..8192, N = K =
    // 4096, and no faster at 128-wide tiles (config 2).
    const bool pair = env_int("PFRT_QGEMM_PAIR", bn == 256 ? 1 : 0) != 0 && splits == 1;
    if (pair) {
        // 256-row pair tiles; the MMA instruction carries M = 256.
        GemmSched ps = sched;
        ps.num_m_blk = static_cast<int>(ceil_div(M, 256));
        ps.num_units = ps.num_m_blk * sched.num_n_blk;
        ps.wide_units = ps.num_units;
        QEpi ep = eg;
        ep.idesc = idesc_make(2, a_is_u8 ? 0u : 1u, 1u, 256, static_cast<uint32_t>(bn));
        st = (bn == 256) ? launch_q2<256, 6>(ctx, tmA, w->tm_b128, ps, ep, s)
                         : launch_q2<128, 8>(ctx, tmA, w->tm_b64, ps, ep, s);
        if (st) return st;
        PFRT_CHECK_LAUNCH("umma_gemm2_kernel<i8>");
        return PFRT_OK;
    }
    st = (bn == 256) ? launch_q<256, 4>(ctx, tmA, w->tm_b256, w->tm_b128, sched, eg, s)
                     : launch_q<128, 6>(ctx, tmA, w->tm_b128, w->tm_b128, sched, eg, s);
    if (st) return st;
    if (splits > 1) {
        const int64_t threads = M * ceil_div(N, 4);
        q_splitk_reduce_kernel<<<static_cast<unsigned>(ceil_div(threads, 256)), 256, 0, s>>>(e, splits);
        PFRT_CHECK_LAUNCH("q_splitk_reduce_kernel");
    }
    return PFRT_OK;
}

pfrt_status pfrt_qlinear_host(pfrt_ctx* ctx, const pfrt_qweight* w, int64_t M, const void* a_host, int64_t lda,
                              int a_is_u8, float a_scale, int32_t a_zp, const float* bias, int relu, int out_mode,
                              float y_scale, int32_t y_zp, void* y_host, int64_t ldy, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!w) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear_host: null weight");
    if (M < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear: negative M");
    if (M == 0) return PFRT_OK;
    if (!a_host || !y_host) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear_host: null input or output");
    if (lda < w->K || ldy < w->N) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear_host: row stride too small");
    if (out_mode != PFRT_OUT_F32 && out_mode != PFRT_OUT_S8 && out_mode != PFRT_OUT_U8)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_qlinear_host: bad output mode");
    const size_t esz = (out_mode == PFRT_OUT_F32) ? 4 : 1;
    // Dense device copies (row stride K and N); the host rows keep their strides.
    const size_t a_bytes = align_up(static_cast<size_t>(M) * w->K, 256);
    const size_t y_bytes = static_cast<size_t>(M) * w->N * esz;
    void* io = nullptr;
    st = io_buffer(ctx, a_bytes + y_bytes, &io);
    if (st) return st;
    uint8_t* a_dev = static_cast<uint8_t*>(io);
    uint8_t* y_dev = a_dev + a_bytes;
    cudaStream_t s = pick_stream(ctx, stream);
    // One linear copy for contiguous rows (a pitched copy moves row by row).
    if (lda == w->K)
        PFRT_CUDA_TRY(cudaMemcpyAsync(a_dev, a_host, static_cast<size_t>(M) * w->K, cudaMemcpyHostToDevice, s));
    else
        PFRT_CUDA_TRY(cudaMemcpy2DAsync(a_dev, w->K, a_host, lda, w->K, M, cudaMemcpyHostToDevice, s));
    st = pfrt_qlinear(ctx, w, M, a_dev, w->K, a_is_u8, a_scale, a_zp, bias, relu, out_mode, y_scale, y_zp, y_dev,
                      w->N, nullptr, stream);
    if (st) return st;
    if (ldy == w->N)
        PFRT_CUDA_TRY(cudaMemcpyAsync(y_host, y_dev, y_bytes, cudaMemcpyDeviceToHost, s));
    else
        PFRT_CUDA_TRY(
            cudaMemcpy2DAsync(y_host, ldy * esz, y_dev, w->N * esz, w->N * esz, M, cudaMemcpyDeviceToHost, s));
    return PFRT_OK;
}

}  // extern "C"
