// gemm_f32.cu -- fp32 Gemm / MatMul on tcgen05 kind::tf32 with the 3xTF32
// split.
//
// Replaces cpu_gemm (src/backends/cpu/ops/math.cpp:377-438) and the 2-D path
// of cpu_matmul (:326-336).  Each fp32 operand x is split once into
// hi = tf32(x) (round to nearest) and lo = x - hi (exact in fp32); the tensor
// cores accumulate lo_a*hi_b + hi_a*lo_b + hi_a*hi_b in fp32, which recovers
// close to fp32 accuracy (the dropped lo*lo term is ~2^-22 relative).
//
// The split writes both parts K-major ([rows, Kpad], Kpad = K rounded up to
// 32 and zero padded), whatever the transA/transB of the input, so one GEMM
// kernel serves all four transpose combinations.  A constant B (a graph
// initializer) is split once by pfrt_fweight_create.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>

#include "epilogues.cuh"
#include "internal.hpp"
#include "umma_gemm.cuh"

struct pfrt_fweight {
    pfrt_ctx* ctx = nullptr;
    int64_t K = 0, N = 0, Kpad = 0;
    float* hi = nullptr;  // [N, Kpad]
    float* lo = nullptr;  // [N, Kpad]
    CUtensorMap tm_hi{}, tm_lo{};
};

namespace pfrt {

constexpr int kF32BN = 128;
constexpr int kF32Stages = 3;

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
    hi = __uint_as_float(h);
    lo = __fsub_rn(x, hi);
}

constexpr int kSplitRows = 8;  // blockDim.y of split_kmajor_kernel

// out_{hi,lo}[r, k] = split(src(r, k)) for k < K, 0 for K <= k < Kpad, where
// src(r, k) = src[r*ld + k] (trans = 0) or src[k*ld + r] (trans = 1).
// 32x32 tiles through shared memory keep both sides coalesced for trans = 1.
// Launched with programmatic stream serialization: it waits for the previous
// kernel (which may write src or still read hi/lo) before any access, and
// lets the GEMM that follows start its set-up at once.
__global__ void split_kmajor_kernel(const float* __restrict__ src, int64_t rows, int64_t K,
                                    int64_t ld, int trans, float* __restrict__ hi,
                                    float* __restrict__ lo, int64_t Kpad) {
    pdl_wait();
    pdl_launch_dependents();
    // Block (32, kSplitRows): each thread's 32 / kSplitRows loads are issued
    // together before any is used.
    constexpr int RPT = 32 / kSplitRows;
    __shared__ float tile[32][33];
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    if (trans) {
        float x[RPT];
#pragma unroll
        for (int t = 0; t < RPT; ++t) {
            const int i = threadIdx.y + kSplitRows * t;
            const int64_t k = k0 + i, r = r0 + threadIdx.x;
            x[t] = (k < K && r < rows) ? src[k * ld + r] : 0.0f;
        }
#pragma unroll
        for (int t = 0; t < RPT; ++t) tile[threadIdx.y + kSplitRows * t][threadIdx.x] = x[t];
        __syncthreads();
#pragma unroll
        for (int t = 0; t < RPT; ++t) {
            const int i = threadIdx.y + kSplitRows * t;
            const int64_t r = r0 + i, k = k0 + threadIdx.x;
            if (r < rows && k < Kpad) {
                float h, l;
                split_tf32(tile[threadIdx.x][i], h, l);
                hi[r * Kpad + k] = h;
                lo[r * Kpad + k] = l;
            }
        }
    } else {
        float x[RPT];
#pragma unroll
        for (int t = 0; t < RPT; ++t) {
            const int64_t r = r0 + threadIdx.y + kSplitRows * t, k = k0 + threadIdx.x;
            x[t] = (r < rows && k < K) ? src[r * ld + k] : 0.0f;
        }
#pragma unroll
        for (int t = 0; t < RPT; ++t) {
            const int64_t r = r0 + threadIdx.y + kSplitRows * t, k = k0 + threadIdx.x;
            if (r < rows && k < Kpad) {
                float h, l;
                split_tf32(x[t], h, l);
                hi[r * Kpad + k] = h;
                lo[r * Kpad + k] = l;
            }
        }
    }
}

// Thread per (row, 4 columns): partials added in split order (IEEE fp32),
// then alpha/beta/C as in the single-pass epilogue.  splits = 0 gives the
// empty-K result beta*C.  Launched with programmatic stream serialization:
// nothing is read before the GEMM that wrote the partials has completed.
__global__ void f_splitk_reduce_kernel(const FEpi e, int splits) {
    pdl_wait();
    pdl_launch_dependents();
    const int quads = (e.N + 3) / 4;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(e.M) * quads) return;
    const int row = static_cast<int>(idx / quads);
    const int col0 = static_cast<int>(idx % quads) * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const bool vec = (e.N % 4) == 0;
    const int64_t plane = static_cast<int64_t>(e.M) * e.N;
    const float* base = e.partial + static_cast<int64_t>(row) * e.N + col0;
    if (vec) {
        // Up to eight partials' loads in flight at once, then added in split
        // order (the sum does not depend on how the loads are grouped).
        constexpr int U = 8;
        for (int k0 = 0; k0 < splits; k0 += U) {
            float4 v[U];
#pragma unroll
            for (int j = 0; j < U; ++j)
                if (k0 + j < splits) v[j] = *reinterpret_cast<const float4*>(base + (k0 + j) * plane);
#pragma unroll
            for (int j = 0; j < U; ++j) {
                if (k0 + j < splits) {
                    acc[0] = __fadd_rn(acc[0], v[j].x);
                    acc[1] = __fadd_rn(acc[1], v[j].y);
                    acc[2] = __fadd_rn(acc[2], v[j].z);
                    acc[3] = __fadd_rn(acc[3], v[j].w);
                }
            }
        }
    } else {
        for (int k = 0; k < splits; ++k) {
            const float* p = base + k * plane;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (col0 + j < e.N) acc[j] = __fadd_rn(acc[j], p[j]);
        }
    }
    e.store_direct<4>(row, col0, acc);
}

namespace {

int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

int default_splits(const pfrt_ctx* ctx, int64_t tiles, int kb_total) {
    if (tiles * 2 > ctx->num_sms || kb_total < 16) return 1;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({8, ctx->num_sms / tiles, kb_total / 4})));
}

pfrt_status launch_split(const float* src, int64_t rows, int64_t K, int64_t ld, int trans,
                         float* hi, float* lo, int64_t Kpad, cudaStream_t s) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(32, kSplitRows);
    cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(Kpad, 32)), static_cast<unsigned>(ceil_div(rows, 32)));
    cfg.stream = s;
    cfg.numAttrs = pdl_attr(attr);
    cfg.attrs = attr;
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, split_kmajor_kernel, src, rows, K, ld, trans, hi, lo, Kpad));
    return PFRT_OK;
}

// Runs the GEMM on prepared K-major hi/lo operands.
pfrt_status run_f32(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t Kpad, const CUtensorMap& tmAh,
                    const CUtensorMap& tmAl, const CUtensorMap& tmBh, const CUtensorMap& tmBl,
                    float alpha, float beta, const float* c, int64_t c_len, float* y, int64_t ldy,
                    void* scratch_tail, size_t tail_bytes, cudaStream_t s, int max_splits = 1 << 20,
                    float* const* peer_y = nullptr, int n_peer_y = 0) {
    using Cfg = GemmCfg<KIND_TF32X3, kF32BN, kF32Stages>;
    const int64_t mblk = ceil_div(M, 128), nblk = ceil_div(N, kF32BN);
    const int64_t tiles = mblk * nblk;
    const int kb_total = static_cast<int>(ceil_div(Kpad, Cfg::BK));
    // Split K when the tiles alone would leave most SMs idle (config 1: 16
    // tiles on 148 SMs ran in 28 us unsplit, 14.7 us with 8 splits).
    int splits = default_splits(ctx, tiles, kb_total);
    splits = env_int("PFRT_GEMM_SPLITS", splits);
    splits = std::max(1, std::min({splits, kb_total, max_splits}));
    const int kb_per = static_cast<int>(ceil_div(kb_total, splits));
    splits = static_cast<int>(ceil_div(kb_total, kb_per));
    if (splits > 1 && sizeof(float) * splits * M * N > tail_bytes)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "internal: split-K scratch too small");

    FEpi e{};
    e.M = static_cast<int>(M);
    e.N = static_cast<int>(N);
    e.alpha = alpha;
    e.beta = beta;
    e.C = (c != nullptr && c_len > 0) ? c : nullptr;
    e.c_len = c_len;
    e.out = y;
    e.ldo = ldy;
    e.out_mode = kOutF32;
    e.vec_ok = ((reinterpret_cast<uintptr_t>(y) & 15u) == 0 && (N % 4) == 0 && (ldy % 4) == 0) ? 1 : 0;
    e.n_peer_out = std::min(n_peer_y, kMaxPeerOut);
    for (int i = 0; i < e.n_peer_out; ++i) {
        e.peer_out[i] = peer_y[i];
        if ((reinterpret_cast<uintptr_t>(peer_y[i]) & 15u) != 0) e.vec_ok = 0;
    }
    FEpi eg = e;
    if (splits > 1) {
        eg.out_mode = kOutPartial;
        eg.partial = static_cast<float*>(scratch_tail);
        e.partial = eg.partial;
    }
    GemmSched sched{};
    sched.num_m_blk = static_cast<int>(mblk);
    sched.num_n_blk = static_cast<int>(nblk);
    sched.splits = splits;
    sched.kb_total = kb_total;
    sched.kb_per_split = kb_per;
    sched.num_units = static_cast<int>(mblk * nblk * splits);
    sched.wide_units = sched.num_units;  // no narrow tail on the fp32 path

    auto kern = umma_gemm_kernel<KIND_TF32X3, kF32BN, kF32Stages, FEpi>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Cfg::SMEM_BYTES));
    const int grid = std::min(sched.num_units, ctx->num_sms);
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = s;
    cfg.numAttrs = pdl_attr(attr);
    cfg.attrs = attr;
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmAh, tmBh, tmAl, tmBl, sched, eg, ctx->d_err));
    if (splits > 1) {
        const int64_t threads = M * ceil_div(N, 4);
        cudaLaunchConfig_t rc{};
        cudaLaunchAttribute rattr[1];
        rc.gridDim = dim3(static_cast<unsigned>(ceil_div(threads, 256)));
        rc.blockDim = dim3(256);
        rc.stream = s;
        rc.numAttrs = pdl_attr(rattr);
        rc.attrs = rattr;
        PFRT_CUDA_TRY(cudaLaunchKernelEx(&rc, f_splitk_reduce_kernel, e, splits));
    }
    return PFRT_OK;
}

size_t splitk_bytes(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t Kpad) {
    // Upper bound of the split-K partial buffer run_f32 may ask for.
    const int64_t kb_total = ceil_div(Kpad, 32);
    const int64_t tiles = ceil_div(M, 128) * ceil_div(N, kF32BN);
    int64_t splits = std::max<int64_t>(1, env_int("PFRT_GEMM_SPLITS", default_splits(ctx, tiles, static_cast<int>(kb_total))));
    splits = std::min<int64_t>(splits, kb_total);
    return splits > 1 ? align_up(sizeof(float) * splits * M * N, 256) : 0;
}

pfrt_status check_common(int64_t M, int64_t N, int64_t K, const float* a, float* y) {
    if (M < 0 || N < 0 || K < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: negative dimension");
    if (M > (int64_t{1} << 31) - 256 || N > (int64_t{1} << 31) - 256)
        return fail(PFRT_ERR_UNSUPPORTED, "Gemm: dimension too large");
    if ((M > 0 && N > 0) && (!y || (K > 0 && !a)))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: null input or output");
    return PFRT_OK;
}

// K == 0: the product is empty and Y = beta*C (or 0).  Reuses the reduction
// kernel with zero splits.
pfrt_status run_empty_k(int64_t M, int64_t N, float alpha, float beta, const float* c,
                        int64_t c_len, float* y, cudaStream_t s) {
    FEpi e{};
    e.M = static_cast<int>(M);
    e.N = static_cast<int>(N);
    e.alpha = alpha;
    e.beta = beta;
    e.C = (c != nullptr && c_len > 0) ? c : nullptr;
    e.c_len = c_len;
    e.out = y;
    e.ldo = N;
    e.out_mode = kOutF32;
    e.vec_ok = 0;
    const int64_t threads = M * ceil_div(N, 4);
    f_splitk_reduce_kernel<<<static_cast<unsigned>(ceil_div(threads, 256)), 256, 0, s>>>(e, 0);
    PFRT_CHECK_LAUNCH("f_splitk_reduce_kernel");
    return PFRT_OK;
}

}  // namespace

// Fixed scratch for pfrt_gemm_f32_noalloc: the hi/lo split of A lives here
// instead of in memory allocated at call time.  Every device that loads this
// library holds these 16 MiB until the process exits.  Host code must not use
// the array's name as a device address (on the host it only stands for the
// symbol); noalloc_scratch() looks up the real device address.
constexpr size_t kNoAllocScratchBytes = size_t{16} << 20;
constexpr int64_t kNoAllocMaxElems = static_cast<int64_t>(kNoAllocScratchBytes / (2 * sizeof(float)));
static __device__ __align__(256) unsigned char g_gemm_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};

// Device address of g_gemm_noalloc_scratch on `device`, looked up once per
// device with that device current (the caller has made it current).
pfrt_status noalloc_scratch(int device, void** out) {
    if (device < 0 || device >= kNoAllocMaxDevices)
        return fail(PFRT_ERR_UNSUPPORTED, "pfrt_gemm_f32_noalloc: device ordinal too large");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[device] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return PFRT_OK;
}

}  // namespace

pfrt_status fweight_from_device_split(pfrt_ctx* ctx, int64_t N, int64_t K, float* hi, float* lo,
                                      pfrt_fweight** out) {
    auto* w = new pfrt_fweight();
    w->ctx = ctx;
    w->K = K;
    w->N = N;
    w->Kpad = static_cast<int64_t>(align_up(K, 32));
    w->hi = hi;
    w->lo = lo;
    pfrt_status st = make_tmap_2d(&w->tm_hi, w->hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, w->Kpad, N,
                                  w->Kpad * 4, 32, kF32BN);
    if (st == PFRT_OK)
        st = make_tmap_2d(&w->tm_lo, w->lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, w->Kpad, N,
                          w->Kpad * 4, 32, kF32BN);
    if (st != PFRT_OK) {
        pfrt_fweight_destroy(w);
        return st;
    }
    *out = w;
    return PFRT_OK;
}

pfrt_status split_tf32_kmajor(const float* src, int64_t rows, int64_t K, int64_t ld, float* hi, float* lo,
                              int64_t Kpad, cudaStream_t s) {
    return launch_split(src, rows, K, ld, 0, hi, lo, Kpad, s);
}

pfrt_status gemm_f32_strided(pfrt_ctx* ctx, int64_t M, const float* a, int64_t lda, const pfrt_fweight* b,
                             float* y, int64_t ldy, cudaStream_t s, float* const* peer_y, int n_peer_y) {
    if (n_peer_y > kMaxPeerOut) return fail(PFRT_ERR_UNSUPPORTED, "Gemm: too many output copies");
    const int64_t N = b->N, K = b->K;
    pfrt_status st = check_common(M, N, K, a, y);
    if (st) return st;
    if (M == 0) return PFRT_OK;
    if (lda < K || ldy < N) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: row stride too small");
    const size_t part_bytes = align_up(sizeof(float) * M * b->Kpad, 256);
    const size_t tail = splitk_bytes(ctx, M, N, b->Kpad);
    void* scr = nullptr;
    st = scratch(ctx, 2 * part_bytes + tail, &scr);
    if (st) return st;
    float* ahi = static_cast<float*>(scr);
    float* alo = reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + part_bytes);
    st = launch_split(a, M, K, lda, 0, ahi, alo, b->Kpad, s);
    if (st) return st;
    CUtensorMap tah, tal;
    st = make_tmap_2d(&tah, ahi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, b->Kpad, M, b->Kpad * 4, 32, 128);
    if (st == PFRT_OK)
        st = make_tmap_2d(&tal, alo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, b->Kpad, M, b->Kpad * 4, 32, 128);
    if (st) return st;
    return run_f32(ctx, M, N, b->Kpad, tah, tal, b->tm_hi, b->tm_lo, 1.0f, 0.0f, nullptr, 0, y, ldy,
                   static_cast<uint8_t*>(scr) + 2 * part_bytes, tail, s, 1 << 20, peer_y, n_peer_y);
}

}  // namespace pfrt

using namespace pfrt;

extern "C" {

pfrt_status pfrt_fweight_create(pfrt_ctx* ctx, int64_t K, int64_t N, int trans_b,
                                const float* b_host, pfrt_fweight** out) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!out || !b_host) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_fweight_create: null argument");
    *out = nullptr;
    if (K <= 0 || N <= 0)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_fweight_create: K and N must be positive");
    auto* w = new pfrt_fweight();
    w->ctx = ctx;
    w->K = K;
    w->N = N;
    w->Kpad = static_cast<int64_t>(align_up(K, 32));
    float* staging = nullptr;
    auto cleanup = [&](pfrt_status s) {
        if (staging) cudaFree(staging);
        if (s != PFRT_OK) pfrt_fweight_destroy(w);
        return s;
    };
    const size_t n_el = static_cast<size_t>(N * w->Kpad);
    cudaError_t e = cudaMalloc(&w->hi, sizeof(float) * n_el);
    if (e == cudaSuccess) e = cudaMalloc(&w->lo, sizeof(float) * n_el);
    if (e == cudaSuccess) e = cudaMalloc(&staging, sizeof(float) * K * N);
    // On the context stream, so the split below is ordered after it (a
    // pageable cudaMemcpy may return before its DMA lands, and the context
    // stream does not wait for the legacy stream).
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(staging, b_host, sizeof(float) * K * N, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "pfrt_fweight_create"));
    // B [K,N] (trans_b = 0) is the transposed view of the K-major [N,K] we want.
    st = launch_split(staging, N, K, trans_b ? K : N, trans_b ? 0 : 1, w->hi, w->lo, w->Kpad,
                      ctx->stream);
    if (st) return cleanup(st);
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "pfrt_fweight_create split"));
    st = make_tmap_2d(&w->tm_hi, w->hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, w->Kpad, N,
                      w->Kpad * 4, 32, kF32BN);
    if (st == PFRT_OK)
        st = make_tmap_2d(&w->tm_lo, w->lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, w->Kpad, N,
                          w->Kpad * 4, 32, kF32BN);
    if (st) return cleanup(st);
    *out = w;
    return cleanup(PFRT_OK);
}

pfrt_status pfrt_fweight_destroy(pfrt_fweight* w) {
    if (!w) return PFRT_OK;
    if (w->ctx) cudaSetDevice(w->ctx->device);
    if (w->hi) cudaFree(w->hi);
    if (w->lo) cudaFree(w->lo);
    delete w;
    return PFRT_OK;
}

pfrt_status pfrt_gemm_f32(pfrt_ctx* ctx, int64_t M, int trans_a, float alpha, const float* a,
                          const pfrt_fweight* b, float beta, const float* c, int64_t c_len,
                          float* y, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!b) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: null weight");
    if (b->ctx != ctx) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: weight belongs to another context");
    const int64_t N = b->N, K = b->K;
    st = check_common(M, N, K, a, y);
    if (st) return st;
    if (M == 0) return PFRT_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t part_bytes = align_up(sizeof(float) * M * b->Kpad, 256);
    const size_t tail = splitk_bytes(ctx, M, N, b->Kpad);
    void* scr = nullptr;
    st = scratch(ctx, 2 * part_bytes + tail, &scr);
    if (st) return st;
    float* ahi = static_cast<float*>(scr);
    float* alo = reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + part_bytes);
    st = launch_split(a, M, K, trans_a ? M : K, trans_a, ahi, alo, b->Kpad, s);
    if (st) return st;
    CUtensorMap tah, tal;
    st = make_tmap_2d(&tah, ahi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, b->Kpad, M, b->Kpad * 4, 32, 128);
    if (st == PFRT_OK)
        st = make_tmap_2d(&tal, alo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, b->Kpad, M, b->Kpad * 4, 32, 128);
    if (st) return st;
    return run_f32(ctx, M, N, b->Kpad, tah, tal, b->tm_hi, b->tm_lo, alpha, beta, c, c_len, y, N,
                   static_cast<uint8_t*>(scr) + 2 * part_bytes, tail, s);
}

pfrt_status pfrt_gemm_f32_dense(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t K, int trans_a,
                                int trans_b, float alpha, const float* a, const float* b,
                                float beta, const float* c, int64_t c_len, float* y,
                                pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    st = check_common(M, N, K, a, y);
    if (st) return st;
    if (M == 0 || N == 0) return PFRT_OK;
    cudaStream_t s = pick_stream(ctx, stream);
    if (K == 0) return run_empty_k(M, N, alpha, beta, c, c_len, y, s);
    if (!b) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: null B");
    const int64_t Kpad = static_cast<int64_t>(align_up(K, 32));
    const size_t pa = align_up(sizeof(float) * M * Kpad, 256);
    const size_t pb = align_up(sizeof(float) * N * Kpad, 256);
    const size_t tail = splitk_bytes(ctx, M, N, Kpad);
    void* scr = nullptr;
    st = scratch(ctx, 2 * pa + 2 * pb + tail, &scr);
    if (st) return st;
    uint8_t* base = static_cast<uint8_t*>(scr);
    float* ahi = reinterpret_cast<float*>(base);
    float* alo = reinterpret_cast<float*>(base + pa);
    float* bhi = reinterpret_cast<float*>(base + 2 * pa);
    float* blo = reinterpret_cast<float*>(base + 2 * pa + pb);
    st = launch_split(a, M, K, trans_a ? M : K, trans_a, ahi, alo, Kpad, s);
    if (st) return st;
    st = launch_split(b, N, K, trans_b ? K : N, trans_b ? 0 : 1, bhi, blo, Kpad, s);
    if (st) return st;
    CUtensorMap tah, tal, tbh, tbl;
    st = make_tmap_2d(&tah, ahi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Kpad, M, Kpad * 4, 32, 128);
    if (!st) st = make_tmap_2d(&tal, alo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Kpad, M, Kpad * 4, 32, 128);
    if (!st) st = make_tmap_2d(&tbh, bhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Kpad, N, Kpad * 4, 32, kF32BN);
    if (!st) st = make_tmap_2d(&tbl, blo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, Kpad, N, Kpad * 4, 32, kF32BN);
    if (st) return st;
    return run_f32(ctx, M, N, Kpad, tah, tal, tbh, tbl, alpha, beta, c, c_len, y, N,
                   base + 2 * pa + 2 * pb, tail, s);
}

// The Gemm of pfrt_gemm_f32, for callers that must not allocate device
// memory during a call.  The per-call split of A goes to the fixed 16 MiB
// array above instead of the context's scratch arena, so the call makes no
// cudaMalloc/cudaFree and no other allocation.  Limit: M * Kpad <= 2^21
// elements (Kpad = K rounded up to 32); larger calls are rejected.  The first
// call on a device does a one-time set-up (the lookup of the array's device
// address), so that first call should come before any stream capture.  All
// calls share the array, so calls that overlap on the GPU (other streams,
// other threads) race on it.  K is never split across CTAs here (there is no
// room for split-K partial sums, and PFRT_GEMM_SPLITS is ignored): the result
// agrees with pfrt_gemm_f32 within fp32 tolerance, not bit for bit, and
// shapes whose tiles leave SMs idle run slower than through pfrt_gemm_f32.
pfrt_status pfrt_gemm_f32_noalloc(pfrt_ctx* ctx, int64_t M, int trans_a, float alpha, const float* a,
                                  const pfrt_fweight* b, float beta, const float* c, int64_t c_len,
                                  float* y, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!b) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: null weight");
    if (b->ctx != ctx) return fail(PFRT_ERR_INVALID_ARGUMENT, "Gemm: weight belongs to another context");
    const int64_t N = b->N, K = b->K;
    st = check_common(M, N, K, a, y);
    if (st) return st;
    if (M == 0) return PFRT_OK;
    if (M > kNoAllocMaxElems / b->Kpad)
        return fail(PFRT_ERR_UNSUPPORTED,
                    "pfrt_gemm_f32_noalloc: M * Kpad = " + std::to_string(M) + " * " +
                        std::to_string(b->Kpad) + " exceeds the fixed scratch limit of " +
                        std::to_string(kNoAllocMaxElems) + " elements; use pfrt_gemm_f32");
    void* base = nullptr;
    st = noalloc_scratch(ctx->device, &base);
    if (st) return st;
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t part_bytes = align_up(sizeof(float) * M * b->Kpad, 256);
    float* ahi = static_cast<float*>(base);
    float* alo = reinterpret_cast<float*>(static_cast<uint8_t*>(base) + part_bytes);
    // The split writes every element of [M, Kpad] (zero padding included), so
    // nothing left in the array by an earlier call is read.
    st = launch_split(a, M, K, trans_a ? M : K, trans_a, ahi, alo, b->Kpad, s);
    if (st) return st;
    CUtensorMap tah, tal;
    st = make_tmap_2d(&tah, ahi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, b->Kpad, M, b->Kpad * 4, 32, 128);
    if (st == PFRT_OK)
        st = make_tmap_2d(&tal, alo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, b->Kpad, M, b->Kpad * 4, 32, 128);
    if (st) return st;
    return run_f32(ctx, M, N, b->Kpad, tah, tal, b->tm_hi, b->tm_lo, alpha, beta, c, c_len, y, N,
                   nullptr, 0, s, /*max_splits=*/1);
}

}  // extern "C"
