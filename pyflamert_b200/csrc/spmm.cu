// spmm.cu -- CSR SpMM over pruned weights, Y[M,N] = X[M,K] * W^T with W [N,K]
// in CSR (one CSR row per output channel).
//
// Replaces pruning::sparse_matmul (src/pruning/sparse_tensor.cpp:473-519):
// Y^T = sparse_matmul(W, X^T).  The reference walks each CSR row's nonzeros
// in storage order; here the nonzeros of a row are split across a warp and
// the partial sums are combined with warp shuffles, so the summation order
// differs and results agree to fp32 rounding (normwise relative error).
//
// The path is memory-bound for small M (SpMV-like: 8 bytes of CSR per
// nonzero, reused by nothing), so it is built for HBM streaming: one warp per
// CSR row, 128-bit loads of indices and values (4 nonzeros per lane per load),
// and grid-stride row assignment over a persistent grid.  Two kernels:
//   skinny (M <= 8):  lanes split the row's nonzeros; each lane keeps M
//                     partial sums; X (a few KB to 256 KB) is read through L1.
//   tiled  (M > 8, CSR uploaded with pfrt_csr_create): the weight is
//                     re-blocked once into 256-column chunks; a block stages a
//                     64-row x 256-column tile of X in shared memory and its
//                     warps walk their CSR rows' nonzeros in that chunk, each
//                     lane owning 2 rows of X; every X operand comes from
//                     shared memory instead of an L2 gather.
//   wide   (M > 8, caller-owned device CSR): X is transposed once to
//                     X^T [K, Mpad]; lanes split M (4 rows of X per lane,
//                     float4) and each nonzero's (index, value) is broadcast
//                     with a shuffle; the X^T rows are gathered from L2.
// Every index is bounds-checked; a bad one is skipped and recorded.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.hpp"

struct pfrt_csr {
    pfrt_ctx* ctx = nullptr;
    int64_t N = 0, K = 0, nnz = 0;
    int32_t* indptr = nullptr;   // [N+1]
    int32_t* indices = nullptr;  // [nnz]
    float* values = nullptr;     // [nnz]
    // Column-blocked copy for the tiled kernel: the nonzeros of column chunk
    // c (columns [c*KT, (c+1)*KT)) of every row, chunk-major, as packed
    // (local column, value bits) pairs, with row pointers cptr[c][N+1].
    int nchunks = 0;
    int32_t* cptr = nullptr;     // [nchunks][N+1]
    uint2* cent = nullptr;       // [nnz]
};

namespace pfrt {

constexpr int kSpmmThreads = 256;  // 8 warps per block

// Row range [j0, j1) clamped to [0, nnz]; an inverted range is empty.
__device__ __forceinline__ void row_range(const int32_t* __restrict__ indptr, int64_t n, int64_t nnz,
                                          int64_t& j0, int64_t& j1) {
    j0 = __ldg(indptr + n);
    j1 = __ldg(indptr + n + 1);
    j0 = j0 < 0 ? 0 : (j0 > nnz ? nnz : j0);
    j1 = j1 < j0 ? j0 : (j1 > nnz ? nnz : j1);
}

template <int MV>
__device__ __forceinline__ void skinny_accum(float (&acc)[MV], int M, int32_t col, float v,
                                             const float* __restrict__ x, int64_t ldx, int64_t K,
                                             bool& bad) {
    if (static_cast<uint32_t>(col) >= static_cast<uint64_t>(K)) {
        bad = true;
        return;
    }
#pragma unroll
    for (int m = 0; m < MV; ++m)
        if (m < M) acc[m] = __fmaf_rn(v, __ldg(x + m * ldx + col), acc[m]);
}

// M <= MV <= 8.  One warp per CSR row; the lanes share the row's nonzeros.
template <int MV>
__global__ void __launch_bounds__(kSpmmThreads)
    spmm_skinny_kernel(int M, int64_t N, int64_t K, int64_t nnz, const int32_t* __restrict__ indptr,
                       const int32_t* __restrict__ indices, const float* __restrict__ values,
                       const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy,
                       int* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kSpmmThreads + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kSpmmThreads) >> 5;
    bool bad = false;
    for (int64_t n = warp0; n < N; n += nwarps) {
        int64_t j0, j1;
        row_range(indptr, n, nnz, j0, j1);
        float acc[MV];
#pragma unroll
        for (int m = 0; m < MV; ++m) acc[m] = 0.0f;
        // Head: up to 3 nonzeros until j is a multiple of 4 (16-byte aligned).
        const int64_t ja = min((j0 + 3) & ~int64_t{3}, j1);
        if (j0 + lane < ja)
            skinny_accum<MV>(acc, M, __ldg(indices + j0 + lane), __ldg(values + j0 + lane), x, ldx, K, bad);
        // Body: 128-bit loads, 4 nonzeros each, four loads per lane issued
        // back to back before any use, so each lane keeps 8 independent
        // 16-byte loads in flight instead of one dependent load per step.
        const int64_t jb = ja + ((j1 - ja) & ~int64_t{3});
        for (int64_t j = ja + 4 * lane; j < jb; j += 512) {
            int4 c4[4];
            float4 v4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int64_t jj = j + 128 * u;
                if (jj < jb) {
                    c4[u] = __ldg(reinterpret_cast<const int4*>(indices + jj));
                    v4[u] = __ldg(reinterpret_cast<const float4*>(values + jj));
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (j + 128 * u < jb) {
                    skinny_accum<MV>(acc, M, c4[u].x, v4[u].x, x, ldx, K, bad);
                    skinny_accum<MV>(acc, M, c4[u].y, v4[u].y, x, ldx, K, bad);
                    skinny_accum<MV>(acc, M, c4[u].z, v4[u].z, x, ldx, K, bad);
                    skinny_accum<MV>(acc, M, c4[u].w, v4[u].w, x, ldx, K, bad);
                }
            }
        }
        // Tail: fewer than 4 nonzeros.
        if (jb + lane < j1)
            skinny_accum<MV>(acc, M, __ldg(indices + jb + lane), __ldg(values + jb + lane), x, ldx, K, bad);
#pragma unroll
        for (int m = 0; m < MV; ++m) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
            acc[m] = v;
        }
        if (lane < M) {
            float v = acc[0];
#pragma unroll
            for (int m = 1; m < MV; ++m)
                if (lane == m) v = acc[m];
            y[static_cast<int64_t>(lane) * ldy + n] = v;
        }
    }
    if (bad) report_error(err, kDevBadIndex);
}

// M > 8.  Warp per (CSR row, block of 128 rows of X).  xt is X^T [K, ldxt]
// with ldxt a multiple of 4 and columns >= M zero.
__global__ void __launch_bounds__(kSpmmThreads)
    spmm_wide_kernel(int M, int64_t N, int64_t K, int64_t nnz, const int32_t* __restrict__ indptr,
                     const int32_t* __restrict__ indices, const float* __restrict__ values,
                     const float* __restrict__ xt, int64_t ldxt, float* __restrict__ y, int64_t ldy,
                     int* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * kSpmmThreads + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kSpmmThreads) >> 5;
    const int64_t mblocks = (M + 127) / 128;
    const int64_t units = N * mblocks;
    bool bad = false;
    for (int64_t u = warp0; u < units; u += nwarps) {
        const int64_t n = u / mblocks;
        const int m0 = static_cast<int>(u % mblocks) * 128;
        const int mm = m0 + 4 * lane;
        const bool active = mm < M;
        int64_t j0, j1;
        row_range(indptr, n, nnz, j0, j1);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int64_t jc = j0; jc < j1; jc += 32) {
            int32_t c = 0;
            float v = 0.0f;
            if (jc + lane < j1) {
                c = __ldg(indices + jc + lane);
                v = __ldg(values + jc + lane);
                if (static_cast<uint32_t>(c) >= static_cast<uint64_t>(K)) {
                    bad = true;
                    c = 0;
                    v = 0.0f;
                }
            }
            const int cnt = static_cast<int>((j1 - jc) < 32 ? (j1 - jc) : 32);
            for (int t = 0; t < cnt; ++t) {
                const int32_t ct = __shfl_sync(0xffffffffu, c, t);
                const float vt = __shfl_sync(0xffffffffu, v, t);
                if (active) {
                    const float4 x4 = __ldg(reinterpret_cast<const float4*>(xt + static_cast<int64_t>(ct) * ldxt + mm));
                    acc.x = __fmaf_rn(vt, x4.x, acc.x);
                    acc.y = __fmaf_rn(vt, x4.y, acc.y);
                    acc.z = __fmaf_rn(vt, x4.z, acc.z);
                    acc.w = __fmaf_rn(vt, x4.w, acc.w);
                }
            }
        }
        if (active) {
            float* yp = y + static_cast<int64_t>(mm) * ldy + n;
            yp[0] = acc.x;
            if (mm + 1 < M) yp[ldy] = acc.y;
            if (mm + 2 < M) yp[2 * ldy] = acc.z;
            if (mm + 3 < M) yp[3 * ldy] = acc.w;
        }
    }
    if (bad) report_error(err, kDevBadIndex);
}

constexpr int kTileKT = 256;  // columns of X per staged chunk
constexpr int kTileMT = 64;   // rows of X per block (2 per lane)

// Dynamic shared memory of spmm_tiled_kernel: the X tile, then one 32-entry
// nonzero buffer per warp.  The output staging reuses the X tile.
constexpr size_t kTileSmem = sizeof(float2) * kTileKT * 32 + sizeof(uint2) * 8 * 32;

// Block = (64 rows of X, 8*RPW CSR rows).  For each 256-column chunk the block
// stages X[m0:m0+64, chunk] transposed into xs[k][pair] (pair p holds rows
// m0+2p and m0+2p+1, stored at position p ^ (k & 31) so that staging writes
// spread over the banks and the reads of one k stay a permutation), then
// each warp walks the chunk's nonzeros of its RPW rows: 32 (index, value)
// pairs are loaded coalesced into a per-warp buffer and broadcast to all
// lanes, and lane l accumulates rows m0+2l and m0+2l+1.
template <int RPW>
__global__ void __launch_bounds__(256)
    spmm_tiled_kernel(int M, int64_t N, int64_t K, int nchunks, const int32_t* __restrict__ cptr,
                      const uint2* __restrict__ cent, const float* __restrict__ x, int64_t ldx,
                      float* __restrict__ y, int64_t ldy, int64_t mtiles, int* err) {
    extern __shared__ __align__(16) uint8_t tsm[];
    float2* xs = reinterpret_cast<float2*>(tsm);
    uint2* ent = reinterpret_cast<uint2*>(tsm + sizeof(float2) * kTileKT * 32);
    constexpr int R = 8 * RPW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t mt = blockIdx.x % mtiles, nt = blockIdx.x / mtiles;
    const int m0 = static_cast<int>(mt) * kTileMT;
    const int64_t n0 = nt * R;
    uint2* wbuf = ent + warp * 32;
    float2 acc[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) acc[r] = make_float2(0.f, 0.f);
    bool bad = false;
    for (int c = 0; c < nchunks; ++c) {
        const int64_t k0 = static_cast<int64_t>(c) * kTileKT;
        const int kt = static_cast<int>((K - k0) < kTileKT ? (K - k0) : kTileKT);
        // Stage: thread i handles column k = i % 256 of pair p (rows m0+2p, +1).
        for (int e = threadIdx.x; e < kTileKT * 32; e += 256) {
            const int k = e % kTileKT, p = e / kTileKT;
            const int m = m0 + 2 * p;
            float2 v = make_float2(0.f, 0.f);
            if (k < kt) {
                if (m < M) v.x = __ldg(x + static_cast<int64_t>(m) * ldx + k0 + k);
                if (m + 1 < M) v.y = __ldg(x + static_cast<int64_t>(m + 1) * ldx + k0 + k);
            }
            xs[k * 32 + (p ^ (k & 31))] = v;
        }
        __syncthreads();
        const int32_t* cp = cptr + static_cast<int64_t>(c) * (N + 1);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int64_t n = n0 + warp * RPW + r;
            if (n < N) {
                const int64_t j0 = __ldg(cp + n), j1 = __ldg(cp + n + 1);
                for (int64_t jc = j0; jc < j1; jc += 32) {
                    if (jc + lane < j1) wbuf[lane] = __ldg(cent + jc + lane);
                    __syncwarp();
                    const int cnt = static_cast<int>((j1 - jc) < 32 ? (j1 - jc) : 32);
                    for (int t = 0; t < cnt; ++t) {
                        const uint2 en = wbuf[t];
                        const int k = static_cast<int>(en.x);
                        if (k >= kt) {  // outside this chunk: skip and record
                            bad = true;
                            continue;
                        }
                        const float v = __uint_as_float(en.y);
                        const float2 xv = xs[k * 32 + (lane ^ (k & 31))];
                        acc[r].x = __fmaf_rn(v, xv.x, acc[r].x);
                        acc[r].y = __fmaf_rn(v, xv.y, acc[r].y);
                    }
                    __syncwarp();
                }
            }
        }
        __syncthreads();
    }
    // Output: stage [64 rows of X][R CSR rows] so the stores run along n.
    float* ys = reinterpret_cast<float*>(tsm);
    constexpr int LDYS = R + 1;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        ys[(2 * lane) * LDYS + warp * RPW + r] = acc[r].x;
        ys[(2 * lane + 1) * LDYS + warp * RPW + r] = acc[r].y;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kTileMT * R; e += 256) {
        const int m = e / R, i = e % R;
        if (m0 + m < M && n0 + i < N) y[static_cast<int64_t>(m0 + m) * ldy + n0 + i] = ys[m * LDYS + i];
    }
    if (bad) report_error(err, kDevBadIndex);
}

// xt[k, m] = x[m, k] for m < M, 0 for M <= m < ldxt.  32x32 tiles.
__global__ void transpose_pad_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx,
                                     float* __restrict__ xt, int64_t ldxt) {
    __shared__ float tile[32][33];
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t m = m0 + i, k = k0 + threadIdx.x;
        tile[i][threadIdx.x] = (m < M && k < K) ? x[m * ldx + k] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int64_t k = k0 + i, m = m0 + threadIdx.x;
        if (k < K && m < ldxt) xt[k * ldxt + m] = tile[threadIdx.x][i];
    }
}

namespace {

pfrt_status validate_host_csr(int64_t N, int64_t K, int64_t nnz, const void* indptr,
                              const void* indices, int bits, std::vector<int32_t>& ip32,
                              std::vector<int32_t>& ix32) {
    if (bits != 32 && bits != 64) return fail(PFRT_ERR_INVALID_ARGUMENT, "CSR index_bits must be 32 or 64");
    if (N < 0 || K < 0 || nnz < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "CSR: negative size");
    if (nnz > INT32_MAX || K > INT32_MAX)
        return fail(PFRT_ERR_UNSUPPORTED, "CSR: nnz and K must fit in int32 for the device format");
    ip32.resize(static_cast<size_t>(N + 1));
    ix32.resize(static_cast<size_t>(nnz));
    auto ip_at = [&](int64_t i) -> int64_t {
        return bits == 32 ? static_cast<const int32_t*>(indptr)[i] : static_cast<const int64_t*>(indptr)[i];
    };
    auto ix_at = [&](int64_t i) -> int64_t {
        return bits == 32 ? static_cast<const int32_t*>(indices)[i] : static_cast<const int64_t*>(indices)[i];
    };
    if (ip_at(0) != 0) return fail(PFRT_ERR_BAD_CSR, "CSR indptr[0] must be 0");
    for (int64_t r = 0; r < N; ++r) {
        const int64_t a = ip_at(r), b = ip_at(r + 1);
        if (b < a)
            return fail(PFRT_ERR_BAD_CSR, "CSR indptr decreases at row " + std::to_string(r));
        ip32[r] = static_cast<int32_t>(a);
    }
    if (ip_at(N) != nnz)
        return fail(PFRT_ERR_BAD_CSR, "CSR indptr[N] = " + std::to_string(ip_at(N)) + " != nnz = " +
                                          std::to_string(nnz));
    ip32[N] = static_cast<int32_t>(nnz);
    for (int64_t j = 0; j < nnz; ++j) {
        const int64_t c = ix_at(j);
        if (c < 0 || c >= K)
            return fail(PFRT_ERR_BAD_CSR, "CSR column index " + std::to_string(c) +
                                              " out of range [0, " + std::to_string(K) + ")");
        ix32[j] = static_cast<int32_t>(c);
    }
    return PFRT_OK;
}

pfrt_status run_spmm(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t K, int64_t nnz,
                     const int32_t* indptr, const int32_t* indices, const float* values,
                     const float* x, int64_t ldx, float* y, int64_t ldy, cudaStream_t s) {
    if (M < 0 || N < 0 || K < 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: negative size");
    if (M == 0 || N == 0) return PFRT_OK;
    if (M > INT32_MAX - 256) return fail(PFRT_ERR_UNSUPPORTED, "SpMM: M too large");
    if (!indptr || !x || !y || (nnz > 0 && (!indices || !values)))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: null pointer");
    if (ldx < K || ldy < N) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: row stride too small");
    const bool aligned = ((reinterpret_cast<uintptr_t>(indices) | reinterpret_cast<uintptr_t>(values)) & 15u) == 0;
    if (!aligned) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: indices/values must be 16-byte aligned");
    const int max_blocks = ctx->num_sms * 8;
    if (M <= 8) {
        const int64_t warps = N;
        const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(warps, kSpmmThreads / 32), max_blocks));
        const int Mi = static_cast<int>(M);
#define PFRT_SKINNY(MV)                                                                        \
    spmm_skinny_kernel<MV><<<blocks, kSpmmThreads, 0, s>>>(Mi, N, K, nnz, indptr, indices, values, \
                                                           x, ldx, y, ldy, ctx->d_err)
        if (M == 1) PFRT_SKINNY(1);
        else if (M == 2) PFRT_SKINNY(2);
        else if (M <= 4) PFRT_SKINNY(4);
        else PFRT_SKINNY(8);
#undef PFRT_SKINNY
        PFRT_CHECK_LAUNCH("spmm_skinny_kernel");
        return PFRT_OK;
    }
    const int64_t ldxt = static_cast<int64_t>(align_up(static_cast<size_t>(M), 4));
    void* scr = nullptr;
    pfrt_status st = scratch(ctx, sizeof(float) * ldxt * std::max<int64_t>(K, 1), &scr);
    if (st) return st;
    float* xt = static_cast<float*>(scr);
    if (K > 0) {
        dim3 tb(32, 8);
        dim3 tg(static_cast<unsigned>(ceil_div(K, 32)), static_cast<unsigned>(ceil_div(ldxt, 32)));
        transpose_pad_kernel<<<tg, tb, 0, s>>>(x, M, K, ldx, xt, ldxt);
        PFRT_CHECK_LAUNCH("transpose_pad_kernel");
    }
    const int64_t warps = N * ceil_div(M, 128);
    const int blocks = static_cast<int>(std::min<int64_t>(ceil_div(warps, kSpmmThreads / 32), max_blocks));
    spmm_wide_kernel<<<blocks, kSpmmThreads, 0, s>>>(static_cast<int>(M), N, K, nnz, indptr, indices,
                                                     values, xt, ldxt, y, ldy, ctx->d_err);
    PFRT_CHECK_LAUNCH("spmm_wide_kernel");
    return PFRT_OK;
}

template <int RPW>
pfrt_status launch_tiled(pfrt_ctx* ctx, const pfrt_csr* w, int64_t M, const float* x, int64_t ldx,
                         float* y, int64_t ldy, cudaStream_t s) {
    auto kern = spmm_tiled_kernel<RPW>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kTileSmem)));
    const int64_t mtiles = ceil_div(M, kTileMT);
    const int64_t units = mtiles * ceil_div(w->N, 8 * RPW);
    if (units > INT32_MAX) return fail(PFRT_ERR_UNSUPPORTED, "SpMM: too many tiles");
    kern<<<static_cast<unsigned>(units), 256, kTileSmem, s>>>(
        static_cast<int>(M), w->N, w->K, w->nchunks, w->cptr, w->cent, x, ldx, y, ldy, mtiles, ctx->d_err);
    PFRT_CHECK_LAUNCH("spmm_tiled_kernel");
    return PFRT_OK;
}

pfrt_status run_spmm_tiled(pfrt_ctx* ctx, const pfrt_csr* w, int64_t M, const float* x, int64_t ldx,
                           float* y, int64_t ldy, cudaStream_t s) {
    if (M > INT32_MAX - 256) return fail(PFRT_ERR_UNSUPPORTED, "SpMM: M too large");
    if (!x || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: null pointer");
    if (ldx < w->K || ldy < w->N) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: row stride too small");
    if (w->N == 0) return PFRT_OK;
    // Rows per warp: the largest that still gives every SM two blocks.
    const int64_t mtiles = ceil_div(M, kTileMT);
    int rpw = 4;
    for (int cand : {32, 16, 8}) {
        if (mtiles * ceil_div(w->N, 8 * cand) >= 2 * ctx->num_sms) {
            rpw = cand;
            break;
        }
    }
    switch (rpw) {
        case 32: return launch_tiled<32>(ctx, w, M, x, ldx, y, ldy, s);
        case 16: return launch_tiled<16>(ctx, w, M, x, ldx, y, ldy, s);
        case 8: return launch_tiled<8>(ctx, w, M, x, ldx, y, ldy, s);
        default: return launch_tiled<4>(ctx, w, M, x, ldx, y, ldy, s);
    }
}

}  // namespace
}  // namespace pfrt

using namespace pfrt;

extern "C" {

pfrt_status pfrt_csr_create(pfrt_ctx* ctx, int64_t N, int64_t K, int64_t nnz,
                            const void* indptr_host, const void* indices_host, int index_bits,
                            const float* values_host, pfrt_csr** out) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!out || !indptr_host || (nnz > 0 && (!indices_host || !values_host)))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_csr_create: null argument");
    *out = nullptr;
    std::vector<int32_t> ip, ix;
    st = validate_host_csr(N, K, nnz, indptr_host, indices_host, index_bits, ip, ix);
    if (st) return st;
    auto* w = new pfrt_csr();
    w->ctx = ctx;
    w->N = N;
    w->K = K;
    w->nnz = nnz;
    // Round the nonzero arrays up to a multiple of 4 so 128-bit loads of the
    // last group stay inside the allocation.
    const size_t cap = align_up(static_cast<size_t>(std::max<int64_t>(nnz, 1)), 4);
    cudaError_t e = cudaMalloc(&w->indptr, sizeof(int32_t) * (N + 1));
    if (e == cudaSuccess) e = cudaMalloc(&w->indices, sizeof(int32_t) * cap);
    if (e == cudaSuccess) e = cudaMalloc(&w->values, sizeof(float) * cap);
    if (e == cudaSuccess) e = cudaMemcpy(w->indptr, ip.data(), sizeof(int32_t) * (N + 1), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && nnz > 0)
        e = cudaMemcpy(w->indices, ix.data(), sizeof(int32_t) * nnz, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && nnz > 0)
        e = cudaMemcpy(w->values, values_host, sizeof(float) * nnz, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        pfrt_csr_destroy(w);
        return cuda_fail(e, "pfrt_csr_create");
    }
    // Column-blocked copy for the tiled kernel (stable within each row).
    w->nchunks = static_cast<int>(std::max<int64_t>(1, ceil_div(K, kTileKT)));
    {
        const int C = w->nchunks;
        std::vector<int32_t> cptr(static_cast<size_t>(C) * (N + 1), 0);
        for (int64_t r = 0; r < N; ++r)
            for (int32_t j = ip[r]; j < ip[r + 1]; ++j) ++cptr[static_cast<size_t>(ix[j] / kTileKT) * (N + 1) + r + 1];
        int64_t run = 0;
        for (int c = 0; c < C; ++c) {
            int32_t* row = cptr.data() + static_cast<size_t>(c) * (N + 1);
            row[0] = static_cast<int32_t>(run);
            for (int64_t r = 0; r < N; ++r) {
                run += row[r + 1];
                row[r + 1] = static_cast<int32_t>(run);
            }
        }
        std::vector<int32_t> fill(cptr);
        std::vector<uint2> cent(static_cast<size_t>(std::max<int64_t>(nnz, 1)));
        const float* vh = values_host;
        for (int64_t r = 0; r < N; ++r)
            for (int32_t j = ip[r]; j < ip[r + 1]; ++j) {
                const int c = ix[j] / kTileKT;
                uint32_t bits;
                std::memcpy(&bits, vh + j, 4);
                cent[fill[static_cast<size_t>(c) * (N + 1) + r]++] =
                    make_uint2(static_cast<uint32_t>(ix[j] - c * kTileKT), bits);
            }
        e = cudaMalloc(&w->cptr, sizeof(int32_t) * cptr.size());
        if (e == cudaSuccess) e = cudaMalloc(&w->cent, sizeof(uint2) * cent.size());
        if (e == cudaSuccess)
            e = cudaMemcpy(w->cptr, cptr.data(), sizeof(int32_t) * cptr.size(), cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(w->cent, cent.data(), sizeof(uint2) * cent.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            pfrt_csr_destroy(w);
            return cuda_fail(e, "pfrt_csr_create (blocked copy)");
        }
    }
    *out = w;
    return PFRT_OK;
}

pfrt_status pfrt_csr_validate_host(int64_t N, int64_t K, int64_t nnz, const void* indptr_host,
                                   const void* indices_host, int index_bits) {
    if (!indptr_host || (nnz > 0 && !indices_host))
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_csr_validate_host: null argument");
    std::vector<int32_t> ip, ix;
    return validate_host_csr(N, K, nnz, indptr_host, indices_host, index_bits, ip, ix);
}

pfrt_status pfrt_csr_destroy(pfrt_csr* w) {
    if (!w) return PFRT_OK;
    if (w->ctx) cudaSetDevice(w->ctx->device);
    if (w->indptr) cudaFree(w->indptr);
    if (w->indices) cudaFree(w->indices);
    if (w->values) cudaFree(w->values);
    if (w->cptr) cudaFree(w->cptr);
    if (w->cent) cudaFree(w->cent);
    delete w;
    return PFRT_OK;
}

pfrt_status pfrt_csr_info(const pfrt_csr* w, int64_t* n, int64_t* k, int64_t* nnz) {
    if (!w) return fail(PFRT_ERR_INVALID_ARGUMENT, "null CSR");
    if (n) *n = w->N;
    if (k) *k = w->K;
    if (nnz) *nnz = w->nnz;
    return PFRT_OK;
}

pfrt_status pfrt_spmm(pfrt_ctx* ctx, const pfrt_csr* w, int64_t M, const float* x, int64_t ldx,
                      float* y, int64_t ldy, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!w) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: null CSR");
    if (w->ctx != ctx) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: CSR belongs to another context");
    const char* tiled = std::getenv("PFRT_SPMM_TILED");
    if (M > 8 && tiled && *tiled == '1')
        return run_spmm_tiled(ctx, w, M, x, ldx, y, ldy, pick_stream(ctx, stream));
    return run_spmm(ctx, M, w->N, w->K, w->nnz, w->indptr, w->indices, w->values, x, ldx, y, ldy,
                    pick_stream(ctx, stream));
}

pfrt_status pfrt_spmm_csr_f32(pfrt_ctx* ctx, int64_t M, int64_t N, int64_t K, int64_t nnz,
                              const int32_t* indptr, const int32_t* indices,
                              const float* values, const float* x, int64_t ldx, float* y,
                              int64_t ldy, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    return run_spmm(ctx, M, N, K, nnz, indptr, indices, values, x, ldx, y, ldy,
                    pick_stream(ctx, stream));
}

}  // extern "C"
