// prune.cu -- magnitude pruning of a dense fp32 weight straight into a CSR
// weight on the GPU.
//
// Reproduces pruning::MagnitudePruning::compute_mask
// (src/pruning/magnitude_pruning.cpp:22-102) and pruning::to_sparse of
// W * mask with threshold 0 (src/pruning/sparse_tensor.cpp:560-587):
//   threshold T = the floor(n*s)-th smallest |w| (0-based, capped at n-1);
//   the mask keeps |w| > T; if more than (size_t)((float)n * s) weights are
//   then pruned, the first entries (in index order) with |w| == T are kept
//   again until that count is reached; the CSR holds the kept entries whose
//   value is not 0, row by row in column order.
//
// |w| as an unsigned 32-bit pattern orders like the float (it is
// non-negative), so T is found by a radix select over the bit patterns: four
// passes of a 256-bin histogram of one byte among the elements that share the
// bytes already chosen.  Each pass also tells how many elements are below
// the chosen prefix, so the counts of |w| < T and |w| == T come for free.
// The index-order rank of a tie is the number of ties in earlier rows (an
// exclusive scan of per-row counts) plus the ties before it in its row
// (ballot/popc within the warp that owns the row).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.hpp"

namespace pfrt {
namespace {

constexpr uint32_t kNanBits = 0x7f800000u;  // |w| bits above this are NaN

// hist[d] += #{ i : (u_i & pmask) == prefix, (u_i >> shift) & 255 == d },
// u_i = bits of |w_i|; nan[0] += #{ u_i > kNanBits } (first pass only).
__global__ void prune_hist_kernel(const float* __restrict__ w, int64_t n, uint32_t prefix, uint32_t pmask,
                                  int shift, unsigned long long* __restrict__ hist,
                                  unsigned long long* __restrict__ nan) {
    __shared__ unsigned int sh[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh[i] = 0;
    __syncthreads();
    unsigned int nn = 0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t u = __float_as_uint(w[i]) & 0x7fffffffu;
        nn += (u > kNanBits);
        if ((u & pmask) == prefix) atomicAdd(&sh[(u >> shift) & 255u], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
        if (sh[i]) atomicAdd(hist + i, static_cast<unsigned long long>(sh[i]));
    if (nan) {
        for (int o = 16; o; o >>= 1) nn += __shfl_xor_sync(0xffffffffu, nn, o);
        if ((threadIdx.x & 31) == 0 && nn) atomicAdd(nan, static_cast<unsigned long long>(nn));
    }
}

// Per row: gt[r] = #{ |w| > T }, eq[r] = #{ |w| == T }.  Warp per row.
__global__ void prune_rowstat_kernel(const float* __restrict__ w, int64_t N, int64_t K, uint32_t T,
                                     int32_t* __restrict__ gt, int32_t* __restrict__ eq) {
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= N) return;
    const float* row = w + r * K;
    int g = 0, e = 0;
    for (int64_t c = lane; c < K; c += 32) {
        const uint32_t u = __float_as_uint(row[c]) & 0x7fffffffu;
        g += (u > T);
        e += (u == T);
    }
    for (int o = 16; o; o >>= 1) {
        g += __shfl_xor_sync(0xffffffffu, g, o);
        e += __shfl_xor_sync(0xffffffffu, e, o);
    }
    if (lane == 0) {
        gt[r] = g;
        eq[r] = e;
    }
}

// Writes the mask (optional) and the CSR entries of each row.  A tie of row
// r with rank eq_base[r] + (ties before it in the row) is kept when that rank
// is below `restore`; a kept tie enters the CSR only when T > 0 (its value
// is then not 0).  Warp per row, 32 columns at a time in column order.
__global__ void prune_compact_kernel(const float* __restrict__ w, int64_t N, int64_t K, uint32_t T,
                                     uint64_t restore, const int64_t* __restrict__ eq_base,
                                     const int32_t* __restrict__ indptr, float* __restrict__ mask,
                                     int32_t* __restrict__ indices, float* __restrict__ values) {
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= N) return;
    const float* row = w + r * K;
    const uint32_t lt = (1u << lane) - 1u;
    uint64_t tie = static_cast<uint64_t>(eq_base[r]);
    int64_t out = indptr[r];
    for (int64_t c0 = 0; c0 < K; c0 += 32) {
        const int64_t c = c0 + lane;
        const bool in = c < K;
        const float v = in ? row[c] : 0.0f;
        const uint32_t u = __float_as_uint(v) & 0x7fffffffu;
        const bool g = in && u > T;
        const bool e = in && u == T;
        const uint32_t eb = __ballot_sync(0xffffffffu, e);
        const bool keep = g || (e && tie + __popc(eb & lt) < restore);
        const bool csr = g || (keep && T > 0u);
        const uint32_t cb = __ballot_sync(0xffffffffu, csr);
        if (in && mask) mask[r * K + c] = keep ? 1.0f : 0.0f;
        if (csr) {
            const int64_t at = out + __popc(cb & lt);
            indices[at] = static_cast<int32_t>(c);
            values[at] = v;
        }
        tie += __popc(eb);
        out += __popc(cb);
    }
}

// ------------------------------------------------------------ N:M pruning
// pruning::NMSparsityPruning::compute_mask (src/pruning/nm_sparsity.cpp:45-126):
// each group of m consecutive weights in flat order keeps its n largest |w|
// (a last group of g < m keeps min(ceil((float)(g*n) / m), g)).  Which of
// equal |w| stay is decided by the reference's std::partial_sort; libstdc++
// (GCC 13) implements it as a heap selection, restated here move for move:
// a binary heap over the first k slots, top = the element no other precedes
// under gt(a, b) = |w[a]| > |w[b]|, built bottom-up; each later element that
// precedes the top replaces it.  A sift moves the hole to a leaf along the
// preferred child (the right one unless it precedes the left), then sifts the
// value up from there.
constexpr int kNmMax = 32;

__device__ __forceinline__ void nm_sift(const float* a, int* h, int hole, int len, int v) {
    const int top = hole;
    int child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (a[h[child]] > a[h[child - 1]]) child--;
        h[hole] = h[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        h[hole] = h[child - 1];
        hole = child - 1;
    }
    int parent = (hole - 1) / 2;
    while (hole > top && a[h[parent]] > a[v]) {
        h[hole] = h[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    h[hole] = v;
}

// One thread per group: mask[i] = 1 for the kept weights of the group, else 0.
__global__ void nm_mask_kernel(const float* __restrict__ w, int64_t total, int n, int m, float* __restrict__ mask) {
    const int64_t grp = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t i0 = grp * m;
    if (i0 >= total) return;
    const int g = static_cast<int>(min(static_cast<int64_t>(m), total - i0));
    int k = n;
    if (g < m) k = min(g, static_cast<int>(ceilf(__fdiv_rn(static_cast<float>(static_cast<uint64_t>(g) * n),
                                                        static_cast<float>(m)))));
    float a[kNmMax];
    int h[kNmMax];
    for (int j = 0; j < g; ++j) a[j] = fabsf(w[i0 + j]);
    for (int j = 0; j < k; ++j) h[j] = j;
    if (k >= 2)
        for (int parent = (k - 2) / 2;; --parent) {
            nm_sift(a, h, parent, k, h[parent]);
            if (parent == 0) break;
        }
    for (int j = k; j < g; ++j)
        if (a[j] > a[h[0]]) nm_sift(a, h, 0, k, j);
    uint32_t kept = 0;
    for (int j = 0; j < k; ++j) kept |= 1u << h[j];
    for (int j = 0; j < g; ++j) mask[i0 + j] = ((kept >> j) & 1u) ? 1.0f : 0.0f;
}

// Per row: the entries to_sparse keeps of W * mask (|w| > 0 where kept).  Warp per row.
__global__ void masked_rowcount_kernel(const float* __restrict__ w, const float* __restrict__ mask, int64_t N,
                                       int64_t K, int32_t* __restrict__ cnt) {
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= N) return;
    int c = 0;
    for (int64_t j = lane; j < K; j += 32) c += (mask[r * K + j] != 0.0f && fabsf(w[r * K + j]) > 0.0f);
    for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) cnt[r] = c;
}

// Those entries, row by row in column order.  Warp per row.
__global__ void masked_compact_kernel(const float* __restrict__ w, const float* __restrict__ mask, int64_t N,
                                      int64_t K, const int32_t* __restrict__ indptr, int32_t* __restrict__ indices,
                                      float* __restrict__ values) {
    const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= N) return;
    const uint32_t lt = (1u << lane) - 1u;
    int64_t out = indptr[r];
    for (int64_t c0 = 0; c0 < K; c0 += 32) {
        const int64_t c = c0 + lane;
        const float v = c < K ? w[r * K + c] : 0.0f;
        const bool keep = c < K && mask[r * K + c] != 0.0f && fabsf(v) > 0.0f;
        const uint32_t b = __ballot_sync(0xffffffffu, keep);
        if (keep) {
            const int64_t at = out + __popc(b & lt);
            indices[at] = static_cast<int32_t>(c);
            values[at] = v;
        }
        out += __popc(b);
    }
}

}  // namespace
}  // namespace pfrt

using namespace pfrt;

extern "C" {

pfrt_status pfrt_csr_from_magnitude_pruning(pfrt_ctx* ctx, int64_t N, int64_t K, const float* w_dev,
                                            float sparsity, float* mask_dev, pfrt_csr** out) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!out || (N * K > 0 && !w_dev)) return fail(PFRT_ERR_INVALID_ARGUMENT, "magnitude pruning: null argument");
    if (N < 0 || K < 0 || N > INT32_MAX || K > INT32_MAX)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "magnitude pruning: bad shape");
    *out = nullptr;
    const int64_t n = N * K;
    if (sparsity > 0.0f && sparsity < 1.0f && n == 0)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "Cannot prune empty weight tensor");  // magnitude_pruning.cpp:54-56
    if (std::isnan(sparsity)) return fail(PFRT_ERR_INVALID_ARGUMENT, "magnitude pruning: sparsity is NaN");
    cudaStream_t s = ctx->stream;
    const int blocks = std::max(1, std::min(ctx->num_sms * 8, static_cast<int>(std::min<int64_t>(ceil_div(n, 256), INT32_MAX))));

    // Device scratch: hist[256] + nan[1] (u64), gt/eq [N] (i32), eq_base [N] (i64), indptr [N+1] (i32).
    unsigned long long* hist = nullptr;
    int32_t *gt = nullptr, *eq = nullptr, *indptr = nullptr, *indices = nullptr;
    int64_t* eq_base = nullptr;
    float* values = nullptr;
    auto cleanup = [&](pfrt_status r) {
        if (hist) cudaFree(hist);
        if (gt) cudaFree(gt);
        if (eq) cudaFree(eq);
        if (eq_base) cudaFree(eq_base);
        if (indptr) cudaFree(indptr);
        if (indices) cudaFree(indices);
        if (values) cudaFree(values);
        return r;
    };
    cudaError_t e = cudaMalloc(&hist, sizeof(unsigned long long) * 257);
    if (e == cudaSuccess) e = cudaMalloc(&gt, sizeof(int32_t) * std::max<int64_t>(N, 1));
    if (e == cudaSuccess) e = cudaMalloc(&eq, sizeof(int32_t) * std::max<int64_t>(N, 1));
    if (e == cudaSuccess) e = cudaMalloc(&eq_base, sizeof(int64_t) * std::max<int64_t>(N, 1));
    if (e == cudaSuccess) e = cudaMalloc(&indptr, sizeof(int32_t) * (N + 1));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "magnitude pruning scratch"));

    // Threshold (as |w| bits) and the number of ties to keep.
    uint32_t T = 0;
    uint64_t restore = 0;
    if (sparsity <= 0.0f) {
        // Keep everything (magnitude_pruning.cpp:33-39): T = 0 with every
        // |w| == 0 restored; the CSR still drops the zeros.
        T = 0;
        restore = UINT64_MAX;
    } else if (sparsity >= 1.0f) {
        T = 0xffffffffu;  // nothing is above it; no tie is restored
        restore = 0;
    } else {
        const uint64_t idx = std::min<uint64_t>(static_cast<uint64_t>(std::floor(static_cast<double>(n) * sparsity)),
                                                static_cast<uint64_t>(n - 1));
        uint64_t k = idx, below = 0, equal = 0;
        uint32_t prefix = 0, pmask = 0;
        std::vector<unsigned long long> h(257);
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            e = cudaMemsetAsync(hist, 0, sizeof(unsigned long long) * 257, s);
            if (e != cudaSuccess) return cleanup(cuda_fail(e, "magnitude pruning"));
            prune_hist_kernel<<<blocks, 256, 0, s>>>(w_dev, n, prefix, pmask, shift, hist, pass == 0 ? hist + 256 : nullptr);
            e = cudaGetLastError();
            if (e == cudaSuccess) e = cudaMemcpyAsync(h.data(), hist, sizeof(unsigned long long) * 257, cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) return cleanup(cuda_fail(e, "prune_hist_kernel"));
            if (pass == 0 && h[256] != 0)
                return cleanup(fail(PFRT_ERR_INVALID_ARGUMENT, "magnitude pruning: NaN in weights"));
            uint64_t cum = 0;
            int d = 0;
            for (; d < 256; ++d) {
                if (k < cum + h[d]) break;
                cum += h[d];
            }
            if (d == 256) return cleanup(fail(PFRT_ERR_CUDA, "magnitude pruning: histogram count mismatch"));
            k -= cum;
            below += cum;
            equal = h[d];
            prefix |= static_cast<uint32_t>(d) << shift;
            pmask |= 0xffu << shift;
        }
        T = prefix;
        // magnitude_pruning.cpp:84-98; size_t * float is evaluated in float.
        const uint64_t target = static_cast<uint64_t>(static_cast<float>(n) * sparsity);
        const uint64_t zeros = below + equal;
        restore = zeros > target ? std::min<uint64_t>(zeros - target, equal) : 0;
    }

    // Per-row counts -> tie ranks and CSR row pointers (host scan).
    const unsigned rb = static_cast<unsigned>(std::max<int64_t>(1, ceil_div(N * 32, 256)));
    std::vector<int32_t> hgt(static_cast<size_t>(N)), heq(static_cast<size_t>(N));
    if (N > 0) {
        prune_rowstat_kernel<<<rb, 256, 0, s>>>(w_dev, N, K, T, gt, eq);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpyAsync(hgt.data(), gt, sizeof(int32_t) * N, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(heq.data(), eq, sizeof(int32_t) * N, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "prune_rowstat_kernel"));
    }
    std::vector<int64_t> hbase(static_cast<size_t>(N));
    std::vector<int32_t> hip(static_cast<size_t>(N + 1));
    int64_t ties = 0, kept = 0;
    hip[0] = 0;
    for (int64_t r = 0; r < N; ++r) {
        hbase[r] = ties;
        int64_t rt = 0;  // restored ties of this row
        if (restore > static_cast<uint64_t>(ties))
            rt = static_cast<int64_t>(std::min<uint64_t>(restore - static_cast<uint64_t>(ties), static_cast<uint64_t>(heq[r])));
        ties += heq[r];
        kept += hgt[r] + (T > 0 ? rt : 0);
        if (kept > INT32_MAX) return cleanup(fail(PFRT_ERR_UNSUPPORTED, "magnitude pruning: more than 2^31 nonzeros"));
        hip[r + 1] = static_cast<int32_t>(kept);
    }
    const int64_t nnz = kept;
    e = cudaMalloc(&indices, sizeof(int32_t) * std::max<int64_t>(nnz, 1));
    if (e == cudaSuccess) e = cudaMalloc(&values, sizeof(float) * std::max<int64_t>(nnz, 1));
    if (e == cudaSuccess && N > 0)
        e = cudaMemcpyAsync(eq_base, hbase.data(), sizeof(int64_t) * N, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(indptr, hip.data(), sizeof(int32_t) * (N + 1), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "magnitude pruning"));
    if (N > 0) {
        prune_compact_kernel<<<rb, 256, 0, s>>>(w_dev, N, K, T, restore, eq_base, indptr, mask_dev, indices, values);
        e = cudaGetLastError();
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "prune_compact_kernel"));
    }
    std::vector<int32_t> hix(static_cast<size_t>(std::max<int64_t>(nnz, 1)));
    std::vector<float> hv(static_cast<size_t>(std::max<int64_t>(nnz, 1)));
    if (nnz > 0) {
        e = cudaMemcpyAsync(hix.data(), indices, sizeof(int32_t) * nnz, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(hv.data(), values, sizeof(float) * nnz, cudaMemcpyDeviceToHost, s);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "magnitude pruning"));
    cleanup(PFRT_OK);
    return pfrt_csr_create(ctx, N, K, nnz, hip.data(), hix.data(), 32, hv.data(), out);
}

pfrt_status pfrt_csr_from_nm_pruning(pfrt_ctx* ctx, int64_t N, int64_t K, const float* w_dev, int32_t n, int32_t m,
                                     float* mask_dev, pfrt_csr** out) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!out || (N * K > 0 && !w_dev)) return fail(PFRT_ERR_INVALID_ARGUMENT, "N:M pruning: null argument");
    if (N < 0 || K < 0 || N > INT32_MAX || K > INT32_MAX)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "N:M pruning: bad shape");
    *out = nullptr;
    // nm_sparsity.cpp:9-18 (the constructor's checks, in its order)
    if (n > m) return fail(PFRT_ERR_INVALID_ARGUMENT, "N must be <= M in N:M sparsity");
    if (n <= 0 || m <= 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "N and M must be > 0");
    if (m > kNmMax) return fail(PFRT_ERR_UNSUPPORTED, "N:M pruning: M above 32");
    const int64_t total = N * K;
    cudaStream_t s = ctx->stream;
    float* mask = mask_dev;
    int32_t *cnt = nullptr, *indptr = nullptr, *indices = nullptr;
    float* values = nullptr;
    float* own_mask = nullptr;
    auto cleanup = [&](pfrt_status r) {
        if (own_mask) cudaFree(own_mask);
        if (cnt) cudaFree(cnt);
        if (indptr) cudaFree(indptr);
        if (indices) cudaFree(indices);
        if (values) cudaFree(values);
        return r;
    };
    cudaError_t e = cudaSuccess;
    if (!mask && total > 0) {
        e = cudaMalloc(&own_mask, sizeof(float) * total);
        mask = own_mask;
    }
    if (e == cudaSuccess) e = cudaMalloc(&cnt, sizeof(int32_t) * std::max<int64_t>(N, 1));
    if (e == cudaSuccess) e = cudaMalloc(&indptr, sizeof(int32_t) * (N + 1));
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "N:M pruning scratch"));
    std::vector<int32_t> hc(static_cast<size_t>(N));
    if (total > 0) {
        const int64_t groups = ceil_div(total, static_cast<int64_t>(m));
        nm_mask_kernel<<<static_cast<unsigned>(ceil_div(groups, 128)), 128, 0, s>>>(w_dev, total, n, m, mask);
        e = cudaGetLastError();
        const unsigned rb = static_cast<unsigned>(std::max<int64_t>(1, ceil_div(N * 32, 256)));
        if (e == cudaSuccess) {
            masked_rowcount_kernel<<<rb, 256, 0, s>>>(w_dev, mask, N, K, cnt);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpyAsync(hc.data(), cnt, sizeof(int32_t) * N, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "nm_mask_kernel"));
    }
    std::vector<int32_t> hip(static_cast<size_t>(N + 1));
    int64_t nnz = 0;
    hip[0] = 0;
    for (int64_t r = 0; r < N; ++r) {
        nnz += hc[r];
        if (nnz > INT32_MAX) return cleanup(fail(PFRT_ERR_UNSUPPORTED, "N:M pruning: more than 2^31 nonzeros"));
        hip[r + 1] = static_cast<int32_t>(nnz);
    }
    std::vector<int32_t> hix(static_cast<size_t>(std::max<int64_t>(nnz, 1)));
    std::vector<float> hv(static_cast<size_t>(std::max<int64_t>(nnz, 1)));
    if (nnz > 0) {
        e = cudaMalloc(&indices, sizeof(int32_t) * nnz);
        if (e == cudaSuccess) e = cudaMalloc(&values, sizeof(float) * nnz);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(indptr, hip.data(), sizeof(int32_t) * (N + 1), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
            const unsigned rb = static_cast<unsigned>(std::max<int64_t>(1, ceil_div(N * 32, 256)));
            masked_compact_kernel<<<rb, 256, 0, s>>>(w_dev, mask, N, K, indptr, indices, values);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpyAsync(hix.data(), indices, sizeof(int32_t) * nnz, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(hv.data(), values, sizeof(float) * nnz, cudaMemcpyDeviceToHost, s);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cleanup(cuda_fail(e, "N:M pruning"));
    cleanup(PFRT_OK);
    return pfrt_csr_create(ctx, N, K, nnz, hip.data(), hix.data(), 32, hv.data(), out);
}

}  // extern "C"
