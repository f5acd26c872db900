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
#include "spmm_sp.cuh"
#include "spmm_tc.cuh"

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
    int32_t* cptr = nullptr;     // [nchunks][N+1] (+4 entries of slack for 16-byte bulk copies)
    uint2* cent = nullptr;       // [nnz] (+2 entries of slack)
    std::vector<int32_t> host_cptr;
    // Row groups of the mid-batch kernel (spmm_xtile_kernel), built on first use.
    int32_t* xt_part = nullptr;  // [xt_groups + 1]
    int64_t xt_groups = 0;
    // Dense tf32-split copy of W for large batches (built on first use).
    pfrt_fweight* dense = nullptr;
    // Row partition of the streaming kernel for `part_warps` warps.
    int64_t part_warps = 0;
    int32_t* part = nullptr;     // [part_warps + 1]
    std::vector<int32_t> host_indptr;
    // Compressed form for the tensor-core kernel (spmm_tc.cuh), built on
    // first use: 0 not built, 1 ready, -1 unusable (a column stored twice
    // in a row).
    int tc_state = 0;
    int64_t tc_npad = 0;
    uint32_t* tc_mask = nullptr;  // [kb_total][tc_npad]
    uint32_t* tc_off = nullptr;   // [kb_total][tc_npad]
    float2* tc_vals = nullptr;    // [nnz]
    // Form of W for the structured-sparse kernel (spmm_sp.cuh): 0 nothing
    // known, 2 the remainder's size counted, 1 built, -1 unusable (rows too
    // long for the count).
    int sp_state = 0;
    int64_t sp_over = 0;          // entries past the second of their group of four (R's size)
    int sp_tiles = 0, sp_kb = 0;
    uint8_t* sp_wimg = nullptr;   // image form: [sp_tiles][sp_kb] images of kSpWImg bytes
    uint4* sp_cmeta = nullptr;    // compressed form (sparser weights): [sp_kb][128 sp_tiles] metadata,
    uint2* sp_cocc = nullptr;     //   slot masks, value indices and bf16 x3 values (spmm_sp.cuh)
    uint32_t* sp_coff = nullptr;
    uint2* sp_cvals = nullptr;
    int64_t* sp_rptr = nullptr;   // R: [N + 1], null when R is empty
    int32_t* sp_rcol = nullptr;
    float* sp_rval = nullptr;
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

// Adds v * X[m, col] for m < M.  X comes from shared memory (xs[col*MV + m],
// staged once per block) when SMEM, else from global memory through L1.
template <int MV, bool SMEM>
__device__ __forceinline__ void skinny_accum(float (&acc)[MV], int M, int32_t col, float v,
                                             const float* __restrict__ x, int64_t ldx, int64_t K,
                                             const float* xs, bool& bad) {
    if (static_cast<uint32_t>(col) >= static_cast<uint64_t>(K)) {
        bad = true;
        return;
    }
    if constexpr (SMEM) {
        if constexpr (MV == 1) {
            acc[0] = __fmaf_rn(v, xs[col], acc[0]);
        } else if constexpr (MV == 2) {
            const float2 xv = reinterpret_cast<const float2*>(xs)[col];
            acc[0] = __fmaf_rn(v, xv.x, acc[0]);
            acc[1] = __fmaf_rn(v, xv.y, acc[1]);
        } else {
#pragma unroll
            for (int q = 0; q < MV; q += 4) {
                const float4 xv = reinterpret_cast<const float4*>(xs + static_cast<int64_t>(col) * MV)[q / 4];
                acc[q] = __fmaf_rn(v, xv.x, acc[q]);
                acc[q + 1] = __fmaf_rn(v, xv.y, acc[q + 1]);
                acc[q + 2] = __fmaf_rn(v, xv.z, acc[q + 2]);
                acc[q + 3] = __fmaf_rn(v, xv.w, acc[q + 3]);
            }
        }
    } else {
#pragma unroll
        for (int m = 0; m < MV; ++m)
            if (m < M) acc[m] = __fmaf_rn(v, __ldg(x + m * ldx + col), acc[m]);
    }
}

// M <= MV <= 8.  One warp per CSR row; the lanes share the row's nonzeros.
// With SMEM the block first stages X (all M rows, interleaved as xs[k][m],
// zero past M) in shared memory, so the per-nonzero gathers of X hit shared
// memory banks instead of L1 tags; the grid is then persistent (a few blocks
// per SM) so X is staged only once per block.
template <int MV, bool SMEM, int THREADS>
__global__ void __launch_bounds__(THREADS)
    spmm_skinny_kernel(int M, int64_t N, int64_t K, int64_t nnz, const int32_t* __restrict__ indptr,
                       const int32_t* __restrict__ indices, const float* __restrict__ values,
                       const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy,
                       int* err) {
    extern __shared__ __align__(16) float xs[];
    if constexpr (SMEM) {
        const int64_t total = K * MV;
        for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
            const int64_t k = i / MV;
            const int m = static_cast<int>(i % MV);
            xs[i] = (m < M) ? __ldg(x + m * ldx + k) : 0.0f;
        }
        __syncthreads();
    }
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * THREADS) >> 5;
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
            skinny_accum<MV, SMEM>(acc, M, __ldg(indices + j0 + lane), __ldg(values + j0 + lane), x, ldx, K,
                                   xs, bad);
        // Body: 128-bit loads of 4 nonzeros each, four loads per lane issued
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
                    skinny_accum<MV, SMEM>(acc, M, c4[u].x, v4[u].x, x, ldx, K, xs, bad);
                    skinny_accum<MV, SMEM>(acc, M, c4[u].y, v4[u].y, x, ldx, K, xs, bad);
                    skinny_accum<MV, SMEM>(acc, M, c4[u].z, v4[u].z, x, ldx, K, xs, bad);
                    skinny_accum<MV, SMEM>(acc, M, c4[u].w, v4[u].w, x, ldx, K, xs, bad);
                }
            }
        }
        // Tail: fewer than 4 nonzeros.
        if (jb + lane < j1)
            skinny_accum<MV, SMEM>(acc, M, __ldg(indices + jb + lane), __ldg(values + jb + lane), x, ldx, K,
                                   xs, bad);
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

// M = 1.  One warp per CSR row on a persistent grid, X staged once per block
// in shared memory (cp.async when X is 16-byte aligned and K % 4 == 0).  Lane
// l takes the entries ja + 128 (R i + u) + 4 l .. + 3 (u < R) of the row's
// 16-byte-aligned body [ja, jb) as R 128-bit index loads and R value loads
// issued together, so a row of up to 128 R + 6 nonzeros costs one round trip;
// the head [j0, ja) and tail [jb, j1) are single loads.  The latency chain of
// a warp is cut in two places: the first row's loads go out before the block
// waits for X, and each row's indptr pair and first round of the NEXT row are
// loaded before the current row's warp reduction.  CHECK: the CSR is not
// known to be valid (caller-owned arrays), so every index is range-checked
// and indptr clamped.
//
// PEER: the output-channel-sharded form fused with the all-gather of Y
// (pfrt_spmm_allgather).  Rank r computes rows [col0, col0 + N) of the
// gathered output y.  Each value is written to y locally and sent to every
// other rank p in one 8-byte relaxed store of (call number << 32 | value
// bits) into recv_p[parity][col0 + n]: the value and its "ready" mark arrive
// together, so no fence or flag is needed (the low-latency protocol NCCL
// uses for small messages).  After its own rows, each block takes a share of
// the values this rank receives, waits for each to carry the current call
// number and unpacks it into y.  The call number e = state[1] + 1 is read
// once per block; the last block to finish (state[0] counts blocks)
// advances state[1].  recv is used by the parity of e: a rank that has
// finished call e has received everyone's values of e, so nobody can be more
// than one call ahead of a reader, and call e+1 writes the other half.
// A wait that runs out (2 s) sets state[3], so the others stop waiting, and
// reports kDevWaitTimeout.
struct PeerArgs {
    int rank;
    int world;
    int64_t col0;
    float* y;
    uint64_t* recv[PFRT_MAX_PEERS];
    uint32_t* state;
    uint64_t wait_ns;  // limit of each wait on another rank
};

template <int R, int THREADS, bool CHECK, bool PEER = false>
__global__ void __launch_bounds__(THREADS)
    spmm_row1_kernel(int64_t N, int64_t K, int64_t nnz, const int32_t* __restrict__ indptr,
                     const int32_t* __restrict__ indices, const float* __restrict__ values,
                     const float* __restrict__ x, int vec_x, float* __restrict__ y, int* err,
                     const PeerArgs pa = PeerArgs{}) {
    extern __shared__ __align__(16) float xs[];
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * THREADS) >> 5;
    uint32_t epoch = 0;
    __shared__ uint32_t s_epoch;
    if constexpr (PEER) {
        if (threadIdx.x == 0) s_epoch = ld_relaxed_gpu(pa.state + 1) + 1u;
    }
    // Programmatic dependent launch (non-PEER): the CSR of an uploaded weight
    // is immutable, so the first row's index and value loads go out before
    // this grid waits for the previous kernel; X and y follow the wait.  A
    // caller-owned CSR (CHECK) may come from the previous kernel: wait first.
    if constexpr (!PEER) {
        if (threadIdx.x == 0) pdl_launch_dependents();
        if constexpr (CHECK) pdl_wait();
    }
    auto bounds = [&](int64_t r, int32_t& a, int32_t& b) {
        if constexpr (CHECK) {
            int64_t j0, j1;
            row_range(indptr, r, nnz, j0, j1);
            a = static_cast<int32_t>(j0);
            b = static_cast<int32_t>(j1);
        } else {
            a = __ldg(indptr + r);
            b = __ldg(indptr + r + 1);
        }
    };
    // One round: R 16-byte loads of indices and of values from j (a multiple
    // of 4, j < jb); loads past jb repeat j's and are masked at use.
    int4 c4[R];
    float4 v4[R];
    auto load_round = [&](int32_t j, int32_t jb) {
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int32_t jj = (j + 128 * u < jb) ? j + 128 * u : j;
            c4[u] = ldg_nc_v4s32(indices + jj);
            v4[u] = ldg_nc_v4f32(values + jj);
        }
    };
    int64_t n = warp0;
    int32_t j0 = 0, j1 = 0;
    if (n < N) bounds(n, j0, j1);
    int32_t ja = min((j0 + 3) & ~3, j1);
    int32_t jb = ja + ((j1 - ja) & ~3);
    if (ja + 4 * lane < jb) load_round(ja + 4 * lane, jb);
    if constexpr (!PEER && !CHECK) pdl_wait();
    if (vec_x) {
        for (int64_t i = threadIdx.x; i < K / 4; i += THREADS) cp_async_16(xs + 4 * i, x + 4 * i);
        cp_async_commit();
        cp_async_wait_all();
    } else {
        for (int64_t i = threadIdx.x; i < K; i += THREADS) xs[i] = __ldg(x + i);
    }
    __syncthreads();
    if constexpr (PEER) epoch = s_epoch;
    bool bad = false;
    auto gx = [&](int32_t c) -> float {
        if constexpr (CHECK) {
            if (static_cast<uint32_t>(c) >= static_cast<uint64_t>(K)) {
                bad = true;
                return 0.0f;
            }
        }
        return xs[c];
    };
    for (; n < N; n += nwarps) {
        const int64_t nn = n + nwarps;
        int32_t k0 = 0, k1 = 0;
        if (nn < N) bounds(nn, k0, k1);
        float hv = 0.0f, tv = 0.0f;
        int32_t hc = 0, tc = 0;
        if (j0 + lane < ja) {
            hc = __ldg(indices + j0 + lane);
            hv = __ldg(values + j0 + lane);
        }
        if (jb + lane < j1) {
            tc = __ldg(indices + jb + lane);
            tv = __ldg(values + jb + lane);
        }
        float acc = 0.0f;
        for (int32_t j = ja + 4 * lane; j < jb;) {
#pragma unroll
            for (int u = 0; u < R; ++u) {
                if (j + 128 * u < jb) {
                    acc = __fmaf_rn(v4[u].x, gx(c4[u].x), acc);
                    acc = __fmaf_rn(v4[u].y, gx(c4[u].y), acc);
                    acc = __fmaf_rn(v4[u].z, gx(c4[u].z), acc);
                    acc = __fmaf_rn(v4[u].w, gx(c4[u].w), acc);
                }
            }
            j += 128 * R;
            if (j < jb) load_round(j, jb);
        }
        if (j0 + lane < ja) acc = __fmaf_rn(hv, gx(hc), acc);
        if (jb + lane < j1) acc = __fmaf_rn(tv, gx(tc), acc);
        // the next row's first round goes out before this row's reduction
        j0 = k0;
        j1 = k1;
        ja = min((j0 + 3) & ~3, j1);
        jb = ja + ((j1 - ja) & ~3);
        if (nn < N && ja + 4 * lane < jb) load_round(ja + 4 * lane, jb);
#pragma unroll
        for (int o = 16; o; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) {
            if constexpr (PEER) {
                pa.y[pa.col0 + n] = acc;
                const uint64_t msg = (static_cast<uint64_t>(epoch) << 32) | __float_as_uint(acc);
                const int64_t at = static_cast<int64_t>(epoch & 1u) * pa.world * N + pa.col0 + n;
                for (int p = 0; p < pa.world; ++p)
                    if (p != pa.rank)
                        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(pa.recv[p] + at), "l"(msg)
                                     : "memory");
            } else {
                y[n] = acc;
            }
        }
    }
    if (bad) report_error(err, kDevBadIndex);
    if constexpr (PEER) {
        // Unpack this block's share of the values the other ranks send.
        const int64_t incoming = static_cast<int64_t>(pa.world - 1) * N;
        const int64_t share = (incoming + gridDim.x - 1) / gridDim.x;
        const int64_t q0 = static_cast<int64_t>(blockIdx.x) * share;
        const int64_t q1 = q0 + share < incoming ? q0 + share : incoming;
        const uint64_t* box = pa.recv[pa.rank] + static_cast<int64_t>(epoch & 1u) * pa.world * N;
        const uint64_t t0 = global_timer_ns();
        bool ok = true;
        for (int64_t q = q0 + threadIdx.x; q < q1 && ok; q += THREADS) {
            const int64_t p = q / N, i = q - p * N;
            const int64_t src = p < pa.rank ? p : p + 1;  // skip this rank's own slot
            const int64_t at = src * N + i;
            for (uint32_t it = 0;; ++it) {
                uint64_t m;
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(m) : "l"(box + at) : "memory");
                if (static_cast<uint32_t>(m >> 32) == epoch) {
                    pa.y[at] = __uint_as_float(static_cast<uint32_t>(m));
                    break;
                }
                if ((it & 255u) == 255u &&
                    (ld_relaxed_gpu(pa.state + 3) != 0 || global_timer_ns() - t0 > pa.wait_ns)) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) {
            atomicExch(pa.state + 3, 1u);
            report_error(err, kDevWaitTimeout);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(pa.state, 1u) == gridDim.x - 1) {
                pa.state[0] = 0u;
                st_release_gpu(pa.state + 1, epoch);
            }
        }
    }
}

// M > 1 all-gather of the output-channel-sharded SpMM (pfrt_spmm_allgather).
// Each rank writes its column block [rank*ns, rank*ns + ns) of Y into its own
// gathered output y [M][ldy]; the block must also land in every other rank's
// y.  Two ways, chosen per rank and per call:
//   copy:  after the shard's SpMM, peer_push_kernel stores the block into
//          every other rank's y over NVLink;
//   fused: the shard's SpMM is the dense-path GEMM, whose epilogue stores each
//          output tile into every rank's y as it is computed (FEpi's
//          peer_out), so the transfer overlaps the GEMM; peer_ready_kernel runs
//          before the GEMM and peer_push_kernel after it only signals.
// Signal words of rank p (sig[p], mapped by every rank):
//   [kSigReady + q]   the last call at which rank q's y was free (written
//                     by q into every other rank's words);
//   [kSigDone + par]  other ranks that have finished writing p's y in the
//                     calls of parity par.
// Call e = state[1] + 1.  "Ready": this rank declares its y free for e (its
// stream has completed everything before this kernel, the consumers of call
// e - 1's output included) by a release store into every other rank's words,
// then waits until every other rank has declared its own; only then may it
// write into their outputs.  "Done": after its copies (each block: a
// system-scope fence, then one count on this rank's state[2]), the last
// block adds one to every other rank's done count and waits until this
// rank's count reaches world - 1; it resets the count (no rank can add to it
// again before this rank's call e + 2 declares its y free) and publishes e.
// One count per rank and call, whatever each rank's grid, so ranks may take
// different ways.  Waits give up after wait_ns or once state[3] is set,
// which they then set.
constexpr int kSigReady = 0;
constexpr int kSigDone = PFRT_MAX_PEERS;
static_assert(kSigDone + 2 <= PFRT_PEER_SIG_WORDS, "signal words");
constexpr int kPushThreads = 512;

struct PushArgs {
    int rank;
    int world;
    int64_t M, ns, ldy;
    int vec;                         // float4 copies (ns and ldy multiples of 4)
    int copy;                        // 0: the block is already in every output (fused)
    int ready_done;                  // 1: peer_ready_kernel ran for this call
    float* y[PFRT_MAX_PEERS];
    uint32_t* sig[PFRT_MAX_PEERS];
    uint32_t* state;
    uint64_t wait_ns;
};

// Waits until *p reaches `target` (modulo 2^32).  Relaxed system-scope polls,
// then one acquire fence.  False when the wait runs out or *abort is set.
__device__ __forceinline__ bool wait_word_reached(const uint32_t* p, uint32_t target, const uint32_t* abort,
                                                  uint64_t t0, uint64_t limit_ns) {
    for (uint32_t it = 0;; ++it) {
        uint32_t v;
        asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (static_cast<int32_t>(v - target) >= 0) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            return true;
        }
        if ((it & 63u) == 63u) {
            if (ld_relaxed_gpu(abort) != 0) return false;
            if (global_timer_ns() - t0 > limit_ns) return false;
        }
        __nanosleep(32);
    }
}

// The "ready" exchange of call e by threads [0, world) of one block; returns
// false (on every thread of the block) when a wait gave up.
__device__ __forceinline__ bool peer_ready(const PushArgs& a, uint32_t e, bool declare, int* s_fail) {
    const int tid = threadIdx.x;
    const uint64_t t0 = global_timer_ns();
    if (declare && tid < a.world && tid != a.rank) st_release_sys(a.sig[tid] + kSigReady + a.rank, e);
    if (tid < a.world && tid != a.rank &&
        !wait_word_reached(a.sig[a.rank] + kSigReady + tid, e, a.state + 3, t0, a.wait_ns))
        *s_fail = 1;
    __syncthreads();
    return *s_fail == 0;
}

__global__ void __launch_bounds__(32) peer_ready_kernel(const PushArgs a, int* err) {
    __shared__ int s_fail;
    if (threadIdx.x == 0) s_fail = ld_relaxed_gpu(a.state + 3) != 0 ? 1 : 0;
    __syncthreads();
    const uint32_t e = ld_relaxed_gpu(a.state + 1) + 1u;
    if (!peer_ready(a, e, true, &s_fail) && threadIdx.x == 0) {
        atomicExch(a.state + 3, 1u);
        report_error(err, kDevWaitTimeout);
    }
}

__global__ void __launch_bounds__(kPushThreads) peer_push_kernel(const PushArgs a, int* err) {
    __shared__ uint32_t s_epoch;
    __shared__ int s_fail;
    const int tid = threadIdx.x;
    if (tid == 0) {
        s_epoch = ld_relaxed_gpu(a.state + 1) + 1u;
        s_fail = ld_relaxed_gpu(a.state + 3) != 0 ? 1 : 0;
    }
    __syncthreads();
    const uint32_t e = s_epoch;
    bool ok = s_fail == 0;
    if (!a.ready_done) ok = peer_ready(a, e, blockIdx.x == 0, &s_fail);
    if (ok && a.copy) {
        const int64_t col0 = static_cast<int64_t>(a.rank) * a.ns;
        const float* src = a.y[a.rank];
        const int64_t stride = static_cast<int64_t>(gridDim.x) * kPushThreads;
        if (a.vec) {
            const int64_t q = a.ns / 4, total = a.M * q;
            for (int64_t i = static_cast<int64_t>(blockIdx.x) * kPushThreads + tid; i < total; i += stride) {
                const int64_t m = i / q;
                const int64_t off = m * a.ldy + col0 + 4 * (i - m * q);
                const float4 v = *reinterpret_cast<const float4*>(src + off);
                for (int p = 0; p < a.world; ++p)
                    if (p != a.rank) *reinterpret_cast<float4*>(a.y[p] + off) = v;
            }
        } else {
            const int64_t total = a.M * a.ns;
            for (int64_t i = static_cast<int64_t>(blockIdx.x) * kPushThreads + tid; i < total; i += stride) {
                const int64_t m = i / a.ns;
                const int64_t off = m * a.ldy + col0 + (i - m * a.ns);
                const float v = src[off];
                for (int p = 0; p < a.world; ++p)
                    if (p != a.rank) a.y[p][off] = v;
            }
        }
    }
    __syncthreads();
    if (tid != 0) return;
    // A block that could not copy says so before it is counted, so the last
    // block cannot report the output complete.
    if (!ok) {
        atomicExch(a.state + 3, 1u);
        report_error(err, kDevWaitTimeout);
    }
    // The block's stores (ordered before this thread by the barrier) before
    // its count; the last block's fence then covers every block's stores.
    __threadfence_system();
    if (atomicAdd(a.state + 2, 1u) != gridDim.x - 1) return;
    __threadfence_system();
    uint32_t* mine = a.sig[a.rank];
    bool fine = ld_relaxed_gpu(a.state + 3) == 0;
    if (fine) {
        for (int p = 0; p < a.world; ++p)
            if (p != a.rank)
                asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.sig[p] + kSigDone + (e & 1u)) : "memory");
        fine = wait_word_reached(mine + kSigDone + (e & 1u), static_cast<uint32_t>(a.world - 1), a.state + 3,
                                 global_timer_ns(), a.wait_ns);
    }
    if (!fine) {
        atomicExch(a.state + 3, 1u);
        report_error(err, kDevWaitTimeout);
    } else {
        atomicExch(mine + kSigDone + (e & 1u), 0u);
    }
    a.state[2] = 0u;
    st_release_gpu(a.state + 1, e);
}

// Streaming form of the skinny kernel, for a CSR uploaded with
// pfrt_csr_create.  Warp w owns the contiguous rows [part[w], part[w+1]),
// chosen on the host so that every warp gets about the same number of
// nonzeros; their nonzeros are one contiguous range of the CSR arrays, which
// the warp streams in 256-entry stages (two 128-bit index loads and two value
// loads per lane), always loading stage s+1 before it works on stage s.
// Rows are reduced segment by segment: the part of a row inside a stage is
// summed over the warp with shuffles and added to the row's running sum, and a
// row is written when its last stage is done.
template <int MV, bool SMEM, int THREADS>
__global__ void __launch_bounds__(THREADS)
    spmm_stream_kernel(int M, int64_t K, const int32_t* __restrict__ indptr,
                       const int32_t* __restrict__ indices, const float* __restrict__ values,
                       const int32_t* __restrict__ part, const float* __restrict__ x, int64_t ldx,
                       float* __restrict__ y, int64_t ldy, int* err) {
    extern __shared__ __align__(16) float xs[];
    if constexpr (SMEM) {
        const int64_t total = K * MV;
        for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
            const int64_t k = i / MV;
            const int m = static_cast<int>(i % MV);
            xs[i] = (m < M) ? __ldg(x + m * ldx + k) : 0.0f;
        }
        __syncthreads();
    }
    const int lane = threadIdx.x & 31;
    const int64_t w = (static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x) >> 5;
    const int32_t rb = __ldg(part + w), re = __ldg(part + w + 1);
    if (rb >= re) return;
    const int32_t lo = __ldg(indptr + rb), hi = __ldg(indptr + re);
    bool bad = false;
    // Row ends of rows base .. base+31, one per lane.
    int32_t base = rb;
    int32_t bnd = (base + 1 + lane <= re) ? __ldg(indptr + base + 1 + lane) : hi;
    int32_t row = rb;
    int32_t row_start = lo;
    int32_t row_end = __shfl_sync(0xffffffffu, bnd, 0);
    float racc[MV];
#pragma unroll
    for (int m = 0; m < MV; ++m) racc[m] = 0.0f;

    auto load_stage = [&](int32_t s, int4 (&c)[2], float4 (&v)[2]) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int32_t g = s + 128 * h + 4 * lane;
            if (g < hi) {
                c[h] = __ldg(reinterpret_cast<const int4*>(indices + g));
                v[h] = __ldg(reinterpret_cast<const float4*>(values + g));
            } else {
                c[h] = make_int4(0, 0, 0, 0);
                v[h] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
    int32_t s0 = lo & ~3;
    int4 ci[2];
    float4 vi[2];
    load_stage(s0, ci, vi);
    bool done = false;
    while (!done) {
        const int32_t s1 = s0 + 256;
        int4 cn[2];
        float4 vn[2];
        if (s1 < hi) load_stage(s1, cn, vn);
        // Products of the lane's 8 entries (entry e: j = s0 + 128*(e/4) + 4*lane + e%4).
        float pv[8][MV];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int h = e >> 2, q = e & 3;
            const int32_t col = (q == 0) ? ci[h].x : (q == 1) ? ci[h].y : (q == 2) ? ci[h].z : ci[h].w;
            const float v = (q == 0) ? vi[h].x : (q == 1) ? vi[h].y : (q == 2) ? vi[h].z : vi[h].w;
            const int32_t j = s0 + 128 * h + 4 * lane + q;
            const bool live = (j >= lo && j < hi);
            const bool ok = static_cast<uint32_t>(col) < static_cast<uint64_t>(K);
            if (live && !ok) bad = true;
#pragma unroll
            for (int m = 0; m < MV; ++m) {
                float xm = 0.0f;
                if (live && ok) {
                    if constexpr (SMEM) xm = xs[static_cast<int64_t>(col) * MV + m];
                    else xm = (m < M) ? __ldg(x + m * ldx + col) : 0.0f;
                }
                pv[e][m] = (live && ok) ? __fmul_rn(v, xm) : 0.0f;
            }
        }
        // Segments of this stage: the rows that end in it, then the row that continues.
        while (true) {
            const int32_t seg_lo = max(row_start, s0), seg_hi = min(row_end, s1);
            float sum[MV];
#pragma unroll
            for (int m = 0; m < MV; ++m) sum[m] = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int32_t j = s0 + 128 * (e >> 2) + 4 * lane + (e & 3);
                if (j >= seg_lo && j < seg_hi) {
#pragma unroll
                    for (int m = 0; m < MV; ++m) sum[m] = __fadd_rn(sum[m], pv[e][m]);
                }
            }
#pragma unroll
            for (int m = 0; m < MV; ++m) {
                float t = sum[m];
#pragma unroll
                for (int o = 16; o; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
                racc[m] = __fadd_rn(racc[m], t);
            }
            if (row_end > s1) break;  // the row continues in the next stage
            if (lane < M) {
                float out = racc[0];
#pragma unroll
                for (int m = 1; m < MV; ++m)
                    if (lane == m) out = racc[m];
                y[static_cast<int64_t>(lane) * ldy + row] = out;
            }
#pragma unroll
            for (int m = 0; m < MV; ++m) racc[m] = 0.0f;
            ++row;
            if (row >= re) {
                done = true;
                break;
            }
            row_start = row_end;
            if (row - base >= 32) {
                base += 32;
                bnd = (base + 1 + lane <= re) ? __ldg(indptr + base + 1 + lane) : hi;
            }
            row_end = __shfl_sync(0xffffffffu, bnd, row - base);
        }
        if (done || s1 >= hi) {
            // Rows left after the last nonzero are empty: write zeros.
            for (; !done && row < re; ++row)
                if (lane < M) y[static_cast<int64_t>(lane) * ldy + row] = 0.0f;
            break;
        }
        s0 = s1;
        ci[0] = cn[0];
        ci[1] = cn[1];
        vi[0] = vn[0];
        vi[1] = vn[1];
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

// Mid-batch kernel (M > 8): one block per row group, over the column-blocked
// copy of the CSR.  The groups are contiguous row ranges chosen on the host
// (about equal nonzeros; at most kXtRows rows and kXtEntMax nonzeros of any
// one column chunk), so the nonzeros of a group in chunk c are one
// contiguous range of `cent`, and its row pointers one range of cptr[c].
// Per chunk, a producer warp brings into a two-stage shared-memory ring:
//   - the tile X^T[c*KT .. +KT][m0 .. m0+MT] by TMA,
//   - the group's entries (local column, value) by a 1-D bulk copy,
//   - the group's row pointers by a 1-D bulk copy,
// all completing on the stage's mbarrier.  The compute warps then work from
// shared memory only: warp w owns rows w, w + kXtWarps, ... of the group;
// lane l owns MV consecutive rows of X (columns of Y), so each nonzero is one
// broadcast read of its (column, value) and one MV-wide read of X^T[k].
// Outputs are staged through shared memory and stored along n.
// The local columns come from the host-side blocking of a validated CSR
// (column - 256 * chunk, in [0, 256) by construction); the kernel masks them
// to the tile instead of checking them, so no entry can address shared memory
// outside the chunk's X tile.
constexpr int kTileKT = 256;    // columns of X (rows of X^T) per chunk, = the column-blocked copy's block
// 15 compute warps + the producer: 16 warps, 4 on each of the SM's four
// schedulers, so each thread may hold up to 128 registers (a scheduler's
// 16 K registers over 4 warps).  With 16 compute warps the fifth warp on one
// scheduler capped threads at 96 registers and the MV = 2 instance spilled
// to local memory, through the L1 pipe this kernel is bound by.
constexpr int kXtWarps = 15;    // compute warps per block
constexpr int kXtRowsPerWarp = 8;
constexpr int kXtRows = kXtWarps * kXtRowsPerWarp;
constexpr int kXtEntMax = 4096; // nonzeros of one group in one chunk
constexpr int kXtOffMax = kXtRows + 8;

template <int MV>
struct XtCfg {
    static constexpr int MT = 32 * MV;
    static constexpr int XS_BYTES = 4 * MT * kTileKT;
    static constexpr int ENT_BYTES = 8 * (kXtEntMax + 2);
    static constexpr int OFF_BYTES = 4 * kXtOffMax;
    static constexpr int STAGE_BYTES = (XS_BYTES + ENT_BYTES + OFF_BYTES + 1023) / 1024 * 1024;
    static constexpr int SMEM = 2 * STAGE_BYTES + 128 + 1024;
    static_assert(4 * MT * (kXtRows + 1) <= STAGE_BYTES, "output staging fits in a stage");
    static_assert(OFF_BYTES % 16 == 0 && ENT_BYTES % 16 == 0 && XS_BYTES % 1024 == 0, "alignment");
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

template <int MV>
__global__ void __launch_bounds__((kXtWarps + 1) * 32, 1)
    spmm_xtile_kernel(const __grid_constant__ CUtensorMap tmx, int M, int mtiles, int64_t N, int nchunks,
                      const int32_t* __restrict__ gpart, const int32_t* __restrict__ cptr,
                      const uint2* __restrict__ cent, float* __restrict__ y, int64_t ldy, int* err) {
    using Cfg = XtCfg<MV>;
    constexpr int MT = Cfg::MT;
    extern __shared__ uint8_t xsm_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(xsm_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + 2 * Cfg::STAGE_BYTES);
    uint64_t* empty = full + 2;
    int32_t* meta = reinterpret_cast<int32_t*>(empty + 2);  // [2][2]: first entry, first row pointer
    volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = static_cast<int>(blockIdx.x % mtiles);
    const int64_t g = blockIdx.x / mtiles;
    const int m0 = mt * MT;
    const int32_t r0 = __ldg(gpart + g), r1 = __ldg(gpart + g + 1);
    const int nr = r1 - r0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kXtWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    float acc[kXtRowsPerWarp][MV];
#pragma unroll
    for (int i = 0; i < kXtRowsPerWarp; ++i)
#pragma unroll
        for (int v = 0; v < MV; ++v) acc[i][v] = 0.0f;

    if (warp == kXtWarps) {
        if (lane == 0) {
            tma_prefetch_desc(&tmx);
            bool ok = true;
            int issued = 0;
            for (int c = 0; c < nchunks; ++c) {
                const int st = c & 1;
                const uint32_t ph = static_cast<uint32_t>(c >> 1) & 1u;
                if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                const int32_t* cp = cptr + static_cast<int64_t>(c) * (N + 1);
                const int32_t e0 = __ldg(cp + r0), e1 = __ldg(cp + r1);
                const int32_t elo = e0 & ~1, ehi = (e1 + 1) & ~1;
                const int64_t olo = (static_cast<int64_t>(c) * (N + 1) + r0) & ~int64_t{3};
                const int64_t ohi = (static_cast<int64_t>(c) * (N + 1) + r1 + 1 + 3) & ~int64_t{3};
                uint8_t* sb = base + st * Cfg::STAGE_BYTES;
                meta[2 * st] = elo;
                meta[2 * st + 1] = static_cast<int32_t>(olo - static_cast<int64_t>(c) * (N + 1));
                const uint32_t ebytes = 8u * static_cast<uint32_t>(ehi - elo);
                const uint32_t obytes = 4u * static_cast<uint32_t>(ohi - olo);
                mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(Cfg::XS_BYTES) + ebytes + obytes);
                tma_load_2d(sb, &tmx, &full[st], m0, c * kTileKT);
                if (ebytes) bulk_g2s(sb + Cfg::XS_BYTES, cent + elo, ebytes, &full[st]);
                bulk_g2s(sb + Cfg::XS_BYTES + Cfg::ENT_BYTES, cptr + olo, obytes, &full[st]);
                ++issued;
            }
            if (!ok) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
            }
            // Everything issued has been consumed by the compute warps, or,
            // after an abort, is waited for here before the block may exit.
            const int zero = 0;
            for (int c = (issued > 2 ? issued - 2 : 0); c < issued && !ok; ++c)
                mbar_wait(&full[c & 1], static_cast<uint32_t>(c >> 1) & 1u, &zero);
        }
    } else {
        for (int c = 0; c < nchunks; ++c) {
            const int st = c & 1;
            const uint32_t ph = static_cast<uint32_t>(c >> 1) & 1u;
            if (!mbar_wait(&full[st], ph, abort_flag)) {
                if (lane == 0) {
                    *abort_flag = 1;
                    report_error(err, kDevWaitTimeout);
                }
                break;
            }
            const uint8_t* sb = base + st * Cfg::STAGE_BYTES;
            const float* xs = reinterpret_cast<const float*>(sb);
            const uint2* ents = reinterpret_cast<const uint2*>(sb + Cfg::XS_BYTES);
            const int32_t* offs = reinterpret_cast<const int32_t*>(sb + Cfg::XS_BYTES + Cfg::ENT_BYTES);
            const int32_t elo = meta[2 * st], olo = meta[2 * st + 1];
#pragma unroll
            for (int i = 0; i < kXtRowsPerWarp; ++i) {
                const int rl = warp + i * kXtWarps;
                if (rl < nr) {
                    const int32_t e0 = offs[r0 + rl - olo] - elo, e1 = offs[r0 + rl + 1 - olo] - elo;
                    int32_t e = e0;
                    for (; e + 3 < e1; e += 4) {
                        uint2 en[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) en[u] = ents[e + u];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const uint32_t k = en[u].x & static_cast<uint32_t>(kTileKT - 1);
                            const float v = __uint_as_float(en[u].y);
                            if constexpr (MV == 2) {
                                const float2 xv = reinterpret_cast<const float2*>(xs + k * MT)[lane];
                                acc[i][0] = __fmaf_rn(v, xv.x, acc[i][0]);
                                acc[i][1] = __fmaf_rn(v, xv.y, acc[i][1]);
                            } else {
                                acc[i][0] = __fmaf_rn(v, xs[k * MT + lane], acc[i][0]);
                            }
                        }
                    }
                    for (; e < e1; ++e) {
                        const uint2 en = ents[e];
                        const uint32_t k = en.x & static_cast<uint32_t>(kTileKT - 1);
                        const float v = __uint_as_float(en.y);
#pragma unroll
                        for (int q = 0; q < MV; ++q) acc[i][q] = __fmaf_rn(v, xs[k * MT + lane * MV + q], acc[i][q]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    }
    __syncthreads();
    // Output: stage [MT rows of X][nr CSR rows] in stage 0, then store along n.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    float* ys = reinterpret_cast<float*>(base);
    const int ld = nr + 1;
    if (warp < kXtWarps) {
#pragma unroll
        for (int i = 0; i < kXtRowsPerWarp; ++i) {
            const int rl = warp + i * kXtWarps;
            if (rl < nr)
#pragma unroll
                for (int q = 0; q < MV; ++q) ys[(lane * MV + q) * ld + rl] = acc[i][q];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < MT * nr; e += blockDim.x) {
        const int m = e / nr, i = e % nr;
        if (m0 + m < M && !*abort_flag) y[static_cast<int64_t>(m0 + m) * ldy + r0 + i] = ys[m * ld + i];
    }
}

// Dense tf32 split of a CSR matrix: hi[n][k] = tf32(v), lo[n][k] = v - hi
// for every stored (n, k, v); the buffers are zero beforehand.  Warp per row.
__global__ void csr_scatter_split_kernel(int64_t N, int64_t Kpad, const int32_t* __restrict__ indptr,
                                         const int32_t* __restrict__ indices, const float* __restrict__ values,
                                         float* __restrict__ hi, float* __restrict__ lo) {
    const int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    for (int32_t j = indptr[n] + lane; j < indptr[n + 1]; j += 32) {
        const float v = values[j];
        uint32_t h;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
        const int64_t at = n * Kpad + indices[j];
        hi[at] = __uint_as_float(h);
        lo[at] = __fsub_rn(v, __uint_as_float(h));
    }
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

// Device order of the nonzeros inside each row.  The row kernel gives lane l
// the entries ja + 128 t + 4 l + q (q = 0..3) of a row's 16-byte-aligned body
// [ja, jb), ja = j0 rounded up to a multiple of 4, and one shared-memory
// gather of X covers the 32 entries with the same (t, q): a "group".  Entries
// whose columns share a bank (col mod 32) in one group serialise that gather.
// The body's entries are therefore dealt out in bank order over the groups,
// one slot of every group before the next slot of any, so the entries of one
// bank fall into different groups while there are groups left.  The set of
// (column, value) pairs of every row is unchanged; only the order in which
// the kernels sum them differs.
void bank_order_rows(const std::vector<int32_t>& ip, std::vector<int32_t>& ix, std::vector<float>& v) {
    const int64_t N = static_cast<int64_t>(ip.size()) - 1;
    std::vector<int32_t> slot, order, tmp_i;
    std::vector<float> tmp_v;
    for (int64_t n = 0; n < N; ++n) {
        const int32_t j0 = ip[n], j1 = ip[n + 1];
        const int32_t ja = std::min((j0 + 3) & ~3, j1);
        const int32_t jb = ja + ((j1 - ja) & ~3);
        const int32_t L = jb - ja;
        if (L <= 4) continue;
        const int32_t groups = 4 * ((L + 127) / 128);
        slot.clear();
        for (int32_t l = 0; l < 32; ++l)
            for (int32_t g = 0; g < groups; ++g) {
                const int32_t p = 128 * (g / 4) + 4 * l + (g % 4);
                if (p < L) slot.push_back(p);
            }
        int32_t cnt[33] = {0};
        for (int32_t k = 0; k < L; ++k) ++cnt[(ix[ja + k] & 31) + 1];
        for (int b = 0; b < 32; ++b) cnt[b + 1] += cnt[b];
        order.assign(static_cast<size_t>(L), 0);
        for (int32_t k = 0; k < L; ++k) order[cnt[ix[ja + k] & 31]++] = k;
        tmp_i.assign(ix.begin() + ja, ix.begin() + jb);
        tmp_v.assign(v.begin() + ja, v.begin() + jb);
        for (int32_t k = 0; k < L; ++k) {
            ix[ja + slot[k]] = tmp_i[order[k]];
            v[ja + slot[k]] = tmp_v[order[k]];
        }
    }
}

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
                     const float* x, int64_t ldx, float* y, int64_t ldy, cudaStream_t s,
                     bool validated = false) {
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
        const int Mi = static_cast<int>(M);
        const int MV = (M == 1) ? 1 : (M == 2) ? 2 : (M <= 4) ? 4 : 8;
        const size_t xs_bytes = sizeof(float) * static_cast<size_t>(K) * MV;
        const char* no_smem = std::getenv("PFRT_SPMM_NO_SMEM");
        // Staging X costs one coalesced copy per block out of L2: worth it
        // when the gathers it replaces cost more.  Each gathered X element
        // moves a 32-byte L2 sector (M of them per nonzero, from separate
        // rows of X when M > 1).
        const int per_sm = static_cast<int>(std::max<size_t>(1, std::min<size_t>(4, (224 * 1024) / (xs_bytes + 1024))));
        const int64_t smem_blocks = std::min<int64_t>(ceil_div(N, 16), int64_t{per_sm} * ctx->num_sms);
        const bool pays = (M >= 2) || (32.0 * nnz >= static_cast<double>(smem_blocks) * xs_bytes);
        const bool smem = xs_bytes <= 96 * 1024 && K > 0 && pays && !(no_smem && *no_smem == '1');
        const size_t shm = smem ? xs_bytes : 0;
        // One persistent wave: exactly the blocks that are resident at once.
        int occ = 1;
        {
            cudaError_t oe;
            switch (MV) {
                case 1: oe = smem ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<1, true, 512>, 512, shm)
                                  : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<1, false, kSpmmThreads>, kSpmmThreads, 0); break;
                case 2: oe = smem ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<2, true, 512>, 512, shm)
                                  : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<2, false, kSpmmThreads>, kSpmmThreads, 0); break;
                case 4: oe = smem ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<4, true, 512>, 512, shm)
                                  : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<4, false, kSpmmThreads>, kSpmmThreads, 0); break;
                default: oe = smem ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<8, true, 512>, 512, shm)
                                   : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmm_skinny_kernel<8, false, kSpmmThreads>, kSpmmThreads, 0); break;
            }
            if (oe != cudaSuccess) return cuda_fail(oe, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
            occ = std::max(1, occ);
        }
        // M = 1 with X in shared memory: the row kernel (batched loads, next
        // row prefetched).  Its 32-bit entry arithmetic needs nnz well inside
        // int32.
        const char* row1_env = std::getenv("PFRT_SPMM_ROW1");
        if (MV == 1 && smem && nnz <= INT32_MAX - 4096 && !(row1_env && *row1_env == '0')) {
            const int vec_x = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (K & 3) == 0) ? 1 : 0;
            int occ1 = 1;
            cudaError_t oe = validated
                ? cudaFuncSetAttribute(spmm_row1_kernel<4, 512, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(shm))
                : cudaFuncSetAttribute(spmm_row1_kernel<4, 512, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(shm));
            if (oe == cudaSuccess)
                oe = validated ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, spmm_row1_kernel<4, 512, false>, 512, shm)
                               : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, spmm_row1_kernel<4, 512, true>, 512, shm);
            if (oe != cudaSuccess) return cuda_fail(oe, "spmm_row1_kernel occupancy");
            const int b1 = static_cast<int>(std::max<int64_t>(
                1, std::min<int64_t>(ceil_div(N, 16), int64_t{std::max(1, occ1)} * ctx->num_sms)));
            cudaLaunchConfig_t lc{};
            cudaLaunchAttribute la[1];
            lc.gridDim = dim3(static_cast<unsigned>(b1));
            lc.blockDim = dim3(512);
            lc.dynamicSmemBytes = shm;
            lc.stream = s;
            lc.numAttrs = pdl_attr(la);
            lc.attrs = la;
            const PeerArgs none{};
            if (validated)
                PFRT_CUDA_TRY(cudaLaunchKernelEx(&lc, spmm_row1_kernel<4, 512, false>, N, K, nnz, indptr, indices,
                                                 values, x, vec_x, y, ctx->d_err, none));
            else
                PFRT_CUDA_TRY(cudaLaunchKernelEx(&lc, spmm_row1_kernel<4, 512, true>, N, K, nnz, indptr, indices,
                                                 values, x, vec_x, y, ctx->d_err, none));
            return PFRT_OK;
        }
        const int tpb = smem ? 512 : kSpmmThreads;
        const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(N, tpb / 32),
                                                                                   int64_t{occ} * ctx->num_sms)));
        (void)smem_blocks;
        (void)max_blocks;
#define PFRT_SKINNY(MVV)                                                                              \
    do {                                                                                              \
        if (smem) {                                                                                   \
            PFRT_CUDA_TRY(cudaFuncSetAttribute(spmm_skinny_kernel<MVV, true, 512>,                    \
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,          \
                                               static_cast<int>(shm)));                              \
            spmm_skinny_kernel<MVV, true, 512><<<blocks, 512, shm, s>>>(                              \
                Mi, N, K, nnz, indptr, indices, values, x, ldx, y, ldy, ctx->d_err);                  \
        } else {                                                                                      \
            spmm_skinny_kernel<MVV, false, kSpmmThreads><<<blocks, kSpmmThreads, 0, s>>>(             \
                Mi, N, K, nnz, indptr, indices, values, x, ldx, y, ldy, ctx->d_err);                  \
        }                                                                                             \
    } while (0)
        if (MV == 1) PFRT_SKINNY(1);
        else if (MV == 2) PFRT_SKINNY(2);
        else if (MV == 4) PFRT_SKINNY(4);
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

// Row partition for `warps` warps with about equal cost per warp, cost of a
// row = its nonzeros + 16 (per-row overhead).  part[w] is non-decreasing,
// part[0] = 0, part[warps] = N.
pfrt_status ensure_partition(pfrt_csr* w, int64_t warps, cudaStream_t s) {
    if (w->part && w->part_warps == warps) return PFRT_OK;
    const int64_t N = w->N;
    std::vector<int32_t> part(static_cast<size_t>(warps + 1));
    const double total = static_cast<double>(w->nnz) + 16.0 * static_cast<double>(N);
    int64_t r = 0;
    for (int64_t k = 0; k <= warps; ++k) {
        const double target = total * static_cast<double>(k) / static_cast<double>(warps);
        while (r < N && static_cast<double>(w->host_indptr[r]) + 16.0 * static_cast<double>(r) < target) ++r;
        part[k] = static_cast<int32_t>(r);
    }
    part[warps] = static_cast<int32_t>(N);
    if (w->part) cudaFree(w->part);
    w->part = nullptr;
    w->part_warps = 0;
    PFRT_CUDA_TRY(cudaMalloc(&w->part, sizeof(int32_t) * part.size()));
    PFRT_CUDA_TRY(cudaMemcpyAsync(w->part, part.data(), sizeof(int32_t) * part.size(), cudaMemcpyHostToDevice, s));
    PFRT_CUDA_TRY(cudaStreamSynchronize(s));
    w->part_warps = warps;
    return PFRT_OK;
}

// Dense copy of W for the tensor-core path, built once on the device.
pfrt_status ensure_dense(pfrt_ctx* ctx, pfrt_csr* w, cudaStream_t s) {
    if (w->dense) return PFRT_OK;
    const int64_t kpad = static_cast<int64_t>(align_up(static_cast<size_t>(w->K), 32));
    const size_t bytes = sizeof(float) * static_cast<size_t>(w->N) * kpad;
    float *hi = nullptr, *lo = nullptr;
    cudaError_t e = cudaMalloc(&hi, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&lo, bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(hi, 0, bytes, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(lo, 0, bytes, s);
    if (e != cudaSuccess) {
        if (hi) cudaFree(hi);
        if (lo) cudaFree(lo);
        return cuda_fail(e, "SpMM dense copy");
    }
    csr_scatter_split_kernel<<<static_cast<unsigned>(ceil_div(w->N * 32, 256)), 256, 0, s>>>(
        w->N, kpad, w->indptr, w->indices, w->values, hi, lo);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cudaFree(hi);
        cudaFree(lo);
        return cuda_fail(e, "csr_scatter_split_kernel");
    }
    return fweight_from_device_split(ctx, w->N, w->K, hi, lo, &w->dense);
}

// Compressed form of W for the tensor-core kernel (spmm_tc.cuh), built once
// on the device.  A row that stores a column twice (the CSR sums them; the
// compressed form has one slot per position) leaves the form unusable and
// the other paths serve the weight.
pfrt_status ensure_tcfmt(pfrt_csr* w, cudaStream_t s) {
    if (w->tc_state != 0) return PFRT_OK;
    const int64_t kb_total = ceil_div(std::max<int64_t>(w->K, 1), kTcBK);
    const int64_t npad = ceil_div(std::max<int64_t>(w->N, 1), kTcWRows) * kTcWRows;
    const size_t words = static_cast<size_t>(kb_total) * static_cast<size_t>(npad);
    int* dup = nullptr;
    cudaError_t e = cudaMalloc(&w->tc_mask, sizeof(uint32_t) * words);
    if (e == cudaSuccess) e = cudaMalloc(&w->tc_off, sizeof(uint32_t) * words);
    // 64 entries of slack: the producers prefetch up to 32 entries past the
    // first value of the k-block they expand.
    if (e == cudaSuccess) e = cudaMalloc(&w->tc_vals, sizeof(float2) * static_cast<size_t>(w->nnz + 64));
    if (e == cudaSuccess) e = cudaMalloc(&dup, sizeof(int));
    if (e == cudaSuccess) e = cudaMemsetAsync(w->tc_mask, 0, sizeof(uint32_t) * words, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(dup, 0, sizeof(int), s);
    const unsigned row_blocks = static_cast<unsigned>(ceil_div(std::max<int64_t>(w->N, 1) * 32, 256));
    if (e == cudaSuccess) {
        tc_mask_kernel<<<row_blocks, 256, 0, s>>>(w->N, npad, w->indptr, w->indices, w->tc_mask, dup);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) {
        tc_off_kernel<<<static_cast<unsigned>(ceil_div(npad, 256)), 256, 0, s>>>(
            w->N, npad, static_cast<int>(kb_total), w->indptr, w->nnz, w->tc_mask, w->tc_off);
        e = cudaGetLastError();
    }
    int h_dup = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h_dup, dup, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && !h_dup) {
        tc_vals_kernel<<<row_blocks, 256, 0, s>>>(w->N, npad, w->indptr, w->indices, w->values, w->tc_mask,
                                                  w->tc_off, w->tc_vals);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    if (dup) cudaFree(dup);
    if (e != cudaSuccess || h_dup) {
        cudaFree(w->tc_mask);
        cudaFree(w->tc_off);
        cudaFree(w->tc_vals);
        w->tc_mask = w->tc_off = nullptr;
        w->tc_vals = nullptr;
        w->tc_state = -1;
        return e != cudaSuccess ? cuda_fail(e, "SpMM compressed form") : PFRT_OK;
    }
    w->tc_npad = npad;
    w->tc_state = 1;
    return PFRT_OK;
}

// Stream-K schedule of the tensor-core kernel: the k-blocks of all units
// split evenly over at most one CTA per SM.
TcSched tc_schedule(const pfrt_ctx* ctx, const pfrt_csr* w, int64_t M) {
    TcSched sc{};
    sc.n_wtiles = static_cast<int>(ceil_div(std::max<int64_t>(w->N, 1), kTcWRows));
    sc.n_xslabs = M <= 64 ? 1 : static_cast<int>(ceil_div(M, 128));
    sc.kb_total = static_cast<int>(ceil_div(std::max<int64_t>(w->K, 1), kTcBK));
    sc.total = static_cast<int64_t>(sc.n_wtiles) * sc.n_xslabs * sc.kb_total;
    sc.per_cta = ceil_div(sc.total, static_cast<int64_t>(ctx->num_sms));
    return sc;
}

// Expected time of the tensor-core kernel, fitted to measurements on
// 4096^2 and 8192^2 weights at 90 % sparsity: per k-block of a CTA's range
// 0.59 us (stacked, 8 MMAs of 128 x 128 x 8) or 0.82 us (wide, 12 MMAs),
// plus the X split, the fix-up of the shared units and the launches.
double tc_time(const pfrt_ctx* ctx, const pfrt_csr* w, int64_t M) {
    const TcSched sc = tc_schedule(ctx, w, M);
    return static_cast<double>(sc.per_cta) * (M <= 64 ? 0.59e-6 : 0.82e-6) + 12.0e-6;
}

// Y = X W^T on the tensor cores from W's compressed form (spmm_tc.cuh).
pfrt_status run_spmm_tc(pfrt_ctx* ctx, pfrt_csr* w, int64_t M, const float* x, int64_t ldx, float* y,
                        int64_t ldy, cudaStream_t s) {
    pfrt_status st = ensure_tcfmt(w, s);
    if (st) return st;
    if (w->tc_state != 1) return PFRT_ERR_UNSUPPORTED;
    const int64_t kpad = static_cast<int64_t>(align_up(static_cast<size_t>(w->K), kTcBK));
    const TcSched sc = tc_schedule(ctx, w, M);
    const int64_t grid = ceil_div(sc.total, sc.per_cta);
    const bool stacked = M <= 64;
    const size_t xbytes = align_up(sizeof(float) * static_cast<size_t>(M * kpad), 256);
    const size_t pbytes = sizeof(float) * static_cast<size_t>(2 * grid * kTcTileElems);
    void* scr = nullptr;
    st = scratch(ctx, 2 * xbytes + pbytes, &scr);
    if (st) return st;
    float* xhi = static_cast<float*>(scr);
    float* xlo = reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + xbytes);
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + 2 * xbytes);
    st = split_tf32_kmajor(x, M, w->K, ldx, xhi, xlo, kpad, s);
    if (st) return st;
    CUtensorMap tmh, tml;
    st = make_tmap_2d(&tmh, xhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, kpad, M, kpad * 4, kTcBK, 64);
    if (st == PFRT_OK)
        st = make_tmap_2d(&tml, xlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, kpad, M, kpad * 4, kTcBK, 64);
    if (st) return st;
    TcArgs a{};
    a.mask = w->tc_mask;
    a.off = w->tc_off;
    a.vals = w->tc_vals;
    a.npad = w->tc_npad;
    a.M = static_cast<int>(M);
    a.N = static_cast<int>(w->N);
    a.y = y;
    a.ldy = ldy;
    a.partial = part;
    auto kern = stacked ? spmm_tc_kernel<true> : spmm_tc_kernel<false>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kTcSmemBytes;
    cfg.stream = s;
    cfg.numAttrs = pdl_attr(attr);
    cfg.attrs = attr;
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tmh, tml, sc, a, ctx->d_err));
    if (grid > 1) {
        cudaLaunchConfig_t rc{};
        rc.gridDim = dim3(static_cast<unsigned>(grid - 1), static_cast<unsigned>((stacked ? 64 : 128) * kTcWRows / 1024));
        rc.blockDim = dim3(256);
        rc.stream = s;
        rc.numAttrs = pdl_attr(attr);
        rc.attrs = attr;
        PFRT_CUDA_TRY(cudaLaunchKernelEx(&rc, tc_fixup_kernel, sc, static_cast<const float*>(part),
                                         static_cast<int>(M), static_cast<int>(w->N), stacked ? 64 : 128, y,
                                         ldy));
    }
    return PFRT_OK;
}

// Size of W's remainder R for the structured-sparse kernel (spmm_sp.cuh):
// the entries past the second of every aligned group of four columns of a
// row, counted once on the device (the cost model needs it before any image
// is built).
pfrt_status ensure_sp_count(pfrt_csr* w, cudaStream_t s) {
    if (w->sp_state != 0) return PFRT_OK;
    w->sp_state = -1;
    if (w->N <= 0 || w->K <= 0) return PFRT_OK;
    const int groups = static_cast<int>(ceil_div(w->K, 4));
    const int64_t row_bytes = 4 * static_cast<int64_t>(groups);
    if (row_bytes > 96 * 1024) return PFRT_OK;  // one row's column marks must fit in shared memory
    const int wpb = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(8, (96 * 1024) / row_bytes)));
    const size_t smem = static_cast<size_t>(wpb) * static_cast<size_t>(row_bytes);
    unsigned long long* over = nullptr;
    cudaError_t e = cudaMalloc(&over, sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemsetAsync(over, 0, sizeof(unsigned long long), s);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(sp_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e == cudaSuccess) {
        sp_count_kernel<<<static_cast<unsigned>(ceil_div(w->N, wpb)), 32 * wpb, smem, s>>>(w->N, groups, w->indptr,
                                                                                         w->indices, over);
        e = cudaGetLastError();
    }
    unsigned long long h_over = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h_over, over, sizeof(h_over), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (over) cudaFree(over);
    if (e != cudaSuccess) return cuda_fail(e, "SpMM 2:4 count");
    w->sp_over = static_cast<int64_t>(h_over);
    w->sp_state = 2;
    return PFRT_OK;
}

// Which form of W24 the structured-sparse kernel reads.  The compressed form
// (28 bytes per row and k-block plus 8 per kept entry) is chosen where it is
// under a quarter of the images' size (W24 under ~5 % dense: 95 %-sparse
// weights and sparser), the images would not stay in L2 (over ~96 MB; a
// smaller weight's images are re-read from L2 by every X slab, which beats
// expanding the compressed form again) and a W tile's values of one k-block
// fit the kernel's value slot on average.  Both kernels are bound by shared
// memory bandwidth, so the compressed form's smaller HBM traffic pays only
// where the images are mostly empty: on B200, 8192^2 at 95 %: M = 64 55
// (compressed) against 55 us (images), M = 256 171 against 174 us; at 90 %
// the images win (M = 64 58 against 59, M = 256 181 against 182, M = 1024
// 676 against 715 us).  Whether every run fits is checked when the form is
// built.  PFRT_SPMM_SP_FORM = image|compressed forces one (read when the
// form is built; a forced compressed form reads runs that do not fit from
// global memory, slowly).
bool sp_form_forced(bool& cform) {
    const char* f = std::getenv("PFRT_SPMM_SP_FORM");
    if (!f) return false;
    if (std::strcmp(f, "image") == 0) cform = false;
    else if (std::strcmp(f, "compressed") == 0) cform = true;
    else return false;
    return true;
}

bool sp_use_cform(const pfrt_csr* w) {
    const double tiles = static_cast<double>(ceil_div(w->N, 128)), KB = static_cast<double>(ceil_div(w->K, kSpBK));
    const double kept = static_cast<double>(std::max<int64_t>(w->nnz - w->sp_over, 0));
    if (kept >= 4.0e9) return false;  // 32-bit value indices
    bool cform = false;
    if (sp_form_forced(cform)) return cform;
    const double i_bytes = tiles * KB * kSpWImg, c_bytes = 28.0 * 128.0 * tiles * KB + 8.0 * kept;
    return i_bytes > 96.0e6 && c_bytes < 0.25 * i_bytes && 8.0 * kept / (tiles * KB) < 0.85 * kSpVSlot;
}

// W's structured-sparse form, built once on the device from a dense scratch
// copy that is freed again: the 2:4 part W24 as images, the remainder R as a
// CSR (each row's entries in column order, so the result does not depend on
// how the build was scheduled).
pfrt_status ensure_sp(pfrt_csr* w, cudaStream_t s) {
    pfrt_status st = ensure_sp_count(w, s);
    if (st) return st;
    if (w->sp_state != 2) return PFRT_OK;
    const int tiles = static_cast<int>(ceil_div(w->N, 128));
    const int KB = static_cast<int>(ceil_div(w->K, kSpBK));
    const int64_t npad = static_cast<int64_t>(tiles) * 128, kpad = static_cast<int64_t>(KB) * kSpBK;
    const size_t wd_bytes = sizeof(float) * static_cast<size_t>(npad) * static_cast<size_t>(kpad);
    bool cform = sp_use_cform(w);
    bool cform_forced = false;
    {
        bool f = false;
        cform_forced = sp_form_forced(f) && f;
    }
    const size_t nrk = static_cast<size_t>(npad) * static_cast<size_t>(KB);  // (k-block, row) pairs
    float* wd = nullptr;
    uint8_t* img = nullptr;
    uint4* cmeta = nullptr;
    uint2* cocc = nullptr;
    uint32_t* coff = nullptr;
    uint2* cvals = nullptr;
    int32_t* rcount = nullptr;
    int64_t* rptr = nullptr;
    int32_t* rcol = nullptr;
    float* rval = nullptr;
    const unsigned row_blocks = static_cast<unsigned>(ceil_div(w->N * 32, 256));
    cudaError_t e = cudaMalloc(&wd, wd_bytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(wd, 0, wd_bytes, s);
    if (e == cudaSuccess) {
        sp_scatter_kernel<<<row_blocks, 256, 0, s>>>(w->N, kpad, w->indptr, w->indices, w->values, wd);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && cform) {
        // Two passes over the scratch: counts (with each row's metadata and
        // slot mask) per (k-block, row), a host scan into value indices,
        // then the values.  A run (one W tile's values of one k-block)
        // longer than the kernel's value slot sends the weight to the images
        // unless the form is forced.
        const unsigned cblocks = static_cast<unsigned>(ceil_div(static_cast<int64_t>(nrk), 256));
        std::vector<uint32_t> hoff(nrk + 1);
        e = cudaMalloc(&cmeta, sizeof(uint4) * nrk);
        if (e == cudaSuccess) e = cudaMalloc(&cocc, sizeof(uint2) * nrk);
        if (e == cudaSuccess) e = cudaMalloc(&coff, sizeof(uint32_t) * (nrk + 1));
        if (e == cudaSuccess) {
            sp_cform_kernel<true><<<cblocks, 256, 0, s>>>(npad, KB, kpad, wd, coff, cmeta, cocc, nullptr, nullptr);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpyAsync(hoff.data(), coff, sizeof(uint32_t) * nrk, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        uint64_t total = 0;
        for (size_t i = 0; e == cudaSuccess && i < nrk; ++i) {
            const uint32_t c = hoff[i];
            hoff[i] = static_cast<uint32_t>(total);
            total += c;
        }
        hoff[nrk] = static_cast<uint32_t>(total);
        uint64_t longest = 0;
        for (size_t r = 0; r < nrk; r += 128) {
            const uint64_t b0 = (uint64_t{hoff[r]} * 8u) & ~uint64_t{15};
            const uint64_t b1 = (uint64_t{hoff[r + 128]} * 8u + 15u) & ~uint64_t{15};
            longest = std::max(longest, b1 - b0);
        }
        if (e == cudaSuccess && longest > static_cast<uint64_t>(kSpVSlot) && !cform_forced) {
            cudaFree(cmeta);
            cudaFree(cocc);
            cudaFree(coff);
            cmeta = nullptr;
            cocc = nullptr;
            coff = nullptr;
            cform = false;
        }
        const size_t vbytes = ((8 * total + 15) & ~size_t{15}) + 16;  // copies end on a 16-byte boundary
        if (e == cudaSuccess && cform) e = cudaMalloc(&cvals, vbytes);
        if (e == cudaSuccess && cform)
            e = cudaMemcpyAsync(coff, hoff.data(), sizeof(uint32_t) * (nrk + 1), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess && cform) {
            sp_cform_kernel<false><<<cblocks, 256, 0, s>>>(npad, KB, kpad, wd, nullptr, nullptr, nullptr, coff, cvals);
            e = cudaGetLastError();
        }
        // hoff is read by the copy above: wait before it goes out of scope.
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    if (e == cudaSuccess && !cform) {
        const size_t img_bytes = static_cast<size_t>(tiles) * static_cast<size_t>(KB) * kSpWImg;
        e = cudaMalloc(&img, img_bytes);
        if (e == cudaSuccess) e = cudaMemsetAsync(img, 0, img_bytes, s);
        const int64_t threads = static_cast<int64_t>(tiles) * KB * 128 * kSpSteps;
        if (e == cudaSuccess) {
            sp_pack_w_kernel<<<static_cast<unsigned>(ceil_div(threads, 256)), 256, 0, s>>>(tiles, KB, kpad, wd, img);
            e = cudaGetLastError();
        }
    }
    if (e == cudaSuccess && w->sp_over > 0) {
        std::vector<int32_t> hcount(static_cast<size_t>(w->N));
        std::vector<int64_t> hptr(static_cast<size_t>(w->N) + 1, 0);
        e = cudaMalloc(&rcount, sizeof(int32_t) * hcount.size());
        if (e == cudaSuccess) {
            sp_remainder_kernel<false><<<row_blocks, 256, 0, s>>>(w->N, kpad, wd, rcount, nullptr, nullptr, nullptr);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(hcount.data(), rcount, sizeof(int32_t) * hcount.size(), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        for (size_t i = 0; e == cudaSuccess && i < hcount.size(); ++i) hptr[i + 1] = hptr[i] + hcount[i];
        const int64_t nr = hptr.back();
        if (e == cudaSuccess && nr > 0) {
            e = cudaMalloc(&rptr, sizeof(int64_t) * hptr.size());
            if (e == cudaSuccess) e = cudaMalloc(&rcol, sizeof(int32_t) * static_cast<size_t>(nr));
            if (e == cudaSuccess) e = cudaMalloc(&rval, sizeof(float) * static_cast<size_t>(nr));
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(rptr, hptr.data(), sizeof(int64_t) * hptr.size(), cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) {
                sp_remainder_kernel<true><<<row_blocks, 256, 0, s>>>(w->N, kpad, wd, nullptr, rptr, rcol, rval);
                e = cudaGetLastError();
            }
        }
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (wd) cudaFree(wd);
    if (rcount) cudaFree(rcount);
    if (e != cudaSuccess) {
        if (img) cudaFree(img);
        if (cmeta) cudaFree(cmeta);
        if (cocc) cudaFree(cocc);
        if (coff) cudaFree(coff);
        if (cvals) cudaFree(cvals);
        if (rptr) cudaFree(rptr);
        if (rcol) cudaFree(rcol);
        if (rval) cudaFree(rval);
        return cuda_fail(e, "SpMM structured-sparse form");
    }
    w->sp_wimg = img;
    w->sp_cmeta = cmeta;
    w->sp_cocc = cocc;
    w->sp_coff = coff;
    w->sp_cvals = cvals;
    w->sp_rptr = rptr;
    w->sp_rcol = rcol;
    w->sp_rval = rval;
    w->sp_tiles = tiles;
    w->sp_kb = KB;
    w->sp_state = 1;
    return PFRT_OK;
}

TcSched sp_schedule(const pfrt_ctx* ctx, const pfrt_csr* w, int64_t M) {
    TcSched sc{};
    sc.n_wtiles = w->sp_tiles;
    sc.n_xslabs = static_cast<int>(ceil_div(M, kSpSlab));
    sc.kb_total = w->sp_kb;
    sc.total = static_cast<int64_t>(sc.n_wtiles) * sc.n_xslabs * sc.kb_total;
    sc.per_cta = ceil_div(sc.total, static_cast<int64_t>(ctx->num_sms));
    return sc;
}

// Y = X W^T on the structured-sparse tensor cores (spmm_sp.cuh): X's bf16
// images, the kernel, and the fix-up of units split between CTAs.
pfrt_status run_spmm_sp(pfrt_ctx* ctx, pfrt_csr* w, int64_t M, const float* x, int64_t ldx, float* y,
                        int64_t ldy, cudaStream_t s) {
    pfrt_status st = ensure_sp(w, s);
    if (st) return st;
    if (w->sp_state != 1) return PFRT_ERR_UNSUPPORTED;
    if (ldx < w->K) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: row stride too small");
    const TcSched sc = sp_schedule(ctx, w, M);
    const int64_t grid = ceil_div(sc.total, sc.per_cta);
    const size_t xbytes = align_up(static_cast<size_t>(sc.n_xslabs) * static_cast<size_t>(sc.kb_total) * kSpXImg, 256);
    const size_t pbytes = align_up(sizeof(float) * static_cast<size_t>(2 * grid * kTcTileElems), 256);
    const int64_t mpad = ceil_div(M, kSpSlab) * kSpSlab;  // X^T's row stride for the remainder
    const size_t tbytes = w->sp_rptr ? sizeof(float) * static_cast<size_t>(w->K) * static_cast<size_t>(mpad) : 0;
    void* scr = nullptr;
    st = scratch(ctx, xbytes + pbytes + tbytes, &scr);
    if (st) return st;
    uint8_t* ximg = static_cast<uint8_t*>(scr);
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + xbytes);
    float* xt = reinterpret_cast<float*>(static_cast<uint8_t*>(scr) + xbytes + pbytes);

    cudaLaunchAttribute attr[1];
    {
        const int64_t threads = static_cast<int64_t>(sc.n_xslabs) * sc.kb_total * kSpSlab * 16;
        cudaLaunchConfig_t pc{};
        pc.gridDim = dim3(static_cast<unsigned>(ceil_div(threads, 256)));
        pc.blockDim = dim3(256);
        pc.stream = s;
        pc.numAttrs = pdl_attr(attr);
        pc.attrs = attr;
        PFRT_CUDA_TRY(cudaLaunchKernelEx(&pc, sp_pack_x_kernel, x, M, w->K, ldx, sc.n_xslabs, sc.kb_total, ximg,
                                         w->sp_rptr ? xt : static_cast<float*>(nullptr), mpad));
    }
    SpArgs a{};
    a.wimg = w->sp_wimg;
    a.ximg = ximg;
    a.cmeta = w->sp_cmeta;
    a.cocc = w->sp_cocc;
    a.coff = w->sp_coff;
    a.cvals = w->sp_cvals;
    a.npad = static_cast<int64_t>(w->sp_tiles) * kTcWRows;
    a.M = static_cast<int>(M);
    a.N = static_cast<int>(w->N);
    a.y = y;
    a.ldy = ldy;
    a.partial = part;
    const bool cform = w->sp_cmeta != nullptr;
    auto kern = cform ? spmm_sp_kernel<true> : spmm_sp_kernel<false>;
    const int smem = cform ? kSpSmemBytesX : kSpSmemBytes;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(cform ? kSpThreadsX : kSpThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.numAttrs = pdl_attr(attr);
    cfg.attrs = attr;
    PFRT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, sc, a, ctx->d_err));
    if (grid > 1) {
        cudaLaunchConfig_t rc{};
        rc.gridDim = dim3(static_cast<unsigned>(grid - 1), static_cast<unsigned>(kSpSlab * kTcWRows / 1024));
        rc.blockDim = dim3(256);
        rc.stream = s;
        rc.numAttrs = pdl_attr(attr);
        rc.attrs = attr;
        PFRT_CUDA_TRY(cudaLaunchKernelEx(&rc, tc_fixup_kernel, sc, static_cast<const float*>(part),
                                         static_cast<int>(M), static_cast<int>(w->N), kSpSlab, y, ldy));
    }
    if (w->sp_rptr) {
        cudaLaunchConfig_t qc{};
        qc.gridDim = dim3(static_cast<unsigned>(ceil_div(w->N, 32)), static_cast<unsigned>(mpad / kSpSlab));
        qc.blockDim = dim3(1024);
        qc.stream = s;
        qc.numAttrs = pdl_attr(attr);
        qc.attrs = attr;
        PFRT_CUDA_TRY(cudaLaunchKernelEx(&qc, sp_remainder_add_kernel, static_cast<const float*>(xt), mpad, M, w->N,
                                         static_cast<const int64_t*>(w->sp_rptr), static_cast<const int32_t*>(w->sp_rcol),
                                         static_cast<const float*>(w->sp_rval), y, ldy));
    }
    return PFRT_OK;
}

// Expected time of the structured-sparse kernel, fitted to 2:4 weights of
// 4096^2 and 8192^2 at M = 64 ... 1024 on B200: 1.4 us per k-block of a
// CTA's range (each moves 104 KB from L2: the kernel runs at the L2 -> SM
// rate, about twice its MMA time) plus 9 us of X packing, fix-up and
// launches; the remainder's kernel ~3 us plus ~0.5 ps per (entry of R, row
// of X).  Once X's images outgrow L2 (above ~96 MB: M > ~2000 at K = 8192)
// every W tile re-reads them from HBM (8192^2 at 90 %, M = 8192: 7.97 ms
// against the dense path's 6.15 ms), charged at 6 TB/s.
double sp_time(const pfrt_ctx* ctx, const pfrt_csr* w, int64_t M) {
    const int64_t tiles = ceil_div(std::max<int64_t>(w->N, 1), 128), kb = ceil_div(std::max<int64_t>(w->K, 1), kSpBK);
    const int64_t slabs = ceil_div(M, kSpSlab);
    const int64_t total = tiles * slabs * kb;
    const double per_cta = std::ceil(static_cast<double>(total) / static_cast<double>(ctx->num_sms));
    const double r_gathers = static_cast<double>(w->sp_over) * static_cast<double>(slabs * kSpSlab);
    const double x_bytes = static_cast<double>(slabs) * static_cast<double>(kb) * kSpXImg;
    const double x_rereads = x_bytes > 96.0e6 ? static_cast<double>(tiles - 1) * x_bytes / 6.0e12 : 0.0;
    return per_cta * 1.4e-6 + 9.0e-6 + x_rereads + (w->sp_over > 0 ? 3.0e-6 + r_gathers * 5.0e-13 : 0.0);
}

template <int MV, bool SMEM>
pfrt_status launch_stream(pfrt_ctx* ctx, pfrt_csr* w, int M, const float* x, int64_t ldx, float* y,
                          int64_t ldy, size_t shm, cudaStream_t s) {
    constexpr int THREADS = SMEM ? 512 : 256;
    auto kern = spmm_stream_kernel<MV, SMEM, THREADS>;
    if (SMEM)
        PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shm)));
    // Exactly the blocks that are resident at once: the partition gives every
    // warp of this grid its own rows, so no warp waits for a second wave.
    int occ = 0;
    PFRT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, THREADS, shm));
    occ = std::max(1, std::min(occ, SMEM ? 2 : 8));
    const int64_t blocks = int64_t{occ} * ctx->num_sms;
    pfrt_status st = ensure_partition(w, blocks * (THREADS / 32), s);
    if (st) return st;
    kern<<<static_cast<unsigned>(blocks), THREADS, shm, s>>>(M, w->K, w->indptr, w->indices, w->values, w->part,
                                                             x, ldx, y, ldy, ctx->d_err);
    PFRT_CHECK_LAUNCH("spmm_stream_kernel");
    return PFRT_OK;
}

pfrt_status run_spmm_stream(pfrt_ctx* ctx, pfrt_csr* w, int64_t M, const float* x, int64_t ldx,
                            float* y, int64_t ldy, cudaStream_t s) {
    if (!x || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: null pointer");
    if (ldx < w->K || ldy < w->N) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: row stride too small");
    if (w->N == 0 || M == 0) return PFRT_OK;
    const int Mi = static_cast<int>(M);
    const int MV = (M == 1) ? 1 : (M == 2) ? 2 : (M <= 4) ? 4 : 8;
    const size_t xs_bytes = sizeof(float) * static_cast<size_t>(w->K) * MV;
    const char* no_smem = std::getenv("PFRT_SPMM_NO_SMEM");
    // Staging X costs one copy per block: worth it when the per-nonzero
    // gathers it replaces (M of them, from separate rows of X when M > 1)
    // cost more than that copy.
    const bool pays = (M >= 2) || (8.0 * w->nnz >= 3.0 * 2.0 * ctx->num_sms * static_cast<double>(xs_bytes));
    const bool smem = xs_bytes <= 96 * 1024 && w->K > 0 && pays && !(no_smem && *no_smem == '1');
    const size_t shm = smem ? xs_bytes : 0;
    switch (MV) {
        case 1: return smem ? launch_stream<1, true>(ctx, w, Mi, x, ldx, y, ldy, shm, s)
                            : launch_stream<1, false>(ctx, w, Mi, x, ldx, y, ldy, 0, s);
        case 2: return smem ? launch_stream<2, true>(ctx, w, Mi, x, ldx, y, ldy, shm, s)
                            : launch_stream<2, false>(ctx, w, Mi, x, ldx, y, ldy, 0, s);
        case 4: return smem ? launch_stream<4, true>(ctx, w, Mi, x, ldx, y, ldy, shm, s)
                            : launch_stream<4, false>(ctx, w, Mi, x, ldx, y, ldy, 0, s);
        default: return smem ? launch_stream<8, true>(ctx, w, Mi, x, ldx, y, ldy, shm, s)
                             : launch_stream<8, false>(ctx, w, Mi, x, ldx, y, ldy, 0, s);
    }
}

// Row groups of spmm_xtile_kernel: contiguous rows, closed when adding the
// next row would exceed kXtRows rows, kXtEntMax nonzeros in some column chunk,
// or the per-group share of nonzeros (total / min_groups, so that there are
// at least about min_groups groups to fill the SMs).  A single row with more
// than kXtEntMax nonzeros in one chunk cannot be placed (returns false).
bool ensure_xt_groups(pfrt_csr* w, int64_t min_groups, cudaStream_t s, pfrt_status* st_out) {
    *st_out = PFRT_OK;
    if (w->xt_part) return true;
    const int64_t N = w->N;
    const int C = w->nchunks;
    // Aim a little under min_groups so that rounding does not spill one group
    // into a second wave.
    const double target = std::max(1.0, 1.04 * static_cast<double>(w->nnz) /
                                             static_cast<double>(std::max<int64_t>(1, min_groups)));
    std::vector<int32_t> part{0};
    std::vector<int32_t> cnt(static_cast<size_t>(C), 0);
    int64_t rows = 0, nz = 0;
    for (int64_t r = 0; r < N; ++r) {
        int64_t rnz = w->host_indptr[r + 1] - w->host_indptr[r];
        bool fits = rows < kXtRows && (rows == 0 || static_cast<double>(nz + rnz) <= target);
        for (int c = 0; c < C && fits; ++c) {
            const int32_t* cp = w->host_cptr.data() + static_cast<size_t>(c) * (N + 1);
            fits = cnt[c] + (cp[r + 1] - cp[r]) <= kXtEntMax;
        }
        if (!fits) {
            part.push_back(static_cast<int32_t>(r));
            std::fill(cnt.begin(), cnt.end(), 0);
            rows = 0;
            nz = 0;
        }
        for (int c = 0; c < C; ++c) {
            const int32_t* cp = w->host_cptr.data() + static_cast<size_t>(c) * (N + 1);
            cnt[c] += cp[r + 1] - cp[r];
            if (cnt[c] > kXtEntMax) return false;
        }
        ++rows;
        nz += rnz;
    }
    part.push_back(static_cast<int32_t>(N));
    cudaError_t e = cudaMalloc(&w->xt_part, sizeof(int32_t) * part.size());
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(w->xt_part, part.data(), sizeof(int32_t) * part.size(), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        if (w->xt_part) cudaFree(w->xt_part);
        w->xt_part = nullptr;
        *st_out = cuda_fail(e, "SpMM row groups");
        return false;
    }
    w->xt_groups = static_cast<int64_t>(part.size()) - 1;
    return true;
}

template <int MV>
pfrt_status launch_xtile(pfrt_ctx* ctx, const pfrt_csr* w, const CUtensorMap& tmx, int64_t M, float* y,
                         int64_t ldy, cudaStream_t s) {
    using Cfg = XtCfg<MV>;
    auto kern = spmm_xtile_kernel<MV>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    const int64_t mtiles = ceil_div(M, Cfg::MT);
    const int64_t blocks = mtiles * w->xt_groups;
    if (blocks > INT32_MAX) return fail(PFRT_ERR_UNSUPPORTED, "SpMM: too many tiles");
    kern<<<static_cast<unsigned>(blocks), (kXtWarps + 1) * 32, Cfg::SMEM, s>>>(
        tmx, static_cast<int>(M), static_cast<int>(mtiles), w->N, w->nchunks, w->xt_part, w->cptr, w->cent, y, ldy,
        ctx->d_err);
    PFRT_CHECK_LAUNCH("spmm_xtile_kernel");
    return PFRT_OK;
}

// M > 8 on an uploaded CSR through spmm_xtile_kernel.  Returns
// PFRT_ERR_UNSUPPORTED (nothing launched) when some row has more than
// kXtEntMax nonzeros in one 256-column chunk.
pfrt_status run_spmm_xtile(pfrt_ctx* ctx, pfrt_csr* w, int64_t M, const float* x, int64_t ldx, float* y,
                           int64_t ldy, cudaStream_t s) {
    if (M > INT32_MAX - 256) return fail(PFRT_ERR_UNSUPPORTED, "SpMM: M too large");
    if (!x || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: null pointer");
    if (ldx < w->K || ldy < w->N) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: row stride too small");
    if (w->N == 0 || M == 0) return PFRT_OK;
    if (w->K == 0) return run_spmm(ctx, M, w->N, w->K, w->nnz, w->indptr, w->indices, w->values, x, ldx, y, ldy, s);
    pfrt_status st;
    if (!ensure_xt_groups(w, ctx->num_sms, s, &st))
        return st ? st : fail(PFRT_ERR_UNSUPPORTED, "SpMM: a row is too dense for the tiled kernel");
    const int mv = (M <= 32) ? 1 : 2;
    const int64_t mt = 32 * mv;
    // X^T [K][Mpad], Mpad a multiple of the tile height (zero padded).
    const int64_t mpad = static_cast<int64_t>(align_up(static_cast<size_t>(M), static_cast<size_t>(mt)));
    void* scr = nullptr;
    st = scratch(ctx, sizeof(float) * mpad * w->K, &scr);
    if (st) return st;
    float* xt = static_cast<float*>(scr);
    dim3 tb(32, 8);
    dim3 tg(static_cast<unsigned>(ceil_div(w->K, 32)), static_cast<unsigned>(ceil_div(mpad, 32)));
    transpose_pad_kernel<<<tg, tb, 0, s>>>(x, M, w->K, ldx, xt, mpad);
    PFRT_CHECK_LAUNCH("transpose_pad_kernel");
    CUtensorMap tmx;
    st = make_tmap_2d_plain(&tmx, xt, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, static_cast<uint64_t>(mpad),
                            static_cast<uint64_t>(w->K), static_cast<uint64_t>(mpad) * 4, static_cast<uint32_t>(mt),
                            kTileKT);
    if (st) return st;
    return mv == 1 ? launch_xtile<1>(ctx, w, tmx, M, y, ldy, s) : launch_xtile<2>(ctx, w, tmx, M, y, ldy, s);
}

// The kernel choice of pfrt_spmm on an uploaded CSR (the context's device
// current, `s` the stream).  M = 1, 2: one warp per row measured fastest;
// M = 3..8: the streaming kernel (its register pipeline pays once each
// nonzero feeds 4-8 rows).  M > 8: the tiled CSR kernel (spmm_xtile_kernel)
// or a 3xTF32 tensor-core GEMM on a dense copy of W made once (8 bytes per
// element of W, capped at 8 GiB), whichever the cost model below expects to
// be faster.  Both estimates are fits to B200 measurements (8192^2 and
// 4096^2 at 90-99 % sparsity, M = 16..256): per 32*MV-row tile of X the
// tiled kernel costs ~1.25 us (MV = 1) or ~1.1 us (MV = 2) per 256-column
// chunk plus ~13.3 or ~12.7 ps per nonzero (it is bound by the shared-memory
// pipe, not by DRAM); the GEMM the larger of reading the dense copy at
// ~5.5 TB/s and its tensor work, plus ~12 us.  The dense copy wins down to
// ~6-7 % density at M <= 64; the tiled kernel serves sparser weights.
// PFRT_SPMM_TILED / PFRT_SPMM_DENSE = 0|1 override the choice.
// A sharded call's output: when the dense path runs and the block is large
// enough, its GEMM stores the block into every rank's output as well (after
// the "ready" exchange), and *fused says so.
struct ShardOut {
    const pfrt_peer_set* peers;
    int64_t ns;
    bool* fused;
};
pfrt_status launch_ready(pfrt_ctx* ctx, const pfrt_peer_set* peers, int64_t M, int64_t ns, cudaStream_t s);

pfrt_status spmm_uploaded(pfrt_ctx* ctx, pfrt_csr* w, int64_t M, const float* x, int64_t ldx, float* y,
                          int64_t ldy, cudaStream_t s, const ShardOut* shard = nullptr) {
    const char* rowwarp = std::getenv("PFRT_SPMM_ROWWARP");
    const char* stream_env = std::getenv("PFRT_SPMM_STREAM");
    const bool want_stream = (stream_env && *stream_env == '1') ||
                             (M >= 3 && M <= 8 && !(rowwarp && *rowwarp == '1'));
    if (M >= 1 && M <= 8 && want_stream) return run_spmm_stream(ctx, w, M, x, ldx, y, ldy, s);
    if (M <= 8)
        return run_spmm(ctx, M, w->N, w->K, w->nnz, w->indptr, w->indices, w->values, x, ldx, y, ldy, s,
                        /*validated=*/true);
    if (!x || !y) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: null pointer");
    if (ldx < w->K || ldy < w->N) return fail(PFRT_ERR_INVALID_ARGUMENT, "SpMM: row stride too small");
    const char* tiled_env = std::getenv("PFRT_SPMM_TILED");
    const char* dense_env = std::getenv("PFRT_SPMM_DENSE");
    const double Nd = static_cast<double>(w->N), Kd = static_cast<double>(w->K), Md = static_cast<double>(M);
    const double dense_bytes = 8.0 * Nd * static_cast<double>(align_up(w->K, 32));
    const bool dense_ok = w->N > 0 && w->K > 0 && dense_bytes <= 8.0 * (1ull << 30);
    const double mv = (M <= 32) ? 1.0 : 2.0;
    const double mtiles = std::ceil(Md / (32.0 * mv));
    const double per_chunk = mv == 1.0 ? 1.25e-6 : 1.1e-6, per_nnz = mv == 1.0 ? 13.3e-12 : 12.7e-12;
    const double t_tiled = mtiles * (per_chunk * static_cast<double>(w->nchunks) + per_nnz * static_cast<double>(w->nnz)) *
                           (148.0 / static_cast<double>(ctx->num_sms));
    const double t_dense = std::max((dense_bytes + 8.0 * Md * Kd) / 5.5e12, 6.0 * Md * Nd * Kd / 6.0e14) + 12.0e-6;
    bool use_dense = dense_ok && t_dense < t_tiled;
    if (dense_env && *dense_env) use_dense = dense_ok && *dense_env == '1';
    if (tiled_env && *tiled_env) use_dense = use_dense && *tiled_env == '0';
    // The tensor-core kernel on W's compressed form: the dense path's
    // arithmetic without reading a dense copy of W.
    const char* tc_env = std::getenv("PFRT_SPMM_TC");
    const bool tc_ok = w->N > 0 && w->K > 0 && w->tc_state >= 0 &&
                       M <= (int64_t{1} << 30) / std::max<int64_t>(w->N, 1);
    // Chosen for up to 256 rows of X: above that the dense copy's Gemm was
    // as fast or faster (8192^2 at 90 %: M = 512 362 against ~400 us,
    // M = 1024 708 against 728 us), and once X's hi/lo split outgrows L2
    // every W tile re-reads it from HBM (M = 8192: 7.2 ms against 5.9 ms).
    // Within 10 % of the dense path it is still preferred: it reads 8 bytes
    // per nonzero instead of 8 per element of W and holds no dense copy.
    // PFRT_SPMM_TC = 0|1 forces it off or on (any M); PFRT_SPMM_DENSE or
    // PFRT_SPMM_TILED set without it chooses among the other paths only.
    bool use_tc = tc_ok && M <= 256 && !(dense_env && *dense_env) && !(tiled_env && *tiled_env) &&
                  tc_time(ctx, w, M) < std::min(t_tiled, dense_ok ? 1.1 * t_dense : 1e30);
    if (tc_env && *tc_env) use_tc = tc_ok && *tc_env == '1';
    pfrt_status st;
    // The structured-sparse tensor cores, for weights with 2:4 structure
    // along K (checked once per weight, on the first call that could use
    // them): half the MMA work of the dense product, W read in compressed
    // form.  PFRT_SPMM_SP = 0|1 forces it off or on (on: where W is 2:4).
    const char* sp_env = std::getenv("PFRT_SPMM_SP");
    const bool sp_forced = sp_env && *sp_env;
    const bool sp_free = !(dense_env && *dense_env) && !(tiled_env && *tiled_env) && !(tc_env && *tc_env);
    if ((sp_forced ? *sp_env == '1' : (M >= 16 && sp_free)) && w->sp_state == 0) {
        st = ensure_sp_count(w, s);
        if (st) return st;
    }
    const bool sp_ok = w->sp_state > 0 && w->N > 0 && w->K > 0 && M <= (int64_t{1} << 30) / std::max<int64_t>(w->N, 1);
    bool use_sp = sp_ok && M >= 16 && sp_free &&
                  sp_time(ctx, w, M) < std::min({t_tiled, dense_ok ? t_dense : 1e30, tc_ok ? tc_time(ctx, w, M) : 1e30});
    if (sp_forced) use_sp = sp_ok && *sp_env == '1';
    if (use_sp) {
        st = run_spmm_sp(ctx, w, M, x, ldx, y, ldy, s);
        if (st != PFRT_ERR_UNSUPPORTED) return st;  // else W is not 2:4 along K
    }
    if (use_tc) {
        st = run_spmm_tc(ctx, w, M, x, ldx, y, ldy, s);
        if (st != PFRT_ERR_UNSUPPORTED) return st;  // else the form is unusable for this weight
    }
    if (use_dense) {
        st = ensure_dense(ctx, w, s);
        if (st) return st;
        // Sharded, on request (PFRT_PEER_FUSE=1): the epilogue also writes
        // every other rank's output, so the all-gather overlaps the GEMM.
        // Off by default: each epilogue thread owns one output row, so its
        // remote stores are 16-byte pieces of 32 different rows per warp
        // instruction, and over NVLink that ran slower than the coalesced copy
        // after the GEMM (4 GPUs, 8192^2 at 90 %: M = 1024 429 us fused
        // against 268 us copied; M = 8192 2.40 ms against 1.88 ms).
        const char* fuse_env = std::getenv("PFRT_PEER_FUSE");
        const bool fuse = shard && shard->peers->world > 1 && fuse_env && *fuse_env == '1';
        if (fuse) {
            const pfrt_peer_set* ps = shard->peers;
            st = launch_ready(ctx, ps, M, shard->ns, s);
            if (st) return st;
            float* py[PFRT_MAX_PEERS];
            int n = 0;
            for (int p = 0; p < ps->world; ++p)
                if (p != ps->rank) py[n++] = ps->y_peer[p] + static_cast<int64_t>(ps->rank) * shard->ns;
            st = gemm_f32_strided(ctx, M, x, ldx, w->dense, y, ldy, s, py, n);
            if (st == PFRT_OK) *shard->fused = true;
            return st;
        }
        return gemm_f32_strided(ctx, M, x, ldx, w->dense, y, ldy, s);
    }
    if (!(tiled_env && *tiled_env == '0')) {
        st = run_spmm_xtile(ctx, w, M, x, ldx, y, ldy, s);
        if (st != PFRT_ERR_UNSUPPORTED) return st;  // else a row too dense for the tile: the wide kernel
    }
    return run_spmm(ctx, M, w->N, w->K, w->nnz, w->indptr, w->indices, w->values, x, ldx, y, ldy, s,
                    /*validated=*/true);
}

uint64_t peer_wait_ns() {
    const char* v = std::getenv("PFRT_PEER_WAIT_MS");
    const long ms = (v && *v) ? std::atol(v) : 0;
    return ms > 0 ? static_cast<uint64_t>(ms) * 1000000ull : kWaitLimitNs;
}

// The checks every call on a peer set makes; M > 1 also needs the mapped
// outputs and signal words.
pfrt_status check_peer_set(const pfrt_peer_set* peers, int64_t M, const char* who) {
    const std::string w(who);
    if (!peers) return fail(PFRT_ERR_INVALID_ARGUMENT, w + ": null peer set");
    const int world = peers->world, rank = peers->rank;
    if (world < 1 || world > PFRT_MAX_PEERS || rank < 0 || rank >= world || !peers->state)
        return fail(PFRT_ERR_INVALID_ARGUMENT, w + ": bad rank/world or null state");
    if (!peers->y) return fail(PFRT_ERR_INVALID_ARGUMENT, w + ": null output");
    if (M < 1) return fail(PFRT_ERR_INVALID_ARGUMENT, w + ": M must be >= 1");
    const int64_t max_m = peers->max_m > 0 ? peers->max_m : 1;
    if (M > max_m)
        return fail(PFRT_ERR_INVALID_ARGUMENT,
                    w + ": M = " + std::to_string(M) + " exceeds the output's max_m = " + std::to_string(max_m));
    if (M > 1 && world > 1) {
        for (int p = 0; p < world; ++p)
            if (!peers->y_peer[p] || !peers->sig[p])
                return fail(PFRT_ERR_INVALID_ARGUMENT, w + ": M > 1 needs every rank's mapped output and signal words");
        if (peers->y_peer[rank] != peers->y) return fail(PFRT_ERR_INVALID_ARGUMENT, w + ": y_peer[rank] must be y");
    }
    return PFRT_OK;
}

PushArgs push_args(const pfrt_peer_set* peers, int64_t M, int64_t ns) {
    const int world = peers->world;
    PushArgs a{};
    a.rank = peers->rank;
    a.world = world;
    a.M = M;
    a.ns = ns;
    a.ldy = static_cast<int64_t>(world) * ns;
    bool vec = (ns % 4) == 0;
    for (int p = 0; p < world; ++p) {
        a.y[p] = peers->y_peer[p];
        a.sig[p] = peers->sig[p];
        vec = vec && (reinterpret_cast<uintptr_t>(a.y[p]) & 15u) == 0;
    }
    a.vec = vec ? 1 : 0;
    a.copy = 1;
    a.state = peers->state;
    a.wait_ns = peer_wait_ns();
    return a;
}

// The "ready" exchange before a GEMM that writes into other ranks' outputs.
pfrt_status launch_ready(pfrt_ctx* ctx, const pfrt_peer_set* peers, int64_t M, int64_t ns, cudaStream_t s) {
    peer_ready_kernel<<<1, 32, 0, s>>>(push_args(peers, M, ns), ctx->d_err);
    PFRT_CHECK_LAUNCH("peer_ready_kernel");
    return PFRT_OK;
}

// After the shard's SpMM: copy the block to the other ranks (unless `fused`:
// the GEMM's epilogue stored it there after launch_ready) and signal.
pfrt_status launch_push(pfrt_ctx* ctx, const pfrt_peer_set* peers, int64_t M, int64_t ns, cudaStream_t s,
                        bool fused = false) {
    if (peers->world == 1 || ns == 0 || M == 0) return PFRT_OK;
    PushArgs a = push_args(peers, M, ns);
    a.copy = fused ? 0 : 1;
    a.ready_done = fused ? 1 : 0;
    const int64_t items = a.vec ? M * ns / 4 : M * ns;
    const int blocks = fused ? 1 : static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(256, ceil_div(items, 4 * kPushThreads))));
    peer_push_kernel<<<blocks, kPushThreads, 0, s>>>(a, ctx->d_err);
    PFRT_CHECK_LAUNCH("peer_push_kernel");
    return PFRT_OK;
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
    // Every copy on the context stream, which is synchronized before the
    // weight is returned: a pageable cudaMemcpy may return before its DMA
    // lands, and later users may be on any stream.
    cudaStream_t cs = ctx->stream;
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(w->indptr, ip.data(), sizeof(int32_t) * (N + 1), cudaMemcpyHostToDevice, cs);
    // Device copy in bank order (bank_order_rows); PFRT_CSR_BANK_ORDER=0
    // keeps the caller's order.
    std::vector<int32_t> ix_dev;
    std::vector<float> v_dev;
    const char* bank_env = std::getenv("PFRT_CSR_BANK_ORDER");
    const bool bank_order = nnz > 0 && !(bank_env && *bank_env == '0');
    if (bank_order) {
        ix_dev = ix;
        v_dev.assign(values_host, values_host + nnz);
        bank_order_rows(ip, ix_dev, v_dev);
    }
    if (e == cudaSuccess && nnz > 0)
        e = cudaMemcpyAsync(w->indices, bank_order ? ix_dev.data() : ix.data(), sizeof(int32_t) * nnz,
                            cudaMemcpyHostToDevice, cs);
    if (e == cudaSuccess && nnz > 0)
        e = cudaMemcpyAsync(w->values, bank_order ? v_dev.data() : values_host, sizeof(float) * nnz,
                            cudaMemcpyHostToDevice, cs);
    if (e != cudaSuccess) {
        pfrt_csr_destroy(w);
        return cuda_fail(e, "pfrt_csr_create");
    }
    w->host_indptr = ip;
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
        e = cudaMalloc(&w->cptr, sizeof(int32_t) * (cptr.size() + 4));
        if (e == cudaSuccess) e = cudaMalloc(&w->cent, sizeof(uint2) * (cent.size() + 2));
        if (e == cudaSuccess) e = cudaMemsetAsync(w->cptr, 0, sizeof(int32_t) * (cptr.size() + 4), cs);
        if (e == cudaSuccess) e = cudaMemsetAsync(w->cent, 0, sizeof(uint2) * (cent.size() + 2), cs);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(w->cptr, cptr.data(), sizeof(int32_t) * cptr.size(), cudaMemcpyHostToDevice, cs);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(w->cent, cent.data(), sizeof(uint2) * cent.size(), cudaMemcpyHostToDevice, cs);
        if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
        w->host_cptr = std::move(cptr);
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
    if (w->xt_part) cudaFree(w->xt_part);
    if (w->part) cudaFree(w->part);
    if (w->dense) pfrt_fweight_destroy(w->dense);
    if (w->tc_mask) cudaFree(w->tc_mask);
    if (w->tc_off) cudaFree(w->tc_off);
    if (w->tc_vals) cudaFree(w->tc_vals);
    if (w->sp_wimg) cudaFree(w->sp_wimg);
    if (w->sp_cmeta) cudaFree(w->sp_cmeta);
    if (w->sp_cocc) cudaFree(w->sp_cocc);
    if (w->sp_coff) cudaFree(w->sp_coff);
    if (w->sp_cvals) cudaFree(w->sp_cvals);
    if (w->sp_rptr) cudaFree(w->sp_rptr);
    if (w->sp_rcol) cudaFree(w->sp_rcol);
    if (w->sp_rval) cudaFree(w->sp_rval);
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
    return spmm_uploaded(ctx, const_cast<pfrt_csr*>(w), M, x, ldx, y, ldy, pick_stream(ctx, stream));
}

pfrt_status pfrt_spmm_allgather(pfrt_ctx* ctx, const pfrt_csr* w, int64_t M, const float* x, int64_t ldx,
                                const pfrt_peer_set* peers, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!w || !x || !peers) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_spmm_allgather: null argument");
    if (w->ctx != ctx) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_spmm_allgather: CSR belongs to another context");
    if (ldx < w->K) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_spmm_allgather: row stride too small");
    st = check_peer_set(peers, M, "pfrt_spmm_allgather");
    if (st) return st;
    const int world = peers->world, rank = peers->rank;
    if (peers->ns != 0 && peers->ns != w->N)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_spmm_allgather: the peer set's ns differs from the shard's rows");
    const int64_t ns = w->N, ldy = static_cast<int64_t>(world) * ns;
    cudaStream_t s = pick_stream(ctx, stream);
    if (M > 1) {
        // This rank's column block of Y, straight into its own gathered
        // output (and, on the fused dense path, into every other rank's).
        bool fused = false;
        const ShardOut so{peers, ns, &fused};
        st = spmm_uploaded(ctx, const_cast<pfrt_csr*>(w), M, x, ldx, peers->y + static_cast<int64_t>(rank) * ns, ldy, s,
                           world > 1 ? &so : nullptr);
        if (st) return st;
        return launch_push(ctx, peers, M, ns, s, fused);
    }
    for (int p = 0; p < world; ++p)
        if (!peers->recv[p]) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_spmm_allgather: null receive buffer");
    const size_t shm = sizeof(float) * static_cast<size_t>(std::max<int64_t>(w->K, 1));
    if (shm > 96 * 1024 || w->nnz > INT32_MAX - 4096)
        return fail(PFRT_ERR_UNSUPPORTED, "pfrt_spmm_allgather: K or nnz too large for the fused M = 1 kernel");
    PeerArgs pa{};
    pa.rank = rank;
    pa.world = world;
    pa.col0 = static_cast<int64_t>(rank) * w->N;
    pa.y = peers->y;
    for (int p = 0; p < world; ++p) pa.recv[p] = peers->recv[p];
    pa.state = peers->state;
    pa.wait_ns = peer_wait_ns();
    auto kern = spmm_row1_kernel<4, 512, false, true>;
    PFRT_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shm)));
    int occ = 1;
    PFRT_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 512, shm));
    const int blocks = static_cast<int>(
        std::max<int64_t>(1, std::min<int64_t>(ceil_div(w->N, 16), int64_t{std::max(1, occ)} * ctx->num_sms)));
    const int vec_x = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (w->K & 3) == 0) ? 1 : 0;
    kern<<<blocks, 512, shm, s>>>(w->N, w->K, w->nnz, w->indptr, w->indices, w->values, x, vec_x, nullptr,
                                   ctx->d_err, pa);
    PFRT_CHECK_LAUNCH("spmm_row1_kernel<peer>");
    return PFRT_OK;
}

pfrt_status pfrt_peer_allgather(pfrt_ctx* ctx, int64_t M, const pfrt_peer_set* peers, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    st = check_peer_set(peers, M, "pfrt_peer_allgather");
    if (st) return st;
    if (peers->ns <= 0) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_peer_allgather: the peer set's ns must be > 0");
    for (int p = 0; p < peers->world && peers->world > 1; ++p)
        if (!peers->y_peer[p] || !peers->sig[p])
            return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_peer_allgather: needs every rank's mapped output and signal words");
    return launch_push(ctx, peers, M, peers->ns, pick_stream(ctx, stream));
}

pfrt_status pfrt_peer_reset(pfrt_ctx* ctx, const pfrt_peer_set* peers, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (!peers || !peers->state) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_peer_reset: null argument");
    const int world = peers->world, rank = peers->rank;
    if (world < 1 || world > PFRT_MAX_PEERS || rank < 0 || rank >= world)
        return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_peer_reset: bad rank/world");
    cudaStream_t s = pick_stream(ctx, stream);
    PFRT_CUDA_TRY(cudaMemsetAsync(peers->state, 0, 4 * sizeof(uint32_t), s));
    if (peers->recv[rank]) {
        if (peers->ns <= 0)
            return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_peer_reset: the peer set's ns is needed to clear its receive buffer");
        PFRT_CUDA_TRY(cudaMemsetAsync(peers->recv[rank], 0, sizeof(uint64_t) * 2 * world * peers->ns, s));
    }
    if (peers->sig[rank]) PFRT_CUDA_TRY(cudaMemsetAsync(peers->sig[rank], 0, sizeof(uint32_t) * PFRT_PEER_SIG_WORDS, s));
    return PFRT_OK;
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
