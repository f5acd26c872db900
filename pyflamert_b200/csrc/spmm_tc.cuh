// spmm_tc.cuh -- CSR SpMM on the tensor cores with W densified on chip.
//
//   Y[M, N] = X[M, K] * W^T,   W [N, K] sparse
//
// computed as the transposed product Y^T = W * X^T on tcgen05 kind::tf32
// with the 3xTF32 split: the MMA's A operand is a 128-row tile of W, built in
// tensor memory (TMEM) from a compressed form of W by producer warps, and
// its B operand is X, split into tf32 hi/lo parts beforehand and loaded by
// TMA.  No dense copy of W exists in HBM: each call reads W's nonzeros once
// per slab of X, and the dense tile lives only in TMEM for the MMAs that use
// it.
//
// A tf32 MMA instruction takes about as long at N = 64 as at N = 128 (~70
// SM clocks for M = 128, K = 8: the N = 128 shape runs at the tensor pipe's
// rate, the narrower one at half of it), so every MMA here is N = 128:
//   stacked (M <= 64): the B tile is X_hi's rows on top of X_lo's rows, and
//       two MMAs per K step, A = W_hi and A = W_lo, accumulate
//       [hh + lh | hl + ll] into one 128-column accumulator; the epilogue
//       adds its two halves.
//   wide (M > 64): slabs of 128 rows of X; three MMAs per K step (lo*hi,
//       hi*lo, hi*hi) into one accumulator.
//
// Compressed form of W (built once per weight, `pfrt_csr` owns it):
//   mask[kb][n]  bit j set <=> W[n, 32 kb + j] is stored      (u32, kb-major)
//   off[kb][n]   index in vals of the first stored value of row n at or
//                after column 32 kb                            (u32, kb-major)
//   vals[]       (hi, lo) tf32 split of every stored value, row by row in
//                column order                                  (float2)
// Rows are padded to a multiple of 128 with empty masks.  Consecutive rows
// are consecutive words of mask and off, so a warp reads its 32 rows' words
// of one k-block in one 128-byte transaction.
//
// One CTA per SM, 448 threads:
//   warps 0..7   producers: warp w builds TMEM lanes 32 (w % 4) .. +31 (a warp
//                may only write its own lane quarter) for every other k-block
//                of the CTA's sequence (w / 4 selects which), so two warps per
//                quarter overlap one k-block's loads with the other's stores.
//                Lane l owns W row 128 t + 32 (w % 4) + l: it expands its
//                row's 32 columns from mask and vals into registers (zeros
//                where the mask bit is clear) and stores them with
//                tcgen05.st, hi part and lo part side by side.
//   warps 8..11  epilogue: tcgen05.ld of the accumulator, IEEE fp32 sums of
//                the per-chunk partials (in registers when stacked, 64 per
//                thread; in shared memory when wide, 128 per thread), stores
//                of Y^T's columns as Y's rows.
//   warp 12      TMA: X hi/lo tiles [64 rows, 32 columns] into a shared ring.
//   warp 13      MMA issuer and TMEM owner.
// TMEM (512 columns): two 128-column accumulators, then kTcStages A stages
// of 64 columns (32 hi, 32 lo).  Stage s of the A ring and of the X ring are
// filled for the same k-block and released by one MMA commit.
//
// Work unit = (W tile of 128 rows, X slab); the k-blocks of all units are
// split evenly over the CTAs (stream-K, see tc_unit).
#pragma once

#include "common.cuh"
#include "umma_gemm.cuh"  // epi_barrier_or

namespace pfrt {

constexpr int kTcWRows = 128;    // W rows per tile = TMEM lanes = MMA M
constexpr int kTcN = 128;        // MMA N = accumulator columns
constexpr int kTcBK = 32;        // K per k-block (128 bytes of fp32)
constexpr int kTcStages = 4;     // even: stage s always belongs to the same producer pair
constexpr int kTcPromoteKb = 4;  // k-blocks per TMEM accumulation (128 K), then an IEEE add
constexpr int kTcProdWarps = 8;
constexpr int kTcEpiWarps = 4;
constexpr int kTcThreads = (kTcProdWarps + kTcEpiWarps + 2) * 32;
constexpr int kTcXBox = 64 * 128;              // bytes of one TMA box of X (64 rows x 32 fp32)
constexpr int kTcStageBytes = 4 * kTcXBox;     // wide: hi and lo of 128 rows; stacked uses half
constexpr int kTcSumBytes = kTcN * 128 * 4;  // wide: running sums [128 X rows][128 W rows]
constexpr int kTcBarBytes = 1024;
constexpr int kTcSmemBytes = kTcStages * kTcStageBytes + kTcSumBytes + kTcBarBytes + 1024;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcAStage0 = 2 * kTcN;      // first A stage column
static_assert(kTcAStage0 + kTcStages * 64 <= kTcTmemCols, "TMEM columns");
static_assert(kTcStages % 2 == 0, "the two producer warps of a quarter alternate k-blocks");

// X rows per unit.
template <bool STACKED>
constexpr int tc_slab() { return STACKED ? 64 : 128; }

struct TcSched {
    int n_wtiles;      // ceil(N / 128)
    int n_xslabs;      // ceil(M / slab): 1 when stacked (M <= 64), else ceil(M / 128)
    int kb_total;      // ceil(K / 32)
    int64_t total;     // k-blocks of all units: n_wtiles * n_xslabs * kb_total
    int64_t per_cta;   // k-blocks per CTA (the last CTA may have fewer)
};

struct TcArgs {
    const uint32_t* mask;  // [kb_total][npad]
    const uint32_t* off;   // [kb_total][npad]
    const float2* vals;    // [nnz]
    int64_t npad;
    int M, N;
    float* y;              // output, row stride ldy
    int64_t ldy;
    float* partial;        // [2 * grid][64][128] partial tiles
};

// Partial tiles of the stream-K fix-up: [X rows of a slab, at most 128][128 W rows].
constexpr int kTcTileElems = kTcN * kTcWRows;

// Unit u = (W tile t, X slab c), slabs innermost: the CTAs that work on the
// slabs of one W tile are neighbours in the grid, run together and find the
// tile's nonzeros in L2.  The k-blocks of all units form one sequence, unit
// by unit; CTA b takes the contiguous range [b L, (b + 1) L) of it (stream-K),
// so every CTA has the same amount of MMA work whatever the unit count.  A
// unit whose k-blocks lie in one CTA's range is finished by that CTA; the
// CTAs that share a unit each write a partial tile (at most two per CTA: the
// first and the last piece of its range) and tc_fixup_kernel adds them up.
__device__ __forceinline__ void tc_unit(const TcSched& s, int64_t u, int& t, int& c) {
    c = static_cast<int>(u % s.n_xslabs);
    t = static_cast<int>(u / s.n_xslabs);
}

// Position (W tile t, X slab c, k-block kb) in a CTA's k-block sequence,
// advanced one k-block at a time without divisions (the per-k-block loops of
// the TMA thread and the producers would otherwise spend most of their
// issue slots on 64-bit division).
struct TcCursor {
    int t, c, kb;
    __device__ __forceinline__ void init(const TcSched& s, int64_t g) {
        const int64_t u = g / s.kb_total;
        kb = static_cast<int>(g - u * s.kb_total);
        tc_unit(s, u, t, c);
    }
    __device__ __forceinline__ void next(const TcSched& s) {
        if (++kb == s.kb_total) {
            kb = 0;
            if (++c == s.n_xslabs) {
                c = 0;
                ++t;
            }
        }
    }
};

// D[tmem] (+)= A[tmem] * B[smem]^T with tf32 inputs, f32 accumulate.  A is
// 128 lanes x 8 columns (one fp32 word per element), K-major.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Stores 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Loads 16 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Non-blocking test of whether the phase with the given parity has
// completed (mbarrier.test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Expands 8 columns [8 G, 8 G + 8) of one row's k-block into hi[j], lo[j]:
// the stored values in column order from *p (advanced past the values it
// used), zeros where the mask bit is clear.  Hand-written PTX so that each
// column costs a predicate, two zeroing moves, one predicated 8-byte load
// and one predicated pointer step: no load depends on another's result, so
// all are in flight at once, and the producers leave the SM's issue slots
// to the MMA thread that shares their scheduler.
template <int G>
__device__ __forceinline__ void tc_expand8(uint32_t m, const float2*& p, uint32_t (&hi)[32], uint32_t (&lo)[32]) {
    uint64_t a = reinterpret_cast<uint64_t>(p);
    asm("{\n\t.reg .pred q0, q1, q2, q3, q4, q5, q6, q7;\n\t"
        ".reg .b32 t;\n\t"
#define PFRT_TC_COL(J, Q, H, L)                                 \
        "and.b32 t, %17, " #J ";\n\t"                          \
        "setp.ne.b32 " #Q ", t, 0;\n\t"                        \
        "mov.b32 " H ", 0;\n\t"                                 \
        "mov.b32 " L ", 0;\n\t"                                 \
        "@" #Q " ld.global.nc.v2.b32 {" H ", " L "}, [%16];\n\t" \
        "@" #Q " add.s64 %16, %16, 8;\n\t"
        PFRT_TC_COL(%18, q0, "%0", "%8")
        PFRT_TC_COL(%19, q1, "%1", "%9")
        PFRT_TC_COL(%20, q2, "%2", "%10")
        PFRT_TC_COL(%21, q3, "%3", "%11")
        PFRT_TC_COL(%22, q4, "%4", "%12")
        PFRT_TC_COL(%23, q5, "%5", "%13")
        PFRT_TC_COL(%24, q6, "%6", "%14")
        PFRT_TC_COL(%25, q7, "%7", "%15")
#undef PFRT_TC_COL
        "}"
        : "=&r"(hi[8 * G + 0]), "=&r"(hi[8 * G + 1]), "=&r"(hi[8 * G + 2]), "=&r"(hi[8 * G + 3]),
          "=&r"(hi[8 * G + 4]), "=&r"(hi[8 * G + 5]), "=&r"(hi[8 * G + 6]), "=&r"(hi[8 * G + 7]),
          "=&r"(lo[8 * G + 0]), "=&r"(lo[8 * G + 1]), "=&r"(lo[8 * G + 2]), "=&r"(lo[8 * G + 3]),
          "=&r"(lo[8 * G + 4]), "=&r"(lo[8 * G + 5]), "=&r"(lo[8 * G + 6]), "=&r"(lo[8 * G + 7]),
          "+l"(a)
        : "r"(m), "n"(1u << (8 * G + 0)), "n"(1u << (8 * G + 1)), "n"(1u << (8 * G + 2)),
          "n"(1u << (8 * G + 3)), "n"(1u << (8 * G + 4)), "n"(1u << (8 * G + 5)), "n"(1u << (8 * G + 6)),
          "n"(1u << (8 * G + 7)));
    p = reinterpret_cast<const float2*>(a);
}

__device__ __forceinline__ void tc_expand(uint32_t m, const float2* p, uint32_t (&hi)[32], uint32_t (&lo)[32]) {
    tc_expand8<0>(m, p, hi, lo);
    tc_expand8<1>(m, p, hi, lo);
    tc_expand8<2>(m, p, hi, lo);
    tc_expand8<3>(m, p, hi, lo);
}

// Partial-tile slot of CTA b's piece of unit u: 2b for the first piece of
// its range, 2b + 1 for the last.
__device__ __forceinline__ int64_t tc_slot(const TcSched& s, int64_t b, int64_t u) {
    return (u == (b * s.per_cta) / s.kb_total) ? 2 * b : 2 * b + 1;
}

template <bool STACKED>
__global__ void __launch_bounds__(kTcThreads, 1)
    spmm_tc_kernel(const __grid_constant__ CUtensorMap tmXh, const __grid_constant__ CUtensorMap tmXl,
                   const TcSched sched, const TcArgs a, int* err) {
    constexpr int SLAB = tc_slab<STACKED>();
    constexpr uint32_t kStageTx = STACKED ? 2 * kTcXBox : 4 * kTcXBox;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* xtiles = smem;
    float* sums = reinterpret_cast<float*>(smem + kTcStages * kTcStageBytes);
    uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes + kTcSumBytes);
    uint64_t* afull = xfull + kTcStages;
    uint64_t* empty = afull + kTcStages;
    uint64_t* tfull = empty + kTcStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr int kEpiThreads = 32 * kTcEpiWarps;
    constexpr int kTmaWarp = kTcProdWarps + kTcEpiWarps;
    constexpr int kMmaWarp = kTmaWarp + 1;
    const int64_t KB = sched.kb_total;
    const int64_t g0 = static_cast<int64_t>(blockIdx.x) * sched.per_cta;
    const int64_t g1 = min(g0 + sched.per_cta, sched.total);  // this CTA's k-blocks [g0, g1)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&afull[s], 4);  // one arrival per lane quarter
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiThreads);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_slot, kTcTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp < kTcProdWarps) {
        // W's compressed form is written once, before any call that uses it,
        // so the producers start before the previous kernel has finished.
        const int q = warp & 3, pw = warp >> 2;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const int nseq = static_cast<int>(g1 - g0);
        const int64_t row_off = q * 32 + lane;
        // mask and off words of this warp's k-blocks, in order, two of its
        // k-blocks ahead of the one being expanded; the row's values about 8
        // (10 % density) k-blocks ahead are prefetched into L1.
        TcCursor ahead;
        ahead.init(sched, g0 + pw);
        int sq_ahead = pw;
        auto load_mo = [&](uint32_t& m, uint32_t& o) {
            m = 0;
            o = 0;
            if (sq_ahead < nseq) {
                const int64_t w = static_cast<int64_t>(ahead.kb) * a.npad + static_cast<int64_t>(ahead.t) * kTcWRows + row_off;
                m = __ldg(a.mask + w);
                o = __ldg(a.off + w);
            }
            ahead.next(sched);
            ahead.next(sched);
            sq_ahead += 2;
        };
        uint32_t m0, o0, m1, o1;
        load_mo(m0, o0);
        load_mo(m1, o1);
        int stage = pw;
        uint32_t phase = 0;
        for (int seq = pw; seq < nseq; seq += 2) {
            uint32_t m2, o2;
            load_mo(m2, o2);
            const float2* p = a.vals + o0;
            asm volatile("prefetch.global.L1 [%0];" ::"l"(p + 16));
            asm volatile("prefetch.global.L1 [%0];" ::"l"(p + 32));
            uint32_t hi[32], lo[32];
            tc_expand(m0, p, hi, lo);
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                break;
            }
            tc_fence_after();
            const uint32_t col = tmem_base + kTcAStage0 + static_cast<uint32_t>(stage * 64) + lane_off;
            tmem_st_32x32b_x32(col, hi);
            tmem_st_32x32b_x32(col + 32, lo);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[stage]);
            if ((stage += 2) >= kTcStages) {
                stage -= kTcStages;
                phase ^= 1u;
            }
            m0 = m1;
            o0 = o1;
            m1 = m2;
            o1 = o2;
        }
    } else if (warp < kTmaWarp) {
        const int q = warp & 3;
        const int nl = q * 32 + lane;  // this thread's TMEM lane = W row within the tile
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        pdl_wait();  // the partial tiles and Y may still be read by the previous kernel
        int tc = 0;  // accumulation chunks consumed
        for (int64_t g = g0; g < g1;) {
            const int64_t u = g / KB;
            const int kb_lo = static_cast<int>(g % KB);
            const int kb_hi = static_cast<int>(KB < kb_lo + (g1 - g) ? KB : kb_lo + (g1 - g));
            g += kb_hi - kb_lo;
            int t, c;
            tc_unit(sched, u, t, c);
            // Running sums of the slab's X rows for this W row: registers
            // (stacked, 64) or this thread's column of `sums` (wide, 128;
            // sums[m * 128 + nl], so a warp's accesses are consecutive words).
            float racc[STACKED ? 64 : 1];
#pragma unroll
            for (int j = 0; j < (STACKED ? 64 : 1); ++j) racc[j] = 0.0f;
            bool stop = false;
            bool first = true;
            for (int kc = kb_lo; kc < kb_hi; kc += kTcPromoteKb, ++tc) {
                const int slot = tc & 1;
                const uint32_t ap = static_cast<uint32_t>(tc >> 1) & 1u;
                const bool got = mbar_wait(&tfull[slot], ap, abort_flag);
                if (epi_barrier_or(!got || *abort_flag != 0, kEpiThreads)) {
                    stop = true;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + static_cast<uint32_t>(slot * kTcN) + lane_off;
                if constexpr (STACKED) {
                    // X row j: columns j (hh + lh) and 64 + j (hl + ll).
#pragma unroll
                    for (int h = 0; h < 4; ++h) {
                        uint32_t v0[16], v1[16];
                        tmem_ld_32x32b_x16(taddr + static_cast<uint32_t>(16 * h), v0);
                        tmem_ld_32x32b_x16(taddr + static_cast<uint32_t>(64 + 16 * h), v1);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            racc[16 * h + j] =
                                __fadd_rn(racc[16 * h + j], __fadd_rn(__uint_as_float(v0[j]), __uint_as_float(v1[j])));
                    }
                } else {
#pragma unroll 1
                    for (int h = 0; h < 4; ++h) {
                        uint32_t v[32];
                        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(32 * h), v);
                        tmem_ld_wait();
                        float* sp = sums + (32 * h) * kTcWRows + nl;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            sp[j * kTcWRows] = first ? __uint_as_float(v[j]) : __fadd_rn(sp[j * kTcWRows], __uint_as_float(v[j]));
                    }
                }
                first = false;
                tc_fence_before();
                mbar_arrive(&tempty[slot]);
            }
            if (stop) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                break;
            }
            auto val = [&](int j) -> float {
                if constexpr (STACKED) return racc[j];
                else return sums[j * kTcWRows + nl];
            };
            // (Fully unrolled, so racc stays in registers when stacked.)
            if (kb_lo == 0 && kb_hi == KB) {
                const int n = t * kTcWRows + nl;
                const int m0 = c * SLAB;
                if (n < a.N) {
                    float* dst = a.y + n;
#pragma unroll
                    for (int j = 0; j < SLAB; ++j)
                        if (m0 + j < a.M) dst[static_cast<int64_t>(m0 + j) * a.ldy] = val(j);
                }
            } else {
                float* dst = a.partial + tc_slot(sched, blockIdx.x, u) * kTcTileElems + nl;
#pragma unroll
                for (int j = 0; j < SLAB; ++j) dst[j * kTcWRows] = val(j);
            }
        }
    } else if (warp == kTmaWarp) {
        if (lane == 0) {
            tma_prefetch_desc(&tmXh);
            tma_prefetch_desc(&tmXl);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            uint32_t last_par[kTcStages];
            bool ok = true;
            pdl_wait();  // X's split comes from the previous kernel
            TcCursor cur;
            cur.init(sched, g0);
            for (int64_t g = g0; g < g1; ++g, cur.next(sched)) {
                const int kx = cur.kb * kTcBK, r0 = cur.c * SLAB;
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* st = xtiles + stage * kTcStageBytes;
                mbar_arrive_expect_tx(&xfull[stage], kStageTx);
                if constexpr (STACKED) {
                    // One 128-row B tile: X_hi's rows 0..63 on top of X_lo's.
                    tma_load_2d(st, &tmXh, &xfull[stage], kx, 0);
                    tma_load_2d(st + kTcXBox, &tmXl, &xfull[stage], kx, 0);
                } else {
                    tma_load_2d(st, &tmXh, &xfull[stage], kx, r0);
                    tma_load_2d(st + kTcXBox, &tmXh, &xfull[stage], kx, r0 + 64);
                    tma_load_2d(st + 2 * kTcXBox, &tmXl, &xfull[stage], kx, r0);
                    tma_load_2d(st + 3 * kTcXBox, &tmXl, &xfull[stage], kx, r0 + 64);
                }
                issued |= 1u << stage;
                last_par[stage] = phase;
                if (++stage == kTcStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                const int zero = 0;
                for (int s = 0; s < kTcStages; ++s)
                    if (issued & (1u << s)) mbar_wait(&xfull[s], last_par[s], &zero);
            }
        }
    } else {
        if (lane == 0) {
            const uint32_t idesc = idesc_make(1, 2, 2, kTcWRows, kTcN);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int tc = 0;
            // The next k-block's barriers are tested while this k-block's
            // MMAs are issued; a waiting test costs no MMA issue time, and
            // a blocking wait (~100+ SM clocks even on a completed phase)
            // is only needed when the test found the phase open.
            bool next_ready = false;
            for (int64_t g = g0; ok && g < g1;) {
                const int kb_lo = static_cast<int>(g % KB);
                const int kb_hi = static_cast<int>(KB < kb_lo + (g1 - g) ? KB : kb_lo + (g1 - g));
                g += kb_hi - kb_lo;
                for (int kc = kb_lo; ok && kc < kb_hi; kc += kTcPromoteKb, ++tc) {
                    const int kce = min(kc + kTcPromoteKb, kb_hi);
                    const int slot = tc & 1;
                    const uint32_t ap = static_cast<uint32_t>(tc >> 1) & 1u;
                    if (!mbar_wait(&tempty[slot], ap ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kTcN);
                    for (int kb = kc; kb < kce; ++kb) {
                        if (!next_ready && (!mbar_wait(&afull[stage], phase, abort_flag) ||
                                            !mbar_wait(&xfull[stage], phase, abort_flag))) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const int ns = stage + 1 == kTcStages ? 0 : stage + 1;
                        const uint32_t nph = stage + 1 == kTcStages ? phase ^ 1u : phase;
                        const bool na = mbar_test_wait(smem_u32(&afull[ns]), nph);
                        const bool nx = mbar_test_wait(smem_u32(&xfull[ns]), nph);
                        const uint32_t ahi = tmem_base + kTcAStage0 + static_cast<uint32_t>(stage * 64);
                        const uint32_t alo = ahi + 32;
                        const uint32_t st = smem_u32(xtiles + stage * kTcStageBytes);
                        const uint64_t dxh = sdesc_kmajor_sw128(st);
#pragma unroll
                        for (int k = 0; k < kTcBK / 8; ++k) {
                            const uint64_t koff = static_cast<uint64_t>((k * 8 * 4) >> 4);
                            const uint32_t acc0 = (kb > kc || k > 0) ? 1u : 0u;
                            if constexpr (STACKED) {
                                umma_tf32_ts(d_tmem, alo + k * 8, dxh + koff, idesc, acc0);
                                umma_tf32_ts(d_tmem, ahi + k * 8, dxh + koff, idesc, 1u);
                            } else {
                                const uint64_t dxl = sdesc_kmajor_sw128(st + 2 * kTcXBox);
                                umma_tf32_ts(d_tmem, alo + k * 8, dxh + koff, idesc, acc0);
                                umma_tf32_ts(d_tmem, ahi + k * 8, dxl + koff, idesc, 1u);
                                umma_tf32_ts(d_tmem, ahi + k * 8, dxh + koff, idesc, 1u);
                            }
                        }
                        umma_commit(&empty[stage]);
                        next_ready = na && nx;
                        if (++stage == kTcStages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    umma_commit(&tfull[slot]);
                }
            }
            if (!ok) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
            }
            umma_commit(drain);
            const int zero = 0;
            mbar_wait(drain, 0, &zero);
        }
    }

    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTcTmemCols);
    }
}

// Finishes the units that several CTAs share: blocks (b, i) for each
// boundary between CTA ranges (b, b + 1) that falls inside a unit (skipped
// when an earlier boundary falls inside the same unit), i over 1024-element
// pieces of the tile.  Each thread adds 4 consecutive elements of the unit's
// partial tiles in CTA order (IEEE fp32), with the loads of several partial
// tiles in flight at once, and stores them to Y.
__global__ void __launch_bounds__(256) tc_fixup_kernel(const TcSched sched, const float* __restrict__ partial, int M,
                                                       int N, int slab, float* __restrict__ y, int64_t ldy) {
    pdl_wait();
    const int64_t KB = sched.kb_total, L = sched.per_cta;
    const int64_t b = blockIdx.x;  // boundary at k-block (b + 1) L
    const int64_t p = (b + 1) * L;
    if (p >= sched.total || p % KB == 0) return;
    const int64_t u = p / KB;
    if (b * L > u * KB) return;  // an earlier boundary is inside u too
    const int64_t bf = (u * KB) / L, bl = ((u + 1) * KB - 1) / L;
    const int e0 = (static_cast<int>(blockIdx.y) * blockDim.x + threadIdx.x) * 4;
    if (e0 >= slab * kTcWRows) return;
    int t, c;
    tc_unit(sched, u, t, c);
    const int ml = e0 / kTcWRows, nl = e0 % kTcWRows;
    const int m = c * slab + ml, n = t * kTcWRows + nl;
    if (m >= M || n >= N) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t cb = bf; cb <= bl; cb += 4) {
        float4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (cb + i <= bl)
                v[i] = *reinterpret_cast<const float4*>(partial + tc_slot(sched, cb + i, u) * kTcTileElems + e0);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (cb + i <= bl) {
                acc.x = __fadd_rn(acc.x, v[i].x);
                acc.y = __fadd_rn(acc.y, v[i].y);
                acc.z = __fadd_rn(acc.z, v[i].z);
                acc.w = __fadd_rn(acc.w, v[i].w);
            }
    }
    float* d = y + static_cast<int64_t>(m) * ldy + n;
    const float r[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (n + j < N) d[j] = r[j];
}

// ---------------------------------------------------------- format build
// mask[kb][n] |= bit of every stored column; a column stored twice in a row
// sets *dup (the compressed form holds one value per position).
__global__ void tc_mask_kernel(int64_t N, int64_t npad, const int32_t* __restrict__ indptr,
                               const int32_t* __restrict__ indices, uint32_t* __restrict__ mask, int* dup) {
    const int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    for (int32_t j = indptr[n] + lane; j < indptr[n + 1]; j += 32) {
        const int32_t col = indices[j];
        const uint32_t bit = 1u << (col & 31);
        const uint32_t old = atomicOr(mask + static_cast<int64_t>(col >> 5) * npad + n, bit);
        if (old & bit) atomicExch(dup, 1);
    }
}

// off[kb][n] = indptr[n] + stored values of row n in k-blocks before kb.
// Thread per row (padding rows get nnz).
__global__ void tc_off_kernel(int64_t N, int64_t npad, int kb_total, const int32_t* __restrict__ indptr,
                              int64_t nnz, const uint32_t* __restrict__ mask, uint32_t* __restrict__ off) {
    const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (n >= npad) return;
    uint32_t run = static_cast<uint32_t>(n < N ? indptr[n] : nnz);
    for (int kb = 0; kb < kb_total; ++kb) {
        const int64_t w = static_cast<int64_t>(kb) * npad + n;
        off[w] = run;
        run += __popc(mask[w]);
    }
}

// vals[off[kb][n] + rank of the column inside its k-block] = split(value).
// Warp per row.
__global__ void tc_vals_kernel(int64_t N, int64_t npad, const int32_t* __restrict__ indptr,
                               const int32_t* __restrict__ indices, const float* __restrict__ values,
                               const uint32_t* __restrict__ mask, const uint32_t* __restrict__ off,
                               float2* __restrict__ vals) {
    const int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    for (int32_t j = indptr[n] + lane; j < indptr[n + 1]; j += 32) {
        const int32_t col = indices[j];
        const int64_t w = static_cast<int64_t>(col >> 5) * npad + n;
        const uint32_t below = mask[w] & ((1u << (col & 31)) - 1u);
        const float v = values[j];
        uint32_t h;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
        vals[off[w] + __popc(below)] = make_float2(__uint_as_float(h), __fsub_rn(v, __uint_as_float(h)));
    }
}

}  // namespace pfrt
