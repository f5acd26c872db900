// umma_gemm_sk.cuh -- the int8 GEMM with K split over a cluster of two CTAs.
//
//   D[M,N] = A[M,K] * B[N,K]^T  (u8/s8 x s8 -> s32), both operands K-major.
//
// For shapes whose 128 x BN tiles number at most half the SMs (config 2:
// 512 x 4096 x 4096 gives 64 tiles of 128 x 256), one tile per cluster of two
// CTAs: CTA r (its rank in the cluster) accumulates about half of the
// k-blocks of the 128 x BN tile in its own TMEM, as umma_gemm_kernel does
// (which k-blocks, and for which columns: "Early exchange" below).  Each CTA
// then finalises half of the tile's columns,
// [r * BN/2, +BN/2): it sends the other half of its partial accumulator to the
// peer through an L2-resident exchange buffer, adds the peer's partial for
// its own half, and runs the fused epilogue on 128 x BN/2 outputs.
//
// Against 128 x 128 tiles on one CTA each, the same SMs pull 768 KB instead of
// 1 MB through L2 per tile at K = 4096 (the mainloop of this shape runs at the
// GPU's aggregate L2 -> SM bandwidth), and each epilogue still covers 16 K
// outputs.  The int32 sum of the two partials is exact: the host admits only
// K for which the whole sum fits in int32.
//
// Exchange: each CTA writes the peer's half of its partial (64 KB at
// BN = 256) to its slot of a global exchange buffer, coalesced and kept in
// L2, and releases it with one remote mbarrier arrival per thread
// (mbarrier.arrive.release.cluster on the peer's xdone); the peer waits with
// cluster-scope acquire and reads the slot with L2-only loads.  (Moving the
// partial through distributed shared memory instead, by remote stores or by
// bulk copies, ran at 20-45 GB/s per SM, several times slower.)  Every wait is
// bounded.
//
// Early exchange.  The k-blocks are not split in two plain halves.  With
// T = kb_total and a tail of t k-blocks, a = (T - t) / 2 and b = a + t:
//   CTA 0: phase 1 = [0, a), all BN columns; phase 2 = [a, b), its own half;
//   CTA 1: phase 1 = [b, T), all BN columns; phase 2 = [a, b), its own half.
// Column half 0 then sums CTA 0's [0, b) and CTA 1's [b, T); half 1 sums
// CTA 0's [0, a) and CTA 1's [a, T): every k-block exactly once.  The peer's
// half of a CTA's partial is complete after phase 1, so its exchange (TMEM ->
// L2 -> the peer) runs while phase 2's N = BN/2 MMAs finish the own half,
// instead of after the whole mainloop.  Phase 2 loads A in full and only the
// own half of B.  t = 0 is the plain split.  The int32 sums are exact in any
// order, so the result does not depend on t.
// A stop (time-out) is written to both CTAs' abort words; both CTAs always
// reach the closing cluster barrier, after which no remote access to either
// CTA's shared memory remains.  No multi-CTA copy is used: each CTA loads its
// own tiles.
#pragma once

#include "umma_gemm2.cuh"

namespace pfrt {

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait with cluster-scope acquire (the phase was completed by arrivals
// from the peer CTA, which also wrote the data the waiter reads next).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, const volatile int* abort) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait_cluster(a, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1; it < kWaitLimitIters; ++it) {
        if (mbar_try_wait_cluster(a, parity)) return true;
        if ((it & 31u) == 0) {
            if (*abort) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) return false;
        }
    }
    return false;
}

// The two halves of a cluster barrier: every thread arrives once and later
// waits once, so the barrier's latency overlaps the work between them.
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

template <int BN, int STAGES>
struct GemmSkCfg {
    using G = GemmCfg<KIND_I8, BN, STAGES>;
    static constexpr int BM = 128;
    static constexpr int HALF = BN / 2;               // columns each CTA finalises
    static constexpr int XGRAN = BM * HALF / 4;       // 16-byte granules in one exchange slot
    static constexpr int BAR_BYTES = 256;
    static constexpr int PARAM_BYTES = 12 * HALF;
    // Eight epilogue warps, two per TMEM lane quarter, each thread taking two
    // 32-column chunks of its row (at BN = 256).  Sixteen (one chunk each)
    // measured 1.4 % slower at config 2: the epilogue is not issue-bound.
    static constexpr int EPI_WARPS = 8;
    static constexpr int EPI_THREADS = 32 * EPI_WARPS;
    static constexpr int GROUPS = EPI_WARPS / 4;      // column groups per lane quarter
    static constexpr int THREADS = 64 + EPI_THREADS;
    static constexpr int SMEM_BYTES = STAGES * G::STAGE_BYTES + BAR_BYTES + PARAM_BYTES + 1024;
    static_assert(HALF % (32 * GROUPS) == 0, "whole 32-column chunks per column group");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
    static_assert((2 * STAGES + 4) * 8 + 8 <= BAR_BYTES, "barrier area");
};

// The k-block ranges of CTA `rank` for kb_total = T and a tail of t k-blocks
// (the host keeps 0 <= t <= T - 2, so both phase-1 ranges are non-empty):
// phase 1 is [p1_lo, p1_lo + n1) over all columns, phase 2 is [a, a + t) over
// the CTA's own half.
__device__ __forceinline__ void sk2_ranges(int T, int t, uint32_t rank, int& p1_lo, int& n1, int& a) {
    a = (T - t) / 2;
    const int b = a + t;
    p1_lo = rank == 0 ? 0 : b;
    n1 = rank == 0 ? a : T - b;
}

// Bytes of the exchange buffer for `tiles` clusters: one slot (128 x BN/2
// int32) per CTA.
template <int BN>
constexpr size_t gemm_sk_xchg_bytes(int64_t tiles) {
    return static_cast<size_t>(tiles) * 2 * 128 * (BN / 2) * sizeof(int32_t);
}

// One 128 x BN tile per cluster (grid = 2 * tiles); sched.splits == 1 and
// 0 <= tail <= sched.kb_total - 2 (both CTAs get phase-1 k-blocks).  tmBh:
// the weight's map with a box of BN/2 rows (phase 2's own half of B).
// xchg: gemm_sk_xchg_bytes.
template <int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(GemmSkCfg<BN, STAGES>::THREADS, 1)
    umma_gemm_sk2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmBh, const GemmSched sched, const int tail,
                         const Epi epi, uint4* xchg, int* err) {
    using Cfg = GemmSkCfg<BN, STAGES>;
    using G = typename Cfg::G;
    constexpr int BM = Cfg::BM;
    constexpr int HALF = Cfg::HALF;
    constexpr int GROUPS = Cfg::GROUPS;
    constexpr int NCH = HALF / (32 * GROUPS);  // 32-column chunks per epilogue thread
    constexpr uint32_t WIDE_BYTES = G::STAGE_BYTES;                  // A + all BN rows of B
    constexpr uint32_t HALF_BYTES = G::A_TILE + HALF * G::BK_BYTES;  // A + the own half of B

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * G::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;  // the own half is complete
    uint64_t* pfull = tfull + 1;       // the peer's half is complete (end of phase 1)
    uint64_t* xdone = pfull + 1;
    uint64_t* drain = xdone + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* params = smem + STAGES * G::STAGE_BYTES + Cfg::BAR_BYTES;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const int unit = static_cast<int>(cluster_id_x());
    const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int*>(abort_flag)), peer);
    int mb, nb, ks;
    decode_unit(sched, unit, mb, nb, ks);
    int p1_lo, n1, p2_lo;
    sk2_ranges(sched.kb_total, tail, rank, p1_lo, n1, p2_lo);
    const int nk = n1 + tail;  // steps of this CTA: n1 over all columns, then `tail` over its own half
    auto kb_of = [&](int i) { return i < n1 ? p1_lo + i : p2_lo + (i - n1); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(tfull, 1);
        mbar_init(pfull, 1);
        mbar_init(xdone, Cfg::EPI_THREADS);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // First half of the cluster barrier that makes both CTAs' barriers and
    // abort words exist before either touches the other's; each thread
    // waits (once) before its first access to the peer.
    cluster_arrive_release();
    bool cl_waited = false;
    auto cluster_ready = [&]() {
        if (!cl_waited) {
            cluster_wait_acquire();
            cl_waited = true;
        }
    };
    if (warp == 1) tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) pdl_launch_dependents();
    bool stopped = false;  // this thread wrote the peer's abort word
    auto stop = [&]() {
        cluster_ready();
        stopped = true;
        *abort_flag = 1;
        st_cluster_u32(peer_abort, 1u);
        report_error(err, kDevWaitTimeout);
    };

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            tma_prefetch_desc(&tmBh);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            uint32_t last_par[STAGES];
            bool ok = true;
            // Step i's B: all BN rows in phase 1, the own half in phase 2
            // (placed at the start of the stage's B area).
            auto load_b = [&](int i, uint8_t* st) {
                if (i < n1)
                    tma_load_2d(st + G::A_TILE, &tmB, &full[stage], kb_of(i) * G::BK, nb * BN);
                else
                    tma_load_2d(st + G::A_TILE, &tmBh, &full[stage], kb_of(i) * G::BK,
                                nb * BN + static_cast<int>(rank) * HALF);
            };
            // B is a prepared weight: written once when it is created, never
            // by a kernel.  So the first stages' B tiles are requested before
            // the dependency wait, while the previous kernel still runs; A
            // (which that kernel may write) follows the wait.  The ring's
            // stages start empty, so these need no empty-barrier wait.
            const int npre = min(STAGES, nk);
            for (int i = 0; i < npre; ++i) {
                stage = i;
                mbar_arrive_expect_tx(&full[i], i < n1 ? WIDE_BYTES : HALF_BYTES);
                load_b(i, tiles + i * G::STAGE_BYTES);
                issued |= 1u << i;
                last_par[i] = 0u;
            }
            pdl_wait();  // A may come from the previous kernel
            for (int i = 0; i < npre; ++i)
                tma_load_2d(tiles + i * G::STAGE_BYTES, &tmA, &full[i], kb_of(i) * G::BK, mb * BM);
            stage = npre % STAGES;
            phase = (npre == STAGES) ? 1u : 0u;
            for (int i = npre; i < nk; ++i) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* st = tiles + stage * G::STAGE_BYTES;
                mbar_arrive_expect_tx(&full[stage], i < n1 ? WIDE_BYTES : HALF_BYTES);
                tma_load_2d(st, &tmA, &full[stage], kb_of(i) * G::BK, mb * BM);
                load_b(i, st);
                issued |= 1u << stage;
                last_par[stage] = phase;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                stop();
                const int zero = 0;
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s)) mbar_wait(&full[s], last_par[s], &zero);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = epi.idesc;  // M = 128, N = BN (set by the host)
            const uint32_t idesc_h = (idesc & ~(0x3Fu << 17)) | (static_cast<uint32_t>(HALF >> 3) << 17);
            const uint32_t d_own = tmem_base + rank * static_cast<uint32_t>(HALF);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int i = 0; i < nk; ++i) {
                if (!mbar_wait(&full[stage], phase, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u32(tiles + stage * G::STAGE_BYTES);
                const uint64_t da = sdesc_kmajor_sw128(st);
                const uint64_t db = sdesc_kmajor_sw128(st + G::A_TILE);
                if (i < n1) {
#pragma unroll
                    for (int k = 0; k < G::BK / G::UMMA_K; ++k) {
                        const uint64_t koff = static_cast<uint64_t>((k * G::UMMA_K) >> 4);
                        umma_i8(tmem_base, da + koff, db + koff, idesc, (i > 0 || k > 0) ? 1u : 0u);
                    }
                } else {
                    // Phase 2: the own columns only (initialised in phase 1).
#pragma unroll
                    for (int k = 0; k < G::BK / G::UMMA_K; ++k) {
                        const uint64_t koff = static_cast<uint64_t>((k * G::UMMA_K) >> 4);
                        umma_i8(d_own, da + koff, db + koff, idesc_h, 1u);
                    }
                }
                umma_commit(&empty[stage]);
                if (i == n1 - 1) umma_commit(pfull);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (ok) umma_commit(tfull);
            else stop();
            umma_commit(drain);
            const int zero = 0;
            mbar_wait(drain, 0, &zero);
        }
    } else {
        const int q = warp & 3;               // TMEM lane quarter
        const int etid = threadIdx.x - 64;
        const int grp = (warp - 2) >> 2;      // column group: chunks grp, grp + GROUPS, ...
        const int rl = q * 32 + lane;         // row within the tile = TMEM lane
        const int row = mb * BM + rl;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const int n_own = nb * BN + static_cast<int>(rank) * HALF;
        pdl_wait();  // parameters, and the output the previous kernel may read
        epi.prepare(params, n_own, HALF, etid, Cfg::EPI_THREADS);
        const bool got = mbar_wait(pfull, 0, abort_flag);
        // Publishes the staged parameters; uniform stop decision.
        bool bad = epi_barrier_or(!got || *abort_flag != 0, Cfg::EPI_THREADS);
        uint4 p[NCH][8];  // the peer's partial of this thread's row, its chunks
        if (!bad) {
            tc_fence_after();
            // The peer's columns of this CTA's partial into this CTA's slot:
            // granule (c*8 + j) of row rl at [(c*8 + j) * 128 + rl], so a
            // warp's 16-byte stores (and the peer's loads) cover 512
            // consecutive bytes.  Kept in L2 (.cg).  Phase 2's MMAs are
            // still accumulating the own columns meanwhile.
            uint4* out = xchg + static_cast<int64_t>(2 * unit + static_cast<int>(rank)) * Cfg::XGRAN;
#pragma unroll 1
            for (int c = grp; c < HALF / 32; c += GROUPS) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + lane_off + static_cast<uint32_t>(peer * HALF + c * 32), v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    __stcg(out + (c * 8 + j) * BM + rl, make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
            }
            cluster_ready();
            // Each thread releases its own stores to the peer (cluster scope
            // covers the global stores of both CTAs' threads).
            mbar_arrive_cluster(mapa_shared(smem_u32(xdone), peer));
            const bool received = mbar_wait_cluster(xdone, 0, abort_flag);
            if (received) {
                // The peer's partial into registers while the own half may
                // still be accumulating.
                const uint4* in = xchg + static_cast<int64_t>(2 * unit + static_cast<int>(peer)) * Cfg::XGRAN;
#pragma unroll
                for (int h = 0; h < NCH; ++h)
#pragma unroll
                    for (int j = 0; j < 8; ++j) p[h][j] = __ldcg(in + ((grp + GROUPS * h) * 8 + j) * BM + rl);
            }
            const bool own = received && mbar_wait(tfull, 0, abort_flag);
            bad = epi_barrier_or(!own || *abort_flag != 0, Cfg::EPI_THREADS);
        }
        if (!bad) {
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < NCH; ++h) {
                const int c = grp + GROUPS * h;
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + lane_off + static_cast<uint32_t>(rank * HALF + c * 32), v);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    v[4 * j] += p[h][j].x;
                    v[4 * j + 1] += p[h][j].y;
                    v[4 * j + 2] += p[h][j].z;
                    v[4 * j + 3] += p[h][j].w;
                }
                epi.store(params, HALF, row, n_own + c * 32, c * 32, 0, v);
            }
        } else if (etid == 0) {
            stop();
        }
    }

    cluster_ready();
    __syncthreads();
    tc_fence_before();
    // Neither CTA exits while the other may still arrive on its barriers or
    // write its abort word.  A thread that wrote the peer's abort word
    // releases it; the others' remote arrivals were all consumed by the
    // peer's waits, so their arrival needs no release (which would also wait
    // for this CTA's output stores).
    if (stopped) cluster_arrive_release();
    else cluster_arrive_relaxed();
    cluster_wait_acquire();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, BN);
    }
}

}  // namespace pfrt
