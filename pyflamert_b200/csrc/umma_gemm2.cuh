// umma_gemm2.cuh -- the int8 GEMM on CTA pairs (tcgen05 cta_group::2).
//
//   D[M,N] = A[M,K] * B[N,K]^T  (u8/s8 x s8 -> s32), both operands K-major.
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x BN tile:
// CTA r (r = 0, 1: its rank in the cluster) holds rows [256 mb + 128 r, +128)
// of A and rows [BN nb + r BN/2, +BN/2) of B in its own shared memory, and a
// single tcgen05.mma.cta_group::2 issued by CTA 0 (the leader) multiplies the
// whole 256 x BN x 32 step, reading both CTAs' shared memory; CTA r's TMEM
// receives the accumulator rows of its half of A, all BN columns.  Each SM
// thus pulls 128 + BN/2 rows per k-block for a 128 x BN accumulator instead of
// 128 + BN: a third less L2 -> SM traffic at BN = 256, the resource the
// one-CTA kernel runs short of.
//
// Roles (320 threads per CTA, as in umma_gemm.cuh):
//   warp 0      TMA producer of this CTA's A and B halves.  The copies use
//               the .cta_group::2 form and complete on the LEADER's full
//               barrier, which the leader's producer armed with both CTAs'
//               bytes.  Each CTA loads only its own halves.
//   warp 1      leader: MMA issuer; both CTAs: the TMEM allocation, made
//               jointly with cta_group::2.
//   warps 2..9  epilogue of this CTA's 128 rows (TMEM -> registers -> Epi).
// Hand-offs: the leader's MMA commits arrive on the empty[stage] and
// tfull[slot] barriers of both CTAs (one commit per CTA, addressed through
// the cluster window); every epilogue warp of both CTAs arrives
// on the leader's tempty[slot] (16 arrivals free a TMEM slot).
// Every mbarrier wait is bounded; a stop is propagated to the peer's abort
// word.  Both CTAs always reach the closing cluster barrier.
#pragma once

#include "umma_gemm.cuh"

namespace pfrt {

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the barrier at this shared-memory offset in both CTAs of
// the pair when the MMAs issued so far have completed: one commit to each
// CTA's barrier, addressed in the cluster's shared window.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
    const uint32_t own = smem_u32(bar);
#pragma unroll
    for (uint32_t r = 0; r < 2; ++r) {
        const uint32_t a = mapa_shared(own, r);
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(a)
                     : "memory");
    }
}

// 2-D tiled load into this CTA's shared memory, completing on the barrier at
// cluster address `bar_cluster` (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* tm, uint32_t bar_cluster,
                                                 int32_t c_inner, int32_t c_outer) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(c_inner), "r"(c_outer)
        : "memory");
}

template <int BN, int STAGES>
struct Gemm2Cfg {
    static constexpr int BM = 128;  // rows per CTA (256 per pair)
    static constexpr int BK_BYTES = 128;
    static constexpr int BK = 128;  // int8 elements
    static constexpr int UMMA_K = 32;
    static constexpr int BH = BN / 2;  // B rows per CTA
    static constexpr int A_TILE = BM * BK_BYTES;
    static constexpr int B_TILE = BH * BK_BYTES;
    static constexpr int STAGE_BYTES = A_TILE + B_TILE;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr int BAR_BYTES = 256;
    static constexpr int EPI_WARPS = 8;
    static constexpr int EPI_THREADS = 32 * EPI_WARPS;
    static constexpr int PARAM_BUF = 16 * BN;  // per-column parameters of one tile
    static constexpr int PARAM_BYTES = 2 * PARAM_BUF;  // the tile in the epilogue and the next
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + PARAM_BYTES + 1024;
    static constexpr int THREADS = 64 + EPI_THREADS;
    static_assert(BN == 128 || BN == 256, "pair tile width");
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM columns");
    static_assert(STAGES <= 8, "stages");
};

// Units are pair tiles (256 x BN); sched.num_m_blk counts 256-row blocks.
template <int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(64 + 32 * Gemm2Cfg<BN, STAGES>::EPI_WARPS, 1)
    umma_gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmSched sched, const Epi epi, int* err) {
    using Cfg = Gemm2Cfg<BN, STAGES>;
    constexpr int BM = Cfg::BM;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* tiles = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* params = smem + STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = static_cast<int>(cluster_id_x());
    const int npairs = static_cast<int>(nclusters_x());
    const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<int*>(abort_flag)), rank ^ 1u);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 2 * Cfg::EPI_WARPS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // Both CTAs' barriers exist before either can arrive on the other's.
    cluster_sync();
    if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) pdl_launch_dependents();
    auto stop = [&]() {
        *abort_flag = 1;
        st_cluster_u32(peer_abort, 1u);
        report_error(err, kDevWaitTimeout);
    };

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            // B is a prepared weight (written once at its creation, never by a
            // kernel): the first unit's first stages of B are requested
            // before the dependency wait, A (which the previous kernel may
            // write) after it.  The ring starts empty: no empty-barrier wait.
            int npre = 0;
            if (pair < sched.num_units) {
                int mb0, nb0, ks0;
                decode_unit(sched, pair, mb0, nb0, ks0);
                npre = min(STAGES, sched.kb_total);
                for (int i = 0; i < npre; ++i) {
                    const uint32_t fbar = mapa_shared(smem_u32(&full[i]), 0u);
                    if (leader) mbar_arrive_expect_tx(&full[i], 2 * Cfg::STAGE_BYTES);
                    tma_load_2d_pair(tiles + i * Cfg::STAGE_BYTES + Cfg::A_TILE, &tmB, fbar, i * Cfg::BK,
                                     nb0 * BN + static_cast<int>(rank) * Cfg::BH);
                }
                pdl_wait();
                for (int i = 0; i < npre; ++i) {
                    const uint32_t fbar = mapa_shared(smem_u32(&full[i]), 0u);
                    tma_load_2d_pair(tiles + i * Cfg::STAGE_BYTES, &tmA, fbar, i * Cfg::BK,
                                     mb0 * 2 * BM + static_cast<int>(rank) * BM);
                }
            } else {
                pdl_wait();
            }
            int stage = npre % STAGES;
            uint32_t phase = (npre == STAGES) ? 1u : 0u;
            bool ok = true;
            for (int unit = pair; ok && unit < sched.num_units; unit += npairs) {
                int mb, nb, ks;
                decode_unit(sched, unit, mb, nb, ks);
                for (int kb = (unit == pair) ? npre : 0; kb < sched.kb_total; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fbar = mapa_shared(smem_u32(&full[stage]), 0u);
                    if (leader) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
                    uint8_t* st = tiles + stage * Cfg::STAGE_BYTES;
                    const int kx = kb * Cfg::BK;
                    tma_load_2d_pair(st, &tmA, fbar, kx, mb * 2 * BM + static_cast<int>(rank) * BM);
                    tma_load_2d_pair(st + Cfg::A_TILE, &tmB, fbar, kx, nb * BN + static_cast<int>(rank) * Cfg::BH);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) stop();
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            const uint32_t idesc = epi.idesc;  // M = 256, N = BN (set by the host)
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int t = 0;
            for (int unit = pair; ok && unit < sched.num_units; unit += npairs, ++t) {
                const int slot = t & 1;
                const uint32_t ap = static_cast<uint32_t>(t >> 1) & 1u;
                if (!mbar_wait(&tempty[slot], ap ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * BN);
                for (int kb = 0; kb < sched.kb_total; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_u32(tiles + stage * Cfg::STAGE_BYTES);
                    const uint64_t da = sdesc_kmajor_sw128(st);
                    const uint64_t db = sdesc_kmajor_sw128(st + Cfg::A_TILE);
#pragma unroll
                    for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
                        const uint64_t koff = static_cast<uint64_t>((k * Cfg::UMMA_K) >> 4);
                        umma_i8_pair(d_tmem, da + koff, db + koff, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    umma_commit_pair(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit_pair(&tfull[slot]);
            }
            if (!ok) stop();
            // Every MMA issued so far must finish before TMEM is released.
            umma_commit_pair(drain);
            const int zero = 0;
            mbar_wait(drain, 0, &zero);
        }
    } else {
        const int q = warp & 3;
        const int etid = threadIdx.x - 64;
        const int half = (warp - 2) >> 2;
        constexpr int CHUNKS = BN / 32 / 2;
        pdl_wait();
        const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0u);
        const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty[1]), 0u);
        int t = 0;
        if (pair < sched.num_units) {
            // The first tile's parameters, staged while its MMAs run.
            int mb, nb, ks;
            decode_unit(sched, pair, mb, nb, ks);
            epi.prepare(params, nb * BN, BN, etid, Cfg::EPI_THREADS);
        }
        for (int unit = pair; unit < sched.num_units; unit += npairs, ++t) {
            int mb, nb, ks;
            decode_unit(sched, unit, mb, nb, ks);
            const int slot = t & 1;
            const uint8_t* pcur = params + slot * Cfg::PARAM_BUF;
            const uint32_t ap = static_cast<uint32_t>(t >> 1) & 1u;
            const bool got = mbar_wait(&tfull[slot], ap, abort_flag);
            // Also publishes this tile's staged parameters; every warp passing
            // it has finished the previous tile, whose buffer is restaged below.
            if (epi_barrier_or(!got || *abort_flag != 0, Cfg::EPI_THREADS)) {
                if (etid == 0) stop();
                break;
            }
            tc_fence_after();
            const int row = mb * 2 * BM + static_cast<int>(rank) * BM + q * 32 + lane;
            const uint32_t taddr =
                tmem_base + static_cast<uint32_t>(slot * BN) + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
            for (int c = half * CHUNKS; c < (half + 1) * CHUNKS; ++c) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 32), acc);
                tmem_ld_wait();
                epi.store(pcur, BN, row, nb * BN + c * 32, c * 32, 0, acc);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(slot ? tempty_leader1 : tempty_leader0);
            if (unit + npairs < sched.num_units) {
                int mb2, nb2, ks2;
                decode_unit(sched, unit + npairs, mb2, nb2, ks2);
                epi.prepare(params + (slot ^ 1) * Cfg::PARAM_BUF, nb2 * BN, BN, etid, Cfg::EPI_THREADS);
            }
        }
    }

    __syncthreads();
    // The leader's MMAs are drained (warp 1 waited above) before either CTA
    // releases TMEM or exits.
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    }
}

}  // namespace pfrt
