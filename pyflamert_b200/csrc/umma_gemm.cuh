// umma_gemm.cuh -- persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M,N] = A[M,K] * B[N,K]^T      (both operands K-major in global memory)
//
// One CTA per SM, 320 threads:
//   warp 0      TMA producer   (one lane)  -- global -> shared, STAGES-deep ring
//   warp 1      MMA issuer     (one lane)  -- tcgen05.mma into TMEM; also owns
//                                             the TMEM allocation
//   warps 2..9  epilogue       (256 threads) -- tcgen05.ld TMEM -> registers,
//                                             fused epilogue, global stores.
//               Two warps per TMEM lane quarter (a warp may only read the
//               32 TMEM lanes of its warp-id % 4), each taking half of the
//               tile's columns, so every SM sub-partition runs two epilogue
//               warps.  Per-column epilogue parameters are staged in shared
//               memory once per tile.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of one tile overlaps the MMAs of the next.
//
// Two element kinds share the pipeline:
//   KIND_I8    A uint8/int8, B int8, s32 accumulate; BK = 128 bytes = 128 elems,
//              UMMA K = 32, one A and one B tile per stage.
//   KIND_TF32X3  fp32 operands pre-split into hi/lo tf32 parts; per UMMA K-step
//              three MMAs lo*hi + hi*lo + hi*hi (the "3xTF32" scheme) so the
//              product keeps ~fp32 accuracy; BK = 32 elems, UMMA K = 8, two A
//              and two B tiles per stage.
//
// Work unit = (m block, n block, k split).  With k_splits > 1 the epilogue
// writes raw partial accumulators and a separate reduction applies the final
// epilogue.  Narrow tail (KIND_I8, one split): when the tiles do not fill
// the last wave of the persistent grid, the units past `wide_units` are
// half-width tiles (BN/2 columns, one MMA of N = BN/2 per K step) so the
// last wave's work is spread over twice as many CTAs; their B tiles come
// through tmB1, a tensor map of B with a BN/2-row box.  No cluster launch: each CTA loads its own
// tiles, so the same binary is safe in multi-GPU jobs.
#pragma once

#include "common.cuh"

namespace pfrt {

constexpr int KIND_I8 = 0;
constexpr int KIND_TF32X3 = 1;

struct GemmSched {
    int num_m_blk;
    int num_n_blk;
    int splits;        // k splits per (m,n) tile
    int kb_total;      // number of BK blocks covering K
    int kb_per_split;  // BK blocks per split (the last split may have fewer)
    int num_units;     // wide_units + 2 * (tiles past wide_units) with a narrow tail, else
                       // num_m_blk * num_n_blk * splits
    int wide_units;    // units [0, wide_units) are full-width tiles; the rest are half tiles
};

template <int KIND, int BN, int STAGES>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BK_BYTES = 128;
    static constexpr int ELEM = (KIND == KIND_I8) ? 1 : 4;
    static constexpr int BK = BK_BYTES / ELEM;
    static constexpr int UMMA_K = (KIND == KIND_I8) ? 32 : 8;
    static constexpr int NPARTS = (KIND == KIND_I8) ? 1 : 2;
    static constexpr int A_TILE = BM * BK_BYTES;
    static constexpr int B_TILE = BN * BK_BYTES;
    static constexpr int STAGE_BYTES = NPARTS * (A_TILE + B_TILE);
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr int BAR_BYTES = 256;
    static constexpr int EPI_WARPS = 8;
    static constexpr int EPI_THREADS = 32 * EPI_WARPS;
    // fp32 (3xTF32) accumulation: the tensor core's fp32 accumulator is not
    // an IEEE round-to-nearest sum, and its error grows with the number of
    // K steps it adds up.  So the MMAs accumulate PROMOTE_KB k-blocks
    // (PROMOTE_KB * BK = 128 K elements) into TMEM, and the epilogue adds each
    // such partial into fp32 registers with IEEE adds.  int8 accumulation is
    // exact, so one TMEM accumulation covers the whole K range.
    static constexpr bool PROMOTE = (KIND == KIND_TF32X3);
    // Per-column parameters: up to 4 words per column, one buffer per tile
    // in flight.  With one accumulation per tile, two buffers let the
    // epilogue stage the next tile's parameters while that tile's MMAs run.
    static constexpr int PARAM_BUF = 16 * BN;
    static constexpr int PARAM_BYTES = PROMOTE ? PARAM_BUF : 2 * PARAM_BUF;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + PARAM_BYTES + 1024;
    static constexpr int THREADS = 64 + EPI_THREADS;
    static constexpr int PROMOTE_KB = 4;
    static constexpr int CHUNK_KB = PROMOTE ? PROMOTE_KB : (1 << 30);
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM columns must be a power of two");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
    static_assert(STAGES <= 8, "stages");
};

__device__ __forceinline__ void decode_unit(const GemmSched& s, int unit, int& mb, int& nb, int& ks) {
    ks = unit % s.splits;
    const int t = unit / s.splits;
    mb = t % s.num_m_blk;
    nb = t / s.num_m_blk;
}

// Unit -> (m block, first column n0, width, k split).  Full-width units cover
// columns [nb*BN, nb*BN + BN); the half tiles of the narrow tail (one split)
// cover [nb*BN + h*BN/2, +BN/2) for h = 0, 1.
template <int BN>
__device__ __forceinline__ void decode_unit_w(const GemmSched& s, int unit, int& mb, int& n0, int& width,
                                              int& ks) {
    int nb;
    if (unit < s.wide_units) {
        decode_unit(s, unit, mb, nb, ks);
        n0 = nb * BN;
        width = BN;
    } else {
        const int v = unit - s.wide_units;
        decode_unit(s, s.wide_units + (v >> 1), mb, nb, ks);
        n0 = nb * BN + (v & 1) * (BN / 2);
        width = BN / 2;
    }
}

// Epi must provide:
//   __device__ void prepare(uint8_t* params, int n0, int bn, int tid, int nthreads) const;
//       stage the per-column parameters of columns [n0, n0 + bn) (called by
//       all epilogue threads, ahead of the tile's accumulator wait where the
//       kernel double-buffers them; params holds 16*bn bytes)
//   __device__ void store(const uint8_t* params, int bn, int row, int col0, int c_local,
//                         int ks, const uint32_t (&acc)[32]) const;
//       row is the global row of this thread; col0 (= n0 + c_local) the first
//       of 32 consecutive global columns held in acc (raw 32-bit accumulator bits).

// Named barrier over the epilogue warps that also ORs a predicate across
// them, so a stop decision is the same in every epilogue warp.
__device__ __forceinline__ bool epi_barrier_or(bool pred, int nthreads) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(out)
        : "r"(pred ? 1u : 0u), "r"(nthreads)
        : "memory");
    return out != 0;
}

__device__ __forceinline__ void epi_barrier(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

template <int KIND, int BN, int STAGES, class Epi>
__global__ void __launch_bounds__(64 + 32 * GemmCfg<KIND, BN, STAGES>::EPI_WARPS, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA0,
                     const __grid_constant__ CUtensorMap tmB0,
                     const __grid_constant__ CUtensorMap tmA1,
                     const __grid_constant__ CUtensorMap tmB1, const GemmSched sched,
                     const Epi epi, int* err) {
    using Cfg = GemmCfg<KIND, BN, STAGES>;
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

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], Cfg::EPI_THREADS);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Every CTA is resident (persistent grid), so the next kernel may launch
    // now; its CTAs wait in pdl_wait until this grid completes.
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tmA0);
            tma_prefetch_desc(&tmB0);
            if (Cfg::NPARTS == 2) {
                tma_prefetch_desc(&tmA1);
                tma_prefetch_desc(&tmB1);
            }
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;          // stages with a load issued
            uint32_t last_par[STAGES];    // parity of the last load issued per stage
            bool ok = true;
            pdl_wait();  // A (and B, C) may come from the previous kernel
            for (int unit = blockIdx.x; ok && unit < sched.num_units; unit += gridDim.x) {
                int mb, n0, width, ks;
                decode_unit_w<BN>(sched, unit, mb, n0, width, ks);
                const int kb0 = ks * sched.kb_per_split;
                const int kb1 = min(kb0 + sched.kb_per_split, sched.kb_total);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = tiles + stage * Cfg::STAGE_BYTES;
                    const int kx = kb * Cfg::BK;
                    if constexpr (Cfg::NPARTS == 2) {
                        mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
                        tma_load_2d(st, &tmA0, &full[stage], kx, mb * BM);
                        tma_load_2d(st + 2 * Cfg::A_TILE, &tmB0, &full[stage], kx, n0);
                        tma_load_2d(st + Cfg::A_TILE, &tmA1, &full[stage], kx, mb * BM);
                        tma_load_2d(st + 2 * Cfg::A_TILE + Cfg::B_TILE, &tmB1, &full[stage], kx, n0);
                    } else {
                        const bool narrow = width != BN;
                        mbar_arrive_expect_tx(&full[stage], narrow ? Cfg::A_TILE + Cfg::B_TILE / 2
                                                                   : Cfg::STAGE_BYTES);
                        tma_load_2d(st, &tmA0, &full[stage], kx, mb * BM);
                        tma_load_2d(st + Cfg::A_TILE, narrow ? &tmB1 : &tmB0, &full[stage], kx, n0);
                    }
                    issued |= 1u << stage;
                    last_par[stage] = phase;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                // Let every copy already issued land before the CTA can exit.
                const int zero = 0;
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s)) mbar_wait(&full[s], last_par[s], &zero);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t idesc_w;
            if constexpr (KIND == KIND_I8) idesc_w = epi.idesc;
            else idesc_w = idesc_make(1, 2, 2, BM, BN);
            // Same descriptor with N = BN/2 (bits 17..22 hold N >> 3).
            const uint32_t idesc_n = (idesc_w & ~(0x3Fu << 17)) | (static_cast<uint32_t>((BN / 2) >> 3) << 17);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int t = 0;  // accumulation chunks issued so far (selects the TMEM slot)
            for (int unit = blockIdx.x; ok && unit < sched.num_units; unit += gridDim.x) {
                int mb, n0, width, ks;
                decode_unit_w<BN>(sched, unit, mb, n0, width, ks);
                const uint32_t idesc = (width == BN) ? idesc_w : idesc_n;
                const int kb0 = ks * sched.kb_per_split;
                const int kb1 = min(kb0 + sched.kb_per_split, sched.kb_total);
                for (int kc = kb0; ok && kc < kb1; kc += Cfg::CHUNK_KB, ++t) {
                    const int kce = min(kc + Cfg::CHUNK_KB, kb1);
                    const int slot = t & 1;
                    const uint32_t ap = static_cast<uint32_t>(t >> 1) & 1u;
                    if (!mbar_wait(&tempty[slot], ap ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * BN);
                    for (int kb = kc; kb < kce; ++kb) {
                        if (!mbar_wait(&full[stage], phase, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t st = smem_u32(tiles + stage * Cfg::STAGE_BYTES);
                        if constexpr (KIND == KIND_I8) {
                            const uint64_t da = sdesc_kmajor_sw128(st);
                            const uint64_t db = sdesc_kmajor_sw128(st + Cfg::A_TILE);
#pragma unroll
                            for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
                                const uint64_t koff = static_cast<uint64_t>((k * Cfg::UMMA_K * Cfg::ELEM) >> 4);
                                umma_i8(d_tmem, da + koff, db + koff, idesc, (kb > kc || k > 0) ? 1u : 0u);
                            }
                        } else {
                            const uint64_t dah = sdesc_kmajor_sw128(st);
                            const uint64_t dal = sdesc_kmajor_sw128(st + Cfg::A_TILE);
                            const uint64_t dbh = sdesc_kmajor_sw128(st + 2 * Cfg::A_TILE);
                            const uint64_t dbl = sdesc_kmajor_sw128(st + 2 * Cfg::A_TILE + Cfg::B_TILE);
#pragma unroll
                            for (int k = 0; k < Cfg::BK / Cfg::UMMA_K; ++k) {
                                const uint64_t koff = static_cast<uint64_t>((k * Cfg::UMMA_K * Cfg::ELEM) >> 4);
                                const uint32_t acc0 = (kb > kc || k > 0) ? 1u : 0u;
                                umma_tf32(d_tmem, dal + koff, dbh + koff, idesc, acc0);
                                umma_tf32(d_tmem, dah + koff, dbl + koff, idesc, 1u);
                                umma_tf32(d_tmem, dah + koff, dbh + koff, idesc, 1u);
                            }
                        }
                        umma_commit(&empty[stage]);
                        if (++stage == STAGES) {
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
            // Every MMA issued so far must finish before TMEM is released.
            umma_commit(drain);
            const int zero = 0;
            mbar_wait(drain, 0, &zero);
        }
    } else {
        const int q = warp & 3;                    // TMEM lane quarter this warp may access
        const int etid = threadIdx.x - 64;         // 0 .. EPI_THREADS-1
        pdl_wait();  // bias/rowsum/C reads and the output writes follow the previous kernel
        const int half = (warp - 2) >> 2;          // which half of the tile's columns
        constexpr int CHUNKS = BN / 32 / 2;        // 32-column chunks per warp
        int t = 0;                                 // accumulation chunks consumed so far
        if constexpr (!Cfg::PROMOTE) {
            // The first tile's parameters, staged while its MMAs run (the
            // accumulator wait's barrier publishes them).
            if (static_cast<int>(blockIdx.x) < sched.num_units) {
                int mb, n0, width, ks;
                decode_unit_w<BN>(sched, blockIdx.x, mb, n0, width, ks);
                epi.prepare(params, n0, width, etid, Cfg::EPI_THREADS);
            }
        }
        for (int unit = blockIdx.x; unit < sched.num_units; unit += gridDim.x) {
            int mb, n0, width, ks;
            decode_unit_w<BN>(sched, unit, mb, n0, width, ks);
            const int kb0 = ks * sched.kb_per_split;
            const int kb1 = min(kb0 + sched.kb_per_split, sched.kb_total);
            const int row = mb * BM + q * 32 + lane;
            const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
            if constexpr (Cfg::PROMOTE) {
                // Sum the TMEM partials of every chunk into registers (IEEE fp32).
                float racc[CHUNKS][32];
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c)
#pragma unroll
                    for (int j = 0; j < 32; ++j) racc[c][j] = 0.0f;
                bool stop = false;
                for (int kc = kb0; kc < kb1; kc += Cfg::CHUNK_KB, ++t) {
                    const int slot = t & 1;
                    const uint32_t ap = static_cast<uint32_t>(t >> 1) & 1u;
                    const bool got = mbar_wait(&tfull[slot], ap, abort_flag);
                    if (epi_barrier_or(!got || *abort_flag != 0, Cfg::EPI_THREADS)) {
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t taddr = tmem_base + static_cast<uint32_t>(slot * BN) + lane_off;
#pragma unroll
                    for (int c = 0; c < CHUNKS; ++c) {
                        uint32_t v[32];
                        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>((half * CHUNKS + c) * 32), v);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; ++j) racc[c][j] = __fadd_rn(racc[c][j], __uint_as_float(v[j]));
                    }
                    tc_fence_before();
                    mbar_arrive(&tempty[slot]);
                }
                if (stop) {
                    *abort_flag = 1;
                    report_error(err, kDevWaitTimeout);
                    break;
                }
                // The barrier of the last chunk also ensures the previous tile's
                // parameters are no longer being read.
                epi.prepare(params, n0, BN, etid, Cfg::EPI_THREADS);
                epi_barrier(Cfg::EPI_THREADS);
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c) {
                    uint32_t bits[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) bits[j] = __float_as_uint(racc[c][j]);
                    const int cl = (half * CHUNKS + c) * 32;
                    epi.store(params, BN, row, n0 + cl, cl, ks, bits);
                }
                epi_barrier(Cfg::EPI_THREADS);  // parameters stay valid until every warp stored
            } else {
                const int slot = t & 1;
                const uint32_t ap = static_cast<uint32_t>(t >> 1) & 1u;
                const uint8_t* pcur = params + slot * Cfg::PARAM_BUF;  // staged before the wait
                ++t;
                const bool got = mbar_wait(&tfull[slot], ap, abort_flag);
                // Uniform stop decision across the epilogue warps.  The barrier
                // also publishes this tile's staged parameters, and every warp
                // passing it has finished the previous tile, whose parameter
                // buffer is restaged below.
                if (epi_barrier_or(!got || *abort_flag != 0, Cfg::EPI_THREADS)) {
                    *abort_flag = 1;
                    report_error(err, kDevWaitTimeout);
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + static_cast<uint32_t>(slot * BN) + lane_off;
                const int wchunks = width / 64;  // 32-column chunks per warp half
#pragma unroll 1
                for (int c = half * wchunks; c < (half + 1) * wchunks; ++c) {
                    uint32_t acc[32];
                    tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 32), acc);
                    tmem_ld_wait();
                    epi.store(pcur, width, row, n0 + c * 32, c * 32, ks, acc);
                }
                tc_fence_before();
                mbar_arrive(&tempty[slot]);
                const int next = unit + static_cast<int>(gridDim.x);
                if (next < sched.num_units) {
                    int mb2, n2, width2, ks2;
                    decode_unit_w<BN>(sched, next, mb2, n2, width2, ks2);
                    epi.prepare(params + (t & 1) * Cfg::PARAM_BUF, n2, width2, etid, Cfg::EPI_THREADS);
                }
            }
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

}  // namespace pfrt
