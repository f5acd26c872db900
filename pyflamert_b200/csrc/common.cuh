// common.cuh -- sm_100a building blocks shared by the kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (UMMA) issue, TMEM allocation and
// loads, and the shared-memory matrix descriptor.
//
// Every wait here is bounded: a wait that does not complete within
// kWaitLimitNs (or kWaitLimitIters polls) reports failure instead of spinning
// forever, so a kernel can record an error flag and return.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace pfrt {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr uint32_t kWaitLimitIters = 1u << 26;

// Device error codes written to the context's error word.
enum DeviceError : int {
    kDevOk = 0,
    kDevWaitTimeout = 1,   // an mbarrier wait gave up
    kDevBadIndex = 2,      // a CSR index outside its bounds was skipped
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false when
// the wait gives up (time or poll limit) or when *abort becomes non-zero.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          const volatile int* abort) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1; it < kWaitLimitIters; ++it) {
        if (mbar_try_wait(a, parity)) return true;
        if ((it & 31u) == 0) {
            if (*abort) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) return false;
        }
    }
    return false;
}

// ------------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization may start before
// the previous kernel on its stream has finished.  pdl_wait() blocks until
// that kernel has completed and its memory is visible; it must precede every
// read of data the previous kernel may write and every write the previous
// kernel may read.  pdl_launch_dependents() lets the next such kernel start.
// Both are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------- cp.async, ld
// 16-byte asynchronous global -> shared copy (both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 16-byte read-only global loads, written so that a batch of them is issued
// back to back before the first use.
__device__ __forceinline__ int4 ldg_nc_v4s32(const int32_t* p) {
    int4 r;
    asm volatile("ld.global.nc.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ float4 ldg_nc_v4f32(const float* p) {
    float4 r;
    asm volatile("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

// ------------------------------------------------- system-scope flags
// Release/acquire accesses of 32-bit flags that other GPUs write or read over
// NVLink (peer mappings), and a bounded wait on them.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until flags[i] has reached e (modulo 2^32) for every i < n (n <= 8).
// Each poll reads all n flags with relaxed system-scope loads, issued
// together; once all have reached e, one acquire fence at system scope orders
// the caller's later accesses after the writers' releases.  Gives up after
// kWaitLimitNs, or as soon as *abort is non-zero; returns false then.
__device__ __forceinline__ bool wait_flags_reached(const uint32_t* flags, int n, uint32_t e,
                                                   const uint32_t* abort) {
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        uint32_t v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < n) asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v[i]) : "l"(flags + i) : "memory");
        bool all = true;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < n) all &= static_cast<int32_t>(v[i] - e) >= 0;
        if (all) {
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            return true;
        }
        if ((it & 63u) == 63u) {
            if (ld_relaxed_gpu(abort) != 0) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs || it > kWaitLimitIters) return false;
        }
        __nanosleep(20);
    }
}

// ----------------------------------------------------------------------- TMA
// 2-D tiled load of one box into shared memory, completing on `bar` with the
// box's byte count.  Every CTA loads its own tiles.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tm,
                                            uint64_t* bar, int32_t c_inner, int32_t c_outer) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c_inner), "r"(c_outer)
        : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(slot_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued
// before it has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, both K-major; int8/uint8 inputs, s32 accumulate.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Same with tf32 inputs (fp32 storage, low mantissa bits not used), f32 accumulate.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Loads 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms
// stacked densely.  Fields: start address >> 4 [0,14); leading byte offset
// (unused for swizzled K-major, 1) [16,30); stride byte offset 1024 >> 4
// [32,46); descriptor version 1 [46,48); layout SWIZZLE_128B = 2 [61,64).
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor (kind::i8 / kind::tf32 / kind::f16 layout):
// D format [4,6) (1 = f32, 2 = s32); A format [7,10); B format [10,13)
// (i8: 0 unsigned, 1 signed; tf32: 2); A/B major [15],[16] (0 = K-major);
// N >> 3 [17,23); M >> 4 [24,29).
__host__ __device__ constexpr uint32_t idesc_make(uint32_t d_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                                  uint32_t m, uint32_t n) {
    return (d_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Records the first device error into the context's error word.
__device__ __forceinline__ void report_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

}  // namespace pfrt
