// epilogues.cuh -- fused epilogues of the tcgen05 GEMM (umma_gemm.cuh) and
// the matching split-K reductions.
//
// QEpi (int8 path) turns the raw s32 accumulator sum_k a*w into the
// reference's quantized linear result (src/quantization/quant_ops.cpp):
//   acc  = sum_k (a - a_zp)(w - w_zp)
//        = raw - a_zp*colsum[n] - w_zp*rowsum[m] + K*a_zp*w_zp   (exact, int64)
//   y    = (float)acc * (a_scale * w_scale[n])          quant_ops.cpp:435,464
//   y    = y + bias[n]                                  math.cpp:225 (fused Add)
//   y    = max(0, y)                                    activation.cpp:56 (fused Relu)
//   q    = clamp((int)round(y * (1/y_scale)) + y_zp)    quant_ops.cpp:42-55
// Every product and sum is rounded separately (__fmul_rn/__fadd_rn): no FMA
// contraction, so the result is bit-identical to the reference CPU code.
//
// FEpi (fp32 path) applies cpu_gemm's tail (src/backends/cpu/ops/math.cpp:
// 427-435): y = alpha*acc + beta*C[(m*N + n) % c_len].
#pragma once

#include "common.cuh"

namespace pfrt {

enum OutMode : int {
    kOutF32 = 0,      // fp32 (dequantized) output
    kOutS8 = 1,       // requantized int8
    kOutU8 = 2,       // requantized uint8
    kOutPartial = 3,  // raw split-K partial accumulators
};

// static_cast<int32_t>(float) as the reference's x86-64 build executes it
// (cvttss2si): a value outside the int32 range, or NaN, becomes INT32_MIN.
// The GPU's own conversion saturates instead, so the range test is explicit.
__device__ __forceinline__ int32_t f2i_like_x86(float r) {
    return (r >= -2147483648.0f && r < 2147483648.0f) ? static_cast<int32_t>(r) : INT32_MIN;
}

// (int32)std::round(t) as the reference's x86-64 build computes it, in three
// instructions.  std::round rounds half away from zero; for every float t,
// round(t) == trunc(t + copysign(p, t)) with p = 0.49999997f, the largest
// float below 1/2, when the addition rounds to nearest (p instead of 1/2 keeps
// t = 0.49999997 from rounding up, and the sum's own rounding carries exact
// halves away from zero).  The truncating conversion saturates: below -2^31
// it already gives INT32_MIN as cvttss2si does, and the `s < 2^31` test
// sends +2^31 and above, and NaN, to INT32_MIN.  Checked against
// f2i_like_x86(roundf(t)) for all 2^32 bit patterns of t.
__device__ __forceinline__ int32_t round_to_i32_like_x86(float t) {
    const float p = __int_as_float(0x3EFFFFFF | (__float_as_int(t) & static_cast<int>(0x80000000u)));
    const float s = __fadd_rn(t, p);
    return (s < 2147483648.0f) ? __float2int_rz(s) : INT32_MIN;
}

// quant_ops.cpp:44-46: clamp((int32)std::round(y * inv_scale) + zp, qmin, qmax),
// with the int32 addition wrapping as it does on the reference's target.
__device__ __forceinline__ int32_t requant_rn(float y, float inv_scale, int32_t zp, bool u8) {
    const int32_t r = round_to_i32_like_x86(__fmul_rn(y, inv_scale));
    const int32_t q = static_cast<int32_t>(static_cast<uint32_t>(r) + static_cast<uint32_t>(zp));
    return u8 ? min(max(q, 0), 255) : min(max(q, -128), 127);
}

// requant_rn with zp == 0 in one saturating conversion: for s < 2^31,
// clamp((int32)trunc(s), qmin, qmax) is cvt.rzi.sat to the 8-bit type (which
// also sends -inf and everything below qmin to qmin); s >= 2^31 and NaN, which
// the reference's conversion turns into INT32_MIN, clamp to qmin as well.
template <bool U8>
__device__ __forceinline__ int32_t requant_rn_zp0(float y, float inv_scale) {
    const float t = __fmul_rn(y, inv_scale);
    const float p = __int_as_float(0x3EFFFFFF | (__float_as_int(t) & static_cast<int>(0x80000000u)));
    const float s = __fadd_rn(t, p);
    int32_t q;
    if constexpr (U8) asm("cvt.rzi.sat.u8.f32 %0, %1;" : "=r"(q) : "f"(s));
    else asm("cvt.rzi.sat.s8.f32 %0, %1;" : "=r"(q) : "f"(s));
    return (s < 2147483648.0f) ? q : (U8 ? 0 : -128);
}

// Low bytes of four values packed little-endian into one word.
__device__ __forceinline__ uint32_t pack_bytes4(int32_t a, int32_t b, int32_t c, int32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

struct QEpi {
    uint32_t idesc;
    int M, N, K;
    int a_zp, w_zp;
    float a_scale;
    const int32_t* colsum;  // [Npad] sum_k W[n,k]
    const int32_t* rowsum;  // [M] sum_k A[m,k]; only read when w_zp != 0
    const float* w_scale;   // [Npad]
    const float* bias;      // [N] or null
    int relu;
    int out_mode;
    float inv_y_scale;
    int y_zp;
    void* out;
    int64_t ldo;            // output row stride, elements
    int32_t* acc_out;       // [M, N] exact accumulators, or null
    int32_t* partial;       // [splits][M][N] when out_mode == kOutPartial
    int vec_ok;             // output rows 16-byte aligned for vector stores
    int acc_vec_ok;         // acc_out 16-byte aligned and N % 4 == 0
    int fast32;             // every intermediate of the zero-point correction fits in int32

    // Exact accumulator and dequantized/biased/activated value of one element.
    __device__ __forceinline__ float finalize(int row, int n, int64_t raw, int32_t rs,
                                              int32_t& acc_true) const {
        int64_t a = raw - static_cast<int64_t>(a_zp) * colsum[n];
        if (w_zp != 0)
            a += static_cast<int64_t>(K) * a_zp * w_zp - static_cast<int64_t>(w_zp) * rs;
        acc_true = static_cast<int32_t>(a);
        float y = __fmul_rn(__ll2float_rn(a), __fmul_rn(a_scale, w_scale[n]));
        if (bias != nullptr && n < N) y = __fadd_rn(y, bias[n]);
        if (relu) y = (0.0f < y) ? y : 0.0f;
        return y;
    }

    // Writes W consecutive outputs (and accumulators) of one row; W is 32 in
    // the GEMM epilogue and 4 in the split-K reduction.
    template <int W>
    __device__ __forceinline__ void emit(int row, int col0, const int32_t (&at)[W],
                                         const float (&y)[W]) const {
        const bool full = (col0 + W <= N);
        if (acc_out != nullptr) {
            int32_t* d = acc_out + static_cast<int64_t>(row) * N + col0;
            if (full && acc_vec_ok) {
#pragma unroll
                for (int j = 0; j < W; j += 4)
                    *reinterpret_cast<int4*>(d + j) = make_int4(at[j], at[j + 1], at[j + 2], at[j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < W; ++j)
                    if (col0 + j < N) d[j] = at[j];
            }
        }
        if (out_mode == kOutF32) {
            float* d = static_cast<float*>(out) + static_cast<int64_t>(row) * ldo + col0;
            if (full && vec_ok) {
#pragma unroll
                for (int j = 0; j < W; j += 4)
                    *reinterpret_cast<float4*>(d + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < W; ++j)
                    if (col0 + j < N) d[j] = y[j];
            }
        } else {
            const bool u8 = (out_mode == kOutU8);
            uint8_t* d = static_cast<uint8_t*>(out) + static_cast<int64_t>(row) * ldo + col0;
            uint32_t packed[W / 4];
#pragma unroll
            for (int w = 0; w < W / 4; ++w)
                packed[w] = pack_bytes4(requant_rn(y[4 * w], inv_y_scale, y_zp, u8),
                                        requant_rn(y[4 * w + 1], inv_y_scale, y_zp, u8),
                                        requant_rn(y[4 * w + 2], inv_y_scale, y_zp, u8),
                                        requant_rn(y[4 * w + 3], inv_y_scale, y_zp, u8));
            if constexpr (W == 32) {
                if (full && vec_ok) {
                    *reinterpret_cast<uint4*>(d) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                    *reinterpret_cast<uint4*>(d + 16) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                    return;
                }
            }
#pragma unroll
            for (int j = 0; j < W; ++j)
                if (col0 + j < N) d[j] = static_cast<uint8_t>((packed[j >> 2] >> (8 * (j & 3))) & 0xFFu);
        }
    }

    // Per-column parameters of one tile, in shared memory (4*bn bytes each):
    // zc[i] = a_zp * colsum[n] (valid when fast32), os[i] = a_scale * w_scale[n],
    // b[i] = bias[n] (0 past N or without bias).
    __device__ __forceinline__ void prepare(uint8_t* p, int n0, int bn, int tid, int nthreads) const {
        int32_t* zc = reinterpret_cast<int32_t*>(p);
        float* os = reinterpret_cast<float*>(p + 4 * bn);
        float* b = reinterpret_cast<float*>(p + 8 * bn);
        for (int i = tid; i < bn; i += nthreads) {
            const int n = n0 + i;
            zc[i] = a_zp * colsum[n];
            os[i] = __fmul_rn(a_scale, w_scale[n]);
            b[i] = (bias != nullptr && n < N) ? bias[n] : 0.0f;
        }
    }

    __device__ __forceinline__ void store_partial(int row, int col0, int ks, const uint32_t (&acc)[32]) const {
        int32_t* d = partial + (static_cast<int64_t>(ks) * M + row) * N + col0;
        if (col0 + 32 <= N && (N % 4) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<int4*>(d + j) =
                    make_int4(static_cast<int>(acc[j]), static_cast<int>(acc[j + 1]),
                              static_cast<int>(acc[j + 2]), static_cast<int>(acc[j + 3]));
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < N) d[j] = static_cast<int32_t>(acc[j]);
        }
    }

    // The requantized int8/uint8 tile row (no accumulator copy, int32-exact
    // zero-point correction): the common case, specialised on the fused
    // bias, ReLU, output type and a zero output zero-point (Z0: one
    // saturating conversion instead of truncation, offset and clamp), so each
    // output costs ~11-15 instructions.
    template <bool HB, bool RL, bool U8, bool Z0>
    __device__ __forceinline__ void store_q8(const uint8_t* p, int bn, int row, int col0, int cl, int32_t rterm,
                                             const uint32_t (&acc)[32]) const {
        const int4* zc4 = reinterpret_cast<const int4*>(p) + cl / 4;
        const float4* os4 = reinterpret_cast<const float4*>(p + 4 * bn) + cl / 4;
        const float4* b4 = reinterpret_cast<const float4*>(p + 8 * bn) + cl / 4;
        uint32_t packed[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const int4 z = zc4[v];
            const float4 o = os4[v];
            const int zz[4] = {z.x, z.y, z.z, z.w};
            const float oo[4] = {o.x, o.y, o.z, o.w};
            float bb[4] = {0.f, 0.f, 0.f, 0.f};
            if constexpr (HB) {
                const float4 b = b4[v];
                bb[0] = b.x; bb[1] = b.y; bb[2] = b.z; bb[3] = b.w;
            }
            int32_t q[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int32_t a = static_cast<int32_t>(acc[4 * v + u]) - zz[u] - rterm;
                float t = __fmul_rn(__int2float_rn(a), oo[u]);
                if constexpr (HB) t = __fadd_rn(t, bb[u]);
                // max(0, t) as activation.cpp:56 computes it, up to the sign of
                // a zero result, which the integer conversion below discards.
                if constexpr (RL) t = fmaxf(t, 0.0f);
                if constexpr (Z0) q[u] = requant_rn_zp0<U8>(t, inv_y_scale);
                else q[u] = requant_rn(t, inv_y_scale, y_zp, U8);
            }
            packed[v] = pack_bytes4(q[0], q[1], q[2], q[3]);
        }
        uint8_t* d = static_cast<uint8_t*>(out) + static_cast<int64_t>(row) * ldo + col0;
        if (col0 + 32 <= N && vec_ok) {
            *reinterpret_cast<uint4*>(d) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            *reinterpret_cast<uint4*>(d + 16) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < N) d[j] = static_cast<uint8_t>((packed[j >> 2] >> (8 * (j & 3))) & 0xFFu);
        }
    }

    template <bool Z0>
    __device__ __forceinline__ void store_q8_sel(const uint8_t* p, int bn, int row, int col0, int cl,
                                                 int32_t rterm, const uint32_t (&acc)[32], bool u8) const {
        if (bias != nullptr) {
            if (relu) u8 ? store_q8<true, true, true, Z0>(p, bn, row, col0, cl, rterm, acc)
                         : store_q8<true, true, false, Z0>(p, bn, row, col0, cl, rterm, acc);
            else u8 ? store_q8<true, false, true, Z0>(p, bn, row, col0, cl, rterm, acc)
                    : store_q8<true, false, false, Z0>(p, bn, row, col0, cl, rterm, acc);
        } else {
            if (relu) u8 ? store_q8<false, true, true, Z0>(p, bn, row, col0, cl, rterm, acc)
                         : store_q8<false, true, false, Z0>(p, bn, row, col0, cl, rterm, acc);
            else u8 ? store_q8<false, false, true, Z0>(p, bn, row, col0, cl, rterm, acc)
                    : store_q8<false, false, false, Z0>(p, bn, row, col0, cl, rterm, acc);
        }
    }

    __device__ __forceinline__ void store(const uint8_t* p, int bn, int row, int col0, int cl, int ks,
                                          const uint32_t (&acc)[32]) const {
        if (row >= M) return;
        if (out_mode == kOutPartial) {
            store_partial(row, col0, ks, acc);
            return;
        }
        int32_t at[32];
        float y[32];
        const int32_t rs = (w_zp != 0) ? rowsum[row] : 0;
        if (fast32 && out_mode != kOutF32 && acc_out == nullptr) {
            const int32_t rterm = (w_zp != 0) ? w_zp * rs - K * a_zp * w_zp : 0;
            const bool u8 = (out_mode == kOutU8);
            if (y_zp == 0) store_q8_sel<true>(p, bn, row, col0, cl, rterm, acc, u8);
            else store_q8_sel<false>(p, bn, row, col0, cl, rterm, acc, u8);
            return;
        }
        if (fast32) {
            // Exact in int32: the host checked that no intermediate can overflow.
            const int32_t rterm = (w_zp != 0) ? w_zp * rs - K * a_zp * w_zp : 0;
            const int4* zc4 = reinterpret_cast<const int4*>(p) + cl / 4;
            const float4* os4 = reinterpret_cast<const float4*>(p + 4 * bn) + cl / 4;
            const float4* b4 = reinterpret_cast<const float4*>(p + 8 * bn) + cl / 4;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const int4 z = zc4[v];
                const float4 o = os4[v];
                const int zz[4] = {z.x, z.y, z.z, z.w};
                const float oo[4] = {o.x, o.y, o.z, o.w};
                float bb[4] = {0.f, 0.f, 0.f, 0.f};
                if (bias != nullptr) {
                    const float4 b = b4[v];
                    bb[0] = b.x; bb[1] = b.y; bb[2] = b.z; bb[3] = b.w;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = 4 * v + u;
                    const int32_t a = static_cast<int32_t>(acc[j]) - zz[u] - rterm;
                    at[j] = a;
                    float t = __fmul_rn(__int2float_rn(a), oo[u]);
                    if (bias != nullptr) t = __fadd_rn(t, bb[u]);
                    if (relu) t = (0.0f < t) ? t : 0.0f;
                    y[j] = t;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                y[j] = finalize(row, col0 + j, static_cast<int64_t>(static_cast<int32_t>(acc[j])), rs, at[j]);
        }
        emit<32>(row, col0, at, y);
    }
};

constexpr int kMaxPeerOut = 7;

struct FEpi {
    int M, N;
    float alpha, beta;
    const float* C;   // bias operand, flat length c_len, or null
    int64_t c_len;
    float* out;
    int64_t ldo;
    int out_mode;     // kOutF32 or kOutPartial
    float* partial;   // [splits][M][N]
    int vec_ok;
    // Further copies of the output written by the same stores: other GPUs'
    // outputs mapped into this process (the sharded SpMM's all-gather), same
    // row stride and offsets as `out`.
    int n_peer_out;
    float* peer_out[kMaxPeerOut];

    __device__ __forceinline__ float finalize(int row, int n, float acc) const {
        float y = __fmul_rn(alpha, acc);
        if (C != nullptr && n < N) {
            const int64_t flat = static_cast<int64_t>(row) * N + n;
            const int64_t ci = (c_len == N) ? n : (c_len == 1 ? 0 : flat % c_len);
            y = __fadd_rn(y, __fmul_rn(beta, C[ci]));
        }
        return y;
    }

    // cb[i] = beta * C[n] when the bias operand is a row vector (c_len == N).
    __device__ __forceinline__ void prepare(uint8_t* p, int n0, int bn, int tid, int nthreads) const {
        if (C == nullptr || c_len != N) return;
        float* cb = reinterpret_cast<float*>(p);
        for (int i = tid; i < bn; i += nthreads) {
            const int n = n0 + i;
            cb[i] = (n < N) ? __fmul_rn(beta, C[n]) : 0.0f;
        }
    }

    template <int W>
    __device__ __forceinline__ void write_to(float* base, int row, int col0, const float (&y)[W]) const {
        float* d = base + static_cast<int64_t>(row) * ldo + col0;
        if (col0 + W <= N && vec_ok) {
#pragma unroll
            for (int j = 0; j < W; j += 4)
                *reinterpret_cast<float4*>(d + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < W; ++j)
                if (col0 + j < N) d[j] = y[j];
        }
    }

    template <int W>
    __device__ __forceinline__ void write(int row, int col0, const float (&y)[W]) const {
        write_to<W>(out, row, col0, y);
        for (int i = 0; i < n_peer_out; ++i) write_to<W>(peer_out[i], row, col0, y);
    }

    // The further output copies of one warp's 32 x 32 block (lane l holds row
    // row0 + l, columns col0 .. col0 + 31; every lane of the warp calls this,
    // rows past M included).  The block is transposed in registers first, so
    // each store instruction writes 32 consecutive floats of one row: over
    // NVLink, 128-byte row pieces instead of 16-byte pieces of 32 rows.
    __device__ __forceinline__ void write_peers_rows(int row0, int col0, float (&y)[32]) const {
        const int lane = threadIdx.x & 31;
        // Recursive block transpose: at block size s, lanes whose bit s differs
        // exchange the off-diagonal s x s blocks (element (r, c) takes
        // (r ^ s, c ^ s) where bit s of r and c differ).
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                if ((j & s) == 0) {
                    const float send = upper ? y[j] : y[j + s];
                    const float recv = __shfl_xor_sync(0xffffffffu, send, s);
                    if (upper) y[j] = recv;
                    else y[j + s] = recv;
                }
            }
        }
        // Now lane l holds column col0 + l of rows row0 .. row0 + 31.
        const int col = col0 + lane;
        if (col >= N) return;
        for (int i = 0; i < n_peer_out; ++i) {
            float* d = peer_out[i] + static_cast<int64_t>(row0) * ldo + col;
#pragma unroll
            for (int r = 0; r < 32; ++r)
                if (row0 + r < M) d[static_cast<int64_t>(r) * ldo] = y[r];
        }
    }

    // Final epilogue from global parameters (split-K reduction, empty K).
    template <int W>
    __device__ __forceinline__ void store_direct(int row, int col0, const float (&acc)[W]) const {
        if (row >= M) return;
        float y[W];
#pragma unroll
        for (int j = 0; j < W; ++j) y[j] = finalize(row, col0 + j, acc[j]);
        write<W>(row, col0, y);
    }

    __device__ __forceinline__ void store(const uint8_t* p, int bn, int row, int col0, int cl, int ks,
                                          const uint32_t (&acc)[32]) const {
        if (out_mode != kOutPartial && n_peer_out > 0) {
            // Warp-collective: every lane, rows past M included.
            float y[32];
            if (row < M) {
                compute(p, row, col0, cl, acc, y);
                write_to<32>(out, row, col0, y);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j) y[j] = 0.0f;
            }
            write_peers_rows(row - (threadIdx.x & 31), col0, y);
            return;
        }
        if (row >= M) return;
        if (out_mode == kOutPartial) {
            float* d = partial + (static_cast<int64_t>(ks) * M + row) * N + col0;
            if (col0 + 32 <= N && (N % 4) == 0) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(d + j) =
                        make_float4(__uint_as_float(acc[j]), __uint_as_float(acc[j + 1]),
                                    __uint_as_float(acc[j + 2]), __uint_as_float(acc[j + 3]));
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (col0 + j < N) d[j] = __uint_as_float(acc[j]);
            }
            return;
        }
        float y[32];
        compute(p, row, col0, cl, acc, y);
        write<32>(row, col0, y);
    }

    __device__ __forceinline__ void compute(const uint8_t* p, int row, int col0, int cl, const uint32_t (&acc)[32],
                                            float (&y)[32]) const {
        if (C != nullptr && c_len == N) {
            const float4* cb4 = reinterpret_cast<const float4*>(p) + cl / 4;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const float4 c = cb4[v];
                const float cc[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    y[4 * v + u] = __fadd_rn(__fmul_rn(alpha, __uint_as_float(acc[4 * v + u])), cc[u]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) y[j] = finalize(row, col0 + j, __uint_as_float(acc[j]));
        }
    }
};

// Split-K reductions: thread per output element, partial sums added in split
// order, then the same finalisation as the single-pass epilogue.
__global__ void q_splitk_reduce_kernel(const QEpi e, int splits);
__global__ void f_splitk_reduce_kernel(const FEpi e, int splits);

}  // namespace pfrt
