// spmm_sp.cuh -- CSR SpMM for weights with 2:4 structure along K, on the
// tensor cores' structured-sparse MMA (tcgen05.mma.sp, kind::f16 with bf16).
//
//   Y[M, N] = X[M, K] * W^T,   W [N, K] with at most two stored entries in
//                               every aligned group of four columns of a row
//
// The 2:4 pattern is what NMSparsityPruning::compute_mask (n = 2, m = 4)
// leaves in a weight stored [N, K] (SparseMatMul, Gemm with transB = 1): its
// groups of m consecutive elements run along K.  A sparse MMA takes the 2:4
// operand in compressed form (two values per group of four, plus a 2-bit
// position for each) and does the work of a dense K = 32 step in the time of
// a dense K = 16 one.
//
// fp32 accuracy from bf16 products: W and X are each split into three bf16
// parts, w = w1 + w2 + w3 and x = x1 + x2 + x3 (each part the bf16 rounding
// of what the earlier parts left), and the six products whose size is at
// least 2^-16 of w1 x1 are summed: w1 x1, w1 x2, w1 x3, w2 x1, w2 x2, w3 x1.
// The dropped ones (w2 x3, w3 x2, w3 x3) are at most ~2^-24 of the product.
// As in the 3xTF32 kernels, TMEM accumulates one k-block (128 K) and the
// epilogue adds each such partial in IEEE fp32.
//
// Orientation Y^T = W X^T: the MMA's A operand (M = 128 lanes) is a tile of
// W in compressed form, its B operand X's parts stacked along N:
//   B = [x1; x2; x3] (64 rows of X each, 192 rows)
//   D[:,   0:192] += w1 * [x1; x2; x3]     (N = 192)
//   D[:,   0:128] += w2 * [x1; x2]         (N = 128)
//   D[:,   0: 64] += w3 * x1               (N = 64)
// so D = [w1x1 + w2x1 + w3x1 | w1x2 + w2x2 | w1x3] and the epilogue adds
// the three 64-column slices.  All three MMAs share one metadata word per
// row: the parts of W have the same sparsity pattern.
//
// Prepared forms (both written in the exact shared-memory image the kernel
// needs, so a stage is filled by plain 1-D bulk copies):
//   W image, per (W tile t of 128 rows, k-block kb of 128 K), 51200 bytes:
//     3 x [128 rows x 64 bf16 = 128 B, 128-byte swizzle]   parts w1, w2, w3
//     [128 lanes][4 u32] metadata: lane l's metadata word of each K = 32 step
//   X image, per (X slab c of 64 rows, kb), 49152 bytes: for each K half
//     (64 K), [x1 | x2 | x3] rows of 128 B, 128-byte swizzle.
// Metadata word of TMEM lane l for one K = 32 step (8 groups of 4 columns),
// as the hardware reads it: for 16-row blocks starting at row b, row
// r = b + 8 h + i (h = 0, 1; i < 8) keeps its groups 0..3 in lane b + i and
// groups 4..7 in lane b + 8 + i, group g at nibble 4 h + g % 4; a nibble is
// (position of the first stored value) | (position of the second) << 2,
// positions in 0..3 within the group, first < second.
//
// Any other sparse W: W = W24 + R, where W24 keeps the first two stored
// entries (by column) of every group of four and R the others.  At 90 %
// unstructured sparsity a group holds three or more entries with
// probability ~0.4 %, so R is a few entries per row; sp_remainder_add_kernel
// adds X R^T to Y afterwards in fp32 (R's entries of a row in column order,
// products of X itself, read from a transposed copy of X).
//
// A third form for sparser weights, the compressed form (sp_cform_kernel),
// holds only W24's values and per row its metadata and slot mask; the
// kernel's producer warps expand it into the same shared-memory parts.
//
// One CTA per SM: warps 0..3 epilogue (TMEM lane quarter = warp), warp 4
// loader (bulk copies), warp 5 MMA issuer and TMEM owner, then (image form)
// four metadata warps 6..9 or (compressed form) eight producer warps 6..13.
// TMEM: two 192-column accumulators at columns 0 and 256, then one 8-column
// slot per (stage, step) from column 448 for the metadata, written with
// tcgen05.st by the warps of the lane quarter (warp % 4): the metadata
// warps copy each lane's four words from the landed image, the producers
// compute them.  Every TMEM address an MMA is
// given is aligned to 8 columns or more.  Work units and
// their stream-K split over the CTAs, the partial tiles and their fix-up are
// those of spmm_tc.cuh with 64-row slabs and 128-K k-blocks.
#pragma once

#include <cuda_bf16.h>

#include "spmm_tc.cuh"

namespace pfrt {

constexpr int kSpBK = 128;                            // K per k-block
constexpr int kSpSteps = kSpBK / 32;                  // sparse MMA steps (K = 32) per k-block
constexpr int kSpSlab = 64;                           // X rows per unit
constexpr int kSpAPart = 128 * 128;                   // one W part: 128 rows x 128 B
constexpr int kSpMetaBytes = 128 * 4 * kSpSteps;      // metadata: [lane][step] u32
constexpr int kSpWImg = 3 * kSpAPart + kSpMetaBytes;  // 51200
constexpr int kSpXPart = kSpSlab * 128;               // one X part of one K half: 64 rows x 128 B
constexpr int kSpXHalf = 3 * kSpXPart;                // 24576
constexpr int kSpXImg = 2 * kSpXHalf;                 // 49152
constexpr int kSpStageBytes = kSpWImg + kSpXImg;      // 100352 (a multiple of 1024)
constexpr int kSpStages = 2;
constexpr int kSpN = 3 * kSpSlab;                     // 192 accumulator columns
constexpr uint32_t kSpAccStride = 256;                // accumulator slots at columns 0 and 256
constexpr uint32_t kSpTmemCols = 512;
constexpr uint32_t kSpMetaCol0 = 448;                 // metadata slot j at 448 + 8 j
constexpr int kSpEpiWarps = 4;
constexpr int kSpMetaWarps = 4;  // image form: one metadata warp per TMEM lane quarter
constexpr int kSpThreads = (kSpEpiWarps + 2 + kSpMetaWarps) * 32;
constexpr int kSpProdWarps = 8;  // compressed form: two producer warps per TMEM lane quarter
constexpr int kSpThreadsX = (kSpEpiWarps + 2 + kSpProdWarps) * 32;
constexpr int kSpBarBytes = 256;
constexpr int kSpSmemBytes = kSpStages * kSpStageBytes + kSpBarBytes + 1024;
// Compressed form: a stage holds the three W parts and X (no metadata
// blocks), and two value slots take one W tile's values of one k-block each.
constexpr int kSpStageBytesX = 3 * kSpAPart + kSpXImg;  // 98304
constexpr int kSpVSlot = 16384;
constexpr int kSpSmemBytesX = kSpStages * kSpStageBytesX + kSpStages * kSpVSlot + kSpBarBytes + 1024;
static_assert(kSpStageBytesX % 1024 == 0 && kSpSmemBytesX <= 227 * 1024, "compressed-form shared memory");
static_assert(kSpStageBytes % 1024 == 0 && kSpWImg % 1024 == 0, "1024-byte aligned swizzle atoms");
static_assert(kSpAccStride + kSpN <= kSpMetaCol0, "accumulators below the metadata");
static_assert(kSpMetaCol0 + 8 * kSpStages * kSpSteps <= kSpTmemCols, "TMEM columns");
static_assert(kSpSmemBytes <= 227 * 1024, "shared memory");

// Byte offset of 16-byte chunk `cb` (0..7) of row r in a 128-byte-swizzled
// image of 128-byte rows (1024-byte atoms of 8 rows).
__host__ __device__ constexpr int sp_swz(int r, int cb) {
    return (r >> 3) * 1024 + (r & 7) * 128 + ((cb ^ (r & 7)) << 4);
}

// 1-D bulk copy global -> shared, completing on `bar` (16-byte aligned, size
// a multiple of 16).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// D[tmem] (+)= A_sparse[smem] * B[smem]^T, bf16 inputs, f32 accumulate; the
// 2:4 metadata in TMEM at `meta`.
__device__ __forceinline__ void umma_sp_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t meta,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(meta), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor: bf16 x bf16 -> f32, M = 128, sparse, N given.
__host__ __device__ constexpr uint32_t sp_idesc(uint32_t n) {
    return idesc_make(1, 1, 1, 128, n) | (1u << 2);
}

__device__ __forceinline__ void bf16x3(float x, uint16_t& p1, uint16_t& p2, uint16_t& p3) {
    const __nv_bfloat16 a = __float2bfloat16_rn(x);
    const float r1 = __fsub_rn(x, __bfloat162float(a));
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const float r2 = __fsub_rn(r1, __bfloat162float(b));
    const __nv_bfloat16 c = __float2bfloat16_rn(r2);
    p1 = __bfloat16_as_ushort(a);
    p2 = __bfloat16_as_ushort(b);
    p3 = __bfloat16_as_ushort(c);
}

// Size of the remainder: one warp per row marks the row's stored columns in
// shared memory (one byte per column, 4 * groups bytes per warp) and adds to
// *over the entries past the second of every group of four columns.  Columns
// come from a validated CSR, so every index is below K <= 4 * groups.
__global__ void sp_count_kernel(int64_t N, int groups, const int32_t* __restrict__ indptr,
                                const int32_t* __restrict__ indices, unsigned long long* over) {
    extern __shared__ uint8_t cnt_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* cnt = cnt_raw + static_cast<int64_t>(warp) * groups * 4;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
    if (n >= N) return;
    for (int g = lane; g < groups * 4; g += 32) cnt[g] = 0;
    __syncwarp();
    const int32_t j0 = indptr[n], j1 = indptr[n + 1];
    for (int32_t j = j0 + lane; j < j1; j += 32) cnt[indices[j]] = 1;
    __syncwarp();
    unsigned long long extra = 0;
    for (int g = lane; g < groups; g += 32) {
        const int c = cnt[4 * g] + cnt[4 * g + 1] + cnt[4 * g + 2] + cnt[4 * g + 3];
        extra += c > 2 ? c - 2 : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) extra += __shfl_xor_sync(0xffffffffu, extra, o);
    if (lane == 0 && extra) atomicAdd(over, extra);
}

// The remainder R from the dense scratch wd [npad][kpad]: one warp per row
// walks the row 32 columns at a time (lane = column); an entry whose group
// of four already has two earlier nonzeros belongs to R.  count: rcount[n]
// = R's entries of row n; fill (rptr given): R's entries in column order.
template <bool FILL>
__global__ void sp_remainder_kernel(int64_t N, int64_t kpad, const float* __restrict__ wd,
                                    int32_t* __restrict__ rcount, const int64_t* __restrict__ rptr,
                                    int32_t* __restrict__ rcol, float* __restrict__ rval) {
    const int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    const float* row = wd + n * kpad;
    int64_t at = FILL ? rptr[n] : 0;
    int32_t total = 0;
    for (int64_t c0 = 0; c0 < kpad; c0 += 32) {
        const float v = row[c0 + lane];
        const uint32_t nz = __ballot_sync(0xffffffffu, v != 0.0f);
        const uint32_t gmask = 0xFu << (lane & ~3);
        const uint32_t before = nz & gmask & ((1u << lane) - 1u);  // earlier nonzeros of my group
        const bool extra = v != 0.0f && __popc(before) >= 2;
        const uint32_t em = __ballot_sync(0xffffffffu, extra);
        if (FILL && extra) {
            const int64_t k = at + __popc(em & ((1u << lane) - 1u));
            rcol[k] = static_cast<int32_t>(c0 + lane);
            rval[k] = v;
        }
        at += __popc(em);
        total += __popc(em);
    }
    if (!FILL && lane == 0) rcount[n] = total;
}

// W[n, c] into the zero-filled dense scratch (one warp per row; a column
// stored twice is summed, as the CSR's product sums it).
__global__ void sp_scatter_kernel(int64_t N, int64_t Kpad, const int32_t* __restrict__ indptr,
                                  const int32_t* __restrict__ indices, const float* __restrict__ values,
                                  float* __restrict__ wd) {
    const int64_t n = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (n >= N) return;
    for (int32_t j = indptr[n] + lane; j < indptr[n + 1]; j += 32) atomicAdd(wd + n * Kpad + indices[j], values[j]);
}

// W images from the dense scratch wd [Npad][Kpad] (zero padded): one thread
// per (tile t, k-block kb, row r, step s) compresses 32 columns (8 groups)
// of one row: its 16 kept values of each part, and its 8 metadata nibbles
// (ORed into the step's words of the two lanes; the image is zeroed first).
__global__ void sp_pack_w_kernel(int tiles, int KB, int64_t Kpad, const float* __restrict__ wd,
                                 uint8_t* __restrict__ img) {
    const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= static_cast<int64_t>(tiles) * KB * 128 * kSpSteps) return;
    const int s = static_cast<int>(id % kSpSteps);
    const int r = static_cast<int>((id / kSpSteps) % 128);
    const int64_t tk = id / (kSpSteps * 128);
    const int kb = static_cast<int>(tk % KB);
    const int t = static_cast<int>(tk / KB);
    const float* src = wd + (static_cast<int64_t>(t) * 128 + r) * Kpad + static_cast<int64_t>(kb) * kSpBK + 32 * s;
    uint8_t* base = img + (static_cast<int64_t>(t) * KB + kb) * kSpWImg;
    uint16_t v[3][16];
    uint32_t nib_lo = 0, nib_hi = 0;  // groups 0..3 and 4..7
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const float4 q = *reinterpret_cast<const float4*>(src + 4 * g);
        const float e[4] = {q.x, q.y, q.z, q.w};
        int p0 = -1, p1 = -1;  // the first two nonzeros; later ones are R's
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (e[i] != 0.0f) {
                if (p0 < 0) p0 = i;
                else if (p1 < 0) p1 = i;
            }
        // Empty slots take zero values at positions that keep p0 < p1.
        if (p0 < 0) {
            p0 = 0;
            p1 = 1;
        } else if (p1 < 0) {
            if (p0 == 3) {
                p0 = 2;
                p1 = 3;
            } else {
                p1 = 3;
            }
        }
        const float a = e[p0], b = e[p1];
        bf16x3(a, v[0][2 * g], v[1][2 * g], v[2][2 * g]);
        bf16x3(b, v[0][2 * g + 1], v[1][2 * g + 1], v[2][2 * g + 1]);
        const uint32_t nib = static_cast<uint32_t>(p0 | (p1 << 2));
        if (g < 4) nib_lo |= nib << (4 * g);
        else nib_hi |= nib << (4 * (g - 4));
    }
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        uint8_t* part = base + p * kSpAPart;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint4 w;
            w.x = v[p][8 * h + 0] | (static_cast<uint32_t>(v[p][8 * h + 1]) << 16);
            w.y = v[p][8 * h + 2] | (static_cast<uint32_t>(v[p][8 * h + 3]) << 16);
            w.z = v[p][8 * h + 4] | (static_cast<uint32_t>(v[p][8 * h + 5]) << 16);
            w.w = v[p][8 * h + 6] | (static_cast<uint32_t>(v[p][8 * h + 7]) << 16);
            *reinterpret_cast<uint4*>(part + sp_swz(r, 2 * s + h)) = w;
        }
    }
    uint32_t* meta = reinterpret_cast<uint32_t*>(base + 3 * kSpAPart);
    const int b16 = r & ~15, i = r & 7, hh = (r >> 3) & 1;
    atomicOr(meta + (b16 + i) * kSpSteps + s, nib_lo << (16 * hh));
    atomicOr(meta + (b16 + 8 + i) * kSpSteps + s, nib_hi << (16 * hh));
}

// X images: one thread per (slab c, k-block kb, 8-column piece q, row j),
// rows fastest: X[64 c + j, 128 kb + 8 q + 0..7] split into three bf16
// parts, 16 bytes of each part written to its swizzled place (zeros past M
// or K).  With xt (the remainder's transposed X, [K][ldxt]) the thread also
// writes its eight values there: a warp's 32 rows make 128-byte stores.
__global__ void sp_pack_x_kernel(const float* __restrict__ x, int64_t M, int64_t K, int64_t ldx, int slabs, int KB,
                                 uint8_t* __restrict__ img, float* __restrict__ xt, int64_t ldxt) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= static_cast<int64_t>(slabs) * KB * kSpSlab * 16) return;
    const int j = static_cast<int>(id % kSpSlab);
    const int q = static_cast<int>((id / kSpSlab) % 16);
    const int64_t ck = id / (16 * kSpSlab);
    const int kb = static_cast<int>(ck % KB);
    const int c = static_cast<int>(ck / KB);
    const int64_t m = static_cast<int64_t>(c) * kSpSlab + j;
    const int64_t k0 = static_cast<int64_t>(kb) * kSpBK + 8 * q;
    float e[8];
    if (m < M && k0 + 8 <= K && (ldx % 4) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        const float4 a = *reinterpret_cast<const float4*>(x + m * ldx + k0);
        const float4 b = *reinterpret_cast<const float4*>(x + m * ldx + k0 + 4);
        e[0] = a.x; e[1] = a.y; e[2] = a.z; e[3] = a.w; e[4] = b.x; e[5] = b.y; e[6] = b.z; e[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = (m < M && k0 + i < K) ? x[m * ldx + k0 + i] : 0.0f;
    }
    if (xt != nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (k0 + i < K) xt[(k0 + i) * ldxt + m] = e[i];
    }
    uint16_t v[3][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) bf16x3(e[i], v[0][i], v[1][i], v[2][i]);
    uint8_t* base = img + (static_cast<int64_t>(c) * KB + kb) * kSpXImg + (q >> 3) * kSpXHalf;
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        uint4 w;
        w.x = v[p][0] | (static_cast<uint32_t>(v[p][1]) << 16);
        w.y = v[p][2] | (static_cast<uint32_t>(v[p][3]) << 16);
        w.z = v[p][4] | (static_cast<uint32_t>(v[p][5]) << 16);
        w.w = v[p][6] | (static_cast<uint32_t>(v[p][7]) << 16);
        *reinterpret_cast<uint4*>(base + p * kSpXPart + sp_swz(j, q & 7)) = w;
    }
}

// Y[m, n] += sum over R's entries (n, c, v) of v * X[m, c], in R's column
// order, after the structured-sparse kernel (and its fix-up) wrote Y.  X
// comes transposed and padded (xt [K][ldxt], ldxt a multiple of 64), so an
// entry's 64 products read 256 contiguous bytes.  One block per (32 W rows,
// 64 X rows), 32 warps: the block's R entries (contiguous in R) staged in
// shared memory, one warp per W row with the lanes over the X rows, the sums
// collected in a shared tile and added to Y row by row (coalesced).
// W rows without R entries are not touched.
constexpr int kSpRStage = 2048;  // R entries staged per block (more are read from global memory)

__global__ void __launch_bounds__(1024) sp_remainder_add_kernel(const float* __restrict__ xt, int64_t ldxt, int64_t M,
                                                               int64_t N, const int64_t* __restrict__ rptr,
                                                               const int32_t* __restrict__ rcol,
                                                               const float* __restrict__ rval, float* __restrict__ y,
                                                               int64_t ldy) {
    __shared__ int32_t s_col[kSpRStage];
    __shared__ float s_val[kSpRStage];
    __shared__ float tile[64][33];
    pdl_wait();
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32, m0 = static_cast<int64_t>(blockIdx.y) * 64;
    const int64_t e_begin = rptr[n0 < N ? n0 : N];
    const int64_t e_end = rptr[n0 + 32 < N ? n0 + 32 : N];
    const bool staged = e_end - e_begin <= kSpRStage;
    if (staged)
        for (int64_t i = threadIdx.x; i < e_end - e_begin; i += blockDim.x) {
            s_col[i] = rcol[e_begin + i];
            s_val[i] = rval[e_begin + i];
        }
    __syncthreads();
    {
        const int r = warp;
        const int64_t n = n0 + r;
        float a0 = 0.0f, a1 = 0.0f;
        if (n < N) {
            const int64_t e1 = rptr[n + 1];
#pragma unroll 4
            for (int64_t e = rptr[n]; e < e1; ++e) {
                const int64_t c = staged ? s_col[e - e_begin] : rcol[e];
                const float v = staged ? s_val[e - e_begin] : rval[e];
                const float* xp = xt + c * ldxt + m0;
                a0 = __fadd_rn(a0, __fmul_rn(v, __ldg(xp + lane)));
                a1 = __fadd_rn(a1, __fmul_rn(v, __ldg(xp + 32 + lane)));
            }
        }
        tile[lane][r] = a0;
        tile[32 + lane][r] = a1;
    }
    __syncthreads();
    const int64_t n = n0 + lane;
    if (n >= N || rptr[n + 1] == rptr[n]) return;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int ml = warp * 2 + i;
        const int64_t m = m0 + ml;
        if (m < M) {
            float* yp = y + m * ldy + n;
            *yp = __fadd_rn(*yp, tile[ml][lane]);
        }
    }
}

// Compressed form of W24 (for sparse weights, where W's images would be
// mostly zeros).  Per (k-block kb, W row n): the row's metadata nibbles of
// each K = 32 step (meta.{x,y,z,w}: groups 0..3 in bits 0..15, groups 4..7
// in bits 16..31, the nibbles sp_pack_w_kernel writes), a 64-bit mask of the
// row's occupied slots (bit 16 s + 2 g + j: slot j of group g of step s;
// slots as in sp_pack_w_kernel: two values in slots 0 and 1, one value at
// position 3 in slot 1, any other single value in slot 0) and the index of
// the row's first value.  Values of (kb, n) pairs in [kb][n] order and,
// within one, in slot order (= column order), each as its three bf16 parts
// in 8 bytes (x = p1 | p2 << 16, y = p3).  A W tile's values of one k-block
// are thus one contiguous run, which the kernel's loader brings into shared
// memory with one bulk copy; the kernel then expands a row with shifts,
// adds and predicated loads only.  Built from the dense scratch copy: one
// thread per (kb, n) counts (COUNT: also the metadata and the slot mask) or
// writes (fill) the row's W24 values of the k-block.
template <bool COUNT>
__global__ void sp_cform_kernel(int64_t npad, int KB, int64_t kpad, const float* __restrict__ wd,
                                uint32_t* __restrict__ counts, uint4* __restrict__ cmeta, uint2* __restrict__ cocc,
                                const uint32_t* __restrict__ coff, uint2* __restrict__ cvals) {
    const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= npad * KB) return;
    const int64_t n = id % npad;
    const int kb = static_cast<int>(id / npad);
    const float* src = wd + n * kpad + static_cast<int64_t>(kb) * kSpBK;
    uint32_t meta[4] = {0u, 0u, 0u, 0u};
    uint32_t occ[2] = {0u, 0u};
    const uint32_t at = COUNT ? 0u : coff[id];
    uint32_t cnt = 0;
#pragma unroll 4
    for (int g = 0; g < kSpBK / 4; ++g) {
        const float4 q = *reinterpret_cast<const float4*>(src + 4 * g);
        const float e[4] = {q.x, q.y, q.z, q.w};
        int p0 = -1, p1 = -1;  // the first two nonzeros of the group are W24's
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (e[i] != 0.0f) {
                if (p0 < 0) p0 = i;
                else if (p1 < 0) p1 = i;
            }
        uint32_t slots;  // bit j: slot j occupied
        if (p0 < 0) {
            slots = 0u;
            p0 = 0;
            p1 = 1;
        } else if (p1 >= 0) {
            slots = 3u;
        } else if (p0 == 3) {
            slots = 2u;
            p0 = 2;
            p1 = 3;
        } else {
            slots = 1u;
            p1 = 3;
        }
        const int step = g >> 3, gg = g & 7;
        meta[step] |= static_cast<uint32_t>(p0 | (p1 << 2)) << (gg < 4 ? 4 * gg : 16 + 4 * (gg - 4));
        occ[step >> 1] |= slots << (16 * (step & 1) + 2 * gg);
        if (!COUNT) {
#pragma unroll
            for (int j = 0; j < 2; ++j)
                if (slots & (1u << j)) {
                    uint16_t a1, a2, a3;
                    bf16x3(e[j == 0 ? p0 : p1], a1, a2, a3);
                    cvals[static_cast<int64_t>(at) + cnt] = make_uint2(a1 | (static_cast<uint32_t>(a2) << 16), a3);
                    ++cnt;
                }
        } else {
            cnt += __popc(slots);
        }
    }
    if (COUNT) {
        counts[id] = cnt;
        cmeta[id] = make_uint4(meta[0], meta[1], meta[2], meta[3]);
        cocc[id] = make_uint2(occ[0], occ[1]);
    }
}

// One value record (the 3 bf16 parts of a W24 entry), loaded only where
// `pred`: from shared memory at byte address `saddr` (SH) or from global
// memory at `g`.  Zero where not loaded.
template <bool SH>
__device__ __forceinline__ uint2 sp_ldrec(uint32_t saddr, const uint2* g, bool pred) {
    uint2 v = make_uint2(0u, 0u);
    if (SH) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %3, 0;\n\t@p ld.shared.v2.u32 {%0, %1}, [%2];\n\t}"
            : "+r"(v.x), "+r"(v.y)
            : "r"(saddr), "r"(pred ? 1u : 0u));
    } else if (pred) {
        v = __ldg(g);
    }
    return v;
}

// Compressed form -> one W row of a stage: for each of the K = 32 steps
// S0 .. S0 + NS - 1, the row's 16 slots of each of the three parts into the
// swizzled W parts at `st`, and the step's metadata word into this thread's
// TMEM lane at column `meta_col` + 8 step (rows rl and rl ^ 8 share a lane
// word: the layout at the top of this file).  Values are record indices
// from the row's first: shared byte address `sbase` + 8 i (SH) or
// gbase + i.  All 16 loads of a step are issued before any is used.
template <bool SH, int S0, int NS>
__device__ __forceinline__ void sp_expand_row(const uint4& rmeta, const uint2& occ, uint32_t sbase,
                                              const uint2* gbase, uint8_t* st, int rl, int h, uint32_t meta_col,
                                              uint32_t lane_off) {
    static_assert((S0 == 0 || S0 == 2) && S0 + NS <= kSpSteps, "steps 0.. or 2..");
    const uint32_t rm[4] = {rmeta.x, rmeta.y, rmeta.z, rmeta.w};
    uint32_t idx = S0 == 0 ? 0u : static_cast<uint32_t>(__popc(occ.x));  // values of the earlier steps
#pragma unroll
    for (int s = S0; s < S0 + NS; ++s) {
        const uint32_t oc = (s < 2 ? occ.x : occ.y) >> (16 * (s & 1));
        uint2 r[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const uint32_t bit = (oc >> k) & 1u;
            r[k] = sp_ldrec<SH>(sbase + 8u * idx, gbase + idx, bit != 0u);
            idx += bit;
        }
        uint32_t w1[8], w2[8], w3[8];
#pragma unroll
        for (int gg = 0; gg < 8; ++gg) {
            w1[gg] = __byte_perm(r[2 * gg].x, r[2 * gg + 1].x, 0x5410);
            w2[gg] = __byte_perm(r[2 * gg].x, r[2 * gg + 1].x, 0x7632);
            w3[gg] = __byte_perm(r[2 * gg].y, r[2 * gg + 1].y, 0x5410);
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int off = sp_swz(rl, 2 * s + hh);
            *reinterpret_cast<uint4*>(st + off) = make_uint4(w1[4 * hh], w1[4 * hh + 1], w1[4 * hh + 2], w1[4 * hh + 3]);
            *reinterpret_cast<uint4*>(st + kSpAPart + off) =
                make_uint4(w2[4 * hh], w2[4 * hh + 1], w2[4 * hh + 2], w2[4 * hh + 3]);
            *reinterpret_cast<uint4*>(st + 2 * kSpAPart + off) =
                make_uint4(w3[4 * hh], w3[4 * hh + 1], w3[4 * hh + 2], w3[4 * hh + 3]);
        }
        // lane word: rows b + i (h = 0) and b + 8 + i (h = 1) of a 16-row
        // block give groups 0..3 to lane b + i and groups 4..7 to lane
        // b + 8 + i, row b + 8 h + i at bits 16 h
        const uint32_t mine = rm[s];
        const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 8);
        const uint32_t word = h == 0 ? ((mine & 0xFFFFu) | (other << 16)) : ((other >> 16) | (mine & 0xFFFF0000u));
        asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(meta_col + 8u * s + lane_off),
                     "r"(word)
                     : "memory");
    }
}

struct SpArgs {
    const uint8_t* wimg;    // [tiles][KB] W images (image form)
    const uint8_t* ximg;    // [slabs][KB] X images
    const uint4* cmeta;     // compressed form: [KB][npad] metadata nibbles
    const uint2* cocc;      // [KB][npad] slot masks
    const uint32_t* coff;   // [KB * npad + 1] value indices (the last one the total)
    const uint2* cvals;     // the 3 bf16 parts of each value
    int64_t npad;
    int M, N;
    float* y;              // output, row stride ldy
    int64_t ldy;
    float* partial;        // [2 * grid][64][128] partial tiles (tc_fixup_kernel's layout)
};

// EXPAND = false: W's images come by bulk copy with their metadata (image
// form), which four metadata warps move into TMEM.  EXPAND = true: the loader brings the W tile's values of the
// k-block into a value slot (one bulk copy) and X into the stage, on
// separate barriers, and eight producer warps (two per TMEM lane quarter,
// one thread per W row and pair of K = 32 steps) expand the values with the
// row's metadata and slot mask into the stage's three swizzled W parts and
// write the metadata words into TMEM themselves.  A run of values longer
// than a slot is read from global memory by the producers instead (slow;
// the host only picks this form where every run fits).
template <bool EXPAND>
__global__ void __launch_bounds__(EXPAND ? kSpThreadsX : kSpThreads, 1)
    spmm_sp_kernel(const TcSched sched, const SpArgs a, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    constexpr int kStage = EXPAND ? kSpStageBytesX : kSpStageBytes;
    constexpr int kXOff = EXPAND ? 3 * kSpAPart : kSpWImg;  // X's place in a stage
    constexpr int kVBytes = EXPAND ? kSpStages * kSpVSlot : 0;
    uint8_t* vslot = smem + kSpStages * kStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSpStages * kStage + kVBytes);
    uint64_t* empty = full + kSpStages;
    uint64_t* tfull = empty + kSpStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* vfull = drain + 1;          // compressed form: stage s's values landed
    uint64_t* xfull = vfull + kSpStages;  // compressed form: stage s's X landed
    uint64_t* mready = xfull + kSpStages;  // image form: stage s's metadata in TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mready + kSpStages);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    // Value slot s: [2 s] index of its first value, [2 s + 1] byte offset of
    // that value in the slot, or ~0 when the run is read from global memory.
    volatile uint32_t* vinfo = tmem_slot + 2;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr int kEpiThreads = 32 * kSpEpiWarps;
    constexpr int kLoadWarp = kSpEpiWarps;
    constexpr int kMmaWarp = kSpEpiWarps + 1;
    constexpr int kProdWarp0 = kSpEpiWarps + 2;
    const int64_t KB = sched.kb_total;
    const int64_t g0 = static_cast<int64_t>(blockIdx.x) * sched.per_cta;
    const int64_t g1 = min(g0 + sched.per_cta, sched.total);  // this CTA's k-blocks [g0, g1)

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSpStages; ++s) {
            mbar_init(&full[s], EXPAND ? kSpProdWarps : 1);  // the loader's copies, or each producer warp
            mbar_init(&empty[s], 1);
            mbar_init(&vfull[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&mready[s], kSpMetaWarps);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiThreads);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_slot, kSpTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    if (threadIdx.x == 0) pdl_launch_dependents();

    if (warp < kSpEpiWarps) {
        const int q = warp;
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
            float racc[kSpSlab];
#pragma unroll
            for (int j = 0; j < kSpSlab; ++j) racc[j] = 0.0f;
            bool stop = false;
            for (int kc = kb_lo; kc < kb_hi; ++kc, ++tc) {
                const int slot = tc & 1;
                const uint32_t ap = static_cast<uint32_t>(tc >> 1) & 1u;
                const bool got = mbar_wait(&tfull[slot], ap, abort_flag);
                if (epi_barrier_or(!got || *abort_flag != 0, kEpiThreads)) {
                    stop = true;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem_base + static_cast<uint32_t>(slot) * kSpAccStride + lane_off;
                // X row j: columns j (x1 products), 64 + j (x2), 128 + j (x3).
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    uint32_t v0[16], v1[16], v2[16];
                    tmem_ld_32x32b_x16(taddr + static_cast<uint32_t>(16 * h), v0);
                    tmem_ld_32x32b_x16(taddr + static_cast<uint32_t>(64 + 16 * h), v1);
                    tmem_ld_32x32b_x16(taddr + static_cast<uint32_t>(128 + 16 * h), v2);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        racc[16 * h + j] = __fadd_rn(
                            racc[16 * h + j],
                            __fadd_rn(__fadd_rn(__uint_as_float(v0[j]), __uint_as_float(v1[j])), __uint_as_float(v2[j])));
                }
                tc_fence_before();
                mbar_arrive(&tempty[slot]);
            }
            if (stop) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                break;
            }
            const int m0 = c * kSpSlab;
            if (kb_lo == 0 && kb_hi == KB) {
                const int n = t * kTcWRows + nl;
                if (n < a.N) {
                    float* dst = a.y + n;
#pragma unroll
                    for (int j = 0; j < kSpSlab; ++j)
                        if (m0 + j < a.M) dst[static_cast<int64_t>(m0 + j) * a.ldy] = racc[j];
                }
            } else {
                float* dst = a.partial + tc_slot(sched, blockIdx.x, u) * kTcTileElems + nl;
#pragma unroll
                for (int j = 0; j < kSpSlab; ++j) dst[j * kTcWRows] = racc[j];
            }
        }
    } else if (warp == kLoadWarp && !EXPAND) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            uint32_t last_par[kSpStages];
            bool ok = true;
            TcCursor cur;
            cur.init(sched, g0);
            // W's images are a prepared weight (written once, never by a
            // kernel that precedes this one): the first stages' W halves are
            // requested before the dependency wait, X (written by the packing
            // kernel just before) after it.
            const int npre = static_cast<int>(g1 - g0 < kSpStages ? g1 - g0 : kSpStages);
            TcCursor pc = cur;
            for (int i = 0; i < npre; ++i, pc.next(sched)) {
                uint8_t* st = smem + i * kSpStageBytes;
                mbar_arrive_expect_tx(&full[i], kSpStageBytes);
                const uint8_t* wsrc = a.wimg + (static_cast<int64_t>(pc.t) * KB + pc.kb) * kSpWImg;
                bulk_load(st, wsrc, kSpWImg / 2, &full[i]);
                bulk_load(st + kSpWImg / 2, wsrc + kSpWImg / 2, kSpWImg / 2, &full[i]);
                issued |= 1u << i;
                last_par[i] = 0u;
            }
            pdl_wait();
            for (int i = 0; i < npre; ++i, cur.next(sched)) {
                uint8_t* st = smem + i * kSpStageBytes + kSpWImg;
                const uint8_t* xsrc = a.ximg + (static_cast<int64_t>(cur.c) * KB + cur.kb) * kSpXImg;
                bulk_load(st, xsrc, kSpXImg / 2, &full[i]);
                bulk_load(st + kSpXImg / 2, xsrc + kSpXImg / 2, kSpXImg / 2, &full[i]);
            }
            stage = npre % kSpStages;
            phase = (npre == kSpStages) ? 1u : 0u;
            for (int64_t g = g0 + npre; g < g1; ++g, cur.next(sched)) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + stage * kSpStageBytes;
                mbar_arrive_expect_tx(&full[stage], kSpStageBytes);
                const uint8_t* wsrc = a.wimg + (static_cast<int64_t>(cur.t) * KB + cur.kb) * kSpWImg;
                const uint8_t* xsrc = a.ximg + (static_cast<int64_t>(cur.c) * KB + cur.kb) * kSpXImg;
                bulk_load(st, wsrc, kSpWImg / 2, &full[stage]);
                bulk_load(st + kSpWImg / 2, wsrc + kSpWImg / 2, kSpWImg / 2, &full[stage]);
                bulk_load(st + kSpWImg, xsrc, kSpXImg / 2, &full[stage]);
                bulk_load(st + kSpWImg + kSpXImg / 2, xsrc + kSpXImg / 2, kSpXImg / 2, &full[stage]);
                issued |= 1u << stage;
                last_par[stage] = phase;
                if (++stage == kSpStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                const int zero = 0;
                for (int s = 0; s < kSpStages; ++s)
                    if (issued & (1u << s)) mbar_wait(&full[s], last_par[s], &zero);
            }
        }
    } else if (warp == kLoadWarp) {
        // Compressed form: values and X on their own barriers.  The values of
        // a stage's next k-block are requested once the producers are done
        // with the slot (full[s]), X once the MMAs are done with the stage
        // (empty[s]), so the producers expand while X is still in flight.
        if (lane == 0) {
            uint32_t vissued = 0, xissued = 0, vpar[kSpStages], xpar[kSpStages];
            bool ok = true;
            TcCursor cur;
            cur.init(sched, g0);
            // The unit's run of values [vo0, vo1) (its W tile's values of the
            // k-block), read one unit ahead; copied into value slot s when
            // it fits, 16-byte aligned at both ends.
            uint32_t vo0 = 0, vo1 = 0;
            auto run_of = [&](const TcCursor& c) {
                const int64_t r0 = static_cast<int64_t>(c.kb) * a.npad + static_cast<int64_t>(c.t) * kTcWRows;
                vo0 = __ldg(a.coff + r0);
                vo1 = __ldg(a.coff + r0 + kTcWRows);
            };
            // vinfo is written before the arrival, which publishes it to the
            // producers.
            auto issue_values = [&](int s, const TcCursor& c, bool fetch_next) {
                const uint64_t b0 = (static_cast<uint64_t>(vo0) * 8u) & ~static_cast<uint64_t>(15);
                const uint64_t b1 = (static_cast<uint64_t>(vo1) * 8u + 15u) & ~static_cast<uint64_t>(15);
                const bool fits = vo1 > vo0 && b1 - b0 <= static_cast<uint64_t>(kSpVSlot);
                vinfo[2 * s] = vo0;
                vinfo[2 * s + 1] =
                    fits ? static_cast<uint32_t>(static_cast<uint64_t>(vo0) * 8u - b0) : (vo1 > vo0 ? ~0u : 0u);
                if (fits) {
                    mbar_arrive_expect_tx(&vfull[s], static_cast<uint32_t>(b1 - b0));
                    bulk_load(vslot + s * kSpVSlot, reinterpret_cast<const uint8_t*>(a.cvals) + b0,
                              static_cast<uint32_t>(b1 - b0), &vfull[s]);
                } else {
                    mbar_arrive(&vfull[s]);
                }
                if (fetch_next) {
                    TcCursor nx = c;
                    nx.next(sched);
                    run_of(nx);
                }
            };
            auto issue_x = [&](int s, const TcCursor& c) {
                uint8_t* st = smem + s * kStage + kXOff;
                const uint8_t* xsrc = a.ximg + (static_cast<int64_t>(c.c) * KB + c.kb) * kSpXImg;
                mbar_arrive_expect_tx(&xfull[s], kSpXImg);
                bulk_load(st, xsrc, kSpXImg / 2, &xfull[s]);
                bulk_load(st + kSpXImg / 2, xsrc + kSpXImg / 2, kSpXImg / 2, &xfull[s]);
            };
            // The compressed form is a prepared weight (written once, never
            // by a kernel that precedes this one): the first values are
            // requested before the dependency wait, X (written by the
            // packing kernel just before) after it.
            const int npre = static_cast<int>(g1 - g0 < kSpStages ? g1 - g0 : kSpStages);
            if (npre > 0) run_of(cur);
            TcCursor pc = cur;
            for (int i = 0; i < npre; ++i, pc.next(sched)) {
                issue_values(i, pc, g0 + i + 1 < g1);
                vissued |= 1u << i;
                vpar[i] = 0u;
            }
            pdl_wait();
            for (int i = 0; i < npre; ++i, cur.next(sched)) {
                issue_x(i, cur);
                xissued |= 1u << i;
                xpar[i] = 0u;
            }
            int stage = npre % kSpStages;
            uint32_t phase = (npre == kSpStages) ? 1u : 0u;
            for (int64_t g = g0 + npre; g < g1; ++g, cur.next(sched)) {
                if (!mbar_wait(&full[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                issue_values(stage, cur, g + 1 < g1);
                vissued |= 1u << stage;
                vpar[stage] = phase;
                if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                issue_x(stage, cur);
                xissued |= 1u << stage;
                xpar[stage] = phase;
                if (++stage == kSpStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                // Copies still in flight land before the CTA exits.
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                const int zero = 0;
                for (int s = 0; s < kSpStages; ++s) {
                    if (vissued & (1u << s)) mbar_wait(&vfull[s], vpar[s], &zero);
                    if (xissued & (1u << s)) mbar_wait(&xfull[s], xpar[s], &zero);
                }
            }
        }
    } else if (!EXPAND && warp >= kProdWarp0) {
        // Metadata warp (image form): once a stage's image has landed, each
        // thread writes its TMEM lane's four step words (the image's
        // [lane][step] block) into the stage's metadata slots; the MMA
        // thread waits for all four warps (mready).  The slots are free: the
        // loader requested the image after the MMAs of the stage's previous
        // k-block were done.
        const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
        const int rl = (warp & 3) * 32 + lane;
        int stage = 0;
        uint32_t phase = 0;
        for (int64_t g = g0; g < g1; ++g) {
            if (!mbar_wait(&full[stage], phase, abort_flag)) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                break;
            }
            tc_fence_after();
            const uint4 mw = *reinterpret_cast<const uint4*>(smem + stage * kStage + 3 * kSpAPart + 16 * rl);
            const uint32_t meta = tmem_base + kSpMetaCol0 + static_cast<uint32_t>(8 * kSpSteps * stage) + lane_off;
            asm volatile(
                "tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};\n\t"
                "tcgen05.st.sync.aligned.32x32b.x1.b32 [%2], {%3};\n\t"
                "tcgen05.st.sync.aligned.32x32b.x1.b32 [%4], {%5};\n\t"
                "tcgen05.st.sync.aligned.32x32b.x1.b32 [%6], {%7};" ::"r"(meta),
                "r"(mw.x), "r"(meta + 8u), "r"(mw.y), "r"(meta + 16u), "r"(mw.z), "r"(meta + 24u), "r"(mw.w)
                : "memory");
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&mready[stage]);
            if (++stage == kSpStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    } else if (EXPAND && warp >= kProdWarp0) {
        // Producer: this thread builds W row n = 128 t + 32 q + lane of each
        // k-block of the CTA's range into the stage's W parts and its TMEM
        // lane's metadata words, from the row's metadata, slot mask and
        // values in the stage's value slot: warps 6..9 the K = 32 steps 0
        // and 1, warps 10..13 steps 2 and 3 (a warp reaches the TMEM lane
        // quarter warp % 4).  The row's data of the next k-block is loaded
        // while this one is built.
        const int q = warp & 3;
        const bool hi_steps = warp >= kProdWarp0 + 4;
        const int rl = q * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        const int h = (rl >> 3) & 1;
        TcCursor cur;
        cur.init(sched, g0);
        int stage = 0;
        uint32_t phase = 0;
        auto load_row = [&](const TcCursor& c, uint4& m, uint2& oc, uint32_t& o) {
            const int64_t w = static_cast<int64_t>(c.kb) * a.npad + static_cast<int64_t>(c.t) * kTcWRows + rl;
            m = __ldg(a.cmeta + w);
            oc = __ldg(a.cocc + w);
            o = __ldg(a.coff + w);
        };
        uint4 m_next{};
        uint2 oc_next{};
        uint32_t o_next = 0;
        if (g0 < g1) load_row(cur, m_next, oc_next, o_next);
        for (int64_t g = g0; g < g1; ++g) {
            const uint4 mk = m_next;
            const uint2 ock = oc_next;
            const uint32_t o_row = o_next;
            TcCursor nx = cur;
            nx.next(sched);
            if (g + 1 < g1) load_row(nx, m_next, oc_next, o_next);
            // The stage's values have landed (vfull) and the MMAs of its
            // previous k-block are done (empty): its W parts and TMEM
            // metadata slots are free.
            if (!mbar_wait(&vfull[stage], phase, abort_flag) || !mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
                *abort_flag = 1;
                report_error(err, kDevWaitTimeout);
                break;
            }
            tc_fence_after();
            uint8_t* st = smem + stage * kStage;
            const uint32_t run0 = vinfo[2 * stage], where = vinfo[2 * stage + 1];
            const uint32_t meta = tmem_base + kSpMetaCol0 + static_cast<uint32_t>(8 * kSpSteps * stage);
            const uint32_t sbase = smem_u32(vslot + stage * kSpVSlot) + where + 8u * (o_row - run0);
            if (where != ~0u) {
                if (hi_steps) sp_expand_row<true, 2, 2>(mk, ock, sbase, a.cvals + o_row, st, rl, h, meta, lane_off);
                else sp_expand_row<true, 0, 2>(mk, ock, sbase, a.cvals + o_row, st, rl, h, meta, lane_off);
            } else {
                if (hi_steps) sp_expand_row<false, 2, 2>(mk, ock, 0u, a.cvals + o_row, st, rl, h, meta, lane_off);
                else sp_expand_row<false, 0, 2>(mk, ock, 0u, a.cvals + o_row, st, rl, h, meta, lane_off);
            }
            tmem_st_wait();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[stage]);
            cur = nx;
            if (++stage == kSpStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int tc = 0;
            for (int64_t g = g0; ok && g < g1; ++g, ++tc) {
                const int slot = tc & 1;
                const uint32_t ap = static_cast<uint32_t>(tc >> 1) & 1u;
                if (!mbar_wait(&tempty[slot], ap ^ 1u, abort_flag) || !mbar_wait(&full[stage], phase, abort_flag) ||
                    !mbar_wait(EXPAND ? &xfull[stage] : &mready[stage], phase, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u32(smem + stage * kStage);
                const uint32_t meta = tmem_base + kSpMetaCol0 + static_cast<uint32_t>(8 * kSpSteps * stage);
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot) * kSpAccStride;
                const uint64_t a1 = sdesc_kmajor_sw128(st), a2 = sdesc_kmajor_sw128(st + kSpAPart),
                               a3 = sdesc_kmajor_sw128(st + 2 * kSpAPart);
#pragma unroll
                for (int k = 0; k < kSpSteps; ++k) {
                    const uint64_t ka = static_cast<uint64_t>((32 * k) >> 4);  // 16 stored bf16 per step
                    const uint64_t db = sdesc_kmajor_sw128(st + kXOff + (k >> 1) * kSpXHalf) +
                                        static_cast<uint64_t>((64 * (k & 1)) >> 4);  // 32 bf16 of X per step
                    const uint32_t mk = meta + static_cast<uint32_t>(8 * k);
                    umma_sp_bf16(d_tmem, a1 + ka, db, mk, sp_idesc(3 * kSpSlab), k > 0 ? 1u : 0u);
                    umma_sp_bf16(d_tmem, a2 + ka, db, mk, sp_idesc(2 * kSpSlab), 1u);
                    umma_sp_bf16(d_tmem, a3 + ka, db, mk, sp_idesc(kSpSlab), 1u);
                }
                umma_commit(&empty[stage]);
                umma_commit(&tfull[slot]);
                if (++stage == kSpStages) {
                    stage = 0;
                    phase ^= 1u;
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
        tmem_dealloc(tmem_base, kSpTmemCols);
    }
}

}  // namespace pfrt
