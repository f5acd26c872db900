/*
 * oracle.c -- CPU restatement of the PyFlameRT reference hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Build with -ffp-contract=off so
 * that no multiply-add is fused: the reference's loops are compiled for the
 * x86-64 baseline, which has no FMA, and every product is rounded before it
 * is added.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* cpu_gemm, src/backends/cpu/ops/math.cpp:377-438.
 * Output zero-filled (:408-409); i-k-j loop with
 * out[i,j] += alpha * a_ik * b_kj (:416-424), i.e. (alpha*a_ik)*b_kj rounded
 * and then added; then out[i] += beta * C[i % c_size] over the flat index
 * (:427-435). */
void oracle_gemm_f32(int64_t M, int64_t N, int64_t K, int trans_a, int trans_b,
                     float alpha, float beta, const float* A, const float* B,
                     const float* C, int64_t c_len, float* Y) {
    memset(Y, 0, (size_t)(M * N) * sizeof(float));
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t k = 0; k < K; ++k) {
            float a_ik = trans_a ? A[k * M + i] : A[i * K + k];
            for (int64_t j = 0; j < N; ++j) {
                float b_kj = trans_b ? B[j * K + k] : B[k * N + j];
                float t = alpha * a_ik;
                t = t * b_kj;
                Y[i * N + j] = Y[i * N + j] + t;
            }
        }
    }
    if (C && c_len > 0) {
        for (int64_t i = 0; i < M * N; ++i) {
            float t = beta * C[i % c_len];
            Y[i] = Y[i] + t;
        }
    }
}

/* cpu_matmul 2-D fast path, src/backends/cpu/ops/math.cpp:326-336:
 * out[i,j] += a_ik * b[k,j] in i-k-j order from a zeroed output. */
void oracle_matmul_f32(int64_t M, int64_t N, int64_t K, const float* A,
                       const float* B, float* Y) {
    memset(Y, 0, (size_t)(M * N) * sizeof(float));
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t k = 0; k < K; ++k) {
            float a_ik = A[i * K + k];
            for (int64_t j = 0; j < N; ++j) {
                float t = a_ik * B[k * N + j];
                Y[i * N + j] = Y[i * N + j] + t;
            }
        }
    }
}

/* quantized_matmul accumulators, src/quantization/quant_ops.cpp:443-498:
 * int64 acc of (a - a_zp) * (b - b_zp), u8/s8 handled per dtype (:480-490).
 * Loop reordered to i-k-j for speed; integer sums are order-independent. */
void oracle_qmm_acc(int64_t M, int64_t N, int64_t K, const void* a, int a_is_u8,
                    int32_t a_zp, const int8_t* w, int32_t w_zp, int64_t* acc) {
    const uint8_t* au = (const uint8_t*)a;
    const int8_t* as = (const int8_t*)a;
    int32_t* row = (int32_t*)malloc((size_t)N * sizeof(int32_t));
    for (int64_t i = 0; i < M; ++i) {
        /* int32 partial sums over a bounded K block, flushed to int64 so the
         * result is exact for any K. */
        for (int64_t j = 0; j < N; ++j) acc[i * N + j] = 0;
        for (int64_t k0 = 0; k0 < K; k0 += 16384) {
            int64_t k1 = k0 + 16384 < K ? k0 + 16384 : K;
            for (int64_t j = 0; j < N; ++j) row[j] = 0;
            for (int64_t k = k0; k < k1; ++k) {
                int32_t av = (a_is_u8 ? (int32_t)au[i * K + k] : (int32_t)as[i * K + k]) - a_zp;
                const int8_t* wk = w + k * N;
                for (int64_t j = 0; j < N; ++j) row[j] += av * ((int32_t)wk[j] - w_zp);
            }
            for (int64_t j = 0; j < N; ++j) acc[i * N + j] += row[j];
        }
    }
    free(row);
}

static inline int32_t clamp_i32(int32_t v, int32_t lo, int32_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

/* One requantization step, quant_ops.cpp:42-55:
 * (int32)std::round(x * inv_scale) + zp, clamped to the dtype range
 * (get_quant_range, quant_params.hpp:143-153). */
static inline int32_t requant_one(float x, float inv_scale, int32_t zp, int out_is_u8) {
    float t = x * inv_scale;
    float r = roundf(t);
    /* static_cast<int32_t>(float) as the reference's x86-64 build executes it
     * (cvttss2si): out of range or NaN gives INT32_MIN; the + zp wraps. */
    int32_t ri = (r >= -2147483648.0f && r < 2147483648.0f) ? (int32_t)r : INT32_MIN;
    int32_t q = (int32_t)((uint32_t)ri + (uint32_t)zp);
    return out_is_u8 ? clamp_i32(q, 0, 255) : clamp_i32(q, -128, 127);
}

void oracle_qepilogue(int64_t M, int64_t N, const int64_t* acc, float a_scale,
                      const float* w_scale, const float* bias, int relu, int out_mode,
                      float y_scale, int32_t y_zp, float* y_f32, void* y_q) {
    float* os = (float*)malloc((size_t)N * sizeof(float));
    for (int64_t j = 0; j < N; ++j) os[j] = a_scale * w_scale[j];   /* quant_ops.cpp:435 */
    float inv_scale = 1.0f / y_scale;                                  /* quant_ops.cpp:41 */
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t j = 0; j < N; ++j) {
            int64_t a64 = acc[i * N + j];
            float y = (float)a64 * os[j];                              /* quant_ops.cpp:464 */
            if (bias) y = y + bias[j];                                 /* math.cpp:225 */
            if (relu) y = (0.0f < y) ? y : 0.0f;                       /* activation.cpp:56, std::max(0.0f, y) */
            if (out_mode == 0) {
                y_f32[i * N + j] = y;
            } else if (out_mode == 1) {
                ((int8_t*)y_q)[i * N + j] = (int8_t)requant_one(y, inv_scale, y_zp, 0);
            } else {
                ((uint8_t*)y_q)[i * N + j] = (uint8_t)requant_one(y, inv_scale, y_zp, 1);
            }
        }
    }
    free(os);
}

void oracle_qlinear(int64_t M, int64_t N, int64_t K, const void* a, int a_is_u8,
                    float a_scale, int32_t a_zp, const int8_t* w, int32_t w_zp,
                    const float* w_scale, const float* bias, int relu,
                    int out_mode, float y_scale, int32_t y_zp, float* y_f32,
                    void* y_q, int32_t* acc_out) {
    int64_t* acc = (int64_t*)malloc((size_t)(M * N) * sizeof(int64_t));
    oracle_qmm_acc(M, N, K, a, a_is_u8, a_zp, w, w_zp, acc);
    if (acc_out)
        for (int64_t i = 0; i < M * N; ++i) acc_out[i] = (int32_t)acc[i];
    oracle_qepilogue(M, N, acc, a_scale, w_scale, bias, relu, out_mode, y_scale, y_zp, y_f32, y_q);
    free(acc);
}

/* quantize_tensor, per-tensor branch, quant_ops.cpp:33-55. */
void oracle_quantize(int64_t n, const float* x, float scale, int32_t zp,
                     int out_is_u8, void* q) {
    float inv_scale = 1.0f / scale;
    for (int64_t i = 0; i < n; ++i) {
        int32_t v = requant_one(x[i], inv_scale, zp, out_is_u8);
        if (out_is_u8) ((uint8_t*)q)[i] = (uint8_t)v;
        else ((int8_t*)q)[i] = (int8_t)v;
    }
}

/* sparse_matmul CSR branch, src/pruning/sparse_tensor.cpp:496-510. */
void oracle_csr_spmm(int64_t R, int64_t C, const int32_t* indptr,
                     const int32_t* indices, const float* values,
                     const float* B, float* Yt) {
    memset(Yt, 0, (size_t)(R * C) * sizeof(float));
    for (int64_t r = 0; r < R; ++r) {
        for (int64_t j = indptr[r]; j < indptr[r + 1]; ++j) {
            int64_t col = indices[j];
            float val = values[j];
            for (int64_t c = 0; c < C; ++c) {
                float t = val * B[col * C + c];
                Yt[r * C + c] = Yt[r * C + c] + t;
            }
        }
    }
}

void oracle_spmm_linear(int64_t M, int64_t N, int64_t K, const int32_t* indptr,
                        const int32_t* indices, const float* values,
                        const float* X, float* Y) {
    (void)K;
    for (int64_t m = 0; m < M; ++m) {
        const float* x = X + m * K;
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int64_t j = indptr[n]; j < indptr[n + 1]; ++j) {
                float t = values[j] * x[indices[j]];
                acc = acc + t;
            }
            Y[m * N + n] = acc;
        }
    }
}

void oracle_spmm_linear_f64(int64_t M, int64_t N, int64_t K,
                            const int32_t* indptr, const int32_t* indices,
                            const float* values, const float* X, double* Y) {
    for (int64_t m = 0; m < M; ++m) {
        const float* x = X + m * K;
        for (int64_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (int64_t j = indptr[n]; j < indptr[n + 1]; ++j)
                acc += (double)values[j] * (double)x[indices[j]];
            Y[m * N + n] = acc;
        }
    }
}

void oracle_gemm_f64(int64_t M, int64_t N, int64_t K, int trans_a, int trans_b,
                     double alpha, double beta, const float* A, const float* B,
                     const float* C, int64_t c_len, double* Y) {
    for (int64_t i = 0; i < M * N; ++i) Y[i] = 0.0;
    for (int64_t i = 0; i < M; ++i) {
        for (int64_t k = 0; k < K; ++k) {
            double a_ik = trans_a ? A[k * M + i] : A[i * K + k];
            for (int64_t j = 0; j < N; ++j) {
                double b_kj = trans_b ? B[j * K + k] : B[k * N + j];
                Y[i * N + j] += alpha * a_ik * b_kj;
            }
        }
    }
    if (C && c_len > 0)
        for (int64_t i = 0; i < M * N; ++i) Y[i] += beta * (double)C[i % c_len];
}

/* ---------------------------------------------------------------- pruning */
static int cmp_float(const void* a, const void* b) {
    const float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

int oracle_magnitude_mask(int64_t n, const float* w, float sparsity, float* mask) {
    if (sparsity <= 0.0f) { /* magnitude_pruning.cpp:33-39 */
        for (int64_t i = 0; i < n; ++i) mask[i] = 1.0f;
        return 0;
    }
    if (sparsity >= 1.0f) { /* :41-47 */
        for (int64_t i = 0; i < n; ++i) mask[i] = 0.0f;
        return 0;
    }
    if (n == 0) return -1; /* :54-56 */
    float* scores = (float*)malloc(sizeof(float) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) scores[i] = fabsf(w[i]);
    qsort(scores, (size_t)n, sizeof(float), cmp_float); /* :66 */
    size_t idx = (size_t)floor((double)n * (double)sparsity); /* :70-73, double */
    if (idx > (size_t)n - 1) idx = (size_t)n - 1;
    const float thr = scores[idx];
    free(scores);
    for (int64_t i = 0; i < n; ++i) mask[i] = (fabsf(w[i]) > thr) ? 1.0f : 0.0f; /* :79-81 */
    /* :84: size_t * float is evaluated in float */
    const size_t target = (size_t)((float)n * sparsity);
    size_t zeros = 0;
    for (int64_t i = 0; i < n; ++i) zeros += (mask[i] == 0.0f);
    if (zeros > target) { /* :91-98: restore ties in index order */
        size_t restore = zeros - target;
        for (int64_t i = 0; i < n && restore > 0; ++i) {
            if (mask[i] == 0.0f && fabsf(w[i]) == thr) {
                mask[i] = 1.0f;
                --restore;
            }
        }
    }
    return 0;
}

void oracle_masked_csr(int64_t rows, int64_t cols, const float* w, const float* mask, int32_t* indptr,
                       int32_t* indices, float* values) {
    int64_t nz = 0;
    indptr[0] = 0;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < cols; ++c) {
            const float d = w[r * cols + c] * mask[r * cols + c];
            if (fabsf(d) > 0.0f) {
                indices[nz] = (int32_t)c;
                values[nz] = d;
                ++nz;
            }
        }
        indptr[r + 1] = (int32_t)nz;
    }
}


/* ------------------------------------------------------------ N:M pruning
 * std::partial_sort(first, middle, last, comp) of libstdc++ (GCC 13) keeps in
 * [first, middle) the set its heap selection leaves there: a binary heap over
 * [first, middle) whose top is the element no other precedes under comp,
 * built bottom-up; then each later element that precedes the top under comp
 * replaces it (pop into the hole at the top).  Each sift moves the hole from
 * the given position to a leaf along the preferred child (the right child
 * unless it precedes the left one under comp), then sifts the new value up
 * from that leaf.  The order of these moves decides which of equal elements
 * stay, so it is restated exactly.  comp(a, b) = |w[a]| > |w[b]| (float
 * compare: any NaN compares false). */
static int nm_gt(const float* w, int a, int b) { return fabsf(w[a]) > fabsf(w[b]); }

static void nm_sift(const float* w, int* h, int hole, int len, int v) {
    const int top = hole;
    int child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (nm_gt(w, h[child], h[child - 1])) child--;
        h[hole] = h[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        h[hole] = h[child - 1];
        hole = child - 1;
    }
    int parent = (hole - 1) / 2;
    while (hole > top && nm_gt(w, h[parent], v)) {
        h[hole] = h[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    h[hole] = v;
}

/* Marks in keep[0..g) the k elements of w[0..g) that partial_sort leaves in
 * its first k positions. */
static void nm_select(const float* w, int g, int k, float* keep) {
    int h[64];
    for (int j = 0; j < k; ++j) h[j] = j;
    if (k >= 2)
        for (int parent = (k - 2) / 2;; --parent) {
            nm_sift(w, h, parent, k, h[parent]);
            if (parent == 0) break;
        }
    for (int j = k; j < g; ++j)
        if (nm_gt(w, j, h[0])) nm_sift(w, h, 0, k, j);
    for (int j = 0; j < g; ++j) keep[j] = 0.0f;
    for (int j = 0; j < k; ++j) keep[h[j]] = 1.0f;
}

int oracle_nm_mask(int64_t total, const float* w, int n, int m, float* mask) {
    if (n <= 0 || m <= 0 || n > m || m > 64) return -1;
    for (int64_t i = 0; i < total; i += m) {
        const int g = (int)((total - i) < m ? (total - i) : m);
        int k = n;
        if (g < m) {
            /* nm_sparsity.cpp:88-90: ceil of a float quotient, capped at g */
            k = (int)ceilf((float)((size_t)g * (size_t)n) / (float)m);
            if (k > g) k = g;
        }
        nm_select(w + i, g, k, mask + i);
    }
    return 0;
}
