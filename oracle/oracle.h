/*
 * oracle.h -- CPU restatement of the PyFlameRT reference hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (pyflamert_b200/, the
 * C-ABI library, the CUDA kernels) may include, link or call this file.  It
 * exists so that tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg can check the CUDA path against the reference's own arithmetic.
 *
 * Each function restates one reference routine, in the same evaluation
 * order, so that fp32 results are bit-identical to the reference built with
 * the same compiler flags (-O2 -ffp-contract=off, x86-64 baseline: no FMA).
 * The restatement is pinned against the reference compiled from its own
 * sources (oracle/_ref, see oracle/Makefile) by tests/test_oracle.py.
 *
 * Layouts are dense row-major, as in the reference Tensor
 * (include/pyflame_rt/tensor.hpp:12-90).
 */
#ifndef PFRT_ORACLE_H
#define PFRT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Gemm: Y = alpha*op(A)*op(B) + beta*C[i % c_len].
 * Follows cpu_gemm, src/backends/cpu/ops/math.cpp:377-438. */
void oracle_gemm_f32(int64_t M, int64_t N, int64_t K, int trans_a, int trans_b,
                     float alpha, float beta, const float* A, const float* B,
                     const float* C, int64_t c_len, float* Y);

/* 2-D MatMul fast path: Y = A[M,K] * B[K,N].
 * Follows cpu_matmul, src/backends/cpu/ops/math.cpp:326-336. */
void oracle_matmul_f32(int64_t M, int64_t N, int64_t K, const float* A,
                       const float* B, float* Y);

/* Exact integer accumulators of the quantized matmul:
 *   acc[m,n] = sum_k (a[m,k]-a_zp) * (w[k,n]-w_zp)   (int64, as quant_ops.cpp:443-466)
 * a is uint8 when a_is_u8 else int8; w is int8 stored [K,N] (reference B layout). */
void oracle_qmm_acc(int64_t M, int64_t N, int64_t K, const void* a, int a_is_u8,
                    int32_t a_zp, const int8_t* w, int32_t w_zp, int64_t* acc);

/* Per-output-channel quantized linear layer, composed from the reference's
 * arithmetic (quant_ops.cpp:435,464 for dequant; math.cpp:225 for the bias
 * add; activation.cpp:56 for ReLU; quant_ops.cpp:42-55 for requant):
 *   os[n] = a_scale * w_scale[n]                      (fp32 product)
 *   y     = (float)acc[m,n] * os[n]
 *   y     = y + bias[n]                               (if bias)
 *   y     = max(0.0f, y)                              (if relu)
 *   q     = clamp((int32)round(y * (1.0f/y_scale)) + y_zp, qmin, qmax)
 * Output: y_f32 when out_mode == 0 (fp32, no requant), else int8 (out_mode 1)
 * or uint8 (out_mode 2) in y_q.  acc_out (nullable) receives the int64
 * accumulators narrowed to int32. */
void oracle_qlinear(int64_t M, int64_t N, int64_t K, const void* a, int a_is_u8,
                    float a_scale, int32_t a_zp, const int8_t* w, int32_t w_zp,
                    const float* w_scale, const float* bias, int relu,
                    int out_mode, float y_scale, int32_t y_zp, float* y_f32,
                    void* y_q, int32_t* acc_out);

/* The dequant / bias / ReLU / requant tail of oracle_qlinear applied to given
 * exact accumulators acc[M,N] (int64). */
void oracle_qepilogue(int64_t M, int64_t N, const int64_t* acc, float a_scale,
                      const float* w_scale, const float* bias, int relu, int out_mode,
                      float y_scale, int32_t y_zp, float* y_f32, void* y_q);

/* Requantize fp32 -> int8/uint8, per tensor.
 * Follows quantize_tensor, src/quantization/quant_ops.cpp:15-55. */
void oracle_quantize(int64_t n, const float* x, float scale, int32_t zp,
                     int out_is_u8, void* q);

/* CSR SpMM, sparse operand on the left:
 *   Yt[r, c] = sum_{j in row r, storage order} values[j] * B[indices[j], c]
 * with W [R, Kw] CSR and B [Kw, C] dense.  Follows sparse_matmul,
 * src/pruning/sparse_tensor.cpp:473-519 (int64 indices there; int32 here,
 * which is the device format). */
void oracle_csr_spmm(int64_t R, int64_t C, const int32_t* indptr,
                     const int32_t* indices, const float* values,
                     const float* B, float* Yt);

/* Linear form used by the backend's SparseMatMul op:
 *   Y[M,N] = X[M,K] * W^T with W [N,K] in CSR.
 * Equal to transpose(oracle_csr_spmm(W, X^T)); computed directly with the
 * same per-output summation order (row r of W, nonzeros in storage order). */
void oracle_spmm_linear(int64_t M, int64_t N, int64_t K, const int32_t* indptr,
                        const int32_t* indices, const float* values,
                        const float* X, float* Y);

/* fp64 restatement of the linear SpMM, for accuracy reporting only. */
void oracle_spmm_linear_f64(int64_t M, int64_t N, int64_t K,
                            const int32_t* indptr, const int32_t* indices,
                            const float* values, const float* X, double* Y);

/* fp64 Gemm, for accuracy reporting only. */
void oracle_gemm_f64(int64_t M, int64_t N, int64_t K, int trans_a, int trans_b,
                     double alpha, double beta, const float* A, const float* B,
                     const float* C, int64_t c_len, double* Y);

/* pruning::MagnitudePruning::compute_mask (src/pruning/magnitude_pruning.cpp:
 * 22-102) on n weights: mask[i] = 1 keeps w[i], 0 prunes it.
 *   sparsity <= 0: keep all; sparsity >= 1: prune all;
 *   threshold = the floor(n*sparsity)-th smallest |w| (0-based, capped at
 *   n-1), keep |w| > threshold; if more than (size_t)((float)n * sparsity)
 *   weights are pruned, keep again the first entries (in index order) with
 *   |w| == threshold until that count is reached.
 * Returns -1 for n == 0 with 0 < sparsity < 1 (the reference throws), else 0.
 * Weights must not be NaN (the reference's sort is then undefined). */
int oracle_magnitude_mask(int64_t n, const float* w, float sparsity, float* mask);

/* pruning::NMSparsityPruning(n, m).compute_mask (src/pruning/nm_sparsity.cpp:
 * 45-126) on `total` weights in flat order: every m consecutive weights keep
 * the n with the largest |w|; a last group of g < m weights keeps
 * min(ceil((float)(g*n) / m), g).  Which of equal |w| are kept follows the
 * reference's std::partial_sort as libstdc++ (GCC 13) implements it: a heap
 * selection keyed by |w[a]| > |w[b]| (oracle.c restates it step for step).
 * Returns 0, or -1 for n == 0, m == 0 or n > m (the constructor's errors). */
int oracle_nm_mask(int64_t total, const float* w, int n, int m, float* mask);

/* pruning::to_sparse(D, threshold, CSR) (src/pruning/sparse_tensor.cpp:
 * 560-587) on D = W * mask (elementwise, fp32), threshold 0: row r keeps the
 * columns with |D[r][c]| > 0, in column order.  indptr [rows+1]; indices and
 * values must hold the number of nonzeros (at most rows*cols). */
void oracle_masked_csr(int64_t rows, int64_t cols, const float* w, const float* mask, int32_t* indptr,
                       int32_t* indices, float* values);

#ifdef __cplusplus
}
#endif

#endif /* PFRT_ORACLE_H */
