// sparsify.hpp -- the "pruning -> CSR" graph pass of the CUDA backend.
//
// Rewrites MatMul / Gemm nodes whose weight is a float32 initializer into the
// backend's SparseMatMul (Y = X W^T with W in CSR, int32 initializers), so
// that a model pruned by the reference's pruner -- or pruned here, with the
// reference's magnitude criterion -- runs on the CSR SpMM kernels.  The
// reference's own conversion route is MagnitudePruning::compute_mask
// (src/pruning/magnitude_pruning.cpp:22-102), WeightPruner::apply (which
// multiplies the weights by the mask; src/pruning/pruning.cpp) and
// pruning::to_sparse (src/pruning/sparse_tensor.cpp:560-587).
//
// A node is rewritten when
//   MatMul(X, B)               B a 2-D [K, N] initializer, or
//   Gemm(X, B[, C])            transA = 0, alpha = 1, B [K, N] (transB = 0) or
//                              [N, K] (transB = 1), and C absent, or beta = 1
//                              with C an [N] initializer (kept as an Add)
// and at least min_zero_fraction of the (pruned) weight is zero.  With
// prune_sparsity > 0 each such weight is first masked by compute_mask's
// criterion over its own element order; with nm_n > 0 instead, by
// NMSparsityPruning(nm_n, nm_m)'s (src/pruning/nm_sparsity.cpp:45-126), also
// over the weight's storage order.  The graph is returned as a new
// Graph; initializers no longer used by any node are dropped.
#pragma once

#include <cstdint>
#include <vector>

#include "pyflame_rt/graph.hpp"

namespace pyflame_rt {
namespace cuda {

struct SparsifyOptions {
    float prune_sparsity = 0.0f;
    float min_zero_fraction = 0.5f;
    int nm_n = 0;  // > 0: N:M pruning (keep nm_n of every nm_m) instead of magnitude
    int nm_m = 4;
};

struct SparsifyReport {
    int rewritten = 0;
    int64_t dense_bytes = 0;  // float32 bytes of the replaced weights
    int64_t csr_bytes = 0;    // bytes of their CSR initializers
};

Graph sparsify_matmuls(const Graph& graph, const SparsifyOptions& options = {}, SparsifyReport* report = nullptr);

// compute_mask's criterion on n weights in their storage order (1 keeps):
// threshold = the floor(n*s)-th smallest |w| (capped at n-1); keep |w| >
// threshold; while more than (size_t)((float)n * s) weights are pruned, keep
// the next tie (|w| == threshold) in index order.  s <= 0 keeps all, s >= 1
// prunes all; n == 0 with 0 < s < 1 throws std::runtime_error, as the
// reference does.
std::vector<float> magnitude_mask(const float* w, int64_t n, float sparsity);

// NMSparsityPruning(n, m)::compute_mask on `total` weights in storage order
// (1 keeps): every m consecutive weights keep the n largest |w|; a last group
// of g < m keeps min(ceil((float)(g*n) / m), g).  Equal |w| are chosen as the
// reference's std::partial_sort (libstdc++, a heap selection) chooses them.
// Throws std::invalid_argument for n > m or n, m == 0, as the reference's
// constructor; m above 64 is rejected too.
std::vector<float> nm_mask(const float* w, int64_t total, int n, int m);

}  // namespace cuda
}  // namespace pyflame_rt
