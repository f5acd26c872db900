// sparsify.cpp -- see sparsify.hpp.
#include "sparsify.hpp"

#include <algorithm>
#include <cmath>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <unordered_set>

#include "pyflame_rt/node.hpp"
#include "pyflame_rt/tensor.hpp"

namespace pyflame_rt {
namespace cuda {

std::vector<float> magnitude_mask(const float* w, int64_t n, float sparsity) {
    std::vector<float> mask(static_cast<size_t>(n), 1.0f);
    if (sparsity <= 0.0f) return mask;  // magnitude_pruning.cpp:33-39
    if (sparsity >= 1.0f) {             // :41-47
        std::fill(mask.begin(), mask.end(), 0.0f);
        return mask;
    }
    if (n == 0) throw std::runtime_error("Cannot prune empty weight tensor");  // :54-56
    std::vector<float> scores(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) scores[i] = std::abs(w[i]);
    // :66-74: the element at floor(n*s) of the sorted magnitudes (double product).
    size_t idx = static_cast<size_t>(std::floor(static_cast<double>(n) * sparsity));
    idx = std::min(idx, static_cast<size_t>(n) - 1);
    std::nth_element(scores.begin(), scores.begin() + static_cast<std::ptrdiff_t>(idx), scores.end());
    const float thr = scores[idx];
    size_t zeros = 0;
    for (int64_t i = 0; i < n; ++i) {
        mask[i] = (std::abs(w[i]) > thr) ? 1.0f : 0.0f;
        zeros += mask[i] == 0.0f;
    }
    // :84-98: size_t * float is evaluated in float; ties restored in index order.
    const size_t target = static_cast<size_t>(static_cast<float>(n) * sparsity);
    if (zeros > target) {
        size_t restore = zeros - target;
        for (int64_t i = 0; i < n && restore > 0; ++i)
            if (mask[i] == 0.0f && std::abs(w[i]) == thr) {
                mask[i] = 1.0f;
                --restore;
            }
    }
    return mask;
}

namespace {

const Tensor* find_init(const Graph& g, const std::string& name) {
    auto t = g.get_initializer(name);
    return t ? &t->get() : nullptr;
}

struct Csr {
    std::vector<int32_t> indptr, indices;
    std::vector<float> values;
};

// CSR of W [N, K] where W[n][k] = B(k, n), B stored [K, N] (trans = false) or
// [N, K] (trans = true), masked elementwise in B's storage order; an entry is
// kept when |B * mask| > 0 (to_sparse with threshold 0), in column order.
Csr build_csr(const float* b, const float* mask, int64_t N, int64_t K, bool trans) {
    Csr c;
    c.indptr.reserve(static_cast<size_t>(N) + 1);
    c.indptr.push_back(0);
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            const int64_t at = trans ? n * K + k : k * N + n;
            const float d = b[at] * (mask ? mask[at] : 1.0f);
            if (std::abs(d) > 0.0f) {
                c.indices.push_back(static_cast<int32_t>(k));
                c.values.push_back(d);
            }
        }
        if (c.indices.size() > static_cast<size_t>(INT32_MAX))
            throw std::runtime_error("sparsify: more than 2^31 nonzeros in one weight");
        c.indptr.push_back(static_cast<int32_t>(c.indices.size()));
    }
    return c;
}

Tensor to_tensor_i32(const std::vector<int32_t>& v) {
    Tensor t(std::vector<int64_t>{static_cast<int64_t>(v.size())}, DType::Int32);
    std::copy(v.begin(), v.end(), t.data_ptr<int32_t>());
    return t;
}

Tensor to_tensor_f32(const std::vector<float>& v) {
    Tensor t(std::vector<int64_t>{static_cast<int64_t>(v.size())}, DType::Float32);
    std::copy(v.begin(), v.end(), t.data_ptr<float>());
    return t;
}

}  // namespace

// The heap selection of libstdc++'s std::partial_sort over one group: a
// binary heap over the first k slots, top = the element no other precedes
// under |w[a]| > |w[b]|, built bottom-up; each later element that precedes the
// top replaces it.  A sift moves the hole to a leaf along the preferred child
// (the right one unless it precedes the left), then sifts the value up.  The
// order of these moves decides which of equal |w| stay.
namespace {
void nm_sift(const float* a, int* h, int hole, int len, int v) {
    const int top = hole;
    int child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (a[h[child]] > a[h[child - 1]]) child--;
        h[hole] = h[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        h[hole] = h[child - 1];
        hole = child - 1;
    }
    int parent = (hole - 1) / 2;
    while (hole > top && a[h[parent]] > a[v]) {
        h[hole] = h[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    h[hole] = v;
}
}  // namespace

std::vector<float> nm_mask(const float* w, int64_t total, int n, int m) {
    if (n > m) throw std::invalid_argument("N must be <= M in N:M sparsity");
    if (n <= 0 || m <= 0) throw std::invalid_argument("N and M must be > 0");
    if (m > 64) throw std::invalid_argument("N:M pruning: M above 64");
    std::vector<float> mask(static_cast<size_t>(total), 0.0f);
    float a[64];
    int h[64];
    for (int64_t i = 0; i < total; i += m) {
        const int g = static_cast<int>(std::min<int64_t>(m, total - i));
        int k = n;
        if (g < m)
            k = std::min(g, static_cast<int>(std::ceil(static_cast<float>(static_cast<size_t>(g) * n) /
                                                       static_cast<float>(m))));
        for (int j = 0; j < g; ++j) a[j] = std::fabs(w[i + j]);
        for (int j = 0; j < k; ++j) h[j] = j;
        if (k >= 2)
            for (int parent = (k - 2) / 2;; --parent) {
                nm_sift(a, h, parent, k, h[parent]);
                if (parent == 0) break;
            }
        for (int j = k; j < g; ++j)
            if (a[j] > a[h[0]]) nm_sift(a, h, 0, k, j);
        for (int j = 0; j < k; ++j) mask[static_cast<size_t>(i + h[j])] = 1.0f;
    }
    return mask;
}

Graph sparsify_matmuls(const Graph& g, const SparsifyOptions& opt, SparsifyReport* report) {
    SparsifyReport rep;
    Graph out(g.name());
    for (const auto& i : g.inputs()) out.add_input(i);
    for (const auto& o : g.outputs()) out.add_output(o);
    std::vector<std::shared_ptr<Node>> nodes;
    std::unordered_map<std::string, Tensor> new_inits;
    for (const auto& np : g.nodes()) {
        const Node& n = *np;
        const bool is_mm = n.op_type() == "MatMul" && n.inputs().size() == 2;
        const bool is_gemm = n.op_type() == "Gemm" && (n.inputs().size() == 2 || n.inputs().size() == 3);
        const Tensor* B = (is_mm || is_gemm) ? find_init(g, n.inputs()[1]) : nullptr;
        bool ok = B && B->dtype() == DType::Float32 && B->shape().size() == 2 && n.outputs().size() == 1;
        bool trans = false;
        const Tensor* C = nullptr;
        if (ok && is_gemm) {
            trans = n.get_attr<int64_t>("transB", 0) != 0;
            ok = n.get_attr<int64_t>("transA", 0) == 0 && n.get_attr<float>("alpha", 1.0f) == 1.0f;
            if (ok && n.inputs().size() == 3 && !n.inputs()[2].empty()) {
                C = find_init(g, n.inputs()[2]);
                const int64_t N = trans ? B->shape()[0] : B->shape()[1];
                ok = C && C->dtype() == DType::Float32 && C->num_elements() == N &&
                     n.get_attr<float>("beta", 1.0f) == 1.0f;
            }
        }
        if (!ok) {
            nodes.push_back(np);
            continue;
        }
        const int64_t K = trans ? B->shape()[1] : B->shape()[0];
        const int64_t N = trans ? B->shape()[0] : B->shape()[1];
        const int64_t total = K * N;
        std::vector<float> mask;
        if (opt.nm_n > 0) mask = nm_mask(B->data_ptr<float>(), total, opt.nm_n, opt.nm_m);
        else if (opt.prune_sparsity > 0.0f) mask = magnitude_mask(B->data_ptr<float>(), total, opt.prune_sparsity);
        Csr csr = build_csr(B->data_ptr<float>(), mask.empty() ? nullptr : mask.data(), N, K, trans);
        const double zero_frac = total > 0 ? 1.0 - static_cast<double>(csr.values.size()) / static_cast<double>(total) : 0.0;
        if (zero_frac < opt.min_zero_fraction) {
            nodes.push_back(np);
            continue;
        }
        const std::string base = n.name() + "_csr";
        new_inits.emplace(base + "_indptr", to_tensor_i32(csr.indptr));
        new_inits.emplace(base + "_indices", to_tensor_i32(csr.indices));
        new_inits.emplace(base + "_values", to_tensor_f32(csr.values));
        const std::string y = C ? n.name() + "_spmm_out" : n.outputs()[0];
        auto sp = std::make_shared<Node>(C ? n.name() + "_spmm" : n.name(), "SparseMatMul",
                                         std::vector<std::string>{n.inputs()[0], base + "_indptr", base + "_indices",
                                                                  base + "_values"},
                                         std::vector<std::string>{y});
        sp->set_attr("shape", std::vector<int64_t>{N, K});
        nodes.push_back(sp);
        if (C)
            nodes.push_back(std::make_shared<Node>(n.name(), "Add", std::vector<std::string>{y, n.inputs()[2]},
                                                   n.outputs()));
        ++rep.rewritten;
        rep.dense_bytes += 4 * total;
        rep.csr_bytes += static_cast<int64_t>(4 * csr.indptr.size() + 8 * csr.values.size());
    }
    // Keep the initializers some node still reads.
    std::unordered_set<std::string> used;
    for (const auto& np : nodes)
        for (const auto& in : np->inputs()) used.insert(in);
    for (const auto& kv : g.initializers())
        if (used.count(kv.first)) out.add_initializer(kv.first, kv.second);
    for (auto& kv : new_inits) out.add_initializer(kv.first, kv.second);
    for (auto& np : nodes) out.add_node(np);
    if (report) *report = rep;
    return out;
}

}  // namespace cuda
}  // namespace pyflame_rt
