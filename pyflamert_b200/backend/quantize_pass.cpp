// quantize_pass.cpp -- see quantize_pass.hpp.
#include "quantize_pass.hpp"

#include <algorithm>
#include <cmath>
#include <limits>
#include <memory>
#include <unordered_set>
#include <vector>

#include "pyflame_rt/node.hpp"
#include "pyflame_rt/tensor.hpp"

namespace pyflame_rt {
namespace cuda {
namespace {

// QuantParams::compute_from_minmax for UInt8, asymmetric (quant_params.cpp:14-55).
void act_params(float min_val, float max_val, float* scale, int32_t* zp) {
    const int32_t qmin = 0, qmax = 255;
    if (std::abs(max_val - min_val) < 1e-8f) {
        *scale = 1.0f;
        *zp = 0;
        return;
    }
    float s = (max_val - min_val) / static_cast<float>(qmax - qmin);
    int32_t z = qmin - static_cast<int32_t>(std::round(min_val / s));
    z = std::clamp(z, qmin, qmax);
    if (s < 1e-10f) s = 1e-10f;
    *scale = s;
    *zp = z;
}

// compute_dynamic_params_per_channel(B, axis 1, Int8, symmetric) + QuantizedTensor
// on B [K, N]: scales[n], Bq (int8, zero point 0).
void quantize_weight_per_channel(const float* b, int64_t K, int64_t N, std::vector<float>& scales,
                                 std::vector<int8_t>& q) {
    std::vector<float> mn(static_cast<size_t>(N), std::numeric_limits<float>::max());
    std::vector<float> mx(static_cast<size_t>(N), std::numeric_limits<float>::lowest());
    for (int64_t k = 0; k < K; ++k)
        for (int64_t n = 0; n < N; ++n) {
            const float v = b[k * N + n];
            if (std::isfinite(v)) {
                mn[n] = std::min(mn[n], v);
                mx[n] = std::max(mx[n], v);
            }
        }
    scales.assign(static_cast<size_t>(N), 1.0f);
    for (int64_t n = 0; n < N; ++n) {
        if (mn[n] > mx[n]) mn[n] = mx[n] = 0.0f;
        if (std::abs(mx[n] - mn[n]) < 1e-8f) {
            scales[n] = 1.0f;  // zero point 0 as well
            continue;
        }
        const float abs_max = std::max(std::abs(mn[n]), std::abs(mx[n]));
        float s = abs_max / 127.0f;
        if (s < 1e-10f) s = 1e-10f;
        scales[n] = s;
    }
    q.resize(static_cast<size_t>(K * N));
    for (int64_t k = 0; k < K; ++k)
        for (int64_t n = 0; n < N; ++n) {
            const float inv = 1.0f / scales[n];
            const int32_t v = static_cast<int32_t>(std::round(b[k * N + n] * inv));
            q[k * N + n] = static_cast<int8_t>(std::clamp(v, -128, 127));
        }
}

}  // namespace

Graph quantize_matmuls_per_channel(const Graph& g, const QuantizePassOptions& opt, QuantizePassReport* report) {
    QuantizePassReport rep;
    Graph out(g.name());
    for (const auto& i : g.inputs()) out.add_input(i);
    for (const auto& o : g.outputs()) out.add_output(o);
    std::vector<std::shared_ptr<Node>> nodes;
    std::vector<std::pair<std::string, Tensor>> new_inits;
    for (const auto& np : g.nodes()) {
        const Node& n = *np;
        auto rng = n.inputs().empty() ? opt.act_ranges.end() : opt.act_ranges.find(n.inputs()[0]);
        const bool mm = n.op_type() == "MatMul" && n.inputs().size() == 2 && n.outputs().size() == 1;
        auto binit = mm ? g.get_initializer(n.inputs()[1]) : std::nullopt;
        if (!mm || rng == opt.act_ranges.end() || !binit || binit->get().dtype() != DType::Float32 ||
            binit->get().shape().size() != 2) {
            nodes.push_back(np);
            continue;
        }
        const Tensor& B = binit->get();
        const int64_t K = B.shape()[0], N = B.shape()[1];
        std::vector<float> scales;
        std::vector<int8_t> q;
        quantize_weight_per_channel(B.data_ptr<float>(), K, N, scales, q);
        float a_scale;
        int32_t a_zp;
        act_params(rng->second.first, rng->second.second, &a_scale, &a_zp);
        Tensor bq(std::vector<int64_t>{K, N}, DType::Int8);
        std::copy(q.begin(), q.end(), bq.data_ptr<int8_t>());
        const std::string wq = n.inputs()[1] + "_q8";
        const std::string xq = n.inputs()[0] + "_q8_" + n.name();
        new_inits.emplace_back(wq, bq);
        auto qz = std::make_shared<Node>(n.name() + "_quantize_input", "Quantize",
                                         std::vector<std::string>{n.inputs()[0]}, std::vector<std::string>{xq});
        qz->set_attr("scale", a_scale);
        qz->set_attr("zero_point", static_cast<int64_t>(a_zp));
        qz->set_attr("dtype", std::string("uint8"));
        auto qm = std::make_shared<Node>(n.name(), "QuantizedMatMul", std::vector<std::string>{xq, wq}, n.outputs());
        qm->set_attr("a_scale", a_scale);
        qm->set_attr("a_zero_point", static_cast<int64_t>(a_zp));
        qm->set_attr("b_scales", scales);
        qm->set_attr("b_zero_point", static_cast<int64_t>(0));
        nodes.push_back(qz);
        nodes.push_back(qm);
        ++rep.rewritten;
    }
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
