// test_session_seam.cpp -- the drop-in check: the reference's own
// InferenceSession (src/session.cpp), built with the seam that lets
// SessionOptions.device = "cuda" (or "cuda:<n>") select CudaBackend
// (options.cpp:12-17 and select_backend, session.cpp:67-95), loads a .pfm
// model written by the reference's PyFlameFormat::save and runs it on "cuda",
// "cuda:0" and "cpu"; the outputs are compared.  Graph, loader, session and run() are the reference's
// code; only the backend differs.  TEST INFRASTRUCTURE; needs a B200.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <random>
#include <string>
#include <unistd.h>

#include "io/pyflame_format.hpp"
#include "pyflame_rt/errors.hpp"
#include "pyflame_rt/graph.hpp"
#include "pyflame_rt/options.hpp"
#include "pyflame_rt/session.hpp"

using namespace pyflame_rt;

namespace {

Shape sh(std::vector<int64_t> d) {
    Shape s;
    for (auto v : d) s.push_back(v);
    return s;
}

Tensor randn(std::vector<int64_t> shape, float stddev, uint64_t seed) {
    Tensor t(shape, DType::Float32);
    std::mt19937_64 rng(seed);
    std::normal_distribution<float> nd(0.0f, stddev);
    for (int64_t i = 0; i < t.num_elements(); ++i) t.data_ptr<float>()[i] = nd(rng);
    return t;
}

Tensor randi8(std::vector<int64_t> shape, int lo, int hi, uint64_t seed) {
    Tensor t(shape, DType::Int8);
    std::mt19937_64 rng(seed);
    std::uniform_int_distribution<int> d(lo, hi);
    for (int64_t i = 0; i < t.num_elements(); ++i) t.data_ptr<int8_t>()[i] = static_cast<int8_t>(d(rng));
    return t;
}

}  // namespace

int main() {
    // One model with the three hot-path forms side by side.
    Graph g("seam_model");
    g.add_input(TensorInfo("X", sh({256, 1024}), DType::Float32));
    g.add_input(TensorInfo("Xq", sh({128, 512}), DType::Int8));
    g.add_initializer("B", randn({1024, 1024}, 1.0f / 32.0f, 2));
    g.add_initializer("C", randn({1024}, 0.1f, 3));
    auto gemm = std::make_shared<Node>("gemm", "Gemm", std::vector<std::string>{"X", "B", "C"},
                                       std::vector<std::string>{"Y"});
    gemm->set_attr("alpha", 1.0f);
    gemm->set_attr("beta", 1.0f);
    g.add_node(gemm);
    g.add_initializer("W", randi8({512, 384}, -127, 127, 4));
    g.add_initializer("bias", randn({384}, 10.0f, 5));
    auto q = std::make_shared<Node>("qmm", "QuantizedMatMul", std::vector<std::string>{"Xq", "W"},
                                    std::vector<std::string>{"t0"});
    q->set_attr("a_scale", 0.02f);
    q->set_attr("b_scale", 0.0125f);
    g.add_node(q);
    g.add_node(std::make_shared<Node>("add", "Add", std::vector<std::string>{"t0", "bias"},
                                      std::vector<std::string>{"t1"}));
    g.add_node(std::make_shared<Node>("relu", "Relu", std::vector<std::string>{"t1"},
                                      std::vector<std::string>{"t2"}));
    auto qz = std::make_shared<Node>("quant", "Quantize", std::vector<std::string>{"t2"},
                                     std::vector<std::string>{"Yq"});
    qz->set_attr("scale", 0.5f);
    qz->set_attr("dtype", std::string("int8"));
    g.add_node(qz);
    g.add_output(TensorInfo("Y", sh({256, 1024}), DType::Float32));
    g.add_output(TensorInfo("Yq", sh({128, 384}), DType::Int8));

    char tmpl[] = "/tmp/pfrt_seam_XXXXXX";
    const int fd = mkstemp(tmpl);
    if (fd < 0) return 2;
    close(fd);
    const std::string path = std::string(tmpl) + ".pfm";
    std::rename(tmpl, path.c_str());
    PyFlameFormat::save(g, path);

    std::unordered_map<std::string, Tensor> feeds;
    feeds["X"] = randn({256, 1024}, 1.0f, 1);
    feeds["Xq"] = randi8({128, 512}, -128, 127, 6);

    int failed = 0;
    try {
        SessionOptions cpu_opts;
        cpu_opts.optimization_level = OptLevel::None;
        SessionOptions cuda_opts = cpu_opts;
        cuda_opts.device = "cuda";
        SessionOptions cuda0_opts = cpu_opts;
        cuda0_opts.device = "cuda:0";  // a device ordinal in the device string
        InferenceSession cpu(path, cpu_opts);
        InferenceSession cuda(path, cuda_opts);
        InferenceSession cuda0(path, cuda0_opts);
        const std::vector<std::string> outs = {"Y", "Yq"};
        for (int rep = 0; rep < 2; ++rep) {
            auto r = cpu.run(outs, feeds);
            auto y = (rep == 0 ? cuda : cuda0).run(outs, feeds);
            double num = 0, den = 0;
            for (int64_t i = 0; i < r[0].num_elements(); ++i) {
                num = std::max(num, std::fabs(static_cast<double>(y[0].data_ptr<float>()[i]) - r[0].data_ptr<float>()[i]));
                den = std::max(den, std::fabs(static_cast<double>(r[0].data_ptr<float>()[i])));
            }
            const bool gemm_ok = num / den <= 1e-5;
            const bool q_ok = y[1].dtype() == DType::Int8 && y[1].shape() == r[1].shape() &&
                              std::memcmp(y[1].data(), r[1].data(), r[1].size_bytes()) == 0;
            std::printf("%s SessionGemm run %d (normwise %.3g)\n", gemm_ok ? "PASS" : "FAIL", rep, num / den);
            std::printf("%s SessionQuantizedChain run %d\n", q_ok ? "PASS" : "FAIL", rep);
            failed += !gemm_ok + !q_ok;
        }
    } catch (const std::exception& e) {
        std::printf("FAIL Session: %s\n", e.what());
        ++failed;
    }
    std::remove(path.c_str());
    std::printf("%s: %d failed\n", failed ? "FAILED" : "OK", failed);
    return failed ? 1 : 0;
}
