// test_cuda_backend.cpp -- the PyFlameRT Backend plugin (CudaBackend) against
// the reference's own CPUExecutor, in the style of the reference's
// tests/cpp/test_executor.cpp: graphs are built in-process from Graph, Node and
// Tensor, run on both backends, and compared.
//
// Links the reference runtime compiled from its sources (oracle/_ref) and the
// C restatement (oracle/_build) as checkers, and the product libraries
// libpfrt_cuda_backend.so / libpfrt_cuda.so.  Needs a B200; run by
// tests/test_gpu_backend.py.  With --cpu it runs only the host-only checks
// (the batch-split plan and device strings; tests/test_backend_host.py).  Prints one "PASS name" or "FAIL name: why" line
// per test and exits non-zero if any test failed.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "backends/cpu/executor.hpp"
#include "cuda_backend.hpp"
#include "oracle.h"
#include "pyflame_rt/errors.hpp"
#include "pyflame_rt/graph.hpp"
#include "pyflame_rt/pruning/pruning.hpp"
#include "sparsify.hpp"
#include "quantize_pass.hpp"
#include "pyflame_rt/quantization/quant_ops.hpp"
#include "pyflame_rt/quantization/quant_params.hpp"

using namespace pyflame_rt;

namespace {

int g_failed = 0;

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

#define EXPECT(cond, msg)                   \
    do {                                    \
        if (!(cond)) throw Failure(msg);    \
    } while (0)

void run_test(const char* name, const std::function<void()>& fn) {
    try {
        fn();
        std::printf("PASS %s\n", name);
    } catch (const std::exception& e) {
        std::printf("FAIL %s: %s\n", name, e.what());
        ++g_failed;
    }
    std::fflush(stdout);
}

Shape sh(std::vector<int64_t> d) {
    Shape s;
    for (auto v : d) s.push_back(v);
    return s;
}

Tensor randn(std::vector<int64_t> shape, float stddev, uint64_t seed) {
    Tensor t(shape, DType::Float32);
    std::mt19937_64 rng(seed);
    std::normal_distribution<float> nd(0.0f, stddev);
    float* p = t.data_ptr<float>();
    for (int64_t i = 0; i < t.num_elements(); ++i) p[i] = nd(rng);
    return t;
}

template <class T>
Tensor randint(std::vector<int64_t> shape, int lo, int hi, DType dt, uint64_t seed) {
    Tensor t(shape, dt);
    std::mt19937_64 rng(seed);
    std::uniform_int_distribution<int> d(lo, hi);
    T* p = t.data_ptr<T>();
    for (int64_t i = 0; i < t.num_elements(); ++i) p[i] = static_cast<T>(d(rng));
    return t;
}

double normwise(const Tensor& a, const Tensor& b) {
    const float* x = a.data_ptr<float>();
    const float* y = b.data_ptr<float>();
    double num = 0, den = 0;
    for (int64_t i = 0; i < a.num_elements(); ++i) {
        num = std::max(num, std::fabs(static_cast<double>(x[i]) - y[i]));
        den = std::max(den, std::fabs(static_cast<double>(y[i])));
    }
    return den > 0 ? num / den : num;
}

bool same_bytes(const Tensor& a, const Tensor& b) {
    return a.shape() == b.shape() && a.dtype() == b.dtype() &&
           std::memcmp(a.data(), b.data(), a.size_bytes()) == 0;
}

std::shared_ptr<Node> node(const std::string& name, const std::string& op, std::vector<std::string> in,
                           std::vector<std::string> out) {
    return std::make_shared<Node>(name, op, std::move(in), std::move(out));
}

std::vector<Tensor> run(Backend& be, const Graph& g, const std::unordered_map<std::string, Tensor>& feeds) {
    return be.execute(g, feeds);
}

// A row-separable graph: X [M, 1024] -> Gemm(B, C[1024]) -> Y, and
// U [M, 512] uint8 -> QuantizedMatMul (per-channel) -> Add bias -> Relu ->
// Quantize uint8 -> Z.
Graph split_graph(int64_t M) {
    Graph g("split");
    g.add_input(TensorInfo("X", sh({M, 1024}), DType::Float32));
    g.add_input(TensorInfo("U", sh({M, 512}), DType::UInt8));
    g.add_initializer("B", randn({1024, 768}, 1.0f / 32.0f, 21));
    g.add_initializer("C", randn({768}, 0.1f, 22));
    auto gm = node("gemm", "Gemm", {"X", "B", "C"}, {"Y"});
    gm->set_attr("alpha", 1.0f);
    gm->set_attr("beta", 1.0f);
    g.add_node(gm);
    g.add_initializer("W", randint<int8_t>({512, 384}, -127, 127, DType::Int8, 23));
    g.add_initializer("bias", randn({384}, 10.0f, 24));
    std::vector<float> scales(384);
    std::mt19937_64 rng(25);
    std::uniform_real_distribution<float> ud(0.005f, 0.02f);
    for (auto& v : scales) v = ud(rng);
    auto q = node("qmm", "QuantizedMatMul", {"U", "W"}, {"t0"});
    q->set_attr("a_scale", 0.02f);
    q->set_attr("a_zero_point", int64_t{128});
    q->set_attr("b_scales", scales);
    g.add_node(q);
    g.add_node(node("add", "Add", {"t0", "bias"}, {"t1"}));
    g.add_node(node("relu", "Relu", {"t1"}, {"t2"}));
    auto qz = node("quant", "Quantize", {"t2"}, {"Z"});
    qz->set_attr("scale", 2.0f);
    qz->set_attr("dtype", std::string("uint8"));
    g.add_node(qz);
    g.add_output(TensorInfo("Y", sh({M, 768}), DType::Float32));
    g.add_output(TensorInfo("Z", sh({M, 384}), DType::UInt8));
    return g;
}

std::unordered_map<std::string, Tensor> split_feeds(int64_t M) {
    std::unordered_map<std::string, Tensor> f;
    f["X"] = randn({M, 1024}, 1.0f, 26);
    f["U"] = randint<uint8_t>({M, 512}, 0, 255, DType::UInt8, 27);
    return f;
}

// Host-only checks (no GPU): the batch-split plan and the device strings.
void host_tests() {
    run_test("BatchSplitPlanRows", [&] {
        Graph g = split_graph(1000);
        auto f = split_feeds(1000);
        auto plan = batch_split_plan(g, f, 4, 64);
        EXPECT(plan.size() == 4, "4 slices");
        EXPECT(plan.front().first == 0 && plan.back().second == 1000, "slices cover the batch");
        for (size_t i = 1; i < plan.size(); ++i) EXPECT(plan[i].first == plan[i - 1].second, "contiguous");
        EXPECT(batch_split_plan(g, f, 4, 300).empty(), "too few rows per device");
        EXPECT(batch_split_plan(g, f, 1, 1).empty(), "one device");
    });
    run_test("BatchSplitPlanRejects", [&] {
        auto f = split_feeds(512);
        {   // C of M*N elements: C[(m*N + n) % c_len] depends on the row
            Graph g = split_graph(512);
            Graph h("full_c");
            h.add_input(TensorInfo("X", sh({512, 64}), DType::Float32));
            h.add_initializer("B", randn({64, 8}, 1.0f, 1));
            h.add_initializer("C", randn({512 * 8}, 1.0f, 2));
            h.add_node(node("gemm", "Gemm", {"X", "B", "C"}, {"Y"}));
            h.add_output(TensorInfo("Y", sh({512, 8}), DType::Float32));
            std::unordered_map<std::string, Tensor> hf;
            hf["X"] = randn({512, 64}, 1.0f, 3);
            EXPECT(batch_split_plan(h, hf, 2, 1).empty(), "full-matrix C accepted");
            (void)g;
        }
        {   // transA
            Graph h("ta");
            h.add_input(TensorInfo("X", sh({512, 64}), DType::Float32));
            h.add_initializer("B", randn({512, 8}, 1.0f, 1));
            auto n = node("gemm", "Gemm", {"X", "B"}, {"Y"});
            n->set_attr("transA", int64_t{1});
            h.add_node(n);
            h.add_output(TensorInfo("Y", sh({64, 8}), DType::Float32));
            std::unordered_map<std::string, Tensor> hf;
            hf["X"] = randn({512, 64}, 1.0f, 3);
            EXPECT(batch_split_plan(h, hf, 2, 1).empty(), "transA accepted");
        }
        {   // a runtime weight
            Graph h("rt");
            h.add_input(TensorInfo("X", sh({512, 64}), DType::Float32));
            h.add_input(TensorInfo("W", sh({64, 8}), DType::Float32));
            h.add_node(node("mm", "MatMul", {"X", "W"}, {"Y"}));
            h.add_output(TensorInfo("Y", sh({512, 8}), DType::Float32));
            std::unordered_map<std::string, Tensor> hf;
            hf["X"] = randn({512, 64}, 1.0f, 3);
            hf["W"] = randn({64, 8}, 1.0f, 4);
            EXPECT(batch_split_plan(h, hf, 2, 1).empty(), "runtime weight accepted");
        }
        {   // inputs with different row counts
            Graph g = split_graph(512);
            auto bad = split_feeds(512);
            bad["U"] = randint<uint8_t>({256, 512}, 0, 255, DType::UInt8, 5);
            EXPECT(batch_split_plan(g, bad, 2, 1).empty(), "ragged inputs accepted");
        }
        (void)f;
    });
    run_test("CudaDeviceStrings", [&] {
        unsetenv("PFRT_CUDA_DEVICES");
        EXPECT(parse_cuda_devices("cuda") == std::vector<int>{0}, "cuda -> {0}");
        EXPECT(parse_cuda_devices("cuda:3") == std::vector<int>{3}, "cuda:3");
        EXPECT((parse_cuda_devices("cuda:0,1,2") == std::vector<int>{0, 1, 2}), "cuda:0,1,2");
        setenv("PFRT_CUDA_DEVICES", "1,0", 1);
        EXPECT((parse_cuda_devices("cuda") == std::vector<int>{1, 0}), "PFRT_CUDA_DEVICES");
        unsetenv("PFRT_CUDA_DEVICES");
        for (const char* bad : {"cpu", "cuda:", "cuda:x", "cuda:1,,2", "gpu:0"}) {
            bool threw = false;
            try {
                parse_cuda_devices(bad);
            } catch (const PyFlameRTError&) {
                threw = true;
            }
            EXPECT(threw, std::string("accepted ") + bad);
        }
    });
}

}  // namespace

int main(int argc, char** argv) {
    host_tests();
    if (argc > 1 && std::strcmp(argv[1], "--cpu") == 0) return g_failed ? 1 : 0;
    CudaBackend cuda(0);
    CPUExecutor cpu(0);

    // Two backends' worth of devices on device 0 (CudaBackend({0, 0})): the
    // batch split runs, with each slice on its own context; the outputs equal
    // the single-device backend's (int8 bit for bit, fp32 within 1e-5 of the
    // reference CPUExecutor).
    run_test("MultiDeviceBatchSplit", [&] {
        setenv("PFRT_SPLIT_MIN_ROWS", "64", 1);
        CudaBackend multi(std::vector<int>{0, 0});
        const int64_t M = 1000;
        Graph g = split_graph(M);
        auto f = split_feeds(M);
        EXPECT(batch_split_plan(g, f, 2, 64).size() == 2, "plan");
        auto y = multi.execute(g, f);
        auto one = cuda.execute(g, f);
        auto r = cpu.execute(g, f);
        EXPECT(y.size() == 2 && y[0].shape() == r[0].shape() && y[1].shape() == one[1].shape(), "shapes");
        const double e = normwise(y[0], r[0]);
        EXPECT(e <= 1e-5, "Gemm normwise error " + std::to_string(e));
        EXPECT(same_bytes(y[1], one[1]), "int8 chain differs from the single-device backend");
        auto y2 = multi.execute(g, f);  // prepared weights reused on both slices
        EXPECT(same_bytes(y[1], y2[1]), "second run differs");
        unsetenv("PFRT_SPLIT_MIN_ROWS");
    });

    // ExecutorTest.SupportedOps analogue (tests/cpp/test_executor.cpp:150-158).
    run_test("SupportedOps", [&] {
        EXPECT(cuda.name() == "cuda", "name");
        EXPECT(cuda.supports_op("MatMul") && cuda.supports_op("Gemm") && cuda.supports_op("QuantizedMatMul"),
               "hot-path ops must be supported");
        EXPECT(!cuda.supports_op("NonExistentOp"), "unknown op reported as supported");
    });

    // ExecutorTest.MatMul (tests/cpp/test_executor.cpp:162-208), same graph and values.
    run_test("MatMulKnownAnswer", [&] {
        Graph graph("test");
        graph.add_input(TensorInfo("a", sh({2, 3}), DType::Float32));
        graph.add_input(TensorInfo("b", sh({3, 2}), DType::Float32));
        graph.add_output(TensorInfo("c", sh({2, 2}), DType::Float32));
        graph.add_node(node("matmul_0", "MatMul", {"a", "b"}, {"c"}));
        Tensor a({2, 3}, DType::Float32), b({3, 2}, DType::Float32);
        float av[] = {1, 2, 3, 4, 5, 6}, bv[] = {1, 2, 3, 4, 5, 6};
        std::memcpy(a.data(), av, sizeof(av));
        std::memcpy(b.data(), bv, sizeof(bv));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["a"] = std::move(a);
        feeds["b"] = std::move(b);
        auto out = cuda.execute(graph, feeds);
        EXPECT(out.size() == 1, "one output");
        const float* o = out[0].data_ptr<float>();
        EXPECT(o[0] == 22.0f && o[1] == 28.0f && o[2] == 49.0f && o[3] == 64.0f, "[[22,28],[49,64]]");
    });

    // Config 1: Gemm with initializer B and bias C, alpha = beta = 1.
    run_test("GemmConfig1", [&] {
        Graph g("gemm");
        g.add_input(TensorInfo("A", sh({256, 1024}), DType::Float32));
        g.add_initializer("B", randn({1024, 1024}, 1.0f / 32.0f, 2));
        g.add_initializer("C", randn({1024}, 0.1f, 3));
        auto n = node("gemm_0", "Gemm", {"A", "B", "C"}, {"Y"});
        n->set_attr("alpha", 1.0f);
        n->set_attr("beta", 1.0f);
        g.add_node(n);
        g.add_output(TensorInfo("Y", sh({256, 1024}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["A"] = randn({256, 1024}, 1.0f, 1);
        auto y = run(cuda, g, feeds);
        auto r = run(cpu, g, feeds);
        const double e = normwise(y[0], r[0]);
        EXPECT(e <= 1e-5, "normwise error " + std::to_string(e));
        auto y2 = run(cuda, g, feeds);  // second run reuses the prepared weight
        EXPECT(same_bytes(y[0], y2[0]), "second run differs");
    });

    run_test("GemmTransposedRuntimeB", [&] {
        Graph g("gemm_t");
        g.add_input(TensorInfo("A", sh({70, 33}), DType::Float32));
        g.add_input(TensorInfo("B", sh({45, 70}), DType::Float32));
        auto n = node("gemm_t", "Gemm", {"A", "B"}, {"Y"});
        n->set_attr("alpha", 0.5f);
        n->set_attr("transA", int64_t{1});
        n->set_attr("transB", int64_t{1});
        g.add_node(n);
        g.add_output(TensorInfo("Y", sh({33, 45}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["A"] = randn({70, 33}, 1.0f, 4);
        feeds["B"] = randn({45, 70}, 1.0f, 5);
        const double e = normwise(run(cuda, g, feeds)[0], run(cpu, g, feeds)[0]);
        EXPECT(e <= 1e-5, "normwise error " + std::to_string(e));
    });

    run_test("MatMulBatchedBroadcast", [&] {
        Graph g("bmm");
        g.add_input(TensorInfo("A", sh({2, 3, 5, 7}), DType::Float32));
        g.add_initializer("W", randn({7, 4}, 1.0f, 6));
        g.add_input(TensorInfo("B", sh({3, 7, 4}), DType::Float32));
        g.add_node(node("mm_w", "MatMul", {"A", "W"}, {"Y1"}));
        g.add_node(node("mm_b", "MatMul", {"A", "B"}, {"Y2"}));
        g.add_output(TensorInfo("Y1", sh({2, 3, 5, 4}), DType::Float32));
        g.add_output(TensorInfo("Y2", sh({2, 3, 5, 4}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["A"] = randn({2, 3, 5, 7}, 1.0f, 7);
        feeds["B"] = randn({3, 7, 4}, 1.0f, 8);
        auto y = run(cuda, g, feeds);
        auto r = run(cpu, g, feeds);
        EXPECT(normwise(y[0], r[0]) <= 1e-5 && normwise(y[1], r[1]) <= 1e-5, "batched MatMul differs");
    });

    // QuantizedMatMul -> Add -> Relu -> Quantize on int8 x int8, where the
    // reference graph op (quantized_ops.cpp:77-167) is exact: fused kernel vs
    // the reference's four CPU ops, bit for bit.
    auto quant_chain = [&](bool expose_intermediate) {
        const int64_t M = 96, K = 256, N = 160;
        Graph g("qchain");
        g.add_input(TensorInfo("X", sh({M, K}), DType::Int8));
        g.add_initializer("W", randint<int8_t>({K, N}, -127, 127, DType::Int8, 9));
        g.add_initializer("bias", randn({N}, 10.0f, 10));
        auto q = node("qmm", "QuantizedMatMul", {"X", "W"}, {"t0"});
        q->set_attr("a_scale", 0.02f);
        q->set_attr("b_scale", 0.0125f);
        q->set_attr("a_zero_point", int64_t{3});
        q->set_attr("b_zero_point", int64_t{0});
        g.add_node(q);
        g.add_node(node("add", "Add", {"t0", "bias"}, {"t1"}));
        g.add_node(node("relu", "Relu", {"t1"}, {"t2"}));
        auto qz = node("quant", "Quantize", {"t2"}, {"Y"});
        qz->set_attr("scale", 0.7f);
        qz->set_attr("zero_point", int64_t{4});
        qz->set_attr("dtype", std::string("uint8"));
        g.add_node(qz);
        g.add_output(TensorInfo("Y", sh({M, N}), DType::UInt8));
        if (expose_intermediate) g.add_output(TensorInfo("t1", sh({M, N}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = randint<int8_t>({M, K}, -128, 127, DType::Int8, 11);
        auto y = run(cuda, g, feeds);
        auto r = run(cpu, g, feeds);
        EXPECT(y.size() == r.size(), "output count");
        for (size_t i = 0; i < y.size(); ++i) EXPECT(same_bytes(y[i], r[i]), "output " + std::to_string(i) + " differs");
    };
    run_test("QuantizedChainFused", [&] { quant_chain(false); });
    run_test("QuantizedChainUnfused", [&] { quant_chain(true); });

    // uint8 activations with per-output-channel scales (b_scales): checked
    // against the C restatement of quant_ops.cpp (the reference graph op
    // reads uint8 as int8, quantized_ops.cpp:143).
    run_test("QuantizedPerChannelUint8", [&] {
        const int64_t M = 64, K = 512, N = 200;
        Graph g("qpc");
        g.add_input(TensorInfo("X", sh({M, K}), DType::UInt8));
        Tensor w = randint<int8_t>({K, N}, -127, 127, DType::Int8, 12);
        g.add_initializer("W", w);
        Tensor bias = randn({N}, 10.0f, 13);
        g.add_initializer("bias", bias);
        std::vector<float> scales(N);
        std::mt19937_64 rng(14);
        std::uniform_real_distribution<float> ud(0.005f, 0.02f);
        for (auto& s : scales) s = ud(rng);
        auto q = node("qmm", "QuantizedMatMul", {"X", "W"}, {"t0"});
        q->set_attr("a_scale", 0.02f);
        q->set_attr("a_zero_point", int64_t{128});
        q->set_attr("b_scales", scales);
        g.add_node(q);
        g.add_node(node("add", "Add", {"t0", "bias"}, {"t1"}));
        g.add_node(node("relu", "Relu", {"t1"}, {"t2"}));
        auto qz = node("quant", "Quantize", {"t2"}, {"Y"});
        qz->set_attr("scale", 2.0f);
        qz->set_attr("dtype", std::string("uint8"));
        g.add_node(qz);
        g.add_output(TensorInfo("Y", sh({M, N}), DType::UInt8));
        Tensor x = randint<uint8_t>({M, K}, 0, 255, DType::UInt8, 15);
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = x;
        auto y = run(cuda, g, feeds);
        Tensor ref({M, N}, DType::UInt8);
        oracle_qlinear(M, N, K, x.data(), 1, 0.02f, 128, w.data_ptr<int8_t>(), 0, scales.data(),
                       bias.data_ptr<float>(), 1, 2, 2.0f, 0, nullptr, ref.data(), nullptr);
        EXPECT(same_bytes(y[0], ref), "per-channel uint8 chain differs from the reference arithmetic");
    });

    // The config-4 network at a small batch: 4 x (QuantizedMatMul -> Add -> Relu -> Quantize).
    run_test("Int8MlpFourLayers", [&] {
        const int64_t M = 32, H = 512;
        Graph g("mlp");
        g.add_input(TensorInfo("X", sh({M, H}), DType::UInt8));
        std::string cur = "X";
        float a_scale = 0.02f;
        int64_t a_zp = 128;
        const float y_scales[4] = {2.86f, 103.25f, 3800.03f, 189326.23f};
        std::vector<Tensor> ws, bs;
        std::vector<std::vector<float>> scs;
        Tensor x = randint<uint8_t>({M, H}, 0, 255, DType::UInt8, 16);
        for (int l = 0; l < 4; ++l) {
            const std::string s = std::to_string(l);
            ws.push_back(randint<int8_t>({H, H}, -127, 127, DType::Int8, 20 + l));
            bs.push_back(randn({H}, 10.0f, 30 + l));
            std::vector<float> sc(H);
            std::mt19937_64 rng(40 + l);
            std::uniform_real_distribution<float> ud(0.005f, 0.02f);
            for (auto& v : sc) v = ud(rng);
            scs.push_back(sc);
            g.add_initializer("W" + s, ws.back());
            g.add_initializer("b" + s, bs.back());
            auto q = node("qmm" + s, "QuantizedMatMul", {cur, "W" + s}, {"q" + s});
            q->set_attr("a_scale", a_scale);
            q->set_attr("a_zero_point", a_zp);
            q->set_attr("b_scales", sc);
            g.add_node(q);
            g.add_node(node("add" + s, "Add", {"q" + s, "b" + s}, {"a" + s}));
            g.add_node(node("relu" + s, "Relu", {"a" + s}, {"r" + s}));
            auto qz = node("quant" + s, "Quantize", {"r" + s}, {"h" + s});
            qz->set_attr("scale", y_scales[l]);
            qz->set_attr("dtype", std::string("uint8"));
            g.add_node(qz);
            cur = "h" + s;
            a_scale = y_scales[l];
            a_zp = 0;
        }
        g.add_output(TensorInfo(cur, sh({M, H}), DType::UInt8));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = x;
        auto y = run(cuda, g, feeds);
        Tensor h = x;
        float as = 0.02f;
        int32_t az = 128;
        for (int l = 0; l < 4; ++l) {
            Tensor nh({M, H}, DType::UInt8);
            oracle_qlinear(M, H, H, h.data(), 1, as, az, ws[l].data_ptr<int8_t>(), 0, scs[l].data(),
                           bs[l].data_ptr<float>(), 1, 2, y_scales[l], 0, nullptr, nh.data(), nullptr);
            h = nh;
            as = y_scales[l];
            az = 0;
        }
        EXPECT(same_bytes(y[0], h), "4-layer MLP output differs from the reference arithmetic");
    });

    // SparseMatMul (pruned Linear): Y = X W^T, W [N,K] CSR int64.
    run_test("SparseMatMul", [&] {
        const int64_t M = 9, N = 300, K = 700;
        std::mt19937_64 rng(17);
        std::bernoulli_distribution keep(0.1);
        std::normal_distribution<float> nd(0.0f, 0.02f);
        std::vector<int64_t> ip(1, 0), ix;
        std::vector<float> vv;
        for (int64_t r = 0; r < N; ++r) {
            for (int64_t c = 0; c < K; ++c)
                if (keep(rng)) {
                    ix.push_back(c);
                    vv.push_back(nd(rng));
                }
            ip.push_back(static_cast<int64_t>(ix.size()));
        }
        Graph g("spmm");
        g.add_input(TensorInfo("X", sh({M, K}), DType::Float32));
        Tensor tip({N + 1}, DType::Int64), tix({static_cast<int64_t>(ix.size())}, DType::Int64),
            tv({static_cast<int64_t>(vv.size())}, DType::Float32);
        std::memcpy(tip.data(), ip.data(), 8 * ip.size());
        std::memcpy(tix.data(), ix.data(), 8 * ix.size());
        std::memcpy(tv.data(), vv.data(), 4 * vv.size());
        g.add_initializer("indptr", tip);
        g.add_initializer("indices", tix);
        g.add_initializer("values", tv);
        auto n = node("spmm", "SparseMatMul", {"X", "indptr", "indices", "values"}, {"Y"});
        n->set_attr("shape", std::vector<int64_t>{N, K});
        g.add_node(n);
        g.add_output(TensorInfo("Y", sh({M, N}), DType::Float32));
        Tensor x = randn({M, K}, 1.0f, 18);
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = x;
        auto y = run(cuda, g, feeds);
        std::vector<int32_t> ip32(ip.begin(), ip.end()), ix32(ix.begin(), ix.end());
        Tensor ref({M, N}, DType::Float32);
        oracle_spmm_linear(M, N, K, ip32.data(), ix32.data(), vv.data(), x.data_ptr<float>(), ref.data_ptr<float>());
        const double e = normwise(y[0], ref);
        EXPECT(e <= 1e-5, "normwise error " + std::to_string(e));
    });

    // The pruning -> CSR graph pass: compute_mask's criterion (checked against
    // the oracle's restatement, itself pinned to the reference), MatMul and
    // Gemm (transB, bias) rewritten to SparseMatMul, and the rewritten graph
    // on the GPU against CPUExecutor on the original graph with pruned weights.
    run_test("MagnitudeMaskCriterion", [&] {
        for (int kind = 0; kind < 3; ++kind) {
            const int64_t n = 97 * 131;
            Tensor w = kind == 0 ? randn({n}, 1.0f, 40) : randint<float>({n}, -3, 3, DType::Float32, 41);
            if (kind == 2) std::fill(w.data_ptr<float>(), w.data_ptr<float>() + n / 2, 0.0f);
            for (float s : {-0.1f, 0.0f, 0.3f, 0.9f, 0.95f, 0.999f, 1.0f}) {
                auto m = cuda::magnitude_mask(w.data_ptr<float>(), n, s);
                std::vector<float> ref(static_cast<size_t>(n));
                EXPECT(oracle_magnitude_mask(n, w.data_ptr<float>(), s, ref.data()) == 0, "oracle");
                EXPECT(std::memcmp(m.data(), ref.data(), 4 * n) == 0,
                       "mask differs (kind " + std::to_string(kind) + ", s " + std::to_string(s) + ")");
            }
        }
    });

    run_test("NMMaskMatchesReference", [&] {
        // The pass's N:M criterion against the reference's own
        // NMSparsityPruning::compute_mask (src/pruning/nm_sparsity.cpp), ties and NaN included.
        std::mt19937_64 rng(77);
        const float tie_vals[] = {0.0f, -0.0f, 1.0f, -1.0f, 2.0f, -2.0f, 0.5f};
        for (auto nm : std::vector<std::pair<int, int>>{{2, 4}, {1, 2}, {3, 4}, {4, 8}, {5, 16}, {16, 32}}) {
            for (int kind = 0; kind < 3; ++kind) {
                const int64_t total = 1000 + nm.second / 2;  // a short last group
                Tensor w({total}, DType::Float32);
                std::normal_distribution<float> nd(0.0f, 1.0f);
                for (int64_t i = 0; i < total; ++i) {
                    float v = kind == 0 ? tie_vals[rng() % 7] : nd(rng);
                    if (kind == 2 && rng() % 5 == 0) v = std::nanf("");
                    w.data_ptr<float>()[i] = v;
                }
                auto mine = cuda::nm_mask(w.data_ptr<float>(), total, nm.first, nm.second);
                pruning::NMSparsityPruning ref(static_cast<size_t>(nm.first), static_cast<size_t>(nm.second));
                auto rm = ref.compute_mask("w", w, 0.0f);
                EXPECT(std::memcmp(mine.data(), rm.mask.data(), 4 * total) == 0,
                       "N:M mask differs (" + std::to_string(nm.first) + ":" + std::to_string(nm.second) +
                           ", kind " + std::to_string(kind) + ")");
            }
        }
        bool threw = false;
        try {
            cuda::nm_mask(nullptr, 0, 5, 4);
        } catch (const std::invalid_argument& e) {
            threw = std::string(e.what()) == "N must be <= M in N:M sparsity";
        }
        EXPECT(threw, "n > m must throw the reference's message");
    });

    run_test("SparsifyNMPrunedMatMul", [&] {
        // 2:4 pruning of a MatMul weight [K, N] in its storage order, then SparseMatMul on
        // the GPU, against CPUExecutor on the original graph with the reference-masked weight.
        const int64_t M = 32, K = 512, N = 384;
        Graph g("nm");
        g.add_input(TensorInfo("X", sh({M, K}), DType::Float32));
        g.add_initializer("B", randn({K, N}, 0.05f, 60));
        g.add_node(node("mm", "MatMul", {"X", "B"}, {"Y"}));
        g.add_output(TensorInfo("Y", sh({M, N}), DType::Float32));
        cuda::SparsifyOptions opt;
        opt.nm_n = 2;
        opt.nm_m = 4;
        cuda::SparsifyReport rep;
        Graph sg = cuda::sparsify_matmuls(g, opt, &rep);
        EXPECT(rep.rewritten == 1, "one node rewritten, got " + std::to_string(rep.rewritten));
        const Tensor& B = g.get_initializer("B")->get();
        pruning::NMSparsityPruning ref(2, 4);
        auto rm = ref.compute_mask("B", B, 0.0f);
        Graph pg("nm_masked");
        pg.add_input(TensorInfo("X", sh({M, K}), DType::Float32));
        Tensor pb({K, N}, DType::Float32);
        for (int64_t i = 0; i < K * N; ++i) pb.data_ptr<float>()[i] = B.data_ptr<float>()[i] * rm.mask.data_ptr<float>()[i];
        pg.add_initializer("B", pb);
        pg.add_node(node("mm", "MatMul", {"X", "B"}, {"Y"}));
        pg.add_output(TensorInfo("Y", sh({M, N}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = randn({M, K}, 1.0f, 61);
        CPUExecutor cpu(0);
        auto r = cpu.execute(pg, feeds, {"Y"});
        CudaBackend gpu(0);
        auto y = gpu.execute(sg, feeds, {"Y"});
        const double e = normwise(y[0], r[0]);
        EXPECT(e <= 1e-5, "normwise error " + std::to_string(e));
    });

    run_test("SparsifyPrunedMatMulAndGemm", [&] {
        const int64_t M = 64, K = 1024, N = 768;
        Graph g("prunable");
        g.add_input(TensorInfo("X", sh({M, K}), DType::Float32));
        g.add_initializer("B1", randn({K, N}, 0.05f, 50));   // MatMul weight [K, N]
        g.add_initializer("B2", randn({N, K}, 0.05f, 51));   // Gemm weight, transB = 1
        g.add_initializer("C2", randn({N}, 0.1f, 52));
        g.add_node(node("mm", "MatMul", {"X", "B1"}, {"Y1"}));
        auto gm = node("gemm", "Gemm", {"X", "B2", "C2"}, {"Y2"});
        gm->set_attr("transB", static_cast<int64_t>(1));
        gm->set_attr("alpha", 1.0f);
        gm->set_attr("beta", 1.0f);
        g.add_node(gm);
        g.add_output(TensorInfo("Y1", sh({M, N}), DType::Float32));
        g.add_output(TensorInfo("Y2", sh({M, N}), DType::Float32));
        cuda::SparsifyOptions opt;
        opt.prune_sparsity = 0.9f;
        cuda::SparsifyReport rep;
        Graph sg = cuda::sparsify_matmuls(g, opt, &rep);
        EXPECT(rep.rewritten == 2, "two nodes rewritten, got " + std::to_string(rep.rewritten));
        EXPECT(!sg.has_initializer("B1") && !sg.has_initializer("B2") && sg.has_initializer("C2"),
               "dense weights dropped, bias kept");
        // The CSR of the MatMul weight equals to_sparse((B1 * mask)^T) with the oracle's mask.
        const Tensor& B1 = g.get_initializer("B1")->get();
        std::vector<float> m1(static_cast<size_t>(K * N));
        oracle_magnitude_mask(K * N, B1.data_ptr<float>(), 0.9f, m1.data());
        std::vector<int32_t> ip(1, 0), ix;
        std::vector<float> vv;
        for (int64_t n = 0; n < N; ++n) {
            for (int64_t k = 0; k < K; ++k) {
                const float d = B1.data_ptr<float>()[k * N + n] * m1[k * N + n];
                if (std::fabs(d) > 0.0f) {
                    ix.push_back(static_cast<int32_t>(k));
                    vv.push_back(d);
                }
            }
            ip.push_back(static_cast<int32_t>(ix.size()));
        }
        const Tensor& sip = sg.get_initializer("mm_csr_indptr")->get();
        const Tensor& six = sg.get_initializer("mm_csr_indices")->get();
        const Tensor& sv = sg.get_initializer("mm_csr_values")->get();
        EXPECT(sip.num_elements() == N + 1 && six.num_elements() == static_cast<int64_t>(ix.size()), "CSR sizes");
        EXPECT(std::memcmp(sip.data(), ip.data(), 4 * ip.size()) == 0 &&
                   std::memcmp(six.data(), ix.data(), 4 * ix.size()) == 0 &&
                   std::memcmp(sv.data(), vv.data(), 4 * vv.size()) == 0,
               "CSR of the pruned MatMul weight differs from to_sparse(W * mask)");
        // GPU on the rewritten graph vs CPUExecutor on the original graph with masked weights.
        Graph pg("pruned");
        pg.add_input(TensorInfo("X", sh({M, K}), DType::Float32));
        Tensor pb1({K, N}, DType::Float32), pb2({N, K}, DType::Float32);
        const Tensor& B2 = g.get_initializer("B2")->get();
        std::vector<float> m2(static_cast<size_t>(K * N));
        oracle_magnitude_mask(K * N, B2.data_ptr<float>(), 0.9f, m2.data());
        for (int64_t i = 0; i < K * N; ++i) {
            pb1.data_ptr<float>()[i] = B1.data_ptr<float>()[i] * m1[i];
            pb2.data_ptr<float>()[i] = B2.data_ptr<float>()[i] * m2[i];
        }
        pg.add_initializer("B1", pb1);
        pg.add_initializer("B2", pb2);
        pg.add_initializer("C2", g.get_initializer("C2")->get());
        pg.add_node(node("mm", "MatMul", {"X", "B1"}, {"Y1"}));
        pg.add_node(gm);
        pg.add_output(TensorInfo("Y1", sh({M, N}), DType::Float32));
        pg.add_output(TensorInfo("Y2", sh({M, N}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = randn({M, K}, 1.0f, 53);
        auto y = run(cuda, sg, feeds);
        auto r = run(cpu, pg, feeds);
        for (int i = 0; i < 2; ++i) {
            const double e = normwise(y[i], r[i]);
            EXPECT(e <= 1e-5, "output " + std::to_string(i) + " normwise error " + std::to_string(e));
        }
    });

    // Quantizer output -> per-channel QuantizedMatMul: the weight scales and
    // int8 weight equal the reference's compute_dynamic_params_per_channel +
    // quantize_tensor, the activation parameters its compute_from_minmax, and
    // the rewritten graph on the GPU is bit-exact to the int8 oracle.
    run_test("QuantizePassPerChannel", [&] {
        namespace q = quantization;
        const int64_t M = 96, K = 512, N = 384;
        Graph g("fp32_layer");
        g.add_input(TensorInfo("X", sh({M, K}), DType::Float32));
        g.add_initializer("W", randn({K, N}, 0.05f, 60));
        g.add_initializer("bias", randn({N}, 0.1f, 61));
        g.add_node(node("mm", "MatMul", {"X", "W"}, {"t"}));
        g.add_node(node("add", "Add", {"t", "bias"}, {"u"}));
        g.add_node(node("relu", "Relu", {"u"}, {"Y"}));
        g.add_output(TensorInfo("Y", sh({M, N}), DType::Float32));
        Tensor x = randn({M, K}, 1.0f, 62);
        const float* xp = x.data_ptr<float>();
        const float xmin = *std::min_element(xp, xp + M * K), xmax = *std::max_element(xp, xp + M * K);
        cuda::QuantizePassOptions opt;
        opt.act_ranges["X"] = {xmin, xmax};
        cuda::QuantizePassReport rep;
        Graph qg = cuda::quantize_matmuls_per_channel(g, opt, &rep);
        EXPECT(rep.rewritten == 1, "one MatMul rewritten");
        const Node* qm = qg.get_node("mm");
        EXPECT(qm && qm->op_type() == "QuantizedMatMul", "mm is a QuantizedMatMul");
        // reference parameters
        const Tensor& W = g.get_initializer("W")->get();
        auto wp = q::compute_dynamic_params_per_channel(W, 1, DType::Int8, true);
        Tensor wq = q::quantize_tensor(W, wp);  // per-channel over axis 1
        const auto scales = qm->get_attr<std::vector<float>>("b_scales", {});
        EXPECT(scales.size() == static_cast<size_t>(N) &&
                   std::memcmp(scales.data(), wp.scales.data(), 4 * N) == 0,
               "b_scales differ from compute_dynamic_params_per_channel");
        const Tensor& Wq = qg.get_initializer("W_q8")->get();
        EXPECT(same_bytes(Wq, wq), "int8 weight differs from quantize_tensor");
        auto ap = q::QuantParams::compute_from_minmax(xmin, xmax, DType::UInt8, false);
        EXPECT(qm->get_attr<float>("a_scale", 0.0f) == ap.scales[0] &&
                   qm->get_attr<int64_t>("a_zero_point", -1) == ap.zero_points[0],
               "activation parameters differ from compute_from_minmax");
        // GPU run vs the oracle on the reference-quantized activations
        std::unordered_map<std::string, Tensor> feeds;
        feeds["X"] = x;
        auto y = run(cuda, qg, feeds);
        Tensor xq = q::quantize_tensor(x, ap);
        std::vector<float> ref(static_cast<size_t>(M * N));
        oracle_qlinear(M, N, K, xq.data(), 1, ap.scales[0], ap.zero_points[0], Wq.data_ptr<int8_t>(), 0,
                       scales.data(), g.get_initializer("bias")->get().data_ptr<float>(), 1, 0, 1.0f, 0,
                       ref.data(), nullptr, nullptr);
        EXPECT(std::memcmp(y[0].data(), ref.data(), 4 * M * N) == 0, "quantized layer not bit-exact to the oracle");
        // and close to the fp32 layer it replaces
        auto f = run(cpu, g, feeds);
        const double e = normwise(y[0], f[0]);
        EXPECT(e < 0.02, "int8 layer far from fp32: normwise " + std::to_string(e));
    });

    // Error behaviour mirrors CPUExecutor (executor.cpp:80-110, 150-212).
    run_test("UnsupportedOperator", [&] {
        Graph g("bad");
        g.add_input(TensorInfo("x", sh({2, 2}), DType::Float32));
        g.add_node(node("sm", "Softmax", {"x"}, {"y"}));
        g.add_output(TensorInfo("y", sh({2, 2}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["x"] = randn({2, 2}, 1.0f, 19);
        bool thrown = false;
        try {
            cuda.execute(g, feeds);
        } catch (const UnsupportedOperatorError& e) {
            thrown = std::string(e.what()).find("'cuda'") != std::string::npos;
        }
        EXPECT(thrown, "UnsupportedOperatorError naming the cuda backend expected");
    });

    run_test("MissingInput", [&] {
        Graph g("missing");
        g.add_input(TensorInfo("a", sh({2, 3}), DType::Float32));
        g.add_input(TensorInfo("b", sh({3, 2}), DType::Float32));
        g.add_node(node("mm", "MatMul", {"a", "b"}, {"c"}));
        g.add_output(TensorInfo("c", sh({2, 2}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["a"] = randn({2, 3}, 1.0f, 20);
        bool thrown = false;
        try {
            cuda.execute(g, feeds);
        } catch (const InputError&) {
            thrown = true;
        }
        EXPECT(thrown, "InputError expected for a missing input");
    });

    run_test("ShapeErrorNamesNode", [&] {
        Graph g("k");
        g.add_input(TensorInfo("A", sh({4, 5}), DType::Float32));
        g.add_initializer("B", randn({6, 3}, 1.0f, 21));
        g.add_node(node("gemm_bad", "Gemm", {"A", "B"}, {"Y"}));
        g.add_output(TensorInfo("Y", sh({4, 3}), DType::Float32));
        std::unordered_map<std::string, Tensor> feeds;
        feeds["A"] = randn({4, 5}, 1.0f, 22);
        bool ok = false;
        try {
            cuda.execute(g, feeds);
        } catch (const BackendError& e) {
            ok = e.node_name().has_value() && *e.node_name() == "gemm_bad" &&
                 std::string(e.what()).find("incompatible dimensions") != std::string::npos;
        }
        EXPECT(ok, "BackendError naming the node expected");
    });

    std::printf("%s: %d failed\n", g_failed ? "FAILED" : "OK", g_failed);
    return g_failed ? 1 : 0;
}
