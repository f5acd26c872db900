// test_batcher.cpp -- the batching caller (cuda::DynamicBatcher,
// pyflamert_b200/backend/batcher.{hpp,cpp}).  Every batched response is
// checked against the same request run alone, byte for byte.  TEST
// INFRASTRUCTURE.
//
//   test_batcher --cpu   host logic on the reference's CPUExecutor as the
//                        backend(s): futures from several client threads,
//                        callbacks, multi-row requests, padding, output
//                        selection, queue capacity, a malformed request among
//                        good ones, two workers, draining on stop.  No GPU.
//   test_batcher         (B200) the same checks on CudaBackend, and the
//                        throughput of config 2's layer for single-row requests:
//                        one at a time vs batched (one and two workers).
// Prints one "PASS name" / "FAIL name: why" line per test.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <functional>
#include <memory>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "backends/cpu/executor.hpp"
#include "batcher.hpp"
#include "cuda_backend.hpp"
#include "pyflame_rt/errors.hpp"
#include "pyflame_rt/graph.hpp"

using namespace pyflame_rt;
using cuda::DynamicBatcher;

namespace {

int g_failed = 0;

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

#define EXPECT(cond, msg)                \
    do {                                 \
        if (!(cond)) throw Failure(msg); \
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
    for (auto v : d) s.push_back(v < 0 ? std::optional<int64_t>() : std::optional<int64_t>(v));
    return s;
}

Tensor rnd(std::vector<int64_t> shape, DType dt, uint64_t seed) {
    Tensor t(shape, dt);
    std::mt19937_64 rng(seed);
    if (dt == DType::Float32) {
        std::normal_distribution<float> nd(0.0f, 1.0f);
        for (int64_t i = 0; i < t.num_elements(); ++i) t.data_ptr<float>()[i] = nd(rng);
    } else {
        auto* p = static_cast<uint8_t*>(t.data());
        for (size_t i = 0; i < t.size_bytes(); ++i) p[i] = static_cast<uint8_t>(rng());
    }
    return t;
}

// Two outputs: an fp32 Gemm with bias and an int8 QuantizedMatMul (signed
// activations, which the reference graph op reads correctly).
std::shared_ptr<Graph> small_graph() {
    auto g = std::make_shared<Graph>("batch_small");
    g->add_input(TensorInfo("X", sh({-1, 64}), DType::Float32));
    g->add_input(TensorInfo("Xq", sh({-1, 48}), DType::Int8));
    g->add_initializer("W", rnd({64, 32}, DType::Float32, 1));
    g->add_initializer("C", rnd({32}, DType::Float32, 2));
    g->add_initializer("Wq", rnd({48, 16}, DType::Int8, 3));
    auto gemm = std::make_shared<Node>("gemm", "Gemm", std::vector<std::string>{"X", "W", "C"},
                                       std::vector<std::string>{"Y"});
    g->add_node(gemm);
    auto q = std::make_shared<Node>("qmm", "QuantizedMatMul", std::vector<std::string>{"Xq", "Wq"},
                                    std::vector<std::string>{"Yq"});
    q->set_attr("a_scale", 0.02f);
    q->set_attr("b_scale", 0.0125f);
    g->add_node(q);
    g->add_output(TensorInfo("Y", sh({-1, 32}), DType::Float32));
    g->add_output(TensorInfo("Yq", sh({-1, 16}), DType::Float32));
    return g;
}

batching::InferenceRequest request(int64_t rows, uint64_t seed) {
    batching::InferenceRequest r;
    r.inputs["X"] = rnd({rows, 64}, DType::Float32, seed);
    r.inputs["Xq"] = rnd({rows, 48}, DType::Int8, seed + 1);
    return r;
}

// Byte-identical, except fp32 results of the CUDA Gemm when `fp32_tol`: its
// summation order may depend on the batch's row count (split-K), so those
// are held to the fp32 parity bound, normwise <= 1e-5.
bool g_fp32_tol = false;
void same(const Tensor& a, const Tensor& b, const std::string& what) {
    EXPECT(a.shape() == b.shape() && a.dtype() == b.dtype(), what + ": shape/dtype");
    if (g_fp32_tol && a.dtype() == DType::Float32) {
        double num = 0, den = 0;
        for (int64_t i = 0; i < a.num_elements(); ++i) {
            num = std::max(num, std::fabs(double(a.data_ptr<float>()[i]) - b.data_ptr<float>()[i]));
            den = std::max(den, std::fabs(double(b.data_ptr<float>()[i])));
        }
        EXPECT(num <= 1e-5 * den, what + ": normwise error " + std::to_string(den > 0 ? num / den : num));
        return;
    }
    EXPECT(a.size_bytes() == 0 || std::memcmp(a.data(), b.data(), a.size_bytes()) == 0, what + ": bytes differ");
}

using BackendFactory = std::function<std::shared_ptr<Backend>()>;

// Request run alone on a fresh backend of the same kind.
struct Alone {
    std::shared_ptr<Backend> be;
    std::shared_ptr<Graph> g;
    std::vector<Tensor> run(const batching::InferenceRequest& r, const std::vector<std::string>& names) {
        return be->execute(*g, r.inputs, names);
    }
};

void host_logic_tests(const BackendFactory& make, const char* tag) {
    auto g = small_graph();
    Alone alone{make(), g};
    const std::vector<std::string> both = {"Y", "Yq"};
    auto check = [&](const batching::InferenceRequest& req, const batching::InferenceResponse& r,
                     const std::vector<std::string>& names) {
        EXPECT(r.success, "request failed: " + r.error_message);
        const auto ref = alone.run(req, names);
        EXPECT(r.outputs.size() == names.size(), "output count");
        for (size_t i = 0; i < names.size(); ++i) same(r.outputs.at(names[i]), ref[i], names[i]);
    };
    std::string t = std::string("BatcherFuturesManyClients_") + tag;
    run_test(t.c_str(), [&] {
        batching::BatchConfig cfg;
        cfg.max_batch_size = 16;
        cfg.enable_padding = false;
        DynamicBatcher b(g, {make()}, cfg);
        b.start();
        std::vector<std::vector<std::pair<batching::InferenceRequest, std::future<batching::InferenceResponse>>>> per(4);
        std::vector<std::thread> clients;
        for (int c = 0; c < 4; ++c)
            clients.emplace_back([&, c] {
                for (int i = 0; i < 50; ++i) {
                    auto req = request(1 + (i + c) % 4, 1000 * c + 7 * i);
                    auto copy = req;
                    per[c].emplace_back(std::move(copy), b.submit(std::move(req)));
                }
            });
        for (auto& th : clients) th.join();
        for (auto& v : per)
            for (auto& [req, f] : v) check(req, f.get(), both);
        const auto s = b.get_stats();
        EXPECT(s.total_requests == 200, "stats.total_requests = " + std::to_string(s.total_requests));
        std::printf("  200 requests in %llu batches (avg %.1f requests)\n",
                    static_cast<unsigned long long>(s.total_batches), s.avg_batch_size);
        b.stop();
    });
    t = std::string("BatcherCallbacksAndOutputSelection_") + tag;
    run_test(t.c_str(), [&] {
        DynamicBatcher b(g, {make()});
        std::mutex m;
        std::condition_variable cv;
        std::vector<std::pair<uint64_t, batching::InferenceResponse>> got;
        std::vector<batching::InferenceRequest> reqs;
        for (int i = 0; i < 40; ++i) {
            auto req = request(2, 5000 + i);
            req.output_names = {"Yq"};
            reqs.push_back(req);
        }
        std::vector<uint64_t> ids;
        for (auto& req : reqs) {
            auto copy = req;
            ids.push_back(b.submit(std::move(copy), [&](batching::InferenceResponse r) {
                std::lock_guard<std::mutex> l(m);
                got.emplace_back(r.request_id, std::move(r));
                cv.notify_all();
            }));
        }
        b.start();
        std::unique_lock<std::mutex> l(m);
        EXPECT(cv.wait_for(l, std::chrono::seconds(60), [&] { return got.size() == reqs.size(); }), "callbacks missing");
        for (auto& [id, r] : got) {
            const size_t i = static_cast<size_t>(std::find(ids.begin(), ids.end(), id) - ids.begin());
            EXPECT(i < reqs.size(), "unknown request id");
            EXPECT(!r.outputs.count("Y"), "output Y was not asked for");
            check(reqs[i], r, {"Yq"});
        }
        l.unlock();
        b.stop();
    });
    t = std::string("BatcherPaddingRows_") + tag;
    run_test(t.c_str(), [&] {
        batching::BatchConfig cfg;
        cfg.max_batch_size = 8;
        cfg.min_batch_size = 8;
        cfg.max_latency = std::chrono::microseconds(200000);
        cfg.preferred_sizes = {16, 64};
        cfg.enable_padding = true;
        DynamicBatcher b(g, {make()}, cfg);
        std::vector<std::pair<batching::InferenceRequest, std::future<batching::InferenceResponse>>> fs;
        for (int i = 0; i < 24; ++i) {
            auto req = request(1 + i % 3, 9000 + i);
            auto copy = req;
            fs.emplace_back(std::move(copy), b.submit(std::move(req)));
        }
        b.start();
        for (auto& [req, f] : fs) check(req, f.get(), both);
        b.stop();
    });
    t = std::string("BatcherQueueFullAndDrain_") + tag;
    run_test(t.c_str(), [&] {
        batching::BatchConfig cfg;
        cfg.queue_capacity = 5;
        DynamicBatcher b(g, {make()}, cfg);
        std::vector<std::pair<batching::InferenceRequest, std::future<batching::InferenceResponse>>> fs;
        for (int i = 0; i < 6; ++i) {
            auto req = request(1, 300 + i);
            auto copy = req;
            fs.emplace_back(std::move(copy), b.submit(std::move(req)));
        }
        auto last = fs.back().second.get();
        EXPECT(!last.success && last.error_message == "Queue full", "sixth request: " + last.error_message);
        EXPECT(b.get_stats().dropped_requests == 1, "dropped count");
        EXPECT(b.queue_size() == 5, "queue size");
        b.start();
        b.stop();  // the five queued requests are answered before stop returns
        for (int i = 0; i < 5; ++i) check(fs[i].first, fs[i].second.get(), both);
    });
    t = std::string("BatcherMalformedRequestFailsAlone_") + tag;
    run_test(t.c_str(), [&] {
        batching::BatchConfig cfg;
        cfg.min_batch_size = 6;
        cfg.max_latency = std::chrono::microseconds(200000);
        DynamicBatcher b(g, {make()}, cfg);
        std::vector<std::pair<batching::InferenceRequest, std::future<batching::InferenceResponse>>> fs;
        for (int i = 0; i < 6; ++i) {
            auto req = request(2, 700 + i);
            if (i == 3) req.inputs["X"] = rnd({2, 63}, DType::Float32, 1);  // wrong row length
            if (i == 4) req.inputs.erase("Xq");
            auto copy = req;
            fs.emplace_back(std::move(copy), b.submit(std::move(req)));
        }
        b.start();
        for (int i = 0; i < 6; ++i) {
            auto r = fs[i].second.get();
            if (i == 3 || i == 4) {
                EXPECT(!r.success && r.error_message.find("DynamicBatcher: request") == 0,
                       "malformed request: " + r.error_message);
            } else {
                check(fs[i].first, r, both);
            }
        }
        b.stop();
    });
    t = std::string("BatcherTwoWorkers_") + tag;
    run_test(t.c_str(), [&] {
        batching::BatchConfig cfg;
        cfg.max_batch_size = 8;
        DynamicBatcher b(g, {make(), make()}, cfg);
        b.start();
        std::vector<std::pair<batching::InferenceRequest, std::future<batching::InferenceResponse>>> fs;
        for (int i = 0; i < 100; ++i) {
            auto req = request(1 + i % 2, 20000 + i);
            auto copy = req;
            fs.emplace_back(std::move(copy), b.submit(std::move(req)));
        }
        for (auto& [req, f] : fs) check(req, f.get(), both);
        b.stop();
    });
}

// ----------------------------------------------------------------- GPU throughput
// Config 2's layer: u8[., 4096] x s8[4096, 4096] (per-channel scales) -> s8.
std::shared_ptr<Graph> layer_graph() {
    auto g = std::make_shared<Graph>("config2_layer");
    g->add_input(TensorInfo("A", sh({-1, 4096}), DType::UInt8));
    g->add_initializer("W", rnd({4096, 4096}, DType::Int8, 41));
    auto q = std::make_shared<Node>("qmm", "QuantizedMatMul", std::vector<std::string>{"A", "W"},
                                    std::vector<std::string>{"acc"});
    std::vector<float> scales(4096);
    std::mt19937_64 rng(42);
    std::uniform_real_distribution<float> us(0.005f, 0.02f);
    for (auto& s : scales) s = us(rng);
    q->set_attr("a_scale", 0.02f);
    q->set_attr("a_zero_point", int64_t{128});
    q->set_attr("b_scales", scales);
    g->add_node(q);
    auto qz = std::make_shared<Node>("quant", "Quantize", std::vector<std::string>{"acc"}, std::vector<std::string>{"Y"});
    qz->set_attr("scale", 0.05f);
    qz->set_attr("dtype", std::string("int8"));
    g->add_node(qz);
    g->add_output(TensorInfo("Y", sh({-1, 4096}), DType::Int8));
    return g;
}

void gpu_throughput() {
    auto g = layer_graph();
    const int n = 2048;
    std::vector<batching::InferenceRequest> reqs;
    for (int i = 0; i < n; ++i) {
        batching::InferenceRequest r;
        r.inputs["A"] = rnd({1, 4096}, DType::UInt8, 100000 + i);
        reqs.push_back(std::move(r));
    }
    std::vector<Tensor> alone(n);
    double alone_rps = 0;
    run_test("BatcherGpuOneAtATime", [&] {
        CudaBackend be(0);
        be.execute(*g, reqs[0].inputs, {"Y"});  // weights prepared, kernels loaded
        const auto t = std::chrono::steady_clock::now();
        for (int i = 0; i < n; ++i) alone[i] = be.execute(*g, reqs[i].inputs, {"Y"})[0];
        alone_rps = n / std::chrono::duration<double>(std::chrono::steady_clock::now() - t).count();
    });
    auto batched = [&](int workers, double& rps) {
        batching::BatchConfig cfg;
        cfg.max_batch_size = 256;
        cfg.min_batch_size = 256;
        cfg.max_latency = std::chrono::microseconds(500);
        cfg.enable_padding = false;
        cfg.queue_capacity = 0;
        std::vector<std::shared_ptr<Backend>> bes;
        for (int w = 0; w < workers; ++w) bes.push_back(std::make_shared<CudaBackend>(0));
        DynamicBatcher b(g, bes, cfg);
        b.start();
        {
            // warm-up: weights prepared on every backend
            std::vector<std::future<batching::InferenceResponse>> fs;
            for (int i = 0; i < 256 * workers; ++i) fs.push_back(b.submit(reqs[i % n]));
            for (auto& f : fs) f.get();
        }
        b.reset_stats();
        std::vector<std::future<batching::InferenceResponse>> fs(n);
        const auto t = std::chrono::steady_clock::now();
        std::vector<std::thread> clients;
        for (int c = 0; c < 8; ++c)
            clients.emplace_back([&, c] {
                for (int i = c; i < n; i += 8) fs[i] = b.submit(reqs[i]);
            });
        for (auto& th : clients) th.join();
        std::vector<batching::InferenceResponse> rs(n);
        for (int i = 0; i < n; ++i) rs[i] = fs[i].get();
        rps = n / std::chrono::duration<double>(std::chrono::steady_clock::now() - t).count();
        const auto s = b.get_stats();
        std::printf("  %d worker(s): %llu batches, avg %.1f requests\n", workers,
                    static_cast<unsigned long long>(s.total_batches), s.avg_batch_size);
        b.stop();
        for (int i = 0; i < n; ++i) {
            EXPECT(rs[i].success, rs[i].error_message);
            same(rs[i].outputs.at("Y"), alone[i], "request " + std::to_string(i));
        }
    };
    double rps1 = 0, rps2 = 0;
    run_test("BatcherGpuBatchedOneWorker", [&] { batched(1, rps1); });
    run_test("BatcherGpuBatchedTwoWorkers", [&] { batched(2, rps2); });
    std::printf("  config 2 layer, %d single-row requests: one at a time %.0f req/s, batched %.0f req/s (1 worker), "
                "%.0f req/s (2 workers)\n",
                n, alone_rps, rps1, rps2);
    std::printf("BATCH_TIMING {\"requests\": %d, \"alone_rps\": %.1f, \"batched_rps\": %.1f, \"batched2_rps\": %.1f}\n",
                n, alone_rps, rps1, rps2);
}

}  // namespace

int main(int argc, char** argv) {
    const bool cpu_only = argc > 1 && std::strcmp(argv[1], "--cpu") == 0;
    host_logic_tests([] { return std::make_shared<CPUExecutor>(0); }, "cpu");
    if (!cpu_only) {
        g_fp32_tol = true;
        host_logic_tests([] { return std::make_shared<CudaBackend>(0); }, "cuda");
        g_fp32_tol = false;
        gpu_throughput();
    }
    std::printf("%s: %d failed\n", g_failed ? "FAILED" : "OK", g_failed);
    return g_failed ? 1 : 0;
}
