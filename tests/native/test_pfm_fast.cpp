// test_pfm_fast.cpp -- the .pfm fast path (PfmImage + CudaBackend::prepare)
// against the reference's own loader, PyFlameFormat::load
// (src/io/pyflame_format.cpp, compiled from the reference's sources into this
// test).  TEST INFRASTRUCTURE.
//
//   test_pfm_fast --cpu   parse parity: the same Graph (inputs, outputs, nodes,
//                         attributes, initializer bytes) from both loaders, and
//                         the same InvalidModelError text for every truncation
//                         of a model file and for targeted corruptions.  No GPU.
//   test_pfm_fast         (B200) a model loaded through PfmImage and prepared by
//                         CudaBackend::prepare gives bit-identical outputs to the
//                         same model loaded by PyFlameFormat::load and prepared
//                         lazily by execute(); prints the load + prepare time of
//                         both paths for a config-4-sized model.
// Prints one "PASS name" / "FAIL name: why" line per test.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <memory>
#include <random>
#include <string>
#include <unistd.h>
#include <vector>

#include "cuda_backend.hpp"
#include "io/pyflame_format.hpp"
#include "pfm_image.hpp"
#include "pyflame_rt/errors.hpp"
#include "pyflame_rt/graph.hpp"

using namespace pyflame_rt;

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

Tensor rand_tensor(std::vector<int64_t> shape, DType dt, uint64_t seed) {
    Tensor t(shape, dt);
    std::mt19937_64 rng(seed);
    auto* p = static_cast<uint8_t*>(t.data());
    if (dt == DType::Float32) {
        std::normal_distribution<float> nd(0.0f, 1.0f);
        for (int64_t i = 0; i < t.num_elements(); ++i) t.data_ptr<float>()[i] = nd(rng) * 0.05f;
    } else {
        for (size_t i = 0; i < t.size_bytes(); ++i) p[i] = static_cast<uint8_t>(rng());
    }
    return t;
}

std::string tmp_path(const char* tag) {
    char tmpl[64];
    std::snprintf(tmpl, sizeof(tmpl), "/tmp/pfrt_%s_XXXXXX", tag);
    const int fd = mkstemp(tmpl);
    if (fd < 0) throw Failure("mkstemp");
    close(fd);
    return tmpl;
}

std::vector<char> read_file(const std::string& p) {
    std::ifstream f(p, std::ios::binary);
    return std::vector<char>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

void write_file(const std::string& p, const char* data, size_t n) {
    std::ofstream f(p, std::ios::binary | std::ios::trunc);
    f.write(data, static_cast<std::streamsize>(n));
}

// A small graph with every attribute type, several dtypes, dynamic dims and
// an empty initializer.
Graph small_graph() {
    Graph g("pfm_parity");
    g.add_input(TensorInfo("X", sh({-1, 64}), DType::Float32));
    g.add_input(TensorInfo("Xq", sh({8, 32}), DType::UInt8));
    g.add_output(TensorInfo("Y", sh({-1, 48}), DType::Float32));
    g.add_initializer("W", rand_tensor({64, 48}, DType::Float32, 1));
    g.add_initializer("Wq", rand_tensor({32, 16}, DType::Int8, 2));
    g.add_initializer("bias", rand_tensor({48}, DType::Float32, 3));
    g.add_initializer("ip", rand_tensor({5}, DType::Int64, 4));
    g.add_initializer("empty", Tensor({0, 7}, DType::Float32));
    auto n1 = std::make_shared<Node>("mm", "MatMul", std::vector<std::string>{"X", "W"}, std::vector<std::string>{"t"});
    n1->set_attr("i", int64_t{-7});
    n1->set_attr("f", 0.25f);
    n1->set_attr("s", std::string("hello"));
    n1->set_attr("iv", std::vector<int64_t>{1, -2, 3});
    n1->set_attr("fv", std::vector<float>{0.5f, -1.5f});
    g.add_node(n1);
    g.add_node(std::make_shared<Node>("add", "Add", std::vector<std::string>{"t", "bias"},
                                      std::vector<std::string>{"Y"}));
    return g;
}

void same_graph(const Graph& a, const Graph& b) {
    EXPECT(a.name() == b.name(), "graph name");
    EXPECT(a.inputs().size() == b.inputs().size() && a.outputs().size() == b.outputs().size(), "io counts");
    for (size_t i = 0; i < a.inputs().size(); ++i)
        EXPECT(a.inputs()[i].name == b.inputs()[i].name && a.inputs()[i].dtype == b.inputs()[i].dtype &&
                   a.inputs()[i].shape == b.inputs()[i].shape,
               "input " + a.inputs()[i].name);
    for (size_t i = 0; i < a.outputs().size(); ++i)
        EXPECT(a.outputs()[i].name == b.outputs()[i].name && a.outputs()[i].shape == b.outputs()[i].shape,
               "output " + a.outputs()[i].name);
    EXPECT(a.initializers().size() == b.initializers().size(), "initializer count");
    for (const auto& [name, t] : a.initializers()) {
        auto it = b.initializers().find(name);
        EXPECT(it != b.initializers().end(), "initializer " + name);
        EXPECT(t.shape() == it->second.shape() && t.dtype() == it->second.dtype(), "initializer meta " + name);
        EXPECT(t.size_bytes() == it->second.size_bytes() &&
                   (t.size_bytes() == 0 || std::memcmp(t.data(), it->second.data(), t.size_bytes()) == 0),
               "initializer bytes " + name);
    }
    EXPECT(a.num_nodes() == b.num_nodes(), "node count");
    for (size_t i = 0; i < a.num_nodes(); ++i) {
        const Node& x = *a.nodes()[i];
        const Node& y = *b.nodes()[i];
        EXPECT(x.name() == y.name() && x.op_type() == y.op_type() && x.inputs() == y.inputs() &&
                   x.outputs() == y.outputs(),
               "node " + x.name());
        EXPECT(x.attributes() == y.attributes(), "attributes of " + x.name());
    }
}

// The error text each loader gives for the file at p ("" if it loads).
std::string ref_error(const std::string& p) {
    try {
        PyFlameFormat::load(p);
    } catch (const std::exception& e) {
        return e.what();
    }
    return "";
}
std::string fast_error(const std::string& p) {
    try {
        cuda::PfmImage::open(p);
    } catch (const std::exception& e) {
        return e.what();
    }
    return "";
}

void cpu_tests() {
    run_test("PfmParseParity", [] {
        const std::string p = tmp_path("parity");
        Graph g = small_graph();
        PyFlameFormat::save(g, p);
        auto ref = PyFlameFormat::load(p);
        auto img = cuda::PfmImage::open(p);
        same_graph(*ref, img->graph());
        for (const auto& [name, t] : img->graph().initializers())
            EXPECT(!t.owns_data(), "initializer " + name + " should view the mapping");
        std::remove(p.c_str());
    });
    run_test("PfmTruncationErrorsMatch", [] {
        const std::string p = tmp_path("trunc");
        PyFlameFormat::save(small_graph(), p);
        const std::vector<char> full = read_file(p);
        const std::string q = tmp_path("trunc_cut");
        int checked = 0;
        for (size_t cut = 0; cut < full.size(); ++cut) {
            write_file(q, full.data(), cut);
            const std::string r = ref_error(q), f = fast_error(q);
            EXPECT(!r.empty(), "reference loaded a truncated file at " + std::to_string(cut));
            EXPECT(r == f, "at " + std::to_string(cut) + ": reference '" + r + "' vs '" + f + "'");
            ++checked;
        }
        std::printf("  %d truncations, identical errors\n", checked);
        std::remove(p.c_str());
        std::remove(q.c_str());
    });
    run_test("PfmCorruptionErrorsMatch", [] {
        const std::string p = tmp_path("corrupt");
        PyFlameFormat::save(small_graph(), p);
        const std::vector<char> full = read_file(p);
        const std::string q = tmp_path("corrupt_x");
        // Offsets of fields in the small graph's file, found by content.
        auto find = [&](const std::string& s) {
            auto it = std::search(full.begin(), full.end(), s.begin(), s.end());
            if (it == full.end()) throw Failure("field not found: " + s);
            return static_cast<size_t>(it - full.begin());
        };
        struct Case {
            const char* what;
            size_t off;
            std::vector<uint8_t> bytes;
        };
        auto le64 = [](uint64_t v) {
            std::vector<uint8_t> b(8);
            std::memcpy(b.data(), &v, 8);
            return b;
        };
        auto le32 = [](uint32_t v) {
            std::vector<uint8_t> b(4);
            std::memcpy(b.data(), &v, 4);
            return b;
        };
        const size_t w_name = find(std::string("\x01\0\0\0\0\0\0\0W", 9));  // u64 length 1, "W"
        const size_t w_dtype = w_name + 9;
        const size_t w_ndim = w_dtype + 4;
        const size_t w_dim0 = w_ndim + 8;
        const size_t w_bytes = w_dim0 + 16;
        const size_t attr_s = find(std::string("\x01\0\0\0\0\0\0\0s", 9)) + 9;  // type tag of attribute "s"
        std::vector<Case> cases = {
            {"magic", 0, {'P', 'F', 'X', 0}},
            {"version", 4, le32(2)},
            {"graph name length", 8, le64(11ull * 1024 * 1024)},
            {"dtype", w_dtype, le32(99)},
            {"ndim", w_ndim, le64(17)},
            {"negative dim", w_dim0, le64(static_cast<uint64_t>(-3))},
            {"huge dim", w_dim0, le64(100000001)},
            {"byte count", w_bytes, le64(12)},
            {"byte count over limit", w_bytes, le64((4ull << 30) + 1)},
            {"attribute type", attr_s, le32(7)},
            {"attribute type 255", attr_s, le32(255)},
        };
        for (const auto& c : cases) {
            std::vector<char> bad = full;
            std::memcpy(bad.data() + c.off, c.bytes.data(), c.bytes.size());
            write_file(q, bad.data(), bad.size());
            const std::string r = ref_error(q), f = fast_error(q);
            EXPECT(r == f, std::string(c.what) + ": reference '" + r + "' vs '" + f + "'");
            std::printf("  %-22s %s\n", c.what, r.empty() ? "(loads)" : r.c_str());
        }
        EXPECT(ref_error("/nonexistent/x.pfm") == fast_error("/nonexistent/x.pfm"), "missing file");
        std::remove(p.c_str());
        std::remove(q.c_str());
    });
}

// ----------------------------------------------------------------- GPU
// Config 4's layer stack (4 x QuantizedMatMul 4096 x 4096 with per-channel
// scales -> FusedAddRelu(bias) -> Quantize uint8) plus an fp32 Gemm, with a
// pruned SparseMatMul.
Graph big_graph(int64_t hidden, int layers, int64_t batch) {
    Graph g("pfm_fast");
    g.add_input(TensorInfo("X", sh({batch, hidden}), DType::UInt8));
    g.add_input(TensorInfo("F", sh({batch, hidden}), DType::Float32));
    std::string cur = "X";
    std::mt19937_64 rng(7);
    std::uniform_real_distribution<float> us(0.005f, 0.02f);
    for (int l = 0; l < layers; ++l) {
        const std::string w = "w" + std::to_string(l), b = "b" + std::to_string(l);
        g.add_initializer(w, rand_tensor({hidden, hidden}, DType::Int8, 100 + l));
        Tensor bias = rand_tensor({hidden}, DType::Float32, 200 + l);
        for (int64_t i = 0; i < hidden; ++i) bias.data_ptr<float>()[i] *= 200.0f;
        g.add_initializer(b, std::move(bias));
        auto q = std::make_shared<Node>("qmm" + std::to_string(l), "QuantizedMatMul", std::vector<std::string>{cur, w},
                                        std::vector<std::string>{"a" + std::to_string(l)});
        std::vector<float> scales(static_cast<size_t>(hidden));
        for (auto& s : scales) s = us(rng);
        q->set_attr("a_scale", 0.02f);
        q->set_attr("a_zero_point", int64_t{0});
        q->set_attr("b_scales", scales);
        g.add_node(q);
        g.add_node(std::make_shared<Node>("far" + std::to_string(l), "FusedAddRelu",
                                          std::vector<std::string>{"a" + std::to_string(l), b},
                                          std::vector<std::string>{"r" + std::to_string(l)}));
        auto qz = std::make_shared<Node>("qz" + std::to_string(l), "Quantize",
                                         std::vector<std::string>{"r" + std::to_string(l)},
                                         std::vector<std::string>{"h" + std::to_string(l)});
        qz->set_attr("scale", 0.5f);
        qz->set_attr("dtype", std::string("uint8"));
        g.add_node(qz);
        cur = "h" + std::to_string(l);
    }
    g.add_initializer("G", rand_tensor({hidden, hidden}, DType::Float32, 300));
    g.add_initializer("C", rand_tensor({hidden}, DType::Float32, 301));
    auto gemm = std::make_shared<Node>("gemm", "Gemm", std::vector<std::string>{"F", "G", "C"},
                                       std::vector<std::string>{"Yf"});
    g.add_node(gemm);
    // A pruned weight in CSR (int64 indices, as the reference's SparseTensor keeps them).
    const int64_t sn = hidden / 2, sk = hidden;
    Tensor ip({sn + 1}, DType::Int64), ix({sn * 16}, DType::Int64), sv = rand_tensor({sn * 16}, DType::Float32, 302);
    for (int64_t r = 0; r <= sn; ++r) ip.data_ptr<int64_t>()[r] = r * 16;
    for (int64_t j = 0; j < sn * 16; ++j) ix.data_ptr<int64_t>()[j] = (j % 16) * (sk / 16) + (j / 16) % (sk / 16);
    g.add_initializer("sp_ip", std::move(ip));
    g.add_initializer("sp_ix", std::move(ix));
    g.add_initializer("sp_v", std::move(sv));
    auto sp = std::make_shared<Node>("spmm", "SparseMatMul", std::vector<std::string>{"F", "sp_ip", "sp_ix", "sp_v"},
                                     std::vector<std::string>{"Ys"});
    sp->set_attr("shape", std::vector<int64_t>{sn, sk});
    g.add_node(sp);
    g.add_output(TensorInfo(cur, sh({batch, hidden}), DType::UInt8));
    g.add_output(TensorInfo("Yf", sh({batch, hidden}), DType::Float32));
    g.add_output(TensorInfo("Ys", sh({batch, sn}), DType::Float32));
    return g;
}

double secs_since(std::chrono::steady_clock::time_point t) {
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t).count();
}

void gpu_tests() {
    const int64_t hidden = 4096, batch = 256;
    const std::string p = tmp_path("big");
    {
        Graph g = big_graph(hidden, 4, batch);
        PyFlameFormat::save(g, p);
    }
    std::unordered_map<std::string, Tensor> feeds;
    feeds["X"] = rand_tensor({batch, hidden}, DType::UInt8, 11);
    feeds["F"] = rand_tensor({batch, hidden}, DType::Float32, 12);
    const std::vector<std::string> outs = {"h3", "Yf", "Ys"};

    std::vector<Tensor> ref_out, fast_out;
    size_t bytes = 0;
    run_test("PfmWarmUp", [&] {
        // Module loading and first-launch costs of the process, paid once
        // before either path is timed.
        CudaBackend be(0);
        auto g = PyFlameFormat::load(p);
        be.execute(*g, feeds, outs);
    });
    // Each path three times on a fresh backend; medians reported.  The cost of
    // a path = load (or open + prepare) + its first run's excess over a steady
    // run, i.e. everything up to a model ready to serve.
    std::vector<double> ref_t, ref_load_t, fast_t, fast_prep_t;
    auto median = [](std::vector<double> v) {
        std::sort(v.begin(), v.end());
        return v[v.size() / 2];
    };
    for (int rep = 0; rep < 3; ++rep) {
        run_test("PfmReferenceLoaderPath", [&] {
            CudaBackend be(0);
            auto t = std::chrono::steady_clock::now();
            auto g = PyFlameFormat::load(p);
            const double load = secs_since(t);
            t = std::chrono::steady_clock::now();
            ref_out = be.execute(*g, feeds, outs);
            const double first = secs_since(t);
            t = std::chrono::steady_clock::now();
            be.execute(*g, feeds, outs);
            const double steady = secs_since(t);
            ref_t.push_back(load + first - steady);
            ref_load_t.push_back(load);
        });
        run_test("PfmFastPathMatchesReferenceLoader", [&] {
            CudaBackend be(0);
            auto t = std::chrono::steady_clock::now();
            auto img = cuda::PfmImage::open(p);
            auto st = be.prepare(img->graph());
            const double prep = secs_since(t);
            bytes = st.bytes;
            std::printf("  prepare: build %.1f ms, page-in thread %.1f ms (overlapped)\n", st.build_seconds * 1e3,
                        st.fault_seconds * 1e3);
            t = std::chrono::steady_clock::now();
            fast_out = be.execute(img->graph(), feeds, outs);
            const double first = secs_since(t);
            t = std::chrono::steady_clock::now();
            be.execute(img->graph(), feeds, outs);
            const double steady = secs_since(t);
            fast_t.push_back(prep + first - steady);
            fast_prep_t.push_back(prep);
            EXPECT(fast_out.size() == ref_out.size(), "output count");
            for (size_t i = 0; i < ref_out.size(); ++i)
                EXPECT(fast_out[i].size_bytes() == ref_out[i].size_bytes() &&
                           std::memcmp(fast_out[i].data(), ref_out[i].data(), ref_out[i].size_bytes()) == 0,
                       "output " + outs[i] + " differs");
        });
    }
    if (ref_t.empty() || fast_t.empty()) return;
    const double rt = median(ref_t), ft = median(fast_t);
    std::printf("  initializers %.1f MB (page cache warm), medians of 3\n", bytes / 1e6);
    std::printf("  reference loader: %.1f ms to a ready model (load %.1f ms), %.2f GB/s\n", rt * 1e3,
                median(ref_load_t) * 1e3, bytes / rt / 1e9);
    std::printf("  fast path: %.1f ms to a ready model (open + prepare %.1f ms), %.2f GB/s\n", ft * 1e3,
                median(fast_prep_t) * 1e3, bytes / ft / 1e9);
    std::printf("PFM_TIMING {\"bytes\": %zu, \"reference_ms\": %.3f, \"fast_ms\": %.3f}\n", bytes, rt * 1e3,
                ft * 1e3);
    std::remove(p.c_str());
}

}  // namespace

int main(int argc, char** argv) {
    const bool cpu_only = argc > 1 && std::strcmp(argv[1], "--cpu") == 0;
    cpu_tests();
    if (!cpu_only) gpu_tests();
    std::printf("%s: %d failed\n", g_failed ? "FAILED" : "OK", g_failed);
    return g_failed ? 1 : 0;
}
