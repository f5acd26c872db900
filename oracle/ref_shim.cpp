// ref_shim.cpp -- extern "C" entry points over the PyFlameRT reference's own
// hot-path code, compiled from the reference sources by oracle/Makefile into
// oracle/_ref/libpfrt_ref.so.
//
// TEST INFRASTRUCTURE ONLY.  Used by tests/ to pin the C restatement
// (oracle.c) and by bench.py's reference arm / cpu_baseline leg to time the
// reference's CPU implementation.  Nothing in the product links this.
//
// Every function returns 0 on success and -1 on a C++ exception, whose
// message is available from pfref_last_error().
#include "pyflame_rt/pruning/pruning.hpp"
#include "pyflame_rt/graph.hpp"
#include "pyflame_rt/node.hpp"
#include "pyflame_rt/tensor.hpp"
#include "pyflame_rt/quantization/quant_ops.hpp"
#include "pyflame_rt/quantization/quant_params.hpp"
#include "pyflame_rt/pruning/sparse_tensor.hpp"
#include "backends/cpu/executor.hpp"

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

using namespace pyflame_rt;

namespace {

thread_local std::string g_err;

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

Shape static_shape(const std::vector<int64_t>& dims) {
    Shape s;
    for (auto d : dims) s.push_back(d);
    return s;
}

// Runs a single-node graph through the reference CPUExecutor
// (src/backends/cpu/executor.cpp:45-147) and returns its outputs.
std::vector<Tensor> run_single_node(
    const std::string& op_type,
    const std::vector<std::pair<std::string, Tensor>>& inputs,
    const std::vector<std::pair<std::string, AttributeValue>>& attrs,
    DType out_dtype) {
    Graph g("pfref");
    std::vector<std::string> in_names;
    std::unordered_map<std::string, Tensor> feeds;
    for (const auto& [name, t] : inputs) {
        g.add_input(TensorInfo(name, static_shape(t.shape()), t.dtype()));
        in_names.push_back(name);
        feeds.emplace(name, t.view());  // non-owning; the executor clones it
    }
    g.add_output(TensorInfo("Y", Shape{}, out_dtype));
    auto node = std::make_shared<Node>("n0", op_type, in_names,
                                       std::vector<std::string>{"Y"});
    for (const auto& [k, v] : attrs) node->set_attr(k, v);
    g.add_node(node);
    CPUExecutor ex(0);
    return ex.execute(g, feeds, {"Y"});
}

Tensor view(const void* p, std::vector<int64_t> shape, DType dt) {
    return Tensor(const_cast<void*>(p), shape, dt);
}

// Splits [0, rows) into nthreads contiguous slices and runs fn(r0, r1) on
// each in its own thread.  The reference backend is single-threaded by
// construction (executor.cpp:10 stores num_threads_ and never uses it); this
// is harness parallelism over independent row slices.
template <class F>
void parallel_rows(int64_t rows, int nthreads, F fn) {
    if (nthreads <= 1 || rows < 2) {
        fn(int64_t{0}, rows);
        return;
    }
    if (nthreads > rows) nthreads = static_cast<int>(rows);
    std::vector<std::thread> ts;
    std::vector<std::string> errs(nthreads);
    for (int t = 0; t < nthreads; ++t) {
        int64_t r0 = rows * t / nthreads, r1 = rows * (t + 1) / nthreads;
        ts.emplace_back([&, t, r0, r1] {
            try {
                fn(r0, r1);
            } catch (const std::exception& e) {
                errs[t] = e.what();
            }
        });
    }
    for (auto& th : ts) th.join();
    for (auto& e : errs)
        if (!e.empty()) throw std::runtime_error(e);
}

}  // namespace

extern "C" {

const char* pfref_last_error() { return g_err.c_str(); }

// Gemm node through CPUExecutor -> cpu_gemm (src/backends/cpu/ops/math.cpp:377-438).
// A is [M,K] ([K,M] if trans_a), B is [K,N] ([N,K] if trans_b), C is [c_len]
// (nullable).
int pfref_gemm(int64_t M, int64_t N, int64_t K, int trans_a, int trans_b,
               float alpha, float beta, const float* A, const float* B,
               const float* C, int64_t c_len, float* Y, int nthreads) {
    return guarded([&] {
        if (trans_a && nthreads > 1) nthreads = 1;  // row slices need row-major A
        parallel_rows(M, nthreads, [&](int64_t r0, int64_t r1) {
            int64_t m = r1 - r0;
            std::vector<std::pair<std::string, Tensor>> in;
            in.emplace_back("A", trans_a ? view(A, {K, M}, DType::Float32)
                                         : view(A + r0 * K, {m, K}, DType::Float32));
            in.emplace_back("B", trans_b ? view(B, {N, K}, DType::Float32)
                                         : view(B, {K, N}, DType::Float32));
            // The flat bias index i % c_len depends on the global row; a row
            // slice starting at r0 only keeps it when N*r0 % c_len == 0.
            if (C && c_len > 0) {
                if ((r0 * N) % c_len != 0)
                    throw std::runtime_error("pfref_gemm: slice breaks bias broadcast");
                in.emplace_back("C", view(C, {c_len}, DType::Float32));
            }
            auto out = run_single_node(
                "Gemm", in,
                {{"alpha", alpha}, {"beta", beta},
                 {"transA", static_cast<int64_t>(trans_a)},
                 {"transB", static_cast<int64_t>(trans_b)}},
                DType::Float32);
            std::memcpy(Y + r0 * N, out[0].data(), sizeof(float) * m * N);
        });
    });
}

// MatMul node through CPUExecutor -> cpu_matmul (math.cpp:268-374), 2-D.
int pfref_matmul(int64_t M, int64_t N, int64_t K, const float* A,
                 const float* B, float* Y, int nthreads) {
    return guarded([&] {
        parallel_rows(M, nthreads, [&](int64_t r0, int64_t r1) {
            int64_t m = r1 - r0;
            auto out = run_single_node(
                "MatMul",
                {{"A", view(A + r0 * K, {m, K}, DType::Float32)},
                 {"B", view(B, {K, N}, DType::Float32)}},
                {}, DType::Float32);
            std::memcpy(Y + r0 * N, out[0].data(), sizeof(float) * m * N);
        });
    });
}

// quantization::quantized_matmul (src/quantization/quant_ops.cpp:387-506),
// per-tensor parameters.  out_mode 0: fp32 dequantized output; 1/2: requant
// to int8/uint8 via quantize_tensor (quant_ops.cpp:501-503).
int pfref_quantized_matmul(int64_t M, int64_t N, int64_t K, const void* a,
                           int a_is_u8, float a_scale, int32_t a_zp,
                           const void* b, int b_is_u8, float b_scale,
                           int32_t b_zp, int out_mode, float y_scale,
                           int32_t y_zp, void* out, int nthreads) {
    return guarded([&] {
        DType adt = a_is_u8 ? DType::UInt8 : DType::Int8;
        DType bdt = b_is_u8 ? DType::UInt8 : DType::Int8;
        auto ap = quantization::QuantParams::per_tensor(a_scale, a_zp, adt);
        auto bp = quantization::QuantParams::per_tensor(b_scale, b_zp, bdt);
        parallel_rows(M, nthreads, [&](int64_t r0, int64_t r1) {
            int64_t m = r1 - r0;
            Tensor at = view(static_cast<const uint8_t*>(a) + r0 * K, {m, K}, adt);
            Tensor bt = view(b, {K, N}, bdt);
            if (out_mode == 0) {
                Tensor r = quantization::quantized_matmul(at, ap, bt, bp, nullptr);
                std::memcpy(static_cast<float*>(out) + r0 * N, r.data(), sizeof(float) * m * N);
            } else {
                auto op = quantization::QuantParams::per_tensor(
                    y_scale, y_zp, out_mode == 2 ? DType::UInt8 : DType::Int8);
                Tensor r = quantization::quantized_matmul(at, ap, bt, bp, &op);
                std::memcpy(static_cast<uint8_t*>(out) + r0 * N, r.data(), m * N);
            }
        });
    });
}

// Per-output-channel quantized linear layer built from reference code only:
// quantized_matmul (quant_ops.cpp:387-506) is called once per output column
// n with b_scale = w_scale[n], which is exactly the per-channel dequant
// (float)acc * (a_scale * w_scale[n]); the result then goes through the
// reference's own Add (math.cpp:222-226), Relu (activation.cpp:45-60) and
// Quantize (quantized_ops.cpp, quantize_tensor) graph ops on CPUExecutor.
// out_mode 0: fp32 output, 1: int8, 2: uint8.
int pfref_qlinear_per_channel(int64_t M, int64_t N, int64_t K, const void* a,
                              int a_is_u8, float a_scale, int32_t a_zp,
                              const int8_t* w, int32_t w_zp,
                              const float* w_scale, const float* bias,
                              int relu, int out_mode, float y_scale,
                              int32_t y_zp, void* out) {
    return guarded([&] {
        DType adt = a_is_u8 ? DType::UInt8 : DType::Int8;
        auto ap = quantization::QuantParams::per_tensor(a_scale, a_zp, adt);
        Tensor at = view(a, {M, K}, adt);
        std::vector<float> y(static_cast<size_t>(M * N));
        std::vector<int8_t> wcol(static_cast<size_t>(K));
        for (int64_t n = 0; n < N; ++n) {
            for (int64_t k = 0; k < K; ++k) wcol[k] = w[k * N + n];
            auto bp = quantization::QuantParams::per_tensor(w_scale[n], w_zp, DType::Int8);
            Tensor bt = view(wcol.data(), {K, 1}, DType::Int8);
            Tensor r = quantization::quantized_matmul(at, ap, bt, bp, nullptr);
            const float* rp = r.data_ptr<float>();
            for (int64_t m = 0; m < M; ++m) y[m * N + n] = rp[m];
        }
        Tensor cur = view(y.data(), {M, N}, DType::Float32);
        std::vector<Tensor> keep;
        if (bias) {
            auto o = run_single_node(
                "Add", {{"x", cur}, {"b", view(bias, {N}, DType::Float32)}}, {},
                DType::Float32);
            keep.push_back(std::move(o[0]));
            cur = keep.back().view();
        }
        if (relu) {
            auto o = run_single_node("Relu", {{"x", cur}}, {}, DType::Float32);
            keep.push_back(std::move(o[0]));
            cur = keep.back().view();
        }
        if (out_mode == 0) {
            std::memcpy(out, cur.data(), sizeof(float) * M * N);
            return;
        }
        auto o = run_single_node(
            "Quantize", {{"x", cur}},
            {{"scale", y_scale}, {"zero_point", static_cast<int64_t>(y_zp)},
             {"dtype", std::string(out_mode == 2 ? "uint8" : "int8")}},
            out_mode == 2 ? DType::UInt8 : DType::Int8);
        std::memcpy(out, o[0].data(), M * N);
    });
}

// The registered graph op QuantizedMatMul -> cpu_quantized_matmul
// (src/backends/cpu/ops/quantized_ops.cpp:77-167), fp32 output.  Kept to
// document its behaviour: it reads both operands as int8 (:143-144).
int pfref_quantized_matmul_op(int64_t M, int64_t N, int64_t K, const void* a,
                              int a_is_u8, float a_scale, int32_t a_zp,
                              const int8_t* b, float b_scale, int32_t b_zp,
                              float* out) {
    return guarded([&] {
        auto o = run_single_node(
            "QuantizedMatMul",
            {{"A", view(a, {M, K}, a_is_u8 ? DType::UInt8 : DType::Int8)},
             {"B", view(b, {K, N}, DType::Int8)}},
            {{"a_scale", a_scale}, {"b_scale", b_scale},
             {"a_zero_point", static_cast<int64_t>(a_zp)},
             {"b_zero_point", static_cast<int64_t>(b_zp)}},
            DType::Float32);
        std::memcpy(out, o[0].data(), sizeof(float) * M * N);
    });
}

// quantize_tensor per-tensor (quant_ops.cpp:15-55).
int pfref_quantize(int64_t n, const float* x, float scale, int32_t zp,
                   int out_is_u8, void* q) {
    return guarded([&] {
        DType dt = out_is_u8 ? DType::UInt8 : DType::Int8;
        auto p = quantization::QuantParams::per_tensor(scale, zp, dt);
        Tensor r = quantization::quantize_tensor(view(x, {n}, DType::Float32), p);
        std::memcpy(q, r.data(), n);
    });
}

// pruning::sparse_matmul (src/pruning/sparse_tensor.cpp:473-519) on a CSR
// SparseTensor built by from_csr (:170-197) from int64 copies.
// W is [R, Kw]; B is dense [Kw, C]; out is [R, C].
int pfref_sparse_matmul(int64_t R, int64_t Kw, int64_t C, const int64_t* indptr,
                        const int64_t* indices, const float* values,
                        int64_t nnz, const float* B, float* out, int nthreads) {
    return guarded([&] {
        parallel_rows(R, nthreads, [&](int64_t r0, int64_t r1) {
            int64_t base = indptr[r0];
            std::vector<int64_t> ip(indptr + r0, indptr + r1 + 1);
            for (auto& v : ip) v -= base;
            std::vector<int64_t> ix(indices + base, indices + indptr[r1]);
            std::vector<float> vv(values + base, values + indptr[r1]);
            auto w = pruning::SparseTensor::from_csr({r1 - r0, Kw}, ip, ix, vv);
            Tensor r = pruning::sparse_matmul(w, view(B, {Kw, C}, DType::Float32));
            std::memcpy(out + r0 * C, r.data(), sizeof(float) * (r1 - r0) * C);
        });
        (void)nnz;
    });
}

// pruning::MagnitudePruning::compute_mask (src/pruning/magnitude_pruning.cpp:
// 22-102) on W [rows, cols]: mask_out [rows*cols] of 0/1 floats.
int pfref_magnitude_mask(int64_t rows, int64_t cols, const float* w, float sparsity, float* mask_out) {
    return guarded([&] {
        pruning::MagnitudePruning mp;
        auto m = mp.compute_mask("w", view(w, {rows, cols}, DType::Float32), sparsity);
        std::memcpy(mask_out, m.mask.data(), sizeof(float) * rows * cols);
    });
}

// pruning::NMSparsityPruning(n, m).compute_mask (src/pruning/nm_sparsity.cpp:
// 45-126) on `total` weights taken in flat order: mask_out [total] of 0/1.
int pfref_nm_mask(int64_t total, const float* w, int64_t n, int64_t m, float* mask_out) {
    return guarded([&] {
        pruning::NMSparsityPruning nm(static_cast<size_t>(n), static_cast<size_t>(m));
        auto mk = nm.compute_mask("w", view(w, {total}, DType::Float32), 0.0f);
        if (total > 0) std::memcpy(mask_out, mk.mask.data(), sizeof(float) * total);
    });
}

// pruning::to_sparse(dense, threshold, CSR) (src/pruning/sparse_tensor.cpp:
// 560-587) on D [rows, cols]; writes indptr [rows+1], and indices/values up
// to `cap` entries, and *nnz_out.
int pfref_to_sparse_csr(int64_t rows, int64_t cols, const float* d, float threshold, int64_t cap,
                        int64_t* indptr, int64_t* indices, float* values, int64_t* nnz_out) {
    return guarded([&] {
        auto sp = pruning::to_sparse(view(d, {rows, cols}, DType::Float32), threshold, pruning::SparseFormat::CSR);
        const auto& ip = sp.indptr();
        const auto& ix = sp.indices();
        const float* v = sp.values().data();
        *nnz_out = static_cast<int64_t>(ix.size());
        std::copy(ip.begin(), ip.end(), indptr);
        const int64_t n = std::min<int64_t>(cap, static_cast<int64_t>(ix.size()));
        std::copy(ix.begin(), ix.begin() + n, indices);
        std::copy(v, v + n, values);
    });
}

}  // extern "C"
