// cuda_backend.hpp -- PyFlameRT execution backend for B200 (sm_100a).
//
// Implements the reference's plugin interface pyflame_rt::Backend
// (include/pyflame_rt/backend.hpp:14-46) over the C ABI in pfrt_cuda.h, so
// that InferenceSession can run a graph with device = "cuda" in place of
// CPUExecutor (src/backends/cpu/executor.cpp:45-147), with no change to the
// graph, the importers or the session's run().
//
// Node types and their reference counterparts:
//   Gemm             cpu_gemm             (src/backends/cpu/ops/math.cpp:377-438)
//   MatMul           cpu_matmul           (math.cpp:268-374)
//   QuantizedMatMul  quantized_matmul     (src/quantization/quant_ops.cpp:387-506);
//                    per-tensor a_scale/b_scale/a_zero_point/b_zero_point as the
//                    graph op (quantized_ops.cpp:87-90), or per-output-channel
//                    b_scales (float vector).  A following Add (initializer
//                    bias [N]) -> Relu -> Quantize chain is fused into it.
//   SparseMatMul     sparse_matmul        (src/pruning/sparse_tensor.cpp:473-519):
//                    inputs X, indptr, indices, values; attr shape = [N, K];
//                    Y[M,N] = X W^T
//   Add, Relu        cpu_add, cpu_relu    (math.cpp:222-226, activation.cpp:45-60):
//                    same shapes, or a row-vector / scalar operand
//   FusedAddRelu     the fusion pass's Add -> Relu (src/opt/fusion_patterns.cpp:40-70),
//                    max(0, a + b); fused into a preceding QuantizedMatMul as
//                    its bias + ReLU
//   Quantize         cpu_quantize         (quantized_ops.cpp, quantize_tensor)
// Any other node type raises UnsupportedOperatorError(op, "cuda"); there is
// no CPU fallback.  Errors inside a node raise BackendError(message, node name)
// as CPUExecutor does (executor.cpp:106-110).
//
// Initializers (weights, biases, CSR arrays) are uploaded and prepared once
// per graph and reused across runs; graph inputs are copied to the device and
// graph outputs back to new host Tensors on every run.  execute() is
// serialised by a mutex, so a session may call it from several threads.
#pragma once

#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "pyflame_rt/backend.hpp"

namespace pyflame_rt {

class CudaBackend : public Backend {
public:
    explicit CudaBackend(int device = 0);
    /// A backend over several GPUs of this process.  execute() splits a batch
    /// over them by rows when the graph allows it (batch_split_plan: every
    /// node is row-separable and each device gets at least
    /// PFRT_SPLIT_MIN_ROWS rows, default 256): each device runs the graph on
    /// its contiguous slice of every input (a view, no host copy) with its
    /// own copy of the weights, and copies its rows of every output straight
    /// into the output Tensors.  There is no collective: the rows are
    /// independent.  Other graphs run on the first device.
    explicit CudaBackend(const std::vector<int>& devices);
    ~CudaBackend() override;

    CudaBackend(const CudaBackend&) = delete;
    CudaBackend& operator=(const CudaBackend&) = delete;

    const std::string& name() const override;
    bool supports_op(const std::string& op_type) const override;
    std::vector<std::string> get_supported_ops() const override;

    std::vector<Tensor> execute(const Graph& graph,
                                const std::unordered_map<std::string, Tensor>& input_feed,
                                const std::vector<std::string>& output_names = {}) override;

    int device() const;  // the first device
    const std::vector<int>& devices() const;

    /// Drops every prepared initializer (the next execute() prepares them
    /// again).  The caches are keyed on a signature of the graph (its nodes,
    /// and each initializer's name, address, dtype, shape and sampled bytes),
    /// so a different or changed graph is noticed by itself; call this after
    /// rewriting an initializer's data in place.
    void invalidate();

    /// Uploads and prepares every initializer the graph's nodes consume (the
    /// device forms of Gemm/MatMul/QuantizedMatMul weights, CSR arrays,
    /// biases), as the first execute() would, and keeps them for later runs.
    /// A second thread faults in the next node's initializer pages (several
    /// threads per tensor) while the current node's device forms are built,
    /// so a PfmImage graph, whose initializers view the mapped file, is read
    /// once, in parallel, with no host copy of a weight.  Raises what
    /// execute() would for a bad weight.  Not needed for correctness:
    /// execute() prepares lazily.
    struct PrepareStats {
        size_t bytes = 0;            // initializer bytes prepared
        double seconds = 0.0;        // wall time of the call
        double build_seconds = 0.0;  // building device forms (copies, kernels)
        double fault_seconds = 0.0;  // the page-in thread's busy time (overlapped)
    };
    PrepareStats prepare(const Graph& graph);

private:
    class Impl;
    std::vector<int> devices_;
    std::vector<std::unique_ptr<Impl>> impls_;
};

/// Factories for the session seam (InferenceSession::select_backend): a
/// CudaBackend on the given device ordinal, or on the devices a
/// SessionOptions.device string names (parse_cuda_devices).
std::unique_ptr<Backend> make_cuda_backend(int device = 0);
std::unique_ptr<Backend> make_cuda_backend(const std::string& device_spec);

/// Device ordinals of a device string: "cuda" -> the list in the environment
/// variable PFRT_CUDA_DEVICES ("0,1,2,3") if it is set, else {0};
/// "cuda:<n>" -> {n}; "cuda:<n>,<m>,..." -> that list.  Throws
/// BackendError for anything else.
std::vector<int> parse_cuda_devices(const std::string& device_spec);

/// Row ranges [m0, m1) of a batch split of the feeds over `parts` devices, or
/// an empty vector when the graph cannot be split by rows: every graph input
/// must be fed a 2-D tensor with the same row count M >= parts * min_rows,
/// every node must compute each output row from the same row of its
/// activation inputs only (Gemm with transA = 0 and a C that broadcasts per
/// row, MatMul / QuantizedMatMul / SparseMatMul on initializer weights,
/// elementwise Add / FusedAddRelu / Relu / Quantize against same-shape
/// activations or row-vector or scalar initializers), and no requested output
/// may be an initializer.  Host-only (no device needed).
std::vector<std::pair<int64_t, int64_t>> batch_split_plan(const Graph& graph,
                                                          const std::unordered_map<std::string, Tensor>& feeds,
                                                          int parts, int64_t min_rows);

}  // namespace pyflame_rt
