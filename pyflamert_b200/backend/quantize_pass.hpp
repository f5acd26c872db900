// quantize_pass.hpp -- the "Quantizer output -> per-channel QuantizedMatMul"
// graph pass of the CUDA backend.
//
// The reference's Quantizer (src/quantization/quantizer.cpp:342-371) turns a
// MatMul into QuantizedMatMul with per-tensor a_/b_scale attributes only.
// This pass produces the per-output-channel form the backend runs on its
// int8 tensor-core GEMM with the requantization epilogue:
//
//   MatMul(X, B)  ->  Quantize(X -> Xq; scale, zero_point, dtype = uint8)
//                     QuantizedMatMul(Xq, Bq; a_scale, a_zero_point,
//                                     b_scales = [N], b_zero_point = 0)
//
// with the reference's own parameter rules:
//   - B [K, N] (a float32 initializer) is quantized per output channel
//     (axis 1), symmetric int8: compute_dynamic_params_per_channel(B, 1,
//     Int8, true) (src/quantization/quant_ops.cpp:324-380), quantized per
//     channel as quantize_tensor / QuantizedTensor do (quant_ops.cpp:15-127,
//     quant_params.cpp:112-235);
//   - X's (scale, zero_point) come from its calibrated range [min, max]:
//     QuantParams::compute_from_minmax(min, max, UInt8, asymmetric)
//     (quant_params.cpp:14-55).
// QuantizedMatMul's output stays float32 (a_scale * b_scale[n] * acc), so a
// following Add (bias) -> Relu [-> Quantize] is fused by the backend.
#pragma once

#include <string>
#include <unordered_map>
#include <utility>

#include "pyflame_rt/graph.hpp"

namespace pyflame_rt {
namespace cuda {

struct QuantizePassOptions {
    // Calibrated range (min, max) of each MatMul activation input, by tensor
    // name; a MatMul whose input has no range is left as it is.
    std::unordered_map<std::string, std::pair<float, float>> act_ranges;
};

struct QuantizePassReport {
    int rewritten = 0;
};

Graph quantize_matmuls_per_channel(const Graph& graph, const QuantizePassOptions& options,
                                   QuantizePassReport* report = nullptr);

}  // namespace cuda
}  // namespace pyflame_rt
