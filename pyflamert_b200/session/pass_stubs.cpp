// pass_stubs.cpp -- the parts of the reference runtime that InferenceSession
// references but whose sources do not compile (src/opt/constant_folding.cpp,
// cse.cpp, dead_code_elimination.cpp, operator_fusion.cpp and
// src/quantization/quantizer.cpp).  The session here runs graphs as saved
// (OptLevel::None, no quantization config), so none of these is reached; each
// raises if it is.  Linked into libpfrt_session.so and the session tests.
#include <stdexcept>

#include "pyflame_rt/opt/constant_folding.hpp"
#include "pyflame_rt/opt/cse.hpp"
#include "pyflame_rt/opt/dead_code_elimination.hpp"
#include "pyflame_rt/opt/operator_fusion.hpp"
#include "pyflame_rt/quantization/quantizer.hpp"

namespace pyflame_rt {
namespace opt {

namespace {
[[noreturn]] void not_built(const char* what) {
    throw std::runtime_error(std::string(what) + " is not available in this build (OptLevel::None only)");
}
}  // namespace

PassResult ConstantFoldingPass::run(Graph&) { not_built("ConstantFoldingPass"); }
PassResult CSEPass::run(Graph&) { not_built("CSEPass"); }
PassResult DeadCodeEliminationPass::run(Graph&) { not_built("DeadCodeEliminationPass"); }
OperatorFusionPass::OperatorFusionPass() = default;
PassResult OperatorFusionPass::run(Graph&) { not_built("OperatorFusionPass"); }

}  // namespace opt

namespace quantization {

Quantizer::Quantizer(const QuantConfig& config) : config_(config) {
    throw std::runtime_error("Quantizer is not available in this build (no quantization config)");
}
Quantizer::~Quantizer() = default;
QuantizationResult Quantizer::quantize_dynamic(const Graph&) { throw std::runtime_error("Quantizer"); }
QuantizationResult Quantizer::convert_to_fp16(const Graph&) { throw std::runtime_error("Quantizer"); }
QuantizationResult Quantizer::convert_to_bfloat16(const Graph&) { throw std::runtime_error("Quantizer"); }
QuantizationResult Quantizer::quantize_with_calibration(const Graph&, CalibrationDataProvider, size_t) {
    throw std::runtime_error("Quantizer");
}

}  // namespace quantization
}  // namespace pyflame_rt
