// pfm_image.hpp -- a PyFlameRT .pfm model mapped read-only, for the CUDA
// backend's load path.
//
// The reference loader (PyFlameFormat::load, src/io/pyflame_format.cpp:
// 392-460) reads every initializer through a temporary std::vector<char> into
// a freshly allocated, zero-filled host Tensor (read_tensor, :178-251): three
// passes over the weights in host memory before a backend sees them, and the
// CUDA backend then copies them again, from pageable memory, to the device.
//
// PfmImage::open maps the file instead and builds the same Graph (same
// inputs, outputs, nodes and attributes, same validation limits and error
// messages, pyflame_format.hpp:11-20) whose initializers are non-owning
// Tensors viewing the mapping (Tensor(void*, shape, dtype), tensor.hpp:21).
// No initializer byte is copied on the host; the pages are read when the
// backend stages them for the device (CudaBackend::prepare).  The image owns
// the mapping: keep it alive as long as the graph (or anything holding views
// of its initializers) is in use.
#pragma once

#include <cstddef>
#include <memory>
#include <string>

#include "pyflame_rt/graph.hpp"

namespace pyflame_rt {
namespace cuda {

class PfmImage {
public:
    /// Maps and parses `path`.  Throws InvalidModelError exactly where
    /// PyFlameFormat::load would, with the same messages.
    static std::shared_ptr<const PfmImage> open(const std::string& path);

    ~PfmImage();
    PfmImage(const PfmImage&) = delete;
    PfmImage& operator=(const PfmImage&) = delete;

    const Graph& graph() const { return *graph_; }
    /// Bytes of initializer data viewed in the mapping.
    size_t initializer_bytes() const { return init_bytes_; }
    size_t file_bytes() const { return size_; }

private:
    PfmImage() = default;
    void* base_ = nullptr;
    size_t size_ = 0;
    size_t init_bytes_ = 0;
    std::unique_ptr<Graph> graph_;
};

}  // namespace cuda
}  // namespace pyflame_rt
