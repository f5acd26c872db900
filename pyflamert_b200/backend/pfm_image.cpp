// pfm_image.cpp -- PfmImage: the .pfm format (src/io/pyflame_format.cpp)
// parsed from a read-only mapping, initializers as views.
//
// The format is the reference's and is kept alike field for field (it is an
// on-disk interface): magic "PFM\0", u32 version (<= 1), the graph name, the
// input and output TensorInfos (name, u32 dtype, u64 ndim, i64 dims with -1 =
// dynamic), the initializers (name, u32 dtype, u64 ndim, i64 dims, u64 byte
// count, bytes), then the nodes (name, op type, inputs, outputs, attributes
// tagged 0 int64 / 1 float / 2 string / 3 int64 vector / 4 float vector /
// 255 skipped), all little-endian.  The checks, their order and their
// messages follow read_tensor_info/read_tensor/read_node/load
// (pyflame_format.cpp:135-460) so that a bad file fails the same way on both
// load paths.
#include "pfm_image.hpp"

#include <cstring>
#include <fcntl.h>
#include <stdexcept>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "pyflame_rt/errors.hpp"
#include "pyflame_rt/types.hpp"

namespace pyflame_rt {
namespace cuda {

namespace {

// pyflame_format.hpp:11-20
constexpr uint64_t kMaxString = 10ULL * 1024 * 1024;
constexpr uint64_t kMaxTensorData = 4ULL * 1024 * 1024 * 1024;
constexpr uint64_t kMaxArray = 1000000;
constexpr uint64_t kMaxDims = 16;
constexpr uint64_t kMaxNodes = 1000000;
constexpr uint64_t kMaxAttrs = 1000;
constexpr int64_t kMaxDim = 100000000LL;
constexpr int64_t kMaxElements = 1000000000LL;

// Bounds-checked reader over the mapping.
class Cursor {
public:
    Cursor(const uint8_t* p, size_t n) : p_(p), n_(n) {}

    // Next `size` bytes, or InvalidModelError("Incomplete read: ...") with the
    // byte count a stream read would have returned.
    const uint8_t* take(size_t size, const char* context) {
        const size_t avail = n_ - off_;
        if (size > avail) {
            off_ = n_;
            throw InvalidModelError(std::string("Incomplete read: ") + context + " (expected " +
                                    std::to_string(size) + " bytes, got " + std::to_string(avail) + ")");
        }
        const uint8_t* q = p_ + off_;
        off_ += size;
        return q;
    }
    template <class T>
    T pod(const char* context) {
        T v;
        std::memcpy(&v, take(sizeof(T), context), sizeof(T));
        return v;
    }
    uint32_t u32() { return pod<uint32_t>("uint32"); }
    uint64_t u64() { return pod<uint64_t>("uint64"); }
    int64_t i64() { return pod<int64_t>("int64"); }

    std::string str() {
        const uint64_t size = u64();
        if (size > kMaxString)
            throw InvalidModelError("String size exceeds limit: " + std::to_string(size) + " > " +
                                    std::to_string(kMaxString));
        if (size == 0) return std::string();
        const uint8_t* q = take(static_cast<size_t>(size), "string data");
        return std::string(reinterpret_cast<const char*>(q), static_cast<size_t>(size));
    }

private:
    const uint8_t* p_;
    size_t n_;
    size_t off_ = 0;
};

DType checked_dtype(uint32_t v, const std::string& msg) {
    if (!validate_dtype_value(v)) throw InvalidModelError(msg + std::to_string(v));
    return static_cast<DType>(v);
}

TensorInfo tensor_info(Cursor& c) {
    TensorInfo info;
    info.name = c.str();
    info.dtype = checked_dtype(c.u32(), "Invalid dtype value: ");
    const uint64_t ndim = c.u64();
    if (ndim > kMaxDims)
        throw InvalidModelError("Too many dimensions: " + std::to_string(ndim) + " > " + std::to_string(kMaxDims));
    info.shape.reserve(static_cast<size_t>(ndim));
    for (uint64_t i = 0; i < ndim; ++i) {
        const int64_t v = c.i64();
        if (v < 0) info.shape.push_back(std::nullopt);
        else info.shape.push_back(v);
    }
    return info;
}

// One initializer: a Tensor viewing its bytes in the mapping.
std::pair<std::string, Tensor> initializer(Cursor& c, size_t& bytes) {
    std::string name = c.str();
    const DType dtype = checked_dtype(c.u32(), "Invalid dtype value in tensor '" + name + "': ");
    const uint64_t ndim = c.u64();
    if (ndim > kMaxDims)
        throw InvalidModelError("Too many dimensions in tensor '" + name + "': " + std::to_string(ndim));
    std::vector<int64_t> shape(static_cast<size_t>(ndim));
    for (uint64_t i = 0; i < ndim; ++i) {
        shape[i] = c.i64();
        if (shape[i] < 0)
            throw InvalidModelError("Negative dimension in tensor '" + name + "' at axis " + std::to_string(i));
        if (shape[i] > kMaxDim)
            throw InvalidModelError("Dimension too large in tensor '" + name + "' at axis " + std::to_string(i) +
                                    ": " + std::to_string(shape[i]) + " > " + std::to_string(kMaxDim));
    }
    int64_t elements;
    try {
        elements = checked_product(shape);
    } catch (const std::overflow_error&) {
        throw InvalidModelError("Tensor '" + name + "' dimension product overflows int64");
    }
    if (elements > kMaxElements)
        throw InvalidModelError("Tensor '" + name + "' has too many elements: " + std::to_string(elements) + " > " +
                                std::to_string(kMaxElements));
    // Tensor::size_bytes of the reference: 0 for a 0-d shape.
    const size_t expected = shape.empty() ? 0 : static_cast<size_t>(elements) * dtype_size(dtype);
    const uint64_t size = c.u64();
    if (size > kMaxTensorData)
        throw InvalidModelError("Data size exceeds limit: " + std::to_string(size) + " > " +
                                std::to_string(kMaxTensorData));
    const uint8_t* data = size ? c.take(static_cast<size_t>(size), "byte data") : nullptr;
    if (size != expected)
        throw InvalidModelError("Data size mismatch for tensor '" + name + "': got " + std::to_string(size) +
                                ", expected " + std::to_string(expected));
    bytes += expected;
    // A 0-byte tensor keeps a null data pointer, as an empty owned Tensor does.
    return {std::move(name), Tensor(expected ? const_cast<uint8_t*>(data) : nullptr, shape, dtype)};
}

std::shared_ptr<Node> node(Cursor& c) {
    std::string name = c.str();
    std::string op_type = c.str();
    const uint64_t ni = c.u64();
    if (ni > kMaxArray) throw InvalidModelError("Too many inputs for node '" + name + "': " + std::to_string(ni));
    std::vector<std::string> inputs;
    inputs.reserve(static_cast<size_t>(ni));
    for (uint64_t i = 0; i < ni; ++i) inputs.push_back(c.str());
    const uint64_t no = c.u64();
    if (no > kMaxArray) throw InvalidModelError("Too many outputs for node '" + name + "': " + std::to_string(no));
    std::vector<std::string> outputs;
    outputs.reserve(static_cast<size_t>(no));
    for (uint64_t i = 0; i < no; ++i) outputs.push_back(c.str());
    auto n = std::make_shared<Node>(name, op_type, inputs, outputs);
    const uint64_t na = c.u64();
    if (na > kMaxAttrs)
        throw InvalidModelError("Too many attributes for node '" + name + "': " + std::to_string(na));
    for (uint64_t i = 0; i < na; ++i) {
        std::string an = c.str();
        const uint32_t type = c.u32();
        if (type == 0) {
            n->set_attr(an, c.i64());
        } else if (type == 1) {
            n->set_attr(an, c.pod<float>("float attribute"));
        } else if (type == 2) {
            n->set_attr(an, c.str());
        } else if (type == 3 || type == 4) {
            const uint64_t len = c.u64();
            if (len > kMaxArray)
                throw InvalidModelError("Vector attribute '" + an + "' too large: " + std::to_string(len));
            if (type == 3) {
                std::vector<int64_t> v(static_cast<size_t>(len));
                for (uint64_t j = 0; j < len; ++j) v[j] = c.i64();
                n->set_attr(an, v);
            } else {
                std::vector<float> v(static_cast<size_t>(len));
                for (uint64_t j = 0; j < len; ++j) v[j] = c.pod<float>("float vector element");
                n->set_attr(an, v);
            }
        } else if (type != 255) {
            throw InvalidModelError("Unknown attribute type " + std::to_string(type) + " for attribute '" + an +
                                    "' in node '" + name + "'");
        }
    }
    return n;
}

}  // namespace

std::shared_ptr<const PfmImage> PfmImage::open(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) throw InvalidModelError("Cannot open file", path);
    struct stat st {};
    if (fstat(fd, &st) != 0 || !S_ISREG(st.st_mode)) {
        ::close(fd);
        throw InvalidModelError("Cannot open file", path);
    }
    std::shared_ptr<PfmImage> img(new PfmImage());
    img->size_ = static_cast<size_t>(st.st_size);
    if (img->size_ > 0) {
        void* p = mmap(nullptr, img->size_, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            ::close(fd);
            throw InvalidModelError("Cannot open file", path);
        }
        img->base_ = p;
    }
    ::close(fd);  // the mapping keeps the file

    Cursor c(static_cast<const uint8_t*>(img->base_), img->size_);
    const uint8_t* magic = c.take(4, "magic bytes");
    if (std::memcmp(magic, "PFM\0", 4) != 0) throw InvalidModelError("Invalid magic bytes", path);
    const uint32_t version = c.u32();
    if (version > 1) throw InvalidModelError("Unsupported version: " + std::to_string(version), path);
    img->graph_ = std::make_unique<Graph>(c.str());
    Graph& g = *img->graph_;
    const uint64_t ni = c.u64();
    if (ni > kMaxArray) throw InvalidModelError("Too many graph inputs: " + std::to_string(ni), path);
    for (uint64_t i = 0; i < ni; ++i) g.add_input(tensor_info(c));
    const uint64_t no = c.u64();
    if (no > kMaxArray) throw InvalidModelError("Too many graph outputs: " + std::to_string(no), path);
    for (uint64_t i = 0; i < no; ++i) g.add_output(tensor_info(c));
    const uint64_t nin = c.u64();
    if (nin > kMaxArray) throw InvalidModelError("Too many initializers: " + std::to_string(nin), path);
    for (uint64_t i = 0; i < nin; ++i) {
        auto [name, t] = initializer(c, img->init_bytes_);
        g.add_initializer(name, std::move(t));
    }
    const uint64_t nn = c.u64();
    if (nn > kMaxNodes) throw InvalidModelError("Too many nodes: " + std::to_string(nn), path);
    for (uint64_t i = 0; i < nn; ++i) g.add_node(node(c));
    return img;
}

PfmImage::~PfmImage() {
    graph_.reset();  // views first, then the bytes they view
    if (base_) munmap(base_, size_);
}

}  // namespace cuda
}  // namespace pyflame_rt
