// session_capi.cpp -- the C entry points of include/pfrt_session.h over the
// reference's InferenceSession (src/session.cpp) with the CUDA seam.
#include "pfrt_session.h"

#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "pyflame_rt/options.hpp"
#include "pyflame_rt/session.hpp"

struct pfrt_session {
    std::unique_ptr<pyflame_rt::InferenceSession> s;
};

struct pfrt_outputs {
    std::vector<pyflame_rt::Tensor> t;
};

namespace {

int report(const std::exception& e, char* err, size_t err_len) {
    if (err && err_len) {
        std::strncpy(err, e.what(), err_len - 1);
        err[err_len - 1] = '\0';
    }
    return 1;
}

}  // namespace

extern "C" {

int pfrt_session_open(const char* pfm_path, const char* device, pfrt_session** out, char* err, size_t err_len) {
    try {
        if (!pfm_path || !device || !out) throw std::invalid_argument("pfrt_session_open: null argument");
        *out = nullptr;
        pyflame_rt::SessionOptions opts;
        opts.device = device;
        opts.optimization_level = pyflame_rt::OptLevel::None;
        auto s = std::make_unique<pfrt_session>();
        s->s = std::make_unique<pyflame_rt::InferenceSession>(pfm_path, opts);
        *out = s.release();
        return 0;
    } catch (const std::exception& e) {
        return report(e, err, err_len);
    }
}

void pfrt_session_close(pfrt_session* s) { delete s; }

int pfrt_session_run(pfrt_session* s, int n_in, const char* const* names, const void* const* data,
                     const int32_t* dtypes, const int32_t* ndims, const int64_t* dims, int n_out,
                     const char* const* out_names, pfrt_outputs** out, char* err, size_t err_len) {
    try {
        if (!s || !out || (n_in > 0 && (!names || !data || !dtypes || !ndims || !dims)) || (n_out > 0 && !out_names))
            throw std::invalid_argument("pfrt_session_run: null argument");
        *out = nullptr;
        std::unordered_map<std::string, pyflame_rt::Tensor> feed;
        const int64_t* d = dims;
        for (int i = 0; i < n_in; ++i) {
            std::vector<int64_t> shape(d, d + ndims[i]);
            d += ndims[i];
            // A view of the caller's buffer: the session reads it during run().
            feed.emplace(names[i], pyflame_rt::Tensor(const_cast<void*>(data[i]), shape,
                                                      static_cast<pyflame_rt::DType>(dtypes[i])));
        }
        std::vector<std::string> outs;
        for (int i = 0; i < n_out; ++i) outs.emplace_back(out_names[i]);
        auto o = std::make_unique<pfrt_outputs>();
        o->t = s->s->run(outs, feed);
        *out = o.release();
        return 0;
    } catch (const std::exception& e) {
        return report(e, err, err_len);
    }
}

int pfrt_outputs_count(const pfrt_outputs* o) { return o ? static_cast<int>(o->t.size()) : 0; }

int pfrt_outputs_get(const pfrt_outputs* o, int i, const void** data, size_t* bytes, int32_t* dtype, int32_t* ndim,
                     int64_t* dims8) {
    if (!o || i < 0 || i >= static_cast<int>(o->t.size())) return 1;
    const pyflame_rt::Tensor& t = o->t[static_cast<size_t>(i)];
    if (data) *data = t.data();
    if (bytes) *bytes = t.size_bytes();
    if (dtype) *dtype = static_cast<int32_t>(t.dtype());
    if (ndim) *ndim = static_cast<int32_t>(t.ndim());
    if (dims8)
        for (size_t k = 0; k < t.ndim() && k < 8; ++k) dims8[k] = t.shape()[k];
    return 0;
}

void pfrt_outputs_free(pfrt_outputs* o) { delete o; }

}  // extern "C"
