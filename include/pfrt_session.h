/*
 * pfrt_session.h -- C entry points of PyFlameRT's InferenceSession with the
 * CUDA backend plugged in, for hosts that cannot call C++ (ctypes, cgo, JNI).
 *
 * libpfrt_session.so is the reference's own session layer (InferenceSession,
 * SessionOptions, the .pfm loader, Graph/Node/Tensor; src/session.cpp,
 * src/options.cpp, src/io/*.cpp, src/tensor.cpp, ...) compiled from a
 * PyFlameRT checkout with the CUDA seam applied (SessionOptions.device
 * "cuda", "cuda:<n>" or "cuda:<n>,<m>,..." selects pyflame_rt::CudaBackend),
 * plus these functions.  Each returns 0 on success; on failure it returns a
 * non-zero code and writes the exception's message into err (err_len bytes,
 * NUL-terminated, may be NULL).
 */
#ifndef PFRT_SESSION_H
#define PFRT_SESSION_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PFRT_SESSION_API __attribute__((visibility("default")))
#else
#define PFRT_SESSION_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct pfrt_session pfrt_session;
typedef struct pfrt_outputs pfrt_outputs;

/* InferenceSession(model_path, options) with options.device = device
 * (src/session.cpp:27-56) and optimization_level None (the graph runs as
 * saved).  Loads the .pfm file with the reference's loader. */
PFRT_SESSION_API int pfrt_session_open(const char* pfm_path, const char* device, pfrt_session** out,
                                       char* err, size_t err_len);
PFRT_SESSION_API void pfrt_session_close(pfrt_session* s);

/* InferenceSession::run(output_names, input_feed) (src/session.cpp:97-120).
 * Input i is `names[i]`, dtype `dtypes[i]` (pyflame_rt::DType values:
 * 0 float32, 7 int8, 8 uint8, ...), `ndims[i]` dimensions taken in order
 * from `dims`, and `data[i]` in host memory (read, not copied, while the call
 * runs).  n_out = 0 asks for all graph outputs.  The returned outputs own
 * their host memory until pfrt_outputs_free. */
PFRT_SESSION_API int pfrt_session_run(pfrt_session* s, int n_in, const char* const* names,
                                      const void* const* data, const int32_t* dtypes, const int32_t* ndims,
                                      const int64_t* dims, int n_out, const char* const* out_names,
                                      pfrt_outputs** out, char* err, size_t err_len);
PFRT_SESSION_API int pfrt_outputs_count(const pfrt_outputs* o);
/* Output i: host data pointer, byte size, dtype and up to 8 dims (ndim set). */
PFRT_SESSION_API int pfrt_outputs_get(const pfrt_outputs* o, int i, const void** data, size_t* bytes,
                                      int32_t* dtype, int32_t* ndim, int64_t* dims8);
PFRT_SESSION_API void pfrt_outputs_free(pfrt_outputs* o);

#ifdef __cplusplus
}
#endif

#endif /* PFRT_SESSION_H */
