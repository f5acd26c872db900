// batcher.hpp -- the batching caller: single requests assembled into large-M
// batches for the GPU backends.
//
// Mirrors the reference's DynamicBatcher (include/pyflame_rt/batching/
// dynamic_batcher.hpp, src/batching/dynamic_batcher.cpp): the same
// BatchConfig, InferenceRequest and InferenceResponse types and the same
// calls (submit with a future or a callback, submit_batch, infer, start,
// stop, flush, queue_size, stats, update_config), the same queueing rule
// (a batch closes when it holds max_batch_size requests, or as soon as it
// holds min_batch_size, or after max_latency) and "Queue full" rejection.
// It runs a graph on one or more Backends instead of an InferenceSession:
// one worker per backend takes whole batches, so with one CudaBackend per
// GPU the batches of a request stream run on all GPUs at once (the
// batch-sharded data-parallel path, no collective).
//
// Differences from the reference, each a fix:
//   - requests may carry several rows: inputs are concatenated along
//     dimension 0 (the reference copies one row's worth per request) and
//     outputs split back by each request's row count;
//   - futures are fulfilled (the reference drops the promises);
//   - preferred_sizes and padding count rows; padding rows are zero and their
//     outputs dropped;
//   - a request whose inputs do not match the batch (missing input, other
//     dtype or trailing shape) fails alone with an error response;
//   - a request's output_names select its outputs (empty = the graph's).
// Each worker assembles batches in its own reused host buffers (no
// per-batch allocation or zero fill of the payload).
#pragma once

#include <condition_variable>
#include <deque>
#include <functional>
#include <future>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "pyflame_rt/backend.hpp"
#include "pyflame_rt/batching/dynamic_batcher.hpp"
#include "pyflame_rt/graph.hpp"

namespace pyflame_rt {
namespace cuda {

using batching::BatchConfig;
using batching::InferenceRequest;
using batching::InferenceResponse;

class DynamicBatcher {
public:
    using Stats = batching::DynamicBatcher::Stats;

    /// Requests run `graph` on `backends` (one worker each; e.g. one
    /// CudaBackend per GPU).  BatchConfig::num_workers is not used: the
    /// workers are the backends.
    DynamicBatcher(std::shared_ptr<const Graph> graph, std::vector<std::shared_ptr<Backend>> backends,
                   const BatchConfig& config = BatchConfig());
    ~DynamicBatcher();

    DynamicBatcher(const DynamicBatcher&) = delete;
    DynamicBatcher& operator=(const DynamicBatcher&) = delete;

    std::future<InferenceResponse> submit(InferenceRequest request);
    uint64_t submit(InferenceRequest request, std::function<void(InferenceResponse)> callback);
    std::vector<std::future<InferenceResponse>> submit_batch(std::vector<InferenceRequest> requests);
    InferenceResponse infer(InferenceRequest request);

    void start();
    /// Stops after every queued request has been answered.
    void stop();
    bool is_running() const { return running_; }
    void flush();
    size_t queue_size() const;

    Stats get_stats() const;
    void reset_stats();
    const BatchConfig& config() const { return config_; }
    void update_config(const BatchConfig& config);

private:
    struct Pending {
        InferenceRequest request;
        std::promise<InferenceResponse> promise;
        std::function<void(InferenceResponse)> callback;
    };
    struct Staging;

    std::vector<Pending> take_batch();
    void worker_loop(size_t w);
    void process(std::vector<Pending>& batch, Backend& backend, Staging& st);
    void deliver(Pending& p, InferenceResponse r);
    void callback_loop();
    uint64_t enqueue(InferenceRequest request, std::promise<InferenceResponse>* promise,
                     std::function<void(InferenceResponse)> callback);

    std::shared_ptr<const Graph> graph_;
    std::vector<std::shared_ptr<Backend>> backends_;
    BatchConfig config_;
    std::atomic<bool> running_{false};
    std::atomic<uint64_t> next_id_{0};

    mutable std::mutex queue_mutex_;
    std::condition_variable queue_cv_;
    std::deque<Pending> queue_;
    bool flush_ = false;

    std::mutex cb_mutex_;
    std::condition_variable cb_cv_;
    std::deque<std::pair<std::function<void(InferenceResponse)>, InferenceResponse>> cb_queue_;
    bool cb_stop_ = false;

    std::vector<std::thread> workers_;
    std::vector<std::unique_ptr<Staging>> staging_;
    std::thread cb_thread_;

    mutable std::mutex stats_mutex_;
    Stats stats_;
    std::chrono::steady_clock::time_point start_time_;
};

}  // namespace cuda
}  // namespace pyflame_rt
