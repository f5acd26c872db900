// batcher.cpp -- cuda::DynamicBatcher (see batcher.hpp).
#include "batcher.hpp"

#include <algorithm>
#include <cstring>
#include <unordered_map>

#include "pyflame_rt/types.hpp"

namespace pyflame_rt {
namespace cuda {

// A worker's reused host buffers, one per graph input.
struct DynamicBatcher::Staging {
    std::unordered_map<std::string, std::vector<uint8_t>> bufs;
};

DynamicBatcher::DynamicBatcher(std::shared_ptr<const Graph> graph, std::vector<std::shared_ptr<Backend>> backends,
                               const BatchConfig& config)
    : graph_(std::move(graph)), backends_(std::move(backends)), config_(config),
      start_time_(std::chrono::steady_clock::now()) {
    if (!graph_) throw std::invalid_argument("DynamicBatcher: graph is null");
    if (backends_.empty()) throw std::invalid_argument("DynamicBatcher: at least one backend is required");
    for (const auto& b : backends_)
        if (!b) throw std::invalid_argument("DynamicBatcher: backend is null");
}

DynamicBatcher::~DynamicBatcher() {
    stop();
    // Requests that never ran (the batcher was not started) are answered.
    std::deque<Pending> left;
    {
        std::lock_guard<std::mutex> l(queue_mutex_);
        left.swap(queue_);
    }
    for (auto& p : left) {
        InferenceResponse r;
        r.request_id = p.request.id;
        r.success = false;
        r.error_message = "DynamicBatcher destroyed before the request ran";
        if (p.callback) {
            try {
                p.callback(std::move(r));
            } catch (...) {
            }
        } else {
            p.promise.set_value(std::move(r));
        }
    }
}

uint64_t DynamicBatcher::enqueue(InferenceRequest request, std::promise<InferenceResponse>* promise,
                                 std::function<void(InferenceResponse)> callback) {
    request.id = next_id_++;
    request.arrival_time = std::chrono::steady_clock::now();
    const uint64_t id = request.id;
    bool full = false;
    {
        std::lock_guard<std::mutex> l(queue_mutex_);
        full = config_.queue_capacity > 0 && queue_.size() >= config_.queue_capacity;
        if (!full) {
            Pending p;
            p.request = std::move(request);
            if (callback) p.callback = std::move(callback);
            else p.promise = std::move(*promise);
            queue_.push_back(std::move(p));
        }
    }
    if (full) {  // answered on the caller's thread, outside the queue lock
        InferenceResponse r;
        r.request_id = id;
        r.success = false;
        r.error_message = "Queue full";
        {
            std::lock_guard<std::mutex> s(stats_mutex_);
            stats_.dropped_requests++;
        }
        if (callback) callback(std::move(r));
        else promise->set_value(std::move(r));
        return id;
    }
    queue_cv_.notify_one();
    return id;
}

std::future<InferenceResponse> DynamicBatcher::submit(InferenceRequest request) {
    std::promise<InferenceResponse> p;
    auto f = p.get_future();
    enqueue(std::move(request), &p, nullptr);
    return f;
}

uint64_t DynamicBatcher::submit(InferenceRequest request, std::function<void(InferenceResponse)> callback) {
    if (!callback) throw std::invalid_argument("DynamicBatcher::submit: callback is empty");
    return enqueue(std::move(request), nullptr, std::move(callback));
}

std::vector<std::future<InferenceResponse>> DynamicBatcher::submit_batch(std::vector<InferenceRequest> requests) {
    std::vector<std::future<InferenceResponse>> out;
    out.reserve(requests.size());
    for (auto& r : requests) out.push_back(submit(std::move(r)));
    return out;
}

InferenceResponse DynamicBatcher::infer(InferenceRequest request) { return submit(std::move(request)).get(); }

void DynamicBatcher::start() {
    if (running_) return;
    running_ = true;
    {
        std::lock_guard<std::mutex> s(stats_mutex_);
        start_time_ = std::chrono::steady_clock::now();
    }
    cb_stop_ = false;
    cb_thread_ = std::thread(&DynamicBatcher::callback_loop, this);
    staging_.clear();
    for (size_t w = 0; w < backends_.size(); ++w) staging_.push_back(std::make_unique<Staging>());
    for (size_t w = 0; w < backends_.size(); ++w) workers_.emplace_back(&DynamicBatcher::worker_loop, this, w);
}

void DynamicBatcher::stop() {
    if (!running_) return;
    running_ = false;
    queue_cv_.notify_all();
    for (auto& t : workers_)
        if (t.joinable()) t.join();
    workers_.clear();
    {
        std::lock_guard<std::mutex> l(cb_mutex_);
        cb_stop_ = true;
    }
    cb_cv_.notify_all();
    if (cb_thread_.joinable()) cb_thread_.join();
}

void DynamicBatcher::flush() {
    {
        std::lock_guard<std::mutex> l(queue_mutex_);
        flush_ = true;
    }
    queue_cv_.notify_all();
}

size_t DynamicBatcher::queue_size() const {
    std::lock_guard<std::mutex> l(queue_mutex_);
    return queue_.size();
}

DynamicBatcher::Stats DynamicBatcher::get_stats() const {
    Stats s;
    double secs;
    {
        std::lock_guard<std::mutex> l(stats_mutex_);
        s = stats_;
        secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - start_time_).count();
    }
    s.queue_depth = queue_size();
    if (secs > 0) s.throughput_rps = static_cast<double>(s.total_requests) / secs;
    return s;
}

void DynamicBatcher::reset_stats() {
    std::lock_guard<std::mutex> l(stats_mutex_);
    stats_ = Stats{};
    start_time_ = std::chrono::steady_clock::now();
}

void DynamicBatcher::update_config(const BatchConfig& config) {
    std::lock_guard<std::mutex> l(queue_mutex_);
    config_ = config;
}

// The reference's rule (dynamic_batcher.cpp create_batch): wait until the
// queue holds max_batch_size requests, or at least min_batch_size, or until
// max_latency has passed (or a flush / stop), then take up to
// max_batch_size requests in arrival order.
std::vector<DynamicBatcher::Pending> DynamicBatcher::take_batch() {
    std::unique_lock<std::mutex> l(queue_mutex_);
    const auto deadline = std::chrono::steady_clock::now() + config_.max_latency;
    queue_cv_.wait_until(l, deadline, [&] {
        return !running_ || flush_ || queue_.size() >= config_.max_batch_size ||
               (!queue_.empty() && queue_.size() >= config_.min_batch_size);
    });
    std::vector<Pending> batch;
    const size_t cap = std::max<size_t>(1, config_.max_batch_size);
    while (!queue_.empty() && batch.size() < cap) {
        batch.push_back(std::move(queue_.front()));
        queue_.pop_front();
    }
    if (queue_.empty()) flush_ = false;
    return batch;
}

void DynamicBatcher::worker_loop(size_t w) {
    Backend& backend = *backends_[w];
    Staging& st = *staging_[w];
    while (running_) {
        auto b = take_batch();
        if (!b.empty()) process(b, backend, st);
    }
    for (;;) {  // drain what was queued before stop()
        auto b = take_batch();
        if (b.empty()) break;
        process(b, backend, st);
    }
}

void DynamicBatcher::deliver(Pending& p, InferenceResponse r) {
    if (p.callback) {
        {
            std::lock_guard<std::mutex> l(cb_mutex_);
            cb_queue_.emplace_back(std::move(p.callback), std::move(r));
        }
        cb_cv_.notify_one();
    } else {
        p.promise.set_value(std::move(r));
    }
}

void DynamicBatcher::callback_loop() {
    std::unique_lock<std::mutex> l(cb_mutex_);
    for (;;) {
        cb_cv_.wait(l, [&] { return cb_stop_ || !cb_queue_.empty(); });
        while (!cb_queue_.empty()) {
            auto item = std::move(cb_queue_.front());
            cb_queue_.pop_front();
            l.unlock();
            try {
                item.first(std::move(item.second));
            } catch (...) {
                // a callback's exception is its own
            }
            l.lock();
        }
        if (cb_stop_) return;
    }
}

void DynamicBatcher::process(std::vector<Pending>& batch, Backend& backend, Staging& st) {
    const auto t0 = std::chrono::steady_clock::now();
    const auto& infos = graph_->inputs();
    auto fail = [&](Pending& p, const std::string& msg) {
        InferenceResponse r;
        r.request_id = p.request.id;
        r.success = false;
        r.error_message = msg;
        r.latency = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() -
                                                                          p.request.arrival_time);
        deliver(p, std::move(r));
    };

    // The batch's per-input layout, from its first well-formed request:
    // dtype and the dimensions after the batch dimension.
    struct Spec {
        DType dtype = DType::Float32;
        std::vector<int64_t> rest;
        size_t row_bytes = 0;
    };
    std::vector<Spec> spec(infos.size());
    bool have_spec = false;
    std::vector<Pending*> ok;
    std::vector<int64_t> rows;
    for (auto& p : batch) {
        std::string why;
        int64_t m = -1;
        std::vector<Spec> mine(infos.size());
        for (size_t k = 0; k < infos.size() && why.empty(); ++k) {
            auto it = p.request.inputs.find(infos[k].name);
            if (it == p.request.inputs.end()) {
                why = "missing input '" + infos[k].name + "'";
                break;
            }
            const Tensor& t = it->second;
            if (t.ndim() < 1) {
                why = "input '" + infos[k].name + "' has no batch dimension";
                break;
            }
            if (m < 0) m = t.shape()[0];
            if (t.shape()[0] != m) {
                why = "inputs disagree on the batch dimension";
                break;
            }
            mine[k].dtype = t.dtype();
            mine[k].rest.assign(t.shape().begin() + 1, t.shape().end());
            int64_t per = 1;
            for (auto d : mine[k].rest) per *= d;
            mine[k].row_bytes = static_cast<size_t>(per) * dtype_size(t.dtype());
            // The graph's declaration: dtype, and every static dimension past the first.
            bool declared_ok = t.dtype() == infos[k].dtype && infos[k].shape.size() == t.ndim();
            for (size_t d = 1; declared_ok && d < infos[k].shape.size(); ++d)
                if (infos[k].shape[d].has_value() && *infos[k].shape[d] != t.shape()[d]) declared_ok = false;
            if (!declared_ok)
                why = "input '" + infos[k].name + "' does not match the graph input (dtype or shape past dimension 0)";
            else if (have_spec && (mine[k].dtype != spec[k].dtype || mine[k].rest != spec[k].rest))
                why = "input '" + infos[k].name + "' does not match the batch (dtype or shape past dimension 0)";
        }
        if (!why.empty()) {
            fail(p, "DynamicBatcher: request " + std::to_string(p.request.id) + ": " + why);
            continue;
        }
        if (!have_spec) {
            spec = mine;
            have_spec = true;
        }
        ok.push_back(&p);
        rows.push_back(std::max<int64_t>(m, 0));
    }
    if (ok.empty()) return;

    int64_t total = 0;
    for (auto r : rows) total += r;
    int64_t padded = total;
    if (config_.enable_padding) {
        std::vector<size_t> pref = config_.preferred_sizes;
        std::sort(pref.begin(), pref.end());
        for (size_t s : pref)
            if (static_cast<int64_t>(s) >= total) {
                padded = static_cast<int64_t>(s);
                break;
            }
    }

    // Inputs: each request's rows back to back in the worker's buffers,
    // then zero padding rows; the feeds are views of those buffers.
    std::unordered_map<std::string, Tensor> feeds;
    for (size_t k = 0; k < infos.size(); ++k) {
        auto& buf = st.bufs[infos[k].name];
        const size_t need = static_cast<size_t>(padded) * spec[k].row_bytes;
        if (buf.size() < std::max<size_t>(need, 1)) buf.resize(std::max<size_t>(need, 1));
        size_t off = 0;
        for (size_t i = 0; i < ok.size(); ++i) {
            const Tensor& t = ok[i]->request.inputs.at(infos[k].name);
            const size_t bytes = static_cast<size_t>(rows[i]) * spec[k].row_bytes;
            if (bytes) std::memcpy(buf.data() + off, t.data(), bytes);
            off += bytes;
        }
        if (need > off) std::memset(buf.data() + off, 0, need - off);
        std::vector<int64_t> shape{padded};
        shape.insert(shape.end(), spec[k].rest.begin(), spec[k].rest.end());
        feeds.emplace(infos[k].name, Tensor(buf.data(), shape, spec[k].dtype));
    }

    // Outputs: the union of what the requests asked for.
    std::vector<std::string> names;
    auto want = [&](const std::string& n) {
        if (std::find(names.begin(), names.end(), n) == names.end()) names.push_back(n);
    };
    for (Pending* p : ok) {
        if (p->request.output_names.empty())
            for (const auto& o : graph_->outputs()) want(o.name);
        for (const auto& n : p->request.output_names) want(n);
    }

    std::vector<Tensor> outs;
    try {
        outs = backend.execute(*graph_, feeds, names);
    } catch (const std::exception& e) {
        for (Pending* p : ok) fail(*p, e.what());
        return;
    }

    const auto t1 = std::chrono::steady_clock::now();
    int64_t off = 0;
    for (size_t i = 0; i < ok.size(); ++i) {
        Pending& p = *ok[i];
        InferenceResponse r;
        r.request_id = p.request.id;
        std::vector<std::string> mine = p.request.output_names;
        if (mine.empty())
            for (const auto& o : graph_->outputs()) mine.push_back(o.name);
        for (const auto& n : mine) {
            const size_t j = static_cast<size_t>(std::find(names.begin(), names.end(), n) - names.begin());
            const Tensor& t = outs[j];
            if (t.ndim() >= 1 && t.shape()[0] == padded) {
                // This request's rows of a batched output.
                std::vector<int64_t> shape = t.shape();
                shape[0] = rows[i];
                Tensor s(shape, t.dtype());
                const size_t row_bytes = padded ? t.size_bytes() / static_cast<size_t>(padded) : 0;
                if (s.size_bytes())
                    std::memcpy(s.data(), static_cast<const uint8_t*>(t.data()) + static_cast<size_t>(off) * row_bytes,
                                s.size_bytes());
                r.outputs.emplace(n, std::move(s));
            } else {
                r.outputs.emplace(n, t.clone());  // not batched along dimension 0: every request gets it
            }
        }
        off += rows[i];
        r.success = true;
        r.latency = std::chrono::duration_cast<std::chrono::microseconds>(t1 - p.request.arrival_time);
        deliver(p, std::move(r));
    }

    {
        std::lock_guard<std::mutex> l(stats_mutex_);
        stats_.total_requests += ok.size();
        stats_.total_batches++;
        stats_.avg_batch_size = static_cast<double>(stats_.total_requests) / static_cast<double>(stats_.total_batches);
        const double lat = std::chrono::duration<double, std::micro>(t1 - t0).count();
        stats_.avg_latency_us = stats_.total_batches == 1 ? lat : stats_.avg_latency_us * 0.9 + lat * 0.1;
    }
}

}  // namespace cuda
}  // namespace pyflame_rt
