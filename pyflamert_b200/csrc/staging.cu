// staging.cu -- copies between pageable host memory and the device through a
// ring of pinned buffers owned by the context.
//
// A host Tensor of the reference runtime lives in ordinary (pageable) memory
// (tensor.cpp allocates it), so every graph input and output crosses the
// host link from pageable memory.  CUDA's own pageable path copies through a
// driver buffer on one thread; here the context keeps kSlots pinned chunks of
// kChunk bytes, the host side of each chunk is copied by a small pool of
// threads (the caller plus kWorkers), and the DMA of one chunk runs while the
// next chunk is copied on the host.  One event per slot says when its DMA is
// done, so a slot is reused only after that.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.hpp"

namespace pfrt {

namespace {

// memcpy of one buffer split over the caller and `workers` threads (3 by
// default; PFRT_COPY_WORKERS overrides, 0 copies on the caller alone).  A
// copy is handed over through atomics, and a worker that has just finished
// one keeps polling for the next for up to `spin` (100 us by default;
// PFRT_COPY_SPIN_US overrides) before it sleeps on the condition variable:
// the chunks of one transfer follow each other within microseconds, and a
// futex wake-up per chunk would cost more than the copy of a 256 KiB chunk.
// Idle workers sleep.
int env_or(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

class CopyPool {
public:
    CopyPool()
        : workers_(std::max(0, std::min(env_or("PFRT_COPY_WORKERS", 3), 15))),
          spin_ns_(static_cast<int64_t>(std::max(0, env_or("PFRT_COPY_SPIN_US", 100))) * 1000) {
        for (int i = 0; i < workers_; ++i) threads_.emplace_back([this, i] { work(i); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> l(m_);
            stop_.store(true);
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }

    void copy(void* dst, const void* src, size_t n) {
        constexpr size_t kMinSplit = 128 * 1024;
        if (n < kMinSplit || workers_ == 0) {
            std::memcpy(dst, src, n);
            return;
        }
        const size_t part = (n / (workers_ + 1) + 63) & ~size_t{63};
        dst_ = static_cast<char*>(dst);
        src_ = static_cast<const char*>(src);
        n_ = n;
        part_ = part;
        pending_.store(workers_, std::memory_order_relaxed);
        {
            // The release publishes the job to polling workers; the lock
            // orders it against a worker that is about to sleep.
            std::lock_guard<std::mutex> l(m_);
            gen_.fetch_add(1, std::memory_order_release);
        }
        if (sleepers_.load(std::memory_order_acquire) > 0) cv_.notify_all();
        std::memcpy(dst, src, std::min(part, n));  // the caller's share: part 0
        while (pending_.load(std::memory_order_acquire) != 0) {
        }
    }

private:
    void work(int i) {
        uint64_t seen = 0;
        for (;;) {
            uint64_t g = gen_.load(std::memory_order_acquire);
            if (g == seen) {
                const auto t0 = std::chrono::steady_clock::now();
                while ((g = gen_.load(std::memory_order_acquire)) == seen && !stop_.load() &&
                       std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0)
                               .count() < spin_ns_) {
                }
                if (g == seen) {
                    std::unique_lock<std::mutex> l(m_);
                    sleepers_.fetch_add(1);
                    cv_.wait(l, [&] { return stop_.load() || gen_.load(std::memory_order_acquire) != seen; });
                    sleepers_.fetch_sub(1);
                    if (stop_.load()) return;
                    g = gen_.load(std::memory_order_acquire);
                }
            }
            if (stop_.load()) return;
            seen = g;
            const size_t n = n_, part = part_;
            const size_t lo = std::min(n, part * static_cast<size_t>(i + 1));
            const size_t hi = (i == workers_ - 1) ? n : std::min(n, part * static_cast<size_t>(i + 2));
            if (hi > lo) std::memcpy(dst_ + lo, src_ + lo, hi - lo);
            pending_.fetch_sub(1, std::memory_order_release);
        }
    }

    const int workers_;
    const int64_t spin_ns_;
    std::vector<std::thread> threads_;
    std::mutex m_;
    std::condition_variable cv_;
    std::atomic<bool> stop_{false};
    std::atomic<uint64_t> gen_{0};
    std::atomic<int> pending_{0};
    std::atomic<int> sleepers_{0};
    char* dst_ = nullptr;
    const char* src_ = nullptr;
    size_t n_ = 0, part_ = 0;
};

}  // namespace

struct StagingRing {
    // 256 KiB chunks: small enough that the host copy of one chunk and the
    // DMA of the previous one overlap within a 1-2 MiB tensor, large enough
    // that each DMA runs at the link's rate.
    static constexpr int kSlots = 8;
    static constexpr size_t kChunk = size_t{256} << 10;
    void* buf[kSlots] = {};
    cudaEvent_t ev[kSlots] = {};
    bool used[kSlots] = {};
    int next = 0;
    CopyPool pool;
};

void staging_release(pfrt_ctx* ctx) {
    StagingRing* r = ctx->staging;
    if (!r) return;
    for (int i = 0; i < StagingRing::kSlots; ++i) {
        if (r->ev[i]) {
            cudaEventSynchronize(r->ev[i]);
            cudaEventDestroy(r->ev[i]);
        }
        if (r->buf[i]) cudaFreeHost(r->buf[i]);
    }
    delete r;
    ctx->staging = nullptr;
}

namespace {

pfrt_status ring(pfrt_ctx* ctx, StagingRing** out) {
    if (!ctx->staging) {
        auto* r = new StagingRing();
        cudaError_t e = cudaSuccess;
        for (int i = 0; i < StagingRing::kSlots && e == cudaSuccess; ++i) {
            e = cudaMallocHost(&r->buf[i], StagingRing::kChunk);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->ev[i], cudaEventDisableTiming);
        }
        ctx->staging = r;
        if (e != cudaSuccess) {
            staging_release(ctx);
            return cuda_fail(e, "pinned staging buffers");
        }
    }
    *out = ctx->staging;
    return PFRT_OK;
}

// The next slot, once the DMA that last used it has completed.
pfrt_status take_slot(StagingRing* r, int* slot) {
    const int s = r->next;
    r->next = (s + 1) % StagingRing::kSlots;
    if (r->used[s]) {
        PFRT_CUDA_TRY(cudaEventSynchronize(r->ev[s]));
        r->used[s] = false;
    }
    *slot = s;
    return PFRT_OK;
}

}  // namespace
}  // namespace pfrt

using namespace pfrt;

extern "C" {

pfrt_status pfrt_memcpy_h2d_staged(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (bytes == 0) return PFRT_OK;
    if (!dst || !src) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_memcpy_h2d_staged: null pointer");
    StagingRing* r = nullptr;
    st = ring(ctx, &r);
    if (st) return st;
    cudaStream_t s = pick_stream(ctx, stream);
    for (size_t off = 0; off < bytes; off += StagingRing::kChunk) {
        const size_t n = std::min(StagingRing::kChunk, bytes - off);
        int slot = 0;
        st = take_slot(r, &slot);
        if (st) return st;
        r->pool.copy(r->buf[slot], static_cast<const char*>(src) + off, n);
        PFRT_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(dst) + off, r->buf[slot], n, cudaMemcpyHostToDevice, s));
        PFRT_CUDA_TRY(cudaEventRecord(r->ev[slot], s));
        r->used[slot] = true;
    }
    return PFRT_OK;
}

pfrt_status pfrt_memcpy_d2h_staged(pfrt_ctx* ctx, void* dst, const void* src, size_t bytes, pfrt_stream stream) {
    pfrt_status st = enter(ctx);
    if (st) return st;
    if (bytes == 0) return PFRT_OK;
    if (!dst || !src) return fail(PFRT_ERR_INVALID_ARGUMENT, "pfrt_memcpy_d2h_staged: null pointer");
    StagingRing* r = nullptr;
    st = ring(ctx, &r);
    if (st) return st;
    cudaStream_t s = pick_stream(ctx, stream);
    const size_t C = StagingRing::kChunk;
    const size_t nch = (bytes + C - 1) / C;
    std::vector<int> slot_of(nch, 0);
    auto issue = [&](size_t i) -> pfrt_status {
        pfrt_status e = take_slot(r, &slot_of[i]);
        if (e) return e;
        const int sl = slot_of[i];
        const size_t n = std::min(C, bytes - i * C);
        PFRT_CUDA_TRY(cudaMemcpyAsync(r->buf[sl], static_cast<const char*>(src) + i * C, n, cudaMemcpyDeviceToHost, s));
        PFRT_CUDA_TRY(cudaEventRecord(r->ev[sl], s));
        r->used[sl] = true;
        return PFRT_OK;
    };
    for (size_t i = 0; i < std::min<size_t>(nch, StagingRing::kSlots); ++i) {
        st = issue(i);
        if (st) return st;
    }
    for (size_t i = 0; i < nch; ++i) {
        const int sl = slot_of[i];
        PFRT_CUDA_TRY(cudaEventSynchronize(r->ev[sl]));
        r->used[sl] = false;
        r->pool.copy(static_cast<char*>(dst) + i * C, r->buf[sl], std::min(C, bytes - i * C));
        if (i + StagingRing::kSlots < nch) {
            st = issue(i + StagingRing::kSlots);
            if (st) return st;
        }
    }
    return PFRT_OK;
}

}  // extern "C"
