// nfx_copy_pool.h -- host threads that split a large memcpy between them.
//
// The host-buffer Run stages pageable caller buffers through pinned memory (the copy
// engines need page-locked memory to run asynchronously); one thread copies at about
// 18 GB/s, below PCIe, so the staging copies are split over a small pool (8 threads
// reach about 67 GB/s on the GPU hosts).  A Run issues several copies in quick
// succession, so a worker spins for up to kSpinNs after each task before it sleeps:
// waking a sleeping thread costs tens of microseconds per copy.
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace nfx {

class CopyPool {
public:
    static constexpr long long kSpinNs = 1000000;

    explicit CopyPool(int workers) {
        for (int i = 0; i < workers; ++i) threads_.emplace_back([this, i] { loop(i); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_.store(true);
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }
    CopyPool(const CopyPool&) = delete;
    CopyPool& operator=(const CopyPool&) = delete;

    // memcpy(dst, src, bytes) split into (workers + 1) parts, the calling thread taking
    // one; returns when all parts are done.  One copy at a time per pool.
    void copy(void* dst, const void* src, size_t bytes) {
        const int parts = static_cast<int>(threads_.size()) + 1;
        if (bytes < (size_t{1} << 20) || parts == 1) {
            std::memcpy(dst, src, bytes);
            return;
        }
        dst_ = static_cast<char*>(dst);
        src_ = static_cast<const char*>(src);
        bytes_ = bytes;
        per_ = ((bytes / parts + 4095) / 4096) * 4096;   // 4 KiB-aligned part boundaries
        pending_.store(static_cast<int>(threads_.size()), std::memory_order_relaxed);
        {
            std::lock_guard<std::mutex> lk(mu_);
            gen_.fetch_add(1, std::memory_order_release);
        }
        cv_.notify_all();
        part(0);
        while (pending_.load(std::memory_order_acquire) != 0) spin_pause();
    }

private:
    static void spin_pause() {
#if defined(__x86_64__) || defined(__i386__)
        __builtin_ia32_pause();
#endif
    }
    void part(int i) const {
        const size_t b0 = per_ * static_cast<size_t>(i);
        if (b0 >= bytes_) return;
        const size_t n = bytes_ - b0 < per_ ? bytes_ - b0 : per_;
        std::memcpy(dst_ + b0, src_ + b0, n);
    }
    void loop(int i) {
        unsigned long long seen = 0;
        for (;;) {
            // spin a while for the next task, then sleep
            const auto t0 = std::chrono::steady_clock::now();
            bool got = false;
            for (int k = 0; !got; ++k) {
                if (stop_.load(std::memory_order_relaxed)) return;
                got = gen_.load(std::memory_order_acquire) != seen;
                if (!got && (k & 255) == 255 &&
                    std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0)
                            .count() > kSpinNs)
                    break;
                if (!got) spin_pause();
            }
            if (!got) {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_.load() || gen_.load(std::memory_order_acquire) != seen; });
                if (stop_.load()) return;
            }
            seen = gen_.load(std::memory_order_acquire);
            part(i + 1);
            pending_.fetch_sub(1, std::memory_order_acq_rel);
        }
    }

    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::atomic<bool> stop_{false};
    std::atomic<unsigned long long> gen_{0};
    std::atomic<int> pending_{0};
    char* dst_ = nullptr;
    const char* src_ = nullptr;
    size_t bytes_ = 0, per_ = 0;
};

}  // namespace nfx
