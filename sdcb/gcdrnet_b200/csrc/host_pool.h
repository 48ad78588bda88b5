// host_pool.h -- a small persistent pool of host threads for a worker's staging copies.
//
// run(n, f) executes f(0) .. f(n-1) on the helper threads and the calling thread and
// returns when all n have finished.  One caller at a time (a worker serves one call at a
// time).  Tasks are claimed by compare-and-swap on a ticket that carries the round number,
// so a helper that wakes late for a finished round can never take a task of the next one
// (whose function object it does not hold).
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace gcdr {

class HostPool {
public:
    // helpers: threads besides the caller; device: made current in each helper (the tasks
    // issue copies on the worker's stream and wait on its events)
    HostPool(int helpers, int device) : device_(device) {
        for (int i = 0; i < helpers; i++) threads_.emplace_back([this] { loop(); });
    }
    ~HostPool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
        }
        wake_.notify_all();
        for (auto &t : threads_) t.join();
    }
    HostPool(const HostPool &) = delete;
    HostPool &operator=(const HostPool &) = delete;

    void run(int n, const std::function<void(int)> &f) {
        if (n <= 0) return;
        uint64_t round;
        {
            std::lock_guard<std::mutex> g(mu_);
            round = ++round_;
            job_ = &f;
            n_ = n;
            left_ = n;
            ticket_.store(round << 32);
        }
        wake_.notify_all();
        work(round, &f, n);
        std::unique_lock<std::mutex> l(mu_);
        done_.wait(l, [&] { return left_ == 0; });
        job_ = nullptr;
    }

private:
    void loop() {
        cudaSetDevice(device_);
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(int)> *job;
            int n;
            uint64_t round;
            {
                std::unique_lock<std::mutex> l(mu_);
                wake_.wait(l, [&] { return stop_ || round_ != seen; });
                if (stop_) return;
                seen = round = round_;
                job = job_;
                n = n_;
            }
            if (job) work(round, job, n);
        }
    }

    void work(uint64_t round, const std::function<void(int)> *job, int n) {
        for (;;) {
            uint64_t t = ticket_.load();
            if ((t >> 32) != round || (int)(t & 0xffffffffu) >= n) return;
            if (!ticket_.compare_exchange_weak(t, t + 1)) continue;
            (*job)((int)(t & 0xffffffffu));
            std::lock_guard<std::mutex> g(mu_);
            if (--left_ == 0) done_.notify_all();
        }
    }

    int device_;
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable wake_, done_;
    const std::function<void(int)> *job_ = nullptr;
    std::atomic<uint64_t> ticket_{0};
    uint64_t round_ = 0;
    int n_ = 0, left_ = 0;
    bool stop_ = false;
};

}  // namespace gcdr
