// Host-side helpers of the matmul service's host-buffer calls (host_copy.cpp).
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace zest {

// A fixed set of worker threads; run() splits [0, n) into pieces of at least
// min_piece, which the workers and the calling thread take in turn, and
// returns when every piece is done. One run at a time per pool.
class host_pool {
public:
    explicit host_pool(int threads);
    ~host_pool();
    void run(int64_t n, int64_t min_piece, const std::function<void(int64_t, int64_t)> &fn);
    int threads() const { return (int) workers_.size() + 1; }

private:
    struct job {
        const std::function<void(int64_t, int64_t)> *fn = nullptr;
        std::atomic<int64_t> *next = nullptr;
        int64_t n = 0, step = 0, pieces = 0;
    };
    static int64_t drain(const job &j);
    void work();

    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable wake_, idle_;
    job cur_;
    std::atomic<int64_t> next_{ 0 };  // the next piece of the current job
    uint64_t gen_ = 0;
    int64_t finished_ = 0;
    int busy_ = 0;  // workers holding the current job
    bool stop_ = false;
};

// dst[i] = the f32 whose high 16 bits are src[i] and low 16 bits zero: a
// bf16 value widened exactly.
void widen_bf16(const uint16_t *src, float *dst, int64_t n);

}  // namespace zest
