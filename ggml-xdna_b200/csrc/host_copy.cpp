// Host-side helpers of the matmul service's host-buffer calls: a fixed pool
// of worker threads, and the widening of bf16 results to f32.
//
// A result the GEMM has rounded to bf16 (the default output mode, and
// SwiGLU) crosses PCIe as its 16 high bits, half the bytes of its f32 form;
// widening puts them back as the same f32 bits. PCIe, not the kernels,
// bounds a host-buffer call, so this halves the copy out.
#include "host_copy.h"

#include <immintrin.h>

#include <algorithm>
#include <cstring>

namespace zest {

host_pool::host_pool(int threads) {
    for (int i = 1; i < threads; i++) workers_.emplace_back([this] { work(); });
}

host_pool::~host_pool() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        stop_ = true;
    }
    wake_.notify_all();
    for (auto &t : workers_) t.join();
}

// Takes pieces of the current job until none is left; returns how many it ran.
int64_t host_pool::drain(const job &j) {
    int64_t done = 0;
    for (;;) {
        const int64_t i = j.next->fetch_add(1);
        if (i >= j.pieces) return done;
        const int64_t lo = i * j.step, hi = std::min(j.n, lo + j.step);
        (*j.fn)(lo, hi);
        done++;
    }
}

void host_pool::work() {
    uint64_t seen = 0;
    for (;;) {
        job j;
        {
            std::unique_lock<std::mutex> lk(mu_);
            wake_.wait(lk, [&] { return stop_ || gen_ != seen; });
            if (stop_) return;
            seen = gen_;
            j = cur_;
            busy_++;  // run() does not return while a worker holds its job
        }
        const int64_t done = drain(j);
        {
            std::lock_guard<std::mutex> lk(mu_);
            finished_ += done;
            busy_--;
        }
        idle_.notify_all();
    }
}

void host_pool::run(int64_t n, int64_t min_piece, const std::function<void(int64_t, int64_t)> &fn) {
    if (n <= 0) return;
    const int64_t lanes = (int64_t) workers_.size() + 1;
    const int64_t step = std::max<int64_t>(min_piece, (n + 4 * lanes - 1) / (4 * lanes));
    const int64_t pieces = (n + step - 1) / step;
    if (pieces == 1 || workers_.empty()) {
        fn(0, n);
        return;
    }
    job j{ &fn, &next_, n, step, pieces };
    {
        // A worker that woke late for the last job may still hold it; the
        // piece counter is shared, so it must let go before the counter
        // starts again for this job (else it could take one of this job's
        // pieces and drop it as out of its own range).
        std::unique_lock<std::mutex> lk(mu_);
        idle_.wait(lk, [&] { return busy_ == 0; });
        next_ = 0;
        cur_ = j;
        finished_ = 0;
        gen_++;
    }
    wake_.notify_all();
    const int64_t mine = drain(j);
    std::unique_lock<std::mutex> lk(mu_);
    finished_ += mine;
    idle_.wait(lk, [&] { return finished_ == pieces && busy_ == 0; });
}

namespace {

void widen_scalar(const uint16_t *src, float *dst, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        const uint32_t u = (uint32_t) src[i] << 16;
        memcpy(dst + i, &u, 4);
    }
}

// Eight values at a time; streaming stores where the destination is 32-byte
// aligned, so the f32 rows are not read into the cache first.
__attribute__((target("avx2"))) void widen_avx2(const uint16_t *src, float *dst, int64_t n) {
    int64_t i = 0;
    while (i < n && ((uintptr_t) (dst + i) & 31)) {
        const uint32_t u = (uint32_t) src[i] << 16;
        memcpy(dst + i, &u, 4);
        i++;
    }
    for (; i + 8 <= n; i += 8) {
        const __m128i h = _mm_loadu_si128(reinterpret_cast<const __m128i *>(src + i));
        const __m256i w = _mm256_slli_epi32(_mm256_cvtepu16_epi32(h), 16);
        _mm256_stream_si256(reinterpret_cast<__m256i *>(dst + i), w);
    }
    _mm_sfence();
    widen_scalar(src + i, dst + i, n - i);
}

}  // namespace

void widen_bf16(const uint16_t *src, float *dst, int64_t n) {
    static const bool avx2 = __builtin_cpu_supports("avx2");
    if (avx2) widen_avx2(src, dst, n);
    else widen_scalar(src, dst, n);
}

}  // namespace zest
