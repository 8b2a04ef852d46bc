// Stress test of the matmul service's host thread pool (csrc/host_copy.cpp):
// many short jobs in a row, workers woken late by random sleeps, every
// piece of every job run exactly once. Built and run by
// tests/test_host_pool.py; exits 0 on success. TEST CODE.
#include "host_copy.h"

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

int main() {
    using namespace zest;
    std::mt19937 rng(7);
    for (int threads : { 2, 3, 8, 17 }) {
        host_pool pool(threads);
        for (int job = 0; job < 3000; job++) {
            const int64_t n = 1 + (int64_t) (rng() % 4096);
            const int64_t min_piece = 1 + (int64_t) (rng() % 64);
            std::vector<std::atomic<int>> hits((size_t) n);
            for (auto &h : hits) h = 0;
            const int delay = (int) (rng() % 4);
            pool.run(n, min_piece, [&](int64_t lo, int64_t hi) {
                if (delay == 0 && ((lo / min_piece) % 7) == 3) std::this_thread::sleep_for(std::chrono::microseconds(50));
                for (int64_t i = lo; i < hi; i++) hits[(size_t) i]++;
            });
            for (int64_t i = 0; i < n; i++)
                if (hits[(size_t) i] != 1) {
                    fprintf(stderr, "threads %d job %d: element %lld run %d times\n", threads, job, (long long) i,
                            (int) hits[(size_t) i]);
                    return 1;
                }
        }
    }
    // widening: the f32 with the bf16's bits on top, at every alignment
    std::vector<uint16_t> src(1000);
    for (size_t i = 0; i < src.size(); i++) src[i] = (uint16_t) (i * 2654435761u >> 16);
    std::vector<float> dst(1100);
    for (int off = 0; off < 9; off++) {
        widen_bf16(src.data(), dst.data() + off, (int64_t) src.size() - off);
        for (size_t i = 0; i + off < src.size(); i++) {
            uint32_t u;
            memcpy(&u, &dst[i + off], 4);
            if (u != (uint32_t) src[i] << 16) {
                fprintf(stderr, "widen: offset %d element %zu\n", off, i);
                return 1;
            }
        }
    }
    printf("POOL OK\n");
    return 0;
}
