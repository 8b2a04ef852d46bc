// zest_mul_mat_noalloc: the activation pack + GEMM path with its one piece
// of scratch memory (the bf16 copy of the activations) in a fixed device
// array instead of memory from cudaMalloc.
//
// Some callers cannot allocate device memory on this path: a host program
// whose GPU memory is planned and owned by its own allocator (ggml's graph
// allocator, for one, lays out every byte of a compute piece ahead of time),
// and latency-sensitive callers for which cudaMalloc / cudaFree, which may
// synchronise the whole device, are not acceptable in the middle of a
// prompt. They still pass their own inputs and outputs; only the scratch
// moves here.
#include "zest_b200.h"
#include "zest_device.cuh"
#include "zest_internal.h"

#include <mutex>

namespace zest {

// The scratch: room for ZEST_NOALLOC_MAX_VALUES bf16 values (32 MiB). Every
// GPU that loads this library holds it until the process exits. All calls
// share it and it keeps the last call's contents.
static __device__ __align__(256) uint16_t g_act_scratch[ZEST_NOALLOC_MAX_VALUES];

// A __device__ array's name means nothing to host code (using it there as a
// pointer would fault, or silently address host memory), so its device
// address is looked up once per device, with that device current.
static std::mutex g_scratch_mu;
static uint16_t *g_scratch_addr[64];

static uint16_t *scratch_for_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        set_error("zest_mul_mat_noalloc: no current CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_act_scratch);
        if (e != cudaSuccess || !p) {
            set_error("zest_mul_mat_noalloc: cannot find the scratch array on this device");
            return nullptr;
        }
        g_scratch_addr[dev] = static_cast<uint16_t *>(p);
    }
    return g_scratch_addr[dev];
}

}  // namespace zest

using namespace zest;

extern "C" int zest_mul_mat_noalloc(const float *x, int64_t T, int64_t K, int64_t ldx, const uint16_t *w_bf16,
                                    int64_t ldw, int64_t N, int mode, float *y, int64_t ldy, unsigned *err,
                                    void *stream) {
    if (T <= 0 || N <= 0) return 0;
    const int64_t m_pad = (T + TILE_M - 1) / TILE_M * TILE_M;
    if (K <= 0 || m_pad > ZEST_NOALLOC_MAX_VALUES / K)
        return set_error("zest_mul_mat_noalloc: roundup(T, 128) * K exceeds ZEST_NOALLOC_MAX_VALUES (16777216); "
                         "split the rows into smaller calls or use zest_mul_mat");
    uint16_t *a = scratch_for_current_device();
    if (!a) return -1;
    cudaStream_t st = (cudaStream_t) stream;
    // every row in [0, m_pad) is written (rows past T as zeros), so nothing
    // left by an earlier call is read
    if (launch_pack_activations(x, T, K, ldx, m_pad, nullptr, a, K, st)) return -1;
    return launch_gemm(a, K, w_bf16, ldw, T, N, K, mode, y, ldy, 0, err, st);
}
