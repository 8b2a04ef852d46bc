// The C ABI of libzest_b200.so (include/zest_b200.h): the stream-level
// kernel entry points and the matmul service zest_npu, the counterpart of
// the reference's xdna_npu (src/xdna-npu.{h,cpp}).
#include "host_copy.h"
#include "zest_b200.h"
#include "zest_device.cuh"
#include "zest_internal.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

namespace zest {

static thread_local std::string g_err;

int set_error(const char *msg) {
    g_err = msg;
    return -1;
}

int check_launch(const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) return 0;
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return -1;
}

// The IQ3_S codebook, kept on the host so every device that converts IQ3_S
// weights gets a copy (a __device__ symbol exists once per device).
static std::mutex g_grid_mu;
static std::vector<uint32_t> g_grid_host;
static uint64_t g_grid_devices = 0;  // bit d: loaded on device d

bool iq3s_grid_loaded() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(g_grid_mu);
    if (dev < 64 && (g_grid_devices >> dev) & 1) return true;
    if (g_grid_host.empty()) return false;
    if (set_iq3s_grid(g_grid_host.data())) return false;
    if (dev < 64) g_grid_devices |= 1ull << dev;
    return true;
}

// Environment knobs read once; empty means unset (src/xdna-env.h:9-17).
static long long env_ll(const char *name, long long def) {
    const char *s = getenv(name);
    return s && *s ? atoll(s) : def;
}

// Flags every result non-finite: the fault-injection counterpart of the
// NPU's damaged results (GGML_XDNA_NAN_AFTER, src/xdna-npu.cpp:102-112).
__global__ void check_finite_kernel(const float *y, int64_t n, unsigned *err) {
    uint32_t bad = 0;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        bad |= (__float_as_uint(y[i]) & 0x7f800000u) == 0x7f800000u;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x % 32) == 0) atomicOr(err, ERR_NOT_FINITE);
}

// The high 16 bits of n floats that hold bf16 values (the low bits zero):
// the values themselves, in half the bytes, for the copy to the host.
__global__ void narrow_bf16_kernel(const float *__restrict__ y, int64_t n, uint16_t *__restrict__ out) {
    const int64_t stride = (int64_t) gridDim.x * blockDim.x;
    const int64_t n4 = n / 4;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n4; i += stride) {
        const uint4 v = reinterpret_cast<const uint4 *>(y)[i];
        reinterpret_cast<uint2 *>(out)[i] = make_uint2((v.x >> 16) | (v.y & 0xffff0000u), (v.z >> 16) | (v.w & 0xffff0000u));
    }
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = (uint16_t) (__float_as_uint(y[i]) >> 16);
}

}  // namespace zest

using namespace zest;

extern "C" {

int zest_version(void) { return ZEST_B200_VERSION; }

const char *zest_last_error(void) { return g_err.c_str(); }

int zest_load_iq3s_grid(const uint32_t *grid512) {
    if (!grid512) return set_error("zest_load_iq3s_grid: no table");
    std::lock_guard<std::mutex> lk(g_grid_mu);
    g_grid_host.assign(grid512, grid512 + 512);
    g_grid_devices = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_error("zest_load_iq3s_grid: no CUDA device");
    if (set_iq3s_grid(grid512)) return -1;
    if (dev < 64) g_grid_devices |= 1ull << dev;
    return 0;
}

int zest_pack_activations(const float *x, int64_t T, int64_t K, int64_t ldx, int64_t m_pad, uint8_t *a_bfp16,
                          uint16_t *a_bf16, int64_t ld_bf16, void *stream) {
    return launch_pack_activations(x, T, K, ldx, m_pad, a_bfp16, a_bf16, ld_bf16, (cudaStream_t) stream);
}

int zest_convert_weight(int type, const void *raw, int64_t rows_total, int64_t row0, int64_t N, int64_t K,
                        int64_t n_pad, uint8_t *b_bfp16, uint16_t *b_bf16, void *stream) {
    if (row0 < 0 || N < 0 || row0 + N > rows_total) return set_error("zest_convert_weight: rows out of range");
    return launch_convert_weight(type, raw, raw, 0, N, row0, rows_total, K, n_pad, b_bfp16, b_bf16,
                                 (cudaStream_t) stream);
}

int zest_convert_gate_up(int type, const void *gate, const void *up, int64_t rows_total, int64_t row0, int64_t F,
                         int64_t K, int64_t f_pad, uint8_t *b_bfp16, uint16_t *b_bf16, void *stream) {
    if (row0 < 0 || F < 0 || row0 + F > rows_total || f_pad % 256 || f_pad < F)
        return set_error("zest_convert_gate_up: rows out of range or f_pad not a multiple of 256");
    return launch_convert_weight(type, gate, up, 1, F, row0, rows_total, K, 2 * f_pad, b_bfp16, b_bf16,
                                 (cudaStream_t) stream);
}

int zest_gemm(const uint16_t *a_bf16, int64_t lda, const uint16_t *b_bf16, int64_t ldb, int64_t M, int64_t N,
              int64_t K, int mode, float *c, int64_t ldc, unsigned *err, void *stream) {
    return launch_gemm(a_bf16, lda, b_bf16, ldb, M, N, K, mode, c, ldc, 0, err, (cudaStream_t) stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// the matmul service
// ---------------------------------------------------------------------------

// One call's device and host buffers and events. Slot 0 serves the
// synchronous calls; slots 1..ZEST_SLOTS the calls zest_submit_group starts
// and zest_wait_group finishes, several of which may be in flight at once
// (their copies in, kernels and copies out queue on the service's three
// streams in submission order, so one call's copy in overlaps another's copy
// out).
struct call_slot {
    static constexpr int MAX_CHUNKS = 16;
    float *x_dev = nullptr, *y_dev = nullptr;
    size_t x_cap = 0, y_cap = 0;
    // bf16-rounded results cross PCIe as bf16 (y16_dev -> pinned y16_host)
    // and host threads widen them into the caller's f32
    uint16_t *y16_dev = nullptr, *y16_host = nullptr;
    size_t y16_cap = 0, y16_host_cap = 0;
    unsigned *err_dev = nullptr, *err_host = nullptr;
    cudaEvent_t start = nullptr, k_done = nullptr, o_done = nullptr;
    cudaEvent_t in_ev[MAX_CHUNKS] = {}, done_ev[MAX_CHUNKS] = {};  // ordering only
    cudaEvent_t copied_ev[MAX_CHUNKS] = {};                          // a chunk's results are in host memory
    cudaEvent_t t_pack[MAX_CHUNKS] = {}, t_gemm[MAX_CHUNKS] = {}, t_end[MAX_CHUNKS] = {};
    // the call in flight, from its submission until it is finished
    bool busy = false, on_device = false;
    int n = 0, nch = 0;
    int64_t T = 0, rows = 0;
    int64_t n_out[4] = {};
    float *y[4] = {};
    bool w16[4] = {};
    size_t y16_off[4] = {};

    cudaError_t create() {
        cudaError_t e = cudaSuccess;
        for (cudaEvent_t *ev : { &start, &k_done, &o_done })
            if (e == cudaSuccess) e = cudaEventCreate(ev);
        for (int c = 0; c < MAX_CHUNKS && e == cudaSuccess; c++) {
            e = cudaEventCreateWithFlags(&in_ev[c], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done_ev[c], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&copied_ev[c], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreate(&t_pack[c]);
            if (e == cudaSuccess) e = cudaEventCreate(&t_gemm[c]);
            if (e == cudaSuccess) e = cudaEventCreate(&t_end[c]);
        }
        if (e == cudaSuccess) e = cudaMalloc(&err_dev, sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMallocHost(&err_host, sizeof(unsigned));
        return e;
    }
    void destroy() {
        cudaFree(x_dev);
        cudaFree(y_dev);
        cudaFree(y16_dev);
        if (y16_host) cudaFreeHost(y16_host);
        cudaFree(err_dev);
        if (err_host) cudaFreeHost(err_host);
        for (cudaEvent_t e : { start, k_done, o_done })
            if (e) cudaEventDestroy(e);
        for (int c = 0; c < MAX_CHUNKS; c++)
            for (cudaEvent_t e : { in_ev[c], done_ev[c], copied_ev[c], t_pack[c], t_gemm[c], t_end[c] })
                if (e) cudaEventDestroy(e);
    }
};

struct zest_npu {
    struct weight {
        uint8_t *bytes = nullptr;   // bfp16 B operand, reference layout
        uint16_t *bf16 = nullptr;   // [n_pad][K]
        int64_t K = 0, N = 0, n_pad = 0, n_out = 0;
        int mode = 0;
        cudaEvent_t ready = nullptr;  // built on the load stream: recorded after its conversion
    };
    using key_t = std::tuple<const void *, const void *, int, int64_t, int64_t, int>;

    // a host-buffer call is cut into at most MAX_CHUNKS row chunks whose input
    // copies (st_in), kernels (st) and output copies (st_out) overlap
    static constexpr int MAX_CHUNKS = call_slot::MAX_CHUNKS;
    int device = 0;
    cudaStream_t st = nullptr, st_in = nullptr, st_out = nullptr;
    // weight copies from device-resident raw bytes are built on st_load
    // without the host waiting, when async_load is on (zest_set_load_async)
    cudaStream_t st_load = nullptr;
    bool async_load = false;
    bool out16 = true;
    std::map<key_t, weight> weights;
    // the packed input, shared by every call: its writers and readers all run
    // on st, in order; grows only
    uint16_t *a_bf16 = nullptr;
    size_t a_cap = 0;
    // per-call buffers and events: slot 0 for the synchronous calls, the
    // others for zest_submit_group / zest_wait_group
    call_slot slots[1 + ZEST_SLOTS];
    std::unique_ptr<host_pool> pool;
    cudaEvent_t ev[2] = {};  // weight-copy timing
    zest_times times = {};
    // whether GGML_XDNA_FAIL_AFTER / _NAN_AFTER apply: not to the start-up
    // self-test, which the reference runs outside its injection points too
    bool inject = true;

    ~zest_npu() {
        cudaSetDevice(device);
        if (st) cudaStreamSynchronize(st);
        if (st_in) cudaStreamSynchronize(st_in);
        if (st_out) cudaStreamSynchronize(st_out);
        if (st_load) cudaStreamSynchronize(st_load);
        for (auto &kv : weights) {
            cudaFree(kv.second.bytes);
            cudaFree(kv.second.bf16);
            if (kv.second.ready) cudaEventDestroy(kv.second.ready);
        }
        cudaFree(a_bf16);
        for (call_slot &cs : slots) cs.destroy();
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        if (st) cudaStreamDestroy(st);
        if (st_in) cudaStreamDestroy(st_in);
        if (st_out) cudaStreamDestroy(st_out);
        if (st_load) cudaStreamDestroy(st_load);
    }

    static key_t key_of(const zest_wkey *k, int fused) { return key_t(k->buffer, k->data, k->type, k->K, k->N, fused); }

    const weight *find(const zest_wkey *k, int fused) const {
        auto it = weights.find(key_of(k, fused));
        return it == weights.end() ? nullptr : &it->second;
    }
};

namespace zest {

static bool grow(void **p, size_t *cap, size_t need) {
    if (need <= *cap) return true;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, need) != cudaSuccess) return false;
    *cap = need;
    return true;
}

static bool grow_pinned(void **p, size_t *cap, size_t need) {
    if (need <= *cap) return true;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMallocHost(p, need) != cudaSuccess) return false;
    *cap = need;
    return true;
}

// Host threads for widening results, GGML_ZEST_HOST_THREADS (default: the
// machine's, at most 32).
static int host_threads() {
    static const int n = [] {
        const long long v = env_ll("GGML_ZEST_HOST_THREADS", 0);
        if (v > 0) return (int) v;
        const unsigned hc = std::thread::hardware_concurrency();
        return (int) std::min<unsigned>(32, hc ? hc : 8);
    }();
    return n;
}

// Whether a host-buffer call sends this weight's results as bf16: they hold
// bf16 values exactly (the bf16 output mode, and SwiGLU's), unless
// GGML_ZEST_WIRE16=0.
static bool wire16(int mode) {
    static const bool on = env_ll("GGML_ZEST_WIRE16", 1) != 0;
    return on && (mode == MODE_BF16 || mode == MODE_SWIGLU);
}

// GGML_XDNA_FAIL_AFTER=n: every submission after the n-th fails, to test the
// caller's failure path (src/xdna-npu.cpp:89-100).
static bool injected_failure() {
    static const long long after = env_ll("GGML_XDNA_FAIL_AFTER", -1);
    static std::atomic<long long> n{ 0 };
    return after >= 0 && ++n > after;
}

// GGML_XDNA_NAN_AFTER=n: every result after the n-th submission comes back
// NaN, to test that such results are caught (src/xdna-npu.cpp:102-112).
static bool injected_nan() {
    static const long long after = env_ll("GGML_XDNA_NAN_AFTER", -1);
    static std::atomic<long long> n{ 0 };
    return after >= 0 && ++n > after;
}

// Rows per chunk of a host-buffer call: whole below 2048 rows, else about a
// sixteenth of the call (at least 512 rows) so the first copy in and the last
// copy out, which nothing hides, stay short; GGML_ZEST_CHUNK_ROWS overrides.
// PCIe, not the kernels, bounds such a call: a B200's Gen5 x16 link moves
// about 55 GB/s one way and 96 GB/s both ways at once.
static int64_t chunk_rows(int64_t T) {
    static const long long force = env_ll("GGML_ZEST_CHUNK_ROWS", 0);
    int64_t rows = force > 0 ? force : (T < 2048 ? T : std::max<int64_t>(512, T / 16));
    rows = std::max<int64_t>(rows, (T + zest_npu::MAX_CHUNKS - 1) / zest_npu::MAX_CHUNKS);
    return (rows + TILE_M - 1) / TILE_M * TILE_M;
}

static int cuda_fail(const char *what, cudaError_t e) {
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return -1;
}

// A weight copy from raw rows of type `ctype` (the key's own type, or F32
// for values the caller dequantised), keyed by `key`.
static int add_copy(zest_npu *npu, const zest_wkey *key, const void *raw0, const void *raw1, int raw_on_device,
                    int fused, int ctype) {
    if (!npu || !key) return set_error("zest_add_weight: no service or key");
    if (cudaSetDevice(npu->device) != cudaSuccess) return set_error("zest_add_weight: cannot select the device");
    const int64_t K = key->K, N = key->N;
    int64_t row_bytes = 0;
    switch (ctype) {
        case TYPE_F32: row_bytes = K * 4; break;
        case TYPE_F16: row_bytes = K * 2; break;
        case TYPE_Q8_0: row_bytes = K / 32 * 34; break;
        case TYPE_Q4_K: row_bytes = K / 256 * 144; break;
        case TYPE_Q6_K: row_bytes = K / 256 * 210; break;
        case TYPE_IQ3_S: row_bytes = K / 256 * 110; break;
        default: return set_error("zest_add_weight: unsupported weight type");
    }
    zest_npu::weight w;
    w.K = K;
    w.N = N;
    w.n_out = N;
    w.n_pad = fused ? 2 * ((N + 255) / 256 * 256) : (N + 511) / 512 * 512;  // pad_f / pad_n (xdna-npu.cpp:46-47)
    w.mode = fused ? MODE_SWIGLU : (npu->out16 ? MODE_BF16 : MODE_F32);
    const size_t raw_bytes = (size_t) (row_bytes * N);
    if (npu->async_load && raw_on_device) {
        // built on the load stream; the first call that uses the copy waits
        // for its event on the GPU, not the host (the reference's background
        // copy builder, src/ggml-zest.cpp:261-330)
        cudaError_t e = cudaMalloc(&w.bytes, (size_t) (w.n_pad * K / 8 * BLOCK_BYTES));
        if (e == cudaSuccess) e = cudaMalloc(&w.bf16, (size_t) (w.n_pad * K) * 2);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&w.ready, cudaEventDisableTiming);
        int rc = e == cudaSuccess ? 0 : cuda_fail("zest_add_weight: allocating the weight copy", e);
        if (!rc)
            rc = launch_convert_weight(ctype, raw0, fused ? raw1 : raw0, fused, N, 0, N, K, w.n_pad, w.bytes, w.bf16,
                                       npu->st_load);
        if (!rc && (e = cudaEventRecord(w.ready, npu->st_load)) != cudaSuccess) rc = cuda_fail("zest_add_weight", e);
        if (rc) {
            cudaFree(w.bytes);
            cudaFree(w.bf16);
            if (w.ready) cudaEventDestroy(w.ready);
            return rc;
        }
        auto k = zest_npu::key_of(key, fused);
        auto old = npu->weights.find(k);
        if (old != npu->weights.end()) {
            // an older copy under the same key may still be read by queued work
            cudaDeviceSynchronize();
            cudaFree(old->second.bytes);
            cudaFree(old->second.bf16);
            if (old->second.ready) cudaEventDestroy(old->second.ready);
        }
        npu->weights[k] = w;
        return 0;
    }
    const void *src0 = raw0, *src1 = raw1;
    void *staged[2] = { nullptr, nullptr };
    cudaEvent_t t0 = npu->ev[0], t1 = npu->ev[1];
    cudaEventRecord(t0, npu->st);
    if (!raw_on_device) {
        for (int i = 0; i < (fused ? 2 : 1); i++) {
            cudaError_t e = cudaMalloc(&staged[i], raw_bytes ? raw_bytes : 16);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(staged[i], i ? raw1 : raw0, raw_bytes, cudaMemcpyHostToDevice, npu->st);
            if (e != cudaSuccess) {
                cudaFree(staged[0]);
                cudaFree(staged[1]);
                return cuda_fail("zest_add_weight: staging the raw weight", e);
            }
        }
        src0 = staged[0];
        src1 = staged[1];
    }
    cudaError_t e = cudaMalloc(&w.bytes, (size_t) (w.n_pad * K / 8 * BLOCK_BYTES));
    if (e == cudaSuccess) e = cudaMalloc(&w.bf16, (size_t) (w.n_pad * K) * 2);
    int rc = e == cudaSuccess ? 0 : cuda_fail("zest_add_weight: allocating the weight copy", e);
    if (!rc)
        rc = fused ? launch_convert_weight(ctype, src0, src1, 1, N, 0, N, K, w.n_pad, w.bytes, w.bf16, npu->st)
                   : launch_convert_weight(ctype, src0, src0, 0, N, 0, N, K, w.n_pad, w.bytes, w.bf16, npu->st);
    cudaEventRecord(t1, npu->st);
    e = cudaStreamSynchronize(npu->st);
    if (!rc && e != cudaSuccess) rc = cuda_fail("zest_add_weight", e);
    cudaFree(staged[0]);
    cudaFree(staged[1]);
    if (rc) {
        cudaFree(w.bytes);
        cudaFree(w.bf16);
        return rc;
    }
    float ms = 0;
    cudaEventElapsedTime(&ms, t0, t1);
    npu->times.pack_ms += ms;
    auto k = zest_npu::key_of(key, fused);
    auto old = npu->weights.find(k);
    if (old != npu->weights.end()) {
        cudaDeviceSynchronize();
        cudaFree(old->second.bytes);
        cudaFree(old->second.bf16);
        if (old->second.ready) cudaEventDestroy(old->second.ready);
    }
    npu->weights[k] = w;
    return 0;
}

// One exact integer multiply through all three kernels, checked against the
// host (npu_self_test, src/xdna-npu.cpp:136-184): small whole numbers that
// bfp16 holds exactly and fp32 sums add exactly, so every answer must match.
static std::string self_test(int device) {
    constexpr int64_t M = 512, K = 128, N = 512;
    std::vector<int8_t> ai((size_t) (M * K)), wi((size_t) (N * K));
    uint32_t seed = 1;
    auto next = [&](int span) {
        seed = seed * 1664525u + 1013904223u;
        return (int8_t) ((int) (seed >> 24) % span - span / 2);
    };
    for (int8_t &v : ai) v = next(5);
    for (int8_t &v : wi) v = next(7);
    std::vector<float> a(ai.begin(), ai.end()), w(wi.begin(), wi.end()), c((size_t) (M * N));
    zest_npu *npu = zest_open(device);
    if (!npu) return std::string("cannot open the GPU (") + g_err + ")";
    zest_set_out16(npu, 0);
    npu->inject = false;
    const zest_wkey key = { nullptr, w.data(), TYPE_F32, K, N };
    std::string why;
    if (zest_add_weight(npu, &key, w.data(), 0) || zest_mul_mat(npu, &key, 0, a.data(), M, c.data(), 0)) {
        why = "a test multiply failed (" + g_err + ")";
    } else {
        for (int64_t r = 0; r < M && why.empty(); r++)
            for (int64_t n = 0; n < N; n++) {
                int want = 0;
                for (int64_t k = 0; k < K; k++) want += ai[r * K + k] * wi[n * K + k];
                if (c[r * N + n] != (float) want) {
                    char where[128];
                    snprintf(where, sizeof(where), "a test multiply came out wrong (row %lld, column %lld: %g, not %d)",
                             (long long) r, (long long) n, c[r * N + n], want);
                    why = where;
                    break;
                }
            }
    }
    zest_close(npu);
    return why;
}

// Queues one group call in `cs`: up to 4 weights sharing the input x.
// Device buffers: one pass. Host buffers: row chunks (multiples of the
// 128-row tile) whose copies in (st_in), kernels (st) and copies out (st_out)
// overlap one another, and the copies of the calls in other slots.
static int submit_call(zest_npu *npu, call_slot &cs, int n, const zest_wkey *keys, const int *fused, const float *x,
                       int64_t T, float *const *y, int on_device, const char *what) {
    if (!keys || n <= 0 || n > 4) return set_error((std::string(what) + ": not 1 to 4 weights").c_str());
    const zest_npu::weight *w[4];
    for (int i = 0; i < n; i++) {
        w[i] = npu->find(&keys[i], fused ? fused[i] : 0);
        if (!w[i]) return set_error((std::string(what) + ": weight not added").c_str());
        if (w[i]->K != w[0]->K) return set_error((std::string(what) + ": a group's weights differ in K").c_str());
    }
    cs.n = 0;
    cs.nch = 0;
    if (T <= 0) {
        cs.busy = true;  // nothing to do; the wait returns at once
        return 0;
    }
    if (cudaSetDevice(npu->device) != cudaSuccess) return set_error((std::string(what) + ": cannot select the device").c_str());
    if (npu->inject && injected_failure()) return set_error("an injected failure (GGML_XDNA_FAIL_AFTER)");
    cudaStream_t st = npu->st;
    for (int i = 0; i < n; i++)
        if (w[i]->ready) cudaStreamWaitEvent(st, w[i]->ready, 0);  // its copy is built (load stream)
    const int64_t K = w[0]->K, m_pad = (T + TILE_M - 1) / TILE_M * TILE_M;
    const size_t x_bytes = (size_t) (T * K) * 4;
    size_t y_off[4], y_total = 0;
    for (int i = 0; i < n; i++) {
        y_off[i] = y_total;
        y_total += (size_t) (T * w[i]->n_out) * 4;
    }
    // (a buffer that must grow is freed first, which waits for the device)
    if (!grow((void **) &npu->a_bf16, &npu->a_cap, (size_t) (m_pad * K) * 2) ||
        (!on_device && (!grow((void **) &cs.x_dev, &cs.x_cap, x_bytes) || !grow((void **) &cs.y_dev, &cs.y_cap, y_total))))
        return set_error((std::string(what) + ": out of GPU memory for the call's buffers").c_str());
    const float *xd = on_device ? x : cs.x_dev;
    float *yd[4];
    for (int i = 0; i < n; i++) yd[i] = on_device ? y[i] : (float *) ((char *) cs.y_dev + y_off[i]);
    const bool nan = npu->inject && injected_nan();
    const int64_t rows = on_device ? T : chunk_rows(T);
    const int nch = (int) ((T + rows - 1) / rows);
    // Host buffers: results that hold bf16 values cross PCIe as bf16 and are
    // widened on the host, chunk by chunk as their copies land.
    size_t y16_total = 0;
    for (int i = 0; i < n; i++) {
        cs.w16[i] = !on_device && wire16(w[i]->mode);
        if (cs.w16[i]) {
            cs.y16_off[i] = y16_total;
            y16_total += (size_t) (T * w[i]->n_out);
        }
    }
    if (y16_total) {
        if (!grow((void **) &cs.y16_dev, &cs.y16_cap, y16_total * 2) ||
            !grow_pinned((void **) &cs.y16_host, &cs.y16_host_cap, y16_total * 2))
            return set_error((std::string(what) + ": out of memory for the bf16 copies of the results").c_str());
        if (!npu->pool) npu->pool.reset(new host_pool(host_threads()));
    }
    cudaEventRecord(cs.start, st);
    cudaMemsetAsync(cs.err_dev, 0, sizeof(unsigned), st);
    int rc = 0;
    for (int c = 0; c < nch && !rc; c++) {
        const int64_t r0 = c * rows, m = std::min(rows, T - r0);
        if (!on_device) {
            cudaMemcpyAsync(cs.x_dev + r0 * K, x + r0 * K, (size_t) (m * K) * 4, cudaMemcpyHostToDevice, npu->st_in);
            cudaEventRecord(cs.in_ev[c], npu->st_in);
            cudaStreamWaitEvent(st, cs.in_ev[c], 0);
        }
        cudaEventRecord(cs.t_pack[c], st);
        rc = launch_pack_activations(xd + r0 * K, m, K, K, (m + TILE_M - 1) / TILE_M * TILE_M, nullptr,
                                     npu->a_bf16 + r0 * K, K, st);
        cudaEventRecord(cs.t_gemm[c], st);
        gemm_seg segs[4];
        for (int i = 0; i < n; i++)
            segs[i] = { w[i]->bf16, K, w[i]->n_pad, w[i]->n_out, w[i]->n_out, w[i]->mode, yd[i] + r0 * w[i]->n_out };
        if (!rc) rc = launch_gemm_group(npu->a_bf16 + r0 * K, K, m, K, n, segs, cs.err_dev, st);
        if (!rc && nan) {
            for (int i = 0; i < n; i++) {
                cudaMemsetAsync(segs[i].c, 0xff, (size_t) (m * w[i]->n_out) * 4, st);
                check_finite_kernel<<<148, 256, 0, st>>>(segs[i].c, m * w[i]->n_out, cs.err_dev);
            }
        }
        if (!rc)
            for (int i = 0; i < n; i++)
                if (cs.w16[i])
                    narrow_bf16_kernel<<<148, 256, 0, st>>>(segs[i].c, m * w[i]->n_out,
                                                             cs.y16_dev + cs.y16_off[i] + r0 * w[i]->n_out);
        cudaEventRecord(cs.t_end[c], st);
        if (!on_device) {
            cudaEventRecord(cs.done_ev[c], st);
            cudaStreamWaitEvent(npu->st_out, cs.done_ev[c], 0);
            for (int i = 0; i < n; i++) {
                const size_t at = cs.y16_off[i] + (size_t) (r0 * w[i]->n_out), cnt = (size_t) (m * w[i]->n_out);
                if (cs.w16[i])
                    cudaMemcpyAsync(cs.y16_host + at, cs.y16_dev + at, cnt * 2, cudaMemcpyDeviceToHost, npu->st_out);
                else
                    cudaMemcpyAsync(y[i] + r0 * w[i]->n_out, segs[i].c, cnt * 4, cudaMemcpyDeviceToHost, npu->st_out);
            }
            cudaEventRecord(cs.copied_ev[c], npu->st_out);
        }
    }
    cudaMemcpyAsync(cs.err_host, cs.err_dev, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
    cudaEventRecord(cs.k_done, st);
    cudaEventRecord(cs.o_done, on_device ? st : npu->st_out);
    if (rc) {
        cudaStreamSynchronize(st);
        cudaStreamSynchronize(npu->st_in);
        cudaStreamSynchronize(npu->st_out);
        return rc;
    }
    cs.busy = true;
    cs.on_device = on_device != 0;
    cs.n = n;
    cs.nch = nch;
    cs.T = T;
    cs.rows = rows;
    for (int i = 0; i < n; i++) {
        cs.n_out[i] = w[i]->n_out;
        cs.y[i] = y[i];
    }
    return 0;
}

// Finishes the call queued in `cs`: widens its bf16 results into the
// caller's f32 rows as each chunk's copy lands, waits for its kernels and
// copies, and reads its error word. The call's results are then in y.
static int finish_call(zest_npu *npu, call_slot &cs, const char *what) {
    cs.busy = false;
    if (cs.n == 0) return 0;
    if (cudaSetDevice(npu->device) != cudaSuccess) return set_error((std::string(what) + ": cannot select the device").c_str());
    int rc = 0;
    bool any16 = false;
    for (int i = 0; i < cs.n; i++) any16 = any16 || cs.w16[i];
    for (int c = 0; c < cs.nch && any16 && !rc; c++) {
        const cudaError_t ce = cudaEventSynchronize(cs.copied_ev[c]);
        if (ce != cudaSuccess) {
            rc = cuda_fail(what, ce);
            break;
        }
        const int64_t r0 = c * cs.rows, m = std::min(cs.rows, cs.T - r0);
        for (int i = 0; i < cs.n; i++) {
            if (!cs.w16[i]) continue;
            const uint16_t *src = cs.y16_host + cs.y16_off[i] + r0 * cs.n_out[i];
            float *dst = cs.y[i] + r0 * cs.n_out[i];
            npu->pool->run(m * cs.n_out[i], 1 << 16,
                           [src, dst](int64_t lo, int64_t hi) { widen_bf16(src + lo, dst + lo, hi - lo); });
        }
    }
    cudaError_t e = cudaEventSynchronize(cs.k_done);
    if (e == cudaSuccess) e = cudaEventSynchronize(cs.o_done);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail(what, e);
    float total = 0, busy = 0;
    cudaEventElapsedTime(&total, cs.start, cs.o_done);
    for (int c = 0; c < cs.nch; c++) {
        float a = 0, b = 0;
        cudaEventElapsedTime(&a, cs.t_pack[c], cs.t_gemm[c]);
        cudaEventElapsedTime(&b, cs.t_gemm[c], cs.t_end[c]);
        npu->times.encode_ms += a;
        npu->times.gemm_ms += b;
        busy += a + b;
    }
    npu->times.copy_ms += std::max(0.0f, total - busy);  // the copies the kernels did not hide
    npu->times.calls += cs.n;
    if (*cs.err_host & ERR_TIMEOUT) return set_error("a GPU kernel's bounded wait ran out");
    if (*cs.err_host & ERR_NOT_FINITE) return set_error("the GPU's results held NaN or infinity");
    return 0;
}

}  // namespace zest

extern "C" {

zest_npu *zest_open(int device) {
    if (cudaSetDevice(device) != cudaSuccess) {
        set_error("zest_open: no such CUDA device");
        return nullptr;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0) {
        set_error("zest_open: this build runs on sm_100 (B200) only");
        return nullptr;
    }
    auto *npu = new zest_npu;
    npu->device = device;
    npu->out16 = env_ll("GGML_XDNA_OUT16", 1) != 0;
    cudaError_t e = cudaStreamCreateWithFlags(&npu->st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&npu->st_in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&npu->st_out, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&npu->st_load, cudaStreamNonBlocking);
    for (cudaEvent_t &ev : npu->ev)
        if (e == cudaSuccess) e = cudaEventCreate(&ev);
    for (call_slot &cs : npu->slots)
        if (e == cudaSuccess) e = cs.create();
    if (e != cudaSuccess) {
        cuda_fail("zest_open", e);
        delete npu;
        return nullptr;
    }
    return npu;
}

void zest_close(zest_npu *npu) { delete npu; }

void zest_set_out16(zest_npu *npu, int on) {
    if (npu) npu->out16 = on != 0;
}

int zest_usable(int device, char *why, size_t why_len) {
    static std::mutex mu;
    static std::map<int, std::string> verdict;  // "" = usable
    std::string v;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = verdict.find(device);
        if (it == verdict.end()) it = verdict.emplace(device, self_test(device)).first;
        v = it->second;
    }
    const std::string said = v.empty() ? "B200 self-test multiply right" : v;
    if (why && why_len) snprintf(why, why_len, "%s", said.c_str());
    if (!v.empty()) return set_error(v.c_str());
    return 0;
}

int zest_has_weight(const zest_npu *npu, const zest_wkey *key) {
    return npu && key && (npu->find(key, 0) || npu->find(key, 1)) ? 1 : 0;
}

int zest_add_weight(zest_npu *npu, const zest_wkey *key, const void *raw, int raw_on_device) {
    return add_copy(npu, key, raw, raw, raw_on_device, 0, key ? key->type : -1);
}

int zest_add_weight_values(zest_npu *npu, const zest_wkey *key, const float *values, int on_device) {
    return add_copy(npu, key, values, values, on_device, 0, TYPE_F32);
}

int zest_add_fused(zest_npu *npu, const zest_wkey *gate, const void *gate_raw, const void *up_raw, int raw_on_device) {
    return add_copy(npu, gate, gate_raw, up_raw, raw_on_device, 1, gate ? gate->type : -1);
}

int64_t zest_out_width(const zest_npu *npu, const zest_wkey *key, int fused) {
    const zest_npu::weight *w = npu && key ? npu->find(key, fused) : nullptr;
    return w ? w->n_out : -1;
}

const uint8_t *zest_weight_bfp16(const zest_npu *npu, const zest_wkey *key, int fused) {
    const zest_npu::weight *w = npu && key ? npu->find(key, fused) : nullptr;
    if (w && w->ready) cudaEventSynchronize(w->ready);  // a copy still being built on the load stream
    return w ? w->bytes : nullptr;
}

const uint16_t *zest_weight_bf16(const zest_npu *npu, const zest_wkey *key, int fused, int64_t *n_pad) {
    const zest_npu::weight *w = npu && key ? npu->find(key, fused) : nullptr;
    if (w && w->ready) cudaEventSynchronize(w->ready);
    if (w && n_pad) *n_pad = w->n_pad;
    return w ? w->bf16 : nullptr;
}

void zest_set_load_async(zest_npu *npu, int on) {
    if (npu) npu->async_load = on != 0;
}

int zest_wait_weights(zest_npu *npu) {
    if (!npu) return set_error("zest_wait_weights: no service");
    if (cudaSetDevice(npu->device) != cudaSuccess) return set_error("zest_wait_weights: cannot select the device");
    const cudaError_t e = cudaStreamSynchronize(npu->st_load);
    return e == cudaSuccess ? 0 : cuda_fail("zest_wait_weights", e);
}

void *zest_stream(zest_npu *npu) { return npu ? (void *) npu->st : nullptr; }

int zest_mul_mat_group(zest_npu *npu, int n, const zest_wkey *keys, const int *fused, const float *x, int64_t T,
                       float *const *y, int on_device) {
    if (!npu) return set_error("zest_mul_mat: no service, or not 1 to 4 weights");
    int rc = submit_call(npu, npu->slots[0], n, keys, fused, x, T, y, on_device, "zest_mul_mat");
    return rc ? rc : finish_call(npu, npu->slots[0], "zest_mul_mat");
}

int zest_submit_group(zest_npu *npu, int slot, int n, const zest_wkey *keys, const int *fused, const float *x,
                      int64_t T, float *const *y, int on_device) {
    if (!npu) return set_error("zest_submit_group: no service");
    if (slot < 0 || slot >= ZEST_SLOTS) return set_error("zest_submit_group: no such slot");
    call_slot &cs = npu->slots[1 + slot];
    if (cs.busy) return set_error("zest_submit_group: the slot's last call is not finished (zest_wait_group)");
    return submit_call(npu, cs, n, keys, fused, x, T, y, on_device, "zest_submit_group");
}

int zest_wait_group(zest_npu *npu, int slot) {
    if (!npu) return set_error("zest_wait_group: no service");
    if (slot < 0 || slot >= ZEST_SLOTS) return set_error("zest_wait_group: no such slot");
    call_slot &cs = npu->slots[1 + slot];
    if (!cs.busy) return set_error("zest_wait_group: nothing submitted in the slot");
    return finish_call(npu, cs, "zest_wait_group");
}

int zest_mul_mat_group_ex(zest_npu *npu, int n, const zest_wkey *keys, const int *fused, const float *x,
                          float norm_eps, const float *norm_w, float *x_normed, const uint16_t *a_bf16, int64_t T,
                          const zest_mm_out *outs) {
    if (!npu || !keys || !outs || n <= 0 || n > 4) return set_error("zest_mul_mat_group_ex: no service, or not 1 to 4 weights");
    const zest_npu::weight *w[4];
    for (int i = 0; i < n; i++) {
        w[i] = npu->find(&keys[i], fused ? fused[i] : 0);
        if (!w[i]) return set_error("zest_mul_mat_group_ex: weight not added");
        if (w[i]->K != w[0]->K) return set_error("zest_mul_mat_group_ex: a group's weights differ in K");
    }
    if (!a_bf16 && !x) return set_error("zest_mul_mat_group_ex: no input");
    if (T <= 0) return 0;
    if (cudaSetDevice(npu->device) != cudaSuccess) return set_error("zest_mul_mat_group_ex: cannot select the device");
    if (npu->inject && injected_failure()) return set_error("an injected failure (GGML_XDNA_FAIL_AFTER)");
    for (int i = 0; i < n; i++)
        if (w[i]->ready) cudaStreamWaitEvent(npu->st, w[i]->ready, 0);  // its copy is built (load stream)
    const int64_t K = w[0]->K, m_pad = (T + TILE_M - 1) / TILE_M * TILE_M;
    cudaStream_t st = npu->st;
    call_slot &cs = npu->slots[0];
    const bool nan = npu->inject && injected_nan();
    cudaEventRecord(cs.t_pack[0], st);
    cudaMemsetAsync(cs.err_dev, 0, sizeof(unsigned), st);
    int rc = 0;
    const uint16_t *a = a_bf16;
    if (!a) {
        if (!grow((void **) &npu->a_bf16, &npu->a_cap, (size_t) (m_pad * K) * 2))
            return set_error("zest_mul_mat_group_ex: out of GPU memory for the packed input");
        rc = norm_eps >= 0.0f ? zest_pack_rms_norm(x, T, K, K, norm_eps, norm_w, x_normed, K, m_pad, npu->a_bf16, K, st)
                              : launch_pack_activations(x, T, K, K, m_pad, nullptr, npu->a_bf16, K, st);
        a = npu->a_bf16;
    }
    cudaEventRecord(cs.t_gemm[0], st);
    gemm_seg segs[4];
    for (int i = 0; i < n; i++) {
        segs[i] = { w[i]->bf16, K, w[i]->n_pad, w[i]->n_out, w[i]->n_out, w[i]->mode, outs[i].y };
        segs[i].resid = outs[i].residual;
        segs[i].ldr = w[i]->n_out;
        segs[i].a_next = outs[i].a_next;
        segs[i].lda_next = w[i]->n_out;
    }
    if (!rc) rc = launch_gemm_group(a, K, T, K, n, segs, cs.err_dev, st);
    if (!rc && nan)
        for (int i = 0; i < n; i++)
            if (outs[i].y) {
                cudaMemsetAsync(outs[i].y, 0xff, (size_t) (T * w[i]->n_out) * 4, st);
                check_finite_kernel<<<148, 256, 0, st>>>(outs[i].y, T * w[i]->n_out, cs.err_dev);
            }
    cudaEventRecord(cs.t_end[0], st);
    cudaMemcpyAsync(cs.err_host, cs.err_dev, sizeof(unsigned), cudaMemcpyDeviceToHost, st);
    const cudaError_t e = cudaStreamSynchronize(st);
    if (rc) return rc;
    if (e != cudaSuccess) return cuda_fail("zest_mul_mat_group_ex", e);
    float pa = 0, gm = 0;
    cudaEventElapsedTime(&pa, cs.t_pack[0], cs.t_gemm[0]);
    cudaEventElapsedTime(&gm, cs.t_gemm[0], cs.t_end[0]);
    npu->times.encode_ms += pa;
    npu->times.gemm_ms += gm;
    npu->times.calls += n;
    if (*cs.err_host & ERR_TIMEOUT) return set_error("a GPU kernel's bounded wait ran out");
    if (*cs.err_host & ERR_NOT_FINITE) return set_error("the GPU's results held NaN or infinity");
    return 0;
}

int zest_mul_mat(zest_npu *npu, const zest_wkey *key, int fused, const float *x, int64_t T, float *y, int on_device) {
    if (!key) return set_error("zest_mul_mat: no service or key");
    float *ys[1] = { y };
    return zest_mul_mat_group(npu, 1, key, &fused, x, T, ys, on_device);
}

int zest_plan_gemm(int64_t M, int64_t K, int n, const int64_t *N, int sms, zest_gemm_plan *out) {
    if (!out || !N || n <= 0 || n > 4 || M <= 0 || K <= 0)
        return set_error("zest_plan_gemm: 1 to 4 weights, M and K positive, and an output");
    for (int i = 0; i < n; i++)
        if (N[i] <= 0) return set_error("zest_plan_gemm: every weight needs rows");
    gemm_plan gp;
    plan_gemm(M, K, n, N, sms, gp);
    out->pair_kernel = gp.pair;
    out->tile_n = gp.bn;
    out->tiles_m = gp.num_m;
    out->tiles_n = gp.num_n;
    out->k_blocks = gp.num_k;
    out->tiles = gp.tiles;
    out->ctas = gp.ctas;
    out->raster = gp.raster;
    out->stream_k = gp.stream_k;
    out->whole_tiles = gp.dp_tiles;
    out->split_tiles = gp.sk_tiles;
    out->run_k_blocks = gp.sk_q;
    return 0;
}

int zest_gemm_segs(const uint16_t *a_bf16, int64_t lda, int64_t M, int64_t K, int n, const zest_gemm_seg *segs,
                   unsigned *err, void *stream) {
    if (n <= 0 || n > 4 || !segs) return set_error("zest_gemm_segs: 1 to 4 weights");
    gemm_seg g[4];
    for (int i = 0; i < n; i++) {
        const zest_gemm_seg &z = segs[i];
        g[i] = { z.b, z.ldb, z.N, z.ldc, 0, z.mode, z.c };
        g[i].resid = z.residual;
        g[i].ldr = z.ldr;
        g[i].a_next = z.a_next;
        g[i].lda_next = z.lda_next;
        g[i].c_mc = z.c_multicast;
        g[i].mc_store = z.multicast_store;
        g[i].c_peers = z.c_peers;
        g[i].n_peers = z.n_peers;
        g[i].c16 = z.c16;
        g[i].n_c16 = z.n_c16;
        g[i].ldc16 = z.ldc16;
    }
    return launch_gemm_group(a_bf16, lda, M, K, n, g, err, (cudaStream_t) stream);
}

int zest_gemm_group(const uint16_t *a_bf16, int64_t lda, int64_t M, int64_t K, int n, const uint16_t *const *b_bf16,
                    const int64_t *ldb, const int64_t *N, const int *mode, float *const *c, const int64_t *ldc,
                    unsigned *err, void *stream) {
    if (n <= 0 || n > 4 || !b_bf16 || !ldb || !N || !mode || !c || !ldc)
        return set_error("zest_gemm_group: 1 to 4 weights, every array given");
    gemm_seg segs[4];
    for (int i = 0; i < n; i++) segs[i] = { b_bf16[i], ldb[i], N[i], ldc[i], 0, mode[i], c[i] };
    return launch_gemm_group(a_bf16, lda, M, K, n, segs, err, (cudaStream_t) stream);
}

int zest_take_times(zest_npu *npu, zest_times *out) {
    if (!npu || !out) return set_error("zest_take_times: no service");
    *out = npu->times;
    npu->times = {};
    return 0;
}

}  // extern "C"
