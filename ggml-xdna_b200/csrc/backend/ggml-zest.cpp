// ggml backend plugin for the B200: device XDNA0 next to llama.cpp's CUDA
// backend. A B200 counterpart of the reference's src/ggml-zest.cpp.
//
// As in the reference, supports_op is the whole policy. The device reports no
// memory of its own (so llama.cpp gives every layer's weights to the GPU
// backend), registers as an integrated GPU ranked above it, and shares the
// CUDA backend's buffer type. The scheduler therefore hands over any op we
// accept with no copies, and the CUDA backend runs the rest as it would
// alone. We claim prompt-sized weight MUL_MATs. Their operands are
// already in device memory, so every claimed matmul runs in place: the
// weight's copy is converted on the GPU from the raw GGUF bytes (K1), and
// each call packs its activations (K2) and runs the tensor-core GEMM (K3),
// writing ggml's f32 result directly (libzest_b200 kernels).
//
// Reference map: gate src/ggml-zest.cpp:1066-1072,1160-1226; graph_compute
// :654-707,768-926; graph_optimize :934-965; budget :429-564; device/reg
// vtables :967-1061,1250-1319; sticky failure :120-130.
#include "ggml-zest.h"
#include "ggml_abi.h"
#include "zest_b200.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#define ZEST_DESCRIPTION "NVIDIA B200 tensor cores (prompt work, next to the CUDA GPU backend)"

namespace {

// ---------------------------------------------------------------------------
// settings: environment variables read once, empty meaning unset
// (src/xdna-env.h:9-17)
// ---------------------------------------------------------------------------

const char *zenv(const char *name) {
    const char *s = getenv(name);
    return s && *s ? s : nullptr;
}

int64_t env_int(const char *name, int64_t def) {
    const char *s = zenv(name);
    return s ? atoll(s) : def;
}

// Prompt rows at or above which a matmul is ours (src/ggml-zest.cpp:65-74).
int64_t min_batch() {
    static const int64_t v = env_int("GGML_XDNA_MIN_BATCH", 1024);
    return v;
}

// Work below which a launch is not worth it (src/ggml-zest.cpp:76-81).
int64_t min_mflop() {
    static const int64_t v = env_int("GGML_XDNA_MIN_MFLOP", 256);
    return v;
}

// The CUDA device the sibling CUDA backend calls CUDA0.
int cuda_device() {
    static const int v = (int) env_int("GGML_ZEST_CUDA_DEVICE", 0);
    return v;
}

bool trace() {
    static const bool v = env_int("GGML_XDNA_TRACE", 0) != 0;
    return v;
}

void log_line(const char *level, const std::string &msg) { fprintf(stderr, "xdna: %s%s\n", level, msg.c_str()); }

bool op_is(const ggml_tensor *t, const char *name) {
    const char *n = ggml_op_name(t->op);
    return n && strcmp(n, name) == 0;
}

// ---------------------------------------------------------------------------
// run mode and the sticky failure (src/ggml-zest.cpp:91-130)
// ---------------------------------------------------------------------------

// Whether the GPU runs the path, decided once, when llama.cpp registers the
// backend: it opens and a small exact multiply through all three kernels
// comes back right (zest_usable). There is no host-only mode: this build has
// no CPU path.
bool gpu_usable() {
    static const bool ok = [] {
        char why[512] = {};
        const bool good = zest_usable(cuda_device(), why, sizeof why) == 0;
        if (good) log_line("", why);
        else log_line("not offering " GGML_XDNA_DEVICE_NAME ": ", why);
        return good;
    }();
    return ok;
}

// Set when a claimed matmul fails. From then on the backend claims nothing,
// so the scheduler hands everything to the GPU backend; the piece that
// failed returns GGML_STATUS_FAILED.
std::atomic<bool> g_broken{ false };

void failed(const std::string &err) {
    if (!g_broken.exchange(true))
        log_line("", "the B200 path failed (" + err + "); claiming nothing from now on");
}

// ---------------------------------------------------------------------------
// the CUDA backend we work next to (src/ggml-zest.cpp:132-169)
// ---------------------------------------------------------------------------

struct sibling_t {
    ggml_backend_dev_t dev = nullptr;
    ggml_backend_buffer_type_t buft = nullptr;
};

const sibling_t &sibling() {
    static sibling_t s;
    static std::once_flag once;
    std::call_once(once, [] {
        char name[32];
        snprintf(name, sizeof name, "CUDA%d", cuda_device());
        ggml_backend_dev_t d = ggml_backend_dev_by_name(name);
        if (!d)
            for (size_t i = 0; i < ggml_backend_dev_count(); i++) {
                ggml_backend_dev_t c = ggml_backend_dev_get(i);
                const enum ggml_backend_dev_type t = ggml_backend_dev_type(c);
                if ((t == GGML_BACKEND_DEVICE_TYPE_GPU || t == GGML_BACKEND_DEVICE_TYPE_IGPU) &&
                    strcmp(ggml_backend_dev_name(c), GGML_XDNA_DEVICE_NAME) != 0) {
                    d = c;
                    break;
                }
            }
        if (!d) {
            log_line("", "no CUDA device registered; " GGML_XDNA_DEVICE_NAME " works next to one");
            return;
        }
        s.dev = d;
        s.buft = ggml_backend_dev_buffer_type(d);
    });
    return s;
}

// ---------------------------------------------------------------------------
// the weight-copy budget (src/ggml-zest.cpp:429-564)
// ---------------------------------------------------------------------------

struct wkey {
    const void *buffer, *data;
    int type;
    int64_t ne0, ne1;
    bool operator==(const wkey &o) const {
        return buffer == o.buffer && data == o.data && type == o.type && ne0 == o.ne0 && ne1 == o.ne1;
    }
};

struct wkey_hash {
    size_t operator()(const wkey &k) const {
        return std::hash<const void *>()(k.buffer) ^ (std::hash<const void *>()(k.data) * 31) ^ (size_t) k.ne1;
    }
};

constexpr double GB = 1024.0 * 1024 * 1024;

// A weight copy on the GPU: the bfp16 bytes (9 per 8 values) and the bf16
// expansion (2 per value), N padded to 512.
double copy_bytes(int64_t K, int64_t N) { return (double) ((N + 511) / 512 * 512) * (double) K * (9.0 / 8 + 2.0); }

int layer_of(const ggml_tensor *w) {
    int layer = -1;
    return sscanf(w->name, "blk.%d.", &layer) == 1 ? layer : -1;
}

// Weights are taken in the order llama.cpp asks about them until the next
// would pass the limit; then that layer and every later weight stay on the
// GPU backend, and what was taken stays taken. The limit is the device
// memory free at the first question, less what is kept back for llama.cpp's
// work buffers (the larger of 4 GB and a tenth of the device), or
// GGML_XDNA_MAX_COPY_GB.
struct budget_t {
    std::mutex mu;
    int contexts = 0;
    bool started = false, cut = false, running = false;
    double limit = 0, taken = 0;
    struct entry {
        int layer;
        double bytes;
    };
    std::unordered_map<wkey, entry, wkey_hash> in, out;
    void reset() {
        started = cut = running = false;
        limit = taken = 0;
        in.clear();
        out.clear();
    }
};
budget_t g_budget;

bool budget_takes(const ggml_tensor *w) {
    if (!w->buffer || !w->data || ggml_backend_buffer_get_usage(w->buffer) != GGML_BACKEND_BUFFER_USAGE_WEIGHTS)
        return true;
    budget_t &b = g_budget;
    std::lock_guard<std::mutex> lk(b.mu);
    if (b.contexts == 0) return true;
    const wkey key = { w->buffer, w->data, (int) w->type, w->ne[0], w->ne[1] };
    if (b.in.count(key)) return true;
    if (b.out.count(key)) return false;
    if (!b.started) {
        b.started = true;
        const char *s = zenv("GGML_XDNA_MAX_COPY_GB");
        if (s) {
            b.limit = atof(s) * GB;
        } else {
            size_t free_b = 0, total_b = 0;
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(cuda_device());
            if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) free_b = total_b = 0;
            cudaSetDevice(prev);
            b.limit = (double) free_b - std::max(4 * GB, (double) total_b / 10);
        }
    }
    const budget_t::entry e = { layer_of(w), copy_bytes(w->ne[0], w->ne[1]) };
    if (!b.cut && b.taken + e.bytes <= b.limit) {
        b.in[key] = e;
        b.taken += e.bytes;
        return true;
    }
    if (!b.cut) {
        b.cut = true;
        // the layer's weights taken so far go back with it: no layer is split
        if (e.layer >= 0 && !b.running)
            for (auto it = b.in.begin(); it != b.in.end();) {
                if (it->second.layer != e.layer) {
                    ++it;
                    continue;
                }
                b.taken -= it->second.bytes;
                b.out.insert(*it);
                it = b.in.erase(it);
            }
        char msg[160];
        snprintf(msg, sizeof msg, "weight copies limited to %.1f GB; later layers stay on the GPU backend",
                 std::max(0.0, b.limit) / GB);
        log_line("", msg);
    }
    b.out[key] = e;
    return false;
}

// ---------------------------------------------------------------------------
// the policy (src/ggml-zest.cpp:54-61,1063-1072,1160-1226)
// ---------------------------------------------------------------------------

int64_t op_batch(const ggml_tensor *op) { return op_is(op, "MUL_MAT") ? op->ne[1] : ggml_nrows(op); }

bool native_type(int t) {
    return t == GGML_TYPE_F32 || t == GGML_TYPE_F16 || t == GGML_TYPE_Q8_0 || t == GGML_TYPE_Q4_K ||
           t == GGML_TYPE_Q6_K || t == GGML_TYPE_IQ3_S;
}

// The weight side of a matmul we can take: a plain 2D leaf (not a view, not
// computed), of a type the GPU converts or ggml can dequantise.
bool is_weight(const ggml_tensor *w) {
    if (w->op != GGML_OP_NONE || w->view_src != nullptr) return false;
    if (w->ne[2] != 1 || w->ne[3] != 1 || !ggml_is_contiguous(w)) return false;
    if (native_type(w->type)) return true;
    const ggml_type_traits *tr = ggml_get_type_traits(w->type);
    return tr && tr->to_float != nullptr;
}

// Shapes the kernels take: K a multiple of 64 (the bfp16 tile's K) and of
// the type's block.
bool has_shape(const ggml_tensor *w) { return w->ne[0] % 64 == 0 && w->ne[0] >= 64 && w->ne[1] >= 1; }

bool claim_mul_mat(const ggml_tensor *op) {
    const ggml_tensor *src0 = op->src[0], *src1 = op->src[1];
    if (!src0 || !src1) return false;
    if (op_batch(op) < min_batch()) return false;
    if (!is_weight(src0)) return false;
    if (op->type != GGML_TYPE_F32 || src1->type != GGML_TYPE_F32) return false;
    if (!ggml_is_contiguous(src1) || src1->ne[2] != 1 || src1->ne[3] != 1) return false;
    if (src0->ne[0] != src1->ne[0]) return false;
    if (!has_shape(src0)) return false;
    const int64_t mflop = 2 * src0->ne[0] * src0->ne[1] * op_batch(op) / 1000000;
    return mflop >= min_mflop() && budget_takes(src0);
}

// The whole policy. Block claiming of the small ops around our matmuls is
// not built yet, so this claims matmuls only (the reference with
// GGML_XDNA_BLOCKS=0).
bool policy(const ggml_tensor *op) { return op_is(op, "MUL_MAT") && claim_mul_mat(op); }

// ---------------------------------------------------------------------------
// the backend context (src/ggml-zest.cpp:184-423)
// ---------------------------------------------------------------------------

struct context {
    zest_npu *npu = nullptr;
    std::vector<float> host_values;  // a weight of a type without a GPU converter, dequantised
    std::vector<uint8_t> host_raw;
    float *stage_x = nullptr, *stage_y = nullptr;
    size_t stage_x_cap = 0, stage_y_cap = 0;
    // where the time goes, printed with GGML_XDNA_TRACE=1
    double compute_ms = 0, copy_ms = 0;
    int64_t matmuls = 0, pieces = 0, late_copies = 0;

    ~context() {
        if (npu) zest_close(npu);
        cudaFree(stage_x);
        cudaFree(stage_y);
    }
};

bool is_host(const ggml_tensor *t) { return t->buffer && ggml_backend_buffer_is_host(t->buffer); }

bool grow(float **p, size_t *cap, size_t need) {
    if (need <= *cap) return true;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    if (cudaMalloc(p, need) != cudaSuccess) return false;
    *cap = need;
    return true;
}

// Builds a weight's copy if it is not there yet: from the raw GGUF bytes
// where they lie (device or host), converted on the GPU, or for a type
// without a GPU converter dequantised once with ggml's own to_float, as the
// reference does for every type (src/xdna-npu.cpp:339-378).
bool ensure_weight(context &ctx, const ggml_tensor *w, std::string &err) {
    const zest_wkey key = { w->buffer, w->data, (int) w->type, w->ne[0], w->ne[1] };
    if (zest_has_weight(ctx.npu, &key)) return true;
    const auto t0 = std::chrono::steady_clock::now();
    int rc;
    if (native_type(w->type)) {
        rc = zest_add_weight(ctx.npu, &key, w->data, is_host(w) ? 0 : 1);
    } else {
        const ggml_type_traits *tr = ggml_get_type_traits(w->type);
        if (!tr || !tr->to_float) {
            err = std::string(w->name) + ": no dequantiser for its type";
            return false;
        }
        const size_t nb = ggml_nbytes(w);
        const uint8_t *raw = (const uint8_t *) w->data;
        if (!is_host(w)) {
            ctx.host_raw.resize(nb);
            if (cudaMemcpy(ctx.host_raw.data(), w->data, nb, cudaMemcpyDeviceToHost) != cudaSuccess) {
                err = std::string(w->name) + ": cannot read the weight";
                return false;
            }
            raw = ctx.host_raw.data();
        }
        const int64_t K = w->ne[0], N = w->ne[1];
        ctx.host_values.resize((size_t) (K * N));
        for (int64_t r = 0; r < N; r++) tr->to_float(raw + r * w->nb[1], ctx.host_values.data() + r * K, K);
        rc = zest_add_weight_values(ctx.npu, &key, ctx.host_values.data(), 0);
    }
    ctx.copy_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (rc) err = std::string(w->name) + ": " + zest_last_error();
    return rc == 0;
}

// One claimed MUL_MAT, in place on device memory where its tensors are
// (src/ggml-zest.cpp:654-707).
bool mul_mat(context &ctx, ggml_tensor *node, std::string &err) {
    const ggml_tensor *src0 = node->src[0], *src1 = node->src[1];
    if (!ensure_weight(ctx, src0, err)) return false;
    ctx.matmuls++;
    const zest_wkey key = { src0->buffer, src0->data, (int) src0->type, src0->ne[0], src0->ne[1] };
    const int64_t K = src0->ne[0], N = src0->ne[1], T = src1->ne[1];
    const bool x_host = is_host(src1), y_host = is_host(node);
    if (x_host == y_host) {
        if (zest_mul_mat(ctx.npu, &key, 0, (const float *) src1->data, T, (float *) node->data, x_host ? 0 : 1)) {
            err = std::string(node->name) + ": " + zest_last_error();
            return false;
        }
        return true;
    }
    // one side in host memory (a graph input, or a host-buffer result): stage it
    const size_t xb = (size_t) (T * K) * 4, yb = (size_t) (T * N) * 4;
    const float *x = (const float *) src1->data;
    float *y = (float *) node->data;
    if (x_host) {
        if (!grow(&ctx.stage_x, &ctx.stage_x_cap, xb) ||
            cudaMemcpy(ctx.stage_x, src1->data, xb, cudaMemcpyHostToDevice) != cudaSuccess) {
            err = "cannot stage the input";
            return false;
        }
        x = ctx.stage_x;
    }
    if (y_host) {
        if (!grow(&ctx.stage_y, &ctx.stage_y_cap, yb)) {
            err = "cannot stage the output";
            return false;
        }
        y = ctx.stage_y;
    }
    if (zest_mul_mat(ctx.npu, &key, 0, x, T, y, 1)) {
        err = std::string(node->name) + ": " + zest_last_error();
        return false;
    }
    if (y_host && cudaMemcpy(node->data, ctx.stage_y, yb, cudaMemcpyDeviceToHost) != cudaSuccess) {
        err = "cannot write the result back";
        return false;
    }
    return true;
}

// ---------------------------------------------------------------------------
// backend vtable (src/ggml-zest.cpp:639-652,768-984)
// ---------------------------------------------------------------------------

const char *backend_get_name(ggml_backend_t) { return GGML_XDNA_DEVICE_NAME; }

void backend_free(ggml_backend_t backend) {
    delete (context *) backend->context;
    delete backend;
    std::lock_guard<std::mutex> lk(g_budget.mu);
    if (--g_budget.contexts == 0) g_budget.reset();
}

enum ggml_status backend_graph_compute(ggml_backend_t backend, ggml_cgraph *cgraph) {
    context &ctx = *(context *) backend->context;
    {
        std::lock_guard<std::mutex> lk(g_budget.mu);
        g_budget.running = true;
    }
    const auto t0 = std::chrono::steady_clock::now();
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cuda_device());
    enum ggml_status status = GGML_STATUS_SUCCESS;
    const int n = ggml_graph_n_nodes(cgraph);
    for (int i = 0; i < n && status == GGML_STATUS_SUCCESS; i++) {
        ggml_tensor *node = ggml_graph_node(cgraph, i);
        if (op_is(node, "NONE") || op_is(node, "RESHAPE") || op_is(node, "VIEW") || op_is(node, "PERMUTE") ||
            op_is(node, "TRANSPOSE"))
            continue;
        std::string err;
        if (op_is(node, "MUL_MAT")) {
            if (!mul_mat(ctx, node, err)) {
                failed(err);
                status = GGML_STATUS_FAILED;
            }
        } else {
            log_line("", std::string("unsupported op ") + ggml_op_name(node->op));
            status = GGML_STATUS_FAILED;
        }
    }
    cudaSetDevice(prev);
    ctx.compute_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    ctx.pieces++;
    if (trace() && ctx.matmuls >= 196) {
        zest_times t = {};
        zest_take_times(ctx.npu, &t);
        fprintf(stderr,
                "xdna times, %lld matmuls in %lld pieces: all %.1f ms | copies %.1f, encode %.1f, GEMM %.1f "
                "(%d calls), weight copies %.1f ms\n",
                (long long) ctx.matmuls, (long long) ctx.pieces, ctx.compute_ms, t.copy_ms, t.encode_ms, t.gemm_ms,
                t.calls, ctx.copy_ms);
        ctx.compute_ms = ctx.copy_ms = 0;
        ctx.matmuls = ctx.pieces = 0;
    }
    return status;
}

// Weight copies made as soon as llama.cpp plans a piece
// (src/ggml-zest.cpp:928-965): the first prompt then need not wait for them.
// GGML_XDNA_COPY_AT_LOAD=0 leaves them to the first prompt.
void backend_graph_optimize(ggml_backend_t backend, ggml_cgraph *cgraph, ggml_backend_graph_optimize_params *) {
    static const bool at_load = env_int("GGML_XDNA_COPY_AT_LOAD", 1) != 0;
    if (!at_load || g_broken) return;
    context &ctx = *(context *) backend->context;
    const int n = ggml_graph_n_nodes(cgraph);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cuda_device());
    for (int i = 0; i < n; i++) {
        const ggml_tensor *node = ggml_graph_node(cgraph, i);
        if (!op_is(node, "MUL_MAT")) continue;
        const ggml_tensor *w = node->src[0];
        // llama.cpp's memory-fitting trial loads no weight data: nothing to build
        if (!w || !w->data || !w->buffer || ggml_backend_buffer_get_usage(w->buffer) != GGML_BACKEND_BUFFER_USAGE_WEIGHTS)
            continue;
        std::string err;
        if (!ensure_weight(ctx, w, err)) {
            failed("building a weight copy at load: " + err);
            break;
        }
    }
    cudaSetDevice(prev);
}

ggml_guid_t backend_guid() {
    static ggml_guid guid = { 0x5a, 0xe5, 0x7b, 0x20, 0x0b, 0x2d, 0x4c, 0x19, 0xa4, 0x61, 0x3e, 0x0f, 0x8c, 0x77, 0x12, 0xd3 };
    return &guid;
}

const ggml_backend_i backend_iface = {
    /* .get_name            = */ backend_get_name,
    /* .free                = */ backend_free,
    /* .set_tensor_async    = */ nullptr,
    /* .get_tensor_async    = */ nullptr,
    /* .set_tensor_2d_async = */ nullptr,
    /* .get_tensor_2d_async = */ nullptr,
    /* .cpy_tensor_async    = */ nullptr,
    /* .synchronize         = */ nullptr,
    /* .graph_plan_create   = */ nullptr,
    /* .graph_plan_free     = */ nullptr,
    /* .graph_plan_update   = */ nullptr,
    /* .graph_plan_compute  = */ nullptr,
    /* .graph_compute       = */ backend_graph_compute,
    /* .event_record        = */ nullptr,
    /* .event_wait          = */ nullptr,
    /* .graph_optimize      = */ backend_graph_optimize,
};

// ---------------------------------------------------------------------------
// device vtable (src/ggml-zest.cpp:992-1061,1228-1267)
// ---------------------------------------------------------------------------

const char *dev_get_name(ggml_backend_dev_t) { return GGML_XDNA_DEVICE_NAME; }
const char *dev_get_description(ggml_backend_dev_t) { return ZEST_DESCRIPTION; }

// No free memory but some in total: llama.cpp gives this device no layers.
void dev_get_memory(ggml_backend_dev_t, size_t *free, size_t *total) {
    *free = 0;
    *total = 1;
}

// An integrated GPU: ranked with the GPUs, where the scheduler asks it first.
enum ggml_backend_dev_type dev_get_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_IGPU; }

void dev_get_props(ggml_backend_dev_t dev, ggml_backend_dev_props *props) {
    props->name = dev_get_name(dev);
    props->description = dev_get_description(dev);
    props->type = dev_get_type(dev);
    props->device_id = nullptr;
    dev_get_memory(dev, &props->memory_free, &props->memory_total);
    // no async and no events: the scheduler hands over with plain synchronizes
    props->caps = { false, false, false, false, false };
}

ggml_backend_t dev_init_backend(ggml_backend_dev_t dev, const char *) {
    if (!sibling().dev || !gpu_usable()) return nullptr;
    auto *ctx = new context;
    ctx->npu = zest_open(cuda_device());
    if (!ctx->npu) {
        log_line("", std::string("cannot open the GPU: ") + zest_last_error());
        delete ctx;
        return nullptr;
    }
    {
        std::lock_guard<std::mutex> lk(g_budget.mu);
        g_budget.contexts++;
    }
    return new ggml_backend{ backend_guid(), backend_iface, dev, ctx };
}

ggml_backend_buffer_type_t dev_get_buffer_type(ggml_backend_dev_t) { return sibling().buft; }

bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor *op) {
    if (!sibling().dev || g_broken || !gpu_usable()) return false;
    return policy(op);
}

// The CUDA backend's buffers, and host memory (graph inputs).
bool dev_supports_buft(ggml_backend_dev_t, ggml_backend_buffer_type_t buft) {
    const sibling_t &s = sibling();
    return (s.buft != nullptr && buft == s.buft) || ggml_backend_buft_is_host(buft);
}

const ggml_backend_device_i device_iface = {
    /* .get_name             = */ dev_get_name,
    /* .get_description      = */ dev_get_description,
    /* .get_memory           = */ dev_get_memory,
    /* .get_type             = */ dev_get_type,
    /* .get_props            = */ dev_get_props,
    /* .init_backend         = */ dev_init_backend,
    /* .get_buffer_type      = */ dev_get_buffer_type,
    /* .get_host_buffer_type = */ nullptr,
    /* .buffer_from_host_ptr = */ nullptr,
    /* .supports_op          = */ dev_supports_op,
    /* .supports_buft        = */ dev_supports_buft,
    // deliberately no offload_op: that path copies the weights per op
    /* .offload_op           = */ nullptr,
    /* .event_new            = */ nullptr,
    /* .event_free           = */ nullptr,
    /* .event_synchronize    = */ nullptr,
};

// ---------------------------------------------------------------------------
// registry (src/ggml-zest.cpp:1269-1319)
// ---------------------------------------------------------------------------

const char *reg_get_name(ggml_backend_reg_t) { return GGML_XDNA_NAME; }

// No device when the GPU cannot run the path: llama.cpp then never sees XDNA0.
size_t reg_device_count(ggml_backend_reg_t) { return gpu_usable() ? 1 : 0; }

ggml_backend_dev_t reg_device_get(ggml_backend_reg_t reg, size_t index);

const ggml_backend_reg_i reg_iface = {
    /* .get_name         = */ reg_get_name,
    /* .get_device_count = */ reg_device_count,
    /* .get_device       = */ reg_device_get,
    /* .get_proc_address = */ nullptr,
};

}  // namespace

extern "C" {

ggml_backend_reg_t ggml_backend_xdna_reg(void) {
    static ggml_backend_reg reg = { GGML_BACKEND_API_VERSION, reg_iface, nullptr };
    return &reg;
}

int ggml_zest_policy_supports(const ggml_tensor *op) { return op && policy(op) ? 1 : 0; }

GGML_BACKEND_API ggml_backend_reg_t ggml_backend_init(void) { return ggml_backend_xdna_reg(); }

GGML_BACKEND_API int ggml_backend_score(void) { return 1; }

}  // extern "C"

namespace {

ggml_backend_dev_t reg_device_get(ggml_backend_reg_t, size_t index) {
    if (index != 0) return nullptr;
    static ggml_backend_device dev = { device_iface, ggml_backend_xdna_reg(), nullptr };
    return &dev;
}

}  // namespace
