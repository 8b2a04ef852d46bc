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
#include <unordered_set>
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

// A node that computes nothing: a leaf, or a new description of existing memory.
bool is_noop(const ggml_tensor *t) {
    return op_is(t, "NONE") || op_is(t, "RESHAPE") || op_is(t, "VIEW") || op_is(t, "PERMUTE") ||
           op_is(t, "TRANSPOSE");
}

// A piece's nodes in graph order, and which tensors are nodes of it. `nodes`
// leaves out leaves, and with compute_only also the nodes that only
// re-describe memory; every node stays a member (count).
struct piece_nodes {
    std::vector<ggml_tensor *> nodes;
    std::unordered_map<const ggml_tensor *, int> index;
    size_t count(const ggml_tensor *t) const { return index.count(t); }
};

piece_nodes collect_piece(ggml_cgraph *g, bool compute_only) {
    piece_nodes p;
    const int n = ggml_graph_n_nodes(g);
    for (int i = 0; i < n; i++) {
        ggml_tensor *node = ggml_graph_node(g, i);
        p.index[node] = i;
        if (compute_only ? !is_noop(node) : !op_is(node, "NONE")) p.nodes.push_back(node);
    }
    return p;
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

// The device whose buffers we share: llama.cpp's CUDA<n> by its name, or,
// registered under another name, the first GPU device that is not this
// plugin's own.
ggml_backend_dev_t find_sibling() {
    char want[32];
    snprintf(want, sizeof want, "CUDA%d", cuda_device());
    if (ggml_backend_dev_t by_name = ggml_backend_dev_by_name(want)) return by_name;
    auto other_gpu = [](ggml_backend_dev_t c) {
        const enum ggml_backend_dev_type t = ggml_backend_dev_type(c);
        const bool gpu = t == GGML_BACKEND_DEVICE_TYPE_GPU || t == GGML_BACKEND_DEVICE_TYPE_IGPU;
        return gpu && std::string(ggml_backend_dev_name(c)) != GGML_XDNA_DEVICE_NAME;
    };
    const size_t n = ggml_backend_dev_count();
    size_t i = 0;
    while (i < n && !other_gpu(ggml_backend_dev_get(i))) i++;
    return i < n ? ggml_backend_dev_get(i) : nullptr;
}

const sibling_t &sibling() {
    static sibling_t s;
    static std::once_flag once;
    std::call_once(once, [] {
        ggml_backend_dev_t d = find_sibling();
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
    const char *source = "";  // where the limit came from
    struct entry {
        int layer;
        double bytes;
    };
    std::unordered_map<wkey, entry, wkey_hash> in, out;
    void reset() {
        started = cut = running = false;
        limit = taken = 0;
        source = "";
        in.clear();
        out.clear();
    }
};
budget_t g_budget;

// The decision for one weight against budget b (its lock held).
bool budget_decide(budget_t &b, const ggml_tensor *w) {
    const wkey key = { w->buffer, w->data, (int) w->type, w->ne[0], w->ne[1] };
    if (b.in.count(key)) return true;
    if (b.out.count(key)) return false;
    if (!b.started) {
        b.started = true;
        const char *s = zenv("GGML_XDNA_MAX_COPY_GB");
        if (s) {
            b.limit = atof(s) * GB;
            b.source = "GGML_XDNA_MAX_COPY_GB";
        } else {
            b.source = "free GPU memory less a reserve of max(4 GB, a tenth)";
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

// Said once, as the first prompt runs, what the weight copies came to
// (src/ggml-zest.cpp:556-564): the report is left out when the budget cut,
// which said so when it happened.
void budget_report() {
    std::lock_guard<std::mutex> lk(g_budget.mu);
    budget_t &b = g_budget;
    if (b.running) return;
    b.running = true;
    if (!b.started || b.cut) return;
    char msg[256];
    snprintf(msg, sizeof msg, "weight copies: %.1f GB for %zu weights (limit %.1f GB: %s)", b.taken / GB, b.in.size(),
             std::max(0.0, b.limit) / GB, b.source);
    log_line("", msg);
}

// What we noticed about the model while llama.cpp planned its graph, said
// once from graph_compute (src/ggml-zest.cpp:566-655): llama.cpp's
// memory-fitting trial plans graphs with warnings hidden but never computes
// one. A mixture-of-experts model's expert step is a MUL_MAT_ID, which is
// not claimed, and rounding its router's multiply to bfp16 can change which
// experts a token uses. (The reference's second note, on narrow models, rests
// on its NPU-against-iGPU measurements and is not made here.)
struct notes_t {
    std::atomic<bool> moe{ false };
    std::atomic<bool> said{ false };
    void reset() {
        moe = false;
        said = false;
    }
};
notes_t g_notes;

void note_model(const ggml_tensor *op) {
    if (op_is(op, "MUL_MAT_ID")) g_notes.moe.store(true, std::memory_order_relaxed);
}

std::string model_notes() {
    std::string s;
    if (g_notes.moe.load())
        s += "mixture-of-experts model: XDNA0 does not take the expert step (MUL_MAT_ID), so it gets only part "
             "of the work, and rounding the router's multiply to bfp16 can change which experts a token uses "
             "(the reference measured such models drifting further from the GPU's answers than dense ones). "
             "Running it on XDNA0 as asked; -dev CUDA0 would use the GPU backend alone";
    return s;
}

void say_notes() {
    if (g_notes.said.exchange(true)) return;
    const std::string s = model_notes();
    if (!s.empty()) log_line("warning: ", s);
}

bool budget_takes(const ggml_tensor *w) {
    if (!w->buffer || !w->data || ggml_backend_buffer_get_usage(w->buffer) != GGML_BACKEND_BUFFER_USAGE_WEIGHTS)
        return true;
    std::lock_guard<std::mutex> lk(g_budget.mu);
    if (g_budget.contexts == 0) return true;
    return budget_decide(g_budget, w);
}

// ---------------------------------------------------------------------------
// the policy (src/ggml-zest.cpp:54-61,1063-1072,1160-1226)
// ---------------------------------------------------------------------------

int64_t op_batch(const ggml_tensor *op) { return op_is(op, "MUL_MAT") ? op->ne[1] : ggml_nrows(op); }

// ggml's IQ3_S codebook (512 entries of four magnitudes), read back through
// the host ggml's own to_float, the dequantiser the reference converts every
// weight type with (src/xdna-npu.cpp:339-348), so no table is built in. One
// 256-value block per entry i: scale 1 (fp16 d = 1, scale nibbles 0), no
// signs, and every 9-bit grid index equal to i (the low byte in all of qs,
// the high bit in all of qh). to_float then gives entry i's four bytes as the
// block's first four values, and every later group of four repeats them.
// Empty when ggml has no IQ3_S dequantiser or it does not answer that way;
// the GPU converter then does not take IQ3_S.
const std::vector<uint32_t> &iq3s_codebook() {
    static const std::vector<uint32_t> grid = []() -> std::vector<uint32_t> {
        const ggml_type_traits *tr = ggml_get_type_traits(GGML_TYPE_IQ3_S);
        if (!tr || !tr->to_float) return {};
        constexpr int QS = 2, QH = QS + 64, SIGNS = QH + 8, SCALES = SIGNS + 32, BLOCK = SCALES + 4;
        static_assert(BLOCK == 110, "block_iq3_s is 110 bytes");
        std::vector<uint32_t> g(512);
        uint8_t blk[BLOCK];
        float y[256];
        for (int i = 0; i < 512; i++) {
            memset(blk, 0, sizeof blk);
            blk[0] = 0x00;  // d = 1.0 as fp16 (0x3c00), little-endian
            blk[1] = 0x3c;
            memset(blk + QS, i & 0xff, 64);
            memset(blk + QH, i >= 256 ? 0xff : 0x00, 8);
            tr->to_float(blk, y, 256);
            uint32_t e = 0;
            for (int j = 0; j < 4; j++) {
                const float v = y[j];
                if (!(v >= 0.0f && v <= 255.0f) || v != (float) (int) v) return {};
                e |= (uint32_t) v << (8 * j);
            }
            for (int j = 4; j < 256; j++)
                if (y[j] != y[j % 4]) return {};
            g[i] = e;
        }
        return g;
    }();
    return grid;
}

bool native_type(int t) {
    if (t == GGML_TYPE_IQ3_S) return !iq3s_codebook().empty();
    return t == GGML_TYPE_F32 || t == GGML_TYPE_F16 || t == GGML_TYPE_Q8_0 || t == GGML_TYPE_Q4_K ||
           t == GGML_TYPE_Q6_K;
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

// --- block claiming: the small ops next to our matmuls
// (src/xdna-exec.cpp:85-131, src/ggml-zest.cpp:1131-1226) ------------------

int32_t param_i32(const ggml_tensor *t, int i) { return t->op_params[i]; }
float param_f32(const ggml_tensor *t, int i) {
    float v;
    memcpy(&v, &t->op_params[i], sizeof v);
    return v;
}

bool same_shape(const ggml_tensor *a, const ggml_tensor *b) {
    return a->ne[0] == b->ne[0] && a->ne[1] == b->ne[1] && a->ne[2] == b->ne[2] && a->ne[3] == b->ne[3];
}

bool f32_contig(const ggml_tensor *t) { return t && t->type == GGML_TYPE_F32 && ggml_is_contiguous(t); }

// a single row as wide as a's rows (a norm's scale, a bias), broadcast over every row of a
bool is_row_of(const ggml_tensor *r, const ggml_tensor *a) {
    return f32_contig(r) && r->ne[0] == a->ne[0] && r->ne[1] == 1 && r->ne[2] == 1 && r->ne[3] == 1;
}

// Rows are prompt tokens, along a tensor's last dimension in use.
int64_t tokens_of(const ggml_tensor *t) { return t->ne[3] > 1 ? t->ne[3] : t->ne[2] > 1 ? t->ne[2] : t->ne[1]; }

bool glu_kind(int g) {
    return g == ZEST_GLU_SWIGLU || g == ZEST_GLU_GEGLU || g == ZEST_GLU_GEGLU_ERF || g == ZEST_GLU_GEGLU_QUICK ||
           g == ZEST_GLU_REGLU;
}

// The input an op keeps as a parameter (a scale or bias row, rope's
// frequency factors); null for none (src/xdna-exec.cpp:85-95).
const ggml_tensor *exec_param(const ggml_tensor *op) {
    if (op_is(op, "MUL")) return op->src[1];
    if (op_is(op, "ADD"))
        return op->src[1] && op->src[0] && is_row_of(op->src[1], op->src[0]) && !same_shape(op->src[0], op->src[1])
                   ? op->src[1]
                   : nullptr;
    if (op_is(op, "ROPE")) return op->src[2];
    return nullptr;
}

// Whether the GPU runs this op in this variant (src/xdna-exec.cpp:97-131).
bool exec_supports(const ggml_tensor *op) {
    const ggml_tensor *a = op->src[0], *b = op->src[1];
    if (op_is(op, "MUL_MAT")) return true;
    if (op_is(op, "RESHAPE")) return a && ggml_is_contiguous(a);
    if (op_is(op, "RMS_NORM")) return f32_contig(a) && f32_contig(op);
    if (op_is(op, "MUL")) return f32_contig(a) && f32_contig(op) && is_row_of(b, a) && same_shape(a, op);
    if (op_is(op, "ADD"))
        return f32_contig(a) && f32_contig(b) && f32_contig(op) && same_shape(a, op) &&
               (same_shape(a, b) || is_row_of(b, a));
    if (op_is(op, "SCALE")) return f32_contig(a) && f32_contig(op) && same_shape(a, op);
    if (op_is(op, "GLU")) {
        if (!glu_kind(param_i32(op, 0)) || !f32_contig(a) || !f32_contig(op)) return false;
        if (b) return param_i32(op, 1) == 0 && f32_contig(b) && same_shape(a, b) && same_shape(a, op);
        return a->ne[0] == 2 * op->ne[0] && ggml_nrows(a) == ggml_nrows(op);
    }
    if (op_is(op, "ROPE")) {
        if (!f32_contig(a) || !f32_contig(op) || !b || b->type != GGML_TYPE_I32) return false;
        const int n_dims = param_i32(op, 1), mode = param_i32(op, 2), n_offs = param_i32(op, 15);
        const ggml_tensor *ff = op->src[2];
        if (ff && (!f32_contig(ff) || ff->ne[0] < n_dims / 2)) return false;
        return (mode == ZEST_ROPE_NEOX || mode == ZEST_ROPE_NORMAL) && n_dims > 0 && n_dims % 2 == 0 &&
               n_dims <= a->ne[0] && n_offs == 0 && a->ne[3] == 1 && b->ne[0] == a->ne[2];
    }
    return false;
}

// Block claiming on, unless GGML_XDNA_BLOCKS=0 (src/ggml-zest.cpp:1131-1140).
bool blocks() {
    static const bool v = env_int("GGML_XDNA_BLOCKS", 1) != 0;
    return v;
}

// GGML_ZEST_GROUPS=0 runs every MUL_MAT on its own (find_groups).
bool groups_on() {
    static const bool v = env_int("GGML_ZEST_GROUPS", 1) != 0;
    return v;
}

// Whether a tensor may live in host memory once allocated: a graph input, an
// embedding lookup, or one in a host buffer (src/ggml-zest.cpp:1149-1158).
bool maybe_host(const ggml_tensor *t) {
    for (; t; t = t->view_src) {
        if ((t->flags & GGML_TENSOR_FLAG_INPUT) || op_is(t, "GET_ROWS")) return true;
        if (t->buffer && ggml_backend_buffer_is_host(t->buffer)) return true;
    }
    return false;
}

// Who reads what, as the scheduler shows us (src/ggml-zest.cpp:1074-1109):
// every supports_op question carries the op's inputs. A fused matmul skips
// writing its own result only when nothing outside its piece reads it.
std::mutex g_read_mu;
std::unordered_map<const ggml_tensor *, std::vector<const ggml_tensor *>> g_readers;

void note_readers(const ggml_tensor *op) {
    std::lock_guard<std::mutex> lk(g_read_mu);
    for (int j = 0; j < GGML_MAX_SRC; j++)
        if (const ggml_tensor *s = op->src[j]) {
            auto &r = g_readers[s];
            if (std::find(r.begin(), r.end(), op) == r.end()) r.push_back(op);
            for (const ggml_tensor *v = s->view_src; v; v = v->view_src) {
                auto &rv = g_readers[v];
                if (std::find(rv.begin(), rv.end(), op) == rv.end()) rv.push_back(op);
            }
        }
}

template <typename Set>
bool read_outside(const ggml_tensor *t, const Set &in_piece) {
    static const bool all = env_int("GGML_XDNA_WRITE_ALL", 0) != 0;
    if (all || (t->flags & GGML_TENSOR_FLAG_OUTPUT)) return true;
    std::lock_guard<std::mutex> lk(g_read_mu);
    auto it = g_readers.find(t);
    if (it == g_readers.end()) return true;
    for (const ggml_tensor *r : it->second)
        if (!in_piece.count(r)) return true;
    return false;
}

// GGML_XDNA_TRACE=1: matmul results with no recorded reader (their readers
// decide what a piece writes back and what it folds), one line each, and a
// count every 100 pieces (src/ggml-zest.cpp:1111-1129).
void trace_piece(ggml_cgraph *cgraph) {
    static std::atomic<int64_t> pieces{ 0 }, results{ 0 }, unseen{ 0 };
    const int64_t p = ++pieces;
    const int n = ggml_graph_n_nodes(cgraph);
    for (int i = 0; i < n; i++) {
        const ggml_tensor *t = ggml_graph_node(cgraph, i);
        if (!op_is(t, "MUL_MAT")) continue;
        results++;
        std::lock_guard<std::mutex> lk(g_read_mu);
        if (!g_readers.count(t)) {
            unseen++;
            log_line("trace: ", std::string(t->name) + " (MUL_MAT) has no recorded reader");
        }
    }
    if (p % 100 == 0) {
        char msg[160];
        snprintf(msg, sizeof msg, "%lld pieces, %lld matmul results, %lld with no recorded reader", (long long) p,
                 (long long) results.load(), (long long) unseen.load());
        log_line("trace: ", msg);
    }
}

// GGML_XDNA_BLOCK_OPS, when set, names the small ops block claiming may take
// (op names split at commas); unset, it may take every op exec_supports runs.
bool block_op_allowed(const ggml_tensor *op) {
    struct allow_list {
        bool given = false;
        std::unordered_set<std::string> names;
    };
    static const allow_list allow = [] {
        allow_list a;
        const char *v = zenv("GGML_XDNA_BLOCK_OPS");
        if (!v) return a;
        a.given = true;
        std::string s(v);
        size_t from = 0;
        while (from <= s.size()) {
            size_t to = s.find(',', from);
            if (to == std::string::npos) to = s.size();
            if (to > from) a.names.insert(s.substr(from, to - from));
            from = to + 1;
        }
        return a;
    }();
    return !allow.given || allow.names.count(ggml_op_name(op->op)) > 0;
}

// The whole policy (src/ggml-zest.cpp:1182-1226): a matmul we can take, or a
// small op the GPU runs that covers a prompt-sized batch, keeps its
// parameters in plain leaves, cannot have its result placed in host memory,
// and is fed by an op we claim.
bool policy(const ggml_tensor *op, int depth = 0) {
    if (op_is(op, "MUL_MAT")) return claim_mul_mat(op);
    if (!blocks() || depth > 8) return false;
    if (!op_is(op, "RESHAPE") && tokens_of(op) < min_batch()) return false;
    if (!exec_supports(op) || !block_op_allowed(op)) return false;
    if (const ggml_tensor *w = exec_param(op))
        if (w->op != GGML_OP_NONE || w->view_src) return false;
    for (int j = 0; j < GGML_MAX_SRC; j++)
        if (const ggml_tensor *s = op->src[j])
            if (maybe_host(s) && same_shape(op, s)) return false;
    for (int j = 0; j < GGML_MAX_SRC; j++) {
        const ggml_tensor *s = op->src[j];
        if (s && s->op != GGML_OP_NONE && policy(s, depth + 1)) return true;
    }
    return false;
}

// ---------------------------------------------------------------------------
// the backend context (src/ggml-zest.cpp:184-423)
// ---------------------------------------------------------------------------

struct context {
    zest_npu *npu = nullptr;
    std::vector<float> host_values;  // a weight of a type without a GPU converter, dequantised
    std::vector<uint8_t> host_raw;
    float *stage_x = nullptr, *stage_y = nullptr;
    size_t stage_x_cap = 0, stage_y_cap = 0;
    // device copies of a piece's host-memory tensors (rotary positions),
    // slot by slot, reused from piece to piece
    std::vector<std::pair<void *, size_t>> stage;
    size_t stage_next = 0;
    float *rope_table = nullptr;
    size_t rope_cap = 0;
    void *a_next = nullptr;  // a SwiGLU's packed result on its way to the next matmul
    size_t a_next_cap = 0;
    // where the time goes, printed with GGML_XDNA_TRACE=1
    double compute_ms = 0, copy_ms = 0;
    int64_t matmuls = 0, pieces = 0, late_copies = 0, small_ops = 0, fused = 0, grouped = 0;

    void *stage_slot(size_t n) {
        if (stage_next == stage.size()) stage.emplace_back(nullptr, 0);
        auto &s = stage[stage_next];
        if (s.second < n) {
            cudaFree(s.first);
            s.first = nullptr;
            s.second = 0;
            if (cudaMalloc(&s.first, n) != cudaSuccess) return nullptr;
            s.second = n;
        }
        stage_next++;
        return s.first;
    }

    ~context() {
        cudaFree(a_next);
        if (npu) zest_close(npu);
        cudaFree(stage_x);
        cudaFree(stage_y);
        cudaFree(rope_table);
        for (auto &s : stage) cudaFree(s.first);
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
    if (--g_budget.contexts == 0) {
        g_budget.reset();
        g_notes.reset();  // the next model gets its own notes
    }
}

const ggml_tensor *owner(const ggml_tensor *t) {
    while (t->view_src) t = t->view_src;
    return t;
}

// SiLU(gate) * up as one GEMM (output mode 2): a SwiGLU whose gate and up are
// matmuls of this piece on the same input, read by nothing else, or one
// matmul whose weight holds the gate's rows and then the up's
// (find_fusions, src/xdna-exec.cpp:392-431).
struct fusion {
    ggml_tensor *gate, *up, *glu;  // up: null for one weight holding both
};

template <typename Set>
std::vector<fusion> find_fusions(const std::vector<ggml_tensor *> &nodes, const Set &in_piece) {
    std::vector<fusion> out;
    for (ggml_tensor *n : nodes) {
        if (!op_is(n, "GLU") || param_i32(n, 0) != ZEST_GLU_SWIGLU || param_i32(n, 1) != 0) continue;
        ggml_tensor *gm = n->src[0], *um = n->src[1];
        if (!op_is(gm, "MUL_MAT") || !in_piece.count(gm) || read_outside(gm, in_piece)) continue;
        if (!native_type(gm->src[0]->type)) continue;
        if (um) {
            if (!op_is(um, "MUL_MAT") || !in_piece.count(um) || read_outside(um, in_piece)) continue;
            if (owner(gm->src[1]) != owner(um->src[1]) || gm->src[0]->type != um->src[0]->type ||
                !same_shape(gm->src[0], um->src[0]))
                continue;
        } else if (gm->src[0]->ne[1] % 2 != 0) {
            continue;
        }
        bool other = false;  // another reader in the piece
        for (ggml_tensor *m : nodes)
            for (int j = 0; j < GGML_MAX_SRC && m != n; j++)
                if (m->src[j] && (owner(m->src[j]) == gm || (um && owner(m->src[j]) == um))) other = true;
        if (!other) out.push_back({ gm, um, n });
    }
    return out;
}

bool ensure_fused(context &ctx, const fusion &f, zest_wkey &key, std::string &err) {
    const ggml_tensor *g = f.gate->src[0];
    key = { g->buffer, g->data, (int) g->type, g->ne[0], f.up ? g->ne[1] : g->ne[1] / 2 };
    if (zest_out_width(ctx.npu, &key, 1) >= 0) return true;
    const char *up_raw = f.up ? (const char *) f.up->src[0]->data : (const char *) g->data + key.N * g->nb[1];
    const auto t0 = std::chrono::steady_clock::now();
    const int rc = zest_add_fused(ctx.npu, &key, g->data, up_raw, is_host(g) ? 0 : 1);
    ctx.copy_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    if (rc) err = std::string(g->name) + ": " + zest_last_error();
    return rc == 0;
}

// MUL_MATs of a piece on one input, run as one grouped call (one pack, one
// launch) at the first one's turn, as the reference submits a piece's
// matmuls as one runlist (src/xdna-npu.cpp:476-531). A later matmul joins
// only where running it early is safe: no node between the two turns
// writes or reads its output's bytes, which ggml's allocator may have lent
// to a tensor whose life ends in between. Input and outputs share one
// residency (all device memory, or all host memory), at most 4 per group.
bool overlaps(const ggml_tensor *a, const ggml_tensor *b) {
    if (!a || !b || !a->data || !b->data) return false;
    const char *a0 = (const char *) a->data, *b0 = (const char *) b->data;
    return a0 < b0 + ggml_nbytes(b) && b0 < a0 + ggml_nbytes(a);
}

template <typename Skip>
std::vector<std::vector<ggml_tensor *>> find_groups(const std::vector<ggml_tensor *> &nodes, const Skip &skip) {
    std::vector<std::vector<ggml_tensor *>> out;
    std::unordered_map<const ggml_tensor *, bool> taken;
    for (size_t i = 0; i < nodes.size(); i++) {
        ggml_tensor *first = nodes[i];
        if (!op_is(first, "MUL_MAT") || skip.count(first) || taken.count(first)) continue;
        const ggml_tensor *x = first->src[1];
        const bool host = is_host(x);
        if (is_host(first) != host) continue;
        std::vector<ggml_tensor *> g{ first };
        for (size_t j = i + 1; j < nodes.size() && g.size() < 4; j++) {
            ggml_tensor *m = nodes[j];
            if (!op_is(m, "MUL_MAT") || skip.count(m) || taken.count(m) || m->src[1] != x || is_host(m) != host)
                continue;
            bool safe = true;
            for (size_t k = i + 1; k < j && safe; k++) {
                const ggml_tensor *p = nodes[k];
                if (std::find(g.begin(), g.end(), p) != g.end()) continue;
                safe = !overlaps(p, m);
                for (int s = 0; s < GGML_MAX_SRC && safe; s++) safe = !overlaps(p->src[s], m);
            }
            for (const ggml_tensor *o : g) safe = safe && !overlaps(o, m) && !overlaps(x, m);
            if (safe) g.push_back(m);
        }
        if (g.size() > 1) {
            for (ggml_tensor *m : g) taken[m] = true;
            out.push_back(std::move(g));
        }
    }
    return out;
}

// One group of MUL_MATs sharing an input (find_groups).
bool mul_mat_group(context &ctx, const std::vector<ggml_tensor *> &g, std::string &err) {
    std::vector<zest_wkey> keys;
    std::vector<float *> ys;
    for (const ggml_tensor *m : g) {
        const ggml_tensor *w = m->src[0];
        if (!ensure_weight(ctx, w, err)) return false;
        keys.push_back({ w->buffer, w->data, (int) w->type, w->ne[0], w->ne[1] });
        ys.push_back((float *) m->data);
    }
    const ggml_tensor *x = g[0]->src[1];
    ctx.matmuls += (int64_t) g.size();
    ctx.grouped += (int64_t) g.size() - 1;
    if (zest_mul_mat_group(ctx.npu, (int) g.size(), keys.data(), nullptr, (const float *) x->data, x->ne[1],
                           ys.data(), is_host(x) ? 0 : 1)) {
        err = std::string(g[0]->name) + ": " + zest_last_error();
        return false;
    }
    return true;
}

// A tensor's bytes on the device: in place, or a staged copy of a
// host-memory tensor (a graph input such as the rotary positions).
const void *device_in(context &ctx, const ggml_tensor *t, cudaStream_t st) {
    if (!t || !is_host(t)) return t ? t->data : nullptr;
    const size_t n = ggml_nbytes(t);
    void *d = ctx.stage_slot(n);
    if (!d || cudaMemcpyAsync(d, t->data, n, cudaMemcpyHostToDevice, st) != cudaSuccess) return nullptr;
    return d;
}

// One small op on the GPU, on the service's stream (run_rows,
// src/xdna-exec.cpp:253-346).
bool small_op(context &ctx, ggml_tensor *n, std::string &err) {
    cudaStream_t st = (cudaStream_t) zest_stream(ctx.npu);
    const ggml_tensor *a = n->src[0], *b = n->src[1];
    const float *x = (const float *) device_in(ctx, a, st);
    float *y = is_host(n) ? (float *) ctx.stage_slot(ggml_nbytes(n)) : (float *) n->data;
    if (!x || !y) {
        err = std::string(n->name) + ": cannot stage a host tensor";
        return false;
    }
    int rc = -1;
    const int64_t d = a->ne[0], rows = ggml_nrows(a);
    if (op_is(n, "RMS_NORM")) {
        rc = zest_rms_norm(x, rows, d, param_f32(n, 0), y, st);
    } else if (op_is(n, "MUL")) {
        rc = zest_mul_row(x, (const float *) device_in(ctx, b, st), rows, d, y, st);
    } else if (op_is(n, "ADD")) {
        rc = zest_add(x, (const float *) device_in(ctx, b, st), same_shape(a, b) ? 0 : 1, rows, d, y, st);
    } else if (op_is(n, "SCALE")) {
        rc = zest_scale(x, rows * d, param_f32(n, 0), param_f32(n, 1), y, st);
    } else if (op_is(n, "GLU")) {
        const int kind = param_i32(n, 0);
        const int64_t f = n->ne[0], out_rows = ggml_nrows(n);
        if (b) {
            rc = zest_glu(kind, x, f, (const float *) device_in(ctx, b, st), f, out_rows, f, y, st);
        } else {
            const bool swapped = param_i32(n, 1) != 0;
            rc = zest_glu(kind, x + (swapped ? f : 0), 2 * f, x + (swapped ? 0 : f), 2 * f, out_rows, f, y, st);
        }
    } else if (op_is(n, "ROPE")) {
        const int n_dims = param_i32(n, 1), mode = param_i32(n, 2), n_ctx_orig = param_i32(n, 4);
        const int64_t T = a->ne[2];
        const float par[6] = { param_f32(n, 5), param_f32(n, 6), param_f32(n, 7),
                               param_f32(n, 8), param_f32(n, 9), param_f32(n, 10) };
        const size_t tb = (size_t) (T * n_dims) * sizeof(float);
        if (tb > ctx.rope_cap) {
            cudaFree(ctx.rope_table);
            ctx.rope_table = nullptr;
            ctx.rope_cap = 0;
            if (cudaMalloc(&ctx.rope_table, tb) != cudaSuccess) {
                err = "cannot allocate the rope table";
                return false;
            }
            ctx.rope_cap = tb;
        }
        const int32_t *pos = (const int32_t *) device_in(ctx, b, st);
        const float *ff = (const float *) device_in(ctx, n->src[2], st);
        rc = zest_rope_table(pos, T, n_dims, n_ctx_orig, par, ff, ctx.rope_table, st);
        if (!rc) rc = zest_rope(x, T, a->ne[1], a->ne[0], n_dims, mode, ctx.rope_table, y, st);
    } else {
        err = std::string("unsupported op ") + ggml_op_name(n->op);
        return false;
    }
    if (rc) {
        err = std::string(n->name) + ": " + zest_last_error();
        return false;
    }
    if (is_host(n) && cudaMemcpyAsync(n->data, y, ggml_nbytes(n), cudaMemcpyDeviceToHost, st) != cudaSuccess) {
        err = std::string(n->name) + ": cannot write the result back";
        return false;
    }
    ctx.small_ops++;
    return true;
}

// ---------------------------------------------------------------------------
// a piece's plan: which matmuls run together and which small ops ride along
// ---------------------------------------------------------------------------

// GGML_ZEST_FUSE=0 runs the block executor's ops one by one.
bool fuse_on() {
    static const bool v = env_int("GGML_ZEST_FUSE", 1) != 0;
    return v;
}

// One call of the matmul service: a group of matmuls on one input (or a
// fused SwiGLU), with what it folds in from the nodes around it (the
// reference folds the same ops into its passes over the rows, run_pass,
// src/xdna-exec.cpp:368-388):
//   norm/mul   the RMS_NORM (and its MUL by a weight row) that makes the
//              input: normalised inside the pack, never written out
//   add[i]     the residual ADD that reads matmul i's result and nothing
//              else does: added in the GEMM epilogue, written to the ADD
//   a_next     a SwiGLU whose result only the next matmul reads: written as
//              that matmul's packed operand, not as f32 (packed_in there)
struct mm_job {
    std::vector<ggml_tensor *> mms;
    const fusion *glu = nullptr;
    ggml_tensor *norm = nullptr, *mul = nullptr;
    std::vector<ggml_tensor *> add;
    bool a_next = false, packed_in = false;
};

// RMS_NORM -> MUL (a weight row) -> ROPE of the same rows: one kernel.
struct rope_job {
    ggml_tensor *norm, *mul, *rope;
};

struct piece_plan {
    std::vector<fusion> fusions;  // the fused SwiGLUs (jobs point into it)
    std::vector<mm_job> jobs;
    std::vector<rope_job> ropes;
    std::unordered_map<const ggml_tensor *, int> job_at, rope_at;  // anchor node -> job
    std::unordered_map<const ggml_tensor *, bool> skip;            // run inside another node's job
    int counts[6] = {};  // SwiGLU fusions, groups, norm prologues, ADD epilogues, packed hand-offs, norm+rope
};

template <typename Set>
piece_plan plan_piece(const std::vector<ggml_tensor *> &nodes, const Set &in_piece) {
    piece_plan pl;
    std::unordered_map<const ggml_tensor *, int> idx;
    for (size_t i = 0; i < nodes.size(); i++) idx[nodes[i]] = (int) i;
    // in-piece readers of a tensor's storage
    std::unordered_map<const ggml_tensor *, std::vector<ggml_tensor *>> readers;
    for (ggml_tensor *m : nodes)
        for (int j = 0; j < GGML_MAX_SRC; j++)
            if (m->src[j]) readers[owner(m->src[j])].push_back(m);
    auto only_read_by = [&](const ggml_tensor *t, const std::vector<ggml_tensor *> &by) {
        if (read_outside(t, in_piece)) return false;
        auto it = readers.find(t);
        if (it == readers.end()) return false;
        for (ggml_tensor *r : it->second)
            if (std::find(by.begin(), by.end(), r) == by.end()) return false;
        return true;
    };
    auto pos = [&](const ggml_tensor *t) { auto it = idx.find(t); return it == idx.end() ? -1 : it->second; };
    auto dev = [](const ggml_tensor *t) { return t && t->data && !is_host(t); };

    if (blocks()) {
        pl.fusions = find_fusions(nodes, in_piece);
        for (const fusion &f : pl.fusions) {
            mm_job j;
            j.mms = { f.gate };
            if (f.up) j.mms.push_back(f.up);
            j.glu = &f;
            pl.job_at[f.gate] = (int) pl.jobs.size();
            pl.jobs.push_back(j);
            if (f.up) pl.skip[f.up] = true;
            pl.skip[f.glu] = true;
            pl.counts[0]++;
        }
    }
    std::unordered_map<const ggml_tensor *, bool> taken;
    for (const auto &kv : pl.job_at) taken[kv.first] = true;
    for (const auto &kv : pl.skip) taken[kv.first] = true;
    const auto groups = groups_on() ? find_groups(nodes, taken) : std::vector<std::vector<ggml_tensor *>>();
    for (const auto &g : groups) {
        mm_job j;
        j.mms = g;
        pl.job_at[g[0]] = (int) pl.jobs.size();
        pl.jobs.push_back(j);
        for (size_t k = 1; k < g.size(); k++) pl.skip[g[k]] = true;
        for (ggml_tensor *m : g) taken[m] = true;
        pl.counts[1]++;
    }
    for (ggml_tensor *m : nodes)
        if (op_is(m, "MUL_MAT") && !taken.count(m)) {
            mm_job j;
            j.mms = { m };
            pl.job_at[m] = (int) pl.jobs.size();
            pl.jobs.push_back(j);
        }
    for (mm_job &j : pl.jobs) j.add.assign(j.mms.size(), nullptr);
    if (!blocks() || !fuse_on()) return pl;

    for (mm_job &j : pl.jobs) {
        const int at = pos(j.mms[0]);
        ggml_tensor *x = j.mms[0]->src[1];
        const ggml_tensor *out0 = j.glu ? j.glu->glu : j.mms[0];
        bool all_dev = dev(x) && dev(out0);
        for (ggml_tensor *m : j.mms) all_dev = all_dev && dev(m->src[1]);
        if (!all_dev) continue;
        // prologue: x = MUL(RMS_NORM(y), w) or RMS_NORM(y), just before the job
        ggml_tensor *mul = op_is(x, "MUL") ? x : nullptr;
        ggml_tensor *nrm = mul ? mul->src[0] : x;
        if (op_is(nrm, "RMS_NORM") && pos(nrm) >= 0 && f32_contig(nrm->src[0]) && dev(nrm->src[0]) &&
            nrm->src[0]->ne[0] == x->ne[0] && (!mul || (pos(mul) == pos(nrm) + 1 && is_row_of(mul->src[1], mul) &&
                                                        dev(mul->src[1]) && mul->src[0] == nrm)) &&
            pos(x) + 1 == at && only_read_by(x, j.mms) && (!mul || only_read_by(nrm, { mul })) &&
            !pl.skip.count(nrm) && !pl.job_at.count(nrm)) {
            j.norm = nrm;
            j.mul = mul;
            pl.skip[nrm] = true;
            if (mul) pl.skip[mul] = true;
            pl.counts[2]++;
        }
        // epilogue: a plain matmul whose only reader is the ADD right after it
        if (!j.glu && j.mms.size() == 1) {
            ggml_tensor *m = j.mms[0];
            const int after = pos(m) + 1;
            if (after < (int) nodes.size()) {
                ggml_tensor *a = nodes[after];
                if (op_is(a, "ADD") && (a->src[0] == m || a->src[1] == m) && only_read_by(m, { a })) {
                    const ggml_tensor *r = a->src[0] == m ? a->src[1] : a->src[0];
                    // the epilogue reads each residual element before writing the same
                    // one: the sum may go in place, or anywhere apart, not half over it
                    const uintptr_t ad = (uintptr_t) a->data, rd = r ? (uintptr_t) r->data : 0;
                    const bool placed = r && (ad == rd || ad + ggml_nbytes(a) <= rd || rd + ggml_nbytes(r) <= ad);
                    if (r && placed && f32_contig(r) && same_shape(r, a) && same_shape(m, a) && f32_contig(a) &&
                        dev(r) && dev(a) && pos(owner(r)) < pos(m)) {
                        j.add[0] = a;
                        pl.skip[a] = true;
                        pl.counts[3]++;
                    }
                }
            }
        }
    }
    // a SwiGLU whose only reader is the matmul right after it hands over its packed result
    for (mm_job &j : pl.jobs) {
        if (!j.glu) continue;
        ggml_tensor *g = j.glu->glu;
        const int after = pos(g) + 1;
        if (after >= (int) nodes.size()) continue;
        auto it = pl.job_at.find(nodes[after]);
        if (it == pl.job_at.end()) continue;
        mm_job &k = pl.jobs[it->second];
        if (k.glu || k.norm || k.mms.size() != 1 || k.mms[0]->src[1] != g || !only_read_by(g, k.mms)) continue;
        if (!f32_contig(g) || g->ne[0] % 64) continue;
        j.a_next = true;
        k.packed_in = true;
        pl.counts[4]++;
    }
    // norm + rope of a head-shaped view: RMS_NORM -> MUL(w) -> ROPE, consecutive
    for (size_t i = 0; i + 2 < nodes.size(); i++) {
        ggml_tensor *nrm = nodes[i], *mul = nodes[i + 1], *rope = nodes[i + 2];
        if (!op_is(nrm, "RMS_NORM") || !op_is(mul, "MUL") || !op_is(rope, "ROPE")) continue;
        if (pl.skip.count(nrm) || pl.skip.count(mul) || mul->src[0] != nrm || rope->src[0] != mul) continue;
        const ggml_tensor *a = nrm->src[0];
        const int mode = param_i32(rope, 2);
        if (!f32_contig(a) || !f32_contig(rope) || !same_shape(a, rope) || a->ne[0] > 256 || a->ne[3] != 1 ||
            !is_row_of(mul->src[1], mul) || (mode != ZEST_ROPE_NORMAL && mode != ZEST_ROPE_NEOX))
            continue;
        if (!dev(a) || !dev(rope) || !dev(mul->src[1]) || !only_read_by(nrm, { mul }) || !only_read_by(mul, { rope }))
            continue;
        pl.rope_at[rope] = (int) pl.ropes.size();
        pl.ropes.push_back({ nrm, mul, rope });
        pl.skip[nrm] = true;
        pl.skip[mul] = true;
        pl.counts[5]++;
    }
    return pl;
}

// The rope table of a ROPE node's positions, in the context's table.
const float *rope_table_of(context &ctx, const ggml_tensor *n, cudaStream_t st, std::string &err) {
    const int n_dims = param_i32(n, 1), n_ctx_orig = param_i32(n, 4);
    const int64_t T = n->src[0]->ne[2];
    const float par[6] = { param_f32(n, 5), param_f32(n, 6), param_f32(n, 7),
                           param_f32(n, 8), param_f32(n, 9), param_f32(n, 10) };
    const size_t tb = (size_t) (T * n_dims) * sizeof(float);
    if (tb > ctx.rope_cap) {
        cudaFree(ctx.rope_table);
        ctx.rope_table = nullptr;
        ctx.rope_cap = 0;
        if (cudaMalloc(&ctx.rope_table, tb) != cudaSuccess) {
            err = "cannot allocate the rope table";
            return nullptr;
        }
        ctx.rope_cap = tb;
    }
    const int32_t *pos = (const int32_t *) device_in(ctx, n->src[1], st);
    const float *ff = (const float *) device_in(ctx, n->src[2], st);
    if (zest_rope_table(pos, T, n_dims, n_ctx_orig, par, ff, ctx.rope_table, st)) {
        err = std::string(n->name) + ": " + zest_last_error();
        return nullptr;
    }
    return ctx.rope_table;
}

bool run_rope_job(context &ctx, const rope_job &r, std::string &err) {
    cudaStream_t st = (cudaStream_t) zest_stream(ctx.npu);
    const float *table = rope_table_of(ctx, r.rope, st, err);
    if (!table) return false;
    const ggml_tensor *a = r.norm->src[0];
    if (zest_norm_rope((const float *) a->data, a->ne[2], a->ne[1], a->ne[0], param_f32(r.norm, 0),
                       (const float *) r.mul->src[1]->data, param_i32(r.rope, 1), param_i32(r.rope, 2), table,
                       (float *) r.rope->data, nullptr, st)) {
        err = std::string(r.rope->name) + ": " + zest_last_error();
        return false;
    }
    ctx.small_ops += 3;
    return true;
}

// One job through zest_mul_mat_group_ex (device memory throughout).
bool run_mm_job(context &ctx, const mm_job &j, std::string &err) {
    std::vector<zest_wkey> keys;
    std::vector<int> fused;
    std::vector<zest_mm_out> outs;
    if (j.glu) {
        zest_wkey key;
        if (!ensure_fused(ctx, *j.glu, key, err)) return false;
        keys.push_back(key);
        fused.push_back(1);
        ggml_tensor *g = j.glu->glu;
        uint16_t *an = nullptr;
        if (j.a_next) {
            const size_t need = (size_t) ((g->ne[1] + 127) / 128 * 128) * (size_t) g->ne[0] * 2;
            if (need > ctx.a_next_cap) {
                cudaFree(ctx.a_next);
                ctx.a_next = nullptr;
                ctx.a_next_cap = 0;
                if (cudaMalloc(&ctx.a_next, need) != cudaSuccess) {
                    err = "cannot allocate the packed hand-off";
                    return false;
                }
                ctx.a_next_cap = need;
            }
            an = (uint16_t *) ctx.a_next;
        }
        outs.push_back({ j.a_next ? nullptr : (float *) g->data, nullptr, an });
        ctx.matmuls += j.glu->up ? 2 : 1;
        ctx.fused++;
    } else {
        for (size_t i = 0; i < j.mms.size(); i++) {
            const ggml_tensor *w = j.mms[i]->src[0];
            if (!ensure_weight(ctx, w, err)) return false;
            keys.push_back({ w->buffer, w->data, (int) w->type, w->ne[0], w->ne[1] });
            fused.push_back(0);
            const ggml_tensor *a = j.add[i];
            const ggml_tensor *r = a ? (a->src[0] == j.mms[i] ? a->src[1] : a->src[0]) : nullptr;
            outs.push_back({ (float *) (a ? a->data : j.mms[i]->data), r ? (const float *) r->data : nullptr, nullptr });
        }
        ctx.matmuls += (int64_t) j.mms.size();
        ctx.grouped += (int64_t) j.mms.size() - 1;
    }
    const ggml_tensor *x = j.mms[0]->src[1];
    const float *xin = j.norm ? (const float *) j.norm->src[0]->data : (const float *) x->data;
    const float eps = j.norm ? param_f32(j.norm, 0) : -1.0f;
    const float *nw = j.mul ? (const float *) j.mul->src[1]->data : nullptr;
    const uint16_t *a = j.packed_in ? (const uint16_t *) ctx.a_next : nullptr;
    if (zest_mul_mat_group_ex(ctx.npu, (int) keys.size(), keys.data(), fused.data(), j.packed_in ? nullptr : xin,
                              eps, nw, nullptr, a, x->ne[1], outs.data())) {
        err = std::string(j.mms[0]->name) + ": " + zest_last_error();
        return false;
    }
    if (j.norm) ctx.small_ops += j.mul ? 2 : 1;
    for (const ggml_tensor *ad : j.add)
        if (ad) ctx.small_ops++;
    return true;
}

// Whether a job must take the one-op-at-a-time route: any of its tensors in
// host memory (staged by mul_mat / mul_mat_group), and nothing fused.
bool plain_job(const mm_job &j) {
    return !j.glu && !j.norm && !j.a_next && !j.packed_in &&
           std::all_of(j.add.begin(), j.add.end(), [](const ggml_tensor *a) { return a == nullptr; });
}

enum ggml_status backend_graph_compute(ggml_backend_t backend, ggml_cgraph *cgraph) {
    context &ctx = *(context *) backend->context;
    budget_report();
    say_notes();
    if (trace()) trace_piece(cgraph);
    const auto t0 = std::chrono::steady_clock::now();
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cuda_device());
    ctx.stage_next = 0;
    enum ggml_status status = GGML_STATUS_SUCCESS;
    const piece_nodes piece = collect_piece(cgraph, true);
    const std::vector<ggml_tensor *> &nodes = piece.nodes;
    const piece_plan plan = plan_piece(nodes, piece);
    cudaStream_t st = (cudaStream_t) zest_stream(ctx.npu);
    for (size_t k = 0; k < nodes.size(); k++) {
        ggml_tensor *node = nodes[k];
        if (status != GGML_STATUS_SUCCESS) break;
        std::string err;
        bool ok = true;
        if (plan.skip.count(node)) continue;
        if (auto it = plan.job_at.find(node); it != plan.job_at.end()) {
            const mm_job &j = plan.jobs[it->second];
            if (j.glu) {
                const ggml_tensor *x = j.glu->gate->src[1];
                if (is_host(x) || is_host(j.glu->glu)) {
                    err = "a fused SwiGLU with host-memory operands";
                    ok = false;
                } else {
                    ok = run_mm_job(ctx, j, err);
                }
            } else if (plain_job(j)) {
                ok = j.mms.size() > 1 ? mul_mat_group(ctx, j.mms, err) : mul_mat(ctx, j.mms[0], err);
            } else {
                ok = run_mm_job(ctx, j, err);
            }
        } else if (auto ri = plan.rope_at.find(node); ri != plan.rope_at.end()) {
            ok = run_rope_job(ctx, plan.ropes[ri->second], err);
        } else {
            ok = small_op(ctx, node, err);
        }
        if (!ok) {
            failed(err);
            status = GGML_STATUS_FAILED;
        }
    }
    if (cudaStreamSynchronize(st) != cudaSuccess && status == GGML_STATUS_SUCCESS) {
        failed(std::string("a kernel failed: ") + cudaGetErrorString(cudaGetLastError()));
        status = GGML_STATUS_FAILED;
    }
    cudaSetDevice(prev);
    ctx.compute_ms += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    ctx.pieces++;
    if (trace() && ctx.matmuls >= 196) {
        zest_times t = {};
        zest_take_times(ctx.npu, &t);
        fprintf(stderr,
                "xdna times, %lld matmuls (%lld grouped, %lld fused) in %lld pieces: all %.1f ms | copies %.1f, "
                "encode %.1f, GEMM %.1f (%d calls), weight copies %.1f ms\n",
                (long long) ctx.matmuls, (long long) ctx.grouped, (long long) ctx.fused, (long long) ctx.pieces,
                ctx.compute_ms, t.copy_ms, t.encode_ms, t.gemm_ms, t.calls, ctx.copy_ms);
        ctx.compute_ms = ctx.copy_ms = 0;
        ctx.matmuls = ctx.pieces = ctx.grouped = ctx.fused = 0;
    }
    return status;
}

// Weight copies made as soon as llama.cpp plans a piece
// (src/ggml-zest.cpp:928-965): the first prompt then need not wait for them.
// Their conversions are queued on the service's load stream and run while
// llama.cpp carries on (the reference's background builder, :261-330); the
// first matmul that uses a copy waits for it on the GPU.
// GGML_XDNA_COPY_AT_LOAD=0 leaves them to the first prompt.
void backend_graph_optimize(ggml_backend_t backend, ggml_cgraph *cgraph, ggml_backend_graph_optimize_params *) {
    static const bool at_load = env_int("GGML_XDNA_COPY_AT_LOAD", 1) != 0;
    if (!at_load || g_broken) return;
    context &ctx = *(context *) backend->context;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cuda_device());
    // the copies the piece will use, as running it would make them
    // (xdna_exec_weights, src/xdna-exec.cpp:435-448): fused gate/up pairs once
    const piece_nodes piece = collect_piece(cgraph, false);
    const std::vector<ggml_tensor *> &nodes = piece.nodes;
    std::unordered_map<const ggml_tensor *, const fusion *> fused;
    const std::vector<fusion> fusions = blocks() ? find_fusions(nodes, piece) : std::vector<fusion>();
    for (const fusion &f : fusions) {
        fused[f.gate] = &f;
        if (f.up) fused[f.up] = nullptr;
    }
    for (const ggml_tensor *node : nodes) {
        if (!op_is(node, "MUL_MAT")) continue;
        const ggml_tensor *w = node->src[0];
        // llama.cpp's memory-fitting trial loads no weight data: nothing to build
        if (!w || !w->data || !w->buffer || ggml_backend_buffer_get_usage(w->buffer) != GGML_BACKEND_BUFFER_USAGE_WEIGHTS)
            continue;
        std::string err;
        bool ok = true;
        auto it = fused.find(node);
        if (it == fused.end()) {
            ok = ensure_weight(ctx, w, err);
        } else if (it->second) {
            zest_wkey key;
            ok = ensure_fused(ctx, *it->second, key, err);
        }
        if (!ok) {
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
    // weight copies from device-resident weights are built on the service's
    // load stream; a claimed matmul waits for its copy on the GPU
    // (GGML_ZEST_ASYNC_COPIES=0: built before graph_optimize returns)
    zest_set_load_async(ctx->npu, env_int("GGML_ZEST_ASYNC_COPIES", 1) != 0 ? 1 : 0);
    // the IQ3_S converter's codebook, as the host ggml dequantises it
    const std::vector<uint32_t> &grid = iq3s_codebook();
    if (!grid.empty() && zest_load_iq3s_grid(grid.data())) {
        log_line("", std::string("cannot load the IQ3_S codebook: ") + zest_last_error());
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
    if (blocks() || trace()) note_readers(op);
    note_model(op);
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

int ggml_zest_piece_groups(ggml_cgraph *cgraph, int *sizes, int max_groups) {
    const piece_nodes piece = collect_piece(cgraph, false);
    const std::unordered_map<const ggml_tensor *, bool> none;
    const auto groups = find_groups(piece.nodes, none);
    for (int i = 0; i < (int) groups.size() && i < max_groups; i++) sizes[i] = (int) groups[i].size();
    return (int) groups.size();
}

int ggml_zest_budget_plan(double limit_gb, const ggml_tensor *const *weights, int n, int *taken) {
    budget_t b;
    b.started = true;
    b.limit = limit_gb * GB;
    int count = 0;
    for (int i = 0; i < n; i++) {
        taken[i] = budget_decide(b, weights[i]) ? 1 : 0;
        count += taken[i];
    }
    // a weight taken before the cut but whose layer the cut gave back
    for (int i = 0; i < n; i++) {
        const ggml_tensor *w = weights[i];
        const wkey key = { w->buffer, w->data, (int) w->type, w->ne[0], w->ne[1] };
        if (taken[i] && !b.in.count(key)) {
            taken[i] = 0;
            count--;
        }
    }
    return count;
}

int ggml_zest_piece_plan(ggml_cgraph *cgraph, int *counts) {
    const piece_nodes piece = collect_piece(cgraph, true);
    const piece_plan pl = plan_piece(piece.nodes, piece);
    for (int i = 0; i < 6; i++) counts[i] = pl.counts[i];
    return (int) pl.jobs.size();
}

int ggml_zest_iq3s_codebook(uint32_t *out) {
    const std::vector<uint32_t> &g = iq3s_codebook();
    if (g.empty()) return 0;
    if (out) memcpy(out, g.data(), g.size() * sizeof(uint32_t));
    return 1;
}

int ggml_zest_model_notes(char *out, int n) {
    const std::string s = model_notes();
    if (out && n > 0) snprintf(out, (size_t) n, "%s", s.c_str());
    return (int) s.size();
}

int ggml_zest_piece_fusions(ggml_cgraph *cgraph) {
    const piece_nodes piece = collect_piece(cgraph, false);
    return (int) find_fusions(piece.nodes, piece).size();
}

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
