// C entry points over the reference's own block executor (src/xdna-exec.cpp,
// compiled unmodified into oracle/_ref/libzest_ref.so by oracle/Makefile):
// each builds a one- to three-op piece of ggml tensors over the caller's
// arrays and runs it through xdna_exec_piece with no NPU, the reference's
// host path, so the small ops are the reference's run_rows
// (src/xdna-exec.cpp:253-346) and its rope table (:199-239).
// TEST INFRASTRUCTURE ONLY: the golden-vector script and the parity tests
// call these; the product never does.
#include "ggml.h"
#include "ggml-impl.h"
#include "thread_pool.h"
#include "xdna-exec.h"

#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace {

struct piece_builder {
    std::vector<ggml_tensor *> all;
    std::vector<ggml_tensor *> nodes;
    std::vector<void *> blocks;

    ~piece_builder() {
        for (ggml_tensor *t : all) delete t;
        for (void *p : blocks) free(p);
    }

    // a contiguous tensor of 4-byte elements over `data`, ne = [n0, n1, n2]
    ggml_tensor *tensor(ggml_type type, int64_t n0, int64_t n1, int64_t n2, void *data, const char *name) {
        ggml_tensor *t = new ggml_tensor();
        t->type = type;
        t->ne[0] = n0;
        t->ne[1] = n1;
        t->ne[2] = n2;
        t->ne[3] = 1;
        t->nb[0] = 4;
        for (int i = 1; i < GGML_MAX_DIMS; i++) t->nb[i] = t->nb[i - 1] * (size_t) t->ne[i - 1];
        t->op = GGML_OP_NONE;
        t->data = data;
        snprintf(t->name, sizeof t->name, "%s", name);
        all.push_back(t);
        return t;
    }

    ggml_tensor *op(ggml_op kind, ggml_tensor *shape_of, void *out, std::initializer_list<ggml_tensor *> srcs,
                    const int32_t *params, int n_params, const char *name) {
        ggml_tensor *t = tensor(GGML_TYPE_F32, shape_of->ne[0], shape_of->ne[1], shape_of->ne[2], out, name);
        t->op = kind;
        int j = 0;
        for (ggml_tensor *s : srcs) t->src[j++] = s;
        if (params) memcpy(t->op_params, params, (size_t) n_params * sizeof(int32_t));
        nodes.push_back(t);
        return t;
    }

    // Runs the nodes as one piece on the host; the last node's result is
    // the one written back (the others stay inside the piece).
    int run(int n_threads, char *err, int err_len) {
        ggml_cgraph g = {};
        g.n_nodes = (int) nodes.size();
        g.nodes = nodes.data();
        g.size = g.n_nodes;
        const ggml_tensor *last = nodes.back();
        xdna_io io;
        io.read = [](const ggml_tensor *t, void *dst) { memcpy(dst, t->data, ggml_nbytes(t)); };
        io.write = [](ggml_tensor *t, const void *src) { memcpy(t->data, src, ggml_nbytes(t)); };
        io.param = [](const ggml_tensor *t) { return (const float *) t->data; };
        io.alloc = [this](size_t n) {
            void *p = malloc(n ? n : 1);
            blocks.push_back(p);
            return p;
        };
        io.needed_outside = [last](const ggml_tensor *t, const ggml_cgraph *) { return t == last; };
        io.ensure_weight = [](const ggml_tensor *, std::string &e) {
            e = "no matmuls here";
            return false;
        };
        io.ensure_fused = [](const ggml_tensor *, const ggml_tensor *, std::string &e) {
            e = "no matmuls here";
            return false;
        };
        io.weight_bytes = [](const ggml_tensor *) -> const void * { return nullptr; };
        thread_pool pool(n_threads > 0 ? n_threads : 1);
        std::string e;
        const bool ok = xdna_exec_piece(&g, nullptr, pool, io, 1, e);
        if (!ok && err && err_len > 0) snprintf(err, (size_t) err_len, "%s", e.c_str());
        return ok ? 0 : -1;
    }
};

int32_t f32_bits(float v) {
    int32_t b;
    memcpy(&b, &v, 4);
    return b;
}

}  // namespace

extern "C" {

// y[rows][d] = RMS_NORM(x, eps)
int zr_rms_norm(float *x, int64_t rows, int64_t d, float eps, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, d, rows, 1, x, "x");
    const int32_t p[1] = { f32_bits(eps) };
    b.op(GGML_OP_RMS_NORM, xt, y, { xt }, p, 1, "norm");
    return b.run(n_threads, nullptr, 0);
}

// y = x * w, w one row of d broadcast over every row
int zr_mul_row(float *x, float *w, int64_t rows, int64_t d, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, d, rows, 1, x, "x");
    ggml_tensor *wt = b.tensor(GGML_TYPE_F32, d, 1, 1, w, "w");
    b.op(GGML_OP_MUL, xt, y, { xt, wt }, nullptr, 0, "mul");
    return b.run(n_threads, nullptr, 0);
}

// y = x + b: b [rows][d], or (bias_row) one row of d broadcast
int zr_add(float *x, float *bb, int bias_row, int64_t rows, int64_t d, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, d, rows, 1, x, "x");
    ggml_tensor *bt = b.tensor(GGML_TYPE_F32, d, bias_row ? 1 : rows, 1, bb, "b");
    b.op(GGML_OP_ADD, xt, y, { xt, bt }, nullptr, 0, "add");
    return b.run(n_threads, nullptr, 0);
}

// y = x * s + bias
int zr_scale(float *x, int64_t rows, int64_t d, float s, float bias, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, d, rows, 1, x, "x");
    const int32_t p[2] = { f32_bits(s), f32_bits(bias) };
    b.op(GGML_OP_SCALE, xt, y, { xt }, p, 2, "scale");
    return b.run(n_threads, nullptr, 0);
}

// GLU of kind (ggml_glu_op). Split: g and u [rows][f]. One tensor (u null):
// g [rows][2f], gate then up, or up then gate when swapped.
int zr_glu(int kind, int swapped, float *g, float *u, int64_t rows, int64_t f, float *y, int n_threads) {
    piece_builder b;
    const int32_t p[2] = { kind, swapped };
    if (u) {
        ggml_tensor *gt = b.tensor(GGML_TYPE_F32, f, rows, 1, g, "g");
        ggml_tensor *ut = b.tensor(GGML_TYPE_F32, f, rows, 1, u, "u");
        b.op(GGML_OP_GLU, gt, y, { gt, ut }, p, 2, "glu");
    } else {
        ggml_tensor *gt = b.tensor(GGML_TYPE_F32, 2 * f, rows, 1, g, "g");
        ggml_tensor *shape = b.tensor(GGML_TYPE_F32, f, rows, 1, nullptr, "shape");
        b.op(GGML_OP_GLU, shape, y, { gt }, p, 2, "glu");
    }
    return b.run(n_threads, nullptr, 0);
}

// ROPE over x [T][heads][hd] at positions pos[T]; par: freq_base,
// freq_scale, ext_factor, attn_factor, beta_fast, beta_slow; ff: n_dims/2
// frequency factors or null.
int zr_rope(float *x, int64_t T, int64_t heads, int64_t hd, int32_t *pos, int n_dims, int mode, int n_ctx_orig,
            const float *par, float *ff, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, hd, heads, T, x, "x");
    ggml_tensor *pt = b.tensor(GGML_TYPE_I32, T, 1, 1, pos, "pos");
    ggml_tensor *ft = ff ? b.tensor(GGML_TYPE_F32, n_dims / 2, 1, 1, ff, "factors") : nullptr;
    int32_t p[16] = {};
    p[1] = n_dims;
    p[2] = mode;
    p[4] = n_ctx_orig;
    for (int i = 0; i < 6; i++) p[5 + i] = f32_bits(par[i]);
    if (ft) b.op(GGML_OP_ROPE, xt, y, { xt, pt, ft }, p, 16, "rope");
    else b.op(GGML_OP_ROPE, xt, y, { xt, pt }, p, 16, "rope");
    return b.run(n_threads, nullptr, 0);
}

// RMS_NORM then MUL by a weight row, as one piece (the attention and FFN
// norms): y = norm(x) * w, x [rows][d]
int zr_norm_mul(float *x, int64_t rows, int64_t d, float eps, float *w, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, d, rows, 1, x, "x");
    ggml_tensor *wt = b.tensor(GGML_TYPE_F32, d, 1, 1, w, "w");
    const int32_t p[1] = { f32_bits(eps) };
    std::vector<float> mid((size_t) (rows * d));
    ggml_tensor *n = b.op(GGML_OP_RMS_NORM, xt, mid.data(), { xt }, p, 1, "norm");
    b.op(GGML_OP_MUL, xt, y, { n, wt }, nullptr, 0, "mul");
    return b.run(n_threads, nullptr, 0);
}

// Per-head RMS_NORM, MUL by a head-wide weight, then ROPE, as one piece
// (Qwen3's q and k): x [T][heads][hd], w [hd]
int zr_norm_mul_rope(float *x, int64_t T, int64_t heads, int64_t hd, float eps, float *w, int32_t *pos, int n_dims,
                     int mode, int n_ctx_orig, const float *par, float *ff, float *y, int n_threads) {
    piece_builder b;
    ggml_tensor *xt = b.tensor(GGML_TYPE_F32, hd, heads, T, x, "x");
    ggml_tensor *wt = b.tensor(GGML_TYPE_F32, hd, 1, 1, w, "w");
    ggml_tensor *pt = b.tensor(GGML_TYPE_I32, T, 1, 1, pos, "pos");
    ggml_tensor *ft = ff ? b.tensor(GGML_TYPE_F32, n_dims / 2, 1, 1, ff, "factors") : nullptr;
    const int32_t pn[1] = { f32_bits(eps) };
    std::vector<float> mid1((size_t) (T * heads * hd)), mid2((size_t) (T * heads * hd));
    ggml_tensor *n = b.op(GGML_OP_RMS_NORM, xt, mid1.data(), { xt }, pn, 1, "norm");
    ggml_tensor *m = b.op(GGML_OP_MUL, xt, mid2.data(), { n, wt }, nullptr, 0, "mul");
    int32_t p[16] = {};
    p[1] = n_dims;
    p[2] = mode;
    p[4] = n_ctx_orig;
    for (int i = 0; i < 6; i++) p[5 + i] = f32_bits(par[i]);
    if (ft) b.op(GGML_OP_ROPE, xt, y, { m, pt, ft }, p, 16, "rope");
    else b.op(GGML_OP_ROPE, xt, y, { m, pt }, p, 16, "rope");
    return b.run(n_threads, nullptr, 0);
}

}  // extern "C"
