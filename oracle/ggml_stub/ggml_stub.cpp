// Bodies for the stand-in ggml.h: the few shape helpers the reference's
// src/xdna-exec.cpp calls, and ggml's YaRN correction range, which comes from
// the oracle's restatement of ggml's published formula (zest_oracle.c), as
// to_float does. TEST INFRASTRUCTURE ONLY.
#include "ggml.h"
#include "zest_oracle.h"

extern "C" {

int64_t ggml_nelements(const struct ggml_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

int64_t ggml_nrows(const struct ggml_tensor *t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

// Every tensor the reference build makes holds 4-byte elements (f32, i32) or
// is a quantised weight row set that xdna-ref.cpp sizes itself.
size_t ggml_nbytes(const struct ggml_tensor *t) {
    size_t n = 0;
    for (int i = 0; i < GGML_MAX_DIMS; i++) n += (size_t) (t->ne[i] - 1) * t->nb[i];
    return n + t->nb[0];
}

bool ggml_is_contiguous(const struct ggml_tensor *t) {
    size_t want = t->nb[0];
    for (int i = 1; i < GGML_MAX_DIMS; i++) {
        want *= (size_t) t->ne[i - 1];
        if (t->ne[i] != 1 && t->nb[i] != want) return false;
    }
    return true;
}

bool ggml_are_same_shape(const struct ggml_tensor *a, const struct ggml_tensor *b) {
    for (int i = 0; i < GGML_MAX_DIMS; i++)
        if (a->ne[i] != b->ne[i]) return false;
    return true;
}

const char *ggml_op_name(enum ggml_op op) {
    static const char *names[GGML_OP_COUNT] = { "NONE", "ADD", "MUL", "SCALE", "RMS_NORM", "MUL_MAT",
                                                "RESHAPE", "VIEW", "PERMUTE", "TRANSPOSE", "ROPE", "GLU" };
    return op >= 0 && op < GGML_OP_COUNT ? names[op] : "UNKNOWN";
}

void ggml_rope_yarn_corr_dims(int n_dims, int n_ctx_orig, float freq_base, float beta_fast, float beta_slow,
                              float dims[2]) {
    zo_rope_corr_dims(n_dims, n_ctx_orig, freq_base, beta_fast, beta_slow, dims);
}

}  // extern "C"
