/*
 * Stand-in for the ggml declarations that the reference's src/xdna-ref.cpp
 * and src/xdna-exec.cpp use, so those files compile unmodified into the
 * oracle's reference build (oracle/Makefile). ggml itself (llama.cpp tag
 * b10944) is fetched over the network by the reference's
 * tools/fetch-llama.sh and is not present. Only what those two files touch
 * is here: the tensor's fields, the op and GLU ids they switch on (their
 * numeric values are this stand-in's own, except the GLU kinds, which
 * follow ggml's order because tests pass them through), and a few shape
 * helpers (ggml_stub.cpp). to_float is the oracle's restated dequantiser.
 * TEST INFRASTRUCTURE ONLY.
 */
#pragma once

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#define GGML_RESTRICT __restrict
#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10
#define GGML_MAX_OP_PARAMS 64
#define GGML_MAX_NAME 64

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q6_K = 14,
    GGML_TYPE_IQ3_S = 21,
    GGML_TYPE_I32 = 26,
};

enum ggml_op {
    GGML_OP_NONE = 0,
    GGML_OP_ADD,
    GGML_OP_MUL,
    GGML_OP_SCALE,
    GGML_OP_RMS_NORM,
    GGML_OP_MUL_MAT,
    GGML_OP_RESHAPE,
    GGML_OP_VIEW,
    GGML_OP_PERMUTE,
    GGML_OP_TRANSPOSE,
    GGML_OP_ROPE,
    GGML_OP_GLU,
    GGML_OP_COUNT,
};

enum ggml_glu_op {
    GGML_GLU_OP_REGLU = 0,
    GGML_GLU_OP_GEGLU = 1,
    GGML_GLU_OP_SWIGLU = 2,
    GGML_GLU_OP_SWIGLU_OAI = 3,
    GGML_GLU_OP_GEGLU_ERF = 4,
    GGML_GLU_OP_GEGLU_QUICK = 5,
};

#define GGML_ROPE_TYPE_NORMAL 0
#define GGML_ROPE_TYPE_NEOX 2

struct ggml_backend_buffer;

struct ggml_tensor {
    enum ggml_type type;
    struct ggml_backend_buffer *buffer;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    enum ggml_op op;
    int32_t op_params[GGML_MAX_OP_PARAMS / sizeof(int32_t)];
    int32_t flags;
    struct ggml_tensor *src[GGML_MAX_SRC];
    struct ggml_tensor *view_src;
    size_t view_offs;
    void *data;
    char name[GGML_MAX_NAME];
    void *extra;
};

struct ggml_cgraph;

typedef void (*ggml_to_float_t)(const void *GGML_RESTRICT x, float *GGML_RESTRICT y, int64_t k);

struct ggml_type_traits {
    const char *type_name;
    ggml_to_float_t to_float;
};

#ifdef __cplusplus
extern "C" {
#endif
const struct ggml_type_traits *ggml_get_type_traits(enum ggml_type type);
int64_t ggml_nelements(const struct ggml_tensor *t);
int64_t ggml_nrows(const struct ggml_tensor *t);
size_t ggml_nbytes(const struct ggml_tensor *t);
bool ggml_is_contiguous(const struct ggml_tensor *t);
bool ggml_are_same_shape(const struct ggml_tensor *a, const struct ggml_tensor *b);
const char *ggml_op_name(enum ggml_op op);
void ggml_rope_yarn_corr_dims(int n_dims, int n_ctx_orig, float freq_base, float beta_fast, float beta_slow,
                              float dims[2]);
#ifdef __cplusplus
}
#endif
