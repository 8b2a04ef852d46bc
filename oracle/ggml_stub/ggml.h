/*
 * Stand-in for the few ggml declarations that the reference's
 * src/xdna-ref.cpp uses, so that file compiles unmodified into the oracle's
 * reference build (oracle/Makefile). ggml itself (llama.cpp tag b10944) is
 * fetched over the network by the reference's tools/fetch-llama.sh and is not
 * present; to_float here is the oracle's restated dequantiser.
 * TEST INFRASTRUCTURE ONLY.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#define GGML_RESTRICT __restrict

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q6_K = 14,
    GGML_TYPE_IQ3_S = 21,
};

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];
    size_t nb[4];
    void *data;
};

typedef void (*ggml_to_float_t)(const void *GGML_RESTRICT x, float *GGML_RESTRICT y, int64_t k);

struct ggml_type_traits {
    const char *type_name;
    ggml_to_float_t to_float;
};

#ifdef __cplusplus
extern "C" {
#endif
const struct ggml_type_traits *ggml_get_type_traits(enum ggml_type type);
#ifdef __cplusplus
}
#endif
