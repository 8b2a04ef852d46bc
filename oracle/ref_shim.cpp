// C entry points over the reference's own packer and CPU matmul, compiled
// unmodified from the reference tree (src/npu/bfp16_pack.cpp,
// src/xdna-ref.cpp) into oracle/_ref/libzest_ref.so by oracle/Makefile.
// TEST INFRASTRUCTURE ONLY: the parity tests and bench.py's cpu_baseline /
// reference arm call these; the product never does.
#include "bfp16_pack.h"
#include "ggml.h"
#include "xdna-ref.h"
#include "zest_oracle.h"

#include <cstring>
#include <vector>

extern "C" {

// ggml's to_float for the stand-in ggml.h: the oracle's restated dequantisers
static void tf_f16(const void *x, float *y, int64_t k) { zo_dequant_row(ZO_TYPE_F16, x, y, k); }
static void tf_q8_0(const void *x, float *y, int64_t k) { zo_dequant_row(ZO_TYPE_Q8_0, x, y, k); }
static void tf_q4_k(const void *x, float *y, int64_t k) { zo_dequant_row(ZO_TYPE_Q4_K, x, y, k); }
static void tf_q6_k(const void *x, float *y, int64_t k) { zo_dequant_row(ZO_TYPE_Q6_K, x, y, k); }
static void tf_iq3_s(const void *x, float *y, int64_t k) { zo_dequant_row(ZO_TYPE_IQ3_S, x, y, k); }

const struct ggml_type_traits *ggml_get_type_traits(enum ggml_type type) {
    static const ggml_type_traits f32 = { "f32", nullptr }, f16 = { "f16", tf_f16 }, q8 = { "q8_0", tf_q8_0 },
                                  q4k = { "q4_K", tf_q4_k }, q6k = { "q6_K", tf_q6_k }, iq3s = { "iq3_s", tf_iq3_s };
    switch (type) {
        case GGML_TYPE_F32: return &f32;
        case GGML_TYPE_F16: return &f16;
        case GGML_TYPE_Q8_0: return &q8;
        case GGML_TYPE_Q4_K: return &q4k;
        case GGML_TYPE_Q6_K: return &q6k;
        case GGML_TYPE_IQ3_S: return &iq3s;
    }
    return nullptr;
}

static bfp16_tiling tiling(int m, int k, int n, int cols) {
    bfp16_tiling t;
    t.m = m; t.k = k; t.n = n; t.cols = cols;
    return t;
}

void zr_encode_block(const float *x, uint8_t *out) { bfp16_encode_block(x, out); }
void zr_decode_block(const uint8_t *in, float *x) { bfp16_decode_block(in, x); }

void zr_pack_a(const float *x, int64_t M, int64_t K, int m, int k, uint8_t *out, int n_threads) {
    std::vector<uint8_t> v;
    bfp16_pack_a(x, M, K, tiling(m, k, 64, 8), v, n_threads);
    memcpy(out, v.data(), v.size());
}

void zr_pack_b(const float *w, int64_t N, int64_t K, int n, int k, int cols, uint8_t *out, int n_threads) {
    std::vector<uint8_t> v;
    bfp16_pack_b(w, N, K, tiling(128, k, n, cols), v, n_threads);
    memcpy(out, v.data(), v.size());
}

void zr_unpack_a(const uint8_t *in, int64_t M, int64_t K, int m, int k, float *x) {
    bfp16_unpack_a(in, M, K, tiling(m, k, 64, 8), x);
}

void zr_unpack_b(const uint8_t *in, int64_t N, int64_t K, int n, int k, int cols, float *w) {
    bfp16_unpack_b(in, N, K, tiling(128, k, n, cols), w);
}

void zr_interleave_gate_up(const float *gate, const float *up, int64_t F, int64_t K, float *out) {
    bfp16_interleave_gate_up(gate, up, F, K, out);
}

// xdna_ref_mul_mat (src/xdna-ref.cpp:62-97) on ggml-shaped tensors: weight
// src0 [K x N] of `type` (raw GGUF rows), src1 f32 [K x M], dst f32 [N x M].
void zr_mul_mat(int type, const void *w, int64_t N, int64_t K, const float *x, int64_t M, float *y, int n_threads) {
    ggml_tensor s0 = {}, s1 = {}, d = {};
    s0.type = (ggml_type) type;
    s0.ne[0] = K; s0.ne[1] = N; s0.ne[2] = 1; s0.ne[3] = 1;
    const size_t rb = (size_t) zo_row_bytes(type, K);
    s0.nb[0] = type == GGML_TYPE_F32 ? 4 : 1; s0.nb[1] = rb; s0.nb[2] = rb * N; s0.nb[3] = rb * N;
    s0.data = (void *) w;
    s1.type = GGML_TYPE_F32;
    s1.ne[0] = K; s1.ne[1] = M; s1.ne[2] = 1; s1.ne[3] = 1;
    s1.nb[0] = 4; s1.nb[1] = 4 * K; s1.nb[2] = 4 * K * M; s1.nb[3] = s1.nb[2];
    s1.data = (void *) x;
    d.type = GGML_TYPE_F32;
    d.ne[0] = N; d.ne[1] = M; d.ne[2] = 1; d.ne[3] = 1;
    d.nb[0] = 4; d.nb[1] = 4 * N; d.nb[2] = 4 * N * M; d.nb[3] = d.nb[2];
    d.data = y;
    xdna_ref_mul_mat(&s0, &s1, &d, n_threads);
}

}
