/*
 * CPU oracle for the prefill MUL_MAT path: TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's arithmetic, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker.
 * Nothing in the product (the CUDA library, the ggml backend) links or calls
 * it. Each function cites the reference file:line it restates
 * (Cyronius/ggml-xdna paths).
 *
 * Parity pins: the bfp16 codec and tile layouts are checked byte for byte
 * against the reference's own src/npu/bfp16_pack.cpp compiled unmodified into
 * oracle/_ref (oracle/Makefile) and against the reference's test
 * tests/test-bfp16-pack.cpp run there. The GGUF dequantisers restate ggml's
 * published block formats (llama.cpp/ggml tag b10944, not vendored in the
 * reference); they are cross-checked against gguf-py's numpy dequantisers.
 */
#ifndef ZEST_ORACLE_H
#define ZEST_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZO_BLOCK_BYTES 9

/* ggml_type values (the GGUF file-format ids) the path handles */
enum {
    ZO_TYPE_F32 = 0,
    ZO_TYPE_F16 = 1,
    ZO_TYPE_Q8_0 = 8,
    ZO_TYPE_Q4_K = 12,
    ZO_TYPE_Q6_K = 14,
    ZO_TYPE_IQ3_S = 21,
};

/* tile sizes of the packed operands (src/npu/bfp16_pack.h:37-41) */
typedef struct {
    int m, k, n, cols;
} zo_tiling;

/* --- bfp16 codec (src/npu/bfp16_pack.cpp:85-144) ------------------------- */
void zo_encode_block(const float *x, uint8_t *out);
void zo_decode_block(const uint8_t *in, float *x);
/* n blocks of 8 values, row-major, to/from 9n bytes in order */
void zo_encode_blocks(const float *x, int64_t n, uint8_t *out);
void zo_decode_blocks(const uint8_t *in, int64_t n, float *x);

/* --- tile layouts (src/npu/bfp16_pack.cpp:29-83,146-186) ----------------- */
size_t zo_a_offset(int64_t r, int64_t cb, int64_t K, const zo_tiling *t);
size_t zo_b_offset(int64_t r, int64_t cb, int64_t N, int64_t K, const zo_tiling *t);
void zo_pack_a(const float *x, int64_t M, int64_t K, const zo_tiling *t, uint8_t *out);
void zo_pack_b(const float *w, int64_t N, int64_t K, const zo_tiling *t, uint8_t *out);
void zo_unpack_a(const uint8_t *in, int64_t M, int64_t K, const zo_tiling *t, float *x);
void zo_unpack_b(const uint8_t *in, int64_t N, int64_t K, const zo_tiling *t, float *w);
/* src/npu/bfp16_pack.cpp:231-237 */
void zo_interleave_gate_up(const float *gate, const float *up, int64_t F, int64_t K, float *out);

/* --- GGUF dequantisers (ggml to_float; called at src/xdna-ref.cpp:44,
 *     src/xdna-npu.cpp:345) ---------------------------------------------- */
float zo_fp16_to_fp32(uint16_t h);
uint16_t zo_fp32_to_fp16(float f);
int64_t zo_row_bytes(int type, int64_t k);
/* the IQ3_S codebook (512 entries of four magnitudes), loaded at run time */
void zo_set_iq3s_grid(const uint32_t *grid512);
int zo_dequant_row(int type, const void *raw, float *y, int64_t k);
int zo_dequant(int type, const void *raw, int64_t rows, int64_t k, float *y);

/* --- quantisers for synthetic weights (any valid encoding will do: parity
 *     is on the dequantised values both sides share) ---------------------- */
int zo_quantize(int type, const float *x, int64_t rows, int64_t k, void *raw);

/* --- reference matmul (src/xdna-ref.cpp:10-60): Y[m][n] = sum_k W[n][k] X[m][k],
 *     float accumulation in k order --------------------------------------- */
void zo_mul_mat(const float *W, int64_t N, const float *X, int64_t M, int64_t K, float *Y, int n_threads);
void zo_mul_mat_f64(const float *W, int64_t N, const float *X, int64_t M, int64_t K, double *Y, int n_threads);

/* --- output epilogues (kernels/bfp16_gemm/aie_kernels/aie2p/mm_bfp_acc.cc:138-278) */
float zo_round_bf16(float x);
float zo_swiglu_bf16(float g, float u);

/* --- the block executor's small ops (src/xdna-exec.cpp:253-346), float
 *     arithmetic in the reference's order; rows are contiguous ne0 runs --- */
/* ggml_glu_op ids */
enum { ZO_GLU_REGLU = 0, ZO_GLU_GEGLU = 1, ZO_GLU_SWIGLU = 2, ZO_GLU_GEGLU_ERF = 4, ZO_GLU_GEGLU_QUICK = 5 };
/* ggml rope modes */
enum { ZO_ROPE_NORMAL = 0, ZO_ROPE_NEOX = 2 };
void zo_rms_norm(const float *x, int64_t rows, int64_t d, float eps, float *y);
void zo_mul_row(const float *x, const float *w, int64_t rows, int64_t d, float *y);
/* b: same shape as x, or (bias_row) one row of d broadcast over every row */
void zo_add(const float *x, const float *b, int bias_row, int64_t rows, int64_t d, float *y);
void zo_scale(const float *x, int64_t n, float s, float bias, float *y);
/* g and u rows with their own strides (split tensors, or the two halves of
 * one tensor); y rows of f */
void zo_glu(int kind, const float *g, int64_t g_stride, const float *u, int64_t u_stride, int64_t rows, int64_t f,
            float *y);
/* ggml_rope_yarn_corr_dims (ggml's published YaRN correction range) */
void zo_rope_corr_dims(int n_dims, int n_ctx_orig, float freq_base, float beta_fast, float beta_slow, float dims[2]);
/* the per-token cos/sin table, [T][n_dims] (src/xdna-exec.cpp:194-239);
 * par = freq_base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow */
void zo_rope_table(const int32_t *pos, int64_t T, int n_dims, int n_ctx_orig, const float *par, const float *ff,
                   float *table);
/* x [T][heads][d] -> y, rotating the first n_dims of each head */
void zo_rope(const float *x, int64_t T, int64_t heads, int64_t d, int n_dims, int mode, const float *table, float *y);

/* --- the start-up self-test's operands (src/xdna-npu.cpp:142-152) -------- */
void zo_selftest_operands(int64_t M, int64_t K, int64_t N, int8_t *a, int8_t *w);

#ifdef __cplusplus
}
#endif
#endif
