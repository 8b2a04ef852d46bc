/*
 * zest_b200: the B200 (sm_100a) implementation of the Zest add-on's prefill
 * MUL_MAT path, as a C ABI (libzest_b200.so). Plain pointers and sizes only.
 *
 * Two layers:
 *   1. stream-level kernels on device memory, on the caller's CUDA stream
 *      (cudaStream_t passed as void *; NULL = the legacy default stream);
 *   2. the matmul service `zest_npu`, the counterpart of the reference's
 *      class xdna_npu (src/xdna-npu.h:40-136): a per-GPU weight-copy cache
 *      keyed like xdna_npu::wkey and y = x * W^T on host or device buffers.
 *
 * Every function returns 0 on success and -1 on failure, with the reason in
 * zest_last_error() (the reference returns bool and fills std::string &err).
 * No function aborts or throws.
 *
 * Data layouts (the reference's, src/npu/bfp16_pack.h:1-60):
 *   bfp16 block   9 bytes: the largest biased float exponent e of 8 values,
 *                 then 8 int8 mantissas q; value = q * 2^(e - 133)
 *   A operand     activations, rows of K values, in 128-row x 64-column tiles
 *   B operand     weights (N rows of K), per array column c of 8, its 64-row
 *                 groups (c + 8t), each in 64 x 64 tiles
 *   bf16 copies   the same decoded values, row-major [rows][ld], which the
 *                 tensor-core GEMM reads (every bfp16 value is exact in bf16)
 */
#ifndef ZEST_B200_H
#define ZEST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZEST_B200_VERSION 1

/* weight types (ggml_type ids, as GGUF stores them) */
#define ZEST_TYPE_F32 0
#define ZEST_TYPE_F16 1
#define ZEST_TYPE_Q8_0 8
#define ZEST_TYPE_Q4_K 12
#define ZEST_TYPE_Q6_K 14
#define ZEST_TYPE_IQ3_S 21

/* GEMM output modes (kernels/bfp16_gemm/aie_kernels/aie2p/mm_bfp_acc.cc:138-148) */
#define ZEST_MODE_F32 0    /* fp32 as accumulated */
#define ZEST_MODE_BF16 1   /* each value rounded to bf16 (nearest even), returned as f32 */
#define ZEST_MODE_SWIGLU 2 /* SiLU(gate) * up rounded to bf16; N/2 outputs a row */

/* bits of the device error word the GEMM raises */
#define ZEST_ERR_NOT_FINITE 1u /* a result was NaN or infinite */
#define ZEST_ERR_TIMEOUT 2u    /* a bounded wait inside a kernel ran out */

int zest_version(void);
/* Why the last call on this thread failed: the reference's `std::string & err`
 * (xdna_npu::mul_mat and friends, src/xdna-npu.h:40-136). */
const char *zest_last_error(void);

/* ---------------------------------------------------------------------------
 * 1. Stream-level kernels (device pointers)
 * ------------------------------------------------------------------------- */

/* The IQ3_S codebook: ggml's iq3s_grid, 512 entries of four magnitudes packed
 * in a uint32 (host pointer). Needed before converting IQ3_S weights.
 * Replaces: nothing in the reference itself; ggml's to_float for IQ3_S reads
 * the table (called at src/xdna-npu.cpp:345). */
int zest_load_iq3s_grid(const uint32_t *grid512);

/* K2, the activation pack. x: f32 rows [T][ldx]; writes rows [0, m_pad) of
 * the A operand (m_pad a multiple of 128, >= T; rows past T are zeros):
 * a_bfp16 (m_pad*K/8*9 bytes, the reference layout; may be NULL) and/or
 * a_bf16 ([m_pad][ld_bf16] decoded values; may be NULL). K % 64 == 0.
 * Replaces: bfp16_pack_a_into (src/npu/bfp16_pack.h:56-58) and the encode
 * loop of xdna_npu::mul_mat / begin / encode_row (src/xdna-npu.cpp:406-420,
 * 476-515). */
int zest_pack_activations(const float *x, int64_t T, int64_t K, int64_t ldx, int64_t m_pad, uint8_t *a_bfp16,
                          uint16_t *a_bf16, int64_t ld_bf16, void *stream);

/* K1, the weight conversion. raw: GGUF rows of `type` (rows_total rows of K
 * values); converts rows [row0, row0 + N) into a B operand of n_pad rows
 * (n_pad % 512 == 0, rows past N zeros): b_bfp16 (n_pad*K/8*9 bytes, the
 * reference layout; may be NULL) and/or b_bf16 ([n_pad][K]; may be NULL).
 * Replaces: xdna_npu::unpack (ggml to_float) + bfp16_pack_b inside
 * xdna_npu::add_weight (src/xdna-npu.cpp:339-378). */
int zest_convert_weight(int type, const void *raw, int64_t rows_total, int64_t row0, int64_t N, int64_t K,
                        int64_t n_pad, uint8_t *b_bfp16, uint16_t *b_bf16, void *stream);

/* K1 for a fused gate/up pair: 8 gate rows, then the 8 up rows that pair
 * with them, F padded to f_pad (a multiple of 256) -> a B operand of 2*f_pad
 * rows. Rows [row0, row0 + F) of gate and up (rows_total rows each).
 * Replaces: xdna_npu::add_fused (src/xdna-npu.cpp:380-390) with
 * bfp16_interleave_gate_up (src/npu/bfp16_pack.cpp:231-237). */
int zest_convert_gate_up(int type, const void *gate, const void *up, int64_t rows_total, int64_t row0, int64_t F,
                         int64_t K, int64_t f_pad, uint8_t *b_bfp16, uint16_t *b_bf16, void *stream);

/* Launches of K3 (zest_gemm, zest_gemm_group, zest_gemm_segs) whose last
 * waves are cut into stream-K runs (zest_plan_gemm reports which) share one
 * partial-sum workspace per device. The library orders such launches across
 * streams: a launch on another stream than the last one waits for it. A
 * launch being captured into a CUDA graph runs whole tiles when a live
 * launch on another stream may still hold the workspace, or when another
 * stream of the same capture took it; so a graph's own stream-K launches are
 * ordered within the graph, and a graph holding them must not replay while
 * another stream runs one (ZEST_GEMM_SK=0 takes stream-K out). */

/* K3, the GEMM: c[M][ldc] = A[M][K] * B[N][K]^T in fp32 on the tensor cores,
 * then `mode`. In ZEST_MODE_SWIGLU, B comes from zest_convert_gate_up and c
 * gets N/2 values a row. err: a device word the kernel ORs ZEST_ERR_* bits
 * into (the caller clears it).
 * Replaces: the NPU kernel's mm_paired + out_epilogue
 * (kernels/bfp16_gemm/aie_kernels/aie2p/mm_bfp_acc.cc:44-100,258-278) and the
 * host read-back read_row / bfp16_c_row / bfp16_c16_row / all_finite
 * (src/xdna-npu.cpp:59-85, src/npu/bfp16_pack.cpp:188-229). */
int zest_gemm(const uint16_t *a_bf16, int64_t lda, const uint16_t *b_bf16, int64_t ldb, int64_t M, int64_t N,
              int64_t K, int mode, float *c, int64_t ldc, unsigned *err, void *stream);

/* K3 for up to 4 weights that share one A (q, k and v; gate and up) in one
 * launch: c_i[M][ldc_i] = A * B_i^T with B_i of N_i rows and its own mode.
 * The weights' tiles run end to end in one persistent launch, with no kernel
 * tail between them.
 * Replaces: a group of NPU calls submitted as one runlist
 * (xdna_npu::begin / submit, src/xdna-npu.cpp:476-531). */
int zest_gemm_group(const uint16_t *a_bf16, int64_t lda, int64_t M, int64_t K, int n, const uint16_t *const *b_bf16,
                    const int64_t *ldb, const int64_t *N, const int *mode, float *const *c, const int64_t *ldc,
                    unsigned *err, void *stream);

/* One weight of zest_gemm_segs, with what its epilogue fuses. */
typedef struct {
    const uint16_t *b;    /* the weight's bf16 copy, N rows of ldb */
    int64_t ldb, N;
    int mode;             /* ZEST_MODE_* */
    float *c;             /* [M][ldc] output; may be NULL in ZEST_MODE_SWIGLU when a_next is given */
    int64_t ldc;
    const float *residual; /* NULL, or (fp32 and bf16 modes) c = residual + result, [M][ldr]: the ADD
                              that follows o and down in a layer. residual may be c itself */
    int64_t ldr;
    uint16_t *a_next;     /* NULL, or (ZEST_MODE_SWIGLU) the result's K2 operand: the bf16 copy of
                             its bfp16 rounding, [M][lda_next], the next GEMM's A */
    int64_t lda_next;
    float *c_multicast;   /* NULL, or (with c NULL) a multicast address of a buffer [M][ldc] that every
                             GPU of a tensor-parallel group holds: the results are added into all the
                             copies through the NVSwitch (multimem.red), so when every rank's launch has
                             finished each copy holds the sum of the ranks' partial products. The
                             caller zeroes the copies and fences the group before and after */
    int multicast_store;  /* with c_multicast: 1 stores the results into every copy instead of adding
                             them (multimem.st): an N-sharded launch writes its slab of output columns
                             into every GPU's whole [M][N] output (c_multicast points at the slab's
                             first column), the all-gather done by the NVSwitch as the tiles finish.
                             The caller fences the group after the launch, before the copies are read */
    float *const *c_peers; /* NULL, or n_peers pointers, each into another GPU's buffer laid out as c
                              (mapped into this process, e.g. peer pointers of symmetric memory): the
                              epilogue stores every tile there too, by TMA, as it stores it into c. An
                              N-sharded launch's all-gather: c and c_peers point at the slab's first
                              column of every GPU's whole [M][N] output. The caller fences the group
                              after the launch, before the copies are read. Plain stores: no multicast */
    int n_peers;          /* 0 .. ZEST_MAX_PEERS */
    uint16_t *const *c16; /* NULL, or (ZEST_MODE_BF16 only, whose results are bf16 values) n_c16 buffers
                             [M][ldc16] of bf16, this GPU's or other GPUs' (mapped into this process):
                             the epilogue TMA-stores every tile there in bf16, half the bytes of f32.
                             c may then be NULL. An N-sharded launch's all-gather at half the link
                             bytes: each pointer at the slab's first column of a GPU's whole bf16
                             output, which zest_widen_bf16 turns into ggml's f32 after the group's
                             fence. Plain stores: no multicast */
    int n_c16;            /* 0 .. ZEST_MAX_PEERS + 1 */
    int64_t ldc16;        /* a multiple of 8 */
} zest_gemm_seg;
#define ZEST_MAX_PEERS 7

/* dst[i] = the f32 value of the bf16 src[i] (exact), i < n: gathered bf16
 * results back into ggml's f32. src and dst 16-byte aligned.
 * Replaces: the f32 rows the reference's read-back writes (bfp16_c16_row,
 * src/npu/bfp16_pack.cpp:213-229) from the NPU's bf16 output. */
int zest_widen_bf16(const uint16_t *src, int64_t n, float *dst, void *stream);

/* zest_gemm_group with fused epilogues: per weight a residual ADD, or for a
 * fused gate/up weight the down projection's packed input instead of (or
 * besides) the f32 SwiGLU result. The same bits as the unfused ops (ADD as
 * an f32 add of the same operands; the pack of the f32 SwiGLU values).
 * Replaces: run_rows' ADD (src/xdna-exec.cpp:253-346) and the decode /
 * encode passes between two NPU calls (src/xdna-exec.cpp:368-388). */
int zest_gemm_segs(const uint16_t *a_bf16, int64_t lda, int64_t M, int64_t K, int n, const zest_gemm_seg *segs,
                   unsigned *err, void *stream);

/* How K3 runs a launch: its kernel, tiles, tile order and stream-K split. */
typedef struct zest_gemm_plan {
    int pair_kernel;      /* 1: CTA pairs on 256-row tiles; 0: one CTA per 128-row tile (M <= 128) */
    int tile_n;           /* output tile width */
    int tiles_m, tiles_n; /* tile rows; tile columns of all the weights end to end */
    int k_blocks;         /* 64-wide k-blocks */
    int64_t tiles;
    int ctas;             /* CTAs launched (the one-CTA kernel: per weight, at most) */
    int raster;           /* order the persistent CTAs walk the tiles in: 0 groups of 8 tile rows,
                             1 rows (A streamed, B re-read from L2), 2 columns (B streamed) */
    int stream_k;         /* 1: the last waves are cut into equal runs of k-blocks, one per pair */
    int whole_tiles;      /* tiles run whole */
    int split_tiles;      /* tiles cut into runs */
    int64_t run_k_blocks; /* k-blocks per pair over the split tiles */
} zest_gemm_plan;

/* The plan zest_gemm_group / zest_gemm_segs make for A [M][K] and n weights
 * of N[i] rows, on `sms` SMs (<= 0: this device's), with the same tuning
 * variables. Host only: needs no GPU. The reference's NPU calls have a fixed
 * design per shape (kernels/bfp16_gemm/whole_array_bfp_rtp.py:61-377); this
 * reports the choices the B200 launch makes instead. */
int zest_plan_gemm(int64_t M, int64_t K, int n, const int64_t *N, int sms, zest_gemm_plan *out);

/* K2 + K3 without allocating anything: y[T][ldy] = x[T][K] * W^T, where w_bf16
 * is a weight's bf16 B operand (zest_convert_weight / zest_weight_bf16) of N
 * rows and the same mode and err word as zest_gemm. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc on this path,
 * such as a host program whose GPU memory is planned and owned by its own
 * allocator, or a latency-sensitive caller that cannot afford cudaMalloc /
 * cudaFree synchronising the device mid-prompt.
 * The bf16 copy of the activations goes to a fixed device array of
 * ZEST_NOALLOC_MAX_VALUES values (32 MiB), held on every GPU that loads the
 * library until the process exits; calls with roundup(T, 128) * K above that
 * fail with a clear error. The first call on each device looks up the array's
 * device address (with that device current); make that first call before any
 * stream capture. Every call shares the one array, so calls that overlap on
 * the GPU (other streams, other threads) race: serialise them. Nothing in
 * the array needs clearing between calls: each call writes every row it
 * reads. A launch that takes the stream-K route (zest_plan_gemm) keeps its
 * partial sums in K3's own fixed workspace, another device array, ordered
 * across streams as below; the first such launch on a device creates the
 * one CUDA event that orders them. */
#define ZEST_NOALLOC_MAX_VALUES (16 * 1024 * 1024)
int zest_mul_mat_noalloc(const float *x, int64_t T, int64_t K, int64_t ldx, const uint16_t *w_bf16, int64_t ldw,
                         int64_t N, int mode, float *y, int64_t ldy, unsigned *err, void *stream);

/* The block executor's small ops, on device rows of d contiguous floats,
 * float arithmetic in the reference's order.
 * Replaces: the host passes' run_rows (src/xdna-exec.cpp:253-346) and its
 * rope table (src/xdna-exec.cpp:194-239), for the ops xdna_exec_supports
 * admits (src/xdna-exec.cpp:97-131). */
#define ZEST_GLU_REGLU 0 /* ggml_glu_op ids */
#define ZEST_GLU_GEGLU 1
#define ZEST_GLU_SWIGLU 2
#define ZEST_GLU_GEGLU_ERF 4
#define ZEST_GLU_GEGLU_QUICK 5
#define ZEST_ROPE_NORMAL 0 /* ggml rope modes */
#define ZEST_ROPE_NEOX 2
/* y = x / sqrt(mean(x^2) + eps), per row of d (RMS_NORM; run_rows, src/xdna-exec.cpp:258-269) */
int zest_rms_norm(const float *x, int64_t rows, int64_t d, float eps, float *y, void *stream);
/* y = x * w, w one row of d broadcast over every row (MUL by a norm's scale;
 * src/xdna-exec.cpp:271-276) */
int zest_mul_row(const float *x, const float *w, int64_t rows, int64_t d, float *y, void *stream);
/* y = x + b, b the same shape or (bias_row) one row of d (ADD; src/xdna-exec.cpp:278-288) */
int zest_add(const float *x, const float *b, int bias_row, int64_t rows, int64_t d, float *y, void *stream);
/* y = x * s + bias (SCALE; src/xdna-exec.cpp:290-294) */
int zest_scale(const float *x, int64_t n, float s, float bias, float *y, void *stream);
/* y = act(g) * u row by row, g and u with their own row strides (GLU: split
 * tensors, or the two halves of one tensor; src/xdna-exec.cpp:296-319) */
int zest_glu(int kind, const float *g, int64_t g_stride, const float *u, int64_t u_stride, int64_t rows, int64_t f,
             float *y, void *stream);
/* the [T][n_dims] cos/sin table of positions pos (device), YaRN and optional
 * per-frequency factors ff (device, may be NULL); par (host) = freq_base,
 * freq_scale, ext_factor, attn_factor, beta_fast, beta_slow
 * (rope_table, src/xdna-exec.cpp:199-239) */
int zest_rope_table(const int32_t *pos, int64_t T, int n_dims, int n_ctx_orig, const float *par, const float *ff,
                    float *table, void *stream);
/* x [T][heads][d] -> y, the first n_dims of each head rotated (ROPE; src/xdna-exec.cpp:321-341) */
int zest_rope(const float *x, int64_t T, int64_t heads, int64_t d, int n_dims, int mode, const float *table, float *y,
              void *stream);

/* RMS_NORM of each row of x [T][ldx] (eps), times w (a row of K; NULL:
 * none), then K2's pack: a_bf16 [m_pad][lda] receives the bf16 copy of the
 * result's bfp16 rounding (rows past T zero), and y [T][ldy] (NULL: not
 * written) the f32 result, as ggml's MUL tensor. The same bits as
 * zest_rms_norm, zest_mul_row and zest_pack_activations in turn, in one pass.
 * Replaces: run_rows' RMS_NORM and MUL (src/xdna-exec.cpp:253-346) with the
 * encode_row of the matmul input they feed (src/xdna-npu.cpp:511-515). */
int zest_pack_rms_norm(const float *x, int64_t T, int64_t K, int64_t ldx, float eps, const float *w, float *y,
                       int64_t ldy, int64_t m_pad, uint16_t *a_bf16, int64_t lda, void *stream);
/* Per-head RMS_NORM (eps) of x [T][heads][d] (d <= 256), times w (a row of
 * d; NULL: none), then ROPE (mode, n_dims, a zest_rope_table table) into
 * y [T][heads][d] f32 and/or y_bf16 (the bf16 rounding, nearest even); either
 * output may be NULL. Qwen3's q/k norm and rope in one pass.
 * Replaces: run_rows' RMS_NORM, MUL and ROPE (src/xdna-exec.cpp:253-346). */
int zest_norm_rope(const float *x, int64_t T, int64_t heads, int64_t d, float eps, const float *w, int n_dims,
                   int mode, const float *table, float *y, uint16_t *y_bf16, void *stream);

/* ---------------------------------------------------------------------------
 * 2. The matmul service (xdna_npu)
 * ------------------------------------------------------------------------- */

typedef struct zest_npu zest_npu;

/* A weight's identity across calls: where it lives and what it is
 * (xdna_npu::wkey, src/xdna-npu.h:46-52). */
typedef struct {
    const void *buffer, *data;
    int type;
    int64_t K, N;
} zest_wkey;

/* Time spent since the last zest_take_times (xdna_npu::times,
 * src/xdna-npu.h:104-107), measured with CUDA events. */
typedef struct {
    double encode_ms, gemm_ms, copy_ms, pack_ms;
    int calls;
} zest_times;

/* Whether GPU `device` can run the path: it opens, and a small exact integer
 * multiply through all three kernels comes back right. Checked once per
 * device; `why` (may be NULL) says what passed or failed.
 * Replaces: xdna_npu_usable + npu_self_test (src/xdna-npu.cpp:142-184,255-291). */
int zest_usable(int device, char *why, size_t why_len);

/* A service on GPU `device` with its own stream. NULL on failure.
 * Replaces: xdna_npu::xdna_npu + init (src/xdna-npu.cpp:304-317). */
zest_npu *zest_open(int device);
void zest_close(zest_npu *npu);

/* Output mode for weights added from now on: 1 = bf16 (the default, as the
 * reference's GGML_XDNA_OUT16), 0 = fp32 (src/xdna-npu.cpp:49-55,374). */
void zest_set_out16(zest_npu *npu, int on);

int zest_has_weight(const zest_npu *npu, const zest_wkey *key);

/* Builds a weight's copy from its raw GGUF bytes (host memory, or device
 * memory when raw_on_device): bfp16 bytes + bf16 expansion, kept on the GPU.
 * Replaces: xdna_npu::add_weight (src/xdna-npu.cpp:369-378). */
int zest_add_weight(zest_npu *npu, const zest_wkey *key, const void *raw, int raw_on_device);

/* The same from the weight already dequantised to f32 rows (N x K, host
 * memory or device memory when on_device), for GGUF types without a GPU
 * converter here: the caller runs ggml's to_float once, as the reference
 * does for every type (xdna_npu::unpack, src/xdna-npu.cpp:339-350). The copy
 * is keyed by `key` (its type stays the GGUF one). */
int zest_add_weight_values(zest_npu *npu, const zest_wkey *key, const float *values, int on_device);

/* A gate and an up weight fused for SiLU(gate) * up, keyed by gate's key.
 * Replaces: xdna_npu::add_fused (src/xdna-npu.cpp:380-390). */
int zest_add_fused(zest_npu *npu, const zest_wkey *gate, const void *gate_raw, const void *up_raw, int raw_on_device);

/* Output values a row of a weight added above: N, or F for a fused pair
 * (xdna_npu::out_width, src/xdna-npu.h:74). -1 if unknown. */
int64_t zest_out_width(const zest_npu *npu, const zest_wkey *key, int fused);

/* Weight copies built without the host waiting. On (on = 1), a copy added
 * from raw bytes already in device memory (zest_add_weight /
 * zest_add_fused with raw_on_device) is converted on the service's load
 * stream and the call returns at once; the first matmul that uses it waits
 * for it on the GPU, and zest_weight_bf16 / zest_weight_bfp16 wait for it on
 * the host before handing out its buffers. The raw bytes must stay in place
 * until then. Copies from host memory are built before the call returns, as
 * with it off (the default). zest_wait_weights waits for every copy queued.
 * Replaces: the background weight-copy builder that graph_optimize queues
 * and graph_compute waits for (queue_copies / build_copies / finish_copies,
 * src/ggml-zest.cpp:261-330). */
void zest_set_load_async(zest_npu *npu, int on);
int zest_wait_weights(zest_npu *npu);

/* The weight copy's device buffers, for callers that run the kernels
 * themselves (NULL if unknown). */
const uint8_t *zest_weight_bfp16(const zest_npu *npu, const zest_wkey *key, int fused);
const uint16_t *zest_weight_bf16(const zest_npu *npu, const zest_wkey *key, int fused, int64_t *n_pad);

/* y[T][out_width] = x[T][K] * W^T, f32 row-major, for a weight added above
 * (fused: the SwiGLU of the pair). x and y are host memory, or device memory
 * when on_device. Checks every result for NaN/Inf.
 * Replaces: xdna_npu::mul_mat (src/xdna-npu.cpp:392-444). */
int zest_mul_mat(zest_npu *npu, const zest_wkey *key, int fused, const float *x, int64_t T, float *y, int on_device);

/* The same for up to 4 weights added above that share the input x (same K):
 * one pack and one grouped launch; y[i] gets weight i's out_width values a
 * row (fused[i]: the SwiGLU of a fused pair).
 * Replaces: xdna_npu::begin / encode_row / submit / wait / decode_row for
 * one group (src/xdna-npu.cpp:476-551). */
int zest_mul_mat_group(zest_npu *npu, int n, const zest_wkey *keys, const int *fused, const float *x, int64_t T,
                       float *const *y, int on_device);

/* Group calls in flight at once: zest_submit_group queues the call
 * zest_mul_mat_group makes, in slot `slot` (0 .. ZEST_SLOTS-1), and returns
 * without waiting; zest_wait_group(slot) finishes it (host buffers: widens
 * the bf16 results into y as their copies land) and returns its status, the
 * results then in y. The calls of all slots queue on the service's streams in
 * submission order, so with host buffers one call's copy in overlaps another's
 * copy out and the host's widening: PCIe's two directions are busy at once.
 * x and y must stay valid, and x unchanged, until the wait returns; a slot
 * takes its next call only after its wait. One thread at a time calls into a
 * service; wait for every submitted call before zest_close.
 * Replaces: xdna_npu::reserve / begin / encode_row / submit / wait /
 * decode_row with one group in flight per stream (src/xdna-npu.h:79-101),
 * as xdna_exec_piece runs several streams in turn (src/xdna-exec.cpp:589-640). */
#define ZEST_SLOTS 4
int zest_submit_group(zest_npu *npu, int slot, int n, const zest_wkey *keys, const int *fused, const float *x,
                      int64_t T, float *const *y, int on_device);
int zest_wait_group(zest_npu *npu, int slot);

/* Where one weight's result of zest_mul_mat_group_ex goes. */
typedef struct {
    float *y;               /* [T][out_width]; may be NULL for a fused gate/up weight that gives a_next */
    const float *residual;  /* NULL, or the ADD that follows: y = residual + result ([T][out_width], may be y) */
    uint16_t *a_next;       /* NULL, or (a fused gate/up weight) the SwiGLU result's K2 operand,
                               [roundup(T,128)][out_width], the next matmul's a_bf16 */
} zest_mm_out;

/* zest_mul_mat_group on device buffers, with the block executor's ops next
 * to the matmuls folded in. The input is one of: a_bf16 (an operand already
 * packed, [roundup(T,128)][K], e.g. another call's a_next); x after
 * RMS_NORM(norm_eps) and a MUL by norm_w (may be NULL) when norm_eps >= 0,
 * the f32 normalised rows going to x_normed unless it is NULL; or x as is.
 * Each weight's result goes where outs[i] says.
 * Replaces: a piece's run_rows passes around its matmuls (RMS_NORM, MUL,
 * ADD, GLU; src/xdna-exec.cpp:253-346,368-388) together with the group's
 * encode / submit / decode (src/xdna-npu.cpp:476-551). */
int zest_mul_mat_group_ex(zest_npu *npu, int n, const zest_wkey *keys, const int *fused, const float *x,
                          float norm_eps, const float *norm_w, float *x_normed, const uint16_t *a_bf16, int64_t T,
                          const zest_mm_out *outs);

/* The service's CUDA stream (a cudaStream_t): the reference's service owns its
 * NPU queue the same way (xdna_npu, src/xdna-npu.h:40-136). */
void *zest_stream(zest_npu *npu);

/* Replaces: xdna_npu::take_times (src/xdna-npu.cpp:555-559). */
int zest_take_times(zest_npu *npu, zest_times *out);

#ifdef __cplusplus
}
#endif
#endif
