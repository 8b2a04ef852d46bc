/*
 * The ggml backend plugin libggml-zest.so, B200 build: a drop-in for the
 * reference's plugin of the same name (include/ggml-zest.h:1-17 there). It
 * registers the device XDNA0, which llama.cpp selects with
 * `-dev XDNA0,CUDA0`. XDNA0 claims large-batch weight MUL_MATs
 * (supports_op, src/ggml-zest.cpp:1160-1226) and runs them on the B200's
 * tensor cores in place, on the CUDA backend's device buffers.
 *
 * Loaded with GGML_BACKEND_PATH=libggml-zest.so, whose exports are
 * ggml_backend_init and ggml_backend_score (GGML_BACKEND_DL_IMPL /
 * GGML_BACKEND_DL_SCORE_IMPL, src/ggml-zest.cpp:1318-1319), or linked and
 * registered through ggml_backend_xdna_reg.
 */
#ifndef GGML_ZEST_H
#define GGML_ZEST_H

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_XDNA_NAME "XDNA"         /* the backend (registry) name */
#define GGML_XDNA_DEVICE_NAME "XDNA0" /* the device, as -dev names it */

#include <stdint.h>

typedef struct ggml_backend_reg *ggml_backend_reg_t;
struct ggml_tensor;

/* Replaces: ggml_backend_xdna_reg (include/ggml-zest.h:9, src/ggml-zest.cpp:1294-1301). */
__attribute__((visibility("default"))) ggml_backend_reg_t ggml_backend_xdna_reg(void);

/* The dispatch policy alone, without the device checks: whether supports_op
 * would claim `op` on a usable GPU (src/ggml-zest.cpp:1167-1226). For tests
 * and for hosts that plan placement themselves; no GPU is touched. */
__attribute__((visibility("default"))) int ggml_zest_policy_supports(const struct ggml_tensor *op);

/* How many SwiGLU gate/up pairs graph_compute would run as one fused GEMM in
 * this piece (find_fusions, src/xdna-exec.cpp:392-431), from the readers the
 * supports_op questions recorded. Host logic only; for tests. */
struct ggml_cgraph;
__attribute__((visibility("default"))) int ggml_zest_piece_fusions(struct ggml_cgraph *cgraph);

/* The MUL_MATs of this piece that graph_compute would run as grouped calls
 * (one activation pack and one launch per input shared by 2 to 4 matmuls,
 * the counterpart of submitting a piece's matmuls as one runlist,
 * src/xdna-npu.cpp:476-531): returns the number of groups and writes each
 * one's size to sizes[0 .. max_groups). Host logic only; for tests. */
__attribute__((visibility("default"))) int ggml_zest_piece_groups(struct ggml_cgraph *cgraph, int *sizes,
                                                                  int max_groups);

/* The weight-copy budget's answers for these weights asked in this order
 * under a limit of limit_gb (GGML_XDNA_MAX_COPY_GB): taken[i] = 1 where the
 * weight's copy is made. Once a weight does not fit, its whole layer (by the
 * "blk.N." name) stays on the GPU backend with every later one
 * (src/ggml-zest.cpp:466-564). Returns how many are taken. Host logic only;
 * for tests. */
__attribute__((visibility("default"))) int ggml_zest_budget_plan(double limit_gb,
                                                                 const struct ggml_tensor *const *weights, int n,
                                                                 int *taken);

/* The plan graph_compute makes for this piece: returns the number of matmul
 * service calls and writes counts[0..5]: fused SwiGLUs, grouped matmul
 * calls, RMS_NORMs folded into a pack, residual ADDs folded into a GEMM
 * epilogue, SwiGLU results handed to the next matmul packed, and
 * RMS_NORM + MUL + ROPE runs done as one kernel: the ops the reference folds
 * into its passes over a piece's rows (run_pass and find_fusions,
 * src/xdna-exec.cpp:368-388,392-431). Host logic only; for tests. */
__attribute__((visibility("default"))) int ggml_zest_piece_plan(struct ggml_cgraph *cgraph, int *counts);

/* The notes about the model that graph_compute says once as the first prompt
 * runs (src/ggml-zest.cpp:566-655), gathered while supports_op was asked:
 * writes them to out (at most n bytes) and returns their length, 0 for none.
 * Host logic only; for tests. */
__attribute__((visibility("default"))) int ggml_zest_model_notes(char *out, int n);

/* The IQ3_S codebook the plugin converts IQ3_S weights with: ggml's own,
 * read back through the host ggml's to_float when the library loads (the
 * reference dequantises every weight type with that to_float,
 * src/xdna-npu.cpp:339-348). Writes the 512 entries (four magnitude bytes
 * each, the first in the low byte) to out and returns 1; returns 0 when
 * ggml offers no IQ3_S dequantiser, and IQ3_S weights are then not
 * claimed. Host logic only; for tests. */
__attribute__((visibility("default"))) int ggml_zest_iq3s_codebook(uint32_t *out);

#ifdef __cplusplus
}
#endif
#endif
