/*
 * A stand-in for the few ggml-base functions the plugin imports, so that the
 * real libggml-zest.so can be loaded and driven through its vtables without
 * llama.cpp (which this image lacks). TEST INFRASTRUCTURE ONLY.
 *
 * Ops are named, not numbered: the plugin identifies them with ggml_op_name,
 * so the ids here are this harness's own.
 */
#include "ggml_abi.h"

#include <stdlib.h>
#include <string.h>

static const char *OP_NAMES[] = { "NONE", "MUL_MAT", "ADD", "RESHAPE", "VIEW", "MUL_MAT_ID", "GET_ROWS",
                                  "RMS_NORM", "MUL", "SCALE", "GLU", "ROPE", "PERMUTE", "TRANSPOSE", "CPY" };

const char *ggml_op_name(enum ggml_op op) {
    return (int) op >= 0 && (int) op < (int) (sizeof OP_NAMES / sizeof OP_NAMES[0]) ? OP_NAMES[op] : "UNKNOWN";
}

/* block size and bytes per block of the types the tests use */
static void type_size(int type, int64_t *blck, size_t *bytes) {
    switch (type) {
        case GGML_TYPE_F32: *blck = 1; *bytes = 4; return;
        case GGML_TYPE_F16: *blck = 1; *bytes = 2; return;
        case GGML_TYPE_Q4_0: *blck = 32; *bytes = 18; return;
        case GGML_TYPE_Q8_0: *blck = 32; *bytes = 34; return;
        case GGML_TYPE_Q4_K: *blck = 256; *bytes = 144; return;
        case GGML_TYPE_Q6_K: *blck = 256; *bytes = 210; return;
        case GGML_TYPE_IQ3_S: *blck = 256; *bytes = 110; return;
        case GGML_TYPE_I32: *blck = 1; *bytes = 4; return;
        default: *blck = 1; *bytes = 4; return;
    }
}

size_t ggml_nbytes(const struct ggml_tensor *t) {
    int64_t blck;
    size_t bytes;
    type_size(t->type, &blck, &bytes);
    size_t n = (size_t) (t->ne[0] / blck) * bytes;
    for (int i = 1; i < GGML_MAX_DIMS; i++) n += (size_t) (t->ne[i] - 1) * t->nb[i];
    return n;
}

bool ggml_is_contiguous(const struct ggml_tensor *t) {
    int64_t blck;
    size_t bytes;
    type_size(t->type, &blck, &bytes);
    size_t next = bytes;
    if (t->nb[0] != bytes) return false;
    next = (size_t) (t->ne[0] / blck) * bytes;
    for (int i = 1; i < GGML_MAX_DIMS; i++) {
        if (t->ne[i] != 1 && t->nb[i] != next) return false;
        next *= (size_t) t->ne[i];
    }
    return true;
}

int64_t ggml_nrows(const struct ggml_tensor *t) { return t->ne[1] * t->ne[2] * t->ne[3]; }

/* to_float for a type without a GPU converter in the plugin: Q4_0
 * ({fp16 d; u8 qs[16]}: y = (q - 8) * d, low nibbles first) */
static float half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t) (h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t u;
    float f;
    if (e == 0) {
        f = (float) m * (1.0f / 16777216.0f);
        return s ? -f : f;
    }
    u = e == 31 ? (s | 0x7f800000u | (m << 13)) : (s | ((e + 112) << 23) | (m << 13));
    memcpy(&f, &u, 4);
    return f;
}

static void q4_0_to_float(const void *x, float *y, int64_t k) {
    const uint8_t *b = (const uint8_t *) x;
    for (int64_t i = 0; i < k / 32; i++, b += 18) {
        const float d = half_to_float((uint16_t) (b[0] | (b[1] << 8)));
        for (int j = 0; j < 16; j++) {
            y[i * 32 + j] = (float) ((b[2 + j] & 0xF) - 8) * d;
            y[i * 32 + j + 16] = (float) ((b[2 + j] >> 4) - 8) * d;
        }
    }
}

/* IQ3_S as ggml stores it, 110 bytes per 256 values: {fp16 d; u8 qs[64];
 * u8 qh[8]; u8 signs[32]; u8 scales[4]}. Value e of 32-value group g:
 * magnitude byte e%4 of codebook entry qs[8g + e/4] | (bit e/4 of qh[g]) << 8,
 * times d * (1 + 2 * (nibble g%2 of scales[g/2])), negated when bit e%8 of
 * signs[4g + e/8] is set. The codebook is the one the tests load from the
 * installed gguf package (fake_ggml_set_iq3s_grid); without it ggml reports
 * no IQ3_S dequantiser. */
static uint32_t IQ3S_GRID[512];
static int IQ3S_READY;

void fake_ggml_set_iq3s_grid(const uint32_t *grid) {
    memcpy(IQ3S_GRID, grid, sizeof IQ3S_GRID);
    IQ3S_READY = 1;
}

static void iq3_s_to_float(const void *x, float *y, int64_t k) {
    const uint8_t *b = (const uint8_t *) x;
    for (int64_t blk = 0; blk < k / 256; blk++, b += 110) {
        const float d = half_to_float((uint16_t) (b[0] | (b[1] << 8)));
        const uint8_t *qs = b + 2, *qh = b + 66, *signs = b + 74, *scales = b + 106;
        for (int g = 0; g < 8; g++) {
            const float db = d * (float) (1 + 2 * ((scales[g / 2] >> (4 * (g % 2))) & 0xf));
            for (int e = 0; e < 32; e++) {
                const int slot = e / 4;
                const uint32_t idx = qs[8 * g + slot] | (((qh[g] >> slot) & 1u) << 8);
                const float mag = (float) ((IQ3S_GRID[idx] >> (8 * (e % 4))) & 0xffu);
                const int neg = (signs[4 * g + e / 8] >> (e % 8)) & 1;
                y[blk * 256 + 32 * g + e] = db * mag * (neg ? -1.0f : 1.0f);
            }
        }
    }
}

static const struct ggml_type_traits Q4_0_TRAITS = { "q4_0", 32, 0, 18, true, q4_0_to_float, NULL };
static const struct ggml_type_traits IQ3_S_TRAITS = { "iq3_s", 256, 0, 110, true, iq3_s_to_float, NULL };
static const struct ggml_type_traits NO_TRAITS = { "other", 1, 0, 4, false, NULL, NULL };

const struct ggml_type_traits *ggml_get_type_traits(enum ggml_type type) {
    if (type == GGML_TYPE_Q4_0) return &Q4_0_TRAITS;
    if (type == GGML_TYPE_IQ3_S && IQ3S_READY) return &IQ3_S_TRAITS;
    return &NO_TRAITS;
}

/* graphs: {int n; ggml_tensor **nodes} */
struct ggml_cgraph {
    int n_nodes;
    struct ggml_tensor **nodes;
};

int ggml_graph_n_nodes(struct ggml_cgraph *g) { return g->n_nodes; }
struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *g, int i) { return i < 0 ? g->nodes[g->n_nodes + i] : g->nodes[i]; }

/* buffers and buffer types */
struct ggml_backend_buffer_type {
    int is_host;
};
struct ggml_backend_buffer {
    int usage;
    int is_host;
};

static struct ggml_backend_buffer_type CUDA_BUFT = { 0 }, CPU_BUFT = { 1 };

enum ggml_backend_buffer_usage ggml_backend_buffer_get_usage(ggml_backend_buffer_t b) {
    return (enum ggml_backend_buffer_usage) b->usage;
}
bool ggml_backend_buffer_is_host(ggml_backend_buffer_t b) { return b->is_host != 0; }
bool ggml_backend_buft_is_host(ggml_backend_buffer_type_t t) { return t->is_host != 0; }

/* two devices: CUDA0 (a GPU) and CPU */
struct fake_dev {
    struct ggml_backend_device dev;
    const char *name;
    enum ggml_backend_dev_type type;
    ggml_backend_buffer_type_t buft;
};
static struct fake_dev DEVS[2] = {
    { { { 0 }, NULL, NULL }, "CUDA0", GGML_BACKEND_DEVICE_TYPE_GPU, &CUDA_BUFT },
    { { { 0 }, NULL, NULL }, "CPU", GGML_BACKEND_DEVICE_TYPE_CPU, &CPU_BUFT },
};

size_t ggml_backend_dev_count(void) { return 2; }
ggml_backend_dev_t ggml_backend_dev_get(size_t i) { return i < 2 ? &DEVS[i].dev : NULL; }
ggml_backend_dev_t ggml_backend_dev_by_name(const char *name) {
    for (int i = 0; i < 2; i++)
        if (strcmp(DEVS[i].name, name) == 0) return &DEVS[i].dev;
    return NULL;
}
const char *ggml_backend_dev_name(ggml_backend_dev_t d) { return ((struct fake_dev *) d)->name; }
enum ggml_backend_dev_type ggml_backend_dev_type(ggml_backend_dev_t d) { return ((struct fake_dev *) d)->type; }
ggml_backend_buffer_type_t ggml_backend_dev_buffer_type(ggml_backend_dev_t d) { return ((struct fake_dev *) d)->buft; }

/* harness helpers the tests call through ctypes */
ggml_backend_buffer_t fake_buffer_new(int usage, int is_host) {
    ggml_backend_buffer_t b = (ggml_backend_buffer_t) calloc(1, sizeof *b);
    b->usage = usage;
    b->is_host = is_host;
    return b;
}
struct ggml_cgraph *fake_graph_new(int n, struct ggml_tensor **nodes) {
    struct ggml_cgraph *g = (struct ggml_cgraph *) calloc(1, sizeof *g);
    g->n_nodes = n;
    g->nodes = nodes;
    return g;
}
ggml_backend_buffer_type_t fake_cuda_buft(void) { return &CUDA_BUFT; }
ggml_backend_buffer_type_t fake_cpu_buft(void) { return &CPU_BUFT; }
int fake_op_id(const char *name) {
    for (int i = 0; i < (int) (sizeof OP_NAMES / sizeof OP_NAMES[0]); i++)
        if (strcmp(OP_NAMES[i], name) == 0) return i;
    return -1;
}
