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

static const struct ggml_type_traits Q4_0_TRAITS = { "q4_0", 32, 0, 18, true, q4_0_to_float, NULL };
static const struct ggml_type_traits NO_TRAITS = { "other", 1, 0, 4, false, NULL, NULL };

const struct ggml_type_traits *ggml_get_type_traits(enum ggml_type type) {
    return type == GGML_TYPE_Q4_0 ? &Q4_0_TRAITS : &NO_TRAITS;
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
    char *base; /* set for buffers the fake CUDA backend allocates (host memory standing in) */
    size_t size;
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

/* The CUDA backend, as far as running a failed piece again needs it: its
 * instances record each graph they are given (how many nodes, how many of
 * their sources lie in a buffer it allocated, and a checksum of those
 * bytes) and answer with a status the test sets. It computes nothing. */
static struct {
    int status, init_fails;
    long runs, last_nodes, moved_srcs, started, stopped, buffers, buffers_freed, sets;
    unsigned long long moved_sum;
} SIB;

static int in_fake_buffer(const struct ggml_tensor *t) {
    return t->buffer && t->buffer->base && (const char *) t->data >= t->buffer->base &&
           (const char *) t->data < t->buffer->base + t->buffer->size;
}

ggml_backend_t ggml_backend_dev_init(ggml_backend_dev_t device, const char *params) {
    (void) params;
    if (SIB.init_fails || ((struct fake_dev *) device)->type != GGML_BACKEND_DEVICE_TYPE_GPU) return NULL;
    ggml_backend_t b = (ggml_backend_t) calloc(1, sizeof *b);
    b->device = device;
    SIB.started++;
    return b;
}
void ggml_backend_free(ggml_backend_t backend) {
    if (!backend) return;
    free(backend);
    SIB.stopped++;
}
enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph *g) {
    (void) backend;
    SIB.runs++;
    SIB.last_nodes = g->n_nodes;
    for (int i = 0; i < g->n_nodes; i++)
        for (int j = 0; j < GGML_MAX_SRC; j++) {
            const struct ggml_tensor *s = g->nodes[i]->src[j];
            if (!s || !in_fake_buffer(s)) continue;
            SIB.moved_srcs++;
            const unsigned char *p = (const unsigned char *) s->data;
            for (size_t k = 0; k < ggml_nbytes(s); k++) SIB.moved_sum += p[k];
        }
    return (enum ggml_status) SIB.status;
}
ggml_backend_buffer_t ggml_backend_buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size) {
    ggml_backend_buffer_t b = (ggml_backend_buffer_t) calloc(1, sizeof *b);
    b->is_host = buft->is_host;
    b->base = (char *) calloc(1, size ? size : 1);
    b->size = size;
    SIB.buffers++;
    return b;
}
size_t ggml_backend_buft_get_alignment(ggml_backend_buffer_type_t buft) {
    (void) buft;
    return 128;
}
void *ggml_backend_buffer_get_base(ggml_backend_buffer_t b) { return b->base; }
void ggml_backend_buffer_free(ggml_backend_buffer_t b) {
    if (!b) return;
    free(b->base);
    free(b);
    SIB.buffers_freed++;
}
void ggml_backend_tensor_set(struct ggml_tensor *t, const void *data, size_t offset, size_t size) {
    memcpy((char *) t->data + offset, data, size);
    SIB.sets++;
}

/* harness helpers the tests call through ctypes */
void fake_sibling_set(int status, int init_fails) {
    SIB.status = status;
    SIB.init_fails = init_fails;
}
/* out[0..8]: runs, nodes of the last graph, moved sources seen, backends
 * started, backends freed, buffers allocated, buffers freed, tensor_set
 * calls; returns the checksum of the moved sources' bytes */
unsigned long long fake_sibling_stats(long *out) {
    const long v[8] = { SIB.runs, SIB.last_nodes, SIB.moved_srcs, SIB.started, SIB.stopped, SIB.buffers,
                        SIB.buffers_freed, SIB.sets };
    memcpy(out, v, sizeof v);
    return SIB.moved_sum;
}
void fake_sibling_reset(void) { memset(&SIB, 0, sizeof SIB); }
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
