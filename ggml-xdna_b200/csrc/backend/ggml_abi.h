// The part of ggml's ABI that the backend plugin touches, declared here
// because ggml's headers (llama.cpp tag b10944) are not part of this tree.
//
// Layouts follow ggml's public ggml.h / ggml-backend.h and the backend
// interface structs of ggml-backend-impl.h, in the slot order the
// reference's initialisers use (src/ggml-zest.cpp:967-984 backend,
// :1250-1267 device, :1287-1292 reg, :1022-1038 device props). When the
// plugin is built inside llama.cpp's tree, define ZEST_USE_GGML_HEADERS and
// ggml's own headers are used instead.
#pragma once

#ifdef ZEST_USE_GGML_HEADERS
#include "ggml-backend-impl.h"
#include "ggml-impl.h"
#include "ggml.h"
#else

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_SRC 10
#define GGML_MAX_NAME 64
#define GGML_MAX_OP_PARAMS 64

#ifndef GGML_BACKEND_API_VERSION
#define GGML_BACKEND_API_VERSION 2
#endif

#define GGML_BACKEND_API __attribute__((visibility("default")))

// ggml_type values are GGUF's on-disk ids and do not change between releases
enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q5_0 = 6,
    GGML_TYPE_Q5_1 = 7,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_Q2_K = 10,
    GGML_TYPE_Q3_K = 11,
    GGML_TYPE_Q4_K = 12,
    GGML_TYPE_Q5_K = 13,
    GGML_TYPE_Q6_K = 14,
    GGML_TYPE_I32 = 26,
    GGML_TYPE_IQ3_S = 21,
    GGML_TYPE_BF16 = 30,
};

// ggml_op ids move between releases: the plugin names ops with ggml_op_name()
enum ggml_op { GGML_OP_NONE = 0 };

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED = -1,
    GGML_STATUS_SUCCESS = 0,
    GGML_STATUS_ABORTED = 1,
};

enum ggml_tensor_flag {
    GGML_TENSOR_FLAG_INPUT = 1,
    GGML_TENSOR_FLAG_OUTPUT = 2,
    GGML_TENSOR_FLAG_PARAM = 4,
    GGML_TENSOR_FLAG_LOSS = 8,
};

struct ggml_backend_buffer;
struct ggml_cgraph;

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
    char padding[8];
};

typedef void (*ggml_to_float_t)(const void *x, float *y, int64_t k);

struct ggml_type_traits {
    const char *type_name;
    int64_t blck_size;
    int64_t blck_size_interleave;
    size_t type_size;
    bool is_quantized;
    ggml_to_float_t to_float;
    void (*from_float_ref)(const float *x, void *y, int64_t k);
};

typedef uint8_t ggml_guid[16];
typedef ggml_guid *ggml_guid_t;

typedef struct ggml_backend_buffer_type *ggml_backend_buffer_type_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
typedef struct ggml_backend_event *ggml_backend_event_t;
typedef struct ggml_backend *ggml_backend_t;
typedef void *ggml_backend_graph_plan_t;
typedef struct ggml_backend_reg *ggml_backend_reg_t;
typedef struct ggml_backend_device *ggml_backend_dev_t;
typedef struct ggml_backend_graph_optimize_params ggml_backend_graph_optimize_params;

enum ggml_backend_buffer_usage {
    GGML_BACKEND_BUFFER_USAGE_ANY = 0,
    GGML_BACKEND_BUFFER_USAGE_WEIGHTS = 1,
    GGML_BACKEND_BUFFER_USAGE_COMPUTE = 2,
};

enum ggml_backend_dev_type {
    GGML_BACKEND_DEVICE_TYPE_CPU,
    GGML_BACKEND_DEVICE_TYPE_GPU,
    GGML_BACKEND_DEVICE_TYPE_IGPU,
    GGML_BACKEND_DEVICE_TYPE_ACCEL,
};

struct ggml_backend_dev_caps {
    bool async;
    bool host_buffer;
    bool buffer_from_host_ptr;
    bool events;
    bool mmap_support;
};

struct ggml_backend_dev_props {
    const char *name;
    const char *description;
    size_t memory_free;
    size_t memory_total;
    enum ggml_backend_dev_type type;
    const char *device_id;
    struct ggml_backend_dev_caps caps;
};

// backend (stream) interface, src/ggml-zest.cpp:967-984
struct ggml_backend_i {
    const char *(*get_name)(ggml_backend_t backend);
    void (*free)(ggml_backend_t backend);
    void (*set_tensor_async)(ggml_backend_t, struct ggml_tensor *, const void *, size_t, size_t);
    void (*get_tensor_async)(ggml_backend_t, const struct ggml_tensor *, void *, size_t, size_t);
    void (*set_tensor_2d_async)(ggml_backend_t, struct ggml_tensor *, const void *, size_t, size_t, size_t, size_t,
                                size_t);
    void (*get_tensor_2d_async)(ggml_backend_t, const struct ggml_tensor *, void *, size_t, size_t, size_t, size_t,
                                size_t);
    bool (*cpy_tensor_async)(ggml_backend_t, ggml_backend_t, const struct ggml_tensor *, struct ggml_tensor *);
    void (*synchronize)(ggml_backend_t backend);
    ggml_backend_graph_plan_t (*graph_plan_create)(ggml_backend_t, const struct ggml_cgraph *);
    void (*graph_plan_free)(ggml_backend_t, ggml_backend_graph_plan_t);
    void (*graph_plan_update)(ggml_backend_t, ggml_backend_graph_plan_t, const struct ggml_cgraph *);
    enum ggml_status (*graph_plan_compute)(ggml_backend_t, ggml_backend_graph_plan_t);
    enum ggml_status (*graph_compute)(ggml_backend_t backend, struct ggml_cgraph *cgraph);
    void (*event_record)(ggml_backend_t, ggml_backend_event_t);
    void (*event_wait)(ggml_backend_t, ggml_backend_event_t);
    void (*graph_optimize)(ggml_backend_t backend, struct ggml_cgraph *cgraph,
                           ggml_backend_graph_optimize_params *params);
};

struct ggml_backend {
    ggml_guid_t guid;
    struct ggml_backend_i iface;
    ggml_backend_dev_t device;
    void *context;
};

// device interface, src/ggml-zest.cpp:1250-1267
struct ggml_backend_device_i {
    const char *(*get_name)(ggml_backend_dev_t dev);
    const char *(*get_description)(ggml_backend_dev_t dev);
    void (*get_memory)(ggml_backend_dev_t dev, size_t *free, size_t *total);
    enum ggml_backend_dev_type (*get_type)(ggml_backend_dev_t dev);
    void (*get_props)(ggml_backend_dev_t dev, struct ggml_backend_dev_props *props);
    ggml_backend_t (*init_backend)(ggml_backend_dev_t dev, const char *params);
    ggml_backend_buffer_type_t (*get_buffer_type)(ggml_backend_dev_t dev);
    ggml_backend_buffer_type_t (*get_host_buffer_type)(ggml_backend_dev_t dev);
    ggml_backend_buffer_t (*buffer_from_host_ptr)(ggml_backend_dev_t dev, void *ptr, size_t size,
                                                  size_t max_tensor_size);
    bool (*supports_op)(ggml_backend_dev_t dev, const struct ggml_tensor *op);
    bool (*supports_buft)(ggml_backend_dev_t dev, ggml_backend_buffer_type_t buft);
    bool (*offload_op)(ggml_backend_dev_t dev, const struct ggml_tensor *op);
    ggml_backend_event_t (*event_new)(ggml_backend_dev_t dev);
    void (*event_free)(ggml_backend_dev_t dev, ggml_backend_event_t event);
    void (*event_synchronize)(ggml_backend_dev_t dev, ggml_backend_event_t event);
};

struct ggml_backend_device {
    struct ggml_backend_device_i iface;
    ggml_backend_reg_t reg;
    void *context;
};

// registry interface, src/ggml-zest.cpp:1287-1292
struct ggml_backend_reg_i {
    const char *(*get_name)(ggml_backend_reg_t reg);
    size_t (*get_device_count)(ggml_backend_reg_t reg);
    ggml_backend_dev_t (*get_device)(ggml_backend_reg_t reg, size_t index);
    void *(*get_proc_address)(ggml_backend_reg_t reg, const char *name);
};

struct ggml_backend_reg {
    int api_version;
    struct ggml_backend_reg_i iface;
    void *context;
};

// ggml-base functions the plugin calls (resolved from the host process)
const char *ggml_op_name(enum ggml_op op);
size_t ggml_nbytes(const struct ggml_tensor *tensor);
bool ggml_is_contiguous(const struct ggml_tensor *tensor);
int64_t ggml_nrows(const struct ggml_tensor *tensor);
const struct ggml_type_traits *ggml_get_type_traits(enum ggml_type type);
int ggml_graph_n_nodes(struct ggml_cgraph *cgraph);
struct ggml_tensor *ggml_graph_node(struct ggml_cgraph *cgraph, int i);
enum ggml_backend_buffer_usage ggml_backend_buffer_get_usage(ggml_backend_buffer_t buffer);
bool ggml_backend_buffer_is_host(ggml_backend_buffer_t buffer);
bool ggml_backend_buft_is_host(ggml_backend_buffer_type_t buft);
ggml_backend_dev_t ggml_backend_dev_by_name(const char *name);
size_t ggml_backend_dev_count(void);
ggml_backend_dev_t ggml_backend_dev_get(size_t index);
const char *ggml_backend_dev_name(ggml_backend_dev_t device);
enum ggml_backend_dev_type ggml_backend_dev_type(ggml_backend_dev_t device);
ggml_backend_buffer_type_t ggml_backend_dev_buffer_type(ggml_backend_dev_t device);

#ifdef __cplusplus
}
#endif

#endif  // ZEST_USE_GGML_HEADERS
