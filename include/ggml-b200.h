/*
 * ggml B200 backend -- the backend-level C ABI (the plugin surface).
 *
 * This mirrors the public API and the ggml vtable methods of gregordinary/ggml-rocket
 * (ggml-rocket.h:24-93, device vtable ggml-rocket.cpp:7830-7842, backend vtable :7234-7238,
 * registry :7875-7880) on plain C types: a ggml host links a thin adapter that copies the
 * fields of each ggml_tensor it passes into a b200_tensor (INTEGRATION.md shows it), and
 * everything the reference decides -- which ops to claim, how to walk a graph, which route
 * computed what -- is decided here, in C++, over those descriptors. The three claimed ops run
 * as sm_100a CUDA kernels (ggml-b200-kernels.h); nothing claimed ever runs on the CPU.
 */
#ifndef GGML_B200_H
#define GGML_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_MAX_DIMS      4
#define B200_MAX_SRC       10
#define B200_MAX_OP_PARAMS 16   /* int32 words, as ggml's GGML_MAX_OP_PARAMS / 4 */
#define B200_MAX_NAME      64

/* The ops the backend distinguishes. A ggml adapter maps ggml_op values by NAME
 * (ggml_op_name), as the reference's op-ordinal check does (ggml-rocket.cpp:8231-8252). */
typedef enum {
    B200_OP_NONE = 0,
    B200_OP_RESHAPE,
    B200_OP_VIEW,
    B200_OP_PERMUTE,
    B200_OP_TRANSPOSE,
    B200_OP_MUL_MAT,
    B200_OP_MUL_MAT_ID,
    B200_OP_FLASH_ATTN_EXT,
    B200_OP_OTHER,
    /* the glue ops of a layer, claimed only under B200_GLUE=1 (the reference leaves them to the
     * host's CPU backend) */
    B200_OP_RMS_NORM,
    B200_OP_ADD,
    B200_OP_MUL,
    B200_OP_UNARY,       /* op_params[0]: B200_UNARY_* */
    B200_OP_GLU,         /* op_params[0]: B200_GLU_*, op_params[1]: swapped */
    B200_OP_ROPE,
    B200_OP_GET_ROWS,
    B200_OP_CPY,
    /* the MoE router's ops, also under B200_GLUE=1 */
    B200_OP_SOFT_MAX,
    B200_OP_ARGSORT,     /* op_params[0]: 0 ascending, 1 descending (ggml_sort_order) */
    B200_OP_SUM_ROWS,
    B200_OP_DIV,
} b200_op;

/* Sub-ops of UNARY and GLU, which a ggml adapter maps by name (ggml_unary_op_name /
 * ggml_glu_op_name) through ggml_backend_b200_subop_from_name; -1 for any other. */
enum { B200_UNARY_SILU = 1, B200_GLU_SWIGLU = 2 };

/* Precision ranks of ggml's precision contract (op_params, ggml-rocket.cpp:7334-7355). */
enum {
    B200_PREC_UNDECLARED = 0,
    B200_PREC_F32 = 10,
    B200_PREC_BF16 = 15,
    B200_PREC_F16 = 20,
    B200_PREC_Q8 = 30,
    B200_PREC_Q4 = 40,
};

/* op_params[1] of a MUL_MAT whose src0 is a Walsh-Hadamard matrix (ggml's
 * GGML_HINT_SRC0_IS_HADAMARD; the adapter translates the host's value to this one). */
#define B200_HINT_SRC0_IS_HADAMARD 1

/* The fields of a ggml_tensor the backend reads. Strides nb[] are in bytes. `data` is host
 * memory unless `on_device` is set, in which case it is device memory of the backend's GPU. */
typedef struct b200_tensor {
    int32_t type;                              /* ggml_type numbering */
    int32_t op;                                /* b200_op */
    int64_t ne[B200_MAX_DIMS];
    size_t  nb[B200_MAX_DIMS];
    int32_t op_params[B200_MAX_OP_PARAMS];
    struct b200_tensor * src[B200_MAX_SRC];
    void *  data;
    int32_t on_device;
    int32_t readable;                          /* 0: the bytes are in a layout the backend cannot read
                                                  (a CPU_REPACK buffer, ggml-rocket.cpp:7773-7794) */
    char    name[B200_MAX_NAME];
} b200_tensor;

typedef struct b200_backend * b200_backend_t;

/* ggml_status values graph_compute returns. */
enum { B200_STATUS_SUCCESS = 0, B200_STATUS_FAILED = -1, B200_STATUS_ALLOC_FAILED = -2 };

/* ---- registry (ggml-rocket.cpp:7848-7880, 7918-7926) ------------------------------------ */
const char * ggml_backend_b200_reg_name(void);                       /* "B200" */
int          ggml_backend_b200_reg_device_count(void);               /* visible CUDA devices */
/* Maps a ggml op name to a b200_op (B200_OP_OTHER when the backend has no use for it). */
int          ggml_backend_b200_op_from_name(const char * ggml_op_name);
/* Maps a ggml unary or GLU op name ("SILU", "SWIGLU") to its B200_UNARY_* / B200_GLU_* value. */
int          ggml_backend_b200_subop_from_name(const char * name);

/* ---- device (ggml-rocket.cpp:7830-7842) ---------------------------------------------------- */
const char * ggml_backend_b200_device_name(int device);
int          ggml_backend_b200_device_description(int device, char * buf, size_t n);
int          ggml_backend_b200_device_memory(int device, size_t * free_bytes, size_t * total_bytes);
/* The claim rules: supports_op (ggml-rocket.cpp:7410-7772) and offload_op (:7820-7827). */
bool         ggml_backend_b200_supports_op(const b200_tensor * op);
bool         ggml_backend_b200_offload_op(const b200_tensor * op);

/* ---- backend (ggml-rocket.h:24-93, ggml-rocket.cpp:8024-8217) ------------------------------ */
/* Creates an instance on the current CUDA device; NULL when there is none. Device state
 * (stream, workspace, weight cache) is created lazily at the first graph_compute. */
b200_backend_t ggml_backend_b200_init(void);
void           ggml_backend_b200_free(b200_backend_t backend);
bool           ggml_backend_is_b200(const void * backend);
/* The number of GPUs an op may be spread over (the reference's set_n_threads, which spreads
 * an op over NPU workers). Clamped to 1..8. */
void           ggml_backend_b200_set_n_gpus(b200_backend_t backend, int n_gpus);
/* Distinct MoE expert stacks held device-resident, and those streamed per call. */
void           ggml_backend_b200_moe_stats(b200_backend_t backend, long * n_resident, long * n_streamed);
/* Ops completed per route ("f16", "q8_0", "q4_K", "q6_K", "fused", "moe", "fa"); NULL: total. */
long           ggml_backend_b200_route_ops(b200_backend_t backend, const char * route);
/* Always 0: a claimed op is never computed on the CPU. Kept so a test can assert it. */
long           ggml_backend_b200_cpu_fallbacks(b200_backend_t backend);
/* Kernel launches and device faults reported through the device error word. */
long           ggml_backend_b200_device_errors(b200_backend_t backend);
/* Computes the claimed nodes of one graph split in order (views are no-ops); any other op, a
 * malformed MUL_MAT_ID id, or a device error returns B200_STATUS_FAILED. */
int            ggml_backend_b200_graph_compute(b200_backend_t backend, b200_tensor * const * nodes, int n_nodes);
/* Bytes held by the device-resident weight cache, and its entry count. */
size_t         ggml_backend_b200_weight_cache_bytes(b200_backend_t backend, long * n_entries);

/* ---- building a graph from a host's tensors (the ggml adapter's converter) ------------------
 * Replaces the reference's direct reads of ggml_tensor in graph_compute (ggml-rocket.cpp:7088-7200)
 * and its load-time check of the host's GGML_OP_* ordinals (:8231-8265): the adapter in the host
 * process declares each tensor of a split with its fields, its op as ggml's op NAME (ggml_op_name)
 * and, for UNARY / GLU nodes, the sub-op name (ggml_unary_op_name / ggml_glu_op_name). Every host
 * tensor gets one descriptor, keyed by an opaque pointer (the ggml_tensor*), so nodes that share a
 * source share its descriptor (graph_compute groups MUL_MATs / MUL_MAT_IDs by source identity).
 * Sources are declared before their consumers; _add returns NULL for an undeclared source key and
 * the existing descriptor when the key was declared before. Unknown op names map to B200_OP_OTHER
 * (never claimed). The descriptors live until _reset or _free. */
typedef struct b200_graph_builder * b200_graph_builder_t;
b200_graph_builder_t ggml_backend_b200_builder_new(void);
void                 ggml_backend_b200_builder_free(b200_graph_builder_t b);
void                 ggml_backend_b200_builder_reset(b200_graph_builder_t b);
b200_tensor *        ggml_backend_b200_builder_find(b200_graph_builder_t b, const void * key);
b200_tensor *        ggml_backend_b200_builder_add(b200_graph_builder_t b, const void * key, const char * op_name,
                                                   const char * subop_name, int32_t type, const int64_t ne[4],
                                                   const size_t nb[4], const int32_t op_params[B200_MAX_OP_PARAMS],
                                                   const void * const src_keys[B200_MAX_SRC], void * data,
                                                   int32_t on_device, int32_t readable, const char * name);
/* appends a declared tensor to the node list (the split's execution order); returns the node count
 * or -1 for an undeclared key */
int                  ggml_backend_b200_builder_push_node(b200_graph_builder_t b, const void * key);
int                  ggml_backend_b200_builder_nodes(b200_graph_builder_t b, b200_tensor * const ** nodes);
/* graph_compute over the pushed nodes */
int                  ggml_backend_b200_builder_compute(b200_backend_t backend, b200_graph_builder_t b);

/* ---- the weight identity (ggml-rocket.cpp:4124-4222) ---------------------------------------- */
/* The cache key of a weight: its name with the scheduler's copy prefixes stripped, the type and
 * shape, and a 64-bit fingerprint of 16 evenly spaced 64-byte samples of its bytes. Writes at most
 * n bytes (NUL-terminated) and returns the key length; 0 for a tensor the cache must not key
 * (an unnamed or scheduler-generated "leaf_N" / "node_N" name). */
size_t         ggml_backend_b200_weight_key(const b200_tensor * w, char * buf, size_t n);

/* ---- device buffers, async transfers and events ----------------------------------------------
 * The reference hands out the host CPU buffer type (get_buffer_type, ggml-rocket.cpp:7326-7328)
 * and reports caps.async = caps.events = caps.host_buffer = false (get_props, :7310-7322): its
 * NPU computes out of system DRAM. A B200 has its own memory, so this backend also offers what a
 * ggml device with memory offers: a buffer type of device memory (buffer_type_i / buffer_i),
 * async set / get / copy on the backend's stream, events, and pinned host memory. A tensor placed
 * in a b200 buffer is passed with on_device = 1 and data = base + offset; graph_compute then
 * reads and writes it in place, with no host staging. Host buffers stay accepted as before.
 * Calls return B200_STATUS_SUCCESS or B200_STATUS_FAILED (bad handle, range outside the buffer,
 * CUDA error). */
typedef struct b200_buffer * b200_buffer_t;
typedef struct b200_event  * b200_event_t;

/* buffer type (ggml_backend_buffer_type_i): "B200", 256-byte alignment, at most the device's
 * memory, the bytes a tensor needs, not host memory */
const char *  ggml_backend_b200_buffer_type_name(void);
size_t        ggml_backend_b200_buffer_type_alignment(void);
size_t        ggml_backend_b200_buffer_type_max_size(int device);
size_t        ggml_backend_b200_buffer_type_alloc_size(const b200_tensor * t);
bool          ggml_backend_b200_buffer_type_is_host(void);

/* buffers (ggml_backend_buffer_i) on the backend's GPU; NULL when the allocation fails. The
 * synchronous calls are ordered after all work already queued on the backend's stream. Writing a
 * range through these calls, or freeing the buffer, drops every packed weight the backend cached
 * from bytes in that range (the next graph packs them again). */
b200_buffer_t ggml_backend_b200_buffer_alloc(b200_backend_t backend, size_t size);
void          ggml_backend_b200_buffer_free(b200_buffer_t buf);
void *        ggml_backend_b200_buffer_base(b200_buffer_t buf);
size_t        ggml_backend_b200_buffer_size(b200_buffer_t buf);
int           ggml_backend_b200_buffer_set(b200_buffer_t buf, size_t offset, const void * src, size_t size);
int           ggml_backend_b200_buffer_get(b200_buffer_t buf, size_t offset, void * dst, size_t size);
int           ggml_backend_b200_buffer_memset(b200_buffer_t buf, size_t offset, uint8_t value, size_t size);
int           ggml_backend_b200_buffer_clear(b200_buffer_t buf, uint8_t value);
int           ggml_backend_b200_buffer_copy(b200_buffer_t src, size_t src_offset, b200_buffer_t dst,
                                            size_t dst_offset, size_t size);

/* pinned host memory (caps.host_buffer): transfers from and to it run asynchronously */
void *        ggml_backend_b200_host_alloc(size_t size);
void          ggml_backend_b200_host_free(void * ptr);

/* async transfers on the backend's stream (backend set_tensor_async / get_tensor_async /
 * cpy_tensor_async) and the wait for everything queued on it (synchronize) */
int           ggml_backend_b200_set_async(b200_backend_t backend, b200_buffer_t buf, size_t offset,
                                          const void * src, size_t size);
int           ggml_backend_b200_get_async(b200_backend_t backend, b200_buffer_t buf, size_t offset,
                                          void * dst, size_t size);
int           ggml_backend_b200_copy_async(b200_backend_t backend, b200_buffer_t src, size_t src_offset,
                                           b200_buffer_t dst, size_t dst_offset, size_t size);
int           ggml_backend_b200_synchronize(b200_backend_t backend);

/* events (device event_new / event_free / event_synchronize, backend event_record / event_wait) */
b200_event_t  ggml_backend_b200_event_new(b200_backend_t backend);
void          ggml_backend_b200_event_free(b200_event_t ev);
int           ggml_backend_b200_event_record(b200_backend_t backend, b200_event_t ev);
int           ggml_backend_b200_event_wait(b200_backend_t backend, b200_event_t ev);   /* the stream waits */
int           ggml_backend_b200_event_synchronize(b200_event_t ev);                    /* the host waits */

/* ggml_backend_dev_caps of a device: async, host_buffer, buffer_from_host_ptr, events */
void          ggml_backend_b200_device_caps(int device, bool * async, bool * host_buffer,
                                            bool * buffer_from_host_ptr, bool * events);

/* ---- the device-route circuit breaker (ggml-rocket.cpp:263-307) ----------------------------- */
/* Replays a sequence of route outcomes through one breaker and writes, per call, whether the
 * route was attempted (1) or bypassed (0); a bypassed call's rc is ignored. For tests. */
void           ggml_backend_b200_breaker_replay(const int * rcs, int n, int * attempted);

#ifdef __cplusplus
}
#endif

#endif /* GGML_B200_H */
