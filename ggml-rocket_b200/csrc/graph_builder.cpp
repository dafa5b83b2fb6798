// The ggml-independent half of the ggml adapter: a graph of b200_tensor descriptors built from a
// host's tensors, field by field.
//
// The reference's plugin reads ggml_tensor directly (its graph_compute walks the cgraph,
// ggml-rocket.cpp:7088-7200, and decides ops by GGML_OP_* ordinals after checking at load time that
// the host's ordinals are the ones it was compiled with, :8231-8265). Here the adapter that sits in
// the host process hands each tensor's fields to this builder instead, with the op and the
// UNARY / GLU sub-op as ggml's NAMES (ggml_op_name, ggml_unary_op_name, ggml_glu_op_name), so the
// backend does not depend on enum ordinals. The builder
//   - maps the names to b200 ops and sub-ops (unknown ops become B200_OP_OTHER: not claimed);
//   - gives every host tensor exactly one descriptor (keyed by the host's tensor pointer), so two
//     nodes that share a source share the descriptor: graph_compute's shared-src1 grouping of
//     MUL_MATs (QKV, gate/up) and of MUL_MAT_IDs compares source pointers;
//   - copies op_params, writing the b200 sub-op value in place of the host's into word 0 of UNARY
//     and GLU nodes (the other words, e.g. GLU's swapped flag, are kept).
#include <cstring>
#include <deque>
#include <unordered_map>
#include <vector>

#include "ggml-b200.h"

struct b200_graph_builder {
    std::deque<b200_tensor> store;                           // stable addresses
    std::unordered_map<const void*, b200_tensor*> by_key;
    std::vector<b200_tensor*> nodes;
};

extern "C" {

b200_graph_builder_t ggml_backend_b200_builder_new(void) { return new b200_graph_builder(); }

void ggml_backend_b200_builder_free(b200_graph_builder_t b) { delete b; }

void ggml_backend_b200_builder_reset(b200_graph_builder_t b) {
    if (!b) return;
    b->store.clear();
    b->by_key.clear();
    b->nodes.clear();
}

b200_tensor* ggml_backend_b200_builder_find(b200_graph_builder_t b, const void* key) {
    if (!b || !key) return nullptr;
    auto it = b->by_key.find(key);
    return it == b->by_key.end() ? nullptr : it->second;
}

b200_tensor* ggml_backend_b200_builder_add(b200_graph_builder_t b, const void* key, const char* op_name,
                                           const char* subop_name, int32_t type, const int64_t ne[4],
                                           const size_t nb[4], const int32_t op_params[B200_MAX_OP_PARAMS],
                                           const void* const src_keys[B200_MAX_SRC], void* data, int32_t on_device,
                                           int32_t readable, const char* name) {
    if (!b || !key || !ne || !nb) return nullptr;
    if (b200_tensor* have = ggml_backend_b200_builder_find(b, key)) return have;
    b200_tensor* src[B200_MAX_SRC] = {};
    if (src_keys) {
        for (int i = 0; i < B200_MAX_SRC; i++) {
            if (!src_keys[i]) continue;
            src[i] = ggml_backend_b200_builder_find(b, src_keys[i]);
            if (!src[i]) return nullptr;   // a source must be declared before its consumer
        }
    }
    b->store.emplace_back();
    b200_tensor* t = &b->store.back();
    memset(t, 0, sizeof *t);
    t->type = type;
    t->op = ggml_backend_b200_op_from_name(op_name);
    for (int i = 0; i < B200_MAX_DIMS; i++) {
        t->ne[i] = ne[i];
        t->nb[i] = nb[i];
    }
    if (op_params) memcpy(t->op_params, op_params, sizeof t->op_params);
    if (t->op == B200_OP_UNARY || t->op == B200_OP_GLU) t->op_params[0] = ggml_backend_b200_subop_from_name(subop_name);
    for (int i = 0; i < B200_MAX_SRC; i++) t->src[i] = src[i];
    t->data = data;
    t->on_device = on_device;
    t->readable = readable;
    if (name) {
        strncpy(t->name, name, B200_MAX_NAME - 1);
        t->name[B200_MAX_NAME - 1] = 0;
    }
    b->by_key[key] = t;
    return t;
}

int ggml_backend_b200_builder_push_node(b200_graph_builder_t b, const void* key) {
    b200_tensor* t = ggml_backend_b200_builder_find(b, key);
    if (!t) return -1;
    b->nodes.push_back(t);
    return (int)b->nodes.size();
}

int ggml_backend_b200_builder_nodes(b200_graph_builder_t b, b200_tensor* const** nodes) {
    if (!b) return 0;
    if (nodes) *nodes = b->nodes.data();
    return (int)b->nodes.size();
}

int ggml_backend_b200_builder_compute(b200_backend_t backend, b200_graph_builder_t b) {
    if (!b) return B200_STATUS_FAILED;
    return ggml_backend_b200_graph_compute(backend, b->nodes.data(), (int)b->nodes.size());
}

}  // extern "C"
