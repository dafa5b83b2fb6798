// The ggml plugin: ggml's backend interfaces (registry, device, backend, buffer types) over the C ABI
// of libggml-b200.so, so that a stock ggml host (llama.cpp, whisper.cpp) loads this backend through
// GGML_BACKEND_PATH / ggml_backend_load, as it loads the reference's libggml-rocket.so.
//
// It replaces the reference's vtables and DL entry (ggml-rocket.cpp: backend vtable :7202-7238,
// device vtable :7830-7842, registry :7848-7926, GGML_BACKEND_DL_IMPL and the op-ordinal check
// :8231-8265). Everything the reference decides -- which ops to claim, how to walk and fuse a
// split, the weight cache, the claimed ops' arithmetic -- stays in libggml-b200.so; this file only
// translates: every ggml_tensor of a split is declared to the library's graph builder with its
// fields and ggml's op NAMES (ggml_op_name, ggml_unary_op_name, ggml_glu_op_name), sources before
// consumers, so shared sources keep one descriptor. No claimed op is computed on the CPU.
//
// Built only against a host's ggml (ggml-rocket_b200/build.py with GGML_DIR set): it needs ggml's
// private ggml-backend-impl.h, which no stock install ships. The vtables are filled member by
// member on a value-initialised struct rather than by positional or designated initialisers, so
// that ggml versions which add optional members (newer ones append to these structs) still compile
// and leave the new members NULL; the load-time check below refuses a host whose op ordinals
// disagree with the headers this file was compiled against.
//
// Device type: ACCEL by default, as the reference's device (ggml-rocket.cpp:7316-7321): the host
// keeps weights and activations in its CPU buffers, the backend claims ops through supports_op /
// offload_op and caches packed weights on the GPU. B200_DEVICE_TYPE=gpu makes it a GPU device whose
// default buffer type is device memory, so a host places whole layers in HBM.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "ggml-backend-impl.h"
#include "ggml-backend.h"
#include "ggml.h"

#include "ggml-b200-kernels.h"
#include "ggml-b200.h"

namespace {

// ---- per-device state: one b200 backend serves every ggml backend instance and buffer of a device,
// so the packed-weight cache sees every write to the device buffers it was packed from ----------------

struct DevState {
    int index = 0;
    std::string name, desc;
    std::mutex mu;
    b200_backend_t b200 = nullptr;
    int refs = 0;
    ggml_backend_device dev{};
    ggml_backend_buffer_type buft_device{};
    ggml_backend_buffer_type buft_host{};
};

std::vector<DevState*>& devices() {
    static std::vector<DevState*> d;
    return d;
}

DevState* state(ggml_backend_dev_t dev) { return static_cast<DevState*>(dev->context); }

// The device's b200 backend, created on the device it serves.
b200_backend_t service(DevState* s) {
    std::lock_guard<std::mutex> lk(s->mu);
    if (!s->b200) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(s->index);
        s->b200 = ggml_backend_b200_init();
        cudaSetDevice(prev);
    }
    return s->b200;
}

bool gpu_mode() {
    const char* e = getenv("B200_DEVICE_TYPE");
    return e && (strcmp(e, "gpu") == 0 || strcmp(e, "GPU") == 0);
}

// ---- tensors -> descriptors -------------------------------------------------------------------------

bool in_device_buffer(const ggml_tensor* t) {
    if (!t->buffer) return false;
    const ggml_backend_buffer_type_t bt = ggml_backend_buffer_get_type(t->buffer);
    for (DevState* s : devices())
        if (bt == &s->buft_device) return true;
    return false;
}

// Bytes the backend cannot read in place: a CPU repack buffer holds weights in the CPU backend's own
// interleaved layout (the reference declines such sources, ggml-rocket.cpp:7773-7794).
bool tensor_readable(const ggml_tensor* t) {
    if (!t->buffer) return true;
    const char* n = ggml_backend_buft_name(ggml_backend_buffer_get_type(t->buffer));
    return !(n && strstr(n, "REPACK"));
}

b200_tensor* declare(b200_graph_builder_t gb, const ggml_tensor* t) {
    if (b200_tensor* d = ggml_backend_b200_builder_find(gb, t)) return d;
    const void* srcs[B200_MAX_SRC] = {};
    for (int i = 0; i < GGML_MAX_SRC && i < B200_MAX_SRC; i++) {
        if (!t->src[i]) continue;
        if (!declare(gb, t->src[i])) return nullptr;
        srcs[i] = t->src[i];
    }
    const char* sub = nullptr;
    if (t->op == GGML_OP_UNARY) sub = ggml_unary_op_name(ggml_get_unary_op(t));
    else if (t->op == GGML_OP_GLU) sub = ggml_glu_op_name(ggml_get_glu_op(t));
    int32_t opp[B200_MAX_OP_PARAMS] = {};
    memcpy(opp, t->op_params, sizeof opp < sizeof t->op_params ? sizeof opp : sizeof t->op_params);
#ifdef GGML_HINT_SRC0_IS_HADAMARD
    // the Walsh-Hadamard hint in op_params[1]: the host's value becomes the library's (a host that
    // spells it as an enumerator rather than a macro passes its value through unchanged)
    if (t->op == GGML_OP_MUL_MAT)
        opp[1] = opp[1] == (int32_t)GGML_HINT_SRC0_IS_HADAMARD ? B200_HINT_SRC0_IS_HADAMARD : 0;
#endif
    return ggml_backend_b200_builder_add(gb, t, ggml_op_name(t->op), sub, (int32_t)t->type, t->ne, t->nb, opp, srcs,
                                         t->data, in_device_buffer(t) ? 1 : 0, tensor_readable(t) ? 1 : 0, t->name);
}

// One op's descriptor, for the claim rules (which read the op and its direct sources only).
template <typename F>
bool with_op(const ggml_tensor* op, F&& f) {
    thread_local b200_graph_builder_t gb = ggml_backend_b200_builder_new();
    ggml_backend_b200_builder_reset(gb);
    const b200_tensor* d = declare(gb, op);
    return d && f(d);
}

// ---- buffers: device memory ---------------------------------------------------------------------------

b200_buffer_t bufh(ggml_backend_buffer_t b) { return static_cast<b200_buffer_t>(b->context); }
size_t off_of(ggml_backend_buffer_t b, const ggml_tensor* t) {
    return (size_t)((const char*)t->data - (const char*)ggml_backend_b200_buffer_base(bufh(b)));
}

void dbuf_free(ggml_backend_buffer_t b) { ggml_backend_b200_buffer_free(bufh(b)); }
void* dbuf_base(ggml_backend_buffer_t b) { return ggml_backend_b200_buffer_base(bufh(b)); }
void dbuf_memset(ggml_backend_buffer_t b, ggml_tensor* t, uint8_t v, size_t o, size_t n) {
    ggml_backend_b200_buffer_memset(bufh(b), off_of(b, t) + o, v, n);
}
void dbuf_set(ggml_backend_buffer_t b, ggml_tensor* t, const void* data, size_t o, size_t n) {
    ggml_backend_b200_buffer_set(bufh(b), off_of(b, t) + o, data, n);
}
void dbuf_get(ggml_backend_buffer_t b, const ggml_tensor* t, void* data, size_t o, size_t n) {
    ggml_backend_b200_buffer_get(bufh(b), off_of(b, t) + o, data, n);
}
bool dbuf_cpy(ggml_backend_buffer_t b, const ggml_tensor* src, ggml_tensor* dst) {
    if (!in_device_buffer(src)) return false;
    return ggml_backend_b200_buffer_copy(bufh(src->buffer), off_of(src->buffer, src), bufh(b), off_of(b, dst),
                                         ggml_nbytes(src)) == B200_STATUS_SUCCESS;
}
void dbuf_clear(ggml_backend_buffer_t b, uint8_t v) { ggml_backend_b200_buffer_clear(bufh(b), v); }

ggml_backend_buffer_i device_buffer_iface() {
    ggml_backend_buffer_i i{};
    i.free_buffer = dbuf_free;
    i.get_base = dbuf_base;
    i.memset_tensor = dbuf_memset;
    i.set_tensor = dbuf_set;
    i.get_tensor = dbuf_get;
    i.cpy_tensor = dbuf_cpy;
    i.clear = dbuf_clear;
    return i;
}

const char* dbuft_name(ggml_backend_buffer_type_t) { return ggml_backend_b200_buffer_type_name(); }
ggml_backend_buffer_t dbuft_alloc(ggml_backend_buffer_type_t bt, size_t size) {
    DevState* s = state(bt->device);
    b200_buffer_t h = ggml_backend_b200_buffer_alloc(service(s), size ? size : 1);
    if (!h) return nullptr;
    return ggml_backend_buffer_init(bt, device_buffer_iface(), h, size);
}
size_t dbuft_align(ggml_backend_buffer_type_t) { return ggml_backend_b200_buffer_type_alignment(); }
size_t dbuft_max(ggml_backend_buffer_type_t bt) { return ggml_backend_b200_buffer_type_max_size(state(bt->device)->index); }
bool dbuft_is_host(ggml_backend_buffer_type_t) { return false; }

// ---- buffers: pinned host memory (the host buffer type) ---------------------------------------------

void hbuf_free(ggml_backend_buffer_t b) { ggml_backend_b200_host_free(b->context); }
void* hbuf_base(ggml_backend_buffer_t b) { return b->context; }
void hbuf_memset(ggml_backend_buffer_t, ggml_tensor* t, uint8_t v, size_t o, size_t n) {
    memset((char*)t->data + o, v, n);
}
void hbuf_set(ggml_backend_buffer_t, ggml_tensor* t, const void* data, size_t o, size_t n) {
    memcpy((char*)t->data + o, data, n);
}
void hbuf_get(ggml_backend_buffer_t, const ggml_tensor* t, void* data, size_t o, size_t n) {
    memcpy(data, (const char*)t->data + o, n);
}
bool hbuf_cpy(ggml_backend_buffer_t, const ggml_tensor* src, ggml_tensor* dst) {
    if (!src->buffer || !ggml_backend_buffer_is_host(src->buffer)) return false;
    memcpy(dst->data, src->data, ggml_nbytes(src));
    return true;
}
void hbuf_clear(ggml_backend_buffer_t b, uint8_t v) { memset(b->context, v, b->size); }

ggml_backend_buffer_i host_buffer_iface() {
    ggml_backend_buffer_i i{};
    i.free_buffer = hbuf_free;
    i.get_base = hbuf_base;
    i.memset_tensor = hbuf_memset;
    i.set_tensor = hbuf_set;
    i.get_tensor = hbuf_get;
    i.cpy_tensor = hbuf_cpy;
    i.clear = hbuf_clear;
    return i;
}

const char* hbuft_name(ggml_backend_buffer_type_t) { return "B200_Host"; }
ggml_backend_buffer_t hbuft_alloc(ggml_backend_buffer_type_t bt, size_t size) {
    void* p = ggml_backend_b200_host_alloc(size ? size : 1);
    if (!p) return nullptr;
    return ggml_backend_buffer_init(bt, host_buffer_iface(), p, size);
}
size_t hbuft_align(ggml_backend_buffer_type_t) { return 64; }
bool hbuft_is_host(ggml_backend_buffer_type_t) { return true; }

// ---- backend ------------------------------------------------------------------------------------------

DevState* bstate(ggml_backend_t be) { return static_cast<DevState*>(be->context); }

const char* be_name(ggml_backend_t) { return ggml_backend_b200_reg_name(); }
void be_free(ggml_backend_t be) {
    DevState* s = bstate(be);
    {
        std::lock_guard<std::mutex> lk(s->mu);
        s->refs--;
    }
    delete be;
}
void be_set_async(ggml_backend_t be, ggml_tensor* t, const void* data, size_t o, size_t n) {
    ggml_backend_b200_set_async(service(bstate(be)), bufh(t->buffer), off_of(t->buffer, t) + o, data, n);
}
void be_get_async(ggml_backend_t be, const ggml_tensor* t, void* data, size_t o, size_t n) {
    ggml_backend_b200_get_async(service(bstate(be)), bufh(t->buffer), off_of(t->buffer, t) + o, data, n);
}
bool be_cpy_async(ggml_backend_t src_be, ggml_backend_t dst_be, const ggml_tensor* src, ggml_tensor* dst) {
    if (!in_device_buffer(src) || !in_device_buffer(dst) || src_be->iface.get_name != dst_be->iface.get_name)
        return false;
    return ggml_backend_b200_copy_async(service(bstate(dst_be)), bufh(src->buffer), off_of(src->buffer, src),
                                        bufh(dst->buffer), off_of(dst->buffer, dst), ggml_nbytes(src)) ==
           B200_STATUS_SUCCESS;
}
void be_sync(ggml_backend_t be) { ggml_backend_b200_synchronize(service(bstate(be))); }

// graph_compute: the split's nodes declared in order (their sources first), then computed by the
// library; any node it cannot compute fails the split (no CPU fallback on a claimed op).
ggml_status be_graph_compute(ggml_backend_t be, ggml_cgraph* cg) {
    thread_local b200_graph_builder_t gb = ggml_backend_b200_builder_new();
    ggml_backend_b200_builder_reset(gb);
    const int n = ggml_graph_n_nodes(cg);
    for (int i = 0; i < n; i++) {
        ggml_tensor* node = ggml_graph_node(cg, i);
        if (!declare(gb, node) || ggml_backend_b200_builder_push_node(gb, node) < 0) return GGML_STATUS_FAILED;
    }
    const int st = ggml_backend_b200_builder_compute(service(bstate(be)), gb);
    return st == B200_STATUS_SUCCESS ? GGML_STATUS_SUCCESS
           : st == B200_STATUS_ALLOC_FAILED ? GGML_STATUS_ALLOC_FAILED : GGML_STATUS_FAILED;
}

void be_event_record(ggml_backend_t be, ggml_backend_event_t ev) {
    ggml_backend_b200_event_record(service(bstate(be)), static_cast<b200_event_t>(ev->context));
}
void be_event_wait(ggml_backend_t be, ggml_backend_event_t ev) {
    ggml_backend_b200_event_wait(service(bstate(be)), static_cast<b200_event_t>(ev->context));
}

ggml_guid_t guid() {
    static ggml_guid g = {0xb2, 0x00, 0x5e, 0x6e, 0x61, 0x74, 0x69, 0x76, 0x65, 0x67, 0x67, 0x6d, 0x6c, 0x72, 0x6b, 0x74};
    return &g;
}

ggml_backend_i backend_iface() {
    ggml_backend_i i{};
    i.get_name = be_name;
    i.free = be_free;
    i.set_tensor_async = be_set_async;
    i.get_tensor_async = be_get_async;
    i.cpy_tensor_async = be_cpy_async;
    i.synchronize = be_sync;
    i.graph_compute = be_graph_compute;
    i.event_record = be_event_record;
    i.event_wait = be_event_wait;
    return i;
}

// ---- device -------------------------------------------------------------------------------------------

const char* dev_name(ggml_backend_dev_t d) { return state(d)->name.c_str(); }
const char* dev_desc(ggml_backend_dev_t d) { return state(d)->desc.c_str(); }
void dev_memory(ggml_backend_dev_t d, size_t* fr, size_t* total) {
    ggml_backend_b200_device_memory(state(d)->index, fr, total);
}
enum ggml_backend_dev_type dev_type(ggml_backend_dev_t) {
    return gpu_mode() ? GGML_BACKEND_DEVICE_TYPE_GPU : GGML_BACKEND_DEVICE_TYPE_ACCEL;
}
void dev_props(ggml_backend_dev_t d, ggml_backend_dev_props* p) {
    p->name = dev_name(d);
    p->description = dev_desc(d);
    dev_memory(d, &p->memory_free, &p->memory_total);
    p->type = dev_type(d);
    bool as = false, hb = false, fp = false, ev = false;
    ggml_backend_b200_device_caps(state(d)->index, &as, &hb, &fp, &ev);
    p->caps.async = as;
    p->caps.host_buffer = hb;
    p->caps.buffer_from_host_ptr = fp;
    p->caps.events = ev;
}
ggml_backend_t dev_init(ggml_backend_dev_t d, const char*) {
    DevState* s = state(d);
    if (!service(s)) return nullptr;
    {
        std::lock_guard<std::mutex> lk(s->mu);
        s->refs++;
    }
    auto* be = new ggml_backend{};
    be->guid = guid();
    be->iface = backend_iface();
    be->device = d;
    be->context = s;
    return be;
}
ggml_backend_buffer_type_t dev_buft(ggml_backend_dev_t d) {
    if (gpu_mode()) return &state(d)->buft_device;
    // the reference's device hands out the host CPU buffer type (ggml-rocket.cpp:7326-7328)
    ggml_backend_dev_t cpu = ggml_backend_dev_by_type(GGML_BACKEND_DEVICE_TYPE_CPU);
    return cpu ? ggml_backend_dev_buffer_type(cpu) : &state(d)->buft_host;
}
ggml_backend_buffer_type_t dev_host_buft(ggml_backend_dev_t d) { return &state(d)->buft_host; }
bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor* op) {
    return with_op(op, [](const b200_tensor* t) { return ggml_backend_b200_supports_op(t); });
}
// host buffers (read by staging them), this device's memory and its pinned host buffers
bool dev_supports_buft(ggml_backend_dev_t d, ggml_backend_buffer_type_t bt) {
    return ggml_backend_buft_is_host(bt) || bt == &state(d)->buft_device || bt == &state(d)->buft_host;
}
bool dev_offload_op(ggml_backend_dev_t, const ggml_tensor* op) {
    return with_op(op, [](const b200_tensor* t) { return ggml_backend_b200_offload_op(t); });
}
ggml_backend_event_t dev_event_new(ggml_backend_dev_t d) {
    b200_event_t e = ggml_backend_b200_event_new(service(state(d)));
    if (!e) return nullptr;
    auto* ev = new ggml_backend_event{};
    ev->device = d;
    ev->context = e;
    return ev;
}
void dev_event_free(ggml_backend_dev_t, ggml_backend_event_t ev) {
    if (!ev) return;
    ggml_backend_b200_event_free(static_cast<b200_event_t>(ev->context));
    delete ev;
}
void dev_event_sync(ggml_backend_dev_t, ggml_backend_event_t ev) {
    ggml_backend_b200_event_synchronize(static_cast<b200_event_t>(ev->context));
}

ggml_backend_device_i device_iface() {
    ggml_backend_device_i i{};
    i.get_name = dev_name;
    i.get_description = dev_desc;
    i.get_memory = dev_memory;
    i.get_type = dev_type;
    i.get_props = dev_props;
    i.init_backend = dev_init;
    i.get_buffer_type = dev_buft;
    i.get_host_buffer_type = dev_host_buft;
    i.supports_op = dev_supports_op;
    i.supports_buft = dev_supports_buft;
    i.offload_op = dev_offload_op;
    i.event_new = dev_event_new;
    i.event_free = dev_event_free;
    i.event_synchronize = dev_event_sync;
    return i;
}

// ---- registry -----------------------------------------------------------------------------------------

const char* reg_name(ggml_backend_reg_t) { return ggml_backend_b200_reg_name(); }
size_t reg_count(ggml_backend_reg_t) { return devices().size(); }
ggml_backend_dev_t reg_device(ggml_backend_reg_t, size_t i) { return i < devices().size() ? &devices()[i]->dev : nullptr; }
// the public entry points a host may look up by name (the reference exports its own this way)
void* reg_proc(ggml_backend_reg_t, const char* name) {
    if (!name) return nullptr;
    if (strcmp(name, "ggml_backend_b200_set_n_gpus") == 0) return (void*)ggml_backend_b200_set_n_gpus;
    if (strcmp(name, "ggml_backend_b200_route_ops") == 0) return (void*)ggml_backend_b200_route_ops;
    if (strcmp(name, "ggml_backend_b200_moe_stats") == 0) return (void*)ggml_backend_b200_moe_stats;
    if (strcmp(name, "ggml_backend_b200_cpu_fallbacks") == 0) return (void*)ggml_backend_b200_cpu_fallbacks;
    return nullptr;
}

// The op-ordinal check (ggml-rocket.cpp:8231-8252, re-derived): the host's ggml must name every op
// this file switches on (by its compiled-in ordinal) the way these headers do. Names are what the
// library maps, so a host whose ordinals moved is refused rather than mistranslated.
bool ordinals_match() {
    static const struct { ggml_op op; const char* name; } ops[] = {
        {GGML_OP_MUL_MAT, "MUL_MAT"}, {GGML_OP_MUL_MAT_ID, "MUL_MAT_ID"}, {GGML_OP_FLASH_ATTN_EXT, "FLASH_ATTN_EXT"},
        {GGML_OP_UNARY, "UNARY"},     {GGML_OP_GLU, "GLU"},                {GGML_OP_VIEW, "VIEW"},
    };
    for (const auto& e : ops) {
        const char* got = ggml_op_name(e.op);
        if (!got || strcmp(got, e.name) != 0) {
            fprintf(stderr, "ggml-b200: the host's op %d is '%s', expected '%s': not loading\n", (int)e.op,
                    got ? got : "(null)", e.name);
            return false;
        }
    }
    return true;
}

}  // namespace

extern "C" ggml_backend_reg_t ggml_backend_b200_reg(void) {
    static std::once_flag once;
    static ggml_backend_reg reg{};
    static bool ok = false;
    std::call_once(once, [] {
        if (!ordinals_match()) return;
        const int n = ggml_backend_b200_reg_device_count();
        for (int i = 0; i < n; i++) {
            auto* s = new DevState();
            s->index = i;
            s->name = ggml_backend_b200_device_name(i);
            char buf[256] = {0};
            ggml_backend_b200_device_description(i, buf, sizeof buf);
            s->desc = buf;
            s->dev.iface = device_iface();
            s->dev.reg = &reg;
            s->dev.context = s;
            s->buft_device.iface = ggml_backend_buffer_type_i{};
            s->buft_device.iface.get_name = dbuft_name;
            s->buft_device.iface.alloc_buffer = dbuft_alloc;
            s->buft_device.iface.get_alignment = dbuft_align;
            s->buft_device.iface.get_max_size = dbuft_max;
            s->buft_device.iface.is_host = dbuft_is_host;
            s->buft_device.device = &s->dev;
            s->buft_host.iface = ggml_backend_buffer_type_i{};
            s->buft_host.iface.get_name = hbuft_name;
            s->buft_host.iface.alloc_buffer = hbuft_alloc;
            s->buft_host.iface.get_alignment = hbuft_align;
            s->buft_host.iface.is_host = hbuft_is_host;
            s->buft_host.device = &s->dev;
            devices().push_back(s);
        }
        reg.api_version = GGML_BACKEND_API_VERSION;
        reg.iface.get_name = reg_name;
        reg.iface.get_device_count = reg_count;
        reg.iface.get_device = reg_device;
        reg.iface.get_proc_address = reg_proc;
        reg.context = nullptr;
        ok = true;
    });
    return ok ? &reg : nullptr;
}

GGML_BACKEND_DL_IMPL(ggml_backend_b200_reg)
