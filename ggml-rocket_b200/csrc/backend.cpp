// The ggml B200 backend's host layer: what ggml-rocket decides on the host, re-implemented
// over plain b200_tensor descriptors (include/ggml-b200.h) and driving the sm_100a kernels
// (include/ggml-b200-kernels.h).
//
//   knobs          B200_* environment variables, read once; set-but-empty reads as unset
//                  (ggml-rocket.cpp:698-724)
//   claim rules    supports_op / offload_op (ggml-rocket.cpp:7334-7827)
//   breaker        the device-route circuit breaker (ggml-rocket.cpp:263-307)
//   weight cache   device-resident packed weights keyed by name + content fingerprint
//                  (ggml-rocket.cpp:4124-4222), so a weight crosses the host link once
//   graph_compute  the serial node walk with shared-src1 grouping (ggml-rocket.cpp:7088-7200)
//
// There is no CPU fallback: a claimed op that fails on the device fails the graph.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <functional>
#include <initializer_list>
#include <list>
#include <map>
#include <set>
#include <chrono>
#include <condition_variable>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "ggml-b200.h"

namespace {

// ------------------------------------------------------------------------------------------------
// logging and knobs
// ------------------------------------------------------------------------------------------------

void logf(const char* level, const char* fmt, ...) {
    static const bool quiet = [] {
        const char* e = getenv("B200_LOG");
        return e && *e && atoi(e) == 0;
    }();
    if (quiet && strcmp(level, "E") != 0) return;
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "[ggml-b200 %s] ", level);
    vfprintf(stderr, fmt, ap);
    va_end(ap);
}

int knob_int(const char* name, int dflt) {
    const char* e = getenv(name);
    return (e && *e) ? atoi(e) : dflt;
}
bool knob_on(const char* name, bool dflt) {
    const char* e = getenv(name);
    return (e && *e) ? (atoi(e) > 0) : dflt;
}

// Minimum rows a dense MUL_MAT must carry to be claimed (ggml-rocket.cpp:846-876), re-derived for
// B200 by the reference's method: the crossover where the claimed op (here graph_compute with the
// activation and result in host memory, copied in and out every call) meets the host CPU computing
// it. Measured on a B200 box (bench.py --workload crossover: one MUL_MAT per call, weights cached,
// 16 host cores; the CPU arm an fp32 BLAS over the dequantized weight, standing in for ggml's CPU
// backend), the device wins at every M >= 4 for F16 and Q4_K at K = 4096, N = 4096 / 14336: at
// M = 16, 80-170 us (pageable host memory) against 0.9-3.6 ms; at M = 4, 58-82 us against 0.4-2.1
// ms. A CPU that reads 4-bit weights directly (ggml's Q4_K path, memory-bound at these M) narrows
// that by up to ~8x, so the default keeps a margin: 16 rows, where even then the device stays ahead.
// Decode (M = 1) and batched-beam decode (M ~ 5) stay on the CPU unless B200_DECODE claims them for
// the decode kernels. Floor 4, as in the reference.
int min_m() {
    static const int m = [] { const int x = knob_int("B200_MIN_M", 16); return x < 4 ? 4 : x; }();
    return m;
}
// The floor for quantized weights (ggml-rocket.cpp:887-894). The reference's 512 pays for a
// per-call host dequant; the fused device dequant has no such cost and the same crossover
// measurement puts Q4_K at the dense floor, so the default equals min_m(). Never below min_m().
int min_m_quant() {
    static const int m = [] {
        const int x = knob_int("B200_MIN_M_QUANT", 16);
        return x < min_m() ? min_m() : x;
    }();
    return m;
}

// B200_GEMM_COMBINE: 1 (default) = a fused MUL_MAT group is one combined-N GEMM launch, 0 = one
// launch per member after the shared activation pack.
int combine_knob() {
    static const int v = knob_int("B200_GEMM_COMBINE", 1);
    return v;
}

enum MoeMode { MOE_OFF = 0, MOE_AUTO = 1, MOE_FORCED = 2 };
int moe_mode() {
    static const int v = [] {
        const char* e = getenv("B200_MOE");
        if (!e || !*e) return (int)MOE_AUTO;
        return atoi(e) > 0 ? (int)MOE_FORCED : (int)MOE_OFF;
    }();
    return v;
}
int moe_min_tokens() {
    static const int m = [] { const int x = knob_int("B200_MOE_MIN_TOKENS", 32); return x < min_m() ? min_m() : x; }();
    return m;
}
// AUTO's first floor: rows an expert receives on average (n_tokens * n_used / n_expert),
// rounded up to a power of two (ggml-rocket.cpp:952-961).
int moe_m_bucket() {
    static const int p = [] {
        int g = knob_int("B200_MOE_M_BUCKET", 8);
        if (g < 1) g = 1;
        int q = 1;
        while (q < g && q < (1 << 20)) q <<= 1;
        return q;
    }();
    return p;
}
// AUTO's second floor: MACs one expert GEMM carries, in millions (0 disables).
int moe_min_work_mmac() {
    static const int w = [] { int v = knob_int("B200_MOE_MIN_WORK", 0); return v < 0 ? 0 : v; }();
    return w;
}
bool flash_attn_on() {
    static const bool v = knob_int("B200_FLASH_ATTN", 1) > 0;
    return v;
}
int flash_attn_min_t() {
    static const int t = [] { const int x = knob_int("B200_FLASH_ATTN_MIN_T", 16); return x < 1 ? 1 : x; }();
    return t;
}
int flash_attn_min_kv() {
    static const int kv = [] { const int x = knob_int("B200_FLASH_ATTN_MIN_KV", 1024); return x < 1 ? 1 : x; }();
    return kv;
}
// FLASH_ATTN_EXT over a quantized KV cache (Q8_0 / Q4_0 K or V): converted to fp16 tiles, then the
// fp16 kernel (b200_kv_to_f16). Off by default: the reference declines these (F16 K / V only).
bool fa_quant_kv_on() {
    static const bool v = knob_on("B200_FA_QUANT_KV", false);
    return v;
}
bool flash_attn_unmasked() {
    static const bool v = knob_int("B200_FLASH_ATTN_UNMASKED", 0) > 0;
    return v;
}
// Decode-size MUL_MAT (M <= 32, Q4_K / Q6_K / Q8_0) on the GPU (b200_mul_mat_vec). Off by default:
// the reference leaves M below its offload threshold on the CPU; B200_DECODE=1 claims it.
bool decode_on() {
    static const bool v = knob_on("B200_DECODE", false);
    return v;
}

bool fuse_on() {
    static const bool v = knob_on("B200_FUSE", true);
    return v;
}
// The glue ops (RMS_NORM, ADD, MUL, SILU, SWIGLU, ROPE, GET_ROWS, CPY). Off by default: the
// reference claims none of them; B200_GLUE=1 keeps a layer's activations on the device.
bool glue_on() {
    static const bool v = knob_on("B200_GLUE", false);
    return v;
}
size_t weight_budget_bytes(int device) {
    const int mb = knob_int("B200_WEIGHT_BUDGET_MB", 0);
    if (mb > 0) return (size_t)mb << 20;
    size_t fr = 0, tot = 0;
    if (ggml_backend_b200_device_memory(device, &fr, &tot) != 0 || tot == 0) return (size_t)64 << 30;
    return tot / 10 * 8;   // 80 % of the device
}

// ------------------------------------------------------------------------------------------------
// tensor helpers (ggml semantics)
// ------------------------------------------------------------------------------------------------

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_I32 = 26, T_BF16 = 30 };

int64_t blck_size(int t) { return (t == T_Q8_0 || t == T_Q4_0) ? 32 : (t == T_Q4_K || t == T_Q6_K) ? 256 : 1; }
size_t type_size(int t) {
    switch (t) {
        case T_F32: case T_I32: return 4;
        case T_F16: case T_BF16: return 2;
        case T_Q4_0: return 18;   // a KV-cache type only (FLASH_ATTN_EXT); no weight route
        case T_Q8_0: return 34;
        case T_Q4_K: return 144;
        case T_Q6_K: return 210;
        default: return 0;
    }
}
bool is_quantized(int t) { return t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K; }
// Weight types the kernels read: F16 and the three GGUF formats natively; F32 and BF16 are
// converted to fp16 once, when the weight enters the cache (the reference decodes both to fp16,
// ggml-rocket.cpp:3853-3890).
bool weight_type_ok(int t) { return t == T_F16 || t == T_F32 || t == T_BF16 || is_quantized(t); }
int kernel_wtype(int t) { return (t == T_F32 || t == T_BF16) ? T_F16 : t; }

size_t row_bytes(int t, int64_t k) { return type_size(t) * (size_t)(k / blck_size(t)); }
size_t nbytes(const b200_tensor* t) {
    size_t n = row_bytes(t->type, t->ne[0]);
    for (int i = 1; i < 4; i++) n += (size_t)(t->ne[i] - 1) * t->nb[i];
    return t->ne[1] && t->ne[2] && t->ne[3] ? n : 0;
}
bool is_contiguous(const b200_tensor* t) {
    size_t next = type_size(t->type);
    if (t->nb[0] != next) return false;
    next = row_bytes(t->type, t->ne[0]);
    for (int i = 1; i < 4; i++) {
        if (t->ne[i] != 1 && t->nb[i] != next) return false;
        next *= (size_t)t->ne[i];
    }
    return true;
}
int32_t op_param_i32(const b200_tensor* op, int i) { return op->op_params[i]; }
float op_param_f32(const b200_tensor* op, int i) {
    float f;
    memcpy(&f, &op->op_params[i], 4);
    return f;
}

// ------------------------------------------------------------------------------------------------
// precision contract (ggml-rocket.cpp:7334-7404)
// ------------------------------------------------------------------------------------------------

// The accumulator of every route here is fp32 (tcgen05 accumulates in TMEM), which meets any
// declaration. The activation is rounded to fp16, so a src1 declaration above F16 (F32, BF16)
// is declined. A Hadamard-tagged MUL_MAT is declined: the CPU evaluates it as an exact
// O(n log n) transform, here it would be a dense fp16 GEMM.
bool prec_declines(const b200_tensor* op) {
    const int32_t src1 = op_param_i32(op, 3);
    if (src1 != B200_PREC_UNDECLARED && src1 < B200_PREC_F16) return true;
    if (op->op == B200_OP_MUL_MAT && op_param_i32(op, 1) == B200_HINT_SRC0_IS_HADAMARD) return true;
    return false;
}

// A Hadamard-tagged MUL_MAT runs on the device as the fast transform (b200_hadamard) when the glue
// ops are claimed and src0 is, exactly, c times the Sylvester-ordered Hadamard matrix of order n
// (H[i][k] = (-1)^popcount(i & k); n a power of two from 32 to 1024; F32 or F16; host-readable):
// then MUL_MAT's row i of dst = sum_k src0[i][k] x[k] = c (H x)[i]. Any other src0 under the hint
// stays declined, as in the reference. The check reads every entry; its result is cached by the
// data pointer with a fingerprint of sampled entries.
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {
            exp = 113;
            while (!(man & 0x400u)) { man <<= 1; exp--; }
            bits = sign | (exp << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

bool hadamard_scale(const b200_tensor* w, float* scale) {
    if (!w || (w->type != T_F32 && w->type != T_F16) || w->on_device || !w->data || !is_contiguous(w)) return false;
    const int64_t n = w->ne[0];
    if (w->ne[1] != n || w->ne[2] != 1 || w->ne[3] != 1 || n < 32 || n > 1024 || (n & (n - 1)) != 0) return false;
    auto at = [&](int64_t i, int64_t k) -> float {
        return w->type == T_F32 ? static_cast<const float*>(w->data)[i * n + k]
                                : half_bits_to_float(static_cast<const uint16_t*>(w->data)[i * n + k]);
    };
    uint64_t fp = 1469598103934665603ull;
    for (int64_t t = 0; t < 64; t++) {
        float v = at((t * 7919) % n, (t * 104729) % n);
        uint32_t b;
        std::memcpy(&b, &v, 4);
        fp = (fp ^ b) * 1099511628211ull;
    }
    struct Entry {
        int64_t n;
        int type;
        uint64_t fp;
        bool ok;
        float c;
    };
    static std::mutex mu;
    static std::unordered_map<const void*, Entry> cache;
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(w->data);
        if (it != cache.end() && it->second.n == n && it->second.type == w->type && it->second.fp == fp) {
            *scale = it->second.c;
            return it->second.ok;
        }
    }
    const float c = at(0, 0);
    bool ok = std::isfinite(c) && c != 0.0f;
    for (int64_t i = 0; i < n && ok; i++)
        for (int64_t k = 0; k < n && ok; k++) ok = at(i, k) == ((__builtin_popcountll(i & k) & 1) ? -c : c);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (cache.size() > 256) cache.clear();
        cache[w->data] = Entry{n, w->type, fp, ok, c};
    }
    *scale = c;
    return ok;
}

bool is_hadamard_op(const b200_tensor* op) {
    return op->op == B200_OP_MUL_MAT && op_param_i32(op, 1) == B200_HINT_SRC0_IS_HADAMARD;
}

// Claimable on the transform route: the glue ops are claimed, src0 passes hadamard_scale, src1 and
// dst are f32 with src1's rows of n values (any strides; dst contiguous). The f32 transform meets
// every precision declaration (accumulator and activation), so none declines it.
bool hadamard_claimable(const b200_tensor* op) {
    const b200_tensor* a = op->src[0];
    const b200_tensor* x = op->src[1];
    float c = 0.0f;
    if (!glue_on() || !a || !x || x->type != T_F32 || op->type != T_F32 || !is_contiguous(op)) return false;
    if (x->ne[0] != a->ne[0] || op->ne[0] != a->ne[1]) return false;
    for (int d = 1; d < 4; d++)
        if (op->ne[d] != x->ne[d]) return false;
    return hadamard_scale(a, &c);
}

bool sources_readable(const b200_tensor* op) {
    for (int i = 0; i < B200_MAX_SRC; i++)
        if (op->src[i] && !op->src[i]->readable) return false;
    return true;
}

// ------------------------------------------------------------------------------------------------
// MoE placement ledger (the reference's pre-flight, ggml-rocket.cpp:6131-6375): a process-wide
// reservation of whole expert stacks against the device budget, decided once per stack.
// ------------------------------------------------------------------------------------------------

struct MoeLedger {
    std::mutex mu;
    std::map<std::string, bool> decided;
    size_t reserved = 0;
};
MoeLedger& moe_ledger() {
    static MoeLedger l;
    return l;
}

}  // namespace

// ================================================================================================
// weight identity
// ================================================================================================

namespace {

uint64_t fingerprint(const b200_tensor* t, const void* host_bytes) {
    const size_t n = nbytes(t);
    const unsigned char* p = static_cast<const unsigned char*>(host_bytes);
    uint64_t h = 1469598103934665603ull ^ ((uint64_t)n * 0x100000001b3ull) ^ ((uint64_t)t->type << 48);
    auto eat = [&](size_t off, size_t len) {
        for (size_t i = 0; i < len; i++) {
            h ^= p[off + i];
            h *= 1099511628211ull;
        }
    };
    const int NS = 16;
    const size_t W = 64;
    if (n <= NS * W) eat(0, n);
    else
        for (int s = 0; s < NS; s++) eat((n - W) / (NS - 1) * (size_t)s, W);
    return h;
}

std::string weight_key(const b200_tensor* t) {
    const char* n = t->name;
    if (!n[0]) return std::string();
    std::string key(n, strnlen(n, B200_MAX_NAME));
    static const char PREFIX[] = "B200#";   // the scheduler's copy name: "<backend>#<tensor>#<copy>"
    const size_t pl = sizeof(PREFIX) - 1;
    if (key.compare(0, pl, PREFIX) == 0 && key.size() > pl) {
        key = key.substr(pl);
        const size_t h = key.rfind('#');
        if (h != std::string::npos && h > 0 && h + 1 < key.size() &&
            key.find_first_not_of("0123456789", h + 1) == std::string::npos)
            key.resize(h);
    }
    auto autoname = [](const std::string& s) {
        if (s.compare(0, 5, "leaf_") != 0 && s.compare(0, 5, "node_") != 0) return false;
        if (s.size() == 5) return false;
        return s.find_first_not_of("0123456789", 5) == std::string::npos;
    };
    if (autoname(key)) return std::string();
    char buf[96];
    snprintf(buf, sizeof buf, ":t%d:%lldx%lldx%lld", t->type, (long long)t->ne[0], (long long)t->ne[1],
             (long long)t->ne[2]);
    key += buf;
    if (t->data && !t->on_device) {
        snprintf(buf, sizeof buf, "@%016llx", (unsigned long long)fingerprint(t, t->data));
        key += buf;
    } else if (t->data) {
        // device bytes: keyed by where they live; writes through the buffer API drop the entry
        snprintf(buf, sizeof buf, "@d%llx", (unsigned long long)(uintptr_t)t->data);
        key += buf;
    }
    return key;
}

// ------------------------------------------------------------------------------------------------
// the breaker (ggml-rocket.cpp:263-307): three consecutive device failures open a route for 64
// calls, doubling per failed probe up to 4096; structural declines do not count.
// ------------------------------------------------------------------------------------------------

struct Breaker {
    int fails = 0;
    long skip = 0;
    long open_len = 0;
};
bool device_failure(int rc) { return rc < 0 && rc != B200_E_UNSUPPORTED && rc != B200_E_WORKSPACE; }
bool breaker_allow(Breaker& b) {
    if (b.skip > 0) {
        b.skip--;
        return false;
    }
    return true;
}
void breaker_note(Breaker& b, int rc, const char* route) {
    if (!device_failure(rc)) {
        if (rc == 0) {
            b.fails = 0;
            b.open_len = 0;
        }
        return;
    }
    if (++b.fails < 3) return;
    const long OPEN0 = 64, OPEN_MAX = 4096;
    b.open_len = b.open_len ? std::min(b.open_len * 2, OPEN_MAX) : OPEN0;
    b.skip = b.open_len;
    logf("W", "%s: %d consecutive device failures (last rc=%d); bypassed for the next %ld calls\n", route, b.fails, rc,
         b.skip);
}

}  // namespace

// ================================================================================================
// the backend context
// ================================================================================================

struct CachedWeight {
    void* dev = nullptr;
    size_t bytes = 0;
    int ktype = 0;            // the type the kernels read
    std::list<std::string>::iterator lru;
    uintptr_t src_lo = 0, src_hi = 0;   // device bytes it was packed from (on-device weights)
};

// Host bytes whose current value, written by an earlier op of the same graph, is still on the
// device in the staging arena: a later op reading them uses the device copy directly.
struct FwdRange {
    uintptr_t lo, hi;
    char* dev;
};
// A staged output on its way back into pageable host memory (copied out of pinned staging once
// the device-to-host copy has completed).
struct HostCopyBack {
    void* dst;
    const void* pinned;
    size_t n;
};

struct b200_backend {
    uint32_t magic = 0xB2000B20u;
    int device = 0;
    int n_gpus = 1;
    bool dev_ready = false;
    // compute, host-to-device and device-to-host streams: an op's input copies, its kernels and its
    // output copies are ordered by events, so one op's copies overlap its neighbours' kernels
    cudaStream_t stream = nullptr;
    cudaStream_t s_in = nullptr, s_out = nullptr;
    int* dev_err = nullptr;
    // grow-only device scratch arenas
    void* ws = nullptr;
    size_t ws_bytes = 0;
    void* pre = nullptr;                     // a norm-fused activation pack for the MUL_MATs after it (grow-only)
    size_t pre_bytes = 0;
    void* kv16 = nullptr;                    // a quantized KV cache's fp16 tiles (grow-only)
    size_t kv16_bytes = 0;
    // staging of host tensors, bump-allocated through one graph: device arena and pinned host
    // arena (for tensors in pageable memory); both are reset when the graph's copies have drained
    void* io = nullptr;
    size_t io_bytes = 0, io_off = 0;
    void* pin = nullptr;
    size_t pin_bytes = 0, pin_off = 0;
    bool in_pending = false;                 // input copies queued on s_in for the current op
    std::vector<FwdRange> fwd;               // host ranges whose newest bytes sit in the device arena
    std::vector<std::pair<uintptr_t, uintptr_t>> dirty;   // every host range an op of the graph wrote
    std::vector<HostCopyBack> copy_back;
    std::vector<cudaEvent_t> events;
    size_t ev_next = 0;
    void* wstage = nullptr;                  // native weight bytes on their way to the packer
    size_t wstage_bytes = 0;
    // weight cache
    std::unordered_map<std::string, CachedWeight> cache;
    std::list<std::string> lru;
    size_t cache_bytes = 0;
    size_t cache_budget = 0;
    // transient (unkeyed) weight uploads of the current graph
    std::vector<void*> transient;
    // counters
    std::map<std::string, long> route_ops;
    long device_errors = 0;
    long moe_resident = 0, moe_streamed = 0;
    std::map<std::string, bool> moe_seen;
    Breaker brk_fused;
    std::mutex mu;            // graph_compute is serial per instance
    std::set<b200_buffer*> buffers;   // live device buffers allocated through this instance
};

struct b200_buffer {
    uint32_t magic = 0xB200BF00u;
    b200_backend* owner = nullptr;    // nullptr once the backend is freed
    int device = 0;
    void* base = nullptr;
    size_t size = 0;
};

struct b200_event {
    uint32_t magic = 0xB200EE00u;
    int device = 0;
    cudaEvent_t ev = nullptr;
};

namespace {

bool cuda_ok(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    logf("E", "%s: %s\n", what, cudaGetErrorString(e));
    return false;
}

bool ensure_device(b200_backend* b) {
    if (b->dev_ready) return true;
    if (!cuda_ok(cudaSetDevice(b->device), "cudaSetDevice")) return false;
    if (!cuda_ok(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
    if (!cuda_ok(cudaStreamCreateWithFlags(&b->s_in, cudaStreamNonBlocking), "cudaStreamCreate(in)")) return false;
    if (!cuda_ok(cudaStreamCreateWithFlags(&b->s_out, cudaStreamNonBlocking), "cudaStreamCreate(out)")) return false;
    if (!cuda_ok(cudaMalloc(&b->dev_err, 256), "cudaMalloc(err)")) return false;
    if (!cuda_ok(cudaMemsetAsync(b->dev_err, 0, 256, b->stream), "cudaMemset(err)")) return false;
    b->cache_budget = weight_budget_bytes(b->device);
    b->dev_ready = true;
    return true;
}

bool grow(void** p, size_t* have, size_t need, cudaStream_t st) {
    if (*have >= need) return true;
    if (*p) {
        cudaStreamSynchronize(st);
        cudaFree(*p);
        *p = nullptr;
        *have = 0;
    }
    size_t sz = std::max(need, (size_t)1 << 20);
    sz = (sz + 4095) & ~(size_t)4095;
    if (cudaMalloc(p, sz) != cudaSuccess) return false;
    *have = sz;
    return true;
}

void evict_until(b200_backend* b, size_t need) {
    while (b->cache_bytes + need > b->cache_budget && !b->lru.empty()) {
        const std::string k = b->lru.back();
        b->lru.pop_back();
        auto it = b->cache.find(k);
        if (it != b->cache.end()) {
            cudaStreamSynchronize(b->stream);
            cudaFree(it->second.dev);
            b->cache_bytes -= it->second.bytes;
            b->cache.erase(it);
        }
    }
}

// Drop the cached packed weights whose device source bytes overlap [lo, hi).
void invalidate_range(b200_backend* b, uintptr_t lo, uintptr_t hi) {
    for (auto it = b->cache.begin(); it != b->cache.end();) {
        const CachedWeight& cw = it->second;
        if (cw.src_hi > lo && cw.src_lo < hi) {
            cudaStreamSynchronize(b->stream);
            cudaFree(cw.dev);
            b->cache_bytes -= cw.bytes;
            b->lru.erase(cw.lru);
            it = b->cache.erase(it);
        } else {
            ++it;
        }
    }
}

// Upload one [N, K] weight slab (native ggml bytes, host or device) into packed device form.
// Returns the packed device pointer (cached under `key` when non-empty).
void* pack_weight(b200_backend* b, const std::string& key, int type, const void* src, bool src_on_device, int64_t N,
                  int64_t K, int* ktype_out) {
    const int kt = kernel_wtype(type);
    *ktype_out = kt;
    if (!key.empty()) {
        auto it = b->cache.find(key);
        if (it != b->cache.end()) {
            b->lru.erase(it->second.lru);
            b->lru.push_front(key);
            it->second.lru = b->lru.begin();
            return it->second.dev;
        }
    }
    const size_t packed = b200_weight_packed_size(kt, N, K);
    const size_t native = row_bytes(type, K) * (size_t)N;
    if (packed == 0) return nullptr;
    if (!key.empty()) evict_until(b, packed);
    void* dst = nullptr;
    if (cudaMalloc(&dst, packed) != cudaSuccess) return nullptr;
    // stage the native bytes on the device, in a grow-only buffer the packer reads on the compute
    // stream (the next upload reuses it in stream order: no allocation or synchronisation per weight)
    const void* dsrc = src;
    if (!src_on_device) {
        if (!grow(&b->wstage, &b->wstage_bytes, native, b->stream) ||
            cudaMemcpyAsync(b->wstage, src, native, cudaMemcpyHostToDevice, b->stream) != cudaSuccess) {
            cudaFree(dst);
            return nullptr;
        }
        dsrc = b->wstage;
    }
    int rc;
    if (type == T_F32 || type == T_BF16) rc = b200_dequantize(type, dsrc, N, K, 1, dst, b->stream);
    else rc = b200_weight_pack(kt, dsrc, N, K, dst, b->stream);
    if (rc != B200_OK) {
        cudaFree(dst);
        return nullptr;
    }
    if (key.empty()) {
        b->transient.push_back(dst);
    } else {
        b->lru.push_front(key);
        CachedWeight cw;
        cw.dev = dst;
        cw.bytes = packed;
        cw.ktype = kt;
        cw.lru = b->lru.begin();
        if (src_on_device) {
            cw.src_lo = reinterpret_cast<uintptr_t>(src);
            cw.src_hi = cw.src_lo + native;
        }
        b->cache[key] = cw;
        b->cache_bytes += packed;
    }
    return dst;
}

// ---- host copies between pageable memory and the pinned arena ----------------------------------
// A pageable tensor of several MB copied by one thread runs at a fraction of the host link's speed,
// so large copies are split over a small process-wide pool of threads.
class CopyPool {
public:
    static CopyPool& get() {
        static CopyPool pool;
        return pool;
    }
    void memcpy_par(void* dst, const void* src, size_t n) {
        const size_t CHUNK = (size_t)1 << 20;
        if (n < 4 * CHUNK || workers_.empty()) {
            memcpy(dst, src, n);
            return;
        }
        std::lock_guard<std::mutex> serial(run_mu_);
        const size_t parts = workers_.size() + 1;
        const size_t per = ((n + parts - 1) / parts + 4095) & ~(size_t)4095;
        {
            std::lock_guard<std::mutex> lk(mu_);
            dst_ = static_cast<char*>(dst);
            src_ = static_cast<const char*>(src);
            n_ = n;
            per_ = per;
            remaining_ = (int)workers_.size();
            gen_++;
        }
        cv_.notify_all();
        part(0);   // the caller takes the first part
        std::unique_lock<std::mutex> lk(mu_);
        done_.wait(lk, [&] { return remaining_ == 0; });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }

private:
    CopyPool() {
        const unsigned hw = std::thread::hardware_concurrency();
        const int n = (int)std::min(7u, hw > 1 ? hw - 1 : 0u);
        for (int i = 0; i < n; i++) workers_.emplace_back([this, i] { loop(i + 1); });
    }
    void part(size_t k) {
        const size_t lo = k * per_;
        if (lo < n_) memcpy(dst_ + lo, src_ + lo, std::min(per_, n_ - lo));
    }
    void loop(size_t k) {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
            }
            part(k);
            std::lock_guard<std::mutex> lk(mu_);
            if (--remaining_ == 0) done_.notify_one();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex mu_, run_mu_;
    std::condition_variable cv_, done_;
    char* dst_ = nullptr;
    const char* src_ = nullptr;
    size_t n_ = 0, per_ = 0;
    int remaining_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

// ---- staging of host tensors ----------------------------------------------------------------
// A graph's host tensors are copied in on s_in and out on s_out; the op's kernels run on the
// compute stream between an event after its inputs and an event before its outputs. Tensors in
// pinned host memory (the backend's host buffers, or memory a host registered) are copied
// directly; pageable ones go through the pinned arena (memcpy on the host, then the copy; outputs
// land in pinned memory and are copied into place when the graph's copies have drained). An
// output written by one op and read by a later op of the same graph is read from its device
// copy, with no round trip through the host.

size_t staged_size(const b200_tensor* t) { return t->on_device ? 0 : ((nbytes(t) + 255) & ~(size_t)255); }

cudaEvent_t next_event(b200_backend* b) {
    if (b->ev_next == b->events.size()) {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
        b->events.push_back(e);
    }
    return b->events[b->ev_next++];
}

bool host_is_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// Wait for every queued copy and kernel, land the pageable outputs, and start both arenas over.
bool io_drain(b200_backend* b) {
    bool ok = cudaStreamSynchronize(b->s_in) == cudaSuccess;
    ok = cudaStreamSynchronize(b->stream) == cudaSuccess && ok;
    ok = cudaStreamSynchronize(b->s_out) == cudaSuccess && ok;
    for (const HostCopyBack& c : b->copy_back) CopyPool::get().memcpy_par(c.dst, c.pinned, c.n);
    b->copy_back.clear();
    b->fwd.clear();
    b->dirty.clear();
    b->io_off = b->pin_off = 0;
    b->ev_next = 0;
    b->in_pending = false;
    return ok;
}

bool grow_pinned(b200_backend* b, size_t need) {
    if (b->pin_bytes >= need) return true;
    if (b->pin) cudaFreeHost(b->pin);
    b->pin = nullptr;
    b->pin_bytes = 0;
    const size_t sz = (std::max(need, (size_t)1 << 22) + 4095) & ~(size_t)4095;
    if (cudaHostAlloc(&b->pin, sz, cudaHostAllocDefault) != cudaSuccess) return false;
    b->pin_bytes = sz;
    return true;
}

// Room for one op's staging (device bytes, pinned bytes), drained and grown first if the arenas
// cannot hold it after what the graph has already staged. After this, the op's own allocations
// never drain, so no copy queued for it can race a reuse of its region.
// An arena that runs out is grown to what the graph has used so far plus this op, so that the
// next graph of the same shape stages every op without draining in between (a drain serialises
// the copies and kernels that the streams would otherwise overlap).
bool io_reserve(b200_backend* b, size_t dev_need, size_t pin_need) {
    if (b->io_off + dev_need <= b->io_bytes && b->pin_off + pin_need <= b->pin_bytes) return true;
    const size_t dev_want = b->io_off + dev_need, pin_want = b->pin_off + pin_need;
    if (!io_drain(b)) return false;
    if (dev_want > b->io_bytes) {
        if (b->io) cudaFree(b->io);
        b->io = nullptr;
        b->io_bytes = 0;
        const size_t sz = (std::max(dev_want, (size_t)1 << 24) + 4095) & ~(size_t)4095;
        if (cudaMalloc(&b->io, sz) != cudaSuccess) return false;
        b->io_bytes = sz;
    }
    return grow_pinned(b, pin_want);
}

char* io_take(b200_backend* b, size_t n) {
    char* p = static_cast<char*>(b->io) + b->io_off;
    b->io_off += (n + 255) & ~(size_t)255;
    return p;
}
char* pin_take(b200_backend* b, size_t n) {
    char* p = static_cast<char*>(b->pin) + b->pin_off;
    b->pin_off += (n + 255) & ~(size_t)255;
    return p;
}

// The staging an op needs for these host tensors (inputs that an earlier op's output does not
// already hold on the device, and outputs); pinned bytes are counted for pageable tensors.
const FwdRange* fwd_find(const b200_backend* b, const b200_tensor* t) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(t->data), hi = lo + nbytes(t);
    for (const FwdRange& f : b->fwd)
        if (lo >= f.lo && hi <= f.hi) return &f;
    return nullptr;
}
// Host bytes an op of this graph wrote (their copy back may still be in flight or pending).
bool dirty_overlaps(const b200_backend* b, const b200_tensor* t) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(t->data), hi = lo + nbytes(t);
    for (const auto& d : b->dirty)
        if (hi > d.first && lo < d.second) return true;
    return false;
}

struct OpStaging {
    std::vector<const b200_tensor*> ins, outs;
};

bool op_reserve(b200_backend* b, const OpStaging& st) {
    // an input that touches bytes an earlier op wrote, without lying inside one device copy of
    // them: land everything first, then read the host
    for (const b200_tensor* t : st.ins)
        if (t && !t->on_device && !fwd_find(b, t) && dirty_overlaps(b, t)) {
            if (!io_drain(b)) return false;
            break;
        }
    size_t dev = 0, pin = 0;
    for (const b200_tensor* t : st.ins) {
        if (!t || t->on_device || fwd_find(b, t)) continue;
        dev += staged_size(t);
        if (!host_is_pinned(t->data)) pin += staged_size(t);
    }
    for (const b200_tensor* t : st.outs) {
        if (!t || t->on_device) continue;
        dev += staged_size(t);
        if (!host_is_pinned(t->data)) pin += staged_size(t);
    }
    return io_reserve(b, dev, pin);
}

// Device pointer holding a tensor's bytes for the op being set up: its own on the device, the
// device copy an earlier op of the graph left, or a fresh copy queued on s_in.
const void* stage_in(b200_backend* b, const b200_tensor* t, bool* ok) {
    if (t->on_device) return t->data;
    if (const FwdRange* f = fwd_find(b, t)) return f->dev + (reinterpret_cast<uintptr_t>(t->data) - f->lo);
    const size_t n = nbytes(t);
    char* d = io_take(b, n);
    const void* src = t->data;
    if (!host_is_pinned(src)) {
        // pageable: through the pinned arena in chunks, each chunk's copy to the device queued as soon
        // as it is in pinned memory, so the host copy of the next chunk overlaps it
        char* p = pin_take(b, n);
        const size_t CH = (size_t)8 << 20;
        for (size_t o = 0; o < n; o += CH) {
            const size_t c = std::min(CH, n - o);
            CopyPool::get().memcpy_par(p + o, static_cast<const char*>(src) + o, c);
            if (cudaMemcpyAsync(d + o, p + o, c, cudaMemcpyHostToDevice, b->s_in) != cudaSuccess) *ok = false;
        }
        b->in_pending = true;
        return d;
    }
    if (cudaMemcpyAsync(d, src, n, cudaMemcpyHostToDevice, b->s_in) != cudaSuccess) *ok = false;
    b->in_pending = true;
    return d;
}

// Device region for a host output of the op; read_in: the op writes only some of its bytes (a
// strided view), so the current host bytes are copied in first.
char* stage_out(b200_backend* b, const b200_tensor* t, bool read_in, bool* ok) {
    if (t->on_device) return static_cast<char*>(t->data);
    if (read_in) return const_cast<char*>(static_cast<const char*>(stage_in(b, t, ok)));
    return io_take(b, nbytes(t));
}

// The op's kernels may start once its input copies have landed.
bool op_inputs_ready(b200_backend* b) {
    if (!b->in_pending) return true;
    b->in_pending = false;
    cudaEvent_t e = next_event(b);
    return e && cudaEventRecord(e, b->s_in) == cudaSuccess && cudaStreamWaitEvent(b->stream, e, 0) == cudaSuccess;
}

// Queue the copies of the op's host outputs (dev: their device regions) after its kernels, and
// remember where their bytes live until the graph's copies drain.
bool op_outputs_done(b200_backend* b, const std::vector<const b200_tensor*>& outs, const std::vector<char*>& dev) {
    bool any = false;
    for (const b200_tensor* t : outs) any = any || !t->on_device;
    if (!any) return true;
    cudaEvent_t e = next_event(b);
    if (!e || cudaEventRecord(e, b->stream) != cudaSuccess || cudaStreamWaitEvent(b->s_out, e, 0) != cudaSuccess)
        return false;
    for (size_t i = 0; i < outs.size(); i++) {
        const b200_tensor* t = outs[i];
        if (t->on_device) continue;
        const size_t n = nbytes(t);
        void* dst = t->data;
        if (!host_is_pinned(dst)) {
            char* p = pin_take(b, n);
            b->copy_back.push_back({t->data, p, n});
            dst = p;
        }
        if (cudaMemcpyAsync(dst, dev[i], n, cudaMemcpyDeviceToHost, b->s_out) != cudaSuccess) return false;
        const uintptr_t lo = reinterpret_cast<uintptr_t>(t->data), hi = lo + n;
        b->dirty.push_back({lo, hi});
        // written in place inside an existing device copy (a strided output read in from it): that
        // copy stays current; otherwise the new region replaces every copy it overlaps
        bool in_place = false;
        for (const FwdRange& f : b->fwd)
            if (lo >= f.lo && hi <= f.hi && dev[i] == f.dev + (lo - f.lo)) in_place = true;
        if (in_place) continue;
        for (auto it = b->fwd.begin(); it != b->fwd.end();)
            it = (hi > it->lo && lo < it->hi) ? b->fwd.erase(it) : it + 1;
        b->fwd.push_back({lo, hi, dev[i]});
    }
    return true;
}


}  // namespace

// ================================================================================================
// claim rules
// ================================================================================================

// The shapes, types and parameters the glue kernels (glue.cu) implement; anything else stays
// with the host's CPU backend.
static bool same_shape(const b200_tensor* a, const b200_tensor* b) {
    return a->ne[0] == b->ne[0] && a->ne[1] == b->ne[1] && a->ne[2] == b->ne[2] && a->ne[3] == b->ne[3];
}
static bool glue_supported(const b200_tensor* op) {
    const b200_tensor* a = op->src[0];
    const b200_tensor* b = op->src[1];
    if (!a) return false;
    for (int i = 0; i < 4; i++)
        if (op->ne[i] <= 0) return false;
    switch (op->op) {
        case B200_OP_RMS_NORM:
            return a->type == T_F32 && op->type == T_F32 && is_contiguous(op) && same_shape(a, op) &&
                   op_param_f32(op, 0) >= 0.0f;
        case B200_OP_ADD:
        case B200_OP_MUL:
        case B200_OP_DIV: {
            if (!b || a->type != T_F32 || b->type != T_F32 || op->type != T_F32 || !is_contiguous(op) ||
                !same_shape(a, op))
                return false;
            for (int i = 0; i < 4; i++)
                if (b->ne[i] <= 0 || a->ne[i] % b->ne[i] != 0) return false;
            return true;
        }
        case B200_OP_UNARY:
            return op->op_params[0] == B200_UNARY_SILU && a->type == T_F32 && op->type == T_F32 &&
                   is_contiguous(op) && same_shape(a, op);
        case B200_OP_GLU: {
            if (op->op_params[0] != B200_GLU_SWIGLU || a->type != T_F32 || op->type != T_F32 || !is_contiguous(op))
                return false;
            if (b) return b->type == T_F32 && same_shape(a, op) && same_shape(b, op);
            // one input: its two halves along ne[0]
            return a->ne[0] == 2 * op->ne[0] && a->ne[1] == op->ne[1] && a->ne[2] == op->ne[2] &&
                   a->ne[3] == op->ne[3];
        }
        case B200_OP_ROPE: {
            const int n_dims = op->op_params[1], mode = op->op_params[2];
            return b && !op->src[2] && a->type == T_F32 && op->type == T_F32 && b->type == T_I32 &&
                   is_contiguous(op) && same_shape(a, op) && a->ne[3] == 1 && b->ne[0] == a->ne[2] &&
                   a->ne[0] % 2 == 0 && n_dims > 0 && n_dims % 2 == 0 && n_dims <= a->ne[0] &&
                   (mode == 0 || mode == 2) && op_param_f32(op, 7) == 0.0f && op_param_f32(op, 5) > 0.0f;
        }
        case B200_OP_GET_ROWS:
            return b && (a->type == T_F32 || a->type == T_F16) && b->type == T_I32 && op->type == T_F32 &&
                   is_contiguous(op) && op->ne[0] == a->ne[0] && op->ne[1] == b->ne[0] && op->ne[2] == b->ne[1] &&
                   op->ne[3] == b->ne[2] && b->ne[3] == 1 && b->ne[1] <= a->ne[2] && b->ne[2] <= a->ne[3];
        case B200_OP_SOFT_MAX:   // no mask, no ALiBi slope, no sinks
            return !b && !op->src[2] && a->type == T_F32 && op->type == T_F32 && is_contiguous(op) &&
                   same_shape(a, op) && op_param_f32(op, 1) == 0.0f;
        case B200_OP_ARGSORT:
            return a->type == T_F32 && op->type == T_I32 && is_contiguous(op) && same_shape(a, op) &&
                   a->ne[0] <= 1024 && (op->op_params[0] == 0 || op->op_params[0] == 1);
        case B200_OP_SUM_ROWS:
            return a->type == T_F32 && op->type == T_F32 && is_contiguous(op) && op->ne[0] == 1 &&
                   op->ne[1] == a->ne[1] && op->ne[2] == a->ne[2] && op->ne[3] == a->ne[3];
        case B200_OP_CPY: {
            const bool types = (a->type == T_F32 || a->type == T_F16) && (op->type == T_F32 || op->type == T_F16);
            const int64_t na = a->ne[0] * a->ne[1] * a->ne[2] * a->ne[3];
            const int64_t nd = op->ne[0] * op->ne[1] * op->ne[2] * op->ne[3];
            return types && na == nd && (same_shape(a, op) || is_contiguous(op));
        }
        default:
            return false;
    }
}

extern "C" bool ggml_backend_b200_supports_op(const b200_tensor* op) {
    if (!op) return false;
    if (!sources_readable(op)) return false;
    switch (op->op) {
        case B200_OP_NONE:
        case B200_OP_RESHAPE:
        case B200_OP_VIEW:
        case B200_OP_PERMUTE:
        case B200_OP_TRANSPOSE:
            return true;
        case B200_OP_MUL_MAT: {
            const b200_tensor* a = op->src[0];
            const b200_tensor* bb = op->src[1];
            if (!a || !bb) return false;
            if (is_hadamard_op(op)) return hadamard_claimable(op);
            if (prec_declines(op)) return false;
            const int64_t K = a->ne[0], N = a->ne[1], M = bb->ne[1];
            const bool aq = is_quantized(a->type);
            const bool base = a->op == B200_OP_NONE && weight_type_ok(a->type) && bb->type == T_F32 &&
                              op->type == T_F32 && is_contiguous(a) && is_contiguous(bb) && is_contiguous(op) &&
                              a->ne[0] == bb->ne[0] && a->ne[2] == 1 && a->ne[3] == 1 &&
                              (!aq || K % blck_size(a->type) == 0) && K % 32 == 0 && N % 16 == 0 && K >= 64 &&
                              N >= 64;
            if (base && M >= (aq ? min_m_quant() : min_m())) return true;
            // decode (opt-in): Q4_K / Q6_K / Q8_0 weights against 1..32 token rows below the floor, one
            // 2-D activation (b200_mul_mat_vec)
            return base && decode_on() && (a->type == T_Q4_K || a->type == T_Q6_K || a->type == T_Q8_0) && M >= 1 &&
                   M <= 32 && bb->ne[2] == 1 && bb->ne[3] == 1;
        }
        case B200_OP_MUL_MAT_ID: {
            const int mode = moe_mode();
            if (mode == MOE_OFF) return false;
            const b200_tensor* a = op->src[0];
            const b200_tensor* bb = op->src[1];
            const b200_tensor* ids = op->src[2];
            if (!a || !bb || !ids) return false;
            if (prec_declines(op)) return false;
            const int64_t K = a->ne[0], N = a->ne[1], n_tokens = ids->ne[1];
            const bool aq = is_quantized(a->type);
            const bool computable = a->op == B200_OP_NONE && weight_type_ok(a->type) && bb->type == T_F32 &&
                                    ids->type == T_I32 && op->type == T_F32 && is_contiguous(a) &&
                                    is_contiguous(bb) && is_contiguous(op) && a->ne[0] == bb->ne[0] &&
                                    a->ne[3] == 1 && (!aq || K % blck_size(a->type) == 0) && K % 32 == 0 &&
                                    N % 16 == 0 && K >= 64 && N >= 64 && n_tokens >= moe_min_tokens() &&
                                    a->ne[2] > 0;
            if (!computable) return false;
            if (mode == MOE_FORCED) return true;
            // AUTO: the rows an expert receives on average and the work one expert GEMM
            // carries, each against its floor; then the whole stack reserved on the device.
            const int64_t n_used = ids->ne[0], n_expert = a->ne[2];
            const int64_t m_e = n_tokens * n_used / n_expert;
            if (m_e < moe_m_bucket()) return false;
            if (m_e * K * N < (int64_t)moe_min_work_mmac() * 1000000) return false;
            const std::string key = weight_key(a);
            const size_t stack = b200_weight_packed_size(kernel_wtype(a->type), N, K) * (size_t)n_expert;
            MoeLedger& L = moe_ledger();
            std::lock_guard<std::mutex> lk(L.mu);
            if (!key.empty()) {
                auto it = L.decided.find(key);
                if (it != L.decided.end()) return it->second;
            }
            const size_t budget = weight_budget_bytes(0);
            const bool fits = L.reserved + stack <= budget;
            if (fits) L.reserved += stack;
            if (!key.empty()) L.decided[key] = fits;
            return fits;
        }
        case B200_OP_FLASH_ATTN_EXT: {
            const b200_tensor* q = op->src[0];
            const b200_tensor* k = op->src[1];
            const b200_tensor* v = op->src[2];
            const b200_tensor* m = op->src[3];
            if (!flash_attn_on() || !q || !k || !v) return false;
            if (!m && !flash_attn_unmasked()) return false;
            if (op->src[4]) return false;   // attention sinks: a different softmax (ggml-rocket.cpp:7703-7721)
            const float max_bias = op_param_f32(op, 1);
            const int64_t D = q->ne[0], T = q->ne[1], H = q->ne[2], DV = v->ne[0];
            const int64_t KV = k->ne[1], HK = k->ne[2];
            auto aligned16 = [](const b200_tensor* t) {
                return (t->nb[1] % 16 == 0) && (t->nb[2] % 16 == 0) && (t->on_device ? ((uintptr_t)t->data % 16 == 0) : true);
            };
            // a quantized cache: 32-value blocks along the head dimension, read as bytes, so no
            // 16-byte alignment is needed of its view
            auto kv_ok = [&](const b200_tensor* t) {
                if (t->type == T_F16) return t->nb[0] == 2 && aligned16(t);
                return fa_quant_kv_on() && (t->type == T_Q8_0 || t->type == T_Q4_0) && t->ne[0] % 32 == 0 &&
                       t->nb[0] == (size_t)(t->type == T_Q8_0 ? 34 : 18) && (t->on_device || is_contiguous(t));
            };
            return max_bias == 0.0f && q->type == T_F32 && kv_ok(k) && kv_ok(v) &&
                   (!m || (m->type == T_F16 && is_contiguous(m))) && op->type == T_F32 && is_contiguous(op) &&
                   q->ne[3] == 1 && k->ne[3] == 1 && v->ne[3] == 1 && k->ne[0] == D && op->ne[0] == DV &&
                   v->ne[1] == KV && v->ne[2] == HK && q->nb[0] == 4 &&
                   (D == 64 || D == 128) && (DV == 64 || DV == 128) && HK > 0 && H % HK == 0 &&
                   (!m || (m->ne[0] >= KV && m->ne[1] >= T)) &&
                   T >= flash_attn_min_t() && KV >= flash_attn_min_kv();
        }
        case B200_OP_RMS_NORM:
        case B200_OP_ADD:
        case B200_OP_MUL:
        case B200_OP_UNARY:
        case B200_OP_GLU:
        case B200_OP_ROPE:
        case B200_OP_GET_ROWS:
        case B200_OP_CPY:
        case B200_OP_SOFT_MAX:
        case B200_OP_ARGSORT:
        case B200_OP_SUM_ROWS:
        case B200_OP_DIV:
            return glue_on() && glue_supported(op);
        default:
            return false;
    }
}

extern "C" bool ggml_backend_b200_offload_op(const b200_tensor* op) {
    return op && (op->op == B200_OP_MUL_MAT || op->op == B200_OP_MUL_MAT_ID) && ggml_backend_b200_supports_op(op);
}

// ================================================================================================
// handlers
// ================================================================================================

namespace {

const char* route_name(int ktype) {
    switch (ktype) {
        case T_F16: return "f16";
        case T_Q8_0: return "q8_0";
        case T_Q4_K: return "q4_K";
        case T_Q6_K: return "q6_K";
        default: return "other";
    }
}

// The device error word, read once per graph after everything queued has drained (kernels record
// bounded-wait give-ups, bad expert ids and bad row indices there; the first writer wins).
bool graph_finish(b200_backend* b) {
    int h = 0;
    bool ok = cudaMemcpyAsync(&h, b->dev_err, sizeof(int), cudaMemcpyDeviceToHost, b->stream) == cudaSuccess;
    ok = io_drain(b) && ok;
    if (!ok) {
        logf("E", "graph_compute: CUDA error %s\n", cudaGetErrorString(cudaGetLastError()));
        b->device_errors++;
        return false;
    }
    if (h == 0) return true;
    if (h == B200_DEV_BAD_IDS) {
        logf("E", "graph_compute: a MUL_MAT_ID expert id outside [0, n_expert)\n");
    } else if (h == 6) {   // the kernels' bounds-check code (GET_ROWS row index outside the table)
        logf("E", "graph_compute: a GET_ROWS row index outside its table\n");
        b->device_errors++;
    } else {
        logf("E", "graph_compute: device error word %d\n", h);
        b->device_errors++;
    }
    cudaMemsetAsync(b->dev_err, 0, sizeof(int), b->stream);
    cudaStreamSynchronize(b->stream);
    return false;
}

// MUL_MAT, including ggml's batch broadcast over dims 2/3 (ggml-rocket.cpp:4725-4750), and a
// group of MUL_MATs sharing src1 (fused: one activation pack, then one combined-N GEMM launch over
// every member's weight tiles, or one GEMM per member when their types differ).
// pre_a16 / pre_scales (not null): src1 was packed by the kernel before it (a norm fused with the
// pack) and its f32 rows were never written; the caller guarantees no member takes the decode kernel.
int do_mul_mat_group(b200_backend* b, b200_tensor* const* nodes, int ng, const void* pre_a16 = nullptr,
                     const float* pre_scales = nullptr) {
    const bool pre = pre_a16 != nullptr;
    const b200_tensor* node0 = nodes[0];
    const b200_tensor* src1 = node0->src[1];
    const int64_t K = src1->ne[0], M = src1->ne[1];
    const int64_t ne12 = src1->ne[2], ne13 = src1->ne[3];
    // weights
    std::vector<void*> wdev(ng);
    std::vector<int> kt(ng);
    for (int g = 0; g < ng; g++) {
        const b200_tensor* a = nodes[g]->src[0];
        const std::string key = weight_key(a);
        const int64_t N = a->ne[1];
        wdev[g] = pack_weight(b, key, a->type, a->data, a->on_device != 0, N * a->ne[2] * a->ne[3], K, &kt[g]);
        if (!wdev[g]) return B200_E_CUDA;
    }
    // staging: src1 and the members' dst when they are host tensors; workspace: A16 + scales + GEMM
    OpStaging stg;
    if (!pre) stg.ins.push_back(src1);
    size_t need_ws = 0;
    for (int g = 0; g < ng; g++) {
        const b200_tensor* d = nodes[g];
        stg.outs.push_back(d);
        need_ws = std::max(need_ws, b200_gemm_packed_workspace_size(kernel_wtype(d->src[0]->type), M, d->src[0]->ne[1], K));
    }
    // decode-size M (claimed only under B200_DECODE, quantized weights): the weight-streaming kernel
    // for those members, the GEMM (after one shared activation pack) for the rest
    std::vector<char> dec(ng, 0);
    bool any_dec = false, any_gemm = false;
    for (int g = 0; g < ng; g++) {
        dec[g] = M < min_m_quant() && M <= 32 && kt[g] != T_F16;   // F32 / BF16 weights run as F16
        any_dec = any_dec || dec[g];
        any_gemm = any_gemm || !dec[g];
        if (dec[g]) need_ws = std::max(need_ws, b200_mul_mat_vec_workspace_size(M, nodes[g]->src[0]->ne[1], K));
    }
    if (pre && any_dec) return B200_E_INVALID;
    // A group of 2-4 GEMM-sized members of one weight type runs as one combined-N launch
    // (B200_GEMM_COMBINE=0: one launch per member, as the single-op path does).
    bool comb = ng >= 2 && ng <= 4 && !any_dec && combine_knob() != 0;
    for (int g = 1; g < ng && comb; g++) comb = kt[g] == kt[0];
    if (comb) {
        std::vector<int64_t> ns(ng);
        for (int g = 0; g < ng; g++) ns[g] = nodes[g]->src[0]->ne[1];
        need_ws = std::max(need_ws, b200_gemm_packed_group_workspace_size(ng, kt[0], M, ns.data(), K));
    }
    const size_t a16_bytes = ((size_t)M * K * 2 + 255) & ~(size_t)255;
    const size_t sc_bytes = ((size_t)M * 4 + 255) & ~(size_t)255;
    need_ws = ((need_ws + 255) & ~(size_t)255) + a16_bytes + sc_bytes;
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    if (!grow(&b->ws, &b->ws_bytes, need_ws, b->stream)) return B200_E_CUDA;
    bool ok = true;
    const char* a_base = pre ? nullptr : static_cast<const char*>(stage_in(b, src1, &ok));
    std::vector<char*> d_base(ng);
    for (int g = 0; g < ng; g++) d_base[g] = stage_out(b, nodes[g], false, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    char* ws = static_cast<char*>(b->ws);
    void* a16 = pre ? const_cast<void*>(pre_a16) : ws;
    float* scales = pre ? const_cast<float*>(pre_scales) : reinterpret_cast<float*>(ws + a16_bytes);
    void* gws = ws + a16_bytes + sc_bytes;
    const size_t gws_bytes = b->ws_bytes - a16_bytes - sc_bytes;
    for (int64_t i3 = 0; i3 < ne13; i3++) {
        for (int64_t i2 = 0; i2 < ne12; i2++) {
            const float* A = pre ? nullptr : reinterpret_cast<const float*>(a_base + i3 * src1->nb[3] + i2 * src1->nb[2]);
            for (int g = 0; g < ng; g++) {
                if (!dec[g]) continue;
                const b200_tensor* d = nodes[g];
                const int64_t N = d->src[0]->ne[1];
                float* C = reinterpret_cast<float*>(d_base[g] + i3 * d->nb[3] + i2 * d->nb[2]);
                const int rc = b200_mul_mat_vec(kt[g], wdev[g], N, K, A, (int64_t)(src1->nb[1] / 4), M, C,
                                                (int64_t)(d->nb[1] / 4), gws, gws_bytes, b->dev_err, b->stream);
                if (rc != B200_OK) return rc;
            }
            if (!any_gemm) continue;
            int rc = pre ? B200_OK : b200_act_pack(A, (int64_t)(src1->nb[1] / 4), M, K, a16, scales, b->stream);
            if (rc != B200_OK) return rc;
            if (comb) {
                // one combined-N launch over every member (all 2-D, one type, GEMM-sized)
                std::vector<const void*> ws_w(ng);
                std::vector<int64_t> ns(ng), lds(ng);
                std::vector<float*> cs(ng);
                for (int g = 0; g < ng; g++) {
                    const b200_tensor* d = nodes[g];
                    ws_w[g] = wdev[g];
                    ns[g] = d->src[0]->ne[1];
                    lds[g] = (int64_t)(d->nb[1] / 4);
                    cs[g] = reinterpret_cast<float*>(d_base[g] + i3 * d->nb[3] + i2 * d->nb[2]);
                }
                rc = b200_gemm_packed_group(ng, kt[0], ws_w.data(), ns.data(), K, a16, scales, M, cs.data(),
                                            lds.data(), gws, gws_bytes, b->dev_err, b->stream);
                if (rc != B200_OK) return rc;
                continue;
            }
            for (int g = 0; g < ng; g++) {
                if (dec[g]) continue;
                const b200_tensor* d = nodes[g];
                const b200_tensor* a = d->src[0];
                const int64_t N = a->ne[1];
                const int64_t r2 = ne12 / a->ne[2], r3 = ne13 / a->ne[3];
                const size_t wslab = b200_weight_packed_size(kt[g], N, K);
                const char* W = static_cast<const char*>(wdev[g]) + ((i3 / r3) * a->ne[2] + (i2 / r2)) * wslab;
                float* C = reinterpret_cast<float*>(d_base[g] + i3 * d->nb[3] + i2 * d->nb[2]);
                rc = b200_gemm_packed(kt[g], W, N, K, a16, scales, M, C, (int64_t)(d->nb[1] / 4), gws, gws_bytes,
                                      b->dev_err, b->stream);
                if (rc != B200_OK) return rc;
            }
        }
    }
    if (!op_outputs_done(b, stg.outs, d_base)) return B200_E_CUDA;
    if (any_dec) b->route_ops["decode"] += std::count(dec.begin(), dec.end(), (char)1);
    if (!any_gemm) {
        // every member ran on the decode kernel
    } else if (ng > 1) b->route_ops["fused"]++;
    else b->route_ops[route_name(kt[0])]++;
    return B200_OK;
}

// Fusable: a static 2-D weight of a kernel-native type feeding off a shared src1
// (ggml-rocket.cpp:4928-4944). Quantized weights fuse too: the shared pack is free here.
bool node_fusable(const b200_tensor* op) {
    if (op->op != B200_OP_MUL_MAT || is_hadamard_op(op)) return false;
    const b200_tensor* a = op->src[0];
    const b200_tensor* bb = op->src[1];
    return a->ne[2] == 1 && a->ne[3] == 1 && bb->ne[2] == 1 && bb->ne[3] == 1 && ggml_backend_b200_supports_op(op);
}

// MUL_MAT_ID, and a group of MUL_MAT_IDs reading the same b and ids (a MoE layer's gate and up
// projections): the route and the packed rows are made once for the group (b200_mul_mat_id_group).
int do_mul_mat_id_group(b200_backend* b, b200_tensor* const* ops, int ng) {
    const b200_tensor* op0 = ops[0];
    const b200_tensor* bb = op0->src[1];
    const b200_tensor* ids = op0->src[2];
    const int64_t K = op0->src[0]->ne[0], n_expert = op0->src[0]->ne[2];
    const int64_t ne11 = bb->ne[1], n_used = ids->ne[0], n_tokens = ids->ne[1];
    std::vector<const void*> w(ng);
    std::vector<int64_t> Ns(ng), nb1(ng), nb2(ng);
    std::vector<float*> dsts(ng);
    int kt = 0;
    for (int g = 0; g < ng; g++) {
        const b200_tensor* as = ops[g]->src[0];
        const std::string key = weight_key(as);
        int ktg = 0;
        w[g] = pack_weight(b, key, as->type, as->data, as->on_device != 0, as->ne[1] * n_expert, K, &ktg);
        if (!w[g]) return B200_E_CUDA;
        if (g == 0) kt = ktg;
        else if (ktg != kt) return B200_E_UNSUPPORTED;
        if (!key.empty() && !b->moe_seen[key]) {
            b->moe_seen[key] = true;
            b->moe_resident++;
        } else if (key.empty()) {
            b->moe_streamed++;
        }
        Ns[g] = as->ne[1];
        nb1[g] = (int64_t)ops[g]->nb[1];
        nb2[g] = (int64_t)ops[g]->nb[2];
    }
    size_t need_ws = 0;
    for (int g = 0; g < ng; g++)
        need_ws = std::max(need_ws, b200_mul_mat_id_workspace_size(K, Ns[g], n_expert, n_used, n_tokens));
    OpStaging stg;
    stg.ins = {bb, ids};
    for (int g = 0; g < ng; g++) stg.outs.push_back(ops[g]);
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    if (!grow(&b->ws, &b->ws_bytes, need_ws, b->stream)) return B200_E_CUDA;
    bool ok = true;
    const void* bd = stage_in(b, bb, &ok);
    const void* idd = stage_in(b, ids, &ok);
    std::vector<char*> d_dev(ng);
    for (int g = 0; g < ng; g++) {
        d_dev[g] = stage_out(b, ops[g], false, &ok);
        dsts[g] = reinterpret_cast<float*>(d_dev[g]);
    }
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    int rc = b200_mul_mat_id_group(ng, kt, w.data(), Ns.data(), K, n_expert, static_cast<const float*>(bd),
                                   (int64_t)bb->nb[1], (int64_t)bb->nb[2], ne11, static_cast<const int32_t*>(idd),
                                   (int64_t)ids->nb[0], (int64_t)ids->nb[1], n_used, n_tokens, dsts.data(), nb1.data(),
                                   nb2.data(), b->ws, b->ws_bytes, b->dev_err, b->stream);
    if (rc != B200_OK) return rc;
    if (!op_outputs_done(b, stg.outs, d_dev)) return B200_E_CUDA;
    b->route_ops["moe"] += ng;
    if (ng > 1) b->route_ops["moe_grouped"] += ng;
    return B200_OK;
}

int do_mul_mat_id(b200_backend* b, b200_tensor* op) { return do_mul_mat_id_group(b, &op, 1); }

// Members of one MUL_MAT_ID group: the same b and ids tensors, the same K, expert count and weight
// type (each member's stack is a leaf, so hoisting a later member cannot skip a dependency).
static bool mmid_groupable(const b200_tensor* a, const b200_tensor* c) {
    return c->op == B200_OP_MUL_MAT_ID && c->src[1] == a->src[1] && c->src[2] == a->src[2] &&
           c->src[0]->ne[0] == a->src[0]->ne[0] && c->src[0]->ne[2] == a->src[0]->ne[2] &&
           c->src[0]->type == a->src[0]->type && ggml_backend_b200_supports_op(c);
}

// A MoE block's expert FFN as ggml builds it: MUL_MAT_ID up and gate over the same x and ids
// (nodes i and i + 1, either order), GLU SWIGLU of the two (i + 2), and the down MUL_MAT_ID of the
// SWIGLU over the same ids (i + 3). It runs as one b200_mul_mat_id_ffn (one route, the SWIGLU fused
// into the down projection's packing) when the three intermediate tensors are device tensors that
// no other node reads: they are then never written. *gate / *up: the nodes silu and the product
// take (the GLU's swapped flag exchanges them).
static bool moe_ffn_match(b200_tensor* const* nodes, int n, int i, const std::vector<bool>& done,
                          const b200_tensor** gate, const b200_tensor** up) {
    if (i + 3 >= n || done[i + 1] || done[i + 2] || done[i + 3]) return false;
    const b200_tensor* p0 = nodes[i];
    const b200_tensor* p1 = nodes[i + 1];
    const b200_tensor* glu = nodes[i + 2];
    const b200_tensor* down = nodes[i + 3];
    if (!mmid_groupable(p0, p1) || glu->op != B200_OP_GLU || glu->op_params[0] != B200_GLU_SWIGLU || !glu->src[1] ||
        !ggml_backend_b200_supports_op(glu))
        return false;
    if (!((glu->src[0] == p0 && glu->src[1] == p1) || (glu->src[0] == p1 && glu->src[1] == p0))) return false;
    const bool swapped = glu->op_params[1] != 0;
    *gate = swapped ? glu->src[1] : glu->src[0];
    *up = swapped ? glu->src[0] : glu->src[1];
    if (down->op != B200_OP_MUL_MAT_ID || down->src[1] != glu || down->src[2] != p0->src[2] ||
        !ggml_backend_b200_supports_op(down))
        return false;
    const b200_tensor* wg = (*gate)->src[0];
    const b200_tensor* wd = down->src[0];
    const int64_t H = wg->ne[0], F = wg->ne[1], E = wg->ne[2];
    if (wd->ne[0] != F || wd->ne[1] != H || wd->ne[2] != E || (*up)->src[0]->ne[1] != F) return false;
    // h [F, n_used, n_tokens]: the down projection reads row (slot, token) of it
    if (glu->ne[0] != F || glu->ne[1] != p0->src[2]->ne[0] || glu->ne[2] != p0->src[2]->ne[1]) return false;
    if (H % 32 || F % 32 || F > 8192) return false;
    const b200_tensor* mid[3] = {p0, p1, glu};
    for (const b200_tensor* t : mid)
        if (!t->on_device) return false;
    for (int j = 0; j < n; j++) {
        if (j >= i && j <= i + 3) continue;
        for (int k = 0; k < B200_MAX_SRC; k++)
            for (const b200_tensor* t : mid)
                if (nodes[j]->src[k] == t) return false;
    }
    return true;
}

int do_moe_ffn(b200_backend* b, const b200_tensor* gate, const b200_tensor* up, const b200_tensor* down) {
    const b200_tensor* x = gate->src[1];
    const b200_tensor* ids = gate->src[2];
    const b200_tensor* st[3] = {gate->src[0], up->src[0], down->src[0]};
    const int64_t H = st[0]->ne[0], F = st[0]->ne[1], n_expert = st[0]->ne[2];
    const int64_t ne11 = x->ne[1], n_used = ids->ne[0], n_tokens = ids->ne[1];
    const void* w[3];
    int kt[3];
    for (int m = 0; m < 3; m++) {
        const std::string key = weight_key(st[m]);
        const int64_t rows = st[m]->ne[1] * n_expert, K = st[m]->ne[0];
        w[m] = pack_weight(b, key, st[m]->type, st[m]->data, st[m]->on_device != 0, rows, K, &kt[m]);
        if (!w[m]) return B200_E_CUDA;
        if (!key.empty() && !b->moe_seen[key]) {
            b->moe_seen[key] = true;
            b->moe_resident++;
        } else if (key.empty()) {
            b->moe_streamed++;
        }
    }
    if (kt[0] != kt[1]) return B200_E_UNSUPPORTED;
    OpStaging stg;
    stg.ins = {x, ids};
    stg.outs = {down};
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    if (!grow(&b->ws, &b->ws_bytes, b200_mul_mat_id_ffn_workspace_size(H, F, n_expert, n_used, n_tokens), b->stream))
        return B200_E_CUDA;
    bool ok = true;
    const void* xd = stage_in(b, x, &ok);
    const void* idd = stage_in(b, ids, &ok);
    char* dd = stage_out(b, down, false, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    const int rc = b200_mul_mat_id_ffn(kt[0], w[0], w[1], kt[2], w[2], H, F, n_expert, static_cast<const float*>(xd),
                                       (int64_t)x->nb[1], (int64_t)x->nb[2], ne11, static_cast<const int32_t*>(idd),
                                       (int64_t)ids->nb[0], (int64_t)ids->nb[1], n_used, n_tokens,
                                       reinterpret_cast<float*>(dd), (int64_t)down->nb[1], (int64_t)down->nb[2], b->ws,
                                       b->ws_bytes, b->dev_err, b->stream);
    if (rc != B200_OK) return rc;
    std::vector<char*> bases{dd};
    if (!op_outputs_done(b, stg.outs, bases)) return B200_E_CUDA;
    b->route_ops["moe"] += 3;
    b->route_ops["moe_grouped"] += 2;
    b->route_ops["moe_ffn"]++;
    b->route_ops["glue"]++;
    return B200_OK;
}

// A dense FFN as ggml builds it: GLU SWIGLU of the gate and up projections (node i, split form) and
// the down MUL_MAT that reads it (i + 1). When the SWIGLU output is a device tensor no other node
// reads, the pair runs as b200_swiglu_act_pack (the SWIGLU inside the down projection's activation
// pack) and the down GEMM: h is never written. *gate / *up: the tensors silu and the product take.
static bool swiglu_mm_match(b200_tensor* const* nodes, int n, int i, const std::vector<bool>& done,
                            const b200_tensor** gate, const b200_tensor** up) {
    if (i + 1 >= n || done[i + 1]) return false;
    const b200_tensor* glu = nodes[i];
    const b200_tensor* mm = nodes[i + 1];
    if (glu->op != B200_OP_GLU || glu->op_params[0] != B200_GLU_SWIGLU || !glu->src[1] || !glu->on_device ||
        glu->ne[2] != 1 || glu->ne[3] != 1 || !ggml_backend_b200_supports_op(glu))
        return false;
    if (mm->op != B200_OP_MUL_MAT || mm->src[1] != glu || !node_fusable(mm)) return false;
    const bool swapped = glu->op_params[1] != 0;
    *gate = swapped ? glu->src[1] : glu->src[0];
    *up = swapped ? glu->src[0] : glu->src[1];
    const int64_t F = glu->ne[0], M = glu->ne[1];
    if (mm->src[0]->ne[0] != F || F % 4 != 0 || F > 16384) return false;
    if (kernel_wtype(mm->src[0]->type) != T_F16 && M < min_m_quant() && M <= 32) return false;   // decode kernel
    for (const b200_tensor* t : {*gate, *up}) {
        if (t->ne[0] != F || t->ne[1] != M || t->nb[0] != 4 || t->nb[1] % 16 != 0) return false;
        if (t->on_device && (reinterpret_cast<uintptr_t>(t->data) & 15u)) return false;
    }
    for (int j = 0; j < n; j++) {
        if (j == i || j == i + 1) continue;
        for (int k = 0; k < B200_MAX_SRC; k++)
            if (nodes[j]->src[k] == glu) return false;
    }
    return true;
}

int do_swiglu_mul_mat(b200_backend* b, const b200_tensor* gate, const b200_tensor* up, const b200_tensor* mm) {
    const b200_tensor* a = mm->src[0];
    const int64_t F = a->ne[0], N = a->ne[1], M = gate->ne[1];
    int kt = 0;
    void* w = pack_weight(b, weight_key(a), a->type, a->data, a->on_device != 0, N, F, &kt);
    if (!w) return B200_E_CUDA;
    OpStaging stg;
    stg.ins = {gate, up};
    stg.outs = {mm};
    const size_t a16_bytes = ((size_t)M * F * 2 + 255) & ~(size_t)255;
    const size_t sc_bytes = ((size_t)M * 4 + 255) & ~(size_t)255;
    const size_t gws_need = (b200_gemm_packed_workspace_size(kt, M, N, F) + 255) & ~(size_t)255;
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    if (!grow(&b->ws, &b->ws_bytes, a16_bytes + sc_bytes + gws_need, b->stream)) return B200_E_CUDA;
    bool ok = true;
    const float* gd = static_cast<const float*>(stage_in(b, gate, &ok));
    const float* ud = static_cast<const float*>(stage_in(b, up, &ok));
    char* dd = stage_out(b, mm, false, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    char* ws = static_cast<char*>(b->ws);
    float* scales = reinterpret_cast<float*>(ws + a16_bytes);
    int rc = b200_swiglu_act_pack(gd, (int64_t)(gate->nb[1] / 4), ud, (int64_t)(up->nb[1] / 4), M, F, ws, scales,
                                  b->stream);
    if (rc != B200_OK) return rc;
    rc = b200_gemm_packed(kt, w, N, F, ws, scales, M, reinterpret_cast<float*>(dd), (int64_t)(mm->nb[1] / 4),
                          ws + a16_bytes + sc_bytes, b->ws_bytes - a16_bytes - sc_bytes, b->dev_err, b->stream);
    if (rc != B200_OK) return rc;
    if (!op_outputs_done(b, stg.outs, {dd})) return B200_E_CUDA;
    b->route_ops["glue"]++;
    b->route_ops[route_name(kt)]++;
    b->route_ops["swiglu_fused"]++;
    return B200_OK;
}

// ROPE (normal mode) whose only reader is a CPY of its result into an fp16 tensor -- llama.cpp's
// write of the rotated K rows into the KV-cache view -- with only view nodes in between: the pair
// runs as one b200_rope_f16 and the f32 rotated rows are never written. Device tensors only, with
// the layouts the fp16-output kernel takes; *cpy_idx: the CPY's node index.
static bool rope_cpy_match(b200_tensor* const* nodes, int n, int i, const std::vector<bool>& done, int* cpy_idx) {
    const b200_tensor* r = nodes[i];
    const b200_tensor* x = r->src[0];
    const b200_tensor* pos = r->src[1];
    if (r->op != B200_OP_ROPE || r->op_params[2] != 0 || !r->on_device || r->type != T_F32 || !x || !pos ||
        !x->on_device || !pos->on_device || !ggml_backend_b200_supports_op(r))
        return false;
    const int64_t half = x->ne[0] / 2;
    if (x->nb[0] != 4 || x->ne[0] % 2 || half <= 0 || (half & (half - 1)) || half * x->ne[1] > 2048 ||
        r->op_params[1] / 2 > 256 || x->nb[1] % 8 || x->nb[2] % 8 || x->nb[3] % 8 ||
        (reinterpret_cast<uintptr_t>(x->data) & 7u))
        return false;
    int j = -1;
    for (int k = 0; k < n; k++) {
        for (int q = 0; q < B200_MAX_SRC; q++) {
            if (nodes[k]->src[q] != r) continue;
            if (j >= 0 || k <= i || q != 0) return false;   // one reader, after the ROPE, as the CPY source
            j = k;
        }
    }
    if (j < 0 || done[j]) return false;
    const b200_tensor* c = nodes[j];
    if (c->op != B200_OP_CPY || c->type != T_F16 || !c->on_device || !ggml_backend_b200_supports_op(c)) return false;
    for (int d = 0; d < 4; d++)
        if (c->ne[d] != r->ne[d]) return false;
    if (c->nb[0] != 2 || c->nb[1] % 4 || c->nb[2] % 4 || c->nb[3] % 4 || (reinterpret_cast<uintptr_t>(c->data) & 3u))
        return false;
    for (int k = i + 1; k < j; k++) {
        const int op = nodes[k]->op;
        if (op != B200_OP_NONE && op != B200_OP_RESHAPE && op != B200_OP_VIEW && op != B200_OP_PERMUTE &&
            op != B200_OP_TRANSPOSE)
            return false;
    }
    *cpy_idx = j;
    return true;
}

int do_rope_cpy(b200_backend* b, const b200_tensor* r, const b200_tensor* c) {
    const b200_tensor* x = r->src[0];
    const b200_tensor* pos = r->src[1];
    OpStaging stg;
    stg.ins = {x, pos};
    stg.outs = {c};
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    bool ok = true;
    const float* sx = static_cast<const float*>(stage_in(b, x, &ok));
    const int32_t* sp = static_cast<const int32_t*>(stage_in(b, pos, &ok));
    char* d = stage_out(b, c, false, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    const int rc = b200_rope_f16(sx, x->ne, x->nb, sp, r->op_params[1], r->op_params[2], op_param_f32(r, 5),
                                 op_param_f32(r, 6), op_param_f32(r, 8), d, c->nb, b->stream);
    if (rc != B200_OK) return rc;
    if (!op_outputs_done(b, stg.outs, {d})) return B200_E_CUDA;
    b->route_ops["glue"] += 2;
    b->route_ops["rope_cpy"]++;
    return B200_OK;
}

int do_flash_attn(b200_backend* b, b200_tensor* op) {
    const b200_tensor* q = op->src[0];
    const b200_tensor* k = op->src[1];
    const b200_tensor* v = op->src[2];
    const b200_tensor* m = op->src[3];
    const int D = (int)q->ne[0], T = (int)q->ne[1], H = (int)q->ne[2];
    const int DV = (int)v->ne[0], KV = (int)k->ne[1], HK = (int)k->ne[2];
    const float scale = op_param_f32(op, 0), max_bias = op_param_f32(op, 1), softcap = op_param_f32(op, 2);
    OpStaging stg;
    stg.ins = {q, k, v, m};
    stg.outs = {op};
    const size_t need_ws = b200_flash_attn_workspace_size(D, DV, T, H, KV, HK);
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    if (!grow(&b->ws, &b->ws_bytes, need_ws, b->stream)) return B200_E_CUDA;
    bool ok = true;
    const void* qd = stage_in(b, q, &ok);
    const void* kd = stage_in(b, k, &ok);
    const void* vd = stage_in(b, v, &ok);
    const void* md = m ? stage_in(b, m, &ok) : nullptr;
    char* dd = stage_out(b, op, false, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    // a quantized cache: its fp16 tiles, contiguous [HK][KV][D], in a grow-only scratch buffer
    int64_t k_nb1 = (int64_t)k->nb[1], k_nb2 = (int64_t)k->nb[2], v_nb1 = (int64_t)v->nb[1], v_nb2 = (int64_t)v->nb[2];
    if (k->type != T_F16 || v->type != T_F16) {
        const size_t kb = k->type != T_F16 ? ((size_t)HK * KV * D * 2 + 255) & ~(size_t)255 : 0;
        const size_t vb = v->type != T_F16 ? (size_t)HK * KV * DV * 2 : 0;
        if (!grow(&b->kv16, &b->kv16_bytes, kb + vb, b->stream)) return B200_E_CUDA;
        char* base = static_cast<char*>(b->kv16);
        if (k->type != T_F16) {
            const int rc = b200_kv_to_f16(k->type, kd, D, KV, HK, k_nb1, k_nb2, base, b->stream);
            if (rc != B200_OK) return rc;
            kd = base, k_nb1 = (int64_t)D * 2, k_nb2 = (int64_t)KV * D * 2;
        }
        if (v->type != T_F16) {
            const int rc = b200_kv_to_f16(v->type, vd, DV, KV, HK, v_nb1, v_nb2, base + kb, b->stream);
            if (rc != B200_OK) return rc;
            vd = base + kb, v_nb1 = (int64_t)DV * 2, v_nb2 = (int64_t)KV * DV * 2;
        }
        b->route_ops["fa_quant_kv"]++;
    }
    int rc = b200_flash_attn_ext(static_cast<const float*>(qd), (int64_t)q->nb[1], (int64_t)q->nb[2], kd, k_nb1,
                                 k_nb2, vd, v_nb1, v_nb2, md,
                                 m ? (int64_t)m->nb[1] : 0, reinterpret_cast<float*>(dd), D, DV, T, H, KV, HK, scale,
                                 max_bias, softcap, b->ws, b->ws_bytes, b->dev_err, b->stream);
    if (rc != B200_OK) return rc;
    if (!op_outputs_done(b, stg.outs, {dd})) return B200_E_CUDA;
    b->route_ops["fa"]++;
    return B200_OK;
}

// One glue op (glue.cu). Host tensors are staged through the io arena (an output that is a
// strided host view is read in first, so the bytes between its elements survive the copy back);
// tensors in device buffers are used in place, with no host synchronisation.
int do_glue(b200_backend* b, const b200_tensor* op) {
    const b200_tensor* a = op->src[0];
    // ggml's CPY carries its destination as src[1]: that one is written, not read
    const b200_tensor* c = op->op == B200_OP_CPY ? nullptr : op->src[1];
    // a strided host output is read in first, so the bytes between its elements survive the copy
    // back; it is then both an input and an output of the op
    const bool read_in = !op->on_device && !is_contiguous(op);
    OpStaging stg;
    stg.ins = {a, c};
    if (read_in) stg.ins.push_back(op);
    stg.outs = {op};
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    bool ok = true;
    const char* sa = static_cast<const char*>(stage_in(b, a, &ok));
    const char* sc = c ? static_cast<const char*>(stage_in(b, c, &ok)) : nullptr;
    char* d = stage_out(b, op, read_in, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    float* df = reinterpret_cast<float*>(d);
    const cudaStream_t st = b->stream;
    int rc = B200_E_UNSUPPORTED;
    switch (op->op) {
        case B200_OP_RMS_NORM:
            rc = b200_rms_norm(reinterpret_cast<const float*>(sa), a->ne, a->nb, op_param_f32(op, 0), df, st);
            break;
        case B200_OP_ADD:
        case B200_OP_MUL:
        case B200_OP_DIV:
            rc = b200_binary(op->op == B200_OP_ADD ? B200_BIN_ADD : op->op == B200_OP_MUL ? B200_BIN_MUL : B200_BIN_DIV,
                             reinterpret_cast<const float*>(sa), a->ne, a->nb, reinterpret_cast<const float*>(sc), c->ne,
                             c->nb, df, st);
            break;
        case B200_OP_SOFT_MAX:
            rc = b200_soft_max(reinterpret_cast<const float*>(sa), a->ne, a->nb, op_param_f32(op, 0), df, st);
            break;
        case B200_OP_ARGSORT:
            rc = b200_argsort(reinterpret_cast<const float*>(sa), a->ne, a->nb, op->op_params[0],
                              reinterpret_cast<int32_t*>(d), st);
            break;
        case B200_OP_SUM_ROWS:
            rc = b200_sum_rows(reinterpret_cast<const float*>(sa), a->ne, a->nb, df, st);
            break;
        case B200_OP_UNARY:
            rc = b200_silu(reinterpret_cast<const float*>(sa), a->ne, a->nb, df, st);
            break;
        case B200_OP_GLU: {
            const bool swapped = op->op_params[1] != 0;
            const char* x = sa;
            const char* g = sc;
            const size_t* gnb = c ? c->nb : a->nb;
            if (!c) g = sa + (size_t)op->ne[0] * a->nb[0];   // one input: its two halves along ne[0]
            if (swapped) std::swap(x, g);
            const size_t* xnb = a->nb;
            if (c && swapped) std::swap(xnb, gnb);
            rc = b200_swiglu(reinterpret_cast<const float*>(x), xnb, reinterpret_cast<const float*>(g), gnb, op->ne,
                             df, st);
            break;
        }
        case B200_OP_ROPE:
            rc = b200_rope(reinterpret_cast<const float*>(sa), a->ne, a->nb, reinterpret_cast<const int32_t*>(sc),
                           op->op_params[1], op->op_params[2], op_param_f32(op, 5), op_param_f32(op, 6),
                           op_param_f32(op, 8), df, st);
            break;
        case B200_OP_GET_ROWS:
            rc = b200_get_rows(a->type == T_F16 ? 1 : 0, sa, a->ne, a->nb, reinterpret_cast<const int32_t*>(sc), c->ne,
                               c->nb, df, b->dev_err, st);
            break;
        case B200_OP_CPY:
            rc = b200_cpy(a->type == T_F16 ? 1 : 0, sa, a->ne, a->nb, op->type == T_F16 ? 1 : 0, d, op->ne, op->nb, st);
            break;
        default:
            break;
    }
    if (rc != B200_OK) return rc;
    if (!op_outputs_done(b, stg.outs, {d})) return B200_E_CUDA;
    b->route_ops["glue"]++;
    return B200_OK;
}

// A Hadamard-tagged MUL_MAT on the transform route: src0 is never read on the device, only its
// scale (hadamard_scale); dst = scale * H x per row of src1.
int do_hadamard(b200_backend* b, const b200_tensor* op) {
    const b200_tensor* x = op->src[1];
    float c = 0.0f;
    if (!hadamard_scale(op->src[0], &c)) return B200_E_UNSUPPORTED;
    OpStaging stg;
    stg.ins = {x};
    stg.outs = {op};
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    bool ok = true;
    const char* sx = static_cast<const char*>(stage_in(b, x, &ok));
    char* d = stage_out(b, op, false, &ok);
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    const int rc = b200_hadamard(reinterpret_cast<const float*>(sx), x->ne, x->nb, c, reinterpret_cast<float*>(d),
                                 b->stream);
    if (rc != B200_OK) return rc;
    if (!op_outputs_done(b, stg.outs, {d})) return B200_E_CUDA;
    b->route_ops["hadamard"]++;
    return B200_OK;
}

// The residual ADD `add` right before a fusable RMS_NORM * MUL pair, as one launch
// (b200_add_rms_norm_mul): both ADD operands dense f32 of the output's shape.
bool add_norm_fusable(const b200_tensor* add, const b200_tensor* nrm) {
    if (add->op != B200_OP_ADD || nrm->src[0] != add || add->type != T_F32 || !is_contiguous(add)) return false;
    for (int i = 0; i < 2; i++) {
        const b200_tensor* t = add->src[i];
        if (!t || t->type != T_F32 || !is_contiguous(t)) return false;
        for (int d = 0; d < 4; d++)
            if (t->ne[d] != add->ne[d]) return false;
    }
    return add->ne[0] % 4 == 0 && ggml_backend_b200_supports_op(add);
}

int do_add_rms_norm_mul(b200_backend* b, const b200_tensor* add, const b200_tensor* nrm, const b200_tensor* mul,
                        bool write_sum, bool write_norm) {
    const b200_tensor* x = add->src[0];
    const b200_tensor* r = add->src[1];
    const b200_tensor* w = mul->src[1];
    OpStaging stg;
    stg.ins = {x, r, w};
    stg.outs = {mul, add};
    if (write_norm) stg.outs.push_back(nrm);
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    bool ok = true;
    const char* sx = static_cast<const char*>(stage_in(b, x, &ok));
    const char* sr = static_cast<const char*>(stage_in(b, r, &ok));
    const char* sw = static_cast<const char*>(stage_in(b, w, &ok));
    char* dm = stage_out(b, mul, false, &ok);
    char* ds = stage_out(b, add, false, &ok);
    char* dn = write_norm ? stage_out(b, nrm, false, &ok) : nullptr;
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    int rc = b200_add_rms_norm_mul(reinterpret_cast<const float*>(sx), reinterpret_cast<const float*>(sr), add->ne,
                                   op_param_f32(nrm, 0), reinterpret_cast<const float*>(sw),
                                   reinterpret_cast<float*>(ds), reinterpret_cast<float*>(dn),
                                   reinterpret_cast<float*>(dm), b->stream);
    if (rc != B200_OK) return rc;
    std::vector<char*> bases{dm, ds};
    if (write_norm) bases.push_back(dn);
    if (!op_outputs_done(b, stg.outs, bases)) return B200_E_CUDA;
    (void)write_sum;
    b->route_ops["glue"] += 3;
    b->route_ops["add_norm_mul"]++;
    return B200_OK;
}

// RMS_NORM `nrm` and the MUL `mul` right after it that multiplies its rows by one weight row, as
// one launch (b200_rms_norm_mul). Fusable when the MUL reads the norm's output as src[0] and a
// dense f32 row of ne[0] as src[1], both claimed, with the norm's shape. The norm's own output is
// written only when something else may read it (a host tensor, or a later node's source).
bool norm_mul_fusable(const b200_tensor* nrm, const b200_tensor* mul) {
    if (nrm->op != B200_OP_RMS_NORM || mul->op != B200_OP_MUL || mul->src[0] != nrm) return false;
    const b200_tensor* w = mul->src[1];
    if (!w || w->type != T_F32 || !is_contiguous(w) || w->ne[0] != nrm->ne[0] || w->ne[1] != 1 || w->ne[2] != 1 ||
        w->ne[3] != 1)
        return false;
    for (int d = 0; d < 4; d++)
        if (mul->ne[d] != nrm->ne[d]) return false;
    return nrm->type == T_F32 && mul->type == T_F32 && is_contiguous(nrm) && is_contiguous(mul) &&
           ggml_backend_b200_supports_op(nrm) && ggml_backend_b200_supports_op(mul);
}

int do_rms_norm_mul(b200_backend* b, const b200_tensor* nrm, const b200_tensor* mul, bool write_norm) {
    const b200_tensor* x = nrm->src[0];
    const b200_tensor* w = mul->src[1];
    OpStaging stg;
    stg.ins = {x, w};
    stg.outs = {mul};
    if (write_norm) stg.outs.push_back(nrm);
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    bool ok = true;
    const char* sx = static_cast<const char*>(stage_in(b, x, &ok));
    const char* sw = static_cast<const char*>(stage_in(b, w, &ok));
    char* dm = stage_out(b, mul, false, &ok);
    char* dn = write_norm ? stage_out(b, nrm, false, &ok) : nullptr;
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    const int rc = b200_rms_norm_mul(reinterpret_cast<const float*>(sx), x->ne, x->nb, op_param_f32(nrm, 0),
                                     reinterpret_cast<const float*>(sw), reinterpret_cast<float*>(dn),
                                     reinterpret_cast<float*>(dm), b->stream);
    if (rc != B200_OK) return rc;
    std::vector<char*> bases{dm};
    if (write_norm) bases.push_back(dn);
    if (!op_outputs_done(b, stg.outs, bases)) return B200_E_CUDA;
    b->route_ops["glue"] += 2;
    b->route_ops["norm_mul"]++;
    return B200_OK;
}

// The MUL_MATs reading `t` (a fused norm's product) as src1, when they are all of t's readers, come
// after node i0 and run as one group on the GEMM path: t's f32 rows are then never written, the norm
// kernel packs them for the group instead (b200_rms_norm_mul_act_pack).
bool pack_readers(b200_tensor* const* nodes, int n, int i0, const std::vector<bool>& done, const b200_tensor* t,
                  std::vector<b200_tensor*>* grp, std::vector<int>* idx) {
    if (!t->on_device || t->type != T_F32 || !is_contiguous(t) || t->ne[2] != 1 || t->ne[3] != 1) return false;
    if (t->ne[0] % 4 != 0 || t->ne[0] > 16384) return false;
    grp->clear();
    idx->clear();
    for (int j = 0; j < n; j++) {
        for (int k = 0; k < B200_MAX_SRC; k++) {
            if (nodes[j]->src[k] != t) continue;
            if (j <= i0 || done[j] || k != 1 || nodes[j]->op != B200_OP_MUL_MAT || !node_fusable(nodes[j])) return false;
            if (idx->empty() || idx->back() != j) {
                grp->push_back(nodes[j]);
                idx->push_back(j);
            }
        }
    }
    if (grp->empty() || grp->size() > 8) return false;
    const int64_t M = t->ne[1];
    for (const b200_tensor* mm : *grp)
        if (kernel_wtype(mm->src[0]->type) != T_F16 && M < min_m_quant() && M <= 32) return false;   // decode kernel
    return true;
}

// The fused norm kernel reads and writes 16-byte vectors: device tensors must start on 16 bytes
// (host tensors are staged into 256-byte aligned device arenas).
bool vec_ready(std::initializer_list<const b200_tensor*> ts) {
    for (const b200_tensor* t : ts)
        if (t && t->on_device && (reinterpret_cast<uintptr_t>(t->data) & 15u)) return false;
    return true;
}

// [ADD ->] RMS_NORM -> MUL -> the MUL_MAT group reading the product: the norm (and the residual sum,
// always written) in one launch that also packs the product for the group, then the group's GEMMs.
int do_norm_pack_group(b200_backend* b, const b200_tensor* add, const b200_tensor* nrm, const b200_tensor* mul,
                       bool write_norm, b200_tensor* const* grp, int ng) {
    const b200_tensor* x = add ? add->src[0] : nrm->src[0];
    const b200_tensor* r = add ? add->src[1] : nullptr;
    const b200_tensor* w = mul->src[1];
    const int64_t K = mul->ne[0], M = mul->ne[1];
    const size_t a16_bytes = ((size_t)M * K * 2 + 255) & ~(size_t)255;
    const size_t sc_bytes = ((size_t)M * 4 + 255) & ~(size_t)255;
    if (!grow(&b->pre, &b->pre_bytes, a16_bytes + sc_bytes, b->stream)) return B200_E_CUDA;
    OpStaging stg;
    stg.ins = {x, w};
    if (r) stg.ins.push_back(r);
    if (add) stg.outs.push_back(add);
    if (write_norm) stg.outs.push_back(nrm);
    if (!op_reserve(b, stg)) return B200_E_CUDA;
    bool ok = true;
    const char* sx = static_cast<const char*>(stage_in(b, x, &ok));
    const char* sr = r ? static_cast<const char*>(stage_in(b, r, &ok)) : nullptr;
    const char* sw = static_cast<const char*>(stage_in(b, w, &ok));
    char* ds = add ? stage_out(b, add, false, &ok) : nullptr;
    char* dn = write_norm ? stage_out(b, nrm, false, &ok) : nullptr;
    if (!ok || !op_inputs_ready(b)) return B200_E_CUDA;
    float* scales = reinterpret_cast<float*>(static_cast<char*>(b->pre) + a16_bytes);
    int rc = b200_rms_norm_mul_act_pack(reinterpret_cast<const float*>(sx), reinterpret_cast<const float*>(sr), mul->ne,
                                        op_param_f32(nrm, 0), reinterpret_cast<const float*>(sw),
                                        reinterpret_cast<float*>(ds), reinterpret_cast<float*>(dn), nullptr, b->pre,
                                        scales, b->stream);
    if (rc != B200_OK) return rc;
    std::vector<char*> bases;
    if (add) bases.push_back(ds);
    if (write_norm) bases.push_back(dn);
    if (!op_outputs_done(b, stg.outs, bases)) return B200_E_CUDA;
    b->route_ops["glue"] += add ? 3 : 2;
    b->route_ops["norm_pack"]++;
    return do_mul_mat_group(b, grp, ng, b->pre, scales);
}

}  // namespace

// ================================================================================================
// public C API
// ================================================================================================

extern "C" {

const char* ggml_backend_b200_reg_name(void) { return "B200"; }

int ggml_backend_b200_reg_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int ggml_backend_b200_op_from_name(const char* name) {
    if (!name) return B200_OP_OTHER;
    static const struct { const char* n; int op; } map[] = {
        {"NONE", B200_OP_NONE},         {"RESHAPE", B200_OP_RESHAPE},       {"VIEW", B200_OP_VIEW},
        {"PERMUTE", B200_OP_PERMUTE},   {"TRANSPOSE", B200_OP_TRANSPOSE},   {"MUL_MAT", B200_OP_MUL_MAT},
        {"MUL_MAT_ID", B200_OP_MUL_MAT_ID}, {"FLASH_ATTN_EXT", B200_OP_FLASH_ATTN_EXT},
        {"RMS_NORM", B200_OP_RMS_NORM}, {"ADD", B200_OP_ADD},   {"MUL", B200_OP_MUL},
        {"UNARY", B200_OP_UNARY},       {"GLU", B200_OP_GLU},   {"ROPE", B200_OP_ROPE},
        {"GET_ROWS", B200_OP_GET_ROWS}, {"CPY", B200_OP_CPY},   {"SOFT_MAX", B200_OP_SOFT_MAX},
        {"ARGSORT", B200_OP_ARGSORT},   {"SUM_ROWS", B200_OP_SUM_ROWS}, {"DIV", B200_OP_DIV},
    };
    for (const auto& e : map)
        if (strcmp(name, e.n) == 0) return e.op;
    return B200_OP_OTHER;
}

int ggml_backend_b200_subop_from_name(const char* name) {
    if (!name) return -1;
    if (strcmp(name, "SILU") == 0) return B200_UNARY_SILU;
    if (strcmp(name, "SWIGLU") == 0) return B200_GLU_SWIGLU;
    return -1;
}

const char* ggml_backend_b200_device_name(int device) {
    static char names[16][16];
    if (device < 0 || device >= 16) return "B200";
    snprintf(names[device], sizeof names[device], "B200_%d", device);
    return names[device];
}

int ggml_backend_b200_device_description(int device, char* buf, size_t n) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return -1;
    snprintf(buf, n, "%s (sm_%d%d, %d SMs)", p.name, p.major, p.minor, p.multiProcessorCount);
    return 0;
}

int ggml_backend_b200_device_memory(int device, size_t* free_bytes, size_t* total_bytes) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return -1;
    if (cur != device && cudaSetDevice(device) != cudaSuccess) return -1;
    size_t f = 0, t = 0;
    const cudaError_t e = cudaMemGetInfo(&f, &t);
    if (cur != device) cudaSetDevice(cur);
    if (e != cudaSuccess) return -1;
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
    return 0;
}

b200_backend_t ggml_backend_b200_init(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) return nullptr;
    auto* b = new b200_backend();
    cudaGetDevice(&b->device);
    return b;
}

void ggml_backend_b200_free(b200_backend_t b) {
    if (!b) return;
    for (b200_buffer* buf : b->buffers) buf->owner = nullptr;   // they stay valid device memory
    if (b->dev_ready) {
        cudaSetDevice(b->device);
        cudaStreamSynchronize(b->stream);
        for (auto& kv : b->cache) cudaFree(kv.second.dev);
        io_drain(b);
        for (void* p : b->transient) cudaFree(p);
        cudaFree(b->ws);
        cudaFree(b->pre);
        cudaFree(b->kv16);
        cudaFree(b->io);
        cudaFree(b->wstage);
        if (b->pin) cudaFreeHost(b->pin);
        for (cudaEvent_t e : b->events) cudaEventDestroy(e);
        cudaFree(b->dev_err);
        cudaStreamDestroy(b->stream);
        cudaStreamDestroy(b->s_in);
        cudaStreamDestroy(b->s_out);
    }
    b->magic = 0;
    delete b;
}

bool ggml_backend_is_b200(const void* backend) {
    return backend && static_cast<const b200_backend*>(backend)->magic == 0xB2000B20u;
}

void ggml_backend_b200_set_n_gpus(b200_backend_t b, int n) {
    if (!b) return;
    int c = n < 1 ? 1 : (n > 8 ? 8 : n);
    if (c != n) logf("W", "set_n_gpus(%d) clamped to %d\n", n, c);
    b->n_gpus = c;
}

void ggml_backend_b200_moe_stats(b200_backend_t b, long* n_resident, long* n_streamed) {
    if (n_resident) *n_resident = b ? b->moe_resident : 0;
    if (n_streamed) *n_streamed = b ? b->moe_streamed : 0;
}

long ggml_backend_b200_route_ops(b200_backend_t b, const char* route) {
    if (!b) return 0;
    std::lock_guard<std::mutex> lk(b->mu);
    if (!route) {
        long t = 0;
        for (auto& kv : b->route_ops) t += kv.second;
        return t;
    }
    auto it = b->route_ops.find(route);
    return it == b->route_ops.end() ? 0 : it->second;
}

long ggml_backend_b200_cpu_fallbacks(b200_backend_t b) {
    (void)b;
    return 0;
}

long ggml_backend_b200_device_errors(b200_backend_t b) { return b ? b->device_errors : 0; }

size_t ggml_backend_b200_weight_cache_bytes(b200_backend_t b, long* n_entries) {
    if (!b) return 0;
    if (n_entries) *n_entries = (long)b->cache.size();
    return b->cache_bytes;
}

size_t ggml_backend_b200_weight_key(const b200_tensor* w, char* buf, size_t n) {
    if (!w) return 0;
    const std::string k = weight_key(w);
    if (buf && n) {
        const size_t c = std::min(n - 1, k.size());
        memcpy(buf, k.data(), c);
        buf[c] = 0;
    }
    return k.size();
}

void ggml_backend_b200_breaker_replay(const int* rcs, int n, int* attempted) {
    Breaker br;
    for (int i = 0; i < n; i++) {
        const bool go = breaker_allow(br);
        attempted[i] = go ? 1 : 0;
        if (go) breaker_note(br, rcs[i], "replay");
    }
}

int ggml_backend_b200_graph_compute(b200_backend_t b, b200_tensor* const* nodes, int n) {
    if (!b || (n > 0 && !nodes)) return B200_STATUS_FAILED;
    std::lock_guard<std::mutex> lk(b->mu);
    const auto t_enter = std::chrono::steady_clock::now();
    if (!ensure_device(b)) return B200_STATUS_FAILED;
    cudaSetDevice(b->device);
    // B200_GRAPH_TIMING=1: report per graph the host's time to queue the work, the device span from
    // the first queued operation to the last, and the whole call (a diagnostic; off by default)
    static const bool timing = knob_on("B200_GRAPH_TIMING", false);
    cudaEvent_t tev[2] = {nullptr, nullptr};
    if (timing) {
        cudaEventCreate(&tev[0]);
        cudaEventCreate(&tev[1]);
        cudaEventRecord(tev[0], b->stream);
    }
    const bool fuse = fuse_on();
    std::vector<bool> done(n, false);
    int status = B200_STATUS_SUCCESS;
    for (int i = 0; i < n && status == B200_STATUS_SUCCESS; i++) {
        b200_tensor* node = nodes[i];
        if (done[i]) continue;
        switch (node->op) {
            case B200_OP_MUL_MAT: {
                if (!ggml_backend_b200_supports_op(node)) {
                    logf("E", "graph_compute: MUL_MAT %s was not claimed\n", node->name);
                    status = B200_STATUS_FAILED;
                    break;
                }
                if (is_hadamard_op(node)) {
                    const int rc = do_hadamard(b, node);
                    if (rc != B200_OK) {
                        logf("E", "graph_compute: Hadamard MUL_MAT %s failed (%d)\n", node->name, rc);
                        status = B200_STATUS_FAILED;
                    }
                    break;
                }
                std::vector<b200_tensor*> group{node};
                std::vector<int> gidx{i};
                if (fuse && node_fusable(node) && breaker_allow(b->brk_fused)) {
                    for (int j = i + 1; j < n && group.size() < 8; j++) {
                        b200_tensor* nj = nodes[j];
                        if (!done[j] && nj->op == B200_OP_MUL_MAT && nj->src[1] == node->src[1] && node_fusable(nj)) {
                            group.push_back(nj);
                            gidx.push_back(j);
                        }
                    }
                }
                int rc = do_mul_mat_group(b, group.data(), (int)group.size());
                if (group.size() > 1) breaker_note(b->brk_fused, rc, "fused MUL_MAT group");
                if (rc != B200_OK && group.size() > 1) {
                    // the fused group's optional route failed: run the members one by one
                    rc = B200_OK;
                    for (size_t g = 0; g < group.size() && rc == B200_OK; g++) rc = do_mul_mat_group(b, &group[g], 1);
                }
                if (rc != B200_OK) {
                    logf("E", "graph_compute: MUL_MAT %s failed (%d)\n", node->name, rc);
                    status = B200_STATUS_FAILED;
                }
                for (int g : gidx) done[g] = true;
                break;
            }
            case B200_OP_MUL_MAT_ID: {
                if (!ggml_backend_b200_supports_op(node)) {
                    status = B200_STATUS_FAILED;
                    break;
                }
                const b200_tensor* ffn_gate = nullptr;
                const b200_tensor* ffn_up = nullptr;
                if (fuse && breaker_allow(b->brk_fused) && moe_ffn_match(nodes, n, i, done, &ffn_gate, &ffn_up)) {
                    // gate, up, SWIGLU and down in one pass over one route
                    const int rc = do_moe_ffn(b, ffn_gate, ffn_up, nodes[i + 3]);
                    breaker_note(b->brk_fused, rc, "fused MoE FFN");
                    if (rc == B200_OK || rc == B200_E_BAD_IDS) {
                        if (rc != B200_OK) {
                            logf("E", "graph_compute: MUL_MAT_ID handler failed (%d)\n", rc);
                            status = B200_STATUS_FAILED;
                        }
                        done[i] = done[i + 1] = done[i + 2] = done[i + 3] = true;
                        break;
                    }
                    // otherwise the four nodes run one by one below
                }
                std::vector<b200_tensor*> group{node};
                std::vector<int> gidx{i};
                if (fuse && breaker_allow(b->brk_fused)) {
                    for (int j = i + 1; j < n && group.size() < 4; j++) {
                        if (!done[j] && mmid_groupable(node, nodes[j])) {
                            group.push_back(nodes[j]);
                            gidx.push_back(j);
                        }
                    }
                }
                int rc = do_mul_mat_id_group(b, group.data(), (int)group.size());
                if (group.size() > 1) breaker_note(b->brk_fused, rc, "grouped MUL_MAT_ID");
                if (rc != B200_OK && rc != B200_E_BAD_IDS && group.size() > 1) {
                    // the group's optional route failed: run the members one by one
                    rc = B200_OK;
                    for (size_t g = 0; g < group.size() && rc == B200_OK; g++) rc = do_mul_mat_id(b, group[g]);
                }
                if (rc != B200_OK) {
                    logf("E", "graph_compute: MUL_MAT_ID handler failed (%d)\n", rc);
                    status = B200_STATUS_FAILED;
                }
                for (int g : gidx) done[g] = true;
                break;
            }
            case B200_OP_FLASH_ATTN_EXT: {
                if (!ggml_backend_b200_supports_op(node)) {
                    status = B200_STATUS_FAILED;
                    break;
                }
                const int rc = do_flash_attn(b, node);
                if (rc != B200_OK) {
                    logf("E", "graph_compute: FLASH_ATTN_EXT handler failed (%d)\n", rc);
                    status = B200_STATUS_FAILED;
                }
                break;
            }
            case B200_OP_RMS_NORM:
            case B200_OP_ADD:
            case B200_OP_MUL:
            case B200_OP_UNARY:
            case B200_OP_GLU:
            case B200_OP_ROPE:
            case B200_OP_GET_ROWS:
            case B200_OP_CPY:
            case B200_OP_SOFT_MAX:
            case B200_OP_ARGSORT:
            case B200_OP_SUM_ROWS:
            case B200_OP_DIV: {
                if (!ggml_backend_b200_supports_op(node)) {
                    status = B200_STATUS_FAILED;
                    break;
                }
                // ROPE -> the CPY of its result into an fp16 KV-cache view: one pass
                int cpy_j = -1;
                if (fuse && breaker_allow(b->brk_fused) && rope_cpy_match(nodes, n, i, done, &cpy_j)) {
                    const int rc = do_rope_cpy(b, node, nodes[cpy_j]);
                    breaker_note(b->brk_fused, rc, "fused ROPE + CPY");
                    if (rc != B200_OK) {
                        logf("E", "graph_compute: fused ROPE + CPY failed (%d) in node %s\n", rc, node->name);
                        status = B200_STATUS_FAILED;
                    }
                    done[cpy_j] = true;
                    break;
                }
                // GLU SWIGLU -> the down MUL_MAT reading it: the SWIGLU inside the down projection's
                // activation pack, h never written
                const b200_tensor* sw_gate = nullptr;
                const b200_tensor* sw_up = nullptr;
                if (fuse && breaker_allow(b->brk_fused) && swiglu_mm_match(nodes, n, i, done, &sw_gate, &sw_up)) {
                    const int rc = do_swiglu_mul_mat(b, sw_gate, sw_up, nodes[i + 1]);
                    breaker_note(b->brk_fused, rc, "fused SWIGLU + MUL_MAT");
                    if (rc != B200_OK) {
                        logf("E", "graph_compute: fused SWIGLU + MUL_MAT failed (%d) in node %s\n", rc, node->name);
                        status = B200_STATUS_FAILED;
                    }
                    done[i + 1] = true;
                    break;
                }
                // ADD (residual) -> RMS_NORM -> MUL (weight row): one launch; the sum is always
                // written (it is the next residual), the norm's rows only when read later
                if (fuse && i + 2 < n && !done[i + 1] && !done[i + 2] && add_norm_fusable(node, nodes[i + 1]) &&
                    norm_mul_fusable(nodes[i + 1], nodes[i + 2])) {
                    const b200_tensor* nrm = nodes[i + 1];
                    bool write_norm = !nrm->on_device;
                    for (int j = i + 3; j < n && !write_norm; j++)
                        for (int k = 0; k < B200_MAX_SRC && !write_norm; k++) write_norm = nodes[j]->src[k] == nrm;
                    std::vector<b200_tensor*> pg;
                    std::vector<int> pidx;
                    if (breaker_allow(b->brk_fused) &&
                        vec_ready({node->src[0], node->src[1], node, nodes[i + 2]->src[1], write_norm ? nrm : nullptr}) &&
                        pack_readers(nodes, n, i + 2, done, nodes[i + 2], &pg, &pidx)) {
                        // ... and the activation pack of the MUL_MATs reading the product
                        const int rc = do_norm_pack_group(b, node, nrm, nodes[i + 2], write_norm, pg.data(), (int)pg.size());
                        breaker_note(b->brk_fused, rc, "fused norm + MUL_MAT pack");
                        if (rc != B200_OK) {
                            logf("E", "graph_compute: fused ADD+RMS_NORM*MUL+pack failed (%d) in node %s\n", rc, node->name);
                            status = B200_STATUS_FAILED;
                        }
                        done[i + 1] = done[i + 2] = true;
                        for (int j : pidx) done[j] = true;
                        break;
                    }
                    const int rc = do_add_rms_norm_mul(b, node, nrm, nodes[i + 2], true, write_norm);
                    if (rc != B200_OK) {
                        logf("E", "graph_compute: fused ADD+RMS_NORM*MUL failed (%d) in node %s\n", rc, node->name);
                        status = B200_STATUS_FAILED;
                    }
                    done[i + 1] = done[i + 2] = true;
                    break;
                }
                if (fuse && i + 1 < n && !done[i + 1] && norm_mul_fusable(node, nodes[i + 1])) {
                    bool write_norm = !node->on_device;
                    for (int j = i + 2; j < n && !write_norm; j++)
                        for (int k = 0; k < B200_MAX_SRC && !write_norm; k++) write_norm = nodes[j]->src[k] == node;
                    std::vector<b200_tensor*> pg;
                    std::vector<int> pidx;
                    const b200_tensor* x0 = node->src[0];
                    if (breaker_allow(b->brk_fused) && x0 && x0->type == T_F32 && is_contiguous(x0) &&
                        vec_ready({x0, nodes[i + 1]->src[1], write_norm ? node : nullptr}) &&
                        pack_readers(nodes, n, i + 1, done, nodes[i + 1], &pg, &pidx)) {
                        const int rc = do_norm_pack_group(b, nullptr, node, nodes[i + 1], write_norm, pg.data(),
                                                          (int)pg.size());
                        breaker_note(b->brk_fused, rc, "fused norm + MUL_MAT pack");
                        if (rc != B200_OK) {
                            logf("E", "graph_compute: fused RMS_NORM*MUL+pack failed (%d) in node %s\n", rc, node->name);
                            status = B200_STATUS_FAILED;
                        }
                        done[i + 1] = true;
                        for (int j : pidx) done[j] = true;
                        break;
                    }
                    const int rc = do_rms_norm_mul(b, node, nodes[i + 1], write_norm);
                    if (rc != B200_OK) {
                        logf("E", "graph_compute: fused RMS_NORM*MUL failed (%d) in node %s\n", rc, node->name);
                        status = B200_STATUS_FAILED;
                    }
                    done[i + 1] = true;
                    break;
                }
                const int rc = do_glue(b, node);
                if (rc != B200_OK) {
                    logf("E", "graph_compute: glue op handler failed (%d) in node %s\n", rc, node->name);
                    status = B200_STATUS_FAILED;
                }
                break;
            }
            case B200_OP_NONE:
            case B200_OP_RESHAPE:
            case B200_OP_VIEW:
            case B200_OP_PERMUTE:
            case B200_OP_TRANSPOSE:
                break;
            default:
                logf("E", "graph_compute: unsupported op in node %s\n", node->name);
                status = B200_STATUS_FAILED;
        }
    }
    const auto t_queued = std::chrono::steady_clock::now();
    if (timing) cudaEventRecord(tev[1], b->stream);
    if (!graph_finish(b)) status = B200_STATUS_FAILED;
    for (void* p : b->transient) cudaFree(p);
    b->transient.clear();
    if (timing) {
        float dev_ms = 0.0f;
        cudaEventSynchronize(tev[1]);
        cudaEventElapsedTime(&dev_ms, tev[0], tev[1]);
        const auto t_exit = std::chrono::steady_clock::now();
        using us = std::chrono::duration<double, std::micro>;
        fprintf(stderr, "B200_GRAPH_TIMING nodes %d queue_us %.1f device_us %.1f call_us %.1f\n", n,
                us(t_queued - t_enter).count(), 1000.0 * dev_ms, us(t_exit - t_enter).count());
        cudaEventDestroy(tev[0]);
        cudaEventDestroy(tev[1]);
    }
    return status;
}


// ---- device buffers, async transfers and events -------------------------------------------------

static bool buf_ok(const b200_buffer* buf) { return buf && buf->magic == 0xB200BF00u && buf->base; }
static bool range_ok(const b200_buffer* buf, size_t offset, size_t size) {
    return offset <= buf->size && size <= buf->size - offset;
}
// The stream a buffer's synchronous calls are ordered on: its backend's (0 once that is freed).
static cudaStream_t buf_stream(const b200_buffer* buf) {
    return buf->owner && buf->owner->dev_ready ? buf->owner->stream : nullptr;
}
static void buf_invalidate(b200_buffer* buf, size_t offset, size_t size) {
    if (!buf->owner) return;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(buf->base) + offset;
    invalidate_range(buf->owner, lo, lo + size);
}

const char* ggml_backend_b200_buffer_type_name(void) { return "B200"; }
size_t ggml_backend_b200_buffer_type_alignment(void) { return 256; }
size_t ggml_backend_b200_buffer_type_max_size(int device) {
    size_t fr = 0, total = 0;
    if (ggml_backend_b200_device_memory(device, &fr, &total) != 0) return 0;
    return total;
}
size_t ggml_backend_b200_buffer_type_alloc_size(const b200_tensor* t) { return t ? nbytes(t) : 0; }
bool ggml_backend_b200_buffer_type_is_host(void) { return false; }

b200_buffer_t ggml_backend_b200_buffer_alloc(b200_backend_t b, size_t size) {
    if (!ggml_backend_is_b200(b) || size == 0) return nullptr;
    std::lock_guard<std::mutex> lk(b->mu);
    if (!ensure_device(b)) return nullptr;
    void* p = nullptr;
    if (!cuda_ok(cudaMalloc(&p, size), "cudaMalloc(buffer)")) return nullptr;
    auto* buf = new b200_buffer();
    buf->owner = b;
    buf->device = b->device;
    buf->base = p;
    buf->size = size;
    b->buffers.insert(buf);
    return buf;
}

void ggml_backend_b200_buffer_free(b200_buffer_t buf) {
    if (!buf_ok(buf)) return;
    cudaSetDevice(buf->device);
    if (buf->owner) {
        std::lock_guard<std::mutex> lk(buf->owner->mu);
        buf_invalidate(buf, 0, buf->size);
        if (buf->owner->dev_ready) cudaStreamSynchronize(buf->owner->stream);
        buf->owner->buffers.erase(buf);
    }
    cudaFree(buf->base);
    buf->magic = 0;
    buf->base = nullptr;
    delete buf;
}

void* ggml_backend_b200_buffer_base(b200_buffer_t buf) { return buf_ok(buf) ? buf->base : nullptr; }
size_t ggml_backend_b200_buffer_size(b200_buffer_t buf) { return buf_ok(buf) ? buf->size : 0; }

// One synchronous transfer into / out of / within buffers, ordered after the owner's queued work.
static int buf_sync_op(b200_buffer* lock_buf, b200_buffer* inval_buf, size_t inval_off, size_t inval_size,
                       const std::function<cudaError_t(cudaStream_t)>& op) {
    cudaSetDevice(lock_buf->device);
    std::unique_lock<std::mutex> lk;
    if (lock_buf->owner) lk = std::unique_lock<std::mutex>(lock_buf->owner->mu);
    if (inval_buf) buf_invalidate(inval_buf, inval_off, inval_size);
    const cudaStream_t st = buf_stream(lock_buf);
    if (op(st) != cudaSuccess) return B200_STATUS_FAILED;
    return cudaStreamSynchronize(st) == cudaSuccess ? B200_STATUS_SUCCESS : B200_STATUS_FAILED;
}

int ggml_backend_b200_buffer_set(b200_buffer_t buf, size_t offset, const void* src, size_t size) {
    if (!buf_ok(buf) || !range_ok(buf, offset, size) || (!src && size)) return B200_STATUS_FAILED;
    if (size == 0) return B200_STATUS_SUCCESS;
    return buf_sync_op(buf, buf, offset, size, [&](cudaStream_t st) {
        return cudaMemcpyAsync(static_cast<char*>(buf->base) + offset, src, size, cudaMemcpyHostToDevice, st);
    });
}

int ggml_backend_b200_buffer_get(b200_buffer_t buf, size_t offset, void* dst, size_t size) {
    if (!buf_ok(buf) || !range_ok(buf, offset, size) || (!dst && size)) return B200_STATUS_FAILED;
    if (size == 0) return B200_STATUS_SUCCESS;
    return buf_sync_op(buf, nullptr, 0, 0, [&](cudaStream_t st) {
        return cudaMemcpyAsync(dst, static_cast<const char*>(buf->base) + offset, size, cudaMemcpyDeviceToHost, st);
    });
}

int ggml_backend_b200_buffer_memset(b200_buffer_t buf, size_t offset, uint8_t value, size_t size) {
    if (!buf_ok(buf) || !range_ok(buf, offset, size)) return B200_STATUS_FAILED;
    if (size == 0) return B200_STATUS_SUCCESS;
    return buf_sync_op(buf, buf, offset, size, [&](cudaStream_t st) {
        return cudaMemsetAsync(static_cast<char*>(buf->base) + offset, value, size, st);
    });
}

int ggml_backend_b200_buffer_clear(b200_buffer_t buf, uint8_t value) {
    if (!buf_ok(buf)) return B200_STATUS_FAILED;
    return ggml_backend_b200_buffer_memset(buf, 0, value, buf->size);
}

int ggml_backend_b200_buffer_copy(b200_buffer_t src, size_t src_offset, b200_buffer_t dst, size_t dst_offset,
                                  size_t size) {
    if (!buf_ok(src) || !buf_ok(dst) || !range_ok(src, src_offset, size) || !range_ok(dst, dst_offset, size))
        return B200_STATUS_FAILED;
    if (src->owner != dst->owner && src->owner && dst->owner) return B200_STATUS_FAILED;   // one backend's buffers
    if (size == 0) return B200_STATUS_SUCCESS;
    return buf_sync_op(dst, dst, dst_offset, size, [&](cudaStream_t st) {
        return cudaMemcpyAsync(static_cast<char*>(dst->base) + dst_offset,
                               static_cast<const char*>(src->base) + src_offset, size, cudaMemcpyDeviceToDevice, st);
    });
}

void* ggml_backend_b200_host_alloc(size_t size) {
    if (size == 0) return nullptr;
    void* p = nullptr;
    return cudaMallocHost(&p, size) == cudaSuccess ? p : nullptr;
}
void ggml_backend_b200_host_free(void* ptr) {
    if (ptr) cudaFreeHost(ptr);
}

// The backend's own buffer, on its device, with the device state ready; locks its mutex.
static bool async_prologue(b200_backend_t b, const b200_buffer* buf, std::unique_lock<std::mutex>* lk) {
    if (!ggml_backend_is_b200(b)) return false;
    if (buf && (!buf_ok(buf) || buf->owner != b)) return false;
    *lk = std::unique_lock<std::mutex>(b->mu);
    if (!ensure_device(b)) return false;
    return cudaSetDevice(b->device) == cudaSuccess;
}

int ggml_backend_b200_set_async(b200_backend_t b, b200_buffer_t buf, size_t offset, const void* src, size_t size) {
    std::unique_lock<std::mutex> lk;
    if (!async_prologue(b, buf, &lk) || !buf || !range_ok(buf, offset, size) || (!src && size))
        return B200_STATUS_FAILED;
    if (size == 0) return B200_STATUS_SUCCESS;
    buf_invalidate(buf, offset, size);
    return cudaMemcpyAsync(static_cast<char*>(buf->base) + offset, src, size, cudaMemcpyHostToDevice, b->stream) ==
                   cudaSuccess
               ? B200_STATUS_SUCCESS
               : B200_STATUS_FAILED;
}

int ggml_backend_b200_get_async(b200_backend_t b, b200_buffer_t buf, size_t offset, void* dst, size_t size) {
    std::unique_lock<std::mutex> lk;
    if (!async_prologue(b, buf, &lk) || !buf || !range_ok(buf, offset, size) || (!dst && size))
        return B200_STATUS_FAILED;
    if (size == 0) return B200_STATUS_SUCCESS;
    return cudaMemcpyAsync(dst, static_cast<const char*>(buf->base) + offset, size, cudaMemcpyDeviceToHost,
                           b->stream) == cudaSuccess
               ? B200_STATUS_SUCCESS
               : B200_STATUS_FAILED;
}

int ggml_backend_b200_copy_async(b200_backend_t b, b200_buffer_t src, size_t src_offset, b200_buffer_t dst,
                                 size_t dst_offset, size_t size) {
    std::unique_lock<std::mutex> lk;
    if (!buf_ok(src) || src->owner != b || !async_prologue(b, dst, &lk) || !dst ||
        !range_ok(src, src_offset, size) || !range_ok(dst, dst_offset, size))
        return B200_STATUS_FAILED;
    if (size == 0) return B200_STATUS_SUCCESS;
    buf_invalidate(dst, dst_offset, size);
    return cudaMemcpyAsync(static_cast<char*>(dst->base) + dst_offset,
                           static_cast<const char*>(src->base) + src_offset, size, cudaMemcpyDeviceToDevice,
                           b->stream) == cudaSuccess
               ? B200_STATUS_SUCCESS
               : B200_STATUS_FAILED;
}

int ggml_backend_b200_synchronize(b200_backend_t b) {
    std::unique_lock<std::mutex> lk;
    if (!async_prologue(b, nullptr, &lk)) return B200_STATUS_FAILED;
    return cudaStreamSynchronize(b->stream) == cudaSuccess ? B200_STATUS_SUCCESS : B200_STATUS_FAILED;
}

b200_event_t ggml_backend_b200_event_new(b200_backend_t b) {
    std::unique_lock<std::mutex> lk;
    if (!async_prologue(b, nullptr, &lk)) return nullptr;
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    auto* ev = new b200_event();
    ev->device = b->device;
    ev->ev = e;
    return ev;
}

static bool ev_ok(const b200_event* ev) { return ev && ev->magic == 0xB200EE00u && ev->ev; }

void ggml_backend_b200_event_free(b200_event_t ev) {
    if (!ev_ok(ev)) return;
    cudaSetDevice(ev->device);
    cudaEventSynchronize(ev->ev);
    cudaEventDestroy(ev->ev);
    ev->magic = 0;
    delete ev;
}

int ggml_backend_b200_event_record(b200_backend_t b, b200_event_t ev) {
    std::unique_lock<std::mutex> lk;
    if (!ev_ok(ev) || !async_prologue(b, nullptr, &lk) || ev->device != b->device) return B200_STATUS_FAILED;
    return cudaEventRecord(ev->ev, b->stream) == cudaSuccess ? B200_STATUS_SUCCESS : B200_STATUS_FAILED;
}

int ggml_backend_b200_event_wait(b200_backend_t b, b200_event_t ev) {
    std::unique_lock<std::mutex> lk;
    if (!ev_ok(ev) || !async_prologue(b, nullptr, &lk)) return B200_STATUS_FAILED;
    return cudaStreamWaitEvent(b->stream, ev->ev, 0) == cudaSuccess ? B200_STATUS_SUCCESS : B200_STATUS_FAILED;
}

int ggml_backend_b200_event_synchronize(b200_event_t ev) {
    if (!ev_ok(ev)) return B200_STATUS_FAILED;
    cudaSetDevice(ev->device);
    return cudaEventSynchronize(ev->ev) == cudaSuccess ? B200_STATUS_SUCCESS : B200_STATUS_FAILED;
}

void ggml_backend_b200_device_caps(int device, bool* async, bool* host_buffer, bool* buffer_from_host_ptr,
                                   bool* events) {
    const bool present = device >= 0 && device < ggml_backend_b200_reg_device_count();
    if (async) *async = present;
    if (host_buffer) *host_buffer = present;
    if (buffer_from_host_ptr) *buffer_from_host_ptr = present;   // host tensors are staged per op
    if (events) *events = present;
}

}  // extern "C"
