// MUL_MAT for callers that cannot allocate device memory.
//
// Some hosts cannot call cudaMalloc on the path that runs an op: a plugin loaded into a
// process whose allocator owns the device and forbids side allocations, code running inside a
// region that must not change the device memory map, or a caller whose memory budget was fixed
// up front. b200_mul_mat needs a workspace (the fp16 activations, their row scales and, when
// CTAs share an output tile, their partial tiles); this entry point takes that workspace from a file-scope device
// array instead, so the caller passes only its inputs and outputs.
//
// The array is NOALLOC_SCRATCH_BYTES (32 MiB); every GPU that loads this library holds it until
// the process exits. Its first 256 bytes are this entry point's device error word (used when
// the caller passes no dev_err of its own); the rest is the workspace. Calls share the array and
// it keeps the last call's contents, so two calls that overlap on the GPU (different streams,
// or different host threads on the same device) race: the caller must order them. The only
// part of that carried-over content a call reads is the stream-K flag block (when CTAs share an
// output tile), so every call clears it on its stream before the GEMM runs: a finisher then
// never mistakes a flag left by an earlier call for this call's. The error word is not
// cleared per call: the first error since the last b200_mul_mat_noalloc_error stays there.
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = (size_t)32 << 20;
constexpr size_t NOALLOC_ERR_BYTES = 256;

__device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// The array's device address, per device. In host code the symbol is only a host-side stand-in,
// so the address is looked up once per device, with that device current.
std::mutex g_mu;
void* g_addr[64] = {nullptr};

int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B200_E_NO_DEVICE;
    if (dev < 0 || dev >= 64) return B200_E_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return B200_E_CUDA;
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return B200_OK;
}

}  // namespace

extern "C" {

size_t b200_mul_mat_noalloc_max_workspace(void) { return NOALLOC_SCRATCH_BYTES - NOALLOC_ERR_BYTES; }

int b200_mul_mat_noalloc(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda,
                         int64_t M, float* dst, int64_t ldd, int* dev_err, void* stream) {
    if (!w_packed || !src1 || !dst || M <= 0 || N <= 0 || K <= 0) return B200_E_INVALID;
    const size_t need = b200::mul_mat_workspace(wtype, M, N, K);
    if (need == 0) return B200_E_UNSUPPORTED;
    if (need > NOALLOC_SCRATCH_BYTES - NOALLOC_ERR_BYTES) return B200_E_TOO_LARGE;
    void* base = nullptr;
    const int rc = scratch_address(&base);
    if (rc != B200_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the error word lives in the array (zero at load, cleared by b200_mul_mat_noalloc_error)
    int* err = dev_err ? dev_err : static_cast<int*>(base);
    unsigned char* ws = static_cast<unsigned char*>(base) + NOALLOC_ERR_BYTES;
    size_t flags_off = 0, flags_bytes = 0;
    b200::mul_mat_flags_range(wtype, M, N, K, &flags_off, &flags_bytes);
    if (flags_bytes && cudaMemsetAsync(ws + flags_off, 0, flags_bytes, st) != cudaSuccess) return B200_E_CUDA;
    return b200::mul_mat_impl(wtype, w_packed, N, K, src1, lda, M, dst, ldd, ws, NOALLOC_SCRATCH_BYTES - NOALLOC_ERR_BYTES,
                              err, st);
}

int b200_mul_mat_noalloc_error(void* stream, int* host_err) {
    if (!host_err) return B200_E_INVALID;
    void* base = nullptr;
    const int rc = scratch_address(&base);
    if (rc != B200_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(host_err, base, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return B200_E_CUDA;
    if (cudaMemsetAsync(base, 0, sizeof(int), st) != cudaSuccess) return B200_E_CUDA;
    return B200_OK;
}

}  // extern "C"
