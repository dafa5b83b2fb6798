// Dense MUL_MAT with its weight rows split across GPUs (N-sharded), the all-gather of the output
// done by the GEMM's own epilogue stores over NVLink.
//
// Rank r of G holds the packed weight rows [col0, col0 + N_shard) of an N-row weight and the
// whole activation. Its tcgen05 GEMM (the plain MUL_MAT kernel, stream-K over this GPU's SMs)
// writes every finished 32 x 32 output box into the dst buffer of EVERY rank -- its own and the
// other ranks', mapped into this process by CUDA IPC -- at column col0. A signal kernel then
// publishes the op's epoch in each rank's flag slot for r; b200_mul_mat_tp_finish waits (bounded)
// until all G slots of this rank carry it, after which this rank's dst holds the full [M, N]. No
// collective library call, no host round trip, no separate gather pass: the transfer of a box
// overlaps the main loop of the next one.
//
// The per-element arithmetic is the single-GPU MUL_MAT's (the same activation pack, decode and
// fp32 accumulation); only the K split of a tile (the stream-K plan over N_shard rows) can
// differ from the single-GPU plan, which reorders the fp32 sums.
#include <atomic>
#include <cstdint>

#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

// How long a kernel waits for another GPU's flag before it gives up (records ERR_WAIT_PEER in the
// error word and returns): process-wide, set by b200_set_peer_wait_limit_ns, 2 s by default.
static std::atomic<uint64_t> g_peer_wait_ns{B200_WAIT_LIMIT_NS};
uint64_t peer_wait_limit_ns() { return g_peer_wait_ns.load(std::memory_order_relaxed); }

__device__ __forceinline__ int tp_ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void tp_st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Thread d: epoch into rank d's flag slot for this rank (flags are [G][4] int32 per rank).
__global__ void tp_signal_kernel(int* const* __restrict__ peer_flags, int me, int G, int epoch) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __threadfence_system();
    const int d = threadIdx.x;
    if (d >= G) return;
    tp_st_release_sys(peer_flags[d] + 4 * me, epoch);
}

// Thread s: wait (bounded) until rank s's slot of this rank's flags holds the epoch.
__global__ void tp_wait_kernel(const int* __restrict__ flags, int G, int epoch, int* err, uint64_t limit_ns) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    const int s = threadIdx.x;
    if (s >= G) return;
    const int* f = flags + 4 * s;
    const uint64_t t0 = globaltimer();
    while (tp_ld_acquire_sys(f) != epoch) {
        __nanosleep(256);
        if (globaltimer() - t0 > limit_ns) {
            atomicCAS(err, 0, ERR_WAIT_PEER);
            return;
        }
    }
}

}  // namespace b200

extern "C" {

void b200_set_peer_wait_limit_ns(uint64_t ns) { b200::g_peer_wait_ns.store(ns ? ns : B200_WAIT_LIMIT_NS); }
uint64_t b200_peer_wait_limit_ns(void) { return b200::peer_wait_limit_ns(); }

size_t b200_mul_mat_tp_workspace_size(int wtype, int64_t M, int64_t N_shard, int64_t K) {
    if (M <= 0 || N_shard <= 0 || K <= 0) return 0;
    return b200::mul_mat_workspace(wtype, M, N_shard, K);
}

int b200_mul_mat_tp(int wtype, const void* w_shard, int64_t N_shard, int64_t col0, int64_t K, const float* src1,
                    int64_t lda, int64_t M, float* const* peer_dst, int64_t ldd, int64_t n_ranks, int64_t rank,
                    int* const* peer_flags, int epoch, void* workspace, size_t workspace_bytes, int* dev_err,
                    void* stream) {
    using namespace b200;
    if (!w_shard || !src1 || !peer_dst || !peer_flags || !dev_err || N_shard <= 0 || col0 < 0 || K <= 0 || M <= 0 ||
        n_ranks <= 0 || rank < 0 || rank >= n_ranks || lda < K || ldd < col0 + N_shard)
        return B200_E_INVALID;
    if (n_ranks > 64 || col0 % 16 != 0 || ldd % 4 != 0) return B200_E_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int rc = mul_mat_impl(wtype, w_shard, N_shard, K, src1, lda, M, nullptr, ldd, workspace, workspace_bytes,
                                dev_err, st, peer_dst, (int)n_ranks, col0);
    if (rc != B200_OK) return rc;
    launch_pdl(tp_signal_kernel, dim3(1), dim3(64), 0, st, peer_flags, (int)rank, (int)n_ranks, epoch);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int b200_mul_mat_tp_finish(const int* flags, int64_t n_ranks, int epoch, int* dev_err, void* stream) {
    using namespace b200;
    if (!flags || !dev_err || n_ranks <= 0) return B200_E_INVALID;
    if (n_ranks > 64) return B200_E_UNSUPPORTED;
    launch_pdl(tp_wait_kernel, dim3(1), dim3(64), 0, static_cast<cudaStream_t>(stream), flags, (int)n_ranks, epoch,
               dev_err, peer_wait_limit_ns());
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
