// Expert-parallel MUL_MAT_ID over NVLink peer memory: the exchange steps are the kernels' own
// stores into other GPUs' buffers, ordered by flags, with no collective library call and no
// host round trip on the data path.
//
// Every rank allocates the same "shared" buffers (cudaMalloc, exported with an IPC handle and
// mapped by every other rank once, at set-up):
//   recv_a16  [G][cap][K_max] fp16   rows pushed to this rank (as owner), one region per source
//   recv_meta [G][cap][n_used + 3]   per row {scale bits, slot mask, home token, ids...}
//   ret       [T_max][n_used][N_max] f32, this rank's (as home) outputs, dst's own layout
//   flags     [2][G][4] int32        {epoch, rows, pairs} from each source; done epoch per owner
// (the caller allocates them; b200_ep_shared_export / _open map them between processes)
// One op (epoch e, every rank in the same order, all on the caller's stream):
//   home   dispatch (moe_ep.cu kernels: rows per owner with slot masks, fp16 pack), then
//          ep_push_kernel stores each row straight into its owner's recv region for this rank
//          and ep_signal_kernel publishes {e, rows, pairs} in every owner's flags
//   owner  ep_wait_kernel waits for all sources' flags (bounded), the route / gather kernels
//          sort the received (row, slot) pairs by local expert, and the grouped tcgen05 GEMM's
//          epilogue stores every output row straight into its home rank's ret (NVLink stores,
//          no return exchange); ep_signal_kernel then publishes e in every home's done flags
//   home   ep_wait_kernel waits for every owner's done flag; ret holds dst.
// A rank reuses recv / ret only after the previous op's flags complete, so one set suffices.
#include <cstdint>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int P2P_THREADS = 256;

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Home: send row p (rows grouped by destination, counts[d] per destination) -> owner d's recv
// region for source `me`. Grid-stride over rows; one warp copies one row.
__global__ void __launch_bounds__(P2P_THREADS) ep_push_kernel(const __half* __restrict__ a16, const float* __restrict__ scale,
                                                              const int32_t* __restrict__ hdr,
                                                              const int32_t* __restrict__ row_tok,
                                                              const int32_t* __restrict__ counts, int G, int me,
                                                              int n_used, int K, int64_t cap,
                                                              __half* const* __restrict__ peer_a16,
                                                              int32_t* const* __restrict__ peer_meta) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    const int n = __ldg(counts + 2 * G);
    const int lane = threadIdx.x & 31;
    const int wpb = P2P_THREADS / 32;
    const int MW = n_used + 3;
    for (int p = blockIdx.x * wpb + (threadIdx.x >> 5); p < n; p += gridDim.x * wpb) {
        int d = 0, base = 0;
        while (d < G - 1 && p >= base + __ldg(counts + d)) base += __ldg(counts + d++);
        const int64_t slot = (int64_t)me * cap + (p - base);
        const uint4* src = reinterpret_cast<const uint4*>(a16 + (int64_t)p * K);
        uint4* dst = reinterpret_cast<uint4*>(peer_a16[d] + slot * K);
        for (int i = lane; i < K / 8; i += 32) dst[i] = __ldg(src + i);
        int32_t* meta = peer_meta[d] + slot * MW;
        const int32_t* h = hdr + (int64_t)p * (n_used + 1);
        for (int i = lane; i < MW; i += 32) {
            int32_t v;
            if (i == 0) v = __float_as_int(__ldg(scale + p));
            else if (i == 1) v = __ldg(h);                    // slot mask
            else if (i == 2) v = __ldg(row_tok + p);          // the home's token index
            else v = __ldg(h + i - 2);                        // ids
            meta[i] = v;
        }
    }
    __threadfence_system();
}

// Publish epoch e (and, with rows/pairs, this rank's counts per destination) in every peer's
// flag slot for this rank: flags[slot_base + me][0..3] on rank d.
__global__ void ep_signal_kernel(int* const* __restrict__ peer_flags, int slot_base, int me, int G, int epoch,
                                 const int32_t* __restrict__ counts) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __threadfence_system();
    const int d = threadIdx.x;
    if (d >= G) return;
    int* f = peer_flags[d] + 4 * (slot_base + me);
    if (counts) {
        f[1] = __ldg(counts + d);
        f[2] = __ldg(counts + G + d);
    }
    __threadfence_system();
    st_release_sys(f, epoch);
}

// Wait (bounded) until every rank's flag in this rank's slots [slot_base, slot_base + G) holds
// the epoch; copy their row counts and prefix into region (region[G] rows, region[G+1] pairs
// total; region[G+2..] row prefixes) when `region` is given.
__global__ void ep_wait_kernel(const int* __restrict__ flags, int slot_base, int G, int epoch, int32_t* __restrict__ region,
                               int* err, uint64_t limit_ns) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    const int s = threadIdx.x;
    bool ok = true;
    if (s < G) {
        const int* f = flags + 4 * (slot_base + s);
        const uint64_t t0 = globaltimer();
        while (ld_acquire_sys(f) != epoch) {
            __nanosleep(256);
            if (globaltimer() - t0 > limit_ns) {
                atomicCAS(err, 0, ERR_WAIT_PEER);
                ok = false;
                break;
            }
        }
    }
    __syncthreads();
    if (region && threadIdx.x == 0) {
        int rows = 0, pairs = 0;
        for (int k = 0; k < G; k++) {
            const int rk = ok ? flags[4 * (slot_base + k) + 1] : 0;
            region[G + 2 + k] = rows;
            region[k] = rk;
            rows += rk;
            pairs += ok ? flags[4 * (slot_base + k) + 2] : 0;
        }
        region[G] = rows;
        region[G + 1] = pairs;
    }
}

// Received row r (over the G source regions, concatenated) -> (source, index in its region).
__device__ __forceinline__ bool p2p_row(const int32_t* region, int G, int r, int& src, int& idx) {
    if (r >= __ldg(region + G)) return false;
    src = 0;
    while (src < G - 1 && r >= __ldg(region + G + 2 + src + 1)) src++;
    idx = r - __ldg(region + G + 2 + src);
    return true;
}

constexpr int P2PC = 256;   // rows per CTA of the route passes

__global__ void __launch_bounds__(P2PC) p2p_route_count_kernel(const int32_t* __restrict__ meta, const int32_t* __restrict__ region,
                                                               int G, int64_t cap, int n_used, int expert0, int e_loc,
                                                               int32_t* __restrict__ ecnt, int32_t* __restrict__ bsum,
                                                               int32_t* __restrict__ bad) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    extern __shared__ int hist[];
    __shared__ int sh[32];
    for (int e = threadIdx.x; e < e_loc; e += P2PC) hist[e] = 0;
    __syncthreads();
    const int MW = n_used + 3;
    const int r = blockIdx.x * P2PC + threadIdx.x;
    int src, idx, b = 0, pc = 0;
    if (p2p_row(region, G, r, src, idx)) {
        const int32_t* mrow = meta + ((int64_t)src * cap + idx) * MW;
        uint32_t m = (uint32_t)mrow[1];
        if (n_used < 32 && (m >> n_used)) b = 1;
        pc = __popc(m);
        while (m) {
            const int s = __ffs(m) - 1;
            m &= m - 1;
            const int x = mrow[3 + s] - expert0;
            if (x < 0 || x >= e_loc) b = 1;
            else atomicAdd(&hist[x], 1);
        }
    }
    int tot;
    block_excl_scan(pc, &tot, sh);
    b = __syncthreads_or(b);
    for (int e = threadIdx.x; e < e_loc; e += P2PC)
        if (hist[e]) atomicAdd(&ecnt[e], hist[e]);
    if (threadIdx.x == 0) {
        bsum[blockIdx.x] = tot;
        bad[blockIdx.x] = b;
    }
}

// Pairs of the received rows -> per-expert order (any order inside an expert), with the pair's
// home rank, home token and slot for the GEMM epilogue.
__global__ void __launch_bounds__(P2PC) p2p_route_place_kernel(const int32_t* __restrict__ meta, const int32_t* __restrict__ region,
                                                               int G, int64_t cap, int n_used, int expert0,
                                                               const int32_t* __restrict__ bad_any,
                                                               int32_t* __restrict__ cursor,
                                                               int32_t* __restrict__ pair_row,
                                                               int32_t* __restrict__ pair_src,
                                                               int32_t* __restrict__ pair_tok,
                                                               int32_t* __restrict__ pair_slot,
                                                               int32_t* __restrict__ pair_self) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    if (__ldg(bad_any)) return;
    const int MW = n_used + 3;
    const int r = blockIdx.x * P2PC + threadIdx.x;
    int src, idx;
    if (!p2p_row(region, G, r, src, idx)) return;
    const int32_t* mrow = meta + ((int64_t)src * cap + idx) * MW;
    uint32_t m = (uint32_t)mrow[1];
    const int tok = mrow[2];
    while (m) {
        const int s = __ffs(m) - 1;
        m &= m - 1;
        const int x = mrow[3 + s] - expert0;
        const int p = atomicAdd(&cursor[x], 1);
        pair_row[p] = (int)((int64_t)src * cap + idx);
        pair_src[p] = src;
        pair_tok[p] = tok;
        pair_slot[p] = s;
        if (pair_self) pair_self[p] = p;   // the expert FFN's own rows: output row p of a [pairs][N] buffer
    }
}

// Sorted pair p <- its received row (fp16 row, scale from the meta record); grid-stride.
__global__ void __launch_bounds__(256) p2p_gather_kernel(const __half* __restrict__ recv, const int32_t* __restrict__ meta,
                                                         const int32_t* __restrict__ pair_row,
                                                         const int32_t* __restrict__ n_pairs, int n_used, int K,
                                                         __half* __restrict__ dst, float* __restrict__ dst_scale) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    const int n = __ldg(n_pairs);
    const int MW = n_used + 3;
    for (int p = blockIdx.x; p < n; p += gridDim.x) {
        const int64_t rr = __ldg(pair_row + p);
        const uint4* s = reinterpret_cast<const uint4*>(recv + rr * K);
        uint4* d = reinterpret_cast<uint4*>(dst + (int64_t)p * K);
        for (int i = threadIdx.x; i < K / 8; i += 256) d[i] = __ldg(s + i);
        if (threadIdx.x == 0) dst_scale[p] = __int_as_float(__ldg(meta + rr * MW));
    }
}

struct P2pLayout {
    size_t region, ecnt, cursor, bsum, bad, off, tiles, prow, psrc, ptok, pslot, a16, scales, total;
};

static P2pLayout p2p_layout(int64_t G, int64_t cap, int64_t K, int64_t e_loc, int64_t n_used) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t rows = (size_t)(G * cap);
    const size_t P = rows;                          // every (token, slot) pair goes to one owner
    const size_t nb = (rows + P2PC - 1) / P2PC;
    (void)n_used;
    P2pLayout L{};
    L.region = 0;
    L.ecnt = al((size_t)(2 * G + 2) * 4);
    L.cursor = L.ecnt + al((size_t)e_loc * 4);
    L.bsum = L.cursor + al((size_t)e_loc * 4);
    L.bad = L.bsum + al(nb * 4);
    L.off = L.bad + al((nb + 1) * 4);
    L.tiles = L.off + al((size_t)(e_loc + 1) * 4);
    L.prow = L.tiles + al((size_t)(e_loc + 1) * 4);
    L.psrc = L.prow + al(P * 4);
    L.ptok = L.psrc + al(P * 4);
    L.pslot = L.ptok + al(P * 4);
    L.a16 = L.pslot + al(P * 4);
    L.scales = L.a16 + al(P * (size_t)K * 2);
    L.total = L.scales + al(P * 4);
    return L;
}

// The expert FFN's extra workspace after the MUL_MAT_ID owner's: pair_self, the gate and up
// outputs in pair order (f32 [P][F]) and the packed down-projection input (fp16 [P][F] + scales).
struct P2pFfnLayout {
    P2pLayout base;
    size_t self, gate, up, h16, hscale, total;
};

static P2pFfnLayout p2p_ffn_layout(int64_t G, int64_t cap, int64_t H, int64_t F, int64_t e_loc, int64_t n_used) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t P = (size_t)(G * cap);
    P2pFfnLayout L{};
    L.base = p2p_layout(G, cap, H, e_loc, n_used);
    L.self = L.base.total;
    L.gate = L.self + al(P * 4);
    L.up = L.gate + al(P * (size_t)F * 4);
    L.h16 = L.up + al(P * (size_t)F * 4);
    L.hscale = L.h16 + al(P * (size_t)F * 2);
    L.total = L.hscale + al(P * 4);
    return L;
}

// The owner's steps in front of its GEMMs, shared by the MUL_MAT_ID step and the expert FFN:
// wait for every source's rows, route the received (row, slot) pairs by local expert, gather
// the fp16 rows in expert order. Fills the route arrays of the layout (pair_self too when given)
// and returns the token tile the grouped GEMMs use.
struct P2pRoute {
    int32_t *off, *tiles, *psrc, *ptok, *pslot;
    __half* a16;
    float* scales;
    int bt;
};

static int p2p_owner_prologue(const P2pLayout& L, char* ws, int64_t K, int64_t n_local, int64_t expert0,
                              const void* recv_a16, const int32_t* recv_meta, const int* flags, int64_t n_ranks,
                              int64_t n_used, int64_t cap, int64_t pairs_hint, int32_t* pair_self, int epoch,
                              int* dev_err, cudaStream_t st, P2pRoute* R) {
    int32_t* region = reinterpret_cast<int32_t*>(ws + L.region);
    int32_t* ecnt = reinterpret_cast<int32_t*>(ws + L.ecnt);
    int32_t* cursor = reinterpret_cast<int32_t*>(ws + L.cursor);
    int32_t* bsum = reinterpret_cast<int32_t*>(ws + L.bsum);
    int32_t* bad = reinterpret_cast<int32_t*>(ws + L.bad);
    int32_t* prow = reinterpret_cast<int32_t*>(ws + L.prow);
    R->off = reinterpret_cast<int32_t*>(ws + L.off);
    R->tiles = reinterpret_cast<int32_t*>(ws + L.tiles);
    R->psrc = reinterpret_cast<int32_t*>(ws + L.psrc);
    R->ptok = reinterpret_cast<int32_t*>(ws + L.ptok);
    R->pslot = reinterpret_cast<int32_t*>(ws + L.pslot);
    R->a16 = reinterpret_cast<__half*>(ws + L.a16);
    R->scales = reinterpret_cast<float*>(ws + L.scales);
    const int G = (int)n_ranks;
    const int64_t rows_max = n_ranks * cap;
    const int nb = (int)((rows_max + P2PC - 1) / P2PC);
    R->bt = ep_token_tile_public(pairs_hint > 0 ? pairs_hint : rows_max / 2, n_local);
    // 1. every source's rows have landed (their flags carry the counts)
    launch_pdl(ep_wait_kernel, dim3(1), dim3(64), 0, st, flags, 0, G, epoch, region, dev_err, peer_wait_limit_ns());
    // 2. route the (row, slot) pairs by local expert
    const size_t hist_smem = (size_t)n_local * sizeof(int);
    if (hist_smem > 48 * 1024 &&
        cudaFuncSetAttribute(p2p_route_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_smem) !=
            cudaSuccess)
        return B200_E_UNSUPPORTED;
    if (cudaMemsetAsync(ecnt, 0, (size_t)n_local * 4, st) != cudaSuccess) return B200_E_CUDA;
    launch_pdl(p2p_route_count_kernel, dim3(nb), dim3(P2PC), hist_smem, st, recv_meta, region, G, cap, (int)n_used,
               (int)expert0, (int)n_local, ecnt, bsum, bad);
    ep_route_scan_public(ecnt, bsum, bad, nb, (int)n_local, R->bt, R->off, R->tiles, cursor, dev_err, st);
    launch_pdl(p2p_route_place_kernel, dim3(nb), dim3(P2PC), 0, st, recv_meta, region, G, cap, (int)n_used,
               (int)expert0, bad + nb, cursor, prow, R->psrc, R->ptok, R->pslot, pair_self);
    // 3. gather the fp16 rows in expert order (once for every GEMM that reads them)
    const int64_t gcap = (int64_t)device_sm_count() * 8;
    launch_pdl(p2p_gather_kernel, dim3((unsigned)(rows_max < gcap ? rows_max : gcap)), dim3(256), 0, st,
               static_cast<const __half*>(recv_a16), recv_meta, prow, R->off + n_local, (int)n_used, (int)K, R->a16,
               R->scales);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // namespace b200

extern "C" {

// Export a device buffer for the other ranks: the IPC handle of the allocation that holds it and
// the buffer's offset inside that allocation (allocators hand out pieces of larger blocks).
int b200_ep_shared_export(const void* ptr, void* handle, size_t* offset) {
    if (!ptr || !handle || !offset) return B200_E_INVALID;
    using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static GetRangeFn range = nullptr;
    if (!range) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return B200_E_CUDA;
        range = reinterpret_cast<GetRangeFn>(fn);
    }
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return B200_E_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return B200_E_CUDA;
    static_assert(sizeof(h) == B200_IPC_HANDLE_BYTES, "IPC handle size");
    __builtin_memcpy(handle, &h, sizeof(h));
    *offset = (size_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return B200_OK;
}

// Map another rank's exported allocation; *base is its start in this process (add the offset).
int b200_ep_shared_open(const void* handle, void** base) {
    if (!handle || !base) return B200_E_INVALID;
    cudaIpcMemHandle_t h;
    __builtin_memcpy(&h, handle, sizeof(h));
    return cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int b200_ep_shared_close(void* base) { return cudaIpcCloseMemHandle(base) == cudaSuccess ? B200_OK : B200_E_CUDA; }

int b200_moe_ep_p2p_push(const void* send_a16, const float* send_scale, const int32_t* send_hdr, const int32_t* row_tok,
                         const int32_t* counts, int64_t n_ranks, int64_t rank, int64_t n_used, int64_t K, int64_t cap,
                         void* const* peer_recv_a16, int32_t* const* peer_recv_meta, int* const* peer_flags,
                         int epoch, int64_t max_rows, void* stream) {
    using namespace b200;
    if (!send_a16 || !send_scale || !send_hdr || !row_tok || !counts || !peer_recv_a16 || !peer_recv_meta ||
        !peer_flags || n_ranks <= 0 || rank < 0 || rank >= n_ranks || n_used <= 0 || K <= 0 || cap <= 0)
        return B200_E_INVALID;
    if (K % 8 || n_ranks > 64) return B200_E_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t gcap = (int64_t)device_sm_count() * 4;
    const int64_t blocks = (max_rows + 7) / 8 < gcap ? (max_rows + 7) / 8 : gcap;
    if (blocks > 0)
        launch_pdl(ep_push_kernel, dim3((unsigned)blocks), dim3(P2P_THREADS), 0, st,
                   static_cast<const __half*>(send_a16), send_scale, send_hdr, row_tok, counts, (int)n_ranks,
                   (int)rank, (int)n_used, (int)K, cap, reinterpret_cast<__half* const*>(peer_recv_a16),
                   peer_recv_meta);
    launch_pdl(ep_signal_kernel, dim3(1), dim3(64), 0, st, peer_flags, 0, (int)rank, (int)n_ranks, epoch, counts);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

size_t b200_moe_ep_p2p_expert_workspace_size(int64_t n_ranks, int64_t cap, int64_t K, int64_t n_local, int64_t n_used) {
    if (n_ranks <= 0 || cap <= 0 || K <= 0 || n_local <= 0 || n_used <= 0) return 0;
    return b200::p2p_layout(n_ranks, cap, K, n_local, n_used).total;
}

int b200_moe_ep_p2p_expert_group(int n_members, int wtype, const void* const* local_stacks, const int64_t* Ns,
                                 int64_t K, int64_t n_local, int64_t expert0, const void* recv_a16,
                                 const int32_t* recv_meta, const int* flags, int64_t n_ranks, int64_t rank,
                                 int64_t n_used, int64_t cap, int64_t pairs_hint, float* const* const* peer_rets,
                                 const int64_t* ret_nb1, const int64_t* ret_nb2, int* const* peer_flags, int epoch,
                                 void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    using namespace b200;
    if (n_members <= 0 || !local_stacks || !Ns || !peer_rets || !ret_nb1 || !ret_nb2 || !recv_a16 || !recv_meta ||
        !flags || !peer_flags || !dev_err || K <= 0 || n_local <= 0 || expert0 < 0 || n_ranks <= 0 || rank < 0 ||
        rank >= n_ranks || n_used <= 0 || cap <= 0)
        return B200_E_INVALID;
    if (n_members > 16 || !weight_type_supported(wtype, K) || K % 32 != 0 || n_used > 32 || n_local > 4096 ||
        n_ranks > 64)
        return B200_E_UNSUPPORTED;
    for (int m = 0; m < n_members; m++) {
        if (!local_stacks[m] || !peer_rets[m] || Ns[m] <= 0) return B200_E_INVALID;
        if (Ns[m] % 16 != 0 || (ret_nb1[m] % 16) || (ret_nb2[m] % 16)) return B200_E_UNSUPPORTED;
    }
    const P2pLayout L = p2p_layout(n_ranks, cap, K, n_local, n_used);
    if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return B200_E_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int G = (int)n_ranks;
    const int64_t rows_max = n_ranks * cap;
    P2pRoute R;
    int rc = p2p_owner_prologue(L, static_cast<char*>(workspace), K, n_local, expert0, recv_a16, recv_meta, flags,
                                n_ranks, n_used, cap, pairs_hint, nullptr, epoch, dev_err, st, &R);
    if (rc != B200_OK) return rc;
    // 4. per member, the grouped GEMM stores each output row into its home rank's ret over NVLink
    for (int m = 0; m < n_members; m++) {
        rc = gemm_grouped_impl(wtype, local_stacks[m], Ns[m], K, n_local, R.a16, R.scales, rows_max, R.bt, R.off,
                               R.tiles, R.pslot, R.ptok, nullptr, ret_nb1[m], ret_nb2[m], dev_err, st, R.psrc,
                               peer_rets[m]);
        if (rc != B200_OK) return rc;
    }
    // 5. tell every home rank its rows are in place
    launch_pdl(ep_signal_kernel, dim3(1), dim3(64), 0, st, peer_flags, G, (int)rank, G, epoch, nullptr);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

size_t b200_moe_ep_p2p_ffn_workspace_size(int64_t n_ranks, int64_t cap, int64_t H, int64_t F, int64_t n_local,
                                          int64_t n_used) {
    if (n_ranks <= 0 || cap <= 0 || H <= 0 || F <= 0 || n_local <= 0 || n_used <= 0) return 0;
    return b200::p2p_ffn_layout(n_ranks, cap, H, F, n_local, n_used).total;
}

int b200_moe_ep_p2p_expert_ffn(int wtype_gate_up, const void* gate_stack, const void* up_stack, int wtype_down,
                               const void* down_stack, int64_t H, int64_t F, int64_t n_local, int64_t expert0,
                               const void* recv_a16, const int32_t* recv_meta, const int* flags, int64_t n_ranks,
                               int64_t rank, int64_t n_used, int64_t cap, int64_t pairs_hint, float* const* peer_ret,
                               int64_t ret_nb1, int64_t ret_nb2, int* const* peer_flags, int epoch, void* workspace,
                               size_t workspace_bytes, int* dev_err, void* stream) {
    using namespace b200;
    if (!gate_stack || !up_stack || !down_stack || !recv_a16 || !recv_meta || !flags || !peer_ret || !peer_flags ||
        !dev_err || H <= 0 || F <= 0 || n_local <= 0 || expert0 < 0 || n_ranks <= 0 || rank < 0 || rank >= n_ranks ||
        n_used <= 0 || cap <= 0)
        return B200_E_INVALID;
    if (!weight_type_supported(wtype_gate_up, H) || !weight_type_supported(wtype_down, F) || H % 32 || F % 32 ||
        H % 16 || F > 8192 || n_used > 32 || n_local > 4096 || n_ranks > 64 || (ret_nb1 % 16) || (ret_nb2 % 16))
        return B200_E_UNSUPPORTED;
    const P2pFfnLayout L = p2p_ffn_layout(n_ranks, cap, H, F, n_local, n_used);
    if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return B200_E_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    int32_t* self = reinterpret_cast<int32_t*>(ws + L.self);
    float* gate = reinterpret_cast<float*>(ws + L.gate);
    float* up = reinterpret_cast<float*>(ws + L.up);
    __half* h16 = reinterpret_cast<__half*>(ws + L.h16);
    float* hscale = reinterpret_cast<float*>(ws + L.hscale);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int G = (int)n_ranks;
    const int64_t rows_max = n_ranks * cap;
    // 1-3. wait, route, gather the pushed x rows (pair_self: each pair's own row index)
    P2pRoute R;
    int rc = p2p_owner_prologue(L.base, ws, H, n_local, expert0, recv_a16, recv_meta, flags, n_ranks, n_used, cap,
                                pairs_hint, self, epoch, dev_err, st, &R);
    if (rc != B200_OK) return rc;
    // 4. gate and up into this GPU's [pairs][F] buffers (row p = pair p: token and slot index both
    //    pair_self, slot stride 0)
    rc = gemm_grouped_impl(wtype_gate_up, gate_stack, F, H, n_local, R.a16, R.scales, rows_max, R.bt, R.off, R.tiles,
                           self, self, gate, 0, F * 4, dev_err, st);
    if (rc != B200_OK) return rc;
    rc = gemm_grouped_impl(wtype_gate_up, up_stack, F, H, n_local, R.a16, R.scales, rows_max, R.bt, R.off, R.tiles,
                           self, self, up, 0, F * 4, dev_err, st);
    if (rc != B200_OK) return rc;
    // 5. h = swiglu(gate, up), packed for the down projection in the same pair order
    rc = launch_swiglu_pack(gate, up, F, R.off + n_local, rows_max, h16, hscale, st);
    if (rc != B200_OK) return rc;
    // 6. down over the same route; the epilogue stores each row into its home rank's ret
    rc = gemm_grouped_impl(wtype_down, down_stack, H, F, n_local, h16, hscale, rows_max, R.bt, R.off, R.tiles, R.pslot,
                           R.ptok, nullptr, ret_nb1, ret_nb2, dev_err, st, R.psrc, peer_ret);
    if (rc != B200_OK) return rc;
    // 7. tell every home rank its rows are in place
    launch_pdl(ep_signal_kernel, dim3(1), dim3(64), 0, st, peer_flags, G, (int)rank, G, epoch, nullptr);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int b200_moe_ep_p2p_expert(int wtype, const void* local_stack, int64_t K, int64_t N, int64_t n_local, int64_t expert0,
                           const void* recv_a16, const int32_t* recv_meta, const int* flags, int64_t n_ranks,
                           int64_t rank, int64_t n_used, int64_t cap, int64_t pairs_hint, float* const* peer_ret,
                           int64_t ret_nb1, int64_t ret_nb2, int* const* peer_flags, int epoch, void* workspace,
                           size_t workspace_bytes, int* dev_err, void* stream) {
    return b200_moe_ep_p2p_expert_group(1, wtype, &local_stack, &N, K, n_local, expert0, recv_a16, recv_meta, flags,
                                        n_ranks, rank, n_used, cap, pairs_hint, &peer_ret, &ret_nb1, &ret_nb2,
                                        peer_flags, epoch, workspace, workspace_bytes, dev_err, stream);
}

int b200_moe_ep_p2p_finish(const int* flags, int64_t n_ranks, int epoch, int* dev_err, void* stream) {
    using namespace b200;
    if (!flags || !dev_err || n_ranks <= 0 || n_ranks > 64) return B200_E_INVALID;
    launch_pdl(ep_wait_kernel, dim3(1), dim3(64), 0, static_cast<cudaStream_t>(stream), flags, (int)n_ranks,
               (int)n_ranks, epoch, nullptr, dev_err, peer_wait_limit_ns());
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
