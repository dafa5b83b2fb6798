// Expert-parallel MUL_MAT_ID: the rank-local kernels around the all-to-all exchanges.
//
// The experts of one MUL_MAT_ID are split across n_ranks GPUs in contiguous blocks of
// E / n_ranks; every rank holds its own tokens ("home" rank). One op runs as
//   dispatch  (home)    route every (token, b row) to the ranks owning its experts: ONE send
//                       row per (token, b row, destination rank), with a slot mask saying which
//                       of the token's slots it serves there, packed to fp16 with its row scale
//                       (the same pack as single-GPU MUL_MAT_ID, ggml-rocket.cpp:1451-1475)
//   exchange            the caller's all-to-all of rows, scales and headers (NCCL)
//   expert    (owner)   expand the received rows into (row, slot) pairs, sort them by local
//                       expert, run the grouped tcgen05 GEMM, and write each pair's output row
//                       to its place in the return buffer (received order, slots ascending)
//   exchange            the caller's all-to-all of the return rows (f32, bit-identical to the
//                       single-GPU result)
//   combine   (home)    scatter every returned row to dst[:, slot, token]
// The per-(token, slot) arithmetic is the single-GPU op's (ggml-rocket.cpp:6692-6944): the
// same fp16 pack of the same b row, the same weight decode, the same fp32 accumulation, so
// every dst row matches b200_mul_mat_id's for the same plan.
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int EP_THREADS = 1024;
constexpr int EP_MAX_RANKS = 64;
constexpr int EP_MAX_SLOTS = 32;   // slot masks are 32-bit

// Exclusive scan of one int over the CTA (EP_THREADS threads); also returns the total.
__device__ __forceinline__ int block_excl_scan(int v, int* total, int* sh /* [32] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = sh[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        sh[lane] = w;                                   // inclusive over warps
    }
    __syncthreads();
    const int before = (warp > 0 ? sh[warp - 1] : 0) + x - v;
    *total = sh[31];
    __syncthreads();                                    // sh is reused by the next call
    return before;
}

// Home side. Candidate c = t * ne11 + j is token t's b row j (serving slots s with s % ne11 == j).
// For destination rank d its slot mask is {s : s % ne11 == j, ids[s, t] / E_loc == d}. Send rows
// are ordered by destination, then token, then b row; their return rows by the same order with
// each row's slots ascending.
__global__ void __launch_bounds__(EP_THREADS) ep_dispatch_kernel(
    const int32_t* __restrict__ ids, int64_t ids_nb0, int64_t ids_nb1, int n_used, int n_tokens, int ne11, int E,
    int G, int32_t* __restrict__ hdr, int32_t* __restrict__ row_tok, int32_t* __restrict__ row_slot,
    int32_t* __restrict__ row_ret, int32_t* __restrict__ counts, int* err) {
    __shared__ int sh[32];
    const int e_loc = E / G;
    const int C = n_tokens * ne11;
    const int chunk = (C + EP_THREADS - 1) / EP_THREADS;
    const int c_beg = min(C, (int)threadIdx.x * chunk), c_end = min(C, c_beg + chunk);
    auto id_at = [&](int s, int t) {
        return __ldg(reinterpret_cast<const int32_t*>(reinterpret_cast<const char*>(ids) + (int64_t)t * ids_nb1 +
                                                      (int64_t)s * ids_nb0));
    };
    int bad = 0;
    for (int c = c_beg; c < c_end; c++) {
        const int t = c / ne11, j = c % ne11;
        for (int s = j; s < n_used; s += ne11) {
            const int x = id_at(s, t);
            if (x < 0 || x >= E) bad = 1;
        }
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) atomicCAS(err, 0, B200_DEV_BAD_IDS);
        for (int i = threadIdx.x; i < 2 * G + 2; i += EP_THREADS) counts[i] = 0;
        return;
    }
    auto mask_of = [&](int c, int d) {
        const int t = c / ne11, j = c % ne11;
        uint32_t m = 0;
        for (int s = j; s < n_used; s += ne11)
            if (id_at(s, t) / e_loc == d) m |= 1u << s;
        return m;
    };
    int row_base = 0, pair_base = 0;
    for (int d = 0; d < G; d++) {
        int nrow = 0, npair = 0;
        for (int c = c_beg; c < c_end; c++) {
            const uint32_t m = mask_of(c, d);
            if (m) { nrow++; npair += __popc(m); }
        }
        int tot_row, tot_pair;
        int p = row_base + block_excl_scan(nrow, &tot_row, sh);
        int q = pair_base + block_excl_scan(npair, &tot_pair, sh);
        for (int c = c_beg; c < c_end; c++) {
            const uint32_t m = mask_of(c, d);
            if (!m) continue;
            const int t = c / ne11;
            int32_t* h = hdr + (int64_t)p * (n_used + 1);
            h[0] = (int32_t)m;
            for (int s = 0; s < n_used; s++) h[1 + s] = id_at(s, t);
            row_tok[p] = t;
            row_slot[p] = __ffs(m) - 1;
            row_ret[p] = q;
            p++;
            q += __popc(m);
        }
        if (threadIdx.x == 0) {
            counts[d] = tot_row;
            counts[G + d] = tot_pair;
        }
        row_base += tot_row;
        pair_base += tot_pair;
    }
    if (threadIdx.x == 0) {
        counts[2 * G] = row_base;
        counts[2 * G + 1] = pair_base;
    }
}

// Owner side: the received rows' (row, slot) pairs, counted per local expert, placed per expert
// (any order inside an expert: a row's output does not depend on its neighbours in a tile), with
// the return index rowpref[r] + (rank of slot s among row r's slots). off/tile_start as in
// moe_route_kernel. Dynamic shared memory: cnt[E_loc], cur[E_loc] ints.
__global__ void __launch_bounds__(EP_THREADS) ep_expert_route_kernel(
    const int32_t* __restrict__ hdr, int n_rows, int n_used, int expert0, int e_loc, int bt,
    int32_t* __restrict__ off, int32_t* __restrict__ tile_start, int32_t* __restrict__ pair_src,
    int32_t* __restrict__ pair_ret, int32_t* __restrict__ pair_zero, int* err) {
    extern __shared__ int smx[];
    __shared__ int sh[32];
    int* cnt = smx;
    int* cur = smx + e_loc;
    for (int e = threadIdx.x; e < e_loc; e += EP_THREADS) cnt[e] = 0;
    __syncthreads();
    const int chunk = (n_rows + EP_THREADS - 1) / EP_THREADS;
    const int r_beg = min(n_rows, (int)threadIdx.x * chunk), r_end = min(n_rows, r_beg + chunk);
    int bad = 0, npair = 0;
    for (int r = r_beg; r < r_end; r++) {
        const int32_t* h = hdr + (int64_t)r * (n_used + 1);
        uint32_t m = (uint32_t)h[0];
        if (n_used < 32 && (m >> n_used)) bad = 1;
        npair += __popc(m);
        while (m) {
            const int s = __ffs(m) - 1;
            m &= m - 1;
            const int x = h[1 + s] - expert0;
            if (x < 0 || x >= e_loc) bad = 1;
            else atomicAdd(&cnt[x], 1);
        }
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) atomicCAS(err, 0, B200_DEV_BAD_IDS);
        for (int e = threadIdx.x; e <= e_loc; e += EP_THREADS) {
            off[e] = 0;
            tile_start[e] = 0;
        }
        return;
    }
    int total;
    int q = block_excl_scan(npair, &total, sh);
    if (threadIdx.x == 0) {
        int acc = 0, tacc = 0;
        for (int e = 0; e < e_loc; e++) {
            off[e] = acc;
            cur[e] = acc;
            tile_start[e] = tacc;
            acc += cnt[e];
            tacc += (cnt[e] + bt - 1) / bt;
        }
        off[e_loc] = acc;
        tile_start[e_loc] = tacc;
    }
    __syncthreads();
    for (int r = r_beg; r < r_end; r++) {
        const int32_t* h = hdr + (int64_t)r * (n_used + 1);
        uint32_t m = (uint32_t)h[0];
        while (m) {
            const int s = __ffs(m) - 1;
            m &= m - 1;
            const int x = h[1 + s] - expert0;
            const int p = atomicAdd(&cur[x], 1);
            pair_src[p] = r;
            pair_ret[p] = q++;
            pair_zero[p] = 0;
        }
    }
}

// Sorted pair p <- received row pair_src[p] (fp16 row and its scale).
__global__ void __launch_bounds__(256) ep_gather_rows_kernel(const __half* __restrict__ src, const float* __restrict__ src_scale,
                                                             const int32_t* __restrict__ pair_src,
                                                             const int32_t* __restrict__ n_pairs, int K,
                                                             __half* __restrict__ dst, float* __restrict__ dst_scale) {
    const int p = blockIdx.x;
    if (p >= __ldg(n_pairs)) return;
    const int r = __ldg(pair_src + p);
    const uint4* s = reinterpret_cast<const uint4*>(src + (int64_t)r * K);
    uint4* d = reinterpret_cast<uint4*>(dst + (int64_t)p * K);
    for (int i = threadIdx.x; i < K / 8; i += 256) d[i] = __ldg(s + i);
    if (threadIdx.x == 0) dst_scale[p] = __ldg(src_scale + r);
}

// Home side: send row p's returned rows (one per slot in its mask, ascending) -> dst[:, s, t].
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ ret, int N,
                                                         const int32_t* __restrict__ hdr, int n_used,
                                                         const int32_t* __restrict__ row_tok,
                                                         const int32_t* __restrict__ row_ret,
                                                         const int32_t* __restrict__ n_rows, float* __restrict__ dst,
                                                         int64_t d_nb1, int64_t d_nb2) {
    const int p = blockIdx.x;
    if (p >= __ldg(n_rows)) return;
    const int t = __ldg(row_tok + p);
    uint32_t m = (uint32_t)__ldg(hdr + (int64_t)p * (n_used + 1));
    int k = __ldg(row_ret + p);
    while (m) {
        const int s = __ffs(m) - 1;
        m &= m - 1;
        const float4* src = reinterpret_cast<const float4*>(ret + (int64_t)k * N);
        float4* out = reinterpret_cast<float4*>(reinterpret_cast<char*>(dst) + (int64_t)t * d_nb2 + (int64_t)s * d_nb1);
        for (int i = threadIdx.x; i < N / 4; i += 256) out[i] = __ldg(src + i);
        k++;
    }
}

struct EpExpertLayout {
    size_t off, tiles, src, ret, zero, a16, scales, total;
};

static EpExpertLayout ep_expert_layout(int64_t K, int64_t e_loc, int64_t n_used, int64_t n_rows) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t P = (size_t)(n_rows * n_used);
    EpExpertLayout L{};
    L.off = 0;
    L.tiles = al((size_t)(e_loc + 1) * 4);
    L.src = L.tiles + al((size_t)(e_loc + 1) * 4);
    L.ret = L.src + al(P * 4);
    L.zero = L.ret + al(P * 4);
    L.a16 = L.zero + al(P * 4);
    L.scales = L.a16 + al(P * (size_t)K * 2);
    L.total = L.scales + al(P * 4);
    return L;
}

static int ep_token_tile(int64_t pairs, int64_t e_loc) {
    const int64_t avg = e_loc > 0 ? pairs / e_loc : pairs;
    return avg <= 32 ? 32 : avg <= 64 ? 64 : 128;
}

}  // namespace b200

extern "C" {

int b200_moe_ep_dispatch(const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                         int64_t n_expert, int64_t n_ranks, const float* b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                         int64_t K, void* send_a16, float* send_scale, int32_t* send_hdr, int32_t* row_tok,
                         int32_t* row_slot, int32_t* row_ret, int32_t* counts, int* dev_err, void* stream) {
    using namespace b200;
    if (!ids || !b || !send_a16 || !send_scale || !send_hdr || !row_tok || !row_slot || !row_ret || !counts ||
        !dev_err || n_used <= 0 || n_tokens <= 0 || n_expert <= 0 || n_ranks <= 0 || ne11 <= 0 || K <= 0)
        return B200_E_INVALID;
    if (n_used > EP_MAX_SLOTS || n_ranks > EP_MAX_RANKS || n_expert % n_ranks != 0 || n_used % ne11 != 0 ||
        K % 8 != 0 || n_tokens * n_used > (1 << 28))
        return B200_E_UNSUPPORTED;
    if ((b_nb1 % 16) || (b_nb2 % 16) || (reinterpret_cast<uintptr_t>(b) & 15u) ||
        (reinterpret_cast<uintptr_t>(send_a16) & 15u))
        return B200_E_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ep_dispatch_kernel<<<1, EP_THREADS, 0, st>>>(ids, ids_nb0, ids_nb1, (int)n_used, (int)n_tokens, (int)ne11,
                                                 (int)n_expert, (int)n_ranks, send_hdr, row_tok, row_slot, row_ret,
                                                 counts, dev_err);
    if (cudaGetLastError() != cudaSuccess) return B200_E_CUDA;
    const int rc = launch_gather_pack(b, b_nb1, b_nb2, ne11, K, row_slot, row_tok, counts + 2 * n_ranks,
                                      n_tokens * n_used, static_cast<__half*>(send_a16), send_scale, st);
    return rc;
}

size_t b200_moe_ep_expert_workspace_size(int64_t K, int64_t n_local, int64_t n_used, int64_t n_rows) {
    if (K <= 0 || n_local <= 0 || n_used <= 0 || n_rows < 0) return 0;
    return b200::ep_expert_layout(K, n_local, n_used, n_rows > 0 ? n_rows : 1).total;
}

int b200_moe_ep_expert(int wtype, const void* local_stack, int64_t K, int64_t N, int64_t n_local, int64_t expert0,
                       const void* recv_a16, const float* recv_scale, const int32_t* recv_hdr, int64_t n_rows,
                       int64_t n_used, int64_t n_pairs_hint, float* ret, void* workspace, size_t workspace_bytes,
                       int* dev_err, void* stream) {
    using namespace b200;
    if (!local_stack || !ret || !dev_err || K <= 0 || N <= 0 || n_local <= 0 || expert0 < 0 || n_rows < 0 ||
        n_used <= 0)
        return B200_E_INVALID;
    if (n_rows == 0) return B200_OK;
    if (!recv_a16 || !recv_scale || !recv_hdr) return B200_E_INVALID;
    if (!weight_type_supported(wtype, K) || K % 32 != 0 || N % 16 != 0 || n_used > EP_MAX_SLOTS || n_local > 4096 ||
        n_rows * n_used > (1 << 28))
        return B200_E_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(recv_a16) & 15u) || (reinterpret_cast<uintptr_t>(ret) & 15u))
        return B200_E_UNSUPPORTED;
    const EpExpertLayout L = ep_expert_layout(K, n_local, n_used, n_rows);
    if (!workspace || workspace_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return B200_E_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    int32_t* off = reinterpret_cast<int32_t*>(ws + L.off);
    int32_t* tiles = reinterpret_cast<int32_t*>(ws + L.tiles);
    int32_t* src = reinterpret_cast<int32_t*>(ws + L.src);
    int32_t* rix = reinterpret_cast<int32_t*>(ws + L.ret);
    int32_t* zero = reinterpret_cast<int32_t*>(ws + L.zero);
    __half* a16 = reinterpret_cast<__half*>(ws + L.a16);
    float* scales = reinterpret_cast<float*>(ws + L.scales);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t pmax = n_rows * n_used;
    const int bt = ep_token_tile(n_pairs_hint > 0 ? n_pairs_hint : n_rows, n_local);
    const size_t smem = (size_t)2 * n_local * sizeof(int);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(ep_expert_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return B200_E_UNSUPPORTED;
    ep_expert_route_kernel<<<1, EP_THREADS, smem, st>>>(recv_hdr, (int)n_rows, (int)n_used, (int)expert0,
                                                        (int)n_local, bt, off, tiles, src, rix, zero, dev_err);
    if (cudaGetLastError() != cudaSuccess) return B200_E_CUDA;
    ep_gather_rows_kernel<<<(unsigned)pmax, 256, 0, st>>>(static_cast<const __half*>(recv_a16), recv_scale, src,
                                                          off + n_local, (int)K, a16, scales);
    if (cudaGetLastError() != cudaSuccess) return B200_E_CUDA;
    return gemm_grouped_impl(wtype, local_stack, N, K, n_local, a16, scales, pmax, bt, off, tiles, zero, rix, ret, 0,
                             N * 4, dev_err, st);
}

int b200_moe_ep_combine(const float* ret, int64_t N, const int32_t* send_hdr, int64_t n_used, const int32_t* row_tok,
                        const int32_t* row_ret, const int32_t* counts, int64_t n_ranks, int64_t max_rows, float* dst,
                        int64_t d_nb1, int64_t d_nb2, void* stream) {
    using namespace b200;
    if (!send_hdr || !row_tok || !row_ret || !counts || !dst || N <= 0 || n_used <= 0 || n_ranks <= 0 || max_rows < 0)
        return B200_E_INVALID;
    if (max_rows == 0) return B200_OK;
    if (!ret) return B200_E_INVALID;
    if (N % 4 || (d_nb1 % 16) || (d_nb2 % 16) || (reinterpret_cast<uintptr_t>(dst) & 15u) ||
        (reinterpret_cast<uintptr_t>(ret) & 15u))
        return B200_E_UNSUPPORTED;
    ep_combine_kernel<<<(unsigned)max_rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        ret, (int)N, send_hdr, (int)n_used, row_tok, row_ret, counts + 2 * n_ranks, dst, d_nb1, d_nb2);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
