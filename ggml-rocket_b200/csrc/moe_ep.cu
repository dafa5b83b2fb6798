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

constexpr int EPC = 256;   // candidates / rows per CTA of the multi-CTA passes

// Home side. Candidate c = t * ne11 + j is token t's b row j (serving slots s with s % ne11 == j).
// For destination rank d its slot mask is {s : s % ne11 == j, ids[s, t] / E_loc == d}. Send rows
// are ordered by destination, then token, then b row; their return rows by the same order with
// each row's slots ascending. Three passes over CTAs of EPC candidates: count per destination,
// one-CTA scan (destination-major, CTA order inside), write.
struct EpIds {
    const int32_t* ids;
    int64_t nb0, nb1;
    int n_used, ne11, e_loc;
    __device__ __forceinline__ int at(int s, int t) const {
        return __ldg(reinterpret_cast<const int32_t*>(reinterpret_cast<const char*>(ids) + (int64_t)t * nb1 +
                                                      (int64_t)s * nb0));
    }
    __device__ __forceinline__ uint32_t mask(int c, int d) const {
        const int t = c / ne11, j = c % ne11;
        uint32_t m = 0;
        for (int s = j; s < n_used; s += ne11)
            if (at(s, t) / e_loc == d) m |= 1u << s;
        return m;
    }
};

// bcounts[b][d] = {rows, return rows} of CTA b for destination d; bad[b] = a bad id seen.
__global__ void __launch_bounds__(EPC) ep_dispatch_count_kernel(EpIds I, int C, int E, int G,
                                                                int32_t* __restrict__ bcounts, int32_t* __restrict__ bad) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __shared__ int cnt[2 * EP_MAX_RANKS];
    for (int k = threadIdx.x; k < 2 * G; k += EPC) cnt[k] = 0;
    __syncthreads();
    const int c = blockIdx.x * EPC + threadIdx.x;
    int b = 0;
    if (c < C) {
        const int t = c / I.ne11, j = c % I.ne11;
        for (int s = j; s < I.n_used; s += I.ne11) {
            const int x = I.at(s, t);
            if (x < 0 || x >= E) b = 1;
        }
        if (!b) {
            for (int d = 0; d < G; d++) {
                const uint32_t m = I.mask(c, d);
                if (m) {
                    atomicAdd(&cnt[2 * d], 1);
                    atomicAdd(&cnt[2 * d + 1], __popc(m));
                }
            }
        }
    }
    b = __syncthreads_or(b);
    for (int k = threadIdx.x; k < 2 * G; k += EPC) bcounts[(int64_t)blockIdx.x * 2 * G + k] = cnt[k];
    if (threadIdx.x == 0) bad[blockIdx.x] = b;
}

// One thread: bcounts becomes each CTA's first {row, return row} per destination; counts[] gets
// the per-destination totals and the grand totals; bad[nb] = any bad id.
__global__ void ep_dispatch_scan_kernel(int32_t* __restrict__ bcounts, int32_t* __restrict__ bad, int nb, int G,
                                        int32_t* __restrict__ counts, int* err) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    if (threadIdx.x != 0) return;
    int any = 0;
    for (int b = 0; b < nb; b++) any |= bad[b];
    bad[nb] = any;
    if (any) {
        atomicCAS(err, 0, B200_DEV_BAD_IDS);
        for (int k = 0; k < 2 * G + 2; k++) counts[k] = 0;
        return;
    }
    int row_base = 0, pair_base = 0;
    for (int d = 0; d < G; d++) {
        int rr = 0, pp = 0;
        for (int b = 0; b < nb; b++) {
            int32_t* e = bcounts + (int64_t)b * 2 * G + 2 * d;
            const int r = e[0], p = e[1];
            e[0] = row_base + rr;
            e[1] = pair_base + pp;
            rr += r;
            pp += p;
        }
        counts[d] = rr;
        counts[G + d] = pp;
        row_base += rr;
        pair_base += pp;
    }
    counts[2 * G] = row_base;
    counts[2 * G + 1] = pair_base;
}

__global__ void __launch_bounds__(EPC) ep_dispatch_write_kernel(EpIds I, int C, int G,
                                                                const int32_t* __restrict__ bcounts,
                                                                const int32_t* __restrict__ bad_any,
                                                                int32_t* __restrict__ hdr, int32_t* __restrict__ row_tok,
                                                                int32_t* __restrict__ row_slot,
                                                                int32_t* __restrict__ row_ret) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __shared__ int sh[32];
    if (__ldg(bad_any)) return;
    const int c = blockIdx.x * EPC + threadIdx.x;
    for (int d = 0; d < G; d++) {
        const uint32_t m = c < C ? I.mask(c, d) : 0u;
        int tot;
        const int pr = block_excl_scan(m ? 1 : 0, &tot, sh);
        const int pq = block_excl_scan(__popc(m), &tot, sh);
        if (m) {
            const int32_t* base = bcounts + (int64_t)blockIdx.x * 2 * G + 2 * d;
            const int p = __ldg(base) + pr;
            const int t = c / I.ne11;
            int32_t* h = hdr + (int64_t)p * (I.n_used + 1);
            h[0] = (int32_t)m;
            for (int s = 0; s < I.n_used; s++) h[1 + s] = I.at(s, t);
            row_tok[p] = t;
            row_slot[p] = __ffs(m) - 1;
            row_ret[p] = __ldg(base + 1) + pq;
        }
    }
}

// Owner side: the received rows' (row, slot) pairs, counted per local expert, placed per expert
// (any order inside an expert: a row's output does not depend on its neighbours in a tile), with
// the return index rowpref[r] + (rank of slot s among row r's slots). Three passes over CTAs of
// EPC rows: expert histogram (into zeroed ecnt) and per-CTA pair sums; one-CTA scans (off /
// tile_start / placement cursors over experts, pair bases over CTAs); placement.
__global__ void __launch_bounds__(EPC) ep_route_count_kernel(const int32_t* __restrict__ hdr, int n_rows, int n_used,
                                                             int expert0, int e_loc, int32_t* __restrict__ ecnt,
                                                             int32_t* __restrict__ bsum, int32_t* __restrict__ bad) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    extern __shared__ int hist[];
    __shared__ int sh[32];
    for (int e = threadIdx.x; e < e_loc; e += EPC) hist[e] = 0;
    __syncthreads();
    const int r = blockIdx.x * EPC + threadIdx.x;
    int b = 0, pc = 0;
    if (r < n_rows) {
        const int32_t* h = hdr + (int64_t)r * (n_used + 1);
        uint32_t m = (uint32_t)h[0];
        if (n_used < 32 && (m >> n_used)) b = 1;
        pc = __popc(m);
        while (m) {
            const int s = __ffs(m) - 1;
            m &= m - 1;
            const int x = h[1 + s] - expert0;
            if (x < 0 || x >= e_loc) b = 1;
            else atomicAdd(&hist[x], 1);
        }
    }
    int tot;
    block_excl_scan(pc, &tot, sh);
    b = __syncthreads_or(b);
    for (int e = threadIdx.x; e < e_loc; e += EPC)
        if (hist[e]) atomicAdd(&ecnt[e], hist[e]);
    if (threadIdx.x == 0) {
        bsum[blockIdx.x] = tot;
        bad[blockIdx.x] = b;
    }
}

// One CTA of EP_THREADS. Dynamic shared memory: none.
__global__ void __launch_bounds__(EP_THREADS) ep_route_scan_kernel(const int32_t* __restrict__ ecnt,
                                                                  int32_t* __restrict__ bsum, int32_t* __restrict__ bad,
                                                                  int nb, int e_loc, int bt, int32_t* __restrict__ off,
                                                                  int32_t* __restrict__ tile_start,
                                                                  int32_t* __restrict__ cursor, int* err) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __shared__ int sh[32];
    __shared__ int carry[3];
    int any = 0;
    for (int b = threadIdx.x; b < nb; b += EP_THREADS) any |= bad[b];
    if (__syncthreads_or(any)) {
        if (threadIdx.x == 0) {
            atomicCAS(err, 0, B200_DEV_BAD_IDS);
            bad[nb] = 1;
        }
        for (int e = threadIdx.x; e <= e_loc; e += EP_THREADS) {
            off[e] = 0;
            tile_start[e] = 0;
        }
        return;
    }
    if (threadIdx.x == 0) {
        bad[nb] = 0;
        carry[0] = carry[1] = carry[2] = 0;
    }
    __syncthreads();
    for (int e0 = 0; e0 < e_loc; e0 += EP_THREADS) {
        const int e = e0 + threadIdx.x;
        const int c = e < e_loc ? ecnt[e] : 0;
        int t1, t2;
        const int x1 = block_excl_scan(c, &t1, sh);
        const int x2 = block_excl_scan((c + bt - 1) / bt, &t2, sh);
        if (e < e_loc) {
            off[e] = carry[0] + x1;
            cursor[e] = carry[0] + x1;
            tile_start[e] = carry[1] + x2;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            carry[0] += t1;
            carry[1] += t2;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        off[e_loc] = carry[0];
        tile_start[e_loc] = carry[1];
    }
    for (int b0 = 0; b0 < nb; b0 += EP_THREADS) {            // pair bases of the row CTAs
        const int b = b0 + threadIdx.x;
        const int v = b < nb ? bsum[b] : 0;
        int t;
        const int x = block_excl_scan(v, &t, sh);
        if (b < nb) bsum[b] = carry[2] + x;
        __syncthreads();
        if (threadIdx.x == 0) carry[2] += t;
        __syncthreads();
    }
}

__global__ void __launch_bounds__(EPC) ep_route_place_kernel(const int32_t* __restrict__ hdr, int n_rows, int n_used,
                                                             int expert0, const int32_t* __restrict__ bsum,
                                                             const int32_t* __restrict__ bad_any,
                                                             int32_t* __restrict__ cursor,
                                                             int32_t* __restrict__ pair_src,
                                                             int32_t* __restrict__ pair_ret,
                                                             int32_t* __restrict__ pair_zero) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __shared__ int sh[32];
    if (__ldg(bad_any)) return;
    const int r = blockIdx.x * EPC + threadIdx.x;
    uint32_t m = 0;
    const int32_t* h = hdr + (int64_t)r * (n_used + 1);
    if (r < n_rows) m = (uint32_t)h[0];
    int tot;
    int q = __ldg(bsum + blockIdx.x) + block_excl_scan(__popc(m), &tot, sh);
    while (m) {
        const int s = __ffs(m) - 1;
        m &= m - 1;
        const int x = h[1 + s] - expert0;
        const int p = atomicAdd(&cursor[x], 1);
        pair_src[p] = r;
        pair_ret[p] = q++;
        pair_zero[p] = 0;
    }
}

// Sorted pair p <- received row pair_src[p] (fp16 row and its scale); grid-stride over pairs.
__global__ void __launch_bounds__(256) ep_gather_rows_kernel(const __half* __restrict__ src, const float* __restrict__ src_scale,
                                                             const int32_t* __restrict__ pair_src,
                                                             const int32_t* __restrict__ n_pairs, int K,
                                                             __half* __restrict__ dst, float* __restrict__ dst_scale) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    const int n = __ldg(n_pairs);
    for (int p = blockIdx.x; p < n; p += gridDim.x) {
        const int r = __ldg(pair_src + p);
        const uint4* s = reinterpret_cast<const uint4*>(src + (int64_t)r * K);
        uint4* d = reinterpret_cast<uint4*>(dst + (int64_t)p * K);
        for (int i = threadIdx.x; i < K / 8; i += 256) d[i] = __ldg(s + i);
        if (threadIdx.x == 0) dst_scale[p] = __ldg(src_scale + r);
    }
}

// Home side: send row p's returned rows (one per slot in its mask, ascending) -> dst[:, s, t];
// grid-stride over send rows.
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ ret, int N,
                                                         const int32_t* __restrict__ hdr, int n_used,
                                                         const int32_t* __restrict__ row_tok,
                                                         const int32_t* __restrict__ row_ret,
                                                         const int32_t* __restrict__ n_rows, float* __restrict__ dst,
                                                         int64_t d_nb1, int64_t d_nb2) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    const int n = __ldg(n_rows);
    for (int p = blockIdx.x; p < n; p += gridDim.x) {
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
}

struct EpExpertLayout {
    size_t off, tiles, src, ret, zero, a16, scales, ecnt, cursor, bsum, bad, total;
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
    const size_t nb = (size_t)((n_rows + EPC - 1) / EPC);
    L.ecnt = L.scales + al(P * 4);
    L.cursor = L.ecnt + al((size_t)e_loc * 4);
    L.bsum = L.cursor + al((size_t)e_loc * 4);
    L.bad = L.bsum + al(nb * 4);
    L.total = L.bad + al((nb + 1) * 4);
    return L;
}

// as moe_token_tile: one 256-token tile once an expert averages ~100+ rows
static int ep_token_tile(int64_t pairs, int64_t e_loc) {
    const int64_t avg = e_loc > 0 ? pairs / e_loc : pairs;
    return avg <= 32 ? 32 : avg <= 64 ? 64 : avg < 96 ? 128 : 256;
}

static size_t ep_dispatch_scratch(int64_t n_tokens, int64_t ne11, int64_t n_ranks) {
    const size_t nb = (size_t)((n_tokens * ne11 + EPC - 1) / EPC);
    return ((nb * 2 * n_ranks * 4 + 255) & ~(size_t)255) + (nb + 1) * 4;
}

int ep_token_tile_public(int64_t pairs, int64_t e_loc) { return ep_token_tile(pairs, e_loc); }

void ep_route_scan_public(const int32_t* ecnt, int32_t* bsum, int32_t* bad, int nb, int e_loc, int bt, int32_t* off,
                          int32_t* tile_start, int32_t* cursor, int* err, cudaStream_t st) {
    launch_pdl(ep_route_scan_kernel, dim3(1), dim3(EP_THREADS), 0, st, ecnt, bsum, bad, nb, e_loc, bt, off,
               tile_start, cursor, err);
}

}  // namespace b200

extern "C" {

size_t b200_moe_ep_dispatch_scratch_size(int64_t n_tokens, int64_t ne11, int64_t n_ranks) {
    if (n_tokens <= 0 || ne11 <= 0 || n_ranks <= 0) return 0;
    return b200::ep_dispatch_scratch(n_tokens, ne11, n_ranks);
}

int b200_moe_ep_dispatch(const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                         int64_t n_expert, int64_t n_ranks, const float* b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                         int64_t K, void* send_a16, float* send_scale, int32_t* send_hdr, int32_t* row_tok,
                         int32_t* row_slot, int32_t* row_ret, int32_t* counts, void* scratch, size_t scratch_bytes,
                         int* dev_err, void* stream) {
    using namespace b200;
    if (!ids || !b || !send_a16 || !send_scale || !send_hdr || !row_tok || !row_slot || !row_ret || !counts ||
        !dev_err || n_used <= 0 || n_tokens <= 0 || n_expert <= 0 || n_ranks <= 0 || ne11 <= 0 || K <= 0)
        return B200_E_INVALID;
    if (!scratch || scratch_bytes < ep_dispatch_scratch(n_tokens, ne11, n_ranks) ||
        (reinterpret_cast<uintptr_t>(scratch) & 255u))
        return B200_E_WORKSPACE;
    if (n_used > EP_MAX_SLOTS || n_ranks > EP_MAX_RANKS || n_expert % n_ranks != 0 || n_used % ne11 != 0 ||
        K % 8 != 0 || n_tokens * n_used > (1 << 28))
        return B200_E_UNSUPPORTED;
    if ((b_nb1 % 16) || (b_nb2 % 16) || (reinterpret_cast<uintptr_t>(b) & 15u) ||
        (reinterpret_cast<uintptr_t>(send_a16) & 15u))
        return B200_E_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int C = (int)(n_tokens * ne11);
    const int nb = (C + EPC - 1) / EPC;
    int32_t* bcounts = static_cast<int32_t*>(scratch);
    int32_t* bad = reinterpret_cast<int32_t*>(static_cast<char*>(scratch) +
                                              (((size_t)nb * 2 * n_ranks * 4 + 255) & ~(size_t)255));
    const EpIds I{ids, ids_nb0, ids_nb1, (int)n_used, (int)ne11, (int)(n_expert / n_ranks)};
    launch_pdl(ep_dispatch_count_kernel, dim3(nb), dim3(EPC), 0, st, I, C, (int)n_expert, (int)n_ranks, bcounts,
               bad);
    launch_pdl(ep_dispatch_scan_kernel, dim3(1), dim3(32), 0, st, bcounts, bad, nb, (int)n_ranks, counts, dev_err);
    launch_pdl(ep_dispatch_write_kernel, dim3(nb), dim3(EPC), 0, st, I, C, (int)n_ranks, bcounts, bad + nb, send_hdr,
               row_tok, row_slot, row_ret);
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
    int32_t* ecnt = reinterpret_cast<int32_t*>(ws + L.ecnt);
    int32_t* cursor = reinterpret_cast<int32_t*>(ws + L.cursor);
    int32_t* bsum = reinterpret_cast<int32_t*>(ws + L.bsum);
    int32_t* bad = reinterpret_cast<int32_t*>(ws + L.bad);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t pmax = n_rows * n_used;
    const int bt = ep_token_tile(n_pairs_hint > 0 ? n_pairs_hint : n_rows, n_local);
    const int nb = (int)((n_rows + EPC - 1) / EPC);
    const size_t hist_smem = (size_t)n_local * sizeof(int);
    if (hist_smem > 48 * 1024 &&
        cudaFuncSetAttribute(ep_route_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_smem) !=
            cudaSuccess)
        return B200_E_UNSUPPORTED;
    if (cudaMemsetAsync(ecnt, 0, (size_t)n_local * 4, st) != cudaSuccess) return B200_E_CUDA;
    launch_pdl(ep_route_count_kernel, dim3(nb), dim3(EPC), hist_smem, st, recv_hdr, (int)n_rows, (int)n_used,
               (int)expert0, (int)n_local, ecnt, bsum, bad);
    launch_pdl(ep_route_scan_kernel, dim3(1), dim3(EP_THREADS), 0, st, ecnt, bsum, bad, nb, (int)n_local, bt, off, tiles,
               cursor, dev_err);
    launch_pdl(ep_route_place_kernel, dim3(nb), dim3(EPC), 0, st, recv_hdr, (int)n_rows, (int)n_used, (int)expert0,
               bsum, bad + nb, cursor, src, rix, zero);
    if (cudaGetLastError() != cudaSuccess) return B200_E_CUDA;
    const int64_t gcap = (int64_t)device_sm_count() * 8;
    launch_pdl(ep_gather_rows_kernel, dim3((unsigned)(pmax < gcap ? pmax : gcap)), dim3(256), 0, st,
               static_cast<const __half*>(recv_a16), recv_scale, src, off + n_local, (int)K, a16, scales);
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
    const int64_t gcap = (int64_t)device_sm_count() * 8;
    launch_pdl(ep_combine_kernel, dim3((unsigned)(max_rows < gcap ? max_rows : gcap)), dim3(256), 0,
               static_cast<cudaStream_t>(stream), ret, (int)N, send_hdr, (int)n_used, row_tok, row_ret,
               counts + 2 * n_ranks, dst, d_nb1, d_nb2);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
