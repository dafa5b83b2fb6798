// MUL_MAT_ID on sm_100a (the reference's ggml_backend_rocket_mul_mat_id,
// ggml-rocket.cpp:6692-6944), with no host round trip:
//   route      the counting sort of (slot, token) rows by expert id (ggml-rocket.cpp:6706-6732),
//              stable in token-major order like the reference's, plus the grouped GEMM's tile
//              table (per-expert prefix of ceil(rows / token tile)); a bad id aborts the op
//   gather     row r of the sorted order -> b[:, slot % ne11, tok], packed to fp16 with its
//              per-row scale (the reference's gather + pack, :6790-6800 / :1451-1475)
//   grouped    the tcgen05 GEMM of gemm.cuh over every (expert, token tile, weight tile) unit the
//              table lists, whose epilogue scatters each row straight to dst[:, slot, tok]
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "glu.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int ROUTE_THREADS = 1024;
constexpr int ROUTE_CHUNK = 1024;   // rows per CTA of the histogram / placement passes

// The route is a stable counting sort over the token-major row order r = t * n_used + s, split
// over CTAs that each own ROUTE_CHUNK consecutive rows:
//   moe_hist_kernel    per-CTA histogram of the experts of its rows (and a bad-id flag)
//   moe_scan_kernel    one CTA: per-expert offsets, the tile table, and every CTA's first
//                      position per expert (CTA-major within an expert, which keeps the order)
//   moe_place_kernel   per CTA: its rows in order, each to its expert's next position
__device__ __forceinline__ int moe_id_at(const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1, int n_used, int r) {
    const int t = r / n_used, e = r % n_used;
    return __ldg(reinterpret_cast<const int32_t*>(reinterpret_cast<const char*>(ids) + (int64_t)t * ids_nb1 +
                                                  (int64_t)e * ids_nb0));
}

// Dynamic shared memory: cnt[E].
__global__ void __launch_bounds__(ROUTE_THREADS) moe_hist_kernel(const int32_t* __restrict__ ids, int64_t ids_nb0,
                                                                int64_t ids_nb1, int n_used, int R, int E,
                                                                int32_t* __restrict__ counts, int32_t* __restrict__ bad) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    extern __shared__ int cnt[];
    for (int e = threadIdx.x; e < E; e += ROUTE_THREADS) cnt[e] = 0;
    __syncthreads();
    const int r0 = blockIdx.x * ROUTE_CHUNK, r1 = min(R, r0 + ROUTE_CHUNK);
    int b = 0;
    for (int r = r0 + threadIdx.x; r < r1; r += ROUTE_THREADS) {
        const int x = moe_id_at(ids, ids_nb0, ids_nb1, n_used, r);
        if (x < 0 || x >= E) b = 1;
        else atomicAdd(&cnt[x], 1);
    }
    b = __syncthreads_or(b);
    for (int e = threadIdx.x; e < E; e += ROUTE_THREADS) counts[(int64_t)blockIdx.x * E + e] = cnt[e];
    if (threadIdx.x == 0) bad[blockIdx.x] = b;
}

// One CTA. counts[nb][E] becomes each CTA's first position per expert (relative to the expert's
// start); off / tile_start are exclusive scans over the experts. Dynamic shared memory: E ints.
__global__ void __launch_bounds__(ROUTE_THREADS) moe_scan_kernel(int32_t* __restrict__ counts,
                                                                const int32_t* __restrict__ bad, int nb, int E, int bt,
                                                                int32_t* __restrict__ off,
                                                                int32_t* __restrict__ tile_start, int* err) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    extern __shared__ int tot[];
    __shared__ int wsum[2][32];
    __shared__ int carry[2];
    int any = 0;
    for (int b = threadIdx.x; b < nb; b += ROUTE_THREADS) any |= __ldg(bad + b);
    if (__syncthreads_or(any)) {
        if (threadIdx.x == 0) atomicCAS(err, 0, B200_DEV_BAD_IDS);
        for (int e = threadIdx.x; e <= E; e += ROUTE_THREADS) {
            off[e] = 0;
            tile_start[e] = 0;
        }
        return;
    }
    for (int e = threadIdx.x; e < E; e += ROUTE_THREADS) {
        int acc = 0;
        for (int b0 = 0; b0 < nb; b0 += 8) {       // eight independent loads per round trip
            int c[8];
#pragma unroll
            for (int k = 0; k < 8; k++) c[k] = b0 + k < nb ? counts[(int64_t)(b0 + k) * E + e] : 0;
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (b0 + k < nb) counts[(int64_t)(b0 + k) * E + e] = acc;
                acc += c[k];
            }
        }
        tot[e] = acc;
    }
    if (threadIdx.x < 2) carry[threadIdx.x] = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // exclusive scans of the row counts and of the tile counts, ROUTE_THREADS experts at a time
    for (int e0 = 0; e0 < E; e0 += ROUTE_THREADS) {
        const int e = e0 + threadIdx.x;
        const int c = e < E ? tot[e] : 0;
        int v[2] = {c, (c + bt - 1) / bt};
        int incl[2];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            int x = v[k];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            incl[k] = x;
            if (lane == 31) wsum[k][warp] = x;
        }
        __syncthreads();
        if (warp == 0) {
#pragma unroll
            for (int k = 0; k < 2; k++) {
                int x = wsum[k][lane];
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, x, o);
                    if (lane >= o) x += y;
                }
                wsum[k][lane] = x;
            }
        }
        __syncthreads();
        const int before0 = carry[0] + (warp > 0 ? wsum[0][warp - 1] : 0) + incl[0] - v[0];
        const int before1 = carry[1] + (warp > 0 ? wsum[1][warp - 1] : 0) + incl[1] - v[1];
        if (e < E) {
            off[e] = before0;
            tile_start[e] = before1;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            carry[0] += wsum[0][31];
            carry[1] += wsum[1][31];
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        off[E] = carry[0];
        tile_start[E] = carry[1];
    }
}

// Dynamic shared memory: base[E], wcnt[32][E] (ints).
__global__ void __launch_bounds__(ROUTE_THREADS) moe_place_kernel(const int32_t* __restrict__ ids, int64_t ids_nb0,
                                                                 int64_t ids_nb1, int n_used, int R, int E,
                                                                 const int32_t* __restrict__ counts,
                                                                 const int32_t* __restrict__ off,
                                                                 int32_t* __restrict__ slot, int32_t* __restrict__ tok) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    extern __shared__ int sm[];
    int* base = sm;
    int* wcnt = sm + E;
    if (__ldg(off + E) != R) return;      // a bad-id op: the scan wrote an empty table
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += ROUTE_THREADS) base[e] = __ldg(off + e) + counts[(int64_t)blockIdx.x * E + e];
    for (int i = threadIdx.x; i < 32 * E; i += ROUTE_THREADS) wcnt[i] = 0;
    __syncthreads();
    const int r0 = blockIdx.x * ROUTE_CHUNK, r1 = min(R, r0 + ROUTE_CHUNK);
    const unsigned lt_mask = (1u << lane) - 1u;
    for (int rb = r0; rb < r1; rb += ROUTE_THREADS) {
        const int r = rb + threadIdx.x;
        const int x = r < r1 ? moe_id_at(ids, ids_nb0, ids_nb1, n_used, r) : -1;
        const unsigned same = __match_any_sync(0xffffffffu, x);
        const int rank = __popc(same & lt_mask);
        if (x >= 0 && rank == 0) wcnt[warp * E + x] = __popc(same);
        __syncthreads();
        if (x >= 0) {
            int prefix = 0;
            for (int w = 0; w < warp; w++) prefix += wcnt[w * E + x];
            const int p = base[x] + prefix + rank;
            slot[p] = r % n_used;
            tok[p] = r / n_used;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < E; e += ROUTE_THREADS) {
            int s = 0;
            for (int w = 0; w < 32; w++) {
                s += wcnt[w * E + e];
                wcnt[w * E + e] = 0;
            }
            base[e] += s;
        }
        __syncthreads();
    }
}

// Row r of the sorted order: gather b[:, slot % ne11, tok] and pack it like act_pack_kernel.
template <int V>
__global__ void __launch_bounds__(256) moe_gather_pack_kernel(const float* __restrict__ b, int64_t b_nb1,
                                                              int64_t b_nb2, int ne11, int K,
                                                              const int32_t* __restrict__ slot,
                                                              const int32_t* __restrict__ tok,
                                                              const int32_t* __restrict__ off_total,
                                                              __half* __restrict__ a16, float* __restrict__ scales,
                                                              int32_t* __restrict__ self) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __shared__ float red[8];
    const int r = blockIdx.x;
    if (r >= __ldg(off_total)) return;   // a bad-id op has no rows
    if (self && threadIdx.x == 0) self[r] = r;   // the expert FFN's own rows: row r of a [rows][N] buffer
    const int s = __ldg(slot + r), t = __ldg(tok + r);
    const float4* row = reinterpret_cast<const float4*>(reinterpret_cast<const char*>(b) + (int64_t)t * b_nb2 +
                                                        (int64_t)(s % ne11) * b_nb1);
    uint2* out = reinterpret_cast<uint2*>(a16 + (int64_t)r * K);
    const int n4 = K / 4;
    float4 v[V];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int idx = threadIdx.x + i * 256;
        v[i] = idx < n4 ? __ldg(row + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < 8; w++) amax = fmaxf(amax, red[w]);
    const float sc = amax > 0.0f ? amax : 1.0f;
    const float inv = __frcp_rn(sc);
    if (threadIdx.x == 0) scales[r] = sc;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int idx = threadIdx.x + i * 256;
        if (idx < n4) {
            uint2 w;
            w.x = pack_half2(__fmul_rn(v[i].x, inv), __fmul_rn(v[i].y, inv));
            w.y = pack_half2(__fmul_rn(v[i].z, inv), __fmul_rn(v[i].w, inv));
            out[idx] = w;
        }
    }
}

int launch_gather_pack(const float* b, int64_t b_nb1, int64_t b_nb2, int64_t ne11, int64_t K, const int32_t* slot,
                       const int32_t* tok, const int32_t* n_rows, int64_t max_rows, __half* a16, float* scales,
                       cudaStream_t st, int32_t* self) {
    if (max_rows <= 0) return B200_OK;
    const int64_t per = (K / 4 + 255) / 256;
    const dim3 grid((unsigned)max_rows);
#define B200_GATHER(V) \
    launch_pdl(moe_gather_pack_kernel<V>, dim3(grid), dim3(256), 0, st, b, b_nb1, b_nb2, (int)ne11, (int)K, slot, tok, \
               n_rows, a16, scales, self)
    if (per <= 1) B200_GATHER(1);
    else if (per <= 2) B200_GATHER(2);
    else if (per <= 4) B200_GATHER(4);
    else if (per <= 8) B200_GATHER(8);
    else if (per <= 16) B200_GATHER(16);
    else return B200_E_UNSUPPORTED;
#undef B200_GATHER
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

// The expert FFN between its projections: row p's down-projection input h = swiglu(gate[p], up[p])
// (f32 rows of F, in the route's sorted order), packed like every activation row of the GEMMs
// (s = max|h| or 1, fp16(h * (1/s))). The arithmetic is the SWIGLU glue kernel's followed by the
// gather-pack's, so the packed rows equal, bit for bit, those the op chain MUL_MAT_ID, SWIGLU,
// MUL_MAT_ID builds for the down projection. One 256-thread CTA per row (grid-stride over the
// device's row count), V float4 per thread.
template <int V>
__global__ void __launch_bounds__(256) swiglu_pack_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                                             int F, const int32_t* __restrict__ n_rows,
                                                             __half* __restrict__ a16, float* __restrict__ scales) {
    grid_dep_wait();   // programmatic launch: the previous kernel's output is complete
    grid_dep_launch();
    __shared__ float red[8];
    const int n = __ldg(n_rows);
    const int n4 = F / 4;
    for (int p = blockIdx.x; p < n; p += gridDim.x) {
        const float4* g4 = reinterpret_cast<const float4*>(gate + (int64_t)p * F);
        const float4* u4 = reinterpret_cast<const float4*>(up + (int64_t)p * F);
        float4 v[V];
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < V; i++) {
            const int idx = threadIdx.x + i * 256;
            if (idx < n4) {
                const float4 x = g4[idx], y = u4[idx];
                v[i] = make_float4(swiglu_f(x.x, y.x), swiglu_f(x.y, y.y), swiglu_f(x.z, y.z), swiglu_f(x.w, y.w));
            } else {
                v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
        __syncthreads();
        amax = red[0];
#pragma unroll
        for (int w = 1; w < 8; w++) amax = fmaxf(amax, red[w]);
        __syncthreads();   // red is rewritten by the next row
        const float sc = amax > 0.0f ? amax : 1.0f;
        const float inv = __frcp_rn(sc);
        if (threadIdx.x == 0) scales[p] = sc;
        uint2* out = reinterpret_cast<uint2*>(a16 + (int64_t)p * F);
#pragma unroll
        for (int i = 0; i < V; i++) {
            const int idx = threadIdx.x + i * 256;
            if (idx < n4) {
                uint2 w;
                w.x = pack_half2(__fmul_rn(v[i].x, inv), __fmul_rn(v[i].y, inv));
                w.y = pack_half2(__fmul_rn(v[i].z, inv), __fmul_rn(v[i].w, inv));
                out[idx] = w;
            }
        }
    }
}

int launch_swiglu_pack(const float* gate, const float* up, int64_t F, const int32_t* n_rows, int64_t max_rows,
                       __half* h16, float* hscale, cudaStream_t st) {
    if (max_rows <= 0) return B200_OK;
    if (F % 8 || F > 8192) return B200_E_UNSUPPORTED;
    const int64_t gcap = (int64_t)device_sm_count() * 8;
    const dim3 grid((unsigned)(max_rows < gcap ? max_rows : gcap));
    const int64_t v = (F / 4 + 255) / 256;
    if (v <= 1) launch_pdl(swiglu_pack_kernel<1>, grid, dim3(256), 0, st, gate, up, (int)F, n_rows, h16, hscale);
    else if (v <= 2) launch_pdl(swiglu_pack_kernel<2>, grid, dim3(256), 0, st, gate, up, (int)F, n_rows, h16, hscale);
    else if (v <= 4) launch_pdl(swiglu_pack_kernel<4>, grid, dim3(256), 0, st, gate, up, (int)F, n_rows, h16, hscale);
    else launch_pdl(swiglu_pack_kernel<8>, grid, dim3(256), 0, st, gate, up, (int)F, n_rows, h16, hscale);
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

struct MoeLayout {
    size_t off, tiles, slot, tok, a16, scales, counts, bad, total;
};

static MoeLayout moe_layout(int64_t K, int64_t n_expert, int64_t n_used, int64_t n_tokens) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t R = (size_t)(n_used * n_tokens);
    MoeLayout L{};
    L.off = 0;
    L.tiles = al((size_t)(n_expert + 1) * 4);
    L.slot = L.tiles + al((size_t)(n_expert + 1) * 4);
    L.tok = L.slot + al(R * 4);
    L.a16 = L.tok + al(R * 4);
    L.scales = L.a16 + al(R * (size_t)K * 2);
    const size_t nb = (R + ROUTE_CHUNK - 1) / ROUTE_CHUNK;
    L.counts = L.scales + al(R * 4);
    L.bad = L.counts + al(nb * (size_t)n_expert * 4);
    L.total = L.bad + al(nb * 4);
    return L;
}

// The grouped GEMM decodes an expert's weight tile once per token tile; at ~100+ rows per expert
// one 256-token tile (tensor-core work on its padding is cheaper than a second decode) wins.
static int moe_token_tile(int64_t R, int64_t n_expert) {
    const int64_t avg = n_expert > 0 ? R / n_expert : R;
    return avg <= 32 ? 32 : avg <= 64 ? 64 : avg < 96 ? 128 : 256;
}

// The route and the packed rows every grouped GEMM of an op reads: the histogram, scan and
// placement of the (token, slot) pairs by expert, then the gather-pack of their b rows in that
// order (self, when given, gets each sorted row's own index).
struct MoeRoute {
    int32_t *off, *tiles, *slot, *tok;
    __half* a16;
    float* scales;
    int64_t R;
    int bt;
};

static int moe_route_gather(const MoeLayout& L, char* ws, int64_t K, int64_t n_expert, const float* b, int64_t b_nb1,
                            int64_t b_nb2, int64_t ne11, const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1,
                            int64_t n_used, int64_t n_tokens, int32_t* self, int* dev_err, cudaStream_t st,
                            MoeRoute* out) {
    int32_t* off = reinterpret_cast<int32_t*>(ws + L.off);
    int32_t* tiles = reinterpret_cast<int32_t*>(ws + L.tiles);
    int32_t* slot = reinterpret_cast<int32_t*>(ws + L.slot);
    int32_t* tok = reinterpret_cast<int32_t*>(ws + L.tok);
    __half* a16 = reinterpret_cast<__half*>(ws + L.a16);
    float* scales = reinterpret_cast<float*>(ws + L.scales);
    const int64_t R = n_used * n_tokens;
    const int bt = moe_token_tile(R, n_expert);
    *out = MoeRoute{off, tiles, slot, tok, a16, scales, R, bt};
    int32_t* counts = reinterpret_cast<int32_t*>(ws + L.counts);
    int32_t* bad = reinterpret_cast<int32_t*>(ws + L.bad);
    const int nb = (int)((R + ROUTE_CHUNK - 1) / ROUTE_CHUNK);
    const size_t hist_smem = (size_t)n_expert * sizeof(int);
    const size_t place_smem = (size_t)33 * n_expert * sizeof(int);
    if (place_smem > 48 * 1024 &&
        cudaFuncSetAttribute(moe_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)place_smem) !=
            cudaSuccess)
        return B200_E_UNSUPPORTED;
    launch_pdl(moe_hist_kernel, dim3(nb), dim3(ROUTE_THREADS), hist_smem, st, ids, ids_nb0, ids_nb1, (int)n_used,
               (int)R, (int)n_expert, counts, bad);
    launch_pdl(moe_scan_kernel, dim3(1), dim3(ROUTE_THREADS), hist_smem, st, counts, bad, nb, (int)n_expert, bt, off,
               tiles, dev_err);
    launch_pdl(moe_place_kernel, dim3(nb), dim3(ROUTE_THREADS), place_smem, st, ids, ids_nb0, ids_nb1, (int)n_used,
               (int)R, (int)n_expert, counts, off, slot, tok);
    if (cudaGetLastError() != cudaSuccess) return B200_E_CUDA;
    return launch_gather_pack(b, b_nb1, b_nb2, ne11, K, slot, tok, off + n_expert, R, a16, scales, st, self);
}

// MUL_MAT_ID over n_members expert stacks that share the input rows b and the routing ids (a
// layer's gate and up projections): the route and the gather-pack run once, then one grouped
// GEMM per member reads the same sorted fp16 rows. n_members = 1 is the plain op.
int mul_mat_id_group_impl(int n_members, int wtype, const void* const* as_packed, const int64_t* Ns, int64_t K,
                          int64_t n_expert, const float* b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                          const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                          float* const* dsts, const int64_t* d_nb1s, const int64_t* d_nb2s, void* workspace,
                          size_t ws_bytes, int* dev_err, cudaStream_t st) {
    if (n_members <= 0 || !as_packed || !Ns || !dsts || !d_nb1s || !d_nb2s || !b || !ids || !dev_err || K <= 0 ||
        n_expert <= 0 || n_used <= 0 || n_tokens <= 0 || ne11 <= 0)
        return B200_E_INVALID;
    for (int m = 0; m < n_members; m++)
        if (!as_packed[m] || !dsts[m] || Ns[m] <= 0) return B200_E_INVALID;
    if (!weight_type_supported(wtype, K) || K % 32 != 0 || K % 4 != 0) return B200_E_UNSUPPORTED;
    for (int m = 0; m < n_members; m++)
        if (Ns[m] % 16 != 0) return B200_E_UNSUPPORTED;
    if (n_expert > 4096 || n_used * n_tokens > (1 << 28)) return B200_E_UNSUPPORTED;
    if ((b_nb1 % 16) || (b_nb2 % 16) || (reinterpret_cast<uintptr_t>(b) & 15u)) return B200_E_UNSUPPORTED;
    const MoeLayout L = moe_layout(K, n_expert, n_used, n_tokens);
    if (!workspace || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return B200_E_WORKSPACE;
    MoeRoute R;
    const int rc = moe_route_gather(L, static_cast<char*>(workspace), K, n_expert, b, b_nb1, b_nb2, ne11, ids, ids_nb0,
                                    ids_nb1, n_used, n_tokens, nullptr, dev_err, st, &R);
    if (rc != B200_OK) return rc;
    for (int m = 0; m < n_members; m++) {
        const int r2 = gemm_grouped_impl(wtype, as_packed[m], Ns[m], K, n_expert, R.a16, R.scales, R.R, R.bt, R.off,
                                         R.tiles, R.slot, R.tok, dsts[m], d_nb1s[m], d_nb2s[m], dev_err, st);
        if (r2 != B200_OK) return r2;
    }
    return B200_OK;
}

int mul_mat_id_impl(int wtype, const void* as_packed, int64_t K, int64_t N, int64_t n_expert, const float* b,
                    int64_t b_nb1, int64_t b_nb2, int64_t ne11, const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1,
                    int64_t n_used, int64_t n_tokens, float* dst, int64_t d_nb1, int64_t d_nb2, void* workspace,
                    size_t ws_bytes, int* dev_err, cudaStream_t st) {
    if (!as_packed || !dst) return B200_E_INVALID;
    return mul_mat_id_group_impl(1, wtype, &as_packed, &N, K, n_expert, b, b_nb1, b_nb2, ne11, ids, ids_nb0, ids_nb1,
                                 n_used, n_tokens, &dst, &d_nb1, &d_nb2, workspace, ws_bytes, dev_err, st);
}

// The expert FFN of a MoE block, down(swiglu(gate(x), up(x))) per (token, slot), in one pass
// over one route: the pairs are routed and x's rows gathered once, gate and up write [R][F]
// buffers in the route's order (each row's token index is the row itself), the SWIGLU and the
// down projection's packing run in one kernel over those rows, and the down GEMM reuses the
// route to store dst. The single-GPU twin of the expert-parallel owner step; the result equals,
// bit for bit, MUL_MAT_ID group (gate, up) -> SWIGLU -> MUL_MAT_ID (down).
struct MoeFfnLayout {
    MoeLayout base;
    size_t self, gate, up, h16, hscale, total;
};

static MoeFfnLayout moe_ffn_layout(int64_t H, int64_t F, int64_t n_expert, int64_t n_used, int64_t n_tokens) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t R = (size_t)(n_used * n_tokens);
    MoeFfnLayout L{};
    L.base = moe_layout(H, n_expert, n_used, n_tokens);
    L.self = L.base.total;
    L.gate = L.self + al(R * 4);
    L.up = L.gate + al(R * (size_t)F * 4);
    L.h16 = L.up + al(R * (size_t)F * 4);
    L.hscale = L.h16 + al(R * (size_t)F * 2);
    L.total = L.hscale + al(R * 4);
    return L;
}

int mul_mat_id_ffn_impl(int wt_gate_up, const void* gate_packed, const void* up_packed, int wt_down,
                        const void* down_packed, int64_t H, int64_t F, int64_t n_expert, const float* x, int64_t x_nb1,
                        int64_t x_nb2, int64_t ne11, const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1,
                        int64_t n_used, int64_t n_tokens, float* dst, int64_t d_nb1, int64_t d_nb2, void* workspace,
                        size_t ws_bytes, int* dev_err, cudaStream_t st) {
    if (!gate_packed || !up_packed || !down_packed || !x || !ids || !dst || !dev_err || H <= 0 || F <= 0 ||
        n_expert <= 0 || n_used <= 0 || n_tokens <= 0 || ne11 <= 0)
        return B200_E_INVALID;
    if (!weight_type_supported(wt_gate_up, H) || !weight_type_supported(wt_down, F) || H % 32 || F % 32 || F > 8192)
        return B200_E_UNSUPPORTED;
    if (n_expert > 4096 || n_used * n_tokens > (1 << 28)) return B200_E_UNSUPPORTED;
    if ((x_nb1 % 16) || (x_nb2 % 16) || (reinterpret_cast<uintptr_t>(x) & 15u)) return B200_E_UNSUPPORTED;
    const MoeFfnLayout L = moe_ffn_layout(H, F, n_expert, n_used, n_tokens);
    if (!workspace || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return B200_E_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    int32_t* self = reinterpret_cast<int32_t*>(ws + L.self);
    float* gate = reinterpret_cast<float*>(ws + L.gate);
    float* up = reinterpret_cast<float*>(ws + L.up);
    __half* h16 = reinterpret_cast<__half*>(ws + L.h16);
    float* hscale = reinterpret_cast<float*>(ws + L.hscale);
    MoeRoute R;
    int rc = moe_route_gather(L.base, ws, H, n_expert, x, x_nb1, x_nb2, ne11, ids, ids_nb0, ids_nb1, n_used, n_tokens,
                              self, dev_err, st, &R);
    if (rc != B200_OK) return rc;
    rc = gemm_grouped_impl(wt_gate_up, gate_packed, F, H, n_expert, R.a16, R.scales, R.R, R.bt, R.off, R.tiles, self,
                           self, gate, 0, F * 4, dev_err, st);
    if (rc != B200_OK) return rc;
    rc = gemm_grouped_impl(wt_gate_up, up_packed, F, H, n_expert, R.a16, R.scales, R.R, R.bt, R.off, R.tiles, self,
                           self, up, 0, F * 4, dev_err, st);
    if (rc != B200_OK) return rc;
    rc = launch_swiglu_pack(gate, up, F, R.off + n_expert, R.R, h16, hscale, st);
    if (rc != B200_OK) return rc;
    return gemm_grouped_impl(wt_down, down_packed, H, F, n_expert, h16, hscale, R.R, R.bt, R.off, R.tiles, R.slot, R.tok,
                             dst, d_nb1, d_nb2, dev_err, st);
}

}  // namespace b200

extern "C" {

size_t b200_mul_mat_id_workspace_size(int64_t K, int64_t N, int64_t n_expert, int64_t n_used, int64_t n_tokens) {
    (void)N;
    if (K <= 0 || n_expert <= 0 || n_used <= 0 || n_tokens <= 0) return 0;
    return b200::moe_layout(K, n_expert, n_used, n_tokens).total;
}

int b200_mul_mat_id(int wtype, const void* as_packed, int64_t K, int64_t N, int64_t n_expert, const float* b,
                    int64_t b_nb1, int64_t b_nb2, int64_t ne11, const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1,
                    int64_t n_used, int64_t n_tokens, float* dst, int64_t d_nb1, int64_t d_nb2, void* workspace,
                    size_t workspace_bytes, int* dev_err, void* stream) {
    return b200::mul_mat_id_impl(wtype, as_packed, K, N, n_expert, b, b_nb1, b_nb2, ne11, ids, ids_nb0, ids_nb1, n_used,
                                 n_tokens, dst, d_nb1, d_nb2, workspace, workspace_bytes, dev_err,
                                 static_cast<cudaStream_t>(stream));
}

int b200_mul_mat_id_group(int n_members, int wtype, const void* const* as_packed, const int64_t* N, int64_t K,
                          int64_t n_expert, const float* b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                          const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                          float* const* dst, const int64_t* d_nb1, const int64_t* d_nb2, void* workspace,
                          size_t workspace_bytes, int* dev_err, void* stream) {
    if (n_members > 16) return B200_E_UNSUPPORTED;
    return b200::mul_mat_id_group_impl(n_members, wtype, as_packed, N, K, n_expert, b, b_nb1, b_nb2, ne11, ids, ids_nb0,
                                       ids_nb1, n_used, n_tokens, dst, d_nb1, d_nb2, workspace, workspace_bytes,
                                       dev_err, static_cast<cudaStream_t>(stream));
}

size_t b200_mul_mat_id_ffn_workspace_size(int64_t H, int64_t F, int64_t n_expert, int64_t n_used, int64_t n_tokens) {
    if (H <= 0 || F <= 0 || n_expert <= 0 || n_used <= 0 || n_tokens <= 0) return 0;
    return b200::moe_ffn_layout(H, F, n_expert, n_used, n_tokens).total;
}

int b200_mul_mat_id_ffn(int wtype_gate_up, const void* gate_packed, const void* up_packed, int wtype_down,
                        const void* down_packed, int64_t H, int64_t F, int64_t n_expert, const float* x, int64_t x_nb1,
                        int64_t x_nb2, int64_t ne11, const int32_t* ids, int64_t ids_nb0, int64_t ids_nb1,
                        int64_t n_used, int64_t n_tokens, float* dst, int64_t d_nb1, int64_t d_nb2, void* workspace,
                        size_t workspace_bytes, int* dev_err, void* stream) {
    return b200::mul_mat_id_ffn_impl(wtype_gate_up, gate_packed, up_packed, wtype_down, down_packed, H, F, n_expert, x,
                                     x_nb1, x_nb2, ne11, ids, ids_nb0, ids_nb1, n_used, n_tokens, dst, d_nb1, d_nb2,
                                     workspace, workspace_bytes, dev_err, static_cast<cudaStream_t>(stream));
}

int b200_mul_mat_id_route_view(int64_t K, int64_t n_expert, int64_t n_used, int64_t n_tokens, size_t* off_offset,
                               size_t* slot_offset, size_t* tok_offset) {
    if (K <= 0 || n_expert <= 0 || n_used <= 0 || n_tokens <= 0) return B200_E_INVALID;
    const b200::MoeLayout L = b200::moe_layout(K, n_expert, n_used, n_tokens);
    if (off_offset) *off_offset = L.off;
    if (slot_offset) *slot_offset = L.slot;
    if (tok_offset) *tok_offset = L.tok;
    return B200_OK;
}

}  // extern "C"
