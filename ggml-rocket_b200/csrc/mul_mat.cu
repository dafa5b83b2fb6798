// MUL_MAT on sm_100a: the activation pre-pass, the weight decode / re-layout kernels, the
// tcgen05 GEMM launches (gemm.cuh, stream-K scheduled), behind the C ABI declared in
// include/ggml-b200-kernels.h.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <utility>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "gemm.cuh"
#include "glu.cuh"
#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"

namespace b200 {

// ------------------------------------------------------------------------------------------
// Activation "sandwich" pre-pass (the reference's rk_pack_act_row, ggml-rocket.cpp:1451-1475):
// per row s = max|A[m,:]| (1 when 0), A16 = fp16(A * (1/s)).
// One 256-thread CTA per row; the row is read from HBM once into registers (V float4 per
// thread), reduced across the CTA, then scaled and written from registers.
// ------------------------------------------------------------------------------------------
constexpr int ACT_THREADS = 256;

template <int V>
__global__ void __launch_bounds__(ACT_THREADS) act_pack_kernel(const float* __restrict__ A, int64_t lda, int K,
                                                               __half* __restrict__ A16, float* __restrict__ scales) {
    __shared__ float red[ACT_THREADS / 32];
    grid_dep_wait();     // the previous kernel may still read A16 / write A (programmatic launch)
    grid_dep_launch();
    const int m = blockIdx.x;
    const float4* row = reinterpret_cast<const float4*>(A + (size_t)m * lda);
    uint2* out = reinterpret_cast<uint2*>(A16 + (size_t)m * K);
    const int n4 = K / 4;
    float4 v[V];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int idx = threadIdx.x + i * ACT_THREADS;
        v[i] = idx < n4 ? __ldg(row + idx) : make_float4(0.f, 0.f, 0.f, 0.f);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
#pragma unroll
    for (int w = 1; w < ACT_THREADS / 32; w++) amax = fmaxf(amax, red[w]);
    const float s = amax > 0.0f ? amax : 1.0f;
    const float inv = __frcp_rn(s);
    if (threadIdx.x == 0) scales[m] = s;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int idx = threadIdx.x + i * ACT_THREADS;
        if (idx < n4) {
            uint2 w;
            w.x = pack_half2(__fmul_rn(v[i].x, inv), __fmul_rn(v[i].y, inv));
            w.y = pack_half2(__fmul_rn(v[i].z, inv), __fmul_rn(v[i].w, inv));
            out[idx] = w;
        }
    }
}

// The dense FFN's SWIGLU fused into the down projection's activation pack: h = silu(gate) * up per
// element (ggml_swiglu_split, the glue kernel's arithmetic), then the sandwich of h's row, exactly as
// act_pack_kernel packs it -- so A16 and the scales equal SWIGLU followed by the pack, bit for bit,
// and h itself is never written. One 256-thread CTA per row, V float4 of gate and of up per thread.
template <int V>
__global__ void __launch_bounds__(ACT_THREADS) swiglu_act_pack_kernel(const float* __restrict__ gate, int64_t ldg,
                                                                      const float* __restrict__ up, int64_t ldu, int F,
                                                                      __half* __restrict__ A16, float* __restrict__ scales) {
    __shared__ float red[ACT_THREADS / 32];
    grid_dep_wait();     // programmatic launch: gate and up are the previous kernel's output
    grid_dep_launch();
    const int m = blockIdx.x;
    const float4* g4 = reinterpret_cast<const float4*>(gate + (size_t)m * ldg);
    const float4* u4 = reinterpret_cast<const float4*>(up + (size_t)m * ldu);
    uint2* out = reinterpret_cast<uint2*>(A16 + (size_t)m * F);
    const int n4 = F / 4;
    float4 v[V];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int idx = threadIdx.x + i * ACT_THREADS;
        if (idx < n4) {
            const float4 x = __ldg(g4 + idx), y = __ldg(u4 + idx);
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
    for (int w = 1; w < ACT_THREADS / 32; w++) amax = fmaxf(amax, red[w]);
    const float s = amax > 0.0f ? amax : 1.0f;
    const float inv = __frcp_rn(s);
    if (threadIdx.x == 0) scales[m] = s;
#pragma unroll
    for (int i = 0; i < V; i++) {
        const int idx = threadIdx.x + i * ACT_THREADS;
        if (idx < n4) {
            uint2 w;
            w.x = pack_half2(__fmul_rn(v[i].x, inv), __fmul_rn(v[i].y, inv));
            w.y = pack_half2(__fmul_rn(v[i].z, inv), __fmul_rn(v[i].w, inv));
            out[idx] = w;
        }
    }
}

// Rows too long (or too unaligned) for the register version: two passes with scalar loads.
__global__ void __launch_bounds__(ACT_THREADS) act_pack_loop_kernel(const float* __restrict__ A, int64_t lda, int K,
                                                                    __half* __restrict__ A16, float* __restrict__ scales) {
    __shared__ float red[ACT_THREADS / 32];
    grid_dep_wait();
    grid_dep_launch();
    const int m = blockIdx.x;
    const float* row = A + (size_t)m * lda;
    __half* out = A16 + (size_t)m * K;
    float amax = 0.0f;
    for (int i = threadIdx.x; i < K; i += ACT_THREADS) amax = fmaxf(amax, fabsf(__ldg(row + i)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int w = 1; w < ACT_THREADS / 32; w++) amax = fmaxf(amax, red[w]);
    const float s = amax > 0.0f ? amax : 1.0f;
    const float inv = __frcp_rn(s);
    if (threadIdx.x == 0) scales[m] = s;
    for (int i = threadIdx.x; i < K; i += ACT_THREADS) out[i] = __float2half_rn(__fmul_rn(__ldg(row + i), inv));
}

static cudaError_t launch_act_pack(const float* A, int64_t lda, int64_t M, int64_t K, __half* a16, float* scales,
                                   cudaStream_t st) {
    const bool vec = ((reinterpret_cast<uintptr_t>(A) & 15u) == 0) && (lda % 4 == 0) && (K % 4 == 0);
    const int64_t per = (K / 4 + ACT_THREADS - 1) / ACT_THREADS;   // float4 per thread
    const dim3 grid((unsigned)M), block(ACT_THREADS);
    const int k = (int)K;
    if (!vec || per > 16) return launch_pdl(act_pack_loop_kernel, grid, block, 0, st, A, lda, k, a16, scales);
    if (per <= 1) return launch_pdl(act_pack_kernel<1>, grid, block, 0, st, A, lda, k, a16, scales);
    if (per <= 2) return launch_pdl(act_pack_kernel<2>, grid, block, 0, st, A, lda, k, a16, scales);
    if (per <= 4) return launch_pdl(act_pack_kernel<4>, grid, block, 0, st, A, lda, k, a16, scales);
    if (per <= 8) return launch_pdl(act_pack_kernel<8>, grid, block, 0, st, A, lda, k, a16, scales);
    return launch_pdl(act_pack_kernel<16>, grid, block, 0, st, A, lda, k, a16, scales);
}

// ------------------------------------------------------------------------------------------
// Standalone dequant of native ggml rows (the K2d check kernel): one thread per element.
// ------------------------------------------------------------------------------------------
template <int WT, bool F16OUT>
__global__ void dequant_native_kernel(const uint8_t* __restrict__ src, int64_t row_bytes, int64_t N,
                                      int64_t K, void* __restrict__ dst) {
    const int64_t total = N * K;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / K;
        const int k = (int)(i % K);
        const uint8_t* row = src + n * row_bytes;
        float v;
        if constexpr (WT == WT_Q8_0) v = decode_native_elem_q8_0(row, k);
        else if constexpr (WT == WT_Q4_K) v = decode_native_elem_q4k(row, k);
        else if constexpr (WT == WT_Q6_K) v = decode_native_elem_q6k(row, k);
        else if constexpr (WT == WT_F16) v = __half2float(reinterpret_cast<const __half*>(row)[k]);
        else if constexpr (WT == WT_BF16) v = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(row)[k] << 16);
        else v = reinterpret_cast<const float*>(row)[k];
        if constexpr (F16OUT) reinterpret_cast<__half*>(dst)[i] = __float2half_rn(v);
        else reinterpret_cast<float*>(dst)[i] = v;
    }
}

// ------------------------------------------------------------------------------------------
// Native -> packed re-layout (the weight cache's device-resident format, quant.cuh).
// One thread per (row, 256-weight super-block).
// ------------------------------------------------------------------------------------------
__global__ void pack_q6k_kernel(const uint8_t* __restrict__ src, int64_t N, int64_t nsb,
                                uint8_t* __restrict__ dstA, uint16_t* __restrict__ dstD) {
    const int64_t total = N * nsb;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / nsb, sb = i % nsb;
        const uint8_t* b = src + i * 210;
        uint8_t* o = dstA + i * 208;
        for (int j = 0; j < 208; j++) o[j] = b[j];
        dstD[sb * N + n] = (uint16_t)(b[208] | (b[209] << 8));   // transposed: [sb][row]
    }
}

__global__ void pack_q8_0_kernel(const uint8_t* __restrict__ src, int64_t N, int64_t nblk, int64_t ngrp,
                                 uint8_t* __restrict__ dst) {
    // nblk native 32-weight blocks per row -> ngrp groups of 8 as {d[8], qs[256]} (zero-padded).
    const int64_t total = N * ngrp * 8;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t n = i / (ngrp * 8);
        const int64_t j = i % (ngrp * 8);
        uint8_t* g = dst + (n * ngrp + j / 8) * 272;
        uint8_t* od = g + 2 * (j % 8);
        uint8_t* oq = g + 16 + 32 * (j % 8);
        if (j < nblk) {
            const uint8_t* b = src + (n * nblk + j) * 34;
            od[0] = b[0];
            od[1] = b[1];
            for (int q = 0; q < 32; q++) oq[q] = b[2 + q];
        } else {
            od[0] = od[1] = 0;
            for (int q = 0; q < 32; q++) oq[q] = 0;
        }
    }
}

// ------------------------------------------------------------------------------------------
// Host side
// ------------------------------------------------------------------------------------------

int device_sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cached[dev] = v;
    }
    return cached[dev];
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// A 2-D fp16 tensor map [rows, cols] (cols innermost), row pitch in elements, box
// [box_rows, box_cols] with the 128-byte swizzle (box_cols * 2 == 128).
bool make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint32_t box_rows, uint32_t box_cols) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_elems * 2};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// A 2-D uint16 tensor map [rows, cols] (cols innermost, row pitch in bytes), box [box_rows,
// box_cols], no swizzle: the raw quantized tiles and the transposed d plane.
bool make_tmap_2d_u16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_bytes,
                             uint32_t box_rows, uint32_t box_cols) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The f32 output [rows, cols] (cols innermost, row pitch in bytes) as store boxes of 8 rows
// (tokens) x 32 columns (weight rows).
static bool make_tmap_2d_f32_out(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, uint64_t pitch_bytes) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {32, 8};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// The launch plan for one MUL_MAT: token tile and the stream-K granule split.
struct GemmPlan {
    int bt, gran, tile_g, nkb, ntn, ntt, grid, pieces;
    bool pair;                 // 2-SM MMA: CTA pairs over 256 weight rows (grid counts CTAs)
    bool csplit;               // cluster split: two CTAs per tile, one K half each (grid counts CTAs)
    int64_t tiles, total_g;
};

// CTA pairs (the 2-SM MMA) halve each SM's activation traffic. Measured on B200 they pay a few
// per cent for F16 weights at large M and cost the quantized path (whose decoded-weight hand-off
// then crosses the pair) a third of its speed, so by default only F16 with M >= 1024 uses them.
// B200_GEMM_PAIR: unset = that rule, 0 = never, 1 = whenever the token tile allows.
static int pair_knob() {
    static const int v = [] {
        const char* e = getenv("B200_GEMM_PAIR");
        return (e && *e) ? atoi(e) : -1;
    }();
    return v;
}

// B200_GEMM_TILE: unset = the cost model's token tile; 32 / 64 / 128 / 256 = that tile; 512 = the
// wide unit (Q4_K).
static int tile_knob() {
    static const int v = [] {
        const char* e = getenv("B200_GEMM_TILE");
        return (e && *e) ? atoi(e) : 0;
    }();
    return v;
}

// B200_GEMM_CSPLIT: unset = the cost model's choice; 0 = never; 1 = whenever the tiles fit on half
// the SMs (two CTAs of a cluster per tile, each one half of its K range).
static int csplit_knob() {
    static const int v = [] {
        const char* e = getenv("B200_GEMM_CSPLIT");
        return (e && *e) ? atoi(e) : -1;
    }();
    return v;
}

// B200_GEMM_STREAMK: unset / 1 = the cost model's choice; 0 = one whole tile per CTA whenever the
// tiles fit in one wave (no partials, idle SMs allowed); 2 = always stream-K over every SM.
static int streamk_knob() {
    static const int v = [] {
        const char* e = getenv("B200_GEMM_STREAMK");
        return (e && *e) ? atoi(e) : 1;
    }();
    return v;
}

// Whether the cluster split's receive and send regions fit in the idle operand stages of the
// kernel instance for this token tile and weight type.
template <int WT>
static bool csplit_fits_wt(int bt) {
    switch (bt) {
        case 32: return GemmCfg<32, WT, false>::CSPLIT_FITS;
        case 64: return GemmCfg<64, WT, false>::CSPLIT_FITS;
        case 128: return GemmCfg<128, WT, false>::CSPLIT_FITS;
        case 256: return GemmCfg<256, WT, false>::CSPLIT_FITS;
        default: return false;
    }
}
static bool csplit_fits(int bt, int wtype) {
    switch (wtype) {
        case WT_F16: return csplit_fits_wt<WT_F16>(bt);
        case WT_Q4_K: return csplit_fits_wt<WT_Q4_K>(bt);
        case WT_Q6_K: return csplit_fits_wt<WT_Q6_K>(bt);
        case WT_Q8_0: return csplit_fits_wt<WT_Q8_0>(bt);
        default: return false;
    }
}

// Choose the token tile from a cost model (SM clocks). Per 64-wide K block a tile costs the
// slowest of the tensor core (128 x BT x 64 MACs at 4096 MAC/clk), the decode of 8192 quantized
// weights by the dequant warps, and the L2 feed of its operand tiles. Stream-K spreads the
// tiles' K blocks evenly over the grid, so the time is the total over the grid plus a fixed
// cost per work item and, where tiles are shared, the partial-tile round trip.
static GemmPlan plan_gemm_knobs(int64_t M, int64_t N, int64_t K, int sms, int wtype, int tile, bool allow_pair) {
    const bool quant = wtype != WT_F16;
    const int nkb = (int)((K + GEMM_BK - 1) / GEMM_BK);
    const int gran = quant ? 4 : 1;
    const int tile_g = (nkb + gran - 1) / gran;
    GemmPlan best{};
    double best_t = 1e30;
    // 512: the wide unit (two 256-token halves on one decoded weight stage), Q4_K only
    const int bts[5] = {32, 64, 128, 256, 512};
    const int n_bts = wtype == WT_Q4_K ? 5 : 4;
    const bool pair_default = !quant && M >= 1024;
    for (int pair = 0; pair < 2; pair++) {
        if (pair && (!allow_pair || pair_knob() == 0 || (pair_knob() < 0 && !pair_default))) continue;
        if (!pair && allow_pair && (pair_knob() == 1 || (pair_knob() < 0 && pair_default)) && M > 64) continue;
        const int tile_n = pair ? 2 * GEMM_BN : GEMM_BN;
        const int ntn = (int)((N + tile_n - 1) / tile_n);
        for (int bi = 0; bi < n_bts; bi++) {
            const int bt = bts[bi];
            if (bi > 0 && bts[bi - 1] >= M) break;      // a smaller tile already covers M
            if (pair && (bt < 128 || bt > 256)) continue;   // each CTA of a pair stages 64..128 tokens
            if (tile > 0 && bt != tile) continue;
            // the wide unit holds one accumulator, so its epilogue never overlaps a main loop: measured
            // slower than 256-token tiles at M = 512 (a single 4096 x 14336 weight, and a layer's
            // combined gate/up launch: 37.1-37.6 k against 38.1-38.3 k prompt tokens/s), faster at
            // M = 2048 (217 against 232 us) -- left to the model only above M = 512 unless forced
            if (bt == 512 && M <= 512 && tile != 512) continue;
            const int ntt = (int)((M + bt - 1) / bt);
            const int64_t tiles = (int64_t)ntn * ntt;
            const int64_t total_g = tiles * tile_g;
            const int per_unit = pair ? 2 : 1;           // CTAs per work unit
            int units = (int)(total_g < sms / per_unit ? total_g : sms / per_unit);
            // per SM and 64-wide K block: tensor-core clocks (128 x BT x 64 MACs at 4096 MAC/clk),
            // the dequant warps' decode and hand-off of 8192 weights, and shared-memory bytes (TMA
            // writes + MMA reads, 128 B/clk): the activation tile is halved in a pair. The quantized
            // block times are measured on B200 at M = 512 (clock64 spans of the dequant warps, and
            // whole-launch times where the tile's epilogue adds to them): ~820-900 clocks at
            // BT <= 128, ~940 at 256, ~1450-1600 for the wide 512-token unit
            const double mma = bt < 64 ? 128.0 : 2.0 * bt;
            const double decode = !quant ? 0.0 : bt <= 128 ? 900.0 : bt == 256 ? 940.0 : 1600.0;
            const double a_bytes = (pair ? bt / 2 : bt) * 128.0 * 2.0;
            const double w_bytes = quant ? 41984.0 : 32768.0;
            const double feed = (a_bytes + w_bytes) / 128.0;
            double per_kb = mma > decode ? mma : decode;
            if (feed > per_kb) per_kb = feed;
            per_kb += 16.0;
            // a shared tile's partials: each piece but the last is written by its CTA, and the
            // finisher reads them all back after its own range (128 x BT f32 each at ~20 B/clk per
            // SM, measured): pieces_sk is how many CTAs share a tile under stream-K
            const int64_t run_sk = total_g / units > 0 ? total_g / units : 1;
            const double pieces_sk = (double)((tile_g - 1) / run_sk + 2 < tile_g ? (tile_g - 1) / run_sk + 2 : tile_g);
            const double part_sk = 25.6 * bt * pieces_sk;
            // whole tiles, one per CTA, when they fit in one wave: no partials
            const bool whole = tiles <= units && streamk_knob() != 2 && (streamk_knob() == 0 || (double)nkb * per_kb + 800.0 <
                (double)tiles * nkb * per_kb / units + 800.0 * (1.0 + (double)tiles / units) + part_sk);
            if (whole) units = (int)tiles;
            const double items = 1.0 + (double)tiles / units;
            const bool shared = total_g % units != 0 || tiles % units != 0;
            double t = (double)tiles * nkb * per_kb / units + 800.0 * items;
            if (shared) t += part_sk;
            // cluster split: when the tiles fit on half the SMs, two CTAs of a cluster take each tile,
            // one K half each, and add the halves over distributed shared memory (no partial round
            // trip through L2); measured on B200 at M = 512, N = 4096: 42 -> 27 us (K = 4096)
            bool csplit = false;
            if (!pair && csplit_fits(bt, wtype) && tile_g >= 2 && tiles * 2 <= sms && csplit_knob() != 0 &&
                streamk_knob() == 1) {
                const double t_cs = (double)((tile_g + 1) / 2) * gran * per_kb + 1600.0 + 12.8 * bt;
                if (csplit_knob() == 1 || t_cs < t) {
                    t = t_cs;
                    csplit = true;
                }
            }
            if (t < best_t * 0.97) {
                best_t = t;
                best.bt = bt;
                best.csplit = csplit;
                best.pair = pair != 0;
                best.gran = gran;
                best.tile_g = tile_g;
                best.nkb = nkb;
                best.ntn = ntn;
                best.ntt = ntt;
                best.grid = units * per_unit;
                best.tiles = tiles;
                best.total_g = total_g;
                const int64_t run = total_g / units;      // shortest granule run of a unit
                best.pieces = (int)((tile_g - 1) / run + 2 < tile_g ? (tile_g - 1) / run + 2 : tile_g);
                if (!shared) best.pieces = 1;
                if (csplit) {
                    best.pieces = 2;
                    best.grid = (int)(2 * tiles);
                }
            }
        }
    }
    return best;
}

// allow_pair = false for a combined-N launch, whose members' tiles are 128 weight rows each.
static GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int sms, int wtype, bool allow_pair = true) {
    GemmPlan p = plan_gemm_knobs(M, N, K, sms, wtype, tile_knob(), allow_pair);
    if (p.bt == 0) p = plan_gemm_knobs(M, N, K, sms, wtype, 0, allow_pair);   // the forced tile does not apply
    return p;
}

// Stream-K scratch: one partial tile per CTA, then four flags per CTA; none when every CTA
// owns whole tiles.
static size_t streamk_partials_bytes(const GemmPlan& p) { return (size_t)p.grid * p.bt * GEMM_BN * 4; }
static size_t streamk_bytes(const GemmPlan& p) {
    return p.pieces > 1 && !p.csplit ? streamk_partials_bytes(p) + (size_t)p.grid * 16 : 0;
}

// A value no earlier launch has published in the flags (0 is skipped, so zeroed memory never
// reads as published).
static uint32_t next_epoch() {
    static std::atomic<uint32_t> ctr{0x9e3779b9u};
    uint32_t e;
    do { e = ctr.fetch_add(1, std::memory_order_relaxed) + 1; } while (e == 0);
    return e;
}

struct MulMatWorkspace {
    size_t a16_off, scales_off, part_off, total;
};

static MulMatWorkspace mm_workspace_layout(int64_t M, int64_t N, int64_t K, const GemmPlan& p) {
    MulMatWorkspace w{};
    w.a16_off = 0;
    w.scales_off = align_up((size_t)M * K * 2, 256);
    w.part_off = align_up(w.scales_off + (size_t)M * 4, 256);
    w.total = w.part_off + streamk_bytes(p);
    return w;
}

template <int BT, int WT, bool GROUPED, bool PAIR>
static cudaError_t launch_gemm_t(const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmD,
                                 const CUtensorMap& tmO, const GemmArgs& a, const GemmMembers& mm, int grid,
                                 cudaStream_t st) {
    const bool cluster2 = PAIR || a.csplit == 2;
    using C = GemmCfg<BT, WT, PAIR>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BT, WT, GROUPED, PAIR>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    // Programmatic launch: the prologue (barriers, TMEM, descriptor prefetch) overlaps the tail of
    // the previous kernel. Stream-K finishers only ever wait for lower-numbered CTAs, which are
    // scheduled no later than themselves, so the grid needs no co-residency guarantee.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (cluster2) {
        // CTA pairs: clusters of two (the 2-SM MMA's peers, or the two K halves of a cluster split)
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, gemm_kernel<BT, WT, GROUPED, PAIR>, tmA, tmW, tmD, tmO, a, mm);
}

template <int WT, bool GROUPED>
static cudaError_t launch_gemm_bt(int bt, bool pair, const CUtensorMap& tmA, const CUtensorMap& tmW,
                                  const CUtensorMap& tmD, const CUtensorMap& tmO, const GemmArgs& a,
                                  const GemmMembers& mm, int grid, cudaStream_t st) {
    if constexpr (!GROUPED) {
        if (pair) {
            switch (bt) {
                case 128: return launch_gemm_t<128, WT, false, true>(tmA, tmW, tmD, tmO, a, mm, grid, st);
                case 256: return launch_gemm_t<256, WT, false, true>(tmA, tmW, tmD, tmO, a, mm, grid, st);
                default: return cudaErrorInvalidValue;
            }
        }
    }
    if constexpr (!GROUPED && WT == WT_Q4_K) {
        if (bt == 512) return launch_gemm_t<512, WT, false, false>(tmA, tmW, tmD, tmO, a, mm, grid, st);
    }
    switch (bt) {
        case 32: return launch_gemm_t<32, WT, GROUPED, false>(tmA, tmW, tmD, tmO, a, mm, grid, st);
        case 64: return launch_gemm_t<64, WT, GROUPED, false>(tmA, tmW, tmD, tmO, a, mm, grid, st);
        case 128: return launch_gemm_t<128, WT, GROUPED, false>(tmA, tmW, tmD, tmO, a, mm, grid, st);
        default: return launch_gemm_t<256, WT, GROUPED, false>(tmA, tmW, tmD, tmO, a, mm, grid, st);
    }
}

// Fill the weight-side tensor maps for `wrows` packed weight rows of K: the F16 weight tile
// (128-byte swizzled), or the raw quantized super-block tile and, for Q6_K, the d plane.
static bool setup_weight_maps(int wtype, const void* w_packed, int64_t wrows, int64_t K, CUtensorMap& tmW,
                              CUtensorMap& tmD, const CUtensorMap& tmA) {
    size_t d_off = 0;
    packed_weight_bytes(wtype, wrows, K, &d_off);
    tmD = tmA;   // unused unless Q6_K
    const uint8_t* base = static_cast<const uint8_t*>(w_packed);
    switch (wtype) {
        case WT_F16:
            return make_tmap_2d_f16(&tmW, w_packed, (uint64_t)wrows, (uint64_t)K, (uint64_t)K, GEMM_BN, GEMM_BK);
        case WT_Q4_K: {
            const uint64_t rb = (uint64_t)(K / 256) * 144;
            return make_tmap_2d_u16(&tmW, base, (uint64_t)wrows, rb / 2, rb, GEMM_BN, RawCfg<WT_Q4_K>::X_ELEMS);
        }
        case WT_Q6_K: {
            const uint64_t rb = (uint64_t)(K / 256) * 208;
            return make_tmap_2d_u16(&tmW, base, (uint64_t)wrows, rb / 2, rb, GEMM_BN, RawCfg<WT_Q6_K>::X_ELEMS) &&
                   make_tmap_2d_u16(&tmD, base + d_off, (uint64_t)(K / 256), (uint64_t)wrows, (uint64_t)wrows * 2, 1,
                                    GEMM_BN);
        }
        case WT_Q8_0: {
            const uint64_t rb = (uint64_t)((K + 255) / 256) * 272;
            return make_tmap_2d_u16(&tmW, base, (uint64_t)wrows, rb / 2, rb, GEMM_BN, RawCfg<WT_Q8_0>::X_ELEMS);
        }
        default:
            return false;
    }
}

bool make_weight_tile_maps(int wtype, const void* w_packed, int64_t wrows, int64_t K, CUtensorMap* tmW,
                           CUtensorMap* tmD) {
    if (wtype != WT_Q4_K && wtype != WT_Q6_K && wtype != WT_Q8_0) return false;
    const CUtensorMap none{};
    return setup_weight_maps(wtype, w_packed, wrows, K, *tmW, *tmD, none);
}

template <bool GROUPED>
cudaError_t launch_gemm_typed(int wtype, int bt, bool pair, const CUtensorMap& tmA, const CUtensorMap& tmW,
                              const CUtensorMap& tmD, const CUtensorMap& tmO, const GemmArgs& a, int grid, cudaStream_t st,
                              const GemmMembers* members = nullptr) {
    static const GemmMembers none{};
    const GemmMembers& mm = members ? *members : none;
    switch (wtype) {
        case WT_F16: return launch_gemm_bt<WT_F16, GROUPED>(bt, pair, tmA, tmW, tmD, tmO, a, mm, grid, st);
        case WT_Q4_K: return launch_gemm_bt<WT_Q4_K, GROUPED>(bt, pair, tmA, tmW, tmD, tmO, a, mm, grid, st);
        case WT_Q6_K: return launch_gemm_bt<WT_Q6_K, GROUPED>(bt, pair, tmA, tmW, tmD, tmO, a, mm, grid, st);
        case WT_Q8_0: return launch_gemm_bt<WT_Q8_0, GROUPED>(bt, pair, tmA, tmW, tmD, tmO, a, mm, grid, st);
        default: return cudaErrorInvalidValue;
    }
}

// The grouped (MUL_MAT_ID) launch: A16 holds `rows` expert-sorted token rows; the route arrays
// live on the device (see moe.cu).
int gemm_grouped_impl(int wtype, const void* w_stack, int64_t N, int64_t K, int64_t n_expert, const __half* a16,
                      const float* scales, int64_t rows, int bt, const int32_t* off, const int32_t* tile_start,
                      const int32_t* slot, const int32_t* tok, float* dst, int64_t d_nb1, int64_t d_nb2, int* dev_err,
                      cudaStream_t st, const int32_t* src, float* const* dst_bases) {
    // dst_bases (a device array) replaces dst when rows go to several buffers
    if ((d_nb1 % 16) || (d_nb2 % 16) || (!dst_bases && (!dst || (reinterpret_cast<uintptr_t>(dst) & 15u))))
        return B200_E_UNSUPPORTED;
    CUtensorMap tmA, tmW, tmD;
    if (!make_tmap_2d_f16(&tmA, a16, (uint64_t)rows, (uint64_t)K, (uint64_t)K, (uint32_t)bt, GEMM_BK)) return B200_E_CUDA;
    GemmArgs a{};
    if (!setup_weight_maps(wtype, w_stack, N * n_expert, K, tmW, tmD, tmA)) return B200_E_CUDA;
    a.scales = scales;
    a.out = dst;
    a.M = (int)rows;
    a.N = (int)N;
    a.K = (int)K;
    a.n_tiles_n = (int)((N + GEMM_BN - 1) / GEMM_BN);
    a.n_tiles_t = 1;
    a.nkb = (int)((K + GEMM_BK - 1) / GEMM_BK);
    a.err = dev_err;
    a.g_off = off;
    a.g_tile_start = tile_start;
    a.g_slot = slot;
    a.g_tok = tok;
    a.n_expert = (int)n_expert;
    a.d_nb1 = d_nb1;
    a.d_nb2 = d_nb2;
    a.g_src = src;
    a.out_bases = dst_bases;
    const int sms = device_sm_count();
    const int64_t max_tiles = (rows + bt - 1) / bt + n_expert;
    const int64_t max_units = max_tiles * a.n_tiles_n;
    const int grid = (int)(max_units < sms ? max_units : sms);
    if (grid <= 0) return B200_OK;
    return launch_gemm_typed<true>(wtype, bt, false, tmA, tmW, tmD, tmA, a, grid, st) == cudaSuccess ? B200_OK : B200_E_CUDA;
}

size_t packed_weight_bytes(int type, int64_t N, int64_t K, size_t* plane_d_off) {
    size_t off = 0, total = 0;
    switch (type) {
        case WT_F16: total = (size_t)N * K * 2; break;
        case WT_Q4_K: total = (size_t)N * (K / 256) * 144; break;
        case WT_Q6_K:
            off = align_up((size_t)N * (K / 256) * 208, 256);
            total = off + (size_t)N * (K / 256) * 2;
            break;
        case WT_Q8_0:
            total = (size_t)N * ((K + 255) / 256) * 272;
            break;
        default: return 0;
    }
    if (plane_d_off) *plane_d_off = off;
    return total;
}

bool weight_type_supported(int type, int64_t K) {
    switch (type) {
        case WT_F16: return K % 8 == 0;
        case WT_Q8_0: return K % 32 == 0;
        case WT_Q4_K:
        case WT_Q6_K: return K % 256 == 0;
        default: return false;
    }
}

// The tcgen05 GEMM over an already packed activation (A16 [M,K] fp16 + per-row scales). With
// dst_bases (a device array of n_dst pointers) the output columns [col0, col0 + N) go to every
// one of those [M][ldd] buffers instead of dst (the weight rows split across GPUs).
int gemm_packed_impl(int wtype, const void* w_packed, int64_t N, int64_t K, const __half* a16, const float* scales,
                     int64_t M, float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err,
                     cudaStream_t st, float* const* dst_bases, int n_dst, int64_t col0) {
    if (!w_packed || !a16 || !scales || !(dst || (dst_bases && n_dst > 0)) || !dev_err || M <= 0 || N <= 0 || K <= 0)
        return B200_E_INVALID;
    if (!weight_type_supported(wtype, K) || K % 32 != 0 || N % 16 != 0) return B200_E_UNSUPPORTED;
    // the epilogue writes 16-byte vectors of dst rows
    if (ldd % 4 != 0 || (dst && (reinterpret_cast<uintptr_t>(dst) & 15u)) || col0 % 16 != 0 || n_dst > 64)
        return B200_E_UNSUPPORTED;
    if (M > (1 << 30) || N > (1 << 30) || K > (1 << 30)) return B200_E_UNSUPPORTED;
    const int sms = device_sm_count();
    const GemmPlan p = plan_gemm(M, N, K, sms, wtype);
    const size_t sk_bytes = streamk_bytes(p);
    // the cluster split receives into its CTAs' idle operand stages: one tile per cluster
    if (p.csplit && ((int64_t)p.grid != 2 * p.tiles || !csplit_fits(p.bt, wtype))) return B200_E_INVALID;
    if (sk_bytes && (!workspace || workspace_bytes < sk_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u)))
        return B200_E_WORKSPACE;
    CUtensorMap tmA, tmW, tmD;
    // the activation box: a CTA of a pair stages half of the token tile; the wide tile two boxes
    const uint32_t a_box = (uint32_t)(p.pair ? p.bt / 2 : (p.bt > 256 ? 256 : p.bt));
    if (!make_tmap_2d_f16(&tmA, a16, (uint64_t)M, (uint64_t)K, (uint64_t)K, a_box, GEMM_BK))
        return B200_E_CUDA;
    GemmArgs a{};
    if (!setup_weight_maps(wtype, w_packed, N, K, tmW, tmD, tmA)) return B200_E_CUDA;
    a.scales = scales;
    a.out = dst;
    a.ldo = ldd;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.n_tiles_n = p.ntn;
    a.n_tiles_t = p.ntt;
    a.nkb = p.nkb;
    a.err = dev_err;
    a.partials = sk_bytes ? static_cast<float*>(workspace) : nullptr;
    a.flags = sk_bytes ? reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + streamk_partials_bytes(p))
                       : nullptr;
    a.epoch = next_epoch();
    a.gran = p.gran;
    a.tile_g = p.tile_g;
    a.total_g = p.total_g;
    a.out_bases = n_dst > 0 ? dst_bases : nullptr;
    a.n_dst = n_dst > 0 ? n_dst : 0;
    a.col0 = (int)col0;
    a.csplit = p.csplit ? 2 : 0;
    CUtensorMap tmO = tmA;   // unused with several destinations
    if (n_dst <= 0 && !make_tmap_2d_f32_out(&tmO, dst, (uint64_t)M, (uint64_t)N, (uint64_t)ldd * 4)) return B200_E_CUDA;
    const cudaError_t e = launch_gemm_typed<false>(wtype, p.bt, p.pair, tmA, tmW, tmD, tmO, a, p.grid, st);
    return e == cudaSuccess ? B200_OK : B200_E_CUDA;
}

// The combined-N GEMM of a fused group (the reference's _mul_mat_group, ggml-rocket.cpp:4956-5020:
// one GEMM over the members' weights laid side by side, each member's columns unpacked into its
// own dst). Here the members' 128-row weight tiles are numbered end to end and one persistent
// launch takes them all under one schedule, so the group pays one launch's start and one tail
// instead of one per member; every tile reads its member's weight and writes its member's dst
// through that member's tensor maps. Weights of one type and K; no CTA pairs.
static int64_t group_n_padded(int n, const int64_t* N) {
    int64_t s = 0;
    for (int m = 0; m < n; m++) s += (N[m] + GEMM_BN - 1) / GEMM_BN * GEMM_BN;
    return s;
}

size_t gemm_packed_group_workspace(int n, int wtype, int64_t M, const int64_t* N, int64_t K) {
    if (n <= 0 || n > GEMM_MAX_MEMBERS || !N || M <= 0 || K <= 0) return 0;
    return streamk_bytes(plan_gemm(M, group_n_padded(n, N), K, device_sm_count(), wtype, false));
}

int gemm_packed_group_impl(int n, int wtype, const void* const* w_packed, const int64_t* N, int64_t K,
                           const __half* a16, const float* scales, int64_t M, float* const* dst, const int64_t* ldd,
                           void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t st) {
    if (n <= 0 || n > GEMM_MAX_MEMBERS || !w_packed || !N || !dst || !ldd || !a16 || !scales || !dev_err || M <= 0 ||
        K <= 0)
        return B200_E_INVALID;
    if (!weight_type_supported(wtype, K) || K % 32 != 0 || M > (1 << 30) || K > (1 << 30)) return B200_E_UNSUPPORTED;
    for (int m = 0; m < n; m++) {
        if (!w_packed[m] || !dst[m] || N[m] <= 0) return B200_E_INVALID;
        if (N[m] % 16 != 0 || N[m] > (1 << 30) || ldd[m] % 4 != 0 || (reinterpret_cast<uintptr_t>(dst[m]) & 15u))
            return B200_E_UNSUPPORTED;
    }
    const int64_t n_all = group_n_padded(n, N);
    if (n_all > (1 << 30)) return B200_E_UNSUPPORTED;
    const GemmPlan p = plan_gemm(M, n_all, K, device_sm_count(), wtype, false);
    const size_t sk_bytes = streamk_bytes(p);
    if (p.pair || (p.csplit && ((int64_t)p.grid != 2 * p.tiles || !csplit_fits(p.bt, wtype)))) return B200_E_INVALID;
    if (sk_bytes && (!workspace || workspace_bytes < sk_bytes || (reinterpret_cast<uintptr_t>(workspace) & 255u)))
        return B200_E_WORKSPACE;
    CUtensorMap tmA, tmW, tmD, tmO;
    const uint32_t a_box = (uint32_t)(p.bt > 256 ? 256 : p.bt);
    if (!make_tmap_2d_f16(&tmA, a16, (uint64_t)M, (uint64_t)K, (uint64_t)K, a_box, GEMM_BK)) return B200_E_CUDA;
    GemmMembers mm{};
    GemmArgs a{};
    int t0 = 0;
    for (int m = 0; m < n; m++) {
        CUtensorMap& w = m == 0 ? tmW : mm.w[m - 1];
        CUtensorMap& d = m == 0 ? tmD : mm.d[m - 1];
        CUtensorMap& o = m == 0 ? tmO : mm.o[m - 1];
        if (!setup_weight_maps(wtype, w_packed[m], N[m], K, w, d, tmA)) return B200_E_CUDA;
        if (!make_tmap_2d_f32_out(&o, dst[m], (uint64_t)M, (uint64_t)N[m], (uint64_t)ldd[m] * 4)) return B200_E_CUDA;
        a.mem_t0[m] = t0;
        t0 += (int)((N[m] + GEMM_BN - 1) / GEMM_BN);
    }
    a.n_mem = n;
    a.scales = scales;
    a.out = dst[0];
    a.ldo = ldd[0];
    a.M = (int)M;
    a.N = (int)n_all;
    a.K = (int)K;
    a.n_tiles_n = p.ntn;
    a.n_tiles_t = p.ntt;
    a.nkb = p.nkb;
    a.err = dev_err;
    a.partials = sk_bytes ? static_cast<float*>(workspace) : nullptr;
    a.flags = sk_bytes ? reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + streamk_partials_bytes(p))
                       : nullptr;
    a.epoch = next_epoch();
    a.gran = p.gran;
    a.tile_g = p.tile_g;
    a.total_g = p.total_g;
    a.csplit = p.csplit ? 2 : 0;
    const cudaError_t e = launch_gemm_typed<false>(wtype, p.bt, false, tmA, tmW, tmD, tmO, a, p.grid, st, &mm);
    return e == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int swiglu_act_pack_impl(const float* gate, int64_t ldg, const float* up, int64_t ldu, int64_t M, int64_t F,
                         __half* a16, float* scales, cudaStream_t st) {
    if (!gate || !up || !a16 || !scales || M <= 0 || F <= 0 || ldg < F || ldu < F) return B200_E_INVALID;
    // rows of 16-byte vectors held in registers: F % 4 == 0, aligned rows, F <= 16 float4 per thread
    const bool vec = F % 4 == 0 && ldg % 4 == 0 && ldu % 4 == 0 && (reinterpret_cast<uintptr_t>(gate) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(up) & 15u) == 0;
    const int64_t per = (F / 4 + ACT_THREADS - 1) / ACT_THREADS;
    if (!vec || per > 16 || M > INT32_MAX) return B200_E_UNSUPPORTED;
    const dim3 grid((unsigned)M), block(ACT_THREADS);
    const int f = (int)F;
    cudaError_t e;
    if (per <= 4) e = launch_pdl(swiglu_act_pack_kernel<4>, grid, block, 0, st, gate, ldg, up, ldu, f, a16, scales);
    else if (per <= 8) e = launch_pdl(swiglu_act_pack_kernel<8>, grid, block, 0, st, gate, ldg, up, ldu, f, a16, scales);
    else e = launch_pdl(swiglu_act_pack_kernel<16>, grid, block, 0, st, gate, ldg, up, ldu, f, a16, scales);
    return e == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int act_pack_impl(const float* src1, int64_t lda, int64_t M, int64_t K, __half* a16, float* scales, cudaStream_t st) {
    if (!src1 || !a16 || !scales || M <= 0 || K <= 0 || lda < K) return B200_E_INVALID;
    return launch_act_pack(src1, lda, M, K, a16, scales, st) == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int mul_mat_impl(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda, int64_t M,
                 float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t st,
                 float* const* dst_bases, int n_dst, int64_t col0) {
    if (!w_packed || !src1 || !(dst || (dst_bases && n_dst > 0)) || !dev_err || M <= 0 || N <= 0 || K <= 0)
        return B200_E_INVALID;
    const GemmPlan p = plan_gemm(M, N, K, device_sm_count(), wtype);
    const MulMatWorkspace wl = mm_workspace_layout(M, N, K, p);
    if (!workspace || workspace_bytes < wl.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return B200_E_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __half* a16 = reinterpret_cast<__half*>(ws + wl.a16_off);
    float* scales = reinterpret_cast<float*>(ws + wl.scales_off);
    int rc = act_pack_impl(src1, lda, M, K, a16, scales, st);
    if (rc != B200_OK) return rc;
    return gemm_packed_impl(wtype, w_packed, N, K, a16, scales, M, dst, ldd, ws + wl.part_off, wl.total - wl.part_off,
                            dev_err, st, dst_bases, n_dst, col0);
}

size_t mul_mat_workspace(int wtype, int64_t M, int64_t N, int64_t K) {
    const GemmPlan p = plan_gemm(M, N, K, device_sm_count(), wtype);
    return mm_workspace_layout(M, N, K, p).total;
}

void mul_mat_flags_range(int wtype, int64_t M, int64_t N, int64_t K, size_t* offset, size_t* bytes) {
    const GemmPlan p = plan_gemm(M, N, K, device_sm_count(), wtype);
    const MulMatWorkspace wl = mm_workspace_layout(M, N, K, p);
    const size_t sk = streamk_bytes(p);
    *offset = sk ? wl.part_off + streamk_partials_bytes(p) : 0;
    *bytes = sk ? sk - streamk_partials_bytes(p) : 0;
}

int weight_pack_impl(int type, const void* src, int64_t N, int64_t K, void* dst, cudaStream_t st) {
    if (!src || !dst || N <= 0 || K <= 0) return B200_E_INVALID;
    if (!weight_type_supported(type, K)) return B200_E_UNSUPPORTED;
    size_t d_off = 0;
    const size_t bytes = packed_weight_bytes(type, N, K, &d_off);
    if (type == WT_F16 || type == WT_Q4_K) {
        if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st) != cudaSuccess) return B200_E_CUDA;
        return B200_OK;
    }
    uint8_t* dA = static_cast<uint8_t*>(dst);
    uint16_t* dD = reinterpret_cast<uint16_t*>(dA + d_off);
    if (type == WT_Q6_K) {
        const int64_t nsb = K / 256;
        const int64_t total = N * nsb;
        int blocks = (int)((total + 255) / 256);
        if (blocks > 65535) blocks = 65535;
        pack_q6k_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint8_t*>(src), N, nsb, dA, dD);
    } else {
        const int64_t nblk = K / 32, ngrp = (K + 255) / 256;
        const int64_t total = N * ngrp * 8;
        int blocks = (int)((total + 255) / 256);
        if (blocks > 65535) blocks = 65535;
        pack_q8_0_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint8_t*>(src), N, nblk, ngrp, dA);
    }
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

int dequantize_impl(int type, const void* src, int64_t N, int64_t K, int f16_out, void* dst, cudaStream_t st) {
    if (!src || !dst || N <= 0 || K <= 0) return B200_E_INVALID;
    if (K % wt_block_elems(type)) return B200_E_UNSUPPORTED;
    const int64_t row_bytes = (K / wt_block_elems(type)) * wt_block_bytes(type);
    const int64_t total = N * K;
    int blocks = (int)((total + 255) / 256);
    if (blocks > device_sm_count() * 16) blocks = device_sm_count() * 16;
    const uint8_t* s = static_cast<const uint8_t*>(src);
#define B200_DQ(T)                                                                                 \
    if (f16_out) dequant_native_kernel<T, true><<<blocks, 256, 0, st>>>(s, row_bytes, N, K, dst); \
    else dequant_native_kernel<T, false><<<blocks, 256, 0, st>>>(s, row_bytes, N, K, dst);
    switch (type) {
        case WT_Q8_0: B200_DQ(WT_Q8_0); break;
        case WT_Q4_K: B200_DQ(WT_Q4_K); break;
        case WT_Q6_K: B200_DQ(WT_Q6_K); break;
        case WT_F16: B200_DQ(WT_F16); break;
        case WT_BF16: B200_DQ(WT_BF16); break;
        case WT_F32: B200_DQ(WT_F32); break;
        default: return B200_E_UNSUPPORTED;
    }
#undef B200_DQ
    return cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // namespace b200

// ------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------
extern "C" {

size_t b200_weight_packed_size(int type, int64_t N, int64_t K) {
    if (!b200::weight_type_supported(type, K) || N <= 0) return 0;
    return b200::packed_weight_bytes(type, N, K, nullptr);
}

int b200_weight_pack(int type, const void* src_native, int64_t N, int64_t K, void* dst_packed, void* stream) {
    return b200::weight_pack_impl(type, src_native, N, K, dst_packed, static_cast<cudaStream_t>(stream));
}

int b200_dequantize(int type, const void* src_native, int64_t N, int64_t K, int f16_out, void* dst, void* stream) {
    return b200::dequantize_impl(type, src_native, N, K, f16_out, dst, static_cast<cudaStream_t>(stream));
}

int b200_act_pack(const float* src1, int64_t lda, int64_t M, int64_t K, void* a16, float* scales, void* stream) {
    return b200::act_pack_impl(src1, lda, M, K, static_cast<__half*>(a16), scales, static_cast<cudaStream_t>(stream));
}

int b200_swiglu_act_pack(const float* gate, int64_t ldg, const float* up, int64_t ldu, int64_t M, int64_t F, void* a16,
                         float* scales, void* stream) {
    return b200::swiglu_act_pack_impl(gate, ldg, up, ldu, M, F, static_cast<__half*>(a16), scales,
                                      static_cast<cudaStream_t>(stream));
}

size_t b200_gemm_packed_workspace_size(int wtype, int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return b200::streamk_bytes(b200::plan_gemm(M, N, K, b200::device_sm_count(), wtype));
}

int b200_gemm_packed(int wtype, const void* w_packed, int64_t N, int64_t K, const void* a16, const float* scales,
                     int64_t M, float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err,
                     void* stream) {
    return b200::gemm_packed_impl(wtype, w_packed, N, K, static_cast<const __half*>(a16), scales, M, dst, ldd,
                                  workspace, workspace_bytes, dev_err, static_cast<cudaStream_t>(stream));
}

size_t b200_gemm_packed_group_workspace_size(int n_members, int wtype, int64_t M, const int64_t* N, int64_t K) {
    return b200::gemm_packed_group_workspace(n_members, wtype, M, N, K);
}

int b200_gemm_packed_group(int n_members, int wtype, const void* const* w_packed, const int64_t* N, int64_t K,
                           const void* a16, const float* scales, int64_t M, float* const* dst, const int64_t* ldd,
                           void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    return b200::gemm_packed_group_impl(n_members, wtype, w_packed, N, K, static_cast<const __half*>(a16), scales, M,
                                        dst, ldd, workspace, workspace_bytes, dev_err,
                                        static_cast<cudaStream_t>(stream));
}

int b200_gemm_packed_group_plan(int n_members, int wtype, int64_t M, const int64_t* N, int64_t K, int* token_tile,
                                int* splits, int* grid) {
    if (n_members <= 0 || n_members > b200::GEMM_MAX_MEMBERS || !N || M <= 0 || K <= 0) return B200_E_INVALID;
    const b200::GemmPlan p =
        b200::plan_gemm(M, b200::group_n_padded(n_members, N), K, b200::device_sm_count(), wtype, false);
    if (token_tile) *token_tile = p.bt;
    if (splits) *splits = p.pieces;
    if (grid) *grid = p.grid;
    return B200_OK;
}

int b200_mul_mat_plan(int wtype, int64_t M, int64_t N, int64_t K, int* token_tile, int* splits, int* grid,
                      int* launches) {
    if (M <= 0 || N <= 0 || K <= 0) return B200_E_INVALID;
    const b200::GemmPlan p = b200::plan_gemm(M, N, K, b200::device_sm_count(), wtype);
    if (token_tile) *token_tile = p.bt;
    if (splits) *splits = p.pieces;
    if (grid) *grid = p.grid;
    if (launches) *launches = 2;
    return B200_OK;
}

size_t b200_mul_mat_workspace_size(int wtype, int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return b200::mul_mat_workspace(wtype, M, N, K);
}

int b200_mul_mat(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda, int64_t M,
                 float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    return b200::mul_mat_impl(wtype, w_packed, N, K, src1, lda, M, dst, ldd, workspace, workspace_bytes, dev_err,
                              static_cast<cudaStream_t>(stream));
}

}  // extern "C"
