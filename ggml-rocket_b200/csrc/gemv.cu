// Decode-size MUL_MAT (b200_mul_mat_vec). This file holds the row-block kernels for Q4_K weights
// at M = 1..8 token rows, the case they stream fastest; every other weight type (Q6_K, Q8_0) and
// row count (up to 32) runs on the tiled kernel of gemv_tiles.cu, behind the same entry point.
// Both are weight-streaming kernels whose dot products run on the warp-level tensor-core MMA, for
// the shapes the tcgen05 GEMM's 128-row tiles cannot fill.
//
// dst[m, n] = sum_k a[m, k] * W[n, k], W the packed (native) Q4_K rows. With M this small the op
// is bound by reading W once from HBM; on the CUDA cores alone a 4-bit weight costs more issue
// slots (nibble -> float, one FMA per token row) than the SM has at HBM speed, so:
//   * weights are decoded straight into mma.sync m16n8k16 A fragments as fp16 integers q*sc
//     (the 6-bit sub-block scale folded in: (1024 + q) * sc - 1024 * sc in one fused f16x2 FMA,
//     exact since q*sc <= 945), nine instructions per 8 weights and no shared-memory round trip
//     of decoded values; one MMA then serves all 8 token rows;
//   * the sub-block minimum term dmin * sum_j m_j * sum(a over sub-block j) is one more MMA per
//     super-block, with the activation sums split into fp16 (hi, lo) pairs;
//   * per super-block: acc += s * (d * C - dmin * Cmin) in fp32, s the activation block scale;
//   * work schedules (B200_GEMV_SCHEDULE; "tiles" sends this case to gemv_tiles.cu too): "rows"
//     (default), one CTA per 16 weight rows whose
//     8 warps split the super-blocks into contiguous ranges, each streaming its 16 x 144-byte
//     super-block columns through a 4-deep cp.async ring, partials added in warp order; and
//     "stream", a one-wave grid whose warps each take an equal contiguous range of the whole
//     weight through a 4-stage TMA ring, row blocks shared by two warps finished by the last to
//     arrive. Both add partials in a fixed order: results do not depend on timing.
// The activations are prepared once per call by gemv_act_kernel: per 256-value block, the
// block's absmax s and fp16(a / s) (the same per-row "sandwich" rule the GEMM's activation pack
// applies, here per block), stored in the MMA's k-slot order, plus the fp16 (hi, lo) sums of
// every 32-value sub-block.
//
// Numerics: weights are the exact Q4_K values (d*sc*q - dmin*m, from exact integer products and
// fp32 scales); products with the fp16 activations are exact in the MMA and summed in fp32. The
// only rounding beyond fp32 sums is the activations' fp16 rounding, as in the prefill GEMM.
// The decode is ggml's dequantize_row_q4_K (ggml-rocket.cpp:3894-3907 calls it through to_float).
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"

namespace b200 {

constexpr int GV_WARPS = 8;                      // warps per CTA
constexpr int GV_ROWS = 16;                      // weight rows per CTA (the MMA's M)
constexpr int GV_STAGES = 4;                     // TMA stages (units) in flight per warp
constexpr int GV_STAGE = GV_ROWS * 144;          // one unit: a super-block column of 16 rows, bytes
constexpr int GV_PIECES = GV_STAGE / 16;         // 16-byte cp.async copies per stage (rows schedule)
constexpr int GV_SMEM = GV_WARPS * GV_STAGES * GV_STAGE;                              // stream schedule
constexpr int GV_SMEM_ROWS = GV_WARPS * GV_STAGES * GV_STAGE + GV_WARPS * GV_ROWS * 8 * 4;   // + reduction
constexpr int GV_MMAX = 8;                       // token rows per call (the MMA's N)

// ---- small PTX helpers ---------------------------------------------------------------------

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));   // (a & b) | c
    return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// D += A(16x16, row) * B(16x8, col), fp16 operands, fp32 accumulators.
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// ---- activation prep -----------------------------------------------------------------------

// One warp per (token row m, super-block column sb); lane l holds values 8l .. 8l+7 of the block.
//   scl[sb * 8 + m]                  s = absmax of the 256 values (1 when all are zero); token
//                                    rows M..7 get 0
//   a16p[m * K + 256 sb + 8l ...]    fp16(a / s), each group of four stored as (x0, x2, x1, x3):
//                                    the order in which a Q4_K word's nibbles reach the MMA's
//                                    k slots
//   asum2[m * K/32 + 8 sb + j]       fp16 pair (hi, lo), hi + lo = the fp32 sum of sub-block j's
//                                    32 fp16 values to ~22 bits
// and zeroes the n_cnt arrival counters of the weight-streaming kernel that follows.
template <bool VEC>
__global__ void __launch_bounds__(256) gemv_act_kernel(const float* __restrict__ a, int64_t lda, int M, int K,
                                                       __half* __restrict__ a16p, uint32_t* __restrict__ asum2,
                                                       float* __restrict__ scl, uint32_t* __restrict__ cnt,
                                                       int64_t n_cnt) {
    grid_dep_wait();   // the previous kernel may still read this workspace (programmatic launch)
    grid_dep_launch();
    // the weight-streaming kernel's arrival counters start at zero
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_cnt; i += (int64_t)gridDim.x * blockDim.x)
        cnt[i] = 0u;
    const int nsb = K / 256;
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= M * nsb) return;
    const int m = gw / nsb, sb = gw % nsb;
    const int k = sb * 256 + 8 * lane;
    const float* p = a + (int64_t)m * lda + k;
    float x[8];
    if constexpr (VEC) {
        const float4 u = __ldg(reinterpret_cast<const float4*>(p));
        const float4 v = __ldg(reinterpret_cast<const float4*>(p + 4));
        x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = v.x, x[5] = v.y, x[6] = v.z, x[7] = v.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++) x[i] = __ldg(p + i);
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = amax > 0.0f ? amax : 1.0f;
    const float inv = __frcp_rn(s);
    __half h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __float2half_rn(__fmul_rn(x[i], inv));
    auto pk = [](__half lo, __half hi) {
        return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
    };
    *reinterpret_cast<uint4*>(a16p + (int64_t)m * K + k) =
        make_uint4(pk(h[0], h[2]), pk(h[1], h[3]), pk(h[4], h[6]), pk(h[5], h[7]));
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) sum += __half2float(h[i]);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((lane & 3) == 0) {
        const __half hi = __float2half_rn(sum);
        const __half lo = __float2half_rn(sum - __half2float(hi));
        asum2[(int64_t)m * (K / 32) + sb * 8 + (lane >> 2)] = pk(hi, lo);
    }
    if (lane == 0) {
        scl[sb * GV_MMAX + m] = s;
        if (m == 0)
            for (int mm = M; mm < GV_MMAX; mm++) scl[sb * GV_MMAX + mm] = 0.0f;
    }
}

// ---- the weight-streaming kernel -------------------------------------------------------------

// Scale constants of one weight row for this lane's two sub-blocks of a super-block (2t: the low
// nibbles of qs chunk t, 2t+1: its high nibbles), from the row's 16-byte header {d, dmin,
// scales[12]}. The 6-bit sc / m values are ggml's get_scale_min_k4 (t >= 2 takes the j >= 4
// form), moved into f16x2 pairs by a byte permute onto 0x64 (1024 + v, then - 1024).
struct GvRowScales {
    uint32_t mul_lo, add_lo, mul_hi, add_hi, m_lo, m_hi;   // f16x2 pairs
    float d, dmin;
};
__device__ __forceinline__ GvRowScales gv_row_scales(const uint4 h, bool upper, uint32_t sel0, uint32_t sel1) {
    const uint32_t scw = upper ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
    const uint32_t mw = upper ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
    const uint32_t H1024 = 0x64006400u;
    const uint32_t sc0 = hsub2(prmt(scw, 0x64646464u, sel0), H1024);   // (sc_2t, sc_2t)
    const uint32_t sc1 = hsub2(prmt(scw, 0x64646464u, sel1), H1024);   // (sc_2t+1, sc_2t+1)
    GvRowScales r;
    r.mul_lo = sc0;
    r.add_lo = hmul2(sc0, 0xE400E400u);    // -1024 sc: (1024 + q) sc - 1024 sc = q sc
    r.mul_hi = hmul2(sc1, 0x2C002C00u);    // sc / 16:  (1024 + 16 q) sc / 16 - 64 sc = q sc
    r.add_hi = hmul2(sc1, 0xD400D400u);    // -64 sc
    r.m_lo = hsub2(prmt(mw, 0x64646464u, sel0), H1024);
    r.m_hi = hsub2(prmt(mw, 0x64646464u, sel1), H1024);
    r.d = h2f_bits(h.x);
    r.dmin = h2f_bits(h.x >> 16);
    return r;
}


// The "rows" schedule: CTA = 16 weight rows n0 .. n0+15, one CTA per row block (several waves);
// warp w takes super-block columns [w nsb / 8, (w+1) nsb / 8), streamed through a 4-deep cp.async
// ring of its own, and the warps' partials are added in warp order in shared memory.
// Lane (g, t) = (lane / 4, lane % 4) is the MMA's thread group g, thread t: it decodes qs chunk t
// (bytes 32t .. 32t+31) of rows n0+g and n0+g+8 and feeds token row g's activations; its
// accumulators are rows n0+g, n0+g+8 x token rows 2t, 2t+1.
__global__ void __launch_bounds__(32 * GV_WARPS, 2)
    gemv_q4k_rows_kernel(const uint8_t* __restrict__ w, int64_t N, int K, const __half* __restrict__ a16p,
                    const uint32_t* __restrict__ asum2, const float* __restrict__ scl, int M, float* __restrict__ dst,
                    int64_t ldd) {
    extern __shared__ __align__(128) uint8_t gv_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nsb = K / 256;
    const int64_t row_bytes = (int64_t)nsb * 144;
    const int64_t n0 = (int64_t)blockIdx.x * GV_ROWS;
    const int sb0 = (int)((int64_t)warp * nsb / GV_WARPS), sb1 = (int)((int64_t)(warp + 1) * nsb / GV_WARPS);
    uint8_t* ring = gv_smem + warp * (GV_STAGES * GV_STAGE);
    const uint32_t ring_s = smem_u32(ring);
    // copy plan: piece p = lane + 32 j of a stage is 16-byte piece p % 9 of row p / 9 (rows past
    // N read row N - 1, whose results are never stored)
    const uint8_t* src[5];
    uint32_t dso[5];
#pragma unroll
    for (int j = 0; j < 5; j++) {
        const int p = lane + 32 * j;
        const int r = p / 9, c = p % 9;
        const int64_t n = n0 + r < N ? n0 + r : N - 1;
        src[j] = w + n * row_bytes + 16 * c;
        dso[j] = (uint32_t)(r * 144 + 16 * c);
    }
    auto issue = [&](int sb, int slot) {
#pragma unroll
        for (int j = 0; j < 5; j++)
            if (lane + 32 * j < GV_PIECES) cp_async16(ring_s + slot * GV_STAGE + dso[j], src[j] + (int64_t)sb * 144);
    };
    // the weights do not depend on the previous kernel: start streaming them before waiting on it
#pragma unroll
    for (int s = 0; s < GV_STAGES - 1; s++) {
        if (sb0 + s < sb1) issue(sb0 + s, s);
        cp_async_commit();
    }
    grid_dep_wait();   // programmatic launch: the activation prep has finished
    grid_dep_launch();

    const bool upper = t >= 2;
    const uint32_t j0 = (2u * t) & 3u;
    const uint32_t sel0 = 0x4040u | (j0 * 0x101u), sel1 = 0x4040u | ((j0 + 1u) * 0x101u);
    const bool has = g < M;   // token rows past M feed zeros
    const __half* arow = a16p + (int64_t)(has ? g : 0) * K + 64 * t;
    const uint32_t* srow = asum2 + (int64_t)(has ? g : 0) * (K / 32) + 2 * t;
    const uint32_t H1024 = 0x64006400u;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int it = 0;
    for (int sb = sb0; sb < sb1; ++sb, ++it) {
        {
            const int nx = sb + GV_STAGES - 1;
            if (nx < sb1) issue(nx, (it + GV_STAGES - 1) % GV_STAGES);
            cp_async_commit();
        }
        uint32_t awl[16], awh[16];
        uint2 as2 = make_uint2(0u, 0u);
        if (has) {
            const uint4* ap = reinterpret_cast<const uint4*>(arow + (int64_t)sb * 256);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint4 l = __ldca(ap + j), h = __ldca(ap + 4 + j);
                awl[4 * j] = l.x, awl[4 * j + 1] = l.y, awl[4 * j + 2] = l.z, awl[4 * j + 3] = l.w;
                awh[4 * j] = h.x, awh[4 * j + 1] = h.y, awh[4 * j + 2] = h.z, awh[4 * j + 3] = h.w;
            }
            as2 = __ldca(reinterpret_cast<const uint2*>(srow + (int64_t)sb * 8));
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) awl[j] = awh[j] = 0u;
        }
        const float2 s2 = __ldca(reinterpret_cast<const float2*>(scl + (int64_t)sb * GV_MMAX + 2 * t));
        cp_async_wait<GV_STAGES - 1>();   // this lane's copies of the stage have landed
        __syncwarp();                     // ... and every lane's
        const uint8_t* r0 = ring + (it % GV_STAGES) * GV_STAGE + g * 144;
        const uint8_t* r1 = r0 + 8 * 144;
        const GvRowScales f0 = gv_row_scales(lds128(r0), upper, sel0, sel1);
        const GvRowScales f1 = gv_row_scales(lds128(r1), upper, sel0, sel1);
        const uint4 q0a = lds128(r0 + 16 + 32 * t), q0b = lds128(r0 + 32 + 32 * t);
        const uint4 q1a = lds128(r1 + 16 + 32 * t), q1b = lds128(r1 + 32 + 32 * t);
        __syncwarp();                     // the slot is free for the copy issued next iteration
        const uint32_t w0[8] = {q0a.x, q0a.y, q0a.z, q0a.w, q0b.x, q0b.y, q0b.z, q0b.w};
        const uint32_t w1[8] = {q1a.x, q1a.y, q1a.z, q1a.w, q1b.x, q1b.y, q1b.z, q1b.w};
        float clo[4] = {0.0f, 0.0f, 0.0f, 0.0f}, chi[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 8; i++) {
            // word i = qs bytes 4i..4i+3 of the chunk: low nibbles are weights 4i..4i+3 of sub-block
            // 2t, high nibbles the same of 2t+1; a0/a1 take bytes (0, 2), a2/a3 bytes (1, 3)
            const uint32_t x0 = w0[i], x1 = w1[i], y0 = x0 >> 8, y1 = x1 >> 8;
            mma16816(clo, hfma2(lop_and_or(x0, 0x000F000Fu, H1024), f0.mul_lo, f0.add_lo),
                     hfma2(lop_and_or(x1, 0x000F000Fu, H1024), f1.mul_lo, f1.add_lo),
                     hfma2(lop_and_or(y0, 0x000F000Fu, H1024), f0.mul_lo, f0.add_lo),
                     hfma2(lop_and_or(y1, 0x000F000Fu, H1024), f1.mul_lo, f1.add_lo), awl[2 * i], awl[2 * i + 1]);
            mma16816(chi, hfma2(lop_and_or(x0, 0x00F000F0u, H1024), f0.mul_hi, f0.add_hi),
                     hfma2(lop_and_or(x1, 0x00F000F0u, H1024), f1.mul_hi, f1.add_hi),
                     hfma2(lop_and_or(y0, 0x00F000F0u, H1024), f0.mul_hi, f0.add_hi),
                     hfma2(lop_and_or(y1, 0x00F000F0u, H1024), f1.mul_hi, f1.add_hi), awh[2 * i], awh[2 * i + 1]);
        }
        // sum_j m_j * (sum of sub-block j's activations), the sums as (hi, lo) fp16 pairs
        mma16816(cm, f0.m_lo, f1.m_lo, f0.m_hi, f1.m_hi, as2.x, as2.y);
        acc[0] = fmaf(s2.x, fmaf(f0.d, clo[0] + chi[0], -f0.dmin * cm[0]), acc[0]);   // row g,   token 2t
        acc[1] = fmaf(s2.y, fmaf(f0.d, clo[1] + chi[1], -f0.dmin * cm[1]), acc[1]);   // row g,   token 2t+1
        acc[2] = fmaf(s2.x, fmaf(f1.d, clo[2] + chi[2], -f1.dmin * cm[2]), acc[2]);   // row g+8, token 2t
        acc[3] = fmaf(s2.y, fmaf(f1.d, clo[3] + chi[3], -f1.dmin * cm[3]), acc[3]);   // row g+8, token 2t+1
    }
    cp_async_wait<0>();
    // the warps' K slices, added in warp order
    float* red = reinterpret_cast<float*>(gv_smem + GV_WARPS * GV_STAGES * GV_STAGE);   // [warp][row][token]
    red[(warp * GV_ROWS + g) * GV_MMAX + 2 * t] = acc[0];
    red[(warp * GV_ROWS + g) * GV_MMAX + 2 * t + 1] = acc[1];
    red[(warp * GV_ROWS + g + 8) * GV_MMAX + 2 * t] = acc[2];
    red[(warp * GV_ROWS + g + 8) * GV_MMAX + 2 * t + 1] = acc[3];
    __syncthreads();
    for (int i = threadIdx.x; i < GV_ROWS * GV_MMAX; i += blockDim.x) {
        const int m = i / GV_ROWS, r = i % GV_ROWS;
        const int64_t n = n0 + r;
        if (m < M && n < N) {
            float v = 0.0f;
#pragma unroll
            for (int q = 0; q < GV_WARPS; q++) v += red[(q * GV_ROWS + r) * GV_MMAX + m];
            dst[(int64_t)m * ldd + n] = v;
        }
    }
}


// The "stream" schedule.
// Work split. A unit is one super-block column (256 weights) of one 16-row block: 16 x 144 bytes,
// one TMA box. The n_rb * nsb units, row block major, are cut into equal contiguous ranges, one
// per warp of a one-wave persistent grid, so every SM streams the same number of bytes. A row
// block covered by one warp is stored directly; one shared by several warps (at most at the two
// ends of each range) is finished by the last of them to arrive: each writes its 16 x 8 partial,
// fences and counts in; the last adds all partials in warp order (so the result does not depend
// on timing) and stores. Nothing waits on another warp.
struct GvSplit {
    int64_t units, warps;
    __device__ __forceinline__ int64_t start(int64_t w) const { return w * units / warps; }
    __device__ __forceinline__ int64_t owner(int64_t u) const { return ((u + 1) * warps - 1) / units; }
};

// Lane (g, t) = (lane / 4, lane % 4) is the MMA's thread group g, thread t: it decodes qs chunk t
// (bytes 32t .. 32t+31) of the block's rows g and g+8 and feeds token row g's activations; its
// accumulators are rows g, g+8 x token rows 2t, 2t+1.
__global__ void __launch_bounds__(32 * GV_WARPS, 2)
    gemv_q4k_kernel(const __grid_constant__ CUtensorMap tmW, int64_t N, int K, const __half* __restrict__ a16p,
                    const uint32_t* __restrict__ asum2, const float* __restrict__ scl, int M, float* __restrict__ dst,
                    int64_t ldd, uint32_t* __restrict__ cnt, float* __restrict__ part, int* __restrict__ err) {
    extern __shared__ __align__(128) uint8_t gv_smem[];
    __shared__ __align__(8) uint64_t bars[GV_WARPS][GV_STAGES];     // stage landed (TMA bytes)
    __shared__ __align__(8) uint64_t empty[GV_WARPS][GV_STAGES];    // stage read by all 32 lanes
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int nsb = K / 256;
    const int64_t n_rb = (N + GV_ROWS - 1) / GV_ROWS;
    // never more working warps than units, so that every working warp's range is non-empty
    const GvSplit split{n_rb * nsb, std::min<int64_t>((int64_t)gridDim.x * GV_WARPS, n_rb * nsb)};
    const int64_t wid = (int64_t)blockIdx.x * GV_WARPS + warp;
    const int64_t u0 = wid < split.warps ? split.start(wid) : 0, u1 = wid < split.warps ? split.start(wid + 1) : 0;
    const uint32_t ring_s = smem_u32(gv_smem + warp * (GV_STAGES * GV_STAGE));
    const uint32_t bar0 = smem_u32(&bars[warp][0]), ebar0 = smem_u32(&empty[warp][0]);
    if (threadIdx.x == 0) abort_flag = 0;
    if (lane == 0) {
        for (int s = 0; s < GV_STAGES; s++) {
            mbar_init(bar0 + 8 * s, 1);
            mbar_init(ebar0 + 8 * s, 32);
        }
        fence_barrier_init();
        tma_prefetch_desc(&tmW);
    }
    __syncthreads();
    // the weights do not depend on the previous kernel: start streaming them before waiting on it
    auto issue = [&](int64_t u, int slot) {
        mbar_arrive_expect_tx(bar0 + 8 * slot, GV_STAGE);
        tma_load_2d(ring_s + slot * GV_STAGE, &tmW, bar0 + 8 * slot, (int32_t)(u % nsb) * 72,
                    (int32_t)(u / nsb) * GV_ROWS);
    };
    if (lane == 0)
        for (int s = 0; s < GV_STAGES && u0 + s < u1; s++) issue(u0 + s, s);
    grid_dep_wait();   // programmatic launch: the activation prep has finished
    grid_dep_launch();

    const bool upper = t >= 2;
    const uint32_t j0 = (2u * t) & 3u;
    const uint32_t sel0 = 0x4040u | (j0 * 0x101u), sel1 = 0x4040u | ((j0 + 1u) * 0x101u);
    const bool has = g < M;   // token rows past M feed zeros
    const __half* arow = a16p + (int64_t)(has ? g : 0) * K + 64 * t;
    const uint32_t* srow = asum2 + (int64_t)(has ? g : 0) * (K / 32) + 2 * t;
    const uint32_t H1024 = 0x64006400u;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int64_t rb = u0 / nsb, seg0 = u0;
    int sb = (int)(u0 % nsb);
    for (int64_t u = u0; u < u1; ++u) {
        const int i = (int)(u - u0), slot = i % GV_STAGES;
        uint32_t awl[16], awh[16];
        uint2 as2 = make_uint2(0u, 0u);
        // the prep kernel wrote these while this grid was already resident (programmatic launch):
        // coherent L1-cached loads (ld.global.ca) after the grid dependency wait, never the
        // non-coherent path
        if (has) {
            const uint4* ap = reinterpret_cast<const uint4*>(arow + (int64_t)sb * 256);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint4 l = __ldca(ap + j), h = __ldca(ap + 4 + j);
                awl[4 * j] = l.x, awl[4 * j + 1] = l.y, awl[4 * j + 2] = l.z, awl[4 * j + 3] = l.w;
                awh[4 * j] = h.x, awh[4 * j + 1] = h.y, awh[4 * j + 2] = h.z, awh[4 * j + 3] = h.w;
            }
            as2 = __ldca(reinterpret_cast<const uint2*>(srow + (int64_t)sb * 8));
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) awl[j] = awh[j] = 0u;
        }
        const float2 s2 = __ldca(reinterpret_cast<const float2*>(scl + (int64_t)sb * GV_MMAX + 2 * t));
        if (!mbar_wait(bar0 + 8 * slot, (uint32_t)(i / GV_STAGES) & 1u, err, ERR_WAIT_STREAM, &abort_flag)) {
            // let the copies this warp issued land before the CTA's shared memory is released
            if (lane == 0)
                for (int64_t v = u; v < u1 && v < u0 + i + GV_STAGES; ++v) {
                    const int vi = (int)(v - u0);
                    if (!mbar_drain(bar0 + 8 * (vi % GV_STAGES), (uint32_t)(vi / GV_STAGES) & 1u))
                        atomicCAS(err, 0, ERR_WAIT_DRAIN);
                }
            return;
        }
        const uint8_t* r0 = gv_smem + warp * (GV_STAGES * GV_STAGE) + slot * GV_STAGE + g * 144;
        const uint8_t* r1 = r0 + 8 * 144;
        const GvRowScales f0 = gv_row_scales(lds128(r0), upper, sel0, sel1);
        const GvRowScales f1 = gv_row_scales(lds128(r1), upper, sel0, sel1);
        const uint4 q0a = lds128(r0 + 16 + 32 * t), q0b = lds128(r0 + 32 + 32 * t);
        const uint4 q1a = lds128(r1 + 16 + 32 * t), q1b = lds128(r1 + 32 + 32 * t);
        // release the slot; the refill's TMA (async proxy) write is issued only once all 32 lanes'
        // reads of it are known complete through the slot's empty barrier
        mbar_arrive(ebar0 + 8 * slot);
        if (lane == 0 && u + GV_STAGES < u1) {
            if (mbar_wait(ebar0 + 8 * slot, (uint32_t)(i / GV_STAGES) & 1u, err, ERR_WAIT_STREAM, &abort_flag))
                issue(u + GV_STAGES, slot);
        }
        __syncwarp();
        const uint32_t w0[8] = {q0a.x, q0a.y, q0a.z, q0a.w, q0b.x, q0b.y, q0b.z, q0b.w};
        const uint32_t w1[8] = {q1a.x, q1a.y, q1a.z, q1a.w, q1b.x, q1b.y, q1b.z, q1b.w};
        float clo[4] = {0.0f, 0.0f, 0.0f, 0.0f}, chi[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cm[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int k = 0; k < 8; k++) {
            // word k = qs bytes 4k..4k+3 of the chunk: low nibbles are weights 4k..4k+3 of sub-block
            // 2t, high nibbles the same of 2t+1; a0/a1 take bytes (0, 2), a2/a3 bytes (1, 3)
            const uint32_t x0 = w0[k], x1 = w1[k], y0 = x0 >> 8, y1 = x1 >> 8;
            mma16816(clo, hfma2(lop_and_or(x0, 0x000F000Fu, H1024), f0.mul_lo, f0.add_lo),
                     hfma2(lop_and_or(x1, 0x000F000Fu, H1024), f1.mul_lo, f1.add_lo),
                     hfma2(lop_and_or(y0, 0x000F000Fu, H1024), f0.mul_lo, f0.add_lo),
                     hfma2(lop_and_or(y1, 0x000F000Fu, H1024), f1.mul_lo, f1.add_lo), awl[2 * k], awl[2 * k + 1]);
            mma16816(chi, hfma2(lop_and_or(x0, 0x00F000F0u, H1024), f0.mul_hi, f0.add_hi),
                     hfma2(lop_and_or(x1, 0x00F000F0u, H1024), f1.mul_hi, f1.add_hi),
                     hfma2(lop_and_or(y0, 0x00F000F0u, H1024), f0.mul_hi, f0.add_hi),
                     hfma2(lop_and_or(y1, 0x00F000F0u, H1024), f1.mul_hi, f1.add_hi), awh[2 * k], awh[2 * k + 1]);
        }
        // sum_j m_j * (sum of sub-block j's activations), the sums as (hi, lo) fp16 pairs
        mma16816(cm, f0.m_lo, f1.m_lo, f0.m_hi, f1.m_hi, as2.x, as2.y);
        acc[0] = fmaf(s2.x, fmaf(f0.d, clo[0] + chi[0], -f0.dmin * cm[0]), acc[0]);   // row g,   token 2t
        acc[1] = fmaf(s2.y, fmaf(f0.d, clo[1] + chi[1], -f0.dmin * cm[1]), acc[1]);   // row g,   token 2t+1
        acc[2] = fmaf(s2.x, fmaf(f1.d, clo[2] + chi[2], -f1.dmin * cm[2]), acc[2]);   // row g+8, token 2t
        acc[3] = fmaf(s2.y, fmaf(f1.d, clo[3] + chi[3], -f1.dmin * cm[3]), acc[3]);   // row g+8, token 2t+1
        if (sb == nsb - 1 || u + 1 == u1) {
            // the end of this warp's part of row block rb
            const int64_t n0 = rb * GV_ROWS;
            float v[4] = {acc[0], acc[1], acc[2], acc[3]};
            bool store = seg0 == rb * nsb && u + 1 == (rb + 1) * nsb;   // the whole row block is ours
            if (!store) {
                const int slot_out = seg0 == u0 ? 0 : 1;                  // first or last block of the range
                *reinterpret_cast<float4*>(part + (wid * 2 + slot_out) * 128 + 4 * lane) =
                    make_float4(acc[0], acc[1], acc[2], acc[3]);
                __threadfence();
                __syncwarp();
                const int64_t w_lo = split.owner(rb * nsb), w_hi = split.owner((rb + 1) * nsb - 1);
                uint32_t old = 0;
                if (lane == 0) old = atomicAdd(cnt + rb, 1u);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == (uint32_t)(w_hi - w_lo)) {
                    __threadfence();
                    v[0] = v[1] = v[2] = v[3] = 0.0f;
                    for (int64_t q = w_lo; q <= w_hi; ++q) {
                        const int sq = (q == w_lo && split.start(q) / nsb != rb) ? 1 : 0;
                        const float4 p = __ldcg(reinterpret_cast<const float4*>(part + (q * 2 + sq) * 128 + 4 * lane));
                        v[0] += p.x, v[1] += p.y, v[2] += p.z, v[3] += p.w;
                    }
                    store = true;
                }
            }
            if (store) {
                const int64_t ra = n0 + g, rc = n0 + g + 8;
                const int ta = 2 * t, tb = 2 * t + 1;
                if (ra < N && ta < M) dst[(int64_t)ta * ldd + ra] = v[0];
                if (ra < N && tb < M) dst[(int64_t)tb * ldd + ra] = v[1];
                if (rc < N && ta < M) dst[(int64_t)ta * ldd + rc] = v[2];
                if (rc < N && tb < M) dst[(int64_t)tb * ldd + rc] = v[3];
            }
            acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
            seg0 = u + 1;
        }
        if (++sb == nsb) sb = 0, ++rb;
    }
}

struct GvWorkspace {
    size_t a16_off, asum_off, scl_off, cnt_off, part_off, total;
};
// warps = the weight-streaming grid's warp count (its partial slots)
static GvWorkspace gv_workspace(int64_t M, int64_t N, int64_t K, int64_t warps) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    GvWorkspace l{};
    l.a16_off = 0;
    l.asum_off = al((size_t)M * K * 2);
    l.scl_off = l.asum_off + al((size_t)M * (K / 32) * 4);
    l.cnt_off = l.scl_off + al((size_t)(K / 256) * GV_MMAX * 4);
    l.part_off = l.cnt_off + al((size_t)((N + GV_ROWS - 1) / GV_ROWS) * 4);
    l.total = l.part_off + al((size_t)warps * 2 * 128 * 4);
    return l;
}

static int gv_sm_count() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (sms[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        sms[dev] = v;
    }
    return sms[dev];
}

// Which kernel runs Q4_K at M <= 8 (read once per process): B200_GEMV_SCHEDULE = rows | stream
// (this file's kernels for every such M) | tiles (the tiled kernel of gemv_tiles.cu, which runs
// every other type and row count). Unset: rows for M <= GV_ROWS_DEFAULT_MMAX, tiles above, the
// crossover measured on B200 (bench.py --workload gemv, the headline's three Q4_K weights: rows
// 1209 / 1068 / 957 GB/s at M = 4 / 6 / 8, tiles 1068-1069 GB/s at each).
// ---------------------------------------------------------------------------------------------
// M = 1, Q8_0 and Q6_K: one launch with no activation prep and no staging of the weights. A CTA of
// NW = ceil(K / 2048) warps spans a row's K; lane l of warp w owns the 64 weights [2048w + 64l,
// +64) (blocks 2c, 2c + 1 of group 8w + l / 4, c = l % 4), keeps their 64 x values in registers
// (brought in by coalesced loads through shared memory), and walks groups of GV1_R rows with the
// next group's scales and quant bytes already loading while the current group is computed. Per
// 32-weight block, acc = sum q * x (the codes exact in fp32, two at a time) times the block's d;
// the lanes' parts are added by shuffles, the warps' in shared memory. fp32 throughout, within the
// decode tolerance of the fp64 oracle (the sums are ordered differently from the reference's).
// Measured on B200 against the tiled kernel at M = 1 (the headline's three weights): Q8_0 2401
// against 1809 GB/s, Q6_K 1678 against 1266. The same scheme for Q4_K (the most decode work per
// byte) ran at 1338 GB/s against the row-block kernel's 1441, so Q4_K keeps that kernel.
// ---------------------------------------------------------------------------------------------
constexpr int GV1_R = 4;
constexpr int GV1_MAXW = 8;                    // K <= 16384
constexpr int GV1_XS = 36;                     // staging row stride (floats): conflict-free 16-byte reads

// x[2048 w + 64 lane + 32 h + j] for h = 0, 1, j < 32 into xv[h][j / 2] as f32x2 pairs (zeros past K).
__device__ __forceinline__ void gv1_load_x(const float* __restrict__ x, int K, int warp, int lane,
                                           float (*stage)[32][GV1_XS], uint64_t (&xv)[2][16]) {
    const int base = warp * 2048;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        // instruction i: lanes 8o' .. 8o'+7 read owner (4i + o')'s 32 values of this half, 128 bytes
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int o = 4 * i + (lane >> 3), j = 4 * (lane & 7);
            const int e = base + 64 * o + 32 * h + j;
            const float4 v = e < K ? __ldg(reinterpret_cast<const float4*>(x + e)) : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(&stage[warp][o][j]) = v;
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(&stage[warp][lane][j]);
            xv[h][j / 2] = f2_pack(v.x, v.y);
            xv[h][j / 2 + 1] = f2_pack(v.z, v.w);
        }
        __syncwarp();
    }
}

// the R rows' parts: shuffles within the warp, then the NW warps' sums in shared memory
template <int R>
__device__ __forceinline__ void gv1_store_rows(const float (&part)[R], float (*red)[GV1_MAXW][GV1_R], int par,
                                               int warp, int lane, int nw, int64_t r0, int64_t N,
                                               float* __restrict__ dst) {
    static_assert(R <= GV1_R, "row group");
#pragma unroll
    for (int r = 0; r < R; r++) {
        float v = part[r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[par][warp][r] = v;
    }
    __syncthreads();
    // red[par] is next written two groups later, after every thread has passed the next barrier
    if (threadIdx.x < R && r0 + threadIdx.x < N) {
        float s = 0.0f;
        for (int i = 0; i < nw; i++) s += red[par][i][threadIdx.x];
        dst[r0 + threadIdx.x] = s;
    }
}

// Q8_0 weights in the packed layout (272-byte groups of eight 32-weight blocks, {d[8] fp16,
// qs[256] int8}): per row the lane loads its two blocks' scales (one 4-byte word) and 64 quant
// bytes. A block past K (K % 256 != 0) has zero quant bytes, a zero scale and zero x.
struct Gv1Q8 {
    uint32_t dd[GV1_R];
    uint4 q[GV1_R][4];
};

__global__ void __launch_bounds__(32 * GV1_MAXW) gemv1_q8_0_kernel(const uint8_t* __restrict__ w, int64_t N, int K,
                                                                   const float* __restrict__ x,
                                                                   float* __restrict__ dst) {
    __shared__ float red[2][GV1_MAXW][GV1_R];
    extern __shared__ __align__(16) float gv1_smem[];   // the x staging rows of the CTA's NW warps
    auto stage = reinterpret_cast<float (*)[32][GV1_XS]>(gv1_smem);
    grid_dep_wait();   // programmatic launch: x may be the previous kernel's output
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = (int)(blockDim.x >> 5);
    const int ngrp = (K + 255) / 256;
    const int g = warp * 8 + (lane >> 2);      // this lane's group
    const int c = lane & 3;                    // its block pair
    const int64_t row_bytes = (int64_t)ngrp * 272;
    const bool live = g < ngrp;
    const int64_t stride = (int64_t)gridDim.x * GV1_R;
    auto load = [&](int64_t r0, Gv1Q8& b) {
#pragma unroll
        for (int r = 0; r < GV1_R; r++) {
            if (live && r0 + r < N) {
                const uint8_t* grp = w + (r0 + r) * row_bytes + (int64_t)g * 272;
                b.dd[r] = __ldg(reinterpret_cast<const uint32_t*>(grp + 4 * c));
#pragma unroll
                for (int j = 0; j < 4; j++) b.q[r][j] = __ldg(reinterpret_cast<const uint4*>(grp + 16 + 64 * c) + j);
            } else {
                b.dd[r] = 0u;   // a zero scale: the row's part is zero whatever the codes
#pragma unroll
                for (int j = 0; j < 4; j++) b.q[r][j] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
    };
    Gv1Q8 cur;
    load((int64_t)blockIdx.x * GV1_R, cur);
    uint64_t xv[2][16];
    gv1_load_x(x, K, warp, lane, stage, xv);
    const uint64_t MAG = f2_pack(-8388736.0f, -8388736.0f);   // -(2^23 + 128)
    int par = 0;
    for (int64_t r0 = (int64_t)blockIdx.x * GV1_R; r0 < N; r0 += stride, par ^= 1) {
        Gv1Q8 nxt;
        load(r0 + stride, nxt);
        float part[GV1_R];
#pragma unroll
        for (int r = 0; r < GV1_R; r++) {
            uint64_t a0 = f2_pack(0.0f, 0.0f), a1 = a0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t wds[4] = {cur.q[r][j].x, cur.q[r][j].y, cur.q[r][j].z, cur.q[r][j].w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint32_t u = wds[k] ^ 0x80808080u;   // int8 -> q + 128
#pragma unroll
                    for (int i = 0; i < 2; i++) {
                        const uint64_t qf = f2_add(magic_pair(u, i), MAG);
                        if (j < 2) a0 = f2_fma(qf, xv[0][8 * j + 2 * k + i], a0);
                        else a1 = f2_fma(qf, xv[1][8 * (j - 2) + 2 * k + i], a1);
                    }
                }
            }
            float l0, l1, h0, h1;
            f2_unpack(a0, l0, l1);
            f2_unpack(a1, h0, h1);
            part[r] = h2f_bits(cur.dd[r]) * (l0 + l1) + h2f_bits(cur.dd[r] >> 16) * (h0 + h1);
        }
        gv1_store_rows(part, red, par, warp, lane, nw, r0, N, dst);
        cur = nxt;
    }
}

// Q6_K weights in the packed layout (208-byte rows {ql[128], qh[64], scales[16]} per super-block,
// d in the transposed plane [nsb][N] after the rows): lane l of warp w owns the 64 weights of
// quarter c = l % 4 of super-block 8w + l / 4 -- half c / 2 of the super-block, its low (c even) or
// high (c odd) 4-bit codes: 64 ql bytes, 32 qh bytes and 4 scales. Two rows per group.
constexpr int GV1_R6 = 2;
struct Gv1Q6 {
    uint4 ql[GV1_R6][4], qh[GV1_R6][2];
    uint32_t sc[GV1_R6];
    uint32_t d[GV1_R6];
};

__global__ void __launch_bounds__(32 * GV1_MAXW) gemv1_q6k_kernel(const uint8_t* __restrict__ w, int64_t N, int K,
                                                                  size_t d_off, const float* __restrict__ x,
                                                                  float* __restrict__ dst) {
    __shared__ float red[2][GV1_MAXW][GV1_R];
    extern __shared__ __align__(16) float gv1_smem[];   // the x staging rows of the CTA's NW warps
    auto stage = reinterpret_cast<float (*)[32][GV1_XS]>(gv1_smem);
    grid_dep_wait();   // programmatic launch: x may be the previous kernel's output
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = (int)(blockDim.x >> 5);
    const int nsb = K / 256;
    const int sb = warp * 8 + (lane >> 2);
    const int hh = (lane & 3) >> 1, hi4 = lane & 1;   // the half, and low / high codes
    const bool live = sb < nsb;
    const int64_t row_bytes = (int64_t)nsb * 208;
    const uint16_t* dplane = reinterpret_cast<const uint16_t*>(w + d_off);
    const int64_t stride = (int64_t)gridDim.x * GV1_R6;
    auto load = [&](int64_t r0, Gv1Q6& b) {
#pragma unroll
        for (int r = 0; r < GV1_R6; r++) {
            if (live && r0 + r < N) {
                const uint8_t* blk = w + (r0 + r) * row_bytes + (int64_t)sb * 208;
#pragma unroll
                for (int j = 0; j < 4; j++) b.ql[r][j] = __ldg(reinterpret_cast<const uint4*>(blk + 64 * hh) + j);
#pragma unroll
                for (int j = 0; j < 2; j++) b.qh[r][j] = __ldg(reinterpret_cast<const uint4*>(blk + 128 + 32 * hh) + j);
                b.sc[r] = __ldg(reinterpret_cast<const uint32_t*>(blk + 192 + 8 * hh + 4 * hi4));
                b.d[r] = __ldg(dplane + (int64_t)sb * N + (r0 + r));
            } else {
#pragma unroll
                for (int j = 0; j < 4; j++) b.ql[r][j] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int j = 0; j < 2; j++) b.qh[r][j] = make_uint4(0u, 0u, 0u, 0u);
                b.sc[r] = 0u;   // zero scales: the row's part is zero whatever the codes
                b.d[r] = 0u;
            }
        }
    };
    Gv1Q6 cur;
    load((int64_t)blockIdx.x * GV1_R6, cur);
    uint64_t xv[2][16];
    gv1_load_x(x, K, warp, lane, stage, xv);
    const uint64_t MAG = f2_pack(-8388640.0f, -8388640.0f);   // -(2^23 + 32)
    int par = 0;
    for (int64_t r0 = (int64_t)blockIdx.x * GV1_R6; r0 < N; r0 += stride, par ^= 1) {
        Gv1Q6 nxt;
        load(r0 + stride, nxt);                // in flight while this group is computed
        float part[GV1_R6];
#pragma unroll
        for (int r = 0; r < GV1_R6; r++) {
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {         // 16 weights t = 16j .. 16j + 15 of the lane's 64, scale j
                const uint4 l4 = cur.ql[r][j];
                const uint4 h4 = cur.qh[r][j & 1];   // qh byte t % 32
                const int hs = 4 * hi4 + 2 * (j >> 1);
                const uint32_t lw[4] = {l4.x, l4.y, l4.z, l4.w}, hw[4] = {h4.x, h4.y, h4.z, h4.w};
                uint64_t acc = f2_pack(0.0f, 0.0f);
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const uint32_t q = ((lw[k] >> (4 * hi4)) & 0x0F0F0F0Fu) | (((hw[k] >> hs) & 0x03030303u) << 4);
#pragma unroll
                    for (int i = 0; i < 2; i++) {
                        const int t2 = (16 * j + 4 * k) / 2 + i;   // pair index of x within the lane's 64
                        acc = f2_fma(f2_add(magic_pair(q, i), MAG), xv[t2 >> 4][t2 & 15], acc);
                    }
                }
                float a0, a1;
                f2_unpack(acc, a0, a1);
                sum += (float)(int8_t)((cur.sc[r] >> (8 * j)) & 0xffu) * (a0 + a1);
            }
            part[r] = h2f_bits(cur.d[r]) * sum;
        }
        gv1_store_rows(part, red, par, warp, lane, nw, r0, N, dst);
        cur = nxt;
    }
}

constexpr int GV_ROWS_DEFAULT_MMAX = 5;
enum GvSchedule { GV_DEFAULT_SCHEDULE, GV_ROWS_SCHEDULE, GV_STREAM_SCHEDULE, GV_TILES_SCHEDULE };
static GvSchedule gv_schedule() {
    static const GvSchedule v = [] {
        const char* e = getenv("B200_GEMV_SCHEDULE");
        if (e && strcmp(e, "stream") == 0) return GV_STREAM_SCHEDULE;
        if (e && strcmp(e, "tiles") == 0) return GV_TILES_SCHEDULE;
        if (e && strcmp(e, "rows") == 0) return GV_ROWS_SCHEDULE;
        return GV_DEFAULT_SCHEDULE;
    }();
    return v;
}
static bool gv_stream_schedule() { return gv_schedule() == GV_STREAM_SCHEDULE; }
// Whether this file's row-block kernels take the call.
static bool gv_row_kernels(int wtype, int64_t M) {
    if (wtype != WT_Q4_K || M > GV_MMAX) return false;
    switch (gv_schedule()) {
        case GV_TILES_SCHEDULE: return false;
        case GV_DEFAULT_SCHEDULE: return M <= GV_ROWS_DEFAULT_MMAX;
        default: return true;
    }
}

// CTAs of the one-wave grid (two per SM), never more warps than units.
static int64_t gv_grid(int64_t N, int64_t K) {
    const int64_t units = ((N + GV_ROWS - 1) / GV_ROWS) * (K / 256);
    return std::max<int64_t>(1, std::min<int64_t>(2 * gv_sm_count(), units / GV_WARPS));
}

}  // namespace b200

extern "C" {

size_t b200_mul_mat_vec_workspace_size(int64_t M, int64_t N, int64_t K) {
    using namespace b200;
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    const size_t tiles = mul_mat_vec_tiles_workspace(M, N, K);   // 0 when M > 32
    if (M > GV_MMAX || K % 256 != 0) return tiles;
    return std::max(tiles, gv_workspace(M, N, K, gv_grid(N, K) * GV_WARPS).total);
}

int b200_mul_mat_vec(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda, int64_t M,
                     float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    using namespace b200;
    if (!w_packed || !src1 || !dst || !dev_err || N <= 0 || K <= 0 || M <= 0 || lda < K || ldd < N)
        return B200_E_INVALID;
    // M = 1, Q6_K or Q8_0 (unless a schedule is forced): the one-launch fp32 kernels, which need no workspace
    if (wtype == WT_Q6_K && M == 1 && gv_schedule() == GV_DEFAULT_SCHEDULE && K % 256 == 0 &&
        K <= 256 * 8 * GV1_MAXW && N <= (1ll << 40) && (reinterpret_cast<uintptr_t>(w_packed) & 15u) == 0 &&
        (reinterpret_cast<uintptr_t>(src1) & 15u) == 0) {
        size_t d_off = 0;
        packed_weight_bytes(WT_Q6_K, N, K, &d_off);
        const int nw = (int)((K / 256 + 7) / 8);
        const int64_t groups = (N + GV1_R6 - 1) / GV1_R6;
        const int64_t per_sm = std::max(1, 12 / nw);
        const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(groups, gv_sm_count() * per_sm));
        const cudaError_t e = launch_pdl(gemv1_q6k_kernel, dim3((unsigned)grid), dim3(32 * nw),
                                         (size_t)nw * 32 * GV1_XS * 4, static_cast<cudaStream_t>(stream),
                                         static_cast<const uint8_t*>(w_packed), N, (int)K, d_off, src1, dst);
        return e == cudaSuccess ? B200_OK : B200_E_CUDA;
    }
    if (wtype == WT_Q8_0 && M == 1 && gv_schedule() == GV_DEFAULT_SCHEDULE && K % 32 == 0 && K <= 256 * 8 * GV1_MAXW &&
        N <= (1ll << 40) && (reinterpret_cast<uintptr_t>(w_packed) & 15u) == 0 &&
        (reinterpret_cast<uintptr_t>(src1) & 15u) == 0) {
        const int nw = (int)(((K + 255) / 256 + 7) / 8);
        const int64_t groups = (N + GV1_R - 1) / GV1_R;
        const int64_t per_sm = std::max(1, 12 / nw);   // one wave: 12 warps of 166 registers per SM
        const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(groups, gv_sm_count() * per_sm));
        const cudaError_t e = launch_pdl(gemv1_q8_0_kernel, dim3((unsigned)grid), dim3(32 * nw),
                                         (size_t)nw * 32 * GV1_XS * 4,
                                         static_cast<cudaStream_t>(stream), static_cast<const uint8_t*>(w_packed), N,
                                         (int)K, src1, dst);
        return e == cudaSuccess ? B200_OK : B200_E_CUDA;
    }
    if (!gv_row_kernels(wtype, M))
        return mul_mat_vec_tiles(wtype, w_packed, N, K, src1, lda, M, dst, ldd, workspace, workspace_bytes, dev_err,
                                 static_cast<cudaStream_t>(stream));
    if (wtype != WT_Q4_K || K % 256 != 0 || M > GV_MMAX || N > (1ll << 30) || K > (1 << 28) ||
        (reinterpret_cast<uintptr_t>(w_packed) & 15u) != 0)
        return B200_E_UNSUPPORTED;
    const int64_t grid = gv_grid(N, K);
    const GvWorkspace l = gv_workspace(M, N, K, grid * GV_WARPS);
    if (!workspace || workspace_bytes < l.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return B200_E_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(gemv_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_SMEM) !=
                cudaSuccess ||
            cudaFuncSetAttribute(gemv_q4k_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_SMEM_ROWS) !=
                cudaSuccess)
            return B200_E_CUDA;
        attr_set[dev] = true;
    }
    // the packed Q4_K weight as a 2-D uint16 tensor [N rows, 72 * nsb]: one unit is a 72 x 16 box
    const int64_t row_bytes = (K / 256) * 144;
    CUtensorMap tmW;
    if (!make_tmap_2d_u16(&tmW, w_packed, (uint64_t)N, (uint64_t)(row_bytes / 2), (uint64_t)row_bytes, GV_ROWS, 72))
        return B200_E_CUDA;
    char* ws = static_cast<char*>(workspace);
    __half* a16p = reinterpret_cast<__half*>(ws + l.a16_off);
    uint32_t* asum2 = reinterpret_cast<uint32_t*>(ws + l.asum_off);
    float* scl = reinterpret_cast<float*>(ws + l.scl_off);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(ws + l.cnt_off);
    float* part = reinterpret_cast<float*>(ws + l.part_off);
    const int64_t n_rb = (N + GV_ROWS - 1) / GV_ROWS;
    const bool vec = (reinterpret_cast<uintptr_t>(src1) & 15u) == 0 && lda % 4 == 0;
    const int warps = (int)(M * (K / 256));
    const dim3 pgrid((unsigned)std::max(1, (warps + 7) / 8)), pblock(256);
    cudaError_t e = vec ? launch_pdl(gemv_act_kernel<true>, pgrid, pblock, 0, st, src1, lda, (int)M, (int)K, a16p,
                                     asum2, scl, cnt, n_rb)
                        : launch_pdl(gemv_act_kernel<false>, pgrid, pblock, 0, st, src1, lda, (int)M, (int)K, a16p,
                                     asum2, scl, cnt, n_rb);
    if (e != cudaSuccess) return B200_E_CUDA;
    if (!gv_stream_schedule()) {
        e = launch_pdl(gemv_q4k_rows_kernel, dim3((unsigned)n_rb), dim3(32 * GV_WARPS), GV_SMEM_ROWS, st,
                       static_cast<const uint8_t*>(w_packed), N, (int)K, (const __half*)a16p, (const uint32_t*)asum2,
                       (const float*)scl, (int)M, dst, ldd);
        return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
    }
    e = launch_pdl(gemv_q4k_kernel, dim3((unsigned)grid), dim3(32 * GV_WARPS), GV_SMEM, st, tmW, N, (int)K,
                   (const __half*)a16p, (const uint32_t*)asum2, (const float*)scl, (int)M, dst, ldd, cnt, part,
                   dev_err);
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
