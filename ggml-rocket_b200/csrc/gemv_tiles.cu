// Decode-size MUL_MAT (M = 1..32 token rows) over Q4_K, Q6_K and Q8_0 weights on a tiled
// weight-streaming kernel: the path of b200_mul_mat_vec for every weight type and row count
// except Q4_K at M <= 8, which the row-block kernels of gemv.cu keep (they stream that case
// faster, measured).
//
// dst[m, n] = sum_k a[m, k] * W[n, k], W the packed weight (b200_weight_pack). With M this small
// the op is bound by reading W once from HBM:
//   * one persistent CTA per SM; the weight is cut into units of 128 rows x one 256-weight
//     super-block column (the prefill GEMM's raw tile: 18 KB Q4_K, 26 KB Q6_K, 34 KB Q8_0), taken
//     row block by row block in equal contiguous ranges, one per CTA (stream-K over the units);
//   * one producer thread streams each unit's weight tile by TMA, together with the unit's
//     prepared activations (one untiled bulk copy), into a ring of stages; eight consumer warps,
//     16 weight rows each, decode the weights straight into warp-level MMA (mma.sync m16n8k16)
//     A fragments -- no shared-memory round trip of decoded values -- and take the activations'
//     B fragments from the stage;
//   * 8 token rows per MMA column tile, NT = ceil(M / 8) tiles: every decoded fragment serves all
//     M token rows;
//   * a row block shared by several CTAs is finished by the last to arrive, which adds the
//     others' partial sums in CTA order: results do not depend on timing, nothing waits on
//     another CTA.
// Arithmetic per type (all products exact in the MMA, sums in fp32):
//   Q4_K  fp16 integers q*sc (the 6-bit sub-block scale folded in: (1024 + q) * sc - 1024 * sc in
//         one fused f16x2 FMA, exact since q*sc <= 945); the minimum term dmin * sum_j m_j *
//         sum(a over sub-block j) is one more MMA per super-block with the activation sums split
//         into fp16 (hi, lo) pairs; per super-block acc += s * (d * C - dmin * Cmin);
//   Q8_0  fp16 integers 1152 + q (a byte permute onto 0x64: 1024 + (q + 128)); each 32-weight
//         block's two MMAs start from C = -1152 * sum(a over the block), so they yield sum q * a
//         exactly, which is scaled by the block's d in fp32;
//   Q6_K  fp16 integers 1024 + q (4 low bits from ql, 2 high bits from qh); each 16-weight
//         sub-block's MMA starts from C = -1056 * sum(a over the sub-block) (1056 = 1024 + 32,
//         ggml's offset), yielding sum (q - 32) * a, scaled by d * sc in fp32.
// The activations are prepared once per call (gw_prep_kernel): per 256-value block the block's
// absmax s and fp16(a / s), written straight into the B-fragment order of the weight type, plus
// the per-block sums the arithmetic above needs. The only rounding beyond fp32 sums is the
// activations' fp16 rounding, as in the prefill GEMM's activation pack.
// The decodes are ggml's dequantize_row_q4_K / _q6_K / _q8_0 (ggml-rocket.cpp:3894-3907 calls
// them through to_float).
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
namespace gw {

constexpr int CWARPS = 8;                        // consumer warps, 16 weight rows each
constexpr int ROWS = 16 * CWARPS;                // weight rows per unit (the raw tile maps' box)
constexpr int THREADS = 32 * (CWARPS + 1);       // + one producer warp
constexpr int NT_MAX = 4;                        // 8-token MMA column tiles: M <= 32
constexpr int MMAX = 8 * NT_MAX;
constexpr int MAX_STAGES = 8;
constexpr int SMEM_BUDGET = 227 * 1024 - 1024;   // dynamic shared memory (barriers are static)
// Prepared activations, per (super-block column, column tile), CHUNK bytes:
//   [0, 4096)     B fragments: [MMA pair 8][token 8][lane t 4][16 B] (two MMAs' b0, b1)
//   [4096, 4608)  per-block data: Q4_K (hi, lo) sub-block sums as the minimum MMA's B fragment
//                 [token 8][t 4][2]; Q8_0 / Q6_K the C start values [token pair 4][block][2] f32
//   [4608, 4640)  s per token, f32
constexpr int CHUNK = 4640;
constexpr int CH_BLK = 4096, CH_SCALE = 4608;

template <int WT>
struct Type {
    static constexpr int ROW = WT == WT_Q4_K ? 144 : WT == WT_Q6_K ? 208 : 272;   // packed bytes / super-block
    static constexpr int W_BYTES = ROW * ROWS;
    static constexpr int D_BYTES = WT == WT_Q6_K ? ROWS * 2 : 0;   // the transposed d plane's box
};
template <int WT, int NT>
struct Cfg {
    static constexpr int ACT_OFF = Type<WT>::W_BYTES + Type<WT>::D_BYTES;
    static constexpr int ACT_BYTES = NT * CHUNK;
    static constexpr int STAGE = (ACT_OFF + ACT_BYTES + 127) / 128 * 128;
    static constexpr int TX = ACT_OFF + ACT_BYTES;   // bytes landing per stage
};

// ---- small PTX helpers ---------------------------------------------------------------------

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));   // (a & b) | c
    return d;
}
__device__ __forceinline__ uint32_t lop_or_and(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xF8;" : "=r"(d) : "r"(a), "r"(b), "r"(c));   // a | (b & c)
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
__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ float2 ldsf2(const uint8_t* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}
// x shifted left by s (right by -s when s < 0); s is a constant once the loops are unrolled
__device__ __forceinline__ uint32_t shl_signed(uint32_t x, int s) { return s >= 0 ? x << s : x >> -s; }
// one arrival on a row block's counter: release of this warp's partial sums, acquire of the others'
__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// ---- activation prep -----------------------------------------------------------------------

// One warp per (token row m of the padded 8 * NT, super-block column sb); lane l holds values
// 8l .. 8l+7 of the block (zeros past K and for the padding rows m >= M). The block's s = absmax
// (1 when all are zero; 0 for the padding rows) and fp16(a / s) go into the B-fragment order of
// the weight type WT (the k slots each lane's decoded weights occupy, see the consumers below),
// with the per-block sums of the fp16 values. Also zeroes the n_cnt arrival counters of the
// weight-streaming kernel that follows.
template <int WT, bool VEC>
__global__ void __launch_bounds__(256) gw_prep_kernel(const float* __restrict__ a, int64_t lda, int M, int K,
                                                      int nsb, int nt_count, uint8_t* __restrict__ act,
                                                      uint32_t* __restrict__ cnt, int64_t n_cnt) {
    grid_dep_wait();   // the previous kernel may still read this workspace (programmatic launch)
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_cnt; i += (int64_t)gridDim.x * blockDim.x)
        cnt[i] = 0u;
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= nt_count * 8 * nsb) return;
    const int m = gw / nsb, sb = gw % nsb;
    const int nt = m >> 3, n = m & 7;
    const int k = sb * 256 + 8 * lane;
    float x[8];
#pragma unroll
    for (int i = 0; i < 8; i++) x[i] = 0.0f;
    if (m < M) {
        const float* p = a + (int64_t)m * lda + k;
        if (VEC && k + 8 <= K) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(p));
            const float4 v = __ldg(reinterpret_cast<const float4*>(p + 4));
            x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = v.x, x[5] = v.y, x[6] = v.z, x[7] = v.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) x[i] = k + i < K ? __ldg(p + i) : 0.0f;
        }
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
    // a word's bytes (0, 2) feed the MMA slots (2t, 2t+1), bytes (1, 3) the slots (2t+8, 2t+9)
    const uint32_t e02 = pack_h2(h[0], h[2]), e13 = pack_h2(h[1], h[3]);
    const uint32_t e46 = pack_h2(h[4], h[6]), e57 = pack_h2(h[5], h[7]);
    uint8_t* ch = act + ((int64_t)sb * nt_count + nt) * CHUNK;
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) sum += __half2float(h[i]);
    if constexpr (WT == WT_Q4_K) {
        // k = 64t + 32hh + 4i + e: lane t's qs chunk t, low (hh = 0) / high nibbles, word i
        const int t = lane >> 3, hh = (lane >> 2) & 1, i0 = 2 * (lane & 3);
        *reinterpret_cast<uint2*>(ch + (i0 * 8 + n) * 64 + t * 16 + hh * 8) = make_uint2(e02, e13);
        *reinterpret_cast<uint2*>(ch + ((i0 + 1) * 8 + n) * 64 + t * 16 + hh * 8) = make_uint2(e46, e57);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((lane & 3) == 0) {
            const int j = lane >> 2;   // sub-block
            const __half hi = __float2half_rn(sum);
            const __half lo = __float2half_rn(sum - __half2float(hi));
            *reinterpret_cast<uint32_t*>(ch + CH_BLK + (n * 4 + (j >> 1)) * 8 + (j & 1) * 4) = pack_h2(hi, lo);
        }
    } else if constexpr (WT == WT_Q8_0) {
        // k = 32b + 8t + 4h + e: block b, lane t's words 2t + h
        const int b = lane >> 2, t = lane & 3;
        *reinterpret_cast<uint4*>(ch + (b * 8 + n) * 64 + t * 16) = make_uint4(e02, e13, e46, e57);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((lane & 3) == 0)
            *reinterpret_cast<float*>(ch + CH_BLK + ((n >> 1) * 8 + b) * 8 + (n & 1) * 4) = -1152.0f * sum;
    } else {
        // k = 16p + 4t + e: sub-block p, lane t's word
        const int p = lane >> 1, t0 = 2 * (lane & 1);
        *reinterpret_cast<uint2*>(ch + ((p >> 1) * 8 + n) * 64 + t0 * 16 + (p & 1) * 8) = make_uint2(e02, e13);
        *reinterpret_cast<uint2*>(ch + ((p >> 1) * 8 + n) * 64 + (t0 + 1) * 16 + (p & 1) * 8) = make_uint2(e46, e57);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        if ((lane & 1) == 0)
            *reinterpret_cast<float*>(ch + CH_BLK + ((n >> 1) * 16 + p) * 8 + (n & 1) * 4) = -1056.0f * sum;
    }
    if (lane == 0) *reinterpret_cast<float*>(ch + CH_SCALE + 4 * n) = m < M ? s : 0.0f;
}

// ---- per-unit consumers: one warp, 16 weight rows (r0 = its row g, r1 = g + 8) x 256 weights --
// Lane (g, t) = (lane / 4, lane % 4) is the MMA's thread group g, thread t: A fragment rows g and
// g+8, k slots {2t, 2t+1, 2t+8, 2t+9}; accumulators rows g, g+8 x tokens 8nt + 2t, 8nt + 2t + 1.

// Q4_K scale constants of one weight row for this lane's two sub-blocks (2t: the low nibbles of
// qs chunk t, 2t+1: its high nibbles), from the row's 16-byte header {d, dmin, scales[12]}. The
// 6-bit sc / m values are ggml's get_scale_min_k4 (t >= 2 takes the j >= 4 form), moved into
// f16x2 pairs by a byte permute onto 0x64 (1024 + v, then - 1024).
struct RowScales {
    uint32_t mul_lo, add_lo, mul_hi, add_hi, m_lo, m_hi;   // f16x2 pairs
    float d, dmin;
};
__device__ __forceinline__ RowScales row_scales(const uint4 h, bool upper, uint32_t sel0, uint32_t sel1) {
    const uint32_t scw = upper ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
    const uint32_t mw = upper ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
    const uint32_t H1024 = 0x64006400u;
    const uint32_t sc0 = hsub2(prmt(scw, 0x64646464u, sel0), H1024);   // (sc_2t, sc_2t)
    const uint32_t sc1 = hsub2(prmt(scw, 0x64646464u, sel1), H1024);   // (sc_2t+1, sc_2t+1)
    RowScales r;
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

// Q4_K: lane t decodes qs chunk t (bytes 32t .. 32t+31: sub-block 2t in the low nibbles, 2t+1 in
// the high ones) of rows r0 and r1; word i gives one MMA over the low nibbles and one over the
// high nibbles (MMA pair i of the B fragments). Even and odd words accumulate apart (shorter MMA
// dependency chains).
template <int NT>
__device__ __forceinline__ void unit_q4k(const uint8_t* W, const uint8_t* A, int row, int g, int t,
                                         float (&acc)[NT][4]) {
    const uint8_t* r0 = W + row * 144;
    const uint8_t* r1 = r0 + 8 * 144;
    const bool upper = t >= 2;
    const uint32_t j0 = (2u * t) & 3u;
    const uint32_t sel0 = 0x4040u | (j0 * 0x101u), sel1 = 0x4040u | ((j0 + 1u) * 0x101u);
    const RowScales f0 = row_scales(lds128(r0), upper, sel0, sel1);
    const RowScales f1 = row_scales(lds128(r1), upper, sel0, sel1);
    const uint4 q0a = lds128(r0 + 16 + 32 * t), q0b = lds128(r0 + 32 + 32 * t);
    const uint4 q1a = lds128(r1 + 16 + 32 * t), q1b = lds128(r1 + 32 + 32 * t);
    const uint32_t w0[8] = {q0a.x, q0a.y, q0a.z, q0a.w, q0b.x, q0b.y, q0b.z, q0b.w};
    const uint32_t w1[8] = {q1a.x, q1a.y, q1a.z, q1a.w, q1b.x, q1b.y, q1b.z, q1b.w};
    const uint32_t H1024 = 0x64006400u;
    const uint8_t* bf = A + (g * 4 + t) * 16;
    float clo[2][NT][4], chi[2][NT][4], cm[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 4; j++) clo[0][nt][j] = clo[1][nt][j] = chi[0][nt][j] = chi[1][nt][j] = cm[nt][j] = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        // word i = qs bytes 4i..4i+3 of the chunk: low nibbles are weights 4i..4i+3 of sub-block
        // 2t, high nibbles the same of 2t+1; a0/a1 take bytes (0, 2), a2/a3 bytes (1, 3)
        const uint32_t x0 = w0[i], x1 = w1[i], y0 = x0 >> 8, y1 = x1 >> 8;
        const uint32_t l0 = hfma2(lop_and_or(x0, 0x000F000Fu, H1024), f0.mul_lo, f0.add_lo);
        const uint32_t l1 = hfma2(lop_and_or(x1, 0x000F000Fu, H1024), f1.mul_lo, f1.add_lo);
        const uint32_t l2 = hfma2(lop_and_or(y0, 0x000F000Fu, H1024), f0.mul_lo, f0.add_lo);
        const uint32_t l3 = hfma2(lop_and_or(y1, 0x000F000Fu, H1024), f1.mul_lo, f1.add_lo);
        const uint32_t h0 = hfma2(lop_and_or(x0, 0x00F000F0u, H1024), f0.mul_hi, f0.add_hi);
        const uint32_t h1 = hfma2(lop_and_or(x1, 0x00F000F0u, H1024), f1.mul_hi, f1.add_hi);
        const uint32_t h2 = hfma2(lop_and_or(y0, 0x00F000F0u, H1024), f0.mul_hi, f0.add_hi);
        const uint32_t h3 = hfma2(lop_and_or(y1, 0x00F000F0u, H1024), f1.mul_hi, f1.add_hi);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint4 b = lds128(bf + nt * CHUNK + i * 512);
            mma16816(clo[i & 1][nt], l0, l1, l2, l3, b.x, b.y);
            mma16816(chi[i & 1][nt], h0, h1, h2, h3, b.z, b.w);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const uint8_t* an = A + nt * CHUNK;
        // sum_j m_j * (sum of sub-block j's activations), the sums as (hi, lo) fp16 pairs
        const uint2 as2 = lds64(an + CH_BLK + (g * 4 + t) * 8);
        mma16816(cm[nt], f0.m_lo, f1.m_lo, f0.m_hi, f1.m_hi, as2.x, as2.y);
        const float2 s2 = ldsf2(an + CH_SCALE + 8 * t);
        float c[4];
#pragma unroll
        for (int j = 0; j < 4; j++) c[j] = (clo[0][nt][j] + clo[1][nt][j]) + (chi[0][nt][j] + chi[1][nt][j]);
        acc[nt][0] = fmaf(s2.x, fmaf(f0.d, c[0], -f0.dmin * cm[nt][0]), acc[nt][0]);
        acc[nt][1] = fmaf(s2.y, fmaf(f0.d, c[1], -f0.dmin * cm[nt][1]), acc[nt][1]);
        acc[nt][2] = fmaf(s2.x, fmaf(f1.d, c[2], -f1.dmin * cm[nt][2]), acc[nt][2]);
        acc[nt][3] = fmaf(s2.y, fmaf(f1.d, c[3], -f1.dmin * cm[nt][3]), acc[nt][3]);
    }
}

// Q8_0: the packed row holds 272-byte groups {d[8] fp16, qs[256] int8}. Block b's two MMAs take
// words 2t (h = 0) and 2t+1 (h = 1) of the block from lane t.
template <int NT>
__device__ __forceinline__ void unit_q8_0(const uint8_t* W, const uint8_t* A, int row, int g, int t,
                                          float (&acc)[NT][4]) {
    const uint8_t* r0 = W + row * 272;
    const uint8_t* r1 = r0 + 8 * 272;
    const uint4 hd0 = lds128(r0), hd1 = lds128(r1);
    const uint32_t dw0[4] = {hd0.x, hd0.y, hd0.z, hd0.w}, dw1[4] = {hd1.x, hd1.y, hd1.z, hd1.w};
    const uint32_t H64 = 0x64646464u, FLIP = 0x80808080u;
    const uint8_t* bf = A + (g * 4 + t) * 16;
    float blk[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 4; j++) blk[nt][j] = 0.0f;
#pragma unroll
    for (int b = 0; b < 8; b++) {
        const uint2 p0 = lds64(r0 + 16 + 32 * b + 8 * t), p1 = lds64(r1 + 16 + 32 * b + 8 * t);
        const uint32_t x00 = p0.x ^ FLIP, x01 = p0.y ^ FLIP, x10 = p1.x ^ FLIP, x11 = p1.y ^ FLIP;   // q + 128
        const float d0 = h2f_bits(dw0[b >> 1] >> (16 * (b & 1))), d1 = h2f_bits(dw1[b >> 1] >> (16 * (b & 1)));
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const uint8_t* an = A + nt * CHUNK;
            const float2 ci = ldsf2(an + CH_BLK + (t * 8 + b) * 8);   // -1152 * block sums
            const uint4 bq = lds128(bf + nt * CHUNK + b * 512);
            float c[4] = {ci.x, ci.y, ci.x, ci.y};
            mma16816(c, prmt(x00, H64, 0x4240u), prmt(x10, H64, 0x4240u), prmt(x00, H64, 0x4341u),
                     prmt(x10, H64, 0x4341u), bq.x, bq.y);
            mma16816(c, prmt(x01, H64, 0x4240u), prmt(x11, H64, 0x4240u), prmt(x01, H64, 0x4341u),
                     prmt(x11, H64, 0x4341u), bq.z, bq.w);
            blk[nt][0] = fmaf(d0, c[0], blk[nt][0]);
            blk[nt][1] = fmaf(d0, c[1], blk[nt][1]);
            blk[nt][2] = fmaf(d1, c[2], blk[nt][2]);
            blk[nt][3] = fmaf(d1, c[3], blk[nt][3]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const float2 s2 = ldsf2(A + nt * CHUNK + CH_SCALE + 8 * t);
        acc[nt][0] = fmaf(s2.x, blk[nt][0], acc[nt][0]);
        acc[nt][1] = fmaf(s2.y, blk[nt][1], acc[nt][1]);
        acc[nt][2] = fmaf(s2.x, blk[nt][2], acc[nt][2]);
        acc[nt][3] = fmaf(s2.y, blk[nt][3], acc[nt][3]);
    }
}

// Q6_K: plane A rows of 208-byte {ql[128], qh[64], scales[16]} super-blocks, d from the d plane's
// box behind the tile. Sub-block p = 8hh + 2q + is (weights 16p .. 16p+15) is
//   ql[64hh + 32(q & 1) + 16is + l'] nibble (q >> 1), qh[32hh + 16is + l'] bits 2q..2q+1,
// l' = 0..15; lane t holds l' = 4t .. 4t+3 (one ql word and one qh word).
template <int NT>
__device__ __forceinline__ void unit_q6k(const uint8_t* W, const uint8_t* A, int row, int g, int t,
                                         float (&acc)[NT][4]) {
    const uint8_t* r0 = W + row * 208;
    const uint8_t* r1 = r0 + 8 * 208;
    const __half* dpl = reinterpret_cast<const __half*>(W + ROWS * 208);
    const float d0 = __half2float(dpl[row]), d1 = __half2float(dpl[row + 8]);
    const uint4 s0 = lds128(r0 + 192), s1 = lds128(r1 + 192);
    const uint32_t sc0[4] = {s0.x, s0.y, s0.z, s0.w}, sc1[4] = {s1.x, s1.y, s1.z, s1.w};
    const uint32_t H1024 = 0x64006400u;
    const uint8_t* bf = A + (g * 4 + t) * 16;
    float blk[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 4; j++) blk[nt][j] = 0.0f;
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        uint32_t qa0[2], qb0[2], qh0[2], qa1[2], qb1[2], qh1[2];
#pragma unroll
        for (int is = 0; is < 2; is++) {
            const int o = 64 * hh + 16 * is + 4 * t, oh = 128 + 32 * hh + 16 * is + 4 * t;
            qa0[is] = lds32(r0 + o), qb0[is] = lds32(r0 + o + 32), qh0[is] = lds32(r0 + oh);
            qa1[is] = lds32(r1 + o), qb1[is] = lds32(r1 + o + 32), qh1[is] = lds32(r1 + oh);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int ns = 4 * (q >> 1);
#pragma unroll
            for (int is = 0; is < 2; is++) {
                const int p = 8 * hh + 2 * q + is;
                const uint32_t l0 = (q & 1) ? qb0[is] : qa0[is], l1 = (q & 1) ? qb1[is] : qa1[is];
                // 1024 + (nibble | qh bits << 4): bytes (0, 2) and (1, 3) of the words
                const uint32_t a0 = lop_or_and(lop_and_or(l0 >> ns, 0x000F000Fu, H1024), shl_signed(qh0[is], 4 - 2 * q),
                                               0x00300030u);
                const uint32_t a1 = lop_or_and(lop_and_or(l1 >> ns, 0x000F000Fu, H1024), shl_signed(qh1[is], 4 - 2 * q),
                                               0x00300030u);
                const uint32_t a2 = lop_or_and(lop_and_or(l0 >> (8 + ns), 0x000F000Fu, H1024), qh0[is] >> (4 + 2 * q),
                                               0x00300030u);
                const uint32_t a3 = lop_or_and(lop_and_or(l1 >> (8 + ns), 0x000F000Fu, H1024), qh1[is] >> (4 + 2 * q),
                                               0x00300030u);
                const float ds0 = d0 * (float)(int8_t)(sc0[p >> 2] >> (8 * (p & 3)));
                const float ds1 = d1 * (float)(int8_t)(sc1[p >> 2] >> (8 * (p & 3)));
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const uint8_t* an = A + nt * CHUNK;
                    const float2 ci = ldsf2(an + CH_BLK + (t * 16 + p) * 8);   // -1056 * sub-block sums
                    const uint2 bq = lds64(bf + nt * CHUNK + (p >> 1) * 512 + (p & 1) * 8);
                    float c[4] = {ci.x, ci.y, ci.x, ci.y};
                    mma16816(c, a0, a1, a2, a3, bq.x, bq.y);
                    blk[nt][0] = fmaf(ds0, c[0], blk[nt][0]);
                    blk[nt][1] = fmaf(ds0, c[1], blk[nt][1]);
                    blk[nt][2] = fmaf(ds1, c[2], blk[nt][2]);
                    blk[nt][3] = fmaf(ds1, c[3], blk[nt][3]);
                }
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const float2 s2 = ldsf2(A + nt * CHUNK + CH_SCALE + 8 * t);
        acc[nt][0] = fmaf(s2.x, blk[nt][0], acc[nt][0]);
        acc[nt][1] = fmaf(s2.y, blk[nt][1], acc[nt][1]);
        acc[nt][2] = fmaf(s2.x, blk[nt][2], acc[nt][2]);
        acc[nt][3] = fmaf(s2.y, blk[nt][3], acc[nt][3]);
    }
}

// ---- the weight-streaming kernel ---------------------------------------------------------------

// Equal contiguous ranges of `units` over `ctas` CTAs.
struct Split {
    int64_t units, ctas;
    __host__ __device__ __forceinline__ int64_t start(int64_t c) const { return c * units / ctas; }
    __host__ __device__ __forceinline__ int64_t owner(int64_t u) const { return ((u + 1) * ctas - 1) / units; }
};

// Units u = rb * nsb + sb (row block rb of 128 rows, super-block column sb), CTA c taking
// [start(c), start(c+1)). Warps 0..7 consume, warp 8's lane 0 produces. Partial sums: per CTA
// two slots (its first and its last row block), per warp 16 rows x 8 NT tokens.
template <int WT, int NT>
__global__ void __launch_bounds__(THREADS, 1)
    gw_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmD, int64_t N, int nsb,
              const uint8_t* __restrict__ act, int M, float* __restrict__ dst, int64_t ldd, int stages,
              uint32_t* __restrict__ cnt, float* __restrict__ part, int* __restrict__ err) {
    using C = Cfg<WT, NT>;
    extern __shared__ __align__(128) uint8_t gw_smem[];
    __shared__ __align__(8) uint64_t full[MAX_STAGES];    // stage landed (TMA transaction bytes)
    __shared__ __align__(8) uint64_t empty[MAX_STAGES];   // stage read by the eight consumer warps
    __shared__ int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n_rb = (N + ROWS - 1) / ROWS;
    const Split split{n_rb * nsb, (int64_t)gridDim.x};
    const int64_t u0 = split.start(blockIdx.x), u1 = split.start(blockIdx.x + 1);
    const uint32_t smem0 = smem_u32(gw_smem);
    const uint32_t fb = smem_u32(&full[0]), eb = smem_u32(&empty[0]);
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < stages; s++) {
            mbar_init(fb + 8 * s, 1);
            mbar_init(eb + 8 * s, CWARPS);
        }
        fence_barrier_init();
    }
    __syncthreads();
    grid_dep_launch();

    if (warp == CWARPS) {
        // ---- producer: weight tile (+ Q6_K d box) by TMA, activations by one bulk copy ----
        if (lane != 0) return;
        tma_prefetch_desc(&tmW);
        if constexpr (WT == WT_Q6_K) tma_prefetch_desc(&tmD);
        const int64_t n_units = u1 - u0;
        auto issue_w = [&](int64_t i) {
            const int slot = (int)(i % stages);
            const int64_t u = u0 + i;
            const int32_t rb = (int32_t)(u / nsb), sb = (int32_t)(u % nsb);
            const uint32_t dst_s = smem0 + slot * C::STAGE, bar = fb + 8 * slot;
            mbar_arrive_expect_tx(bar, C::TX);
            tma_load_2d(dst_s, &tmW, bar, sb * (Type<WT>::ROW / 2), rb * ROWS);
            if constexpr (WT == WT_Q6_K) tma_load_2d(dst_s + Type<WT>::W_BYTES, &tmD, bar, rb * ROWS, sb);
        };
        auto issue_a = [&](int64_t i) {
            const int slot = (int)(i % stages);
            const int64_t sb = (u0 + i) % nsb;
            bulk_load_g2s(smem0 + slot * C::STAGE + C::ACT_OFF, act + sb * C::ACT_BYTES, C::ACT_BYTES, fb + 8 * slot);
        };
        // the weights do not depend on the previous kernels: start streaming them before waiting
        const int64_t pre = stages < n_units ? stages : n_units;
        for (int64_t i = 0; i < pre; i++) issue_w(i);
        grid_dep_wait();   // programmatic launch: the activation prep has finished
        for (int64_t i = 0; i < pre; i++) issue_a(i);
        int64_t issued = pre;
        for (int64_t i = pre; i < n_units; i++) {
            const int slot = (int)(i % stages);
            if (!mbar_wait(eb + 8 * slot, (uint32_t)(i / stages - 1) & 1u, err, ERR_WAIT_PRODUCER, &abort_flag)) break;
            issue_w(i);
            issue_a(i);
            issued = i + 1;
        }
        if (abort_flag) {
            // let the copies in flight land before the CTA's shared memory is released
            for (int64_t v = issued > stages ? issued - stages : 0; v < issued; v++)
                if (!mbar_drain(fb + 8 * (int)(v % stages), (uint32_t)(v / stages) & 1u)) {
                    atomicCAS(err, 0, ERR_WAIT_DRAIN);
                    break;
                }
        }
        return;
    }

    // ---- consumers ----
    grid_dep_wait();   // dst, the counters and the partial slots are written below
    const int g = lane >> 2, t = lane & 3;
    const int row = 16 * warp + g;
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[nt][j] = 0.0f;
    int64_t seg0 = u0;
    for (int64_t u = u0; u < u1; ++u) {
        const int64_t i = u - u0;
        const int slot = (int)(i % stages);
        const int64_t rb = u / nsb;
        const int sb = (int)(u % nsb);
        if (!mbar_wait(fb + 8 * slot, (uint32_t)(i / stages) & 1u, err, ERR_WAIT_STREAM, &abort_flag)) {
            // let copies that may be in flight land before the CTA's shared memory is released
            if (warp == 0 && lane == 0)
                for (int64_t v = i; v < u1 - u0 && v < i + stages; v++)
                    if (!mbar_drain(fb + 8 * (int)(v % stages), (uint32_t)(v / stages) & 1u)) {
                        atomicCAS(err, 0, ERR_WAIT_DRAIN);
                        break;
                    }
            return;
        }
        const uint8_t* W = gw_smem + slot * C::STAGE;
        const uint8_t* A = W + C::ACT_OFF;
        if constexpr (WT == WT_Q4_K) unit_q4k<NT>(W, A, row, g, t, acc);
        else if constexpr (WT == WT_Q8_0) unit_q8_0<NT>(W, A, row, g, t, acc);
        else unit_q6k<NT>(W, A, row, g, t, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(eb + 8 * slot);   // this warp's reads of the stage are done
        if (sb == nsb - 1 || u + 1 == u1) {
            // the end of this CTA's part of row block rb
            float v[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int j = 0; j < 4; j++) v[nt][j] = acc[nt][j];
            bool store = seg0 == rb * nsb && u + 1 == (rb + 1) * nsb;   // the whole row block is ours
            if (!store) {
                const int slot_out = seg0 == u0 ? 0 : 1;                  // first or last block of the range
                float* mine = part + (((int64_t)blockIdx.x * 2 + slot_out) * CWARPS + warp) * (128 * NT);
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
                    *reinterpret_cast<float4*>(mine + nt * 128 + 4 * lane) =
                        make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
                __syncwarp();   // every lane's part is written before lane 0's release
                const int64_t c_lo = split.owner(rb * nsb), c_hi = split.owner((rb + 1) * nsb - 1);
                uint32_t old = 0;
                if (lane == 0) old = atom_add_acq_rel(cnt + rb * CWARPS + warp, 1u);
                old = __shfl_sync(0xffffffffu, old, 0);
                __syncwarp();   // lane 0's acquire orders the other lanes' reads below
                if (old == (uint32_t)(c_hi - c_lo)) {
                    // the last of the row block's CTAs: add every CTA's part, in CTA order
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int j = 0; j < 4; j++) v[nt][j] = 0.0f;
                    for (int64_t q = c_lo; q <= c_hi; ++q) {
                        const int sq = (q == c_lo && split.start(q) / nsb != rb) ? 1 : 0;
                        const float* pq = part + ((q * 2 + sq) * CWARPS + warp) * (128 * NT);
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            const float4 p = __ldcg(reinterpret_cast<const float4*>(pq + nt * 128 + 4 * lane));
                            v[nt][0] += p.x, v[nt][1] += p.y, v[nt][2] += p.z, v[nt][3] += p.w;
                        }
                    }
                    store = true;
                }
            }
            if (store) {
                const int64_t ra = rb * ROWS + row, rc = ra + 8;
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const int ta = 8 * nt + 2 * t, tb = ta + 1;
                    if (ra < N && ta < M) dst[(int64_t)ta * ldd + ra] = v[nt][0];
                    if (ra < N && tb < M) dst[(int64_t)tb * ldd + ra] = v[nt][1];
                    if (rc < N && ta < M) dst[(int64_t)ta * ldd + rc] = v[nt][2];
                    if (rc < N && tb < M) dst[(int64_t)tb * ldd + rc] = v[nt][3];
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[nt][j] = 0.0f;
            seg0 = u + 1;
        }
    }
}

// ---- host side ----------------------------------------------------------------------------------

static int nt_of(int64_t M) { return (int)((M + 7) / 8); }
static int64_t nsb_of(int64_t K) { return (K + 255) / 256; }

struct Workspace {
    size_t act_off, cnt_off, part_off, total;
};
// ctas = the weight-streaming grid (its partial slots)
static Workspace workspace_layout(int64_t M, int64_t N, int64_t K, int64_t ctas) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const int nt = nt_of(M);
    Workspace l{};
    l.act_off = 0;
    l.cnt_off = al((size_t)nsb_of(K) * nt * CHUNK);
    l.part_off = l.cnt_off + al((size_t)((N + ROWS - 1) / ROWS) * CWARPS * 4);
    l.total = l.part_off + al((size_t)ctas * 2 * CWARPS * 128 * nt * 4);
    return l;
}

static int64_t grid_of(int64_t N, int64_t K) {
    const int64_t units = ((N + ROWS - 1) / ROWS) * nsb_of(K);
    return std::max<int64_t>(1, std::min<int64_t>((int64_t)device_sm_count(), units));
}

template <int WT>
static cudaError_t launch_prep(const float* src1, int64_t lda, int64_t M, int64_t K, uint8_t* act, uint32_t* cnt,
                               int64_t n_cnt, cudaStream_t st) {
    const int nt = nt_of(M), nsb = (int)nsb_of(K);
    const bool vec = (reinterpret_cast<uintptr_t>(src1) & 15u) == 0 && lda % 4 == 0;
    const int warps = nt * 8 * nsb;
    const dim3 grid((unsigned)std::max(1, (warps + 7) / 8)), block(256);
    return vec ? launch_pdl(gw_prep_kernel<WT, true>, grid, block, 0, st, src1, lda, (int)M, (int)K, nsb, nt, act,
                            cnt, n_cnt)
               : launch_pdl(gw_prep_kernel<WT, false>, grid, block, 0, st, src1, lda, (int)M, (int)K, nsb, nt, act,
                            cnt, n_cnt);
}

template <int WT, int NT>
static cudaError_t launch_stream(const CUtensorMap& tmW, const CUtensorMap& tmD, int64_t N, int nsb,
                                 const uint8_t* act, int M, float* dst, int64_t ldd, int64_t grid, uint32_t* cnt,
                                 float* part, int* err, cudaStream_t st) {
    using C = Cfg<WT, NT>;
    const int stages = std::max(2, std::min(MAX_STAGES, SMEM_BUDGET / C::STAGE));
    const size_t smem = (size_t)stages * C::STAGE;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(gw_kernel<WT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BUDGET);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return launch_pdl(gw_kernel<WT, NT>, dim3((unsigned)grid), dim3(THREADS), smem, st, tmW, tmD, N, nsb, act, M,
                      dst, ldd, stages, cnt, part, err);
}

template <int WT>
static cudaError_t launch_all(const float* src1, int64_t lda, int64_t M, int64_t K, const CUtensorMap& tmW,
                              const CUtensorMap& tmD, int64_t N, float* dst, int64_t ldd, int64_t grid,
                              const Workspace& l, char* ws, int* err, cudaStream_t st) {
    uint8_t* act = reinterpret_cast<uint8_t*>(ws + l.act_off);
    uint32_t* cnt = reinterpret_cast<uint32_t*>(ws + l.cnt_off);
    float* part = reinterpret_cast<float*>(ws + l.part_off);
    const int64_t n_cnt = ((N + ROWS - 1) / ROWS) * CWARPS;
    cudaError_t e = launch_prep<WT>(src1, lda, M, K, act, cnt, n_cnt, st);
    if (e != cudaSuccess) return e;
    const int nsb = (int)nsb_of(K), m = (int)M;
    switch (nt_of(M)) {
        case 1: return launch_stream<WT, 1>(tmW, tmD, N, nsb, act, m, dst, ldd, grid, cnt, part, err, st);
        case 2: return launch_stream<WT, 2>(tmW, tmD, N, nsb, act, m, dst, ldd, grid, cnt, part, err, st);
        case 3: return launch_stream<WT, 3>(tmW, tmD, N, nsb, act, m, dst, ldd, grid, cnt, part, err, st);
        default: return launch_stream<WT, 4>(tmW, tmD, N, nsb, act, m, dst, ldd, grid, cnt, part, err, st);
    }
}

}  // namespace gw

size_t mul_mat_vec_tiles_workspace(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || M > gw::MMAX || N <= 0 || K <= 0) return 0;
    return gw::workspace_layout(M, N, K, gw::grid_of(N, K)).total;
}

int mul_mat_vec_tiles(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda,
                      int64_t M, float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err,
                      cudaStream_t st) {
    if (!w_packed || !src1 || !dst || !dev_err || N <= 0 || K <= 0 || M <= 0 || lda < K || ldd < N)
        return B200_E_INVALID;
    const bool k_ok = wtype == WT_Q8_0 ? K % 32 == 0 : (wtype == WT_Q4_K || wtype == WT_Q6_K) && K % 256 == 0;
    if (!k_ok || M > gw::MMAX || N > (1ll << 30) || K > (1 << 28) ||
        (reinterpret_cast<uintptr_t>(w_packed) & 15u) != 0)
        return B200_E_UNSUPPORTED;
    const int64_t grid = gw::grid_of(N, K);
    const gw::Workspace l = gw::workspace_layout(M, N, K, grid);
    if (!workspace || workspace_bytes < l.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return B200_E_INVALID;
    CUtensorMap tmW, tmD;
    if (!make_weight_tile_maps(wtype, w_packed, N, K, &tmW, &tmD)) return B200_E_CUDA;
    char* ws = static_cast<char*>(workspace);
    cudaError_t e;
    switch (wtype) {
        case WT_Q4_K: e = gw::launch_all<WT_Q4_K>(src1, lda, M, K, tmW, tmD, N, dst, ldd, grid, l, ws, dev_err, st); break;
        case WT_Q6_K: e = gw::launch_all<WT_Q6_K>(src1, lda, M, K, tmW, tmD, N, dst, ldd, grid, l, ws, dev_err, st); break;
        default: e = gw::launch_all<WT_Q8_0>(src1, lda, M, K, tmW, tmD, N, dst, ldd, grid, l, ws, dev_err, st); break;
    }
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // namespace b200
