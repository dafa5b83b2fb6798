// Decode-size MUL_MAT (M = 1..8 token rows) over Q4_K weights: a weight-streaming kernel whose
// dot products run on the warp-level tensor-core MMA, for the shapes the tcgen05 GEMM's 128-row
// tiles cannot fill.
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
//   * a CTA owns 16 weight rows; its 8 warps split the super-blocks into contiguous ranges, each
//     streaming its 16 x 144-byte super-block columns through a 4-deep cp.async ring in shared
//     memory, and add their partials in warp order (the result does not depend on timing).
// The activations are prepared once per call by gemv_act_kernel: per 256-value block, the
// block's absmax s and fp16(a / s) (the same per-row "sandwich" rule the GEMM's activation pack
// applies, here per block), stored in the MMA's k-slot order, plus the fp16 (hi, lo) sums of
// every 32-value sub-block.
//
// Numerics: weights are the exact Q4_K values (d*sc*q - dmin*m, from exact integer products and
// fp32 scales); products with the fp16 activations are exact in the MMA and summed in fp32. The
// only rounding beyond fp32 sums is the activations' fp16 rounding, as in the prefill GEMM.
// The decode is ggml's dequantize_row_q4_K (ggml-rocket.cpp:3894-3907 calls it through to_float).
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"

namespace b200 {

constexpr int GV_WARPS = 8;                      // warps per CTA, splitting the super-blocks
constexpr int GV_ROWS = 16;                      // weight rows per CTA (the MMA's M)
constexpr int GV_STAGES = 4;                     // super-block columns in flight per warp
constexpr int GV_STAGE = GV_ROWS * 144;          // one super-block of 16 rows, bytes
constexpr int GV_PIECES = GV_STAGE / 16;         // 16-byte copies per stage (144)
constexpr int GV_SMEM = GV_WARPS * GV_STAGES * GV_STAGE + GV_WARPS * GV_ROWS * 8 * 4;
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
template <bool VEC>
__global__ void __launch_bounds__(256) gemv_act_kernel(const float* __restrict__ a, int64_t lda, int M, int K,
                                                       __half* __restrict__ a16p, uint32_t* __restrict__ asum2,
                                                       float* __restrict__ scl) {
    grid_dep_wait();   // the previous kernel may still read this workspace (programmatic launch)
    grid_dep_launch();
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

// CTA = 16 weight rows n0 .. n0+15; warp w takes super-block columns [w nsb / 8, (w+1) nsb / 8).
// Lane (g, t) = (lane / 4, lane % 4) is the MMA's thread group g, thread t: it decodes qs chunk t
// (bytes 32t .. 32t+31) of rows n0+g and n0+g+8 and feeds token row g's activations; its
// accumulators are rows n0+g, n0+g+8 x token rows 2t, 2t+1.
__global__ void __launch_bounds__(32 * GV_WARPS, 2)
    gemv_q4k_kernel(const uint8_t* __restrict__ w, int64_t N, int K, const __half* __restrict__ a16p,
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
                const uint4 l = __ldg(ap + j), h = __ldg(ap + 4 + j);
                awl[4 * j] = l.x, awl[4 * j + 1] = l.y, awl[4 * j + 2] = l.z, awl[4 * j + 3] = l.w;
                awh[4 * j] = h.x, awh[4 * j + 1] = h.y, awh[4 * j + 2] = h.z, awh[4 * j + 3] = h.w;
            }
            as2 = __ldg(reinterpret_cast<const uint2*>(srow + (int64_t)sb * 8));
        } else {
#pragma unroll
            for (int j = 0; j < 16; j++) awl[j] = awh[j] = 0u;
        }
        const float2 s2 = __ldg(reinterpret_cast<const float2*>(scl + (int64_t)sb * GV_MMAX + 2 * t));
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

struct GvWorkspace {
    size_t a16_off, asum_off, scl_off, total;
};
static GvWorkspace gv_workspace(int64_t M, int64_t K) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    GvWorkspace l{};
    l.a16_off = 0;
    l.asum_off = al((size_t)M * K * 2);
    l.scl_off = l.asum_off + al((size_t)M * (K / 32) * 4);
    l.total = l.scl_off + al((size_t)(K / 256) * GV_MMAX * 4);
    return l;
}

}  // namespace b200

extern "C" {

size_t b200_mul_mat_vec_workspace_size(int64_t M, int64_t K) {
    if (M <= 0 || K <= 0) return 0;
    return b200::gv_workspace(M, K).total;
}

int b200_mul_mat_vec(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda, int64_t M,
                     float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    using namespace b200;
    if (!w_packed || !src1 || !dst || !dev_err || N <= 0 || K <= 0 || M <= 0 || lda < K || ldd < N)
        return B200_E_INVALID;
    if (wtype != WT_Q4_K || K % 256 != 0 || M > GV_MMAX || N > (1ll << 30) || K > (1 << 28))
        return B200_E_UNSUPPORTED;
    const GvWorkspace l = gv_workspace(M, K);
    if (!workspace || workspace_bytes < l.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
        return B200_E_INVALID;
    (void)dev_err;   // nothing in these kernels waits or can fail on the device
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(gemv_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_SMEM) != cudaSuccess)
            return B200_E_CUDA;
        attr_set[dev] = true;
    }
    char* ws = static_cast<char*>(workspace);
    __half* a16p = reinterpret_cast<__half*>(ws + l.a16_off);
    uint32_t* asum2 = reinterpret_cast<uint32_t*>(ws + l.asum_off);
    float* scl = reinterpret_cast<float*>(ws + l.scl_off);
    const bool vec = (reinterpret_cast<uintptr_t>(src1) & 15u) == 0 && lda % 4 == 0;
    const int warps = (int)(M * (K / 256));
    const dim3 pgrid((unsigned)((warps + 7) / 8)), pblock(256);
    cudaError_t e = vec ? launch_pdl(gemv_act_kernel<true>, pgrid, pblock, 0, st, src1, lda, (int)M, (int)K, a16p,
                                     asum2, scl)
                        : launch_pdl(gemv_act_kernel<false>, pgrid, pblock, 0, st, src1, lda, (int)M, (int)K, a16p,
                                     asum2, scl);
    if (e != cudaSuccess) return B200_E_CUDA;
    e = launch_pdl(gemv_q4k_kernel, dim3((unsigned)((N + GV_ROWS - 1) / GV_ROWS)), dim3(32 * GV_WARPS), GV_SMEM, st,
                   static_cast<const uint8_t*>(w_packed), N, (int)K, (const __half*)a16p, (const uint32_t*)asum2,
                   (const float*)scl, (int)M, dst, ldd);
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
