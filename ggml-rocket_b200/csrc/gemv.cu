// Decode-size MUL_MAT (M = 1..8 token rows) over Q4_K weights: a weight-streaming kernel on the
// CUDA cores, for the shapes the tensor-core GEMM's tiles cannot fill.
//
// dst[m, n] = sum_k a[m, k] * W[n, k], W the packed (native) Q4_K rows. With M this small the op
// is bound by reading W once from HBM, so the kernel is built to keep HBM busy and to spend as
// few instructions per weight as it can:
//   * the dot product is taken per 32-weight sub-block in the factored form
//       sum_i (d*sc * q_i - dmin*m) * a_i = d*sc * sum_i q_i a_i - dmin*m * sum_i a_i,
//     the sub-block sums of a taken as the activations are loaded, so a weight costs one
//     nibble-to-float conversion and one FMA per token row;
//   * lane (r, j) of a warp reads chunk j (64 weights, 32 bytes of qs) of the super-blocks of
//     rows r, r + 8, ... (4 rows up to two token rows, 2 above): each activation value it loads
//     feeds all of them, and the 8 lanes sharing j load the same addresses (a broadcast);
//   * the 8 warps of a CTA split a row block's super-blocks (stride 8) and add their partials in
//     warp order through shared memory: the result does not depend on timing; each warp has
//     the next super-block's bytes requested before it uses the current one.
// The arithmetic is ggml's dequantize_row_q4_K (ggml-rocket.cpp:3894-3907 calls it through
// to_float) followed by an fp32 dot product; only the order of the fp32 sums differs from a
// decode-then-dot loop.
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"
#include "quant.cuh"

namespace b200 {

constexpr int GV_ROWS = 8;     // weight rows per warp (and per CTA)
constexpr int GV_KSPLIT = 8;   // warps per CTA, splitting the super-blocks of the row block

// Four nibble codes (the low nibbles of x's bytes, 0..15) as floats, two per f32x2 word.
__device__ __forceinline__ void q4_codes(uint32_t x, float (&q)[4]) {
    const uint64_t MAG = f2_pack(-8388608.0f, -8388608.0f);
    f2_unpack(f2_add(magic_pair(x, 0), MAG), q[0], q[1]);
    f2_unpack(f2_add(magic_pair(x, 1), MAG), q[2], q[3]);
}

template <int MR, bool VEC>
__device__ __forceinline__ float4 act4(const float* __restrict__ a, int64_t lda, int m, int k) {
    const float* p = a + (int64_t)m * lda + k;
    if constexpr (VEC) return __ldg(reinterpret_cast<const float4*>(p));
    return make_float4(__ldg(p), __ldg(p + 1), __ldg(p + 2), __ldg(p + 3));
}

// Rows per lane: each activation load feeds RPL weight rows (RPL = 4 up to two token rows, 2
// above, to stay inside the register file).
template <int MR>
constexpr int gv_rpl() { return MR <= 2 ? 4 : 2; }

template <int MR, bool VEC>
__global__ void __launch_bounds__(32 * GV_KSPLIT, MR == 1 ? 2 : 1) gemv_q4k_kernel(const uint8_t* __restrict__ w, int64_t N,
                                                                     int K, const float* __restrict__ a, int64_t lda,
                                                                     int M, float* __restrict__ dst, int64_t ldd) {
    constexpr int RPL = gv_rpl<MR>();
    constexpr int BLOCK = GV_ROWS * RPL;                // weight rows per CTA
    grid_dep_wait();   // programmatic launch: the activations may be the previous kernel's output
    grid_dep_launch();
    __shared__ float red[GV_KSPLIT][BLOCK][MR];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = lane >> 2, j = lane & 3;
    const int64_t n0 = (int64_t)blockIdx.x * BLOCK;
    const int nsb = K / 256;
    const int64_t row_bytes = (int64_t)nsb * 144;
    // lane (r, j) owns rows n0 + r + GV_ROWS * q, q < RPL (a row past N reads row N - 1)
    const uint8_t* rows[RPL];
#pragma unroll
    for (int q = 0; q < RPL; q++) {
        const int64_t n = n0 + r + GV_ROWS * q;
        rows[q] = w + (n < N ? n : N - 1) * row_bytes;
    }
    float acc[RPL][MR];
#pragma unroll
    for (int q = 0; q < RPL; q++)
#pragma unroll
        for (int m = 0; m < MR; m++) acc[q][m] = 0.0f;
    // this lane's 48 bytes of a super-block of each of its rows: header and 32-byte qs chunk; the
    // next super-block's are requested before this one's are used
    uint4 hdr[RPL], qa[RPL], qb[RPL], nhdr[RPL], nqa[RPL], nqb[RPL];
    auto load = [&](int sb, uint4(&h)[RPL], uint4(&x)[RPL], uint4(&y)[RPL]) {
#pragma unroll
        for (int q = 0; q < RPL; q++) {
            const uint8_t* blk = rows[q] + (int64_t)sb * 144;
            h[q] = __ldg(reinterpret_cast<const uint4*>(blk));
            x[q] = __ldg(reinterpret_cast<const uint4*>(blk + 16 + 32 * j));
            y[q] = __ldg(reinterpret_cast<const uint4*>(blk + 32 + 32 * j));
        }
    };
    if (warp < nsb) load(warp, hdr, qa, qb);
    for (int sb = warp; sb < nsb; sb += GV_KSPLIT) {
        if (sb + GV_KSPLIT < nsb) load(sb + GV_KSPLIT, nhdr, nqa, nqb);
        const int k0 = sb * 256 + 64 * j;
        float s_lo[RPL][MR], s_hi[RPL][MR], as_lo[MR], as_hi[MR];
#pragma unroll
        for (int q = 0; q < RPL; q++)
#pragma unroll
            for (int m = 0; m < MR; m++) s_lo[q][m] = s_hi[q][m] = 0.0f;
#pragma unroll
        for (int m = 0; m < MR; m++) as_lo[m] = as_hi[m] = 0.0f;
#pragma unroll
        for (int w4 = 0; w4 < 8; w4++) {
            float4 al[MR], ah[MR];
#pragma unroll
            for (int m = 0; m < MR; m++) {
                // token rows past M read row M - 1 (in bounds) and are never stored
                const int mr = m < M ? m : M - 1;
                al[m] = act4<MR, VEC>(a, lda, mr, k0 + 4 * w4);
                ah[m] = act4<MR, VEC>(a, lda, mr, k0 + 32 + 4 * w4);
                // the sub-block sums of the activations, added in index order
                as_lo[m] = as_lo[m] + al[m].x + al[m].y + al[m].z + al[m].w;
                as_hi[m] = as_hi[m] + ah[m].x + ah[m].y + ah[m].z + ah[m].w;
            }
#pragma unroll
            for (int q = 0; q < RPL; q++) {
                const uint32_t word = (w4 < 4 ? (&qa[q].x)[w4] : (&qb[q].x)[w4 - 4]);
                float lo[4], hi[4];
                q4_codes(word & 0x0F0F0F0Fu, lo);             // bytes 4*w4 .. 4*w4+3, low nibbles
                q4_codes((word >> 4) & 0x0F0F0F0Fu, hi);      // and their high nibbles
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    s_lo[q][m] = fmaf(lo[0], al[m].x, s_lo[q][m]);
                    s_lo[q][m] = fmaf(lo[1], al[m].y, s_lo[q][m]);
                    s_lo[q][m] = fmaf(lo[2], al[m].z, s_lo[q][m]);
                    s_lo[q][m] = fmaf(lo[3], al[m].w, s_lo[q][m]);
                    s_hi[q][m] = fmaf(hi[0], ah[m].x, s_hi[q][m]);
                    s_hi[q][m] = fmaf(hi[1], ah[m].y, s_hi[q][m]);
                    s_hi[q][m] = fmaf(hi[2], ah[m].z, s_hi[q][m]);
                    s_hi[q][m] = fmaf(hi[3], ah[m].w, s_hi[q][m]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < RPL; q++) {
            uint32_t sc0, mn0, sc1, mn1;
            q4k_sm(2 * j, hdr[q].y, hdr[q].z, hdr[q].w, sc0, mn0);
            q4k_sm(2 * j + 1, hdr[q].y, hdr[q].z, hdr[q].w, sc1, mn1);
            const float d = h2f_bits(hdr[q].x), dmin = h2f_bits(hdr[q].x >> 16);
            const float d_lo = __fmul_rn(d, (float)sc0), m_lo = __fmul_rn(dmin, (float)mn0);
            const float d_hi = __fmul_rn(d, (float)sc1), m_hi = __fmul_rn(dmin, (float)mn1);
#pragma unroll
            for (int m = 0; m < MR; m++)
                acc[q][m] += d_lo * s_lo[q][m] + d_hi * s_hi[q][m] - (m_lo * as_lo[m] + m_hi * as_hi[m]);
            hdr[q] = nhdr[q];
            qa[q] = nqa[q];
            qb[q] = nqb[q];
        }
    }
    // each row's four chunks (lanes j = 0..3), then the CTA's K slices in warp order
#pragma unroll
    for (int q = 0; q < RPL; q++)
#pragma unroll
        for (int m = 0; m < MR; m++) {
            acc[q][m] += __shfl_xor_sync(0xffffffffu, acc[q][m], 1);
            acc[q][m] += __shfl_xor_sync(0xffffffffu, acc[q][m], 2);
        }
    if (j == 0) {
#pragma unroll
        for (int q = 0; q < RPL; q++)
#pragma unroll
            for (int m = 0; m < MR; m++) red[warp][r + GV_ROWS * q][m] = acc[q][m];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < BLOCK * MR; i += blockDim.x) {
        const int rr = i / MR, mm = i % MR;
        const int64_t nn = n0 + rr;
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < GV_KSPLIT; q++) v += red[q][rr][mm];
        if (nn < N && mm < M) dst[(int64_t)mm * ldd + nn] = v;
    }
}

template <int MR>
static cudaError_t launch_gemv_q4k(bool vec, const uint8_t* w, int64_t N, int K, const float* a, int64_t lda, int M,
                                   float* dst, int64_t ldd, cudaStream_t st) {
    constexpr int BLOCK = GV_ROWS * gv_rpl<MR>();
    const dim3 grid((unsigned)((N + BLOCK - 1) / BLOCK)), block(32 * GV_KSPLIT);
    return vec ? launch_pdl(gemv_q4k_kernel<MR, true>, grid, block, 0, st, w, N, K, a, lda, M, dst, ldd)
               : launch_pdl(gemv_q4k_kernel<MR, false>, grid, block, 0, st, w, N, K, a, lda, M, dst, ldd);
}

}  // namespace b200

extern "C" {

size_t b200_mul_mat_vec_workspace_size(int64_t M, int64_t K) {
    (void)M;
    (void)K;
    return 0;   // the kernel needs no scratch; the argument is kept for callers that size one
}

int b200_mul_mat_vec(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda, int64_t M,
                     float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    using namespace b200;
    if (!w_packed || !src1 || !dst || !dev_err || N <= 0 || K <= 0 || M <= 0 || lda < K || ldd < N)
        return B200_E_INVALID;
    if (wtype != WT_Q4_K || K % 256 != 0 || M > 8 || N > (1ll << 30) || K > (1 << 28)) return B200_E_UNSUPPORTED;
    (void)workspace;
    (void)workspace_bytes;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool vec = (reinterpret_cast<uintptr_t>(src1) & 15u) == 0 && lda % 4 == 0;
    const uint8_t* w = static_cast<const uint8_t*>(w_packed);
    cudaError_t e;
    if (M == 1) e = launch_gemv_q4k<1>(vec, w, N, (int)K, src1, lda, (int)M, dst, ldd, st);
    else if (M == 2) e = launch_gemv_q4k<2>(vec, w, N, (int)K, src1, lda, (int)M, dst, ldd, st);
    else if (M <= 4) e = launch_gemv_q4k<4>(vec, w, N, (int)K, src1, lda, (int)M, dst, ldd, st);
    else e = launch_gemv_q4k<8>(vec, w, N, (int)K, src1, lda, (int)M, dst, ldd, st);
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // extern "C"
