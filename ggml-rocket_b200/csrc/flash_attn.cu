// FLASH_ATTN_EXT prefill on sm_100a (the reference's ggml_backend_rocket_flash_attn,
// ggml-rocket.cpp:5444-5691, without its gathers, host softmax or range fallback).
//
// Three kernels:
//   q_pack     Q F32 [D, T, H] (strided) -> Q16 [H][T][D] fp16 holding scale*q, with a per-row
//              power-of-two divisor for rows whose scaled values leave fp16's range; the
//              divisor is multiplied back into that row's scores.
//   mask_flags per (token block, 128-key block) of the F16 mask: all -inf (skipped), all zero
//              (no mask loads), or mixed. Causal prefill skips ~half the key blocks.
//   fa_kernel  one CTA per (group of GP query heads that share a KV head, TQ tokens) = 128 query
//              rows. Per key block: S = Q.K^T by tcgen05 into one of two TMEM buffers; 256
//              softmax threads (two per row, 64 keys each, the row max exchanged through shared
//              memory) read S from TMEM once, keep the online max / sum in fp32 (log2 units),
//              write P (fp16) to shared memory; O += P.V by tcgen05 accumulates in TMEM for the
//              whole key range, rescaled in place only when a row max grows by more than 2^8.
//              K and V tiles arrive by TMA straight from the op's strided cache views, two
//              stages deep.
#include <algorithm>
#include <cstdint>
#include <cstring>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int FA_ROWS = 128;      // query rows per CTA (tcgen05 M)
constexpr int FA_KB = 128;        // keys per block (tcgen05 N of Q.K^T, K of P.V)
constexpr int FA_SPLIT = 2;                          // softmax threads per query row
constexpr int FA_SOFTMAX_WARPS = 4 * FA_SPLIT;
constexpr int FA_THREADS = 64 + 32 * FA_SOFTMAX_WARPS;   // warp 0 TMA, warp 1 MMA, then softmax
constexpr float FA_RESCALE_LOG2 = 8.0f;   // rescale O only when the row max grows by more than 2^8
enum : uint8_t { MF_MIXED = 0, MF_ZERO = 1, MF_MASKED = 2 };

struct FaArgs {
    const float* qscale;       // [H*T] per-row divisor (1 unless out of fp16 range)
    const uint16_t* mask;      // F16 mask or nullptr
    int64_t m_stride;          // mask row stride, elements
    bool mask_vec;             // rows 16-byte aligned: 16-byte loads
    const uint8_t* flags;      // [n_tb][n_kvb]
    float* dst;                // [T][H][DV]
    int T, H, KV, HK, GP, TQ, n_hg, n_tb, n_kvb;
    float softcap;
    int* err;
};

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared-memory descriptor of an MN-major operand in 128-byte-swizzled rows: 64 MN elements per
// 128-byte row, rows (K) 128 B apart, 8-row groups 1024 B apart, 64-element MN groups `lbo` apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

__host__ __device__ constexpr uint32_t idesc_f16_f32_bmn(int M, int N) {
    return idesc_f16_f32(M, N) | (1u << 16);   // B operand MN-major
}

// 32 mask values (fp16 bits) of one row starting at key k0; keys at or past KV read as 0
// (the score of such a key is forced to -inf separately).
__device__ __forceinline__ void load_mask32(const uint16_t* mrow, int k0, int KV, bool vec, uint4 (&mv)[4]) {
    if (vec && k0 + 32 <= KV) {
        const uint4* mp = reinterpret_cast<const uint4*>(mrow + k0);
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) mv[q4] = __ldg(mp + q4);
    } else {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
            const uint32_t lo = (k0 + e < KV) ? (uint32_t)__ldg(mrow + k0 + e) : 0u;
            const uint32_t hi = (k0 + e + 1 < KV) ? (uint32_t)__ldg(mrow + k0 + e + 1) : 0u;
            w[e >> 1] = lo | (hi << 16);
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) mv[q4] = make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
    }
}

// ---------------------------------------------------------------------------------------------
// Set-up pass, one launch: CTAs [0, q_ctas) pack Q, one warp per (h, t) row; the rest classify
// the mask, one CTA per (token block, key block). Launched programmatically; the attention
// kernel that follows starts its prologue while this pass drains.
// ---------------------------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void fa_q_pack_row(const float* __restrict__ q, int64_t q_nb1, int64_t q_nb2, int T,
                                              int H, float scale, __half* __restrict__ q16,
                                              float* __restrict__ qscale, int row, int lane) {
    if (row >= H * T) return;
    const int h = row / T, t = row % T;
    const float* src = reinterpret_cast<const float*>(reinterpret_cast<const char*>(q) + (int64_t)t * q_nb1 +
                                                      (int64_t)h * q_nb2);
    constexpr int PER = D / 32;
    float x[PER];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; i++) {
        x[i] = scale * __ldg(src + lane * PER + i);
        amax = fmaxf(amax, fabsf(x[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float div = 1.0f, inv = 1.0f;
    if (amax > 65504.0f && amax <= 3.0e38f) {
        int e;
        frexpf(amax / 65504.0f, &e);        // amax / 2^e <= 65504
        div = ldexpf(1.0f, e);
        inv = ldexpf(1.0f, -e);
    }
    __half* dst = q16 + ((int64_t)h * T + t) * D + lane * PER;
#pragma unroll
    for (int i = 0; i < PER; i += 2) {
        const uint32_t w = pack_half2(x[i] * inv, x[i + 1] * inv);
        *reinterpret_cast<uint32_t*>(dst + i) = w;
    }
    if (lane == 0) qscale[row] = div;
}

// 256 threads: thread (token row trow of every 32, 16-key segment key_seg) of one 128-key block.
// With 16-byte aligned mask rows a segment is two 16-byte loads.
__device__ __forceinline__ void fa_mask_block(const uint16_t* __restrict__ mask, int64_t m_stride, bool vec, int T,
                                              int KV, int TQ, int tb, int j, int n_kvb, uint8_t* __restrict__ flags) {
    const int key_seg = threadIdx.x & 7;          // 16 keys each
    const int trow = threadIdx.x >> 3;            // 32 token rows per pass
    const int key0 = j * FA_KB + key_seg * 16;
    const bool full_seg = key0 + 16 <= KV;
    bool all_masked = true, all_zero = key0 < KV && full_seg;
    for (int tr = trow; tr < TQ; tr += 32) {
        const int t = tb * TQ + tr;
        if (t >= T) continue;
        const uint16_t* mrow = mask + (int64_t)t * m_stride + key0;
        if (vec && full_seg) {
            const uint4 a = __ldg(reinterpret_cast<const uint4*>(mrow));
            const uint4 b = __ldg(reinterpret_cast<const uint4*>(mrow) + 1);
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (w[i] != 0xFC00FC00u) all_masked = false;         // two -inf
                if ((w[i] & 0x7FFF7FFFu) != 0) all_zero = false;     // two +-0
            }
        } else {
            for (int i = 0; i < 16; i++) {
                if (key0 + i >= KV) break;
                const uint16_t v = __ldg(mrow + i);
                if (v != 0xFC00u) all_masked = false;
                if ((v & 0x7FFFu) != 0) all_zero = false;
            }
        }
    }
    const int am = __syncthreads_and(all_masked ? 1 : 0);
    const int az = __syncthreads_and(all_zero ? 1 : 0);
    if (threadIdx.x == 0) flags[(int64_t)tb * n_kvb + j] = am ? MF_MASKED : (az ? MF_ZERO : MF_MIXED);
}

template <int D>
__global__ void __launch_bounds__(256) fa_prep_kernel(const float* __restrict__ q, int64_t q_nb1, int64_t q_nb2,
                                                      int T, int H, float scale, __half* __restrict__ q16,
                                                      float* __restrict__ qscale, int q_ctas,
                                                      const uint16_t* __restrict__ mask, int64_t m_stride,
                                                      bool mask_vec, int KV, int TQ, int n_kvb, int n_tb,
                                                      uint8_t* __restrict__ flags) {
    grid_dep_wait();          // q and the mask may be the previous kernel's output
    grid_dep_launch();
    if ((int)blockIdx.x < q_ctas) {
        fa_q_pack_row<D>(q, q_nb1, q_nb2, T, H, scale, q16, qscale, (int)(blockIdx.x * 8 + (threadIdx.x >> 5)),
                         (int)(threadIdx.x & 31));
        return;
    }
    const int mi = (int)blockIdx.x - q_ctas;
    if (!mask) {              // no mask: every block is all zero (one CTA writes them)
        if (mi == 0)
            for (int i = threadIdx.x; i < n_tb * n_kvb; i += blockDim.x) flags[i] = MF_ZERO;
        return;
    }
    fa_mask_block(mask, m_stride, mask_vec, T, KV, TQ, mi / n_kvb, mi % n_kvb, n_kvb, flags);
}

// A P row segment of N 32-bit columns (2N fp16 keys) into TMEM.
template <int N>
__device__ __forceinline__ void tmem_st_p(uint32_t taddr, const uint32_t (&w)[N]) {
    if constexpr (N == 64) {
        tmem_st32(taddr, reinterpret_cast<const uint32_t(&)[32]>(w[0]));
        tmem_st32(taddr + 32u, reinterpret_cast<const uint32_t(&)[32]>(w[32]));
    } else if constexpr (N == 32) {
        tmem_st32(taddr, w);
    } else {
        static_assert(N == 16, "P segments are 16, 32 or 64 columns");
        tmem_st16(taddr, w);
    }
}

// ---------------------------------------------------------------------------------------------
// The attention kernel.
// ---------------------------------------------------------------------------------------------
template <int D, int DV>
struct FaCfg {
    static constexpr int Q_BYTES = FA_ROWS * D * 2;
    static constexpr int K_BYTES = FA_KB * D * 2;
    static constexpr int V_BYTES = FA_KB * DV * 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_K = OFF_Q + Q_BYTES;
    static constexpr int OFF_V = OFF_K + 2 * K_BYTES;
    // exchange between the FA_SPLIT threads of a row: maxima [2][SPLIT][128] f32 and their
    // sequence numbers (same shape, int), then sums [SPLIT][128] + sequence numbers
    static constexpr int XCH_MAX = 2 * FA_SPLIT * 128 * 4;
    static constexpr int XCH_SUM = FA_SPLIT * 128 * 4;
    static constexpr int OFF_XCH = OFF_V + 2 * V_BYTES;
    static constexpr int OFF_BAR = OFF_XCH + 2 * XCH_MAX + 2 * XCH_SUM;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
    // TMEM columns: S0 [0,128) | S1 [128,256) | O [256, 256+DV) | P0 [384,448) | P1 [448,512)
    // (P is fp16, two keys per 32-bit column, read by the P.V MMA as its A operand)
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t P_TMEM0 = 384;
    static constexpr uint32_t IDESC_S = idesc_f16_f32(FA_ROWS, FA_KB);
    static constexpr uint32_t IDESC_O = idesc_f16_f32_bmn(FA_ROWS, DV);
};

template <int D, int DV>
__global__ void __launch_bounds__(FA_THREADS, 1)
fa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
          const __grid_constant__ CUtensorMap tmV, const FaArgs args) {
    using C = FaCfg<D, DV>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sb = smem_u32(smem);
    const uint32_t bar = sb + C::OFF_BAR;
    const uint32_t q_full = bar;
    auto k_full = [&](int s) { return bar + 8u * (1 + s); };
    auto k_empty = [&](int s) { return bar + 8u * (3 + s); };
    auto v_full = [&](int s) { return bar + 8u * (5 + s); };
    auto v_empty = [&](int s) { return bar + 8u * (7 + s); };
    auto s_full = [&](int s) { return bar + 8u * (9 + s); };
    auto s_empty = [&](int s) { return bar + 8u * (11 + s); };
    // P of blocks b, b+2, ... written (per parity: a softmax warp may run one block ahead of
    // another, never two, because P buffer b is reused only after the P.V two blocks back)
    auto p_full = [&](int b) { return bar + 8u * (17 + b); };
    auto pv_done = [&](int b) { return bar + 8u * (14 + b); };   // P.V of blocks b, b+2, ... completed
    const uint32_t drain = bar + 8u * 16;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * 19);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 8 * 19 + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // heavier (later) token blocks first
    const int tb = args.n_tb - 1 - (int)(blockIdx.x / args.n_hg);
    const int hg = (int)(blockIdx.x % args.n_hg);
    const int G = args.H / args.HK;
    const int hk = (hg * args.GP) / G;
    const uint8_t* flags = args.flags + (int64_t)tb * args.n_kvb;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(k_full(s), 1);
            mbar_init(k_empty(s), 1);
            mbar_init(v_full(s), 1);
            mbar_init(v_empty(s), 1);
            mbar_init(s_full(s), 1);
            mbar_init(s_empty(s), FA_SOFTMAX_WARPS);
        }
        mbar_init(p_full(0), FA_SOFTMAX_WARPS);
        mbar_init(p_full(1), FA_SOFTMAX_WARPS);
        mbar_init(pv_done(0), 1);
        mbar_init(pv_done(1), 1);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    {
        int* seqs = reinterpret_cast<int*>(smem + C::OFF_XCH + C::XCH_MAX);
        for (int k = threadIdx.x; k < 2 * FA_SPLIT * 128; k += FA_THREADS) seqs[k] = 0;
        int* seql = reinterpret_cast<int*>(smem + C::OFF_XCH + 2 * C::XCH_MAX + C::XCH_SUM);
        for (int k = threadIdx.x; k < FA_SPLIT * 128; k += FA_THREADS) seql[k] = 0;
    }
    tc_fence_before();
    cta_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The prologue above overlapped the set-up pass (programmatic launch): Q16, its row divisors
    // and the mask flags are that pass's output, so wait for it before the first read.
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, C::Q_BYTES);
            for (int c = 0; c < D / 64; c++)
                tma_load_3d(sb + C::OFF_Q + c * (FA_ROWS * 128), &tmQ, q_full, c * 64, tb * args.TQ, hg * args.GP);
            int i = 0;
            bool ok = true;
            int k_issued[2] = {-1, -1}, v_issued[2] = {-1, -1};
            for (int j = 0; j < args.n_kvb && ok; j++) {
                if (flags[j] == MF_MASKED) continue;
                const int s = i & 1;
                const uint32_t ph = (uint32_t)(i >> 1) & 1u;
                if (!mbar_wait(k_empty(s), ph ^ 1u, args.err, ERR_WAIT_PRODUCER, abort_flag)) { ok = false; break; }
                k_issued[s] = (int)ph;
                mbar_arrive_expect_tx(k_full(s), C::K_BYTES);
                for (int c = 0; c < D / 64; c++)
                    tma_load_3d(sb + C::OFF_K + s * C::K_BYTES + c * (FA_KB * 128), &tmK, k_full(s), c * 64, j * FA_KB, hk);
                if (!mbar_wait(v_empty(s), ph ^ 1u, args.err, ERR_WAIT_PRODUCER, abort_flag)) { ok = false; break; }
                v_issued[s] = (int)ph;
                mbar_arrive_expect_tx(v_full(s), C::V_BYTES);
                for (int c = 0; c < DV / 64; c++)
                    tma_load_3d(sb + C::OFF_V + s * C::V_BYTES + c * (FA_KB * 128), &tmV, v_full(s), c * 64, j * FA_KB, hk);
                i++;
            }
            if (!ok) {   // let every copy already issued land before the CTA exits
                bool drained = mbar_drain(q_full, 0);
                for (int s = 0; s < 2; s++) {
                    if (k_issued[s] >= 0) drained &= mbar_drain(k_full(s), (uint32_t)k_issued[s]);
                    if (v_issued[s] >= 0) drained &= mbar_drain(v_full(s), (uint32_t)v_issued[s]);
                }
                if (!drained) atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = mbar_wait(q_full, 0, args.err, ERR_WAIT_MMA, abort_flag);
            tc_fence_after();
            int n_active = 0;
            auto issue_pv = [&](int i) -> bool {
                const int s = i & 1;
                const uint32_t ph = (uint32_t)(i >> 1) & 1u;
                if (!mbar_wait(p_full(i & 1), (uint32_t)(i >> 1) & 1u, args.err, ERR_WAIT_MMA, abort_flag)) return false;
                if (!mbar_wait(v_full(s), ph, args.err, ERR_WAIT_MMA, abort_flag)) return false;
                tc_fence_after();
                const uint32_t vb = sb + C::OFF_V + s * C::V_BYTES;
                const uint32_t p_tmem = tmem + C::P_TMEM0 + (uint32_t)(64 * (i & 1));
#pragma unroll
                for (int ks = 0; ks < FA_KB / 16; ks++) {
                    const uint64_t bdesc = sdesc_mn_sw128(vb + ks * 2048, FA_KB * 128);
                    mma_f16_ts(tmem + 256, p_tmem + 8u * ks, bdesc, C::IDESC_O, (i > 0 || ks > 0) ? 1u : 0u);
                }
                mma_commit(pv_done(i & 1));
                mma_commit(v_empty(s));
                return true;
            };
            for (int j = 0; j < args.n_kvb && ok; j++) {
                if (flags[j] == MF_MASKED) continue;
                const int i = n_active;
                const int s = i & 1;
                const uint32_t ph = (uint32_t)(i >> 1) & 1u;
                if (!mbar_wait(k_full(s), ph, args.err, ERR_WAIT_MMA, abort_flag)) { ok = false; break; }
                if (!mbar_wait(s_empty(s), ph ^ 1u, args.err, ERR_WAIT_MMA, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t kb = sb + C::OFF_K + s * C::K_BYTES;
#pragma unroll
                for (int ks = 0; ks < D / 16; ks++) {
                    const uint64_t a = sdesc_k_sw128(sb + C::OFF_Q + (ks >> 2) * (FA_ROWS * 128) + (ks & 3) * 32);
                    const uint64_t bdesc = sdesc_k_sw128(kb + (ks >> 2) * (FA_KB * 128) + (ks & 3) * 32);
                    mma_f16(tmem + (uint32_t)(s * FA_KB), a, bdesc, C::IDESC_S, ks > 0 ? 1u : 0u);
                }
                mma_commit(s_full(s));
                mma_commit(k_empty(s));
                n_active++;
                if (i > 0 && !issue_pv(i - 1)) { ok = false; break; }
            }
            if (ok && n_active > 0) issue_pv(n_active - 1);
            mma_commit(drain);
            if (!mbar_drain(drain, 0)) atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
        }
    } else {
        // ---------------- softmax / output: FA_SPLIT threads per query row ----------------
        // Warps w, w+4, ... share TMEM lane quarter (w & 3); thread (row r, part pt) owns keys
        // [KPT*pt, KPT*(pt+1)) of every block and O columns [OPT*pt, OPT*(pt+1)). Scores are kept
        // in log2 units. O accumulates in TMEM across blocks (P.V MMAs with accumulate); it is
        // rescaled only when a row's max grows by more than 2^FA_RESCALE_LOG2 over the max the
        // exponentials were taken against (so P <= 2^8 and nothing overflows).
        constexpr int KPT = FA_KB / FA_SPLIT;            // keys per thread per block
        constexpr int OPT = DV / FA_SPLIT;               // O columns per thread
        const int quad = warp & 3;
        const int pt = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int g = r / args.TQ, tq = r % args.TQ;
        const int h = hg * args.GP + g;
        const int t = tb * args.TQ + tq;
        const bool row_valid = t < args.T;
        const float qs = row_valid ? __ldg(args.qscale + (int64_t)h * args.T + t) : 1.0f;
        const uint16_t* mrow = (args.mask && row_valid) ? args.mask + (int64_t)t * args.m_stride : nullptr;
        const float LOG2E = 1.4426950408889634f;
        const float c2 = qs * LOG2E;                     // raw score -> log2 units
        const float softcap = args.softcap;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t o_tmem = tmem + lane_base + 256u + (uint32_t)(pt * OPT);
        volatile float* xv = reinterpret_cast<volatile float*>(smem + C::OFF_XCH);
        volatile int* xs = reinterpret_cast<volatile int*>(smem + C::OFF_XCH + C::XCH_MAX);
        volatile float* xl = reinterpret_cast<volatile float*>(smem + C::OFF_XCH + 2 * C::XCH_MAX);
        volatile int* xls = reinterpret_cast<volatile int*>(smem + C::OFF_XCH + 2 * C::XCH_MAX + C::XCH_SUM);
        // this thread's keys of a block are P columns [KPT/2*pt, KPT/2*(pt+1)) of the P buffer
        const uint32_t p_lane = tmem + lane_base + C::P_TMEM0 + (uint32_t)(pt * (KPT / 2));
        // wait until the P.V MMA of block k has completed (pv_done[k & 1], completion k >> 1)
        auto wait_pv = [&](int k) {
            return mbar_wait(pv_done(k & 1), (uint32_t)(k >> 1) & 1u, args.err, ERR_WAIT_EPILOGUE, abort_flag);
        };
        // Publish a value to the other threads of this row and wait for theirs: a bounded spin on
        // sequence numbers in shared memory (the threads are in different warps). vals[k] gets
        // part k's value.
        auto exchange = [&](volatile float* v, volatile int* sq, float mine, int seq, float (&vals)[FA_SPLIT]) -> bool {
            v[pt * 128 + r] = mine;
            __threadfence_block();
            sq[pt * 128 + r] = seq;
            const uint64_t t0 = globaltimer();
            uint32_t n = 0;
#pragma unroll
            for (int k = 0; k < FA_SPLIT; k++) {
                while (sq[k * 128 + r] != seq) {
                    if ((++n & 255u) == 0) {
                        if (*abort_flag) return false;
                        if (globaltimer() - t0 > B200_WAIT_LIMIT_NS) {
                            atomicCAS(args.err, 0, ERR_WAIT_EPILOGUE);
                            *abort_flag = 1;
                            return false;
                        }
                    }
                }
            }
            __threadfence_block();
#pragma unroll
            for (int k = 0; k < FA_SPLIT; k++) vals[k] = v[k * 128 + r];
            return true;
        };
        float m = -INFINITY;                             // running max (log2 units)
        float l = 0.0f;                                  // this thread's partial row sum
        int i = 0;
        bool ok = true;
        for (int j = 0; j < args.n_kvb && ok; j++) {
            const uint8_t fl = flags[j];
            if (fl == MF_MASKED) continue;
            const bool use_mask = (fl == MF_MIXED) && (mrow != nullptr);
            const bool general = use_mask || softcap != 0.0f || (j + 1) * FA_KB > args.KV;
            const int s = i & 1;
            const uint32_t ph = (uint32_t)(i >> 1) & 1u;
            if (!mbar_wait(s_full(s), ph, args.err, ERR_WAIT_EPILOGUE, abort_flag)) { ok = false; break; }
            tc_fence_after();
            float x[KPT];
#pragma unroll
            for (int c0 = 0; c0 < KPT; c0 += 32) {
                uint32_t rv[32];
                tmem_ld32(tmem + lane_base + (uint32_t)(s * FA_KB + pt * KPT + c0), rv);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; e++) x[c0 + e] = __uint_as_float(rv[e]);
            }
            // S is in registers: the buffer may take the next Q.K^T
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty(s));
            const int k0 = j * FA_KB + pt * KPT;
            float bmax = -INFINITY;
            if (!general) {
#pragma unroll
                for (int e = 0; e < KPT; e++) bmax = fmaxf(bmax, x[e]);
                bmax *= c2;
            } else {
#pragma unroll
                for (int c0 = 0; c0 < KPT; c0 += 32) {
                    uint4 mv[4];
                    if (use_mask) load_mask32(mrow, k0 + c0, args.KV, args.mask_vec, mv);
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        float sv = x[c0 + e] * qs;
                        if (softcap != 0.0f) sv = softcap * tanhf(sv / softcap);
                        sv *= LOG2E;
                        if (use_mask) {
                            const uint32_t mw = (&mv[e >> 3].x)[(e & 7) >> 1];
                            const uint16_t mb = (uint16_t)((e & 1) ? (mw >> 16) : (mw & 0xFFFFu));
                            sv = fmaf(__half2float(__ushort_as_half(mb)), LOG2E, sv);
                        }
                        if (k0 + c0 + e >= args.KV) sv = -INFINITY;
                        x[c0 + e] = sv;
                        bmax = fmaxf(bmax, sv);
                    }
                }
            }
            // the row max over all parts (double-buffered by block parity)
            float maxes[FA_SPLIT];
            if (!exchange(xv + (i & 1) * (FA_SPLIT * 128), xs + (i & 1) * (FA_SPLIT * 128), bmax, i + 1, maxes)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int k = 0; k < FA_SPLIT; k++) bmax = fmaxf(bmax, maxes[k]);
            const bool grow = bmax > m + FA_RESCALE_LOG2;
            const float m_new = grow ? bmax : m;
            const float alpha = (grow && m != -INFINITY) ? ex2_approx(m - m_new) : 1.0f;
            // O is rescaled in place only after the previous block's P.V has landed in it
            if (i > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                if (!wait_pv(i - 1)) { ok = false; break; }
                tc_fence_after();
                {
#pragma unroll
                    for (int c0 = 0; c0 < OPT; c0 += 16) {
                        uint32_t ov[16];
                        tmem_ld16(o_tmem + (uint32_t)c0, ov);
                        tmem_ld_wait();
#pragma unroll
                        for (int e = 0; e < 16; e++) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                        tmem_st16(o_tmem + (uint32_t)c0, ov);
                    }
                    tmem_st_wait();
                }
            }
            l *= alpha;
            m = m_new;
            const float mu = (m == -INFINITY) ? 0.0f : m;
            uint32_t pw[KPT / 2];
            if (!general) {
#pragma unroll
                for (int e = 0; e < KPT; e += 2) {
                    const float p0 = ex2_approx(fmaf(x[e], c2, -mu));
                    const float p1 = ex2_approx(fmaf(x[e + 1], c2, -mu));
                    l += p0 + p1;
                    pw[e >> 1] = pack_half2(p0, p1);
                }
            } else {
#pragma unroll
                for (int e = 0; e < KPT; e += 2) {
                    const float p0 = ex2_approx(x[e] - mu);
                    const float p1 = ex2_approx(x[e + 1] - mu);
                    l += p0 + p1;
                    pw[e >> 1] = pack_half2(p0, p1);
                }
            }
            // P buffer (i & 1) is free once the P.V of block i-2 has completed
            if (i >= 2) {
                if (!wait_pv(i - 2)) { ok = false; break; }
                tc_fence_after();
            }
            tmem_st_p<KPT / 2>(p_lane + (uint32_t)(64 * (i & 1)), pw);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full(i & 1));
            i++;
        }
        bool have_o = false;
        if (ok && i > 0) {
            have_o = wait_pv(i - 1);
            tc_fence_after();
        }
        // row sum over all parts, added in part order so every thread of the row agrees
        float sums[FA_SPLIT];
        if (ok && !exchange(xl, xls, l, 1, sums)) ok = false;
        float l_tot = 0.0f;
#pragma unroll
        for (int k = 0; k < FA_SPLIT; k++) l_tot += sums[k];
        if (ok && have_o) {
            const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
            float* out = args.dst + ((int64_t)t * args.H + h) * DV + pt * OPT;
#pragma unroll
            for (int c0 = 0; c0 < OPT; c0 += 16) {
                uint32_t ov[16];
                tmem_ld16(o_tmem + (uint32_t)c0, ov);
                tmem_ld_wait();
                if (row_valid) {
#pragma unroll
                    for (int e = 0; e < 16; e += 4)
                        *reinterpret_cast<float4*>(out + c0 + e) =
                            make_float4(__uint_as_float(ov[e]) * inv, __uint_as_float(ov[e + 1]) * inv,
                                        __uint_as_float(ov[e + 2]) * inv, __uint_as_float(ov[e + 3]) * inv);
                }
            }
        } else if (ok && row_valid) {
            // no key block survived the mask: the row is all zeros
            float* out = args.dst + ((int64_t)t * args.H + h) * DV + pt * OPT;
            for (int c = 0; c < OPT; c += 4) *reinterpret_cast<float4*>(out + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }

    tc_fence_before();
    cta_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------------------------

static bool make_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t nb1,
                             uint64_t nb2, uint32_t b0, uint32_t b1, uint32_t b2);

struct FaLayout {
    int GP, TQ, n_hg, n_tb, n_kvb;
    size_t q16_off, qs_off, flags_off, total;
};

static FaLayout fa_layout(int D, int T, int H, int KV, int HK) {
    FaLayout L{};
    const int G = H / HK;
    int gp = 1;
    while (gp * 2 <= 16 && G % (gp * 2) == 0) gp *= 2;
    L.GP = gp;
    L.TQ = FA_ROWS / gp;
    L.n_hg = H / gp;
    L.n_tb = (T + L.TQ - 1) / L.TQ;
    L.n_kvb = (KV + FA_KB - 1) / FA_KB;
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    L.q16_off = 0;
    L.qs_off = al((size_t)H * T * D * 2);
    L.flags_off = L.qs_off + al((size_t)H * T * 4);
    L.total = L.flags_off + al((size_t)L.n_tb * L.n_kvb);
    return L;
}

template <int D, int DV>
static cudaError_t launch_fa(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FaArgs& a,
                             int grid, cudaStream_t st) {
    using C = FaCfg<D, DV>;
    static bool set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fa_kernel<D, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        set[dev] = true;
    }
    return launch_pdl(fa_kernel<D, DV>, dim3((unsigned)grid), dim3(FA_THREADS), C::SMEM, st, tq, tk, tv, a);
}

int flash_attn_impl(const float* q, int64_t q_nb1, int64_t q_nb2, const void* k, int64_t k_nb1, int64_t k_nb2,
                    const void* v, int64_t v_nb1, int64_t v_nb2, const void* mask, int64_t m_nb1, float* dst, int D,
                    int DV, int T, int H, int KV, int HK, float scale, float max_bias, float softcap, void* workspace,
                    size_t ws_bytes, int* dev_err, cudaStream_t st) {
    if (!q || !k || !v || !dst || !dev_err || T <= 0 || H <= 0 || KV <= 0 || HK <= 0) return B200_E_INVALID;
    if (H % HK != 0 || max_bias != 0.0f) return B200_E_UNSUPPORTED;
    if (!((D == 64 || D == 128) && (DV == 64 || DV == 128))) return B200_E_UNSUPPORTED;
    if ((k_nb1 | k_nb2 | v_nb1 | v_nb2) % 16 != 0) return B200_E_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(dst)) & 15u)
        return B200_E_UNSUPPORTED;
    if (mask && ((m_nb1 % 2) != 0 || (reinterpret_cast<uintptr_t>(mask) & 1u))) return B200_E_UNSUPPORTED;
    const FaLayout L = fa_layout(D, T, H, KV, HK);
    if (!workspace || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return B200_E_WORKSPACE;
    char* ws = static_cast<char*>(workspace);
    __half* q16 = reinterpret_cast<__half*>(ws + L.q16_off);
    float* qs = reinterpret_cast<float*>(ws + L.qs_off);
    uint8_t* flags = reinterpret_cast<uint8_t*>(ws + L.flags_off);

    {
        const int q_ctas = (H * T + 7) / 8;
        const int m_ctas = mask ? L.n_tb * L.n_kvb : 1;
        const bool mvec = mask && (m_nb1 % 16) == 0 && (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
        const dim3 grid((unsigned)(q_ctas + m_ctas)), block(256);
        const uint16_t* m16 = static_cast<const uint16_t*>(mask);
        const cudaError_t e = D == 64
            ? launch_pdl(fa_prep_kernel<64>, grid, block, 0, st, q, q_nb1, q_nb2, T, H, scale, q16, qs, q_ctas, m16,
                         (int64_t)(m_nb1 / 2), mvec, KV, L.TQ, L.n_kvb, L.n_tb, flags)
            : launch_pdl(fa_prep_kernel<128>, grid, block, 0, st, q, q_nb1, q_nb2, T, H, scale, q16, qs, q_ctas, m16,
                         (int64_t)(m_nb1 / 2), mvec, KV, L.TQ, L.n_kvb, L.n_tb, flags);
        if (e != cudaSuccess) return B200_E_CUDA;
    }

    CUtensorMap tq, tk, tv;
    if (!make_tmap_3d_f16(&tq, q16, D, T, H, (uint64_t)D * 2, (uint64_t)T * D * 2, 64, L.TQ, L.GP)) return B200_E_CUDA;
    if (!make_tmap_3d_f16(&tk, k, D, KV, HK, k_nb1, k_nb2, 64, FA_KB, 1)) return B200_E_CUDA;
    if (!make_tmap_3d_f16(&tv, v, DV, KV, HK, v_nb1, v_nb2, 64, FA_KB, 1)) return B200_E_CUDA;
    FaArgs a{};
    a.qscale = qs;
    a.mask = static_cast<const uint16_t*>(mask);
    a.m_stride = m_nb1 / 2;
    a.mask_vec = mask && (m_nb1 % 16) == 0 && (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
    a.flags = flags;
    a.dst = dst;
    a.T = T;
    a.H = H;
    a.KV = KV;
    a.HK = HK;
    a.GP = L.GP;
    a.TQ = L.TQ;
    a.n_hg = L.n_hg;
    a.n_tb = L.n_tb;
    a.n_kvb = L.n_kvb;
    a.softcap = softcap;
    a.err = dev_err;
    const int grid = L.n_hg * L.n_tb;
    cudaError_t e;
    if (D == 128 && DV == 128) e = launch_fa<128, 128>(tq, tk, tv, a, grid, st);
    else if (D == 64 && DV == 64) e = launch_fa<64, 64>(tq, tk, tv, a, grid, st);
    else if (D == 128 && DV == 64) e = launch_fa<128, 64>(tq, tk, tv, a, grid, st);
    else e = launch_fa<64, 128>(tq, tk, tv, a, grid, st);
    return e == cudaSuccess ? B200_OK : B200_E_CUDA;
}

}  // namespace b200

// The 3-D fp16 tensor map [d2][d1][d0] with byte strides nb1, nb2 and a 128-byte-swizzled box.
namespace b200 {
using EncodeTiledFn3 = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static bool make_tmap_3d_f16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t nb1,
                             uint64_t nb2, uint32_t b0, uint32_t b1, uint32_t b2) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    static EncodeTiledFn3 fn = nullptr;
    if (!fn) {
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return false;
        fn = reinterpret_cast<EncodeTiledFn3>(p);
    }
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {nb1, nb2};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace b200

namespace b200 {

// ---- a quantized KV cache (Q8_0 / Q4_0) as the fp16 tiles the kernel reads ----------------------
// One thread per 32-value block of a [HK][KV][D] view (rows nb1 bytes apart, heads nb2): ggml's
// dequantize_row_q8_0 / _q4_0 (y = q * d, resp. (nibble - 8) * d, in f32), then fp16 (nearest
// even), written contiguous [HK][KV][D]. Blocks are 2-byte aligned only: byte loads.
template <int TYPE>
__global__ void kv_to_f16_kernel(const uint8_t* __restrict__ src, int64_t D, int64_t KV, int64_t HK, int64_t nb1,
                                 int64_t nb2, __half* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t per_row = D / 32, total = HK * KV * per_row;
    constexpr int BYTES = TYPE == 8 ? 34 : 18;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = i % per_row, r = (i / per_row) % KV, h = i / (per_row * KV);
        const uint8_t* b = src + h * nb2 + r * nb1 + c * BYTES;
        const float d = __half2float(__ushort_as_half((unsigned short)(b[0] | (b[1] << 8))));
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
            float v0, v1;
            if constexpr (TYPE == 8) {
                v0 = __fmul_rn((float)(int8_t)b[2 + e], d);
                v1 = __fmul_rn((float)(int8_t)b[3 + e], d);
            } else {   // Q4_0: element j < 16 is the low nibble of byte j, j >= 16 the high nibble of byte j - 16
                const int j0 = e, j1 = e + 1;
                const int q0 = j0 < 16 ? (b[2 + j0] & 0x0f) : (b[2 + j0 - 16] >> 4);
                const int q1 = j1 < 16 ? (b[2 + j1] & 0x0f) : (b[2 + j1 - 16] >> 4);
                v0 = __fmul_rn((float)(q0 - 8), d);
                v1 = __fmul_rn((float)(q1 - 8), d);
            }
            w[e / 2] = (uint32_t)__half_as_ushort(__float2half_rn(v0)) |
                       ((uint32_t)__half_as_ushort(__float2half_rn(v1)) << 16);
        }
        uint4* o = reinterpret_cast<uint4*>(dst + (h * KV + r) * D + 32 * c);
#pragma unroll
        for (int q = 0; q < 4; q++) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
}

}  // namespace b200

extern "C" {

int b200_kv_to_f16(int type, const void* src, int64_t D, int64_t KV, int64_t HK, int64_t nb1, int64_t nb2, void* dst,
                   void* stream) {
    using namespace b200;
    if (!src || !dst || D <= 0 || KV <= 0 || HK <= 0 || nb1 <= 0 || nb2 <= 0) return B200_E_INVALID;
    if ((type != 8 && type != 2) || D % 32 != 0 || (reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
        return B200_E_UNSUPPORTED;
    const int64_t total = HK * KV * (D / 32);
    const int threads = 256;
    const int64_t want = (total + threads - 1) / threads;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)device_sm_count() * 16));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e =
        type == 8 ? launch_pdl(kv_to_f16_kernel<8>, dim3(grid), dim3(threads), 0, st,
                               static_cast<const uint8_t*>(src), D, KV, HK, nb1, nb2, static_cast<__half*>(dst))
                  : launch_pdl(kv_to_f16_kernel<2>, dim3(grid), dim3(threads), 0, st,
                               static_cast<const uint8_t*>(src), D, KV, HK, nb1, nb2, static_cast<__half*>(dst));
    return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA;
}


size_t b200_flash_attn_workspace_size(int D, int DV, int T, int H, int KV, int HK) {
    (void)DV;
    if (T <= 0 || H <= 0 || KV <= 0 || HK <= 0 || H % HK) return 0;
    return b200::fa_layout(D, T, H, KV, HK).total;
}

int b200_flash_attn_ext(const float* q, int64_t q_nb1, int64_t q_nb2, const void* k, int64_t k_nb1, int64_t k_nb2,
                        const void* v, int64_t v_nb1, int64_t v_nb2, const void* mask, int64_t m_nb1, float* dst,
                        int D, int DV, int T, int H, int KV, int HK, float scale, float max_bias, float softcap,
                        void* workspace, size_t workspace_bytes, int* dev_err, void* stream) {
    return b200::flash_attn_impl(q, q_nb1, q_nb2, k, k_nb1, k_nb2, v, v_nb1, v_nb2, mask, m_nb1, dst, D, DV, T, H, KV,
                                 HK, scale, max_bias, softcap, workspace, workspace_bytes, dev_err,
                                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
