// The MUL_MAT kernel family: dst[M,N] = s[m] * (A16[M,K] . W[N,K]^T) on the sm_100a tensor
// cores, with fp32 accumulation in TMEM.
//
// Operand roles ("swap AB"): the tcgen05 M dimension (128 lanes of TMEM) runs over WEIGHT
// rows n and the tcgen05 N dimension over TOKENS t. The accumulator for one tile therefore
// holds D[n, t] with lane = n, and the epilogue's 32 lanes of a warp write 32 consecutive n
// of one output row t: every store is a coalesced 128-byte line of ggml's dst (ne0 = N
// contiguous). Small token counts (M = 32..64) keep the full 128-row weight tile.
//
// Warp roles in one CTA (persistent over work units):
//   warp 0        TMA producer: the activation tile [BT x 64] (and the F16 weight tile)
//   warp 1        TMEM allocator and the single-thread tcgen05.mma issuer
//   warps 2..5    epilogue: TMEM -> registers -> scaled f32 stores (or split-K partials)
//   warps 6..9    (quantized weights only) dequant producers: each thread decodes one
//                 weight row's 64-weight chunk to fp16 and writes it, 128-byte swizzled,
//                 straight into the stage the MMA reads -- no fp16 weight copy in HBM.
// Two TMEM accumulators alternate, so the epilogue of one unit overlaps the next unit's
// main loop. Every wait is bounded (ptx.cuh).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "ptx.cuh"
#include "quant.cuh"

namespace b200 {

constexpr int GEMM_BN = 128;   // weight rows per tile (tcgen05 M)
constexpr int GEMM_BK = 64;    // K per pipeline stage (one 128-byte swizzle row of fp16)

struct GemmArgs {
    const uint8_t* w;          // packed weight plane A (quantized types)
    const uint16_t* wd;        // packed weight plane D (Q6_K / Q8_0 scales)
    int64_t w_row_bytes;       // plane A row stride, bytes
    int64_t wd_row_elems;      // plane D row stride, fp16 elements
    const float* scales;       // [M] per-token activation scale
    float* out;                // dst (splits == 1) or split-K partials
    int64_t ldo;               // row stride of out, floats
    int64_t split_stride;      // floats between split-K partial planes
    int M, N, K;
    int n_tiles_n, n_tiles_t, splits, kb_per_split, nkb, num_units;
    int* err;                  // device error word
    // grouped (MUL_MAT_ID) mode: the token rows are sorted by expert; expert e owns rows
    // [g_off[e], g_off[e+1]) of A16 and weight rows [e*N, (e+1)*N) of the packed stack.
    const int32_t* g_off;          // [n_expert + 1]
    const int32_t* g_tile_start;   // [n_expert + 1] prefix of ceil(rows_e / BT)
    const int32_t* g_slot;         // sorted row -> expert slot
    const int32_t* g_tok;          // sorted row -> token
    int n_expert;
    int64_t d_nb1, d_nb2;          // dst strides over (slot, token), bytes
};

struct UnitCoords {
    int t0, t_end, n0, wrow0, ks, kb0, kb1;
};

template <int BT, int WT>
struct GemmCfg {
    static constexpr bool QUANT = (WT != WT_F16);
    static constexpr int A_BYTES = BT * GEMM_BK * 2;
    static constexpr int W_BYTES = GEMM_BN * GEMM_BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + W_BYTES;
    static constexpr int STAGES = (196608 / STAGE_BYTES) > 8 ? 8 : (196608 / STAGE_BYTES);
    static constexpr int THREADS = QUANT ? 320 : 192;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
    static constexpr uint32_t TMEM_COLS = 2 * BT;
    static constexpr uint32_t IDESC = idesc_f16_f32(GEMM_BN, BT);
};

template <int BT, int WT, bool GROUPED>
__global__ void __launch_bounds__(GemmCfg<BT, WT>::THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
            const GemmArgs args) {
    using C = GemmCfg<BT, WT>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_base = sbase + STAGES * C::STAGE_BYTES;
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
    uint8_t* misc = smem + STAGES * C::STAGE_BYTES + 8 * (2 * STAGES + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), C::QUANT ? 5 : 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), 4);
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        if (!C::QUANT) tma_prefetch_desc(&tmW);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int ntt = args.n_tiles_t, ntn = args.n_tiles_n;
    int num_units = args.num_units;
    if constexpr (GROUPED) num_units = __ldg(args.g_tile_start + args.n_expert) * ntn;
    auto unit_coords = [&](int u) {
        UnitCoords c;
        if constexpr (GROUPED) {
            const int tg = u / ntn;
            const int nt = u % ntn;
            int lo = 0, hi = args.n_expert;            // last e with tile_start[e] <= tg
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (__ldg(args.g_tile_start + mid) <= tg) lo = mid;
                else hi = mid;
            }
            const int e = lo;
            c.t0 = __ldg(args.g_off + e) + (tg - __ldg(args.g_tile_start + e)) * BT;
            c.t_end = __ldg(args.g_off + e + 1);
            c.n0 = nt * GEMM_BN;
            c.wrow0 = e * args.N + c.n0;
            c.ks = 0;
            c.kb0 = 0;
            c.kb1 = args.nkb;
        } else {
            const int tt = u % ntt;
            const int rest = u / ntt;
            const int nt = rest % ntn;
            c.ks = rest / ntn;
            c.t0 = tt * BT;
            c.t_end = args.M;
            c.n0 = nt * GEMM_BN;
            c.wrow0 = c.n0;
            c.kb0 = c.ks * args.kb_per_split;
            c.kb1 = min(args.nkb, c.kb0 + args.kb_per_split);
        }
        return c;
    };

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued_phase[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; s++) issued_phase[s] = -1;
            bool ok = true;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const UnitCoords uc = unit_coords(u);
                for (int kb = uc.kb0; kb < uc.kb1; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, args.err, ERR_WAIT_PRODUCER, abort_flag)) { ok = false; break; }
                    const uint32_t sa = sbase + stage * C::STAGE_BYTES;
                    mbar_arrive_expect_tx(full_bar(stage), C::QUANT ? C::A_BYTES : C::A_BYTES + C::W_BYTES);
                    tma_load_2d(sa, &tmA, full_bar(stage), kb * GEMM_BK, uc.t0);
                    if (!C::QUANT) tma_load_2d(sa + C::A_BYTES, &tmW, full_bar(stage), kb * GEMM_BK, uc.wrow0);
                    issued_phase[stage] = (int)phase;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {   // let every copy already issued land before the CTA exits
#pragma unroll
                for (int s = 0; s < STAGES; s++)
                    if (issued_phase[s] >= 0 && !mbar_drain(full_bar(s), (uint32_t)issued_phase[s]))
                        atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int lt = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, lt++) {
                const UnitCoords uc = unit_coords(u);
                const int kb0 = uc.kb0, kb1 = uc.kb1;
                const int acc = lt & 1;
                const uint32_t aphase = (uint32_t)(lt >> 1) & 1u;
                if (!mbar_wait(tempty_bar(acc), aphase ^ 1u, args.err, ERR_WAIT_MMA, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BT);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, args.err, ERR_WAIT_MMA, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = sbase + stage * C::STAGE_BYTES;
                    const uint32_t sw = sa + C::A_BYTES;
#pragma unroll
                    for (int k = 0; k < GEMM_BK / 16; k++) {
                        mma_f16(d_tmem, sdesc_k_sw128(sw + 32u * k), sdesc_k_sw128(sa + 32u * k), C::IDESC,
                                (kb > kb0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(empty_bar(stage));
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                mma_commit(tfull_bar(acc));
            }
            // Every MMA this thread issued has completed once drain_bar fires.
            mma_commit(drain_bar);
            if (!mbar_drain(drain_bar, 0)) atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
        }
    } else if (warp < 6) {
        // ---------------- epilogue ----------------
        const int q = warp & 3;                       // TMEM lane quadrant this warp may read
        int lt = 0;
        for (int u = blockIdx.x; u < num_units; u += gridDim.x, lt++) {
            const UnitCoords uc = unit_coords(u);
            const int acc = lt & 1;
            const uint32_t aphase = (uint32_t)(lt >> 1) & 1u;
            if (!mbar_wait(tfull_bar(acc), aphase, args.err, ERR_WAIT_EPILOGUE, abort_flag)) break;
            tc_fence_after();
            const int n = uc.n0 + 32 * q + lane;
            float* obase = args.out + (size_t)uc.ks * args.split_stride;
            const bool scaled = args.splits == 1;
            for (int c0 = 0; c0 < BT; c0 += 16) {
                if (uc.t0 + c0 >= uc.t_end) break;
                uint32_t r[16];
                tmem_ld16(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BT + c0), r);
                tmem_ld_wait();
                if (n < args.N) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int t = uc.t0 + c0 + j;
                        if (t < uc.t_end) {
                            float v = __uint_as_float(r[j]);
                            if (scaled) v *= __ldg(args.scales + t);
                            if constexpr (GROUPED) {
                                char* drow = reinterpret_cast<char*>(args.out) + (int64_t)__ldg(args.g_tok + t) * args.d_nb2 +
                                             (int64_t)__ldg(args.g_slot + t) * args.d_nb1;
                                reinterpret_cast<float*>(drow)[n] = v;
                            } else {
                                obase[(size_t)t * args.ldo + n] = v;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
        }
    } else {
        // ---------------- dequant producers (quantized weights) ----------------
        if constexpr (C::QUANT) {
            const int r = threadIdx.x - 192;          // weight row within the tile, 0..127
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const UnitCoords uc = unit_coords(u);
                const int n = uc.n0 + r;
                const int64_t wr = (int64_t)uc.wrow0 + r;
                const uint8_t* wrow = args.w + (size_t)wr * args.w_row_bytes;
                const uint16_t* drow = args.wd ? args.wd + (size_t)wr * args.wd_row_elems : nullptr;
                for (int kb = uc.kb0; kb < uc.kb1; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, args.err, ERR_WAIT_DEQUANT, abort_flag)) { ok = false; break; }
                    uint32_t h[32];
                    if (n < args.N) {
                        if constexpr (WT == WT_Q4_K) decode_q4k_chunk(wrow, kb, h);
                        else if constexpr (WT == WT_Q6_K) decode_q6k_chunk(wrow, drow, kb, h);
                        else decode_q8_0_chunk(wrow, drow, kb, h);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; i++) h[i] = 0u;
                    }
                    const uint32_t sw = sbase + stage * C::STAGE_BYTES + C::A_BYTES;
#pragma unroll
                    for (int c = 0; c < 8; c++)
                        st_shared_v4(sw + sw128_offset((uint32_t)r, (uint32_t)c), h[4 * c], h[4 * c + 1], h[4 * c + 2], h[4 * c + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(full_bar(stage));
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace b200
