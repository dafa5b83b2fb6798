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
//   warp 0        TMA producer of the activation tile [BT x 64]
//   warp 1        TMEM allocator and the single-thread tcgen05.mma issuer
//   warps 2..5    epilogue: TMEM -> registers -> scaled into a 32 x 32 shared-memory box ->
//                 one TMA store per box (grouped mode: 16-byte stores of whole 128-byte lines
//                 of the scattered rows); a stream-K partial goes straight from registers
//   warp 6        TMA producer of the F16 weight tile, or (quantized weights) of the raw
//                 quantized super-block tile: 128 rows x 256 weights into a 2-3 deep ring,
//                 with the TMA's L2 prefetch running 4 super-blocks further ahead
//   (quantized weights only)
//   warps 7..14   dequant, two per scheduler:
//                 thread (row r, half h) decodes 32 weights of row r's 64-weight chunk from
//                 the ring to fp16 and writes them, 128-byte swizzled, straight into the
//                 stage the MMA reads -- no fp16 weight copy in HBM.
// Each producer thread only issues: one TMA or barrier operation costs it ~70-180 clocks, so
// the two operands have separate producers.
// Two TMEM accumulators alternate, so the epilogue of one unit overlaps the next unit's
// main loop. Every wait is bounded (ptx.cuh).
//
// Scheduling (plain MUL_MAT): stream-K. The K range of every 128 x BT output tile is cut into
// granules (one 64-wide K block for F16, one 256-weight super-block for quantized weights);
// the grid (at most one CTA per SM, all resident: cooperative launch) takes equal contiguous
// runs of the tile-after-tile granule sequence, so every SM gets the same number of K steps
// whatever the tile count -- no partial last wave. A tile split between CTAs is finished by
// the CTA holding its last granule, which adds the other CTAs' f32 partials in CTA order:
// deterministic, with no atomics and no second kernel. The finisher gathers those partials
// into its idle second TMEM accumulator while its own K range is still on the tensor core.
//
// Cluster split (plain MUL_MAT with at most one tile per two SMs, e.g. N = 4096 at M = 512): a
// cluster of two CTAs takes one tile, each CTA half of its K range. Stream-K would share every
// such tile between three or four CTAs, and when every piece ends together the partial tiles make
// three serial trips through L2 at the end of the launch (written, read back, the result
// written). Here the two halves meet over distributed shared memory instead: CTA r finishes
// tokens [r BT/2, (r+1) BT/2) of the tile; each epilogue warp sends the other half of its TMEM
// rows into the peer's idle operand stages (st.shared::cluster, mbarrier arrives at cluster
// scope), and adds what it receives to its own half. Addition of two terms commutes, so both
// halves of the tile carry the same sums whichever CTA adds them.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "ptx.cuh"
#include "quant.cuh"

namespace b200 {

constexpr int GEMM_BN = 128;   // weight rows per tile (tcgen05 M)
constexpr int GEMM_BK = 64;    // K per pipeline stage (one 128-byte swizzle row of fp16)
constexpr int GEMM_MAX_MEMBERS = 4;   // weights in one combined-N launch (a fused QKV group has 3)

struct GemmArgs {
    const float* scales;       // [M] per-token activation scale
    float* out;                // dst
    int64_t ldo;               // row stride of out, floats
    int M, N, K;
    int n_tiles_n, n_tiles_t, nkb;
    int* err;                  // device error word
    // Stream-K schedule (plain MUL_MAT): the K-granules of all tiles, tile after tile, are
    // split into gridDim.x contiguous ranges of equal length. A tile whose granules span
    // several CTAs is finished by the CTA holding its last granule (the "finisher"); every
    // other CTA holding part of it writes an unscaled f32 partial tile to its slot of
    // `partials` and publishes `epoch` in its flags. The finisher adds the partials in CTA
    // order, so the result does not depend on timing.
    float* partials;           // [gridDim.x][BT][128] f32
    uint32_t* flags;           // [gridDim.x][4] (one per epilogue warp)
    uint32_t epoch;            // unique per launch
    int gran;                  // K-blocks per granule (4 = one super-block for quantized weights)
    int tile_g;                // granules per tile
    int64_t total_g;           // n_tiles_n * n_tiles_t * tile_g
    // grouped (MUL_MAT_ID) mode: the token rows are sorted by expert; expert e owns rows
    // [g_off[e], g_off[e+1]) of A16 and weight rows [e*N, (e+1)*N) of the packed stack.
    const int32_t* g_off;          // [n_expert + 1]
    const int32_t* g_tile_start;   // [n_expert + 1] prefix of ceil(rows_e / BT)
    const int32_t* g_slot;         // sorted row -> expert slot
    const int32_t* g_tok;          // sorted row -> token
    int n_expert;
    int64_t d_nb1, d_nb2;          // dst strides over (slot, token), bytes
    // optional (expert parallelism over peer memory): sorted row -> index into out_bases, the
    // destination of that row (another GPU's buffer, reached by plain stores over NVLink)
    const int32_t* g_src;
    float* const* out_bases;
    // plain MUL_MAT with its weight rows split across GPUs: when n_dst > 0 every finished box
    // goes to all n_dst buffers out_bases[d] (this GPU's dst and the other GPUs', [M][ldo] f32),
    // at column col0 + n -- the all-gather done by the epilogue's own stores over NVLink
    int n_dst;
    int col0;
    // cluster split: 2 = the two CTAs of a cluster take the two K halves of each tile (launched in
    // clusters of two, grid = 2 x the clusters; no partials or flags), 0 = off
    int csplit;
    // combined-N launch (plain MUL_MAT, one CTA per tile): n_mem weights of the same type and K
    // against one packed activation, each with its own dst. Their 128-row weight tiles are laid
    // end to end: member m owns weight tiles [mem_t0[m], mem_t0[m + 1]) of the n_tiles_n (the
    // last member's end is n_tiles_n), and its weight, d plane and dst tensor maps are the
    // kernel's own maps for m = 0 and GemmMembers' entry m - 1 otherwise. n_mem = 1: one weight.
    int n_mem;
    int mem_t0[GEMM_MAX_MEMBERS];
};

// The tensor maps of a combined-N launch's members 1 .. n_mem - 1 (a kernel parameter, so the
// TMA reads them from parameter memory like the kernel's own maps).
struct GemmMembers {
    CUtensorMap w[GEMM_MAX_MEMBERS - 1], d[GEMM_MAX_MEMBERS - 1], o[GEMM_MAX_MEMBERS - 1];
};

// One work item of a CTA: a tile (or, in stream-K, the piece of a tile's K range this CTA owns).
struct UnitCoords {
    int t0, t_end, n0, wrow0, kb0, kb1;
    int mem;                   // combined-N launch: the member whose weight tile this is (n0, wrow0 are its own)
    bool finishes;             // this piece completes the tile: scale and store dst
    int c_first;               // first CTA holding a piece of this tile (partials c_first..blockIdx.x-1)
    int64_t next;              // cursor of the CTA's next item
};

// Raw quantized tile of one 256-weight super-block x 128 rows, as the TMA writes it.
template <int WT>
struct RawCfg {
    static constexpr int ROW = WT == WT_Q4_K ? 144 : WT == WT_Q6_K ? 208 : WT == WT_Q8_0 ? 272 : 0;   // bytes
    static constexpr int A_BYTES = ROW * GEMM_BN;
    static constexpr int D_BYTES = WT == WT_Q6_K ? GEMM_BN * 2 : 0;    // transposed d plane box
    static constexpr int STAGE = (A_BYTES + D_BYTES + 1023) / 1024 * 1024;
    // the ring covers L2 latency; the L2 prefetch ahead of it covers HBM latency
    static constexpr int STAGES = WT == WT_F16 ? 0 : WT == WT_Q4_K ? 3 : 2;
    static constexpr int PREFETCH = 4;                                   // super-blocks ahead into L2
    static constexpr int X_ELEMS = ROW / 2;                              // uint16 box width
};

// Warp roles: producers 0 and 6, MMA 1, epilogue 2-5, dequant 7-14. The eight dequant warps
// sit two per scheduler (warp % 4), the MMA warp's included: the decode is ALU-heavy, and three
// on one scheduler (beside an epilogue warp) made that scheduler the straggler every stage
// waits for (measured: 5-10 % slower).
constexpr int W_APROD = 0, W_MMA = 1, W_EPI0 = 2, W_WPROD = 6, W_DEQ0 = 7;
constexpr int DEQ_WARPS = 8;
__device__ __forceinline__ int dequant_slot(int warp) {
    return (warp >= W_DEQ0 && warp < W_DEQ0 + DEQ_WARPS) ? warp - W_DEQ0 : -1;
}

template <int BT, int WT, bool PAIR = false>
struct GemmCfg {
    static constexpr bool QUANT = (WT != WT_F16);
    // WIDE (BT = 512): one work unit is a 128-row weight tile against 512 tokens, two 256-token
    // halves sharing every decoded weight stage, so each weight is decoded once per 512 tokens
    // (twice as much tensor-core work per decoded weight as BT = 256). The two halves' fp32
    // accumulators fill the 512 TMEM columns: there is one accumulator, not two alternating ones.
    static constexpr bool WIDE = BT == 512;
    static constexpr int MMA_N = WIDE ? 256 : BT;        // tcgen05 N of one MMA
    static constexpr int N_ACC = WIDE ? 1 : 2;
    // A CTA pair splits the token tile: each CTA stages BT/2 activation rows.
    static constexpr int A_ROWS = PAIR ? BT / 2 : BT;
    static constexpr int A_BOX = WIDE ? 256 : A_ROWS;   // rows per activation TMA box (<= 256)
    static constexpr int A_BYTES = A_ROWS * GEMM_BK * 2;
    static constexpr int W_BYTES = GEMM_BN * GEMM_BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + W_BYTES;
    static constexpr int RAW_STAGES = QUANT ? (WIDE ? 2 : RawCfg<WT>::STAGES) : 0;
    static constexpr int RAW_TOTAL = RawCfg<WT>::STAGE * RAW_STAGES;
    static constexpr int EPI_BYTES = 4 * 32 * 32 * 4;          // a 32 x 32 f32 transpose tile per epilogue warp
    static constexpr int BUDGET = 232448 - 1024 - 512 - RAW_TOTAL - EPI_BYTES;
    static constexpr int STAGES = (BUDGET / STAGE_BYTES) > 8 ? 8 : (BUDGET / STAGE_BYTES);
    static constexpr int THREADS = QUANT ? (W_DEQ0 + DEQ_WARPS) * 32 : 7 * 32;
    static constexpr int DEQ_THREADS = DEQ_WARPS * 32;
    // 3 * STAGES + 11 barriers, the TMEM slot and abort flag, the cluster split's 16 barriers
    static constexpr int BAR_BYTES = 512;
    static constexpr int RAW_OFF = STAGES * STAGE_BYTES;
    static constexpr int EPI_OFF = RAW_OFF + RAW_TOTAL;
    static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
    static constexpr int SMEM = BAR_OFF + BAR_BYTES + 1024;
    static constexpr uint32_t TMEM_COLS = WIDE ? 512 : 2 * BT;
    static constexpr uint32_t IDESC = idesc_f16_f32(PAIR ? 2 * GEMM_BN : GEMM_BN, MMA_N);
    static constexpr int TILE_N = PAIR ? 2 * GEMM_BN : GEMM_BN;   // weight rows per work tile
    static_assert(STAGES >= 2, "pipeline too shallow");
    static_assert(8 * (3 * STAGES + 11) + 8 + 16 * 8 <= BAR_BYTES, "barrier area");
    // the cluster split's receive and send regions (four warps x two halves' rows) in the idle stages
    static constexpr bool CSPLIT_FITS = !WIDE && !PAIR && BT * 512 <= STAGES * STAGE_BYTES;
    static_assert(!(WIDE && PAIR), "the wide tile runs on one SM");
};

template <int BT, int WT, bool GROUPED, bool PAIR>
__global__ void __launch_bounds__(GemmCfg<BT, WT, PAIR>::THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
            const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmO, const GemmArgs args,
            const __grid_constant__ GemmMembers mm) {
    static_assert(!(GROUPED && PAIR), "the grouped GEMM runs one CTA per tile");
    static_assert(!(GROUPED && BT == 512), "the grouped GEMM's tiles are at most 256 rows of one expert");
    using C = GemmCfg<BT, WT, PAIR>;
    using RC = RawCfg<WT>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_base = sbase + C::BAR_OFF;
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = bar_base + 8u * (2 * STAGES + 4);
    auto rfull_bar = [&](int s) { return bar_base + 8u * (2 * STAGES + 5 + s); };
    auto rempty_bar = [&](int s) { return bar_base + 8u * (2 * STAGES + 8 + s); };
    // CTA pair, quantized weights: the peer's dequant warps arrive on a local barrier per stage and
    // one thread of the peer ("announcer") forwards each completed stage to the leader's full barrier
    // with a single cluster-scope arrive, so no dequant warp waits on a remote arrive
    auto pfull_bar = [&](int s) { return bar_base + 8u * (2 * STAGES + 11 + s); };
    uint8_t* misc = smem + C::BAR_OFF + 8 * (3 * STAGES + 11);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + 4);
    // cluster split: per epilogue warp q, xfree(q, 0) completes when the peer's warp q has its
    // receive region free (its main loop is over), xfull(q, 0) when the peer's bulk copy of its rows
    // of this CTA's half has landed in this CTA's region (slots (q, 1) are unused)
    const uint32_t xbar_base = bar_base + 8u * (3 * STAGES + 11) + 8u;
    auto xfull_bar = [&](int q, int sl) { return xbar_base + 8u * (2 * q + sl); };
    auto xfree_bar = [&](int q, int sl) { return xbar_base + 64u + 8u * (2 * q + sl); };
    const bool csplit = !GROUPED && C::CSPLIT_FITS && args.csplit == 2;
    const uint32_t xrank = csplit ? cluster_ctarank() : 0u;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CTA pair (2-SM MMA): the even CTA (leader) issues the MMAs and owns the full / tempty
    // barriers both CTAs feed; the MMA commits arrive in both CTAs.
    const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
    const bool leader = crank == 0;
    const int unit_id = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int n_units_grid = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    auto leader_addr = [&](uint32_t a) { return PAIR ? mapa_shared(a, 0) : a; };
    // arrive on the leader's copy of a barrier (a local arrive in the leader itself)
    auto arrive_leader = [&](uint32_t a) {
        if (!PAIR || leader) mbar_arrive(a);
        else mbar_arrive_cluster(mapa_shared(a, 0));
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            // quantized: the A TMA's expect_tx arrive + the local dequant warps (+ the peer's announcer)
            mbar_init(full_bar(s), C::QUANT ? 1 + DEQ_WARPS / 2 + (PAIR ? 1 : 0) : 2);
            mbar_init(empty_bar(s), 1);
            if (PAIR && C::QUANT) mbar_init(pfull_bar(s), DEQ_WARPS / 2);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(tfull_bar(a), 1);
            mbar_init(tempty_bar(a), PAIR ? 8 : 4);
        }
        for (int s = 0; s < C::RAW_STAGES; s++) {
            mbar_init(rfull_bar(s), 1);
            mbar_init(rempty_bar(s), DEQ_WARPS);
        }
        mbar_init(drain_bar, 1);
        if (csplit) {
            for (int i = 0; i < 8; i++) {
                mbar_init(xfull_bar(i >> 1, i & 1), 1);
                mbar_init(xfree_bar(i >> 1, i & 1), 1);
            }
        }
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        if (WT == WT_Q6_K) tma_prefetch_desc(&tmD);
        for (int m = 1; m < args.n_mem && !GROUPED; m++) {
            tma_prefetch_desc(&mm.w[m - 1]);
            if (WT == WT_Q6_K) tma_prefetch_desc(&mm.d[m - 1]);
        }
    }
    if (warp == W_MMA) {
        if constexpr (PAIR) {
            tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if (PAIR || csplit) cluster_sync();   // the peer's barriers exist before anything arrives on them
    else cta_sync();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int ntt = args.n_tiles_t, ntn = args.n_tiles_n;
    // Work cursor: the grouped mode walks units blockIdx.x, +gridDim.x, ...; stream-K walks this
    // CTA's granule range [g_beg, g_end) from its end backwards, so the pieces other CTAs finish
    // (at the end of the range) come first and the piece this CTA finishes, whose partials come
    // from lower-numbered CTAs, comes last.
    int64_t num_units = 0, g_beg = 0, g_end = 0;   // num_units (grouped): set after the wait below
    if constexpr (!GROUPED) {
        g_beg = (int64_t)unit_id * args.total_g / n_units_grid;
        g_end = (int64_t)(unit_id + 1) * args.total_g / n_units_grid;
    }
    // cluster split: cluster c takes tiles c, c + clusters, ...
    const int64_t n_tiles_all = (int64_t)ntn * ntt;
    const int64_t cursor0 = GROUPED ? (int64_t)blockIdx.x : csplit ? (int64_t)(blockIdx.x >> 1) : g_end;
    auto cursor_ok = [&](int64_t c) { return GROUPED ? c < num_units : csplit ? c < n_tiles_all : c > g_beg; };
    // combined-N launch: the member owning global weight tile nt, which becomes the member's own tile index
    auto member_of = [&](int& nt) {
        int m = 0, base = 0;
        if constexpr (!GROUPED) {
#pragma unroll
            for (int i = 1; i < GEMM_MAX_MEMBERS; i++) {
                if (i < args.n_mem && nt >= args.mem_t0[i]) {
                    m = i;
                    base = args.mem_t0[i];
                }
            }
        }
        nt -= base;
        return m;
    };
    auto wmap = [&](int m) { return m == 0 ? &tmW : &mm.w[m - 1]; };
    auto dmap = [&](int m) { return m == 0 ? &tmD : &mm.d[m - 1]; };
    auto omap = [&](int m) { return m == 0 ? &tmO : &mm.o[m - 1]; };
    auto unit_coords = [&](int64_t cur) {
        UnitCoords c;
        if constexpr (GROUPED) {
            const int tg = (int)(cur / ntn);
            const int nt = (int)(cur % ntn);
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
            c.mem = 0;
            c.kb0 = 0;
            c.kb1 = args.nkb;
            c.finishes = true;
            c.c_first = unit_id;
            c.next = cur + gridDim.x;
        } else if (csplit) {
            const int tt = (int)(cur % ntt);
            int nt = (int)(cur / ntt);
            c.mem = member_of(nt);
            c.t0 = tt * BT;
            c.t_end = args.M;
            c.n0 = nt * GEMM_BN;
            c.wrow0 = c.n0;
            // this CTA's half of the K range, in whole granules
            c.kb0 = (int)(((int64_t)args.tile_g * xrank) / 2) * args.gran;
            c.kb1 = min(args.nkb, (int)(((int64_t)args.tile_g * (xrank + 1)) / 2) * args.gran);
            c.finishes = true;
            c.c_first = unit_id;
            c.next = cur + (gridDim.x >> 1);
        } else {
            const int64_t tile = (cur - 1) / args.tile_g;
            const int64_t tstart = tile * args.tile_g;
            const int64_t s0 = tstart > g_beg ? tstart : g_beg;
            const int tt = (int)(tile % ntt);          // neighbouring tiles share a weight tile
            int nt = (int)(tile / ntt);
            c.mem = member_of(nt);
            c.t0 = tt * BT;
            c.t_end = args.M;
            c.n0 = nt * C::TILE_N + (int)crank * GEMM_BN;   // this CTA's 128 weight rows
            c.wrow0 = c.n0;
            c.kb0 = (int)(s0 - tstart) * args.gran;
            c.kb1 = min(args.nkb, (int)(cur - tstart) * args.gran);
            c.finishes = cur - tstart == args.tile_g;
            // the CTA whose range holds granule tstart: largest c with c*total/grid <= tstart
            c.c_first = (int)(((tstart + 1) * (int64_t)n_units_grid - 1) / args.total_g);
            c.next = s0;
        }
        return c;
    };

    // Everything above overlapped the previous kernel of the stream (programmatic launch). The
    // weights are not that kernel's output, so the weight producer first starts its first
    // tile's weights on their way into L2 (a prefetch only warms L2, the point of coherence, so
    // it cannot return stale data). From here on the grid reads and writes global memory: it
    // waits for the previous kernel to finish, then lets the next one begin its launch.
    if constexpr (!GROUPED) {
        if (warp == W_WPROD && lane == 0 && cursor_ok(cursor0)) {
            const UnitCoords uc = unit_coords(cursor0);
            if constexpr (C::QUANT) {
                const int sb0 = uc.kb0 >> 2, sb_end = (uc.kb1 + 3) >> 2;
                for (int pf = sb0; pf < sb0 + RC::PREFETCH && pf < sb_end; pf++)
                    tma_prefetch_l2_2d(wmap(uc.mem), pf * RC::X_ELEMS, uc.wrow0);
            } else {
                for (int kb = uc.kb0; kb < uc.kb0 + 2 * STAGES && kb < uc.kb1; kb++)
                    tma_prefetch_l2_2d(wmap(uc.mem), kb * GEMM_BK, uc.wrow0);
            }
        }
    }
    grid_dep_wait();
    grid_dep_launch();
    if constexpr (GROUPED) num_units = (int64_t)__ldg(args.g_tile_start + args.n_expert) * ntn;

    // One operand's TMA producer over the A/W stage ring (W only for F16 weights).
    auto produce_stages = [&](bool is_w) {
        int stage = 0;
        uint32_t phase = 0;
        int issued = -1;                                 // phase of the last issue per stage, packed
        uint32_t issued_mask = 0, issued_par = 0;
        bool ok = true;
        for (int64_t cur = cursor0; cursor_ok(cur) && ok;) {
            const UnitCoords uc = unit_coords(cur);
            cur = uc.next;
            for (int kb = uc.kb0; kb < uc.kb1; kb++) {
                if (!mbar_wait(empty_bar(stage), phase ^ 1u, args.err, ERR_WAIT_PRODUCER, abort_flag)) { ok = false; break; }
                const uint32_t sa = sbase + stage * C::STAGE_BYTES;
                if constexpr (PAIR) {
                    // both CTAs' tiles complete on the leader's barrier; the leader expects both
                    const uint32_t fb = leader_addr(full_bar(stage));
                    if (is_w) {
                        if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * C::W_BYTES);
                        tma_load_2d_pair(sa + C::A_BYTES, wmap(uc.mem), fb, kb * GEMM_BK, uc.wrow0);
                    } else {
                        if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * C::A_BYTES);
                        tma_load_2d_pair(sa, &tmA, fb, kb * GEMM_BK, uc.t0 + (int)crank * C::A_ROWS);
                    }
                } else if (is_w) {
                    mbar_arrive_expect_tx(full_bar(stage), C::W_BYTES);
                    tma_load_2d(sa + C::A_BYTES, wmap(uc.mem), full_bar(stage), kb * GEMM_BK, uc.wrow0);
                } else {
                    mbar_arrive_expect_tx(full_bar(stage), C::A_BYTES);
                    tma_load_2d(sa, &tmA, full_bar(stage), kb * GEMM_BK, uc.t0);
                    if constexpr (C::WIDE)   // the second 256-token half of the tile
                        tma_load_2d(sa + C::A_BYTES / 2, &tmA, full_bar(stage), kb * GEMM_BK, uc.t0 + C::A_BOX);
                }
                issued_mask |= 1u << stage;
                issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
        }
        (void)issued;
        if (!ok && (!PAIR || leader)) {   // let every copy already issued land before the CTA exits
            for (int s = 0; s < STAGES; s++)
                if (((issued_mask >> s) & 1u) && !mbar_drain(full_bar(s), (issued_par >> s) & 1u))
                    atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
        }
    };

    if (warp == W_APROD) {
        if (lane == 0) produce_stages(false);
    } else if (warp == W_WPROD) {
        if (lane == 0) {
            if constexpr (!C::QUANT) {
                produce_stages(true);
            } else {
                // ---------------- raw quantized tiles ----------------
                int rs = 0;
                uint32_t rph = 0;
                uint32_t issued_mask = 0, issued_par = 0;
                bool ok = true;
                for (int64_t cur = cursor0; cursor_ok(cur) && ok;) {
                    const UnitCoords uc = unit_coords(cur);
                    cur = uc.next;
                    const int sb0 = uc.kb0 >> 2, sb_end = (uc.kb1 + 3) >> 2;
                    // the L2 prefetch runs PREFETCH super-blocks ahead, on into the next work
                    // unit's first ones, so a unit (an expert's tile in the grouped mode) does not
                    // start on cold weights
                    const bool has_next = cursor_ok(cur);
                    const UnitCoords un = has_next ? unit_coords(cur) : uc;
                    const int nsb0 = un.kb0 >> 2, nsb_end = (un.kb1 + 3) >> 2;
                    const CUtensorMap* tw = wmap(uc.mem);
                    for (int pf = sb0; pf < sb0 + RC::PREFETCH && pf < sb_end; pf++)
                        tma_prefetch_l2_2d(tw, pf * RC::X_ELEMS, uc.wrow0);
                    for (int sb = sb0; sb < sb_end; sb++) {
                        const int ahead = sb + RC::PREFETCH;
                        if (ahead < sb_end) tma_prefetch_l2_2d(tw, ahead * RC::X_ELEMS, uc.wrow0);
                        else if (has_next && nsb0 + (ahead - sb_end) < nsb_end)
                            tma_prefetch_l2_2d(wmap(un.mem), (nsb0 + (ahead - sb_end)) * RC::X_ELEMS, un.wrow0);
                        if (!mbar_wait(rempty_bar(rs), rph ^ 1u, args.err, ERR_WAIT_PRODUCER, abort_flag)) { ok = false; break; }
                        const uint32_t dst = sbase + C::RAW_OFF + rs * RC::STAGE;
                        mbar_arrive_expect_tx(rfull_bar(rs), RC::A_BYTES + RC::D_BYTES);
                        tma_load_2d(dst, tw, rfull_bar(rs), sb * RC::X_ELEMS, uc.wrow0);
                        if constexpr (WT == WT_Q6_K) tma_load_2d(dst + RC::A_BYTES, dmap(uc.mem), rfull_bar(rs), uc.wrow0, sb);
                        issued_mask |= 1u << rs;
                        issued_par = (issued_par & ~(1u << rs)) | (rph << rs);
                        if (++rs == C::RAW_STAGES) { rs = 0; rph ^= 1u; }
                    }
                }
                if (!ok) {
                    for (int s2 = 0; s2 < C::RAW_STAGES; s2++)
                        if (((issued_mask >> s2) & 1u) && !mbar_drain(rfull_bar(s2), (issued_par >> s2) & 1u))
                            atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
                }
            }
        }
    } else if (warp == W_MMA) {
        // ---------------- MMA issuer (the leader's, for a pair) ----------------
        if (lane == 0 && (!PAIR || leader)) {
            int stage = 0;
            uint32_t phase = 0;
            int lt = 0;
            bool ok = true;
            // descriptors of stage 0; a stage adds STAGE_BYTES, a 16-element K step 32 bytes (>> 4)
            const uint64_t wdesc0 = sdesc_k_sw128(sbase + C::A_BYTES);
            const uint64_t adesc0 = sdesc_k_sw128(sbase);
            for (int64_t cur = cursor0; cursor_ok(cur) && ok; lt++) {
                const UnitCoords uc = unit_coords(cur);
                cur = uc.next;
                const int kb0 = uc.kb0, kb1 = uc.kb1;
                const int acc = C::N_ACC == 1 ? 0 : (lt & 1);
                const uint32_t aphase = C::N_ACC == 1 ? (uint32_t)lt & 1u : (uint32_t)(lt >> 1) & 1u;
                if (!mbar_wait<PAIR>(tempty_bar(acc), aphase ^ 1u, args.err, ERR_WAIT_MMA, abort_flag)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BT);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait<PAIR>(full_bar(stage), phase, args.err, ERR_WAIT_MMA, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t soff = (uint64_t)((stage * C::STAGE_BYTES) >> 4);
#pragma unroll
                    for (int k = 0; k < GEMM_BK / 16; k++) {
                        if constexpr (PAIR)
                            mma_f16_pair(d_tmem, wdesc0 + soff + 2 * k, adesc0 + soff + 2 * k, C::IDESC,
                                         (kb > kb0 || k > 0) ? 1u : 0u);
                        else
                            mma_f16(d_tmem, wdesc0 + soff + 2 * k, adesc0 + soff + 2 * k, C::IDESC,
                                    (kb > kb0 || k > 0) ? 1u : 0u);
                        if constexpr (C::WIDE)   // the same decoded weights against tokens 256..511
                            mma_f16(d_tmem + (uint32_t)C::MMA_N, wdesc0 + soff + 2 * k,
                                    adesc0 + soff + (uint64_t)((C::A_BYTES / 2) >> 4) + 2 * k, C::IDESC,
                                    (kb > kb0 || k > 0) ? 1u : 0u);
                    }
                    if constexpr (PAIR) mma_commit_pair(empty_bar(stage));
                    else mma_commit(empty_bar(stage));
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                if constexpr (PAIR) mma_commit_pair(tfull_bar(acc));
                else mma_commit(tfull_bar(acc));
            }
            // Every MMA this thread issued has completed once drain_bar fires.
            if constexpr (PAIR) mma_commit_pair(drain_bar);
            else mma_commit(drain_bar);
            if (!mbar_drain(drain_bar, 0)) atomicCAS(args.err, 0, ERR_WAIT_DRAIN);
        }
        if constexpr (PAIR && C::QUANT) {
            if (lane == 0 && !leader) {
                // the announcer: one cluster-scope arrive on the leader's full barrier per stage, after
                // this CTA's eight dequant warps have filled it (their release at CTA scope, acquired
                // here, is carried to the leader by this arrive's release at cluster scope)
                int stage = 0;
                uint32_t phase = 0;
                bool ok = true;
                for (int64_t cur = cursor0; cursor_ok(cur) && ok;) {
                    const UnitCoords uc = unit_coords(cur);
                    cur = uc.next;
                    for (int kb = uc.kb0; kb < uc.kb1; kb++) {
                        if (!mbar_wait(pfull_bar(stage), phase, args.err, ERR_WAIT_DEQUANT, abort_flag)) { ok = false; break; }
                        mbar_arrive_cluster(mapa_shared(full_bar(stage), 0));
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    }
                }
            }
        }
    } else if (warp >= W_EPI0 && warp < W_EPI0 + 4) {
        // ---------------- epilogue ----------------
        // Thread i of warp q owns TMEM lane (weight row) 32q + i and reads its tokens 16 at a time
        // (tcgen05.ld 32x32b.x16), the next 16 already in flight while the current ones are
        // stored. Every store is one token's 32 consecutive rows: 128 contiguous bytes per warp.
        constexpr int NG = BT / 32;                      // 32-token groups (one value per lane)
        const int q = warp & 3;                          // TMEM lane quadrant this warp may read
        const uint32_t lane_tmem = tmem_base + ((uint32_t)(32 * q) << 16);
        int lt = 0;
        uint32_t xn = 0;                                 // cluster split: tiles exchanged so far
        for (int64_t cur = cursor0; cursor_ok(cur); lt++) {
            const UnitCoords uc = unit_coords(cur);
            cur = uc.next;
            const int acc = C::N_ACC == 1 ? 0 : (lt & 1);
            const uint32_t aphase = C::N_ACC == 1 ? (uint32_t)lt & 1u : (uint32_t)(lt >> 1) & 1u;
            const int ntok = min(BT, uc.t_end - uc.t0);  // tokens of this tile
            bool with_part = false;
            // WIDE: no idle accumulator to gather the partials into; the store loop adds them from
            // global memory instead, once the lower-numbered CTAs have published them
            bool part_direct = false;
            if constexpr (C::WIDE) {
                if (uc.finishes && uc.c_first < unit_id) {
                    bool ok = true;
                    for (int c = uc.c_first; c < unit_id && ok; c++)
                        ok = wait_flag(args.flags + 4 * c + q, args.epoch, args.err, abort_flag);
                    if (!ok) break;
                    part_direct = true;
                }
            } else if constexpr (!GROUPED) {
                if (uc.finishes && uc.c_first < unit_id) {
                    // A finisher sums the partials of the lower-numbered CTAs sharing its tile
                    // (they computed them first) into the idle accumulator while its own K range
                    // is still on the tensor core; this is always the CTA's last item, so the MMA
                    // issuer no longer uses that accumulator.
                    bool ok = true;
                    // partial slot of work unit c for this CTA's rows: 2c + rank for a pair
                    for (int c = uc.c_first; c < unit_id && ok; c++)
                        ok = wait_flag(args.flags + 4 * (PAIR ? 2 * c + (int)crank : c) + q, args.epoch, args.err,
                                       abort_flag);
                    if (!ok) break;
                    for (int c0 = 0; c0 < ntok; c0 += 32) {
                        const int slot0 = PAIR ? 2 * uc.c_first + (int)crank : uc.c_first;
                        const float* p = args.partials + (size_t)slot0 * (BT * GEMM_BN) +
                                         (size_t)c0 * GEMM_BN + 32 * q + lane;
                        float sum[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) sum[j] = __ldcg(p + j * GEMM_BN);
                        for (int c = uc.c_first + 1; c < unit_id; c++) {
                            p += (PAIR ? 2 : 1) * BT * GEMM_BN;
#pragma unroll
                            for (int j = 0; j < 32; j++) sum[j] += __ldcg(p + j * GEMM_BN);
                        }
                        uint32_t r[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) r[j] = __float_as_uint(sum[j]);
                        tmem_st32(lane_tmem + (uint32_t)((acc ^ 1) * BT + c0), r);
                    }
                    tmem_st_wait();
                    with_part = true;
                }
            }
            // Per-token values of a finished tile, fetched before the accumulator is ready: lane
            // i holds those of tokens 32g + i and hands them to the storing lanes by shuffle.
            float scl[NG];
            uint64_t rowp[GROUPED ? NG : 1];
            if (uc.finishes) {
#pragma unroll
                for (int g = 0; g < NG; g++) {
                    const int t = uc.t0 + 32 * g + lane;
                    const bool live = 32 * g < ntok && t < uc.t_end;
                    scl[g] = live ? __ldg(args.scales + t) : 0.0f;
                    if constexpr (GROUPED) {
                        const char* ob = reinterpret_cast<const char*>(
                            args.g_src && live ? args.out_bases[__ldg(args.g_src + t)] : args.out);
                        rowp[g] = live ? reinterpret_cast<uint64_t>(ob + (int64_t)__ldg(args.g_tok + t) * args.d_nb2 +
                                                                   (int64_t)__ldg(args.g_slot + t) * args.d_nb1)
                                       : 0ull;
                    }
                }
            }
            if (!mbar_wait(tfull_bar(acc), aphase, args.err, ERR_WAIT_EPILOGUE, abort_flag)) break;
            tc_fence_after();
            const bool fin = uc.finishes;
            if (!fin) {
                // A piece another CTA finishes: this warp's 32 weight rows of the unscaled
                // partial, stored [token][128] f32 straight from TMEM (coalesced per token).
                float* p = args.partials + (size_t)blockIdx.x * (BT * GEMM_BN) + 32 * q + lane;
                for (int c0 = 0; c0 < ntok; c0 += 32) {
                    uint32_t r[32];
                    tmem_ld32(lane_tmem + (uint32_t)(acc * BT + c0), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 32; j++) __stcg(p + (size_t)(c0 + j) * GEMM_BN, __uint_as_float(r[j]));
                }
            } else if (csplit) {
                // Cluster split: this CTA finishes tokens [own0, own0 + BT/2) of the tile. A cluster
                // holds one tile, so once the accumulator is full this CTA's operand stages are idle.
                // Each epilogue warp stages its rows of the peer's half there ([token][32 rows] f32,
                // HALF x 128 bytes), and one bulk copy moves them into the peer's receive region (also
                // in its idle stages) once the peer says the region is free; then the warp adds what
                // arrived in its own region to its own half, scales it in place and stores it by TMA.
                constexpr int HALF = BT / 2;
                constexpr uint32_t WBYTES = HALF * 128;  // one warp's rows of one half
                const uint32_t wi = (uint32_t)(warp - W_EPI0);
                const uint32_t recv_addr = sbase + wi * WBYTES;
                const uint32_t send_addr = sbase + 4 * WBYTES + wi * WBYTES;
                float* recv = reinterpret_cast<float*>(smem + wi * WBYTES);
                float* send = reinterpret_cast<float*>(smem + 4 * WBYTES + wi * WBYTES);
                const float4* recv4 = reinterpret_cast<const float4*>(recv);
                const uint32_t peer = xrank ^ 1u;
                const int own0 = (int)xrank * HALF, oth0 = HALF - own0;
                const int cc = lane & 7;                 // float4 column of the read-back
                const int nb = uc.n0 + 32 * q + 4 * cc;  // this lane's 4 output columns
                const uint32_t par = xn & 1u;
                xn++;
                // this warp's receive region is free (its MMAs are done): expect the peer's bytes, and
                // tell the peer
                if (lane == 0) {
                    mbar_arrive_expect_tx(xfull_bar(q, 0), WBYTES);
                    mbar_arrive_cluster(mapa_shared(xfree_bar(q, 0), peer));
                }
                for (int ch = 0; ch < HALF / 16; ch++) {
                    uint32_t r[16];
                    tmem_ld16(lane_tmem + (uint32_t)(acc * BT + oth0 + 16 * ch), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int j = 0; j < 16; j++) send[(16 * ch + j) * 32 + lane] = __uint_as_float(r[j]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (mbar_wait<true>(xfree_bar(q, 0), par, args.err, ERR_WAIT_EPILOGUE, abort_flag))
                        bulk_copy_s2cluster(mapa_shared(recv_addr, peer), send_addr, WBYTES,
                                            mapa_shared(xfull_bar(q, 0), peer));
                }
                if (!mbar_wait<true>(xfull_bar(q, 0), par, args.err, ERR_WAIT_EPILOGUE, abort_flag)) break;
                for (int ch = 0; ch < HALF / 16; ch++) {
                    uint32_t o[16];
                    tmem_ld16(lane_tmem + (uint32_t)(acc * BT + own0 + 16 * ch), o);
                    tmem_ld_wait();
                    const int tk0 = own0 + 16 * ch;      // first token (of the tile) of the chunk
                    const int g = tk0 >> 5;
                    float sg = scl[0];
#pragma unroll
                    for (int i = 1; i < NG; i++)
                        if (g == i) sg = scl[i];
                    float* rc = recv + 16 * ch * 32;
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        rc[j * 32 + lane] = (__uint_as_float(o[j]) + rc[j * 32 + lane]) *
                                            __shfl_sync(0xffffffffu, sg, (tk0 & 31) + j);
                    if (args.n_dst == 0) {
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0 && tk0 < ntok) {
                            const uint32_t src = recv_addr + (uint32_t)(16 * ch * 128);
                            tma_store_2d(omap(uc.mem), src, uc.n0 + 32 * q, uc.t0 + tk0);
                            if (tk0 + 8 < ntok) tma_store_2d(omap(uc.mem), src + 1024u, uc.n0 + 32 * q, uc.t0 + tk0 + 8);
                            bulk_commit();
                        }
                    } else {
                        // several destinations (weight rows split across GPUs): 16-byte stores of whole
                        // 128-byte output lines, four tokens per instruction
                        __syncwarp();
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int jr = (lane >> 3) + 4 * i;
                            const float4 v = recv4[(16 * ch + jr) * 8 + cc];
                            const int t = uc.t0 + tk0 + jr;
                            if (t < uc.t_end && nb < args.N) {
                                const size_t o4 = (size_t)t * args.ldo + args.col0 + nb;
                                for (int d = 0; d < args.n_dst; d++)
                                    *reinterpret_cast<float4*>(args.out_bases[d] + o4) = v;
                            }
                        }
                    }
                }
            } else {
                // 32 tokens at a time, through this warp's 32 x 32 f32 box of shared memory
                float* es = reinterpret_cast<float*>(smem + C::EPI_OFF) + (warp - W_EPI0) * 1024;
                const float4* es4 = reinterpret_cast<const float4*>(es);
                const int cc = lane & 7;                 // float4 column of the read-back (grouped)
                const int nb = uc.n0 + 32 * q + 4 * cc;  // this lane's 4 output columns (grouped)
                const uint32_t es_addr = smem_u32(es);
                for (int c0 = 0; c0 < ntok; c0 += 32) {
                    const int g = c0 >> 5;
                    float sg = scl[0];
                    uint64_t rg = GROUPED ? rowp[0] : 0ull;
#pragma unroll
                    for (int i = 1; i < NG; i++) {
                        if (g == i) {
                            sg = scl[i];
                            if constexpr (GROUPED) rg = rowp[i];
                        }
                    }
                    uint32_t r[32];
                    tmem_ld32(lane_tmem + (uint32_t)(acc * BT + c0), r);
                    if (with_part) {
                        uint32_t r2[32];
                        tmem_ld32(lane_tmem + (uint32_t)((acc ^ 1) * BT + c0), r2);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; j++) r[j] = __float_as_uint(__uint_as_float(r[j]) + __uint_as_float(r2[j]));
                    } else {
                        tmem_ld_wait();
                    }
                    if constexpr (C::WIDE) {
                        if (part_direct) {
                            const float* p = args.partials + (size_t)uc.c_first * (BT * GEMM_BN) +
                                             (size_t)c0 * GEMM_BN + 32 * q + lane;
                            for (int c = uc.c_first; c < unit_id; c++, p += BT * GEMM_BN) {
#pragma unroll
                                for (int j = 0; j < 32; j++)
                                    r[j] = __float_as_uint(__uint_as_float(r[j]) + __ldcg(p + j * GEMM_BN));
                            }
                        }
                    }
                    if (!GROUPED && args.n_dst == 0) {
                        // the scaled [token][32 rows] values as four [8 tokens][32 rows] boxes, each
                        // written by one TMA store (rows past M and columns past N are clipped by the
                        // tensor map); four box buffers per warp, so three stores are still reading
                        // shared memory while the next box is written
#pragma unroll
                        for (int sbx = 0; sbx < 4; sbx++) {
                            if (lane == 0) bulk_wait_read<3>();   // this buffer's previous store has read it
                            __syncwarp();
#pragma unroll
                            for (int j = 0; j < 8; j++)
                                es[sbx * 256 + j * 32 + lane] =
                                    __uint_as_float(r[8 * sbx + j]) * __shfl_sync(0xffffffffu, sg, 8 * sbx + j);
                            fence_proxy_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_2d(omap(uc.mem), es_addr + 1024u * sbx, uc.n0 + 32 * q, uc.t0 + c0 + 8 * sbx);
                                bulk_commit();
                            }
                        }
                    } else {
                        // scattered rows (grouped) or several destinations (split weight rows): a
                        // transpose, then 16-byte stores, each instruction four whole 128-byte
                        // output lines (plain stores: the destinations may be other GPUs')
#pragma unroll
                        for (int j = 0; j < 32; j++) es[j * 32 + lane] = __uint_as_float(r[j]);
                        __syncwarp();
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const int jr = (lane >> 3) + 4 * i;
                            const float sc = __shfl_sync(0xffffffffu, sg, jr);
                            float4 v = es4[jr * 8 + cc];
                            v.x *= sc; v.y *= sc; v.z *= sc; v.w *= sc;
                            if constexpr (GROUPED) {
                                const uint64_t rp = __shfl_sync(0xffffffffu, rg, jr);
                                if (rp && nb < args.N) *reinterpret_cast<float4*>(reinterpret_cast<float*>(rp) + nb) = v;
                            } else {
                                const int t = uc.t0 + c0 + jr;
                                if (t < uc.t_end && nb < args.N) {
                                    const size_t o = (size_t)t * args.ldo + args.col0 + nb;
                                    for (int d = 0; d < args.n_dst; d++)
                                        *reinterpret_cast<float4*>(args.out_bases[d] + o) = v;
                                }
                            }
                        }
                        __syncwarp();
                    }
                }
            }
            if (!fin) {
                __threadfence();
                __syncwarp();
                if (lane == 0) st_release_gpu(args.flags + 4 * blockIdx.x + q, args.epoch);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader(tempty_bar(acc));
        }
        if (lane == 0) bulk_wait_all();   // this warp's output stores are complete before it exits
        // rows stored into other GPUs' memory must be visible there before the kernel that follows
        // signals their owners: one system fence per thread after its last store (a fence per
        // tile would hold the accumulator until every store of the tile had crossed NVLink)
        if (GROUPED ? args.g_src != nullptr : args.n_dst > 0) __threadfence_system();
    } else if (C::QUANT && dequant_slot(warp) >= 0) {
        // ---------------- dequant (quantized weights) ----------------
        if constexpr (C::QUANT) {
            // Two groups of four warps take alternate K blocks: in its blocks a warp group decodes all
            // 64 weights of every row of the tile (thread: one row, both 32-weight halves of the chunk,
            // from one read of the raw bytes) and fills the whole stage, with one proxy fence and one
            // arrive per thread per block, while the other group fills the next stage.
            const int dq = dequant_slot(warp);
            const int r = (dq & 3) * 32 + lane;          // weight row within the tile
            const int grp = dq >> 2;                     // this group fills the stages of blocks n with n % 2 == grp
            int rs = 0;
            uint32_t rph = 0, n = 0;                     // n: the CTA's running K-block count
            bool ok = true;
            for (int64_t cur = cursor0; cursor_ok(cur) && ok;) {
                const UnitCoords uc = unit_coords(cur);
                cur = uc.next;
                for (int sb = uc.kb0 >> 2; sb * 4 < uc.kb1 && ok; sb++) {
                    const int k_lo = max(uc.kb0, 4 * sb), k_hi = min(uc.kb1, 4 * sb + 4);
                    // does this group own a block of this super-block?
                    const bool mine = (k_hi - k_lo) > 1 || ((n & 1u) == (uint32_t)grp);
                    if (!mbar_wait(rfull_bar(rs), rph, args.err, ERR_WAIT_DEQUANT, abort_flag)) { ok = false; break; }
                    const uint8_t* raw = smem + C::RAW_OFF + rs * RC::STAGE;
                    const uint8_t* rrow = raw + r * RC::ROW;
                    float d6 = 0.0f;
                    Q4kFactors f0{}, f1{};
                    if (mine) {
                        if constexpr (WT == WT_Q6_K) d6 = __half2float(reinterpret_cast<const __half*>(raw + RC::A_BYTES)[r]);
                        if constexpr (WT == WT_Q4_K) {
                            f0 = q4k_factors(rrow, 0);
                            f1 = q4k_factors(rrow, 1);
                        }
                    }
                    for (int kb = k_lo; kb < k_hi; kb++, n++) {
                        if ((n & 1u) != (uint32_t)grp) continue;
                        uint32_t o0[16], o1[16];
                        if constexpr (WT == WT_Q4_K) {
                            float da, ma, db, mb;
                            f0.pick(kb & 3, da, ma);
                            f1.pick(kb & 3, db, mb);
                            decode_q4k_both(rrow, kb & 3, da, ma, db, mb, o0, o1);
                        } else if constexpr (WT == WT_Q6_K) {
                            decode_q6k_half(rrow, d6, kb & 3, 0, o0);
                            decode_q6k_half(rrow, d6, kb & 3, 1, o1);
                        } else {
                            decode_q8_0_half(rrow, kb & 3, 0, o0);
                            decode_q8_0_half(rrow, kb & 3, 1, o1);
                        }
                        const int stage = (int)(n % (uint32_t)STAGES);
                        const uint32_t phase = (n / (uint32_t)STAGES) & 1u;
                        // decoded first: the arithmetic overlaps the wait for the stage to free up
                        if (!mbar_wait(empty_bar(stage), phase ^ 1u, args.err, ERR_WAIT_DEQUANT, abort_flag)) { ok = false; break; }
                        const uint32_t sw = sbase + stage * C::STAGE_BYTES + C::A_BYTES;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            st_shared_v4(sw + sw128_offset((uint32_t)r, (uint32_t)c), o0[4 * c], o0[4 * c + 1], o0[4 * c + 2],
                                         o0[4 * c + 3]);
                            st_shared_v4(sw + sw128_offset((uint32_t)r, (uint32_t)(4 + c)), o1[4 * c], o1[4 * c + 1],
                                         o1[4 * c + 2], o1[4 * c + 3]);
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(PAIR && !leader ? pfull_bar(stage) : full_bar(stage));
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(rempty_bar(rs));
                    if (++rs == C::RAW_STAGES) { rs = 0; rph ^= 1u; }
                }
            }
        }
    }

    tc_fence_before();
    // a pair: neither CTA leaves while the leader's MMAs may still read the peer's shared memory
    // or write its TMEM (the leader's MMA thread passes here only after its drain); a cluster
    // split: neither leaves while the peer may still write into its shared memory or barriers
    if (PAIR || csplit) cluster_sync();
    else cta_sync();
    if (warp == W_MMA) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        else tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace b200
