/*
 * ggml B200 backend -- the kernel-level C ABI.
 *
 * These entry points run the three prefill ops that gregordinary/ggml-rocket offloads, on
 * device memory and a caller-supplied CUDA stream (passed as void*). They are what the
 * backend layer (ggml-b200.h) calls from graph_compute, and what a host that already keeps
 * its tensors in device memory can call directly. All pointers are device pointers unless
 * stated; all sizes are element counts unless stated; strides named nb* are in bytes, as in
 * ggml. Every function returns 0 (B200_OK) or a negative b200_status; launches are
 * asynchronous, and a kernel that fails at run time (a bounded wait that gave up, a failed
 * bounds check) writes a nonzero code into *dev_err, which the caller reads after the stream
 * synchronises. No entry point falls back to the CPU.
 *
 * Weight types use ggml's ggml_type numbering: F32 0, F16 1, Q8_0 8, Q4_K 12, Q6_K 14, BF16 30.
 */
#ifndef GGML_B200_KERNELS_H
#define GGML_B200_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    B200_OK = 0,
    B200_E_INVALID = -1,       /* a NULL pointer, a non-positive size, malformed strides */
    B200_E_UNSUPPORTED = -2,   /* a shape or type outside what the kernels tile (the claim rules exclude it) */
    B200_E_CUDA = -3,          /* a CUDA API call or launch failed */
    B200_E_DEVICE = -4,        /* a kernel reported a run-time fault through dev_err */
    B200_E_WORKSPACE = -5,     /* the workspace is missing, too small or not 256-byte aligned */
    B200_E_BAD_IDS = -6,       /* a MUL_MAT_ID expert id outside [0, n_expert) */
    B200_E_NO_DEVICE = -7,     /* no CUDA device */
    B200_E_TOO_LARGE = -8,     /* the op needs more scratch than b200_mul_mat_noalloc's fixed array holds */
} b200_status;

/* ---- weights ------------------------------------------------------------------------------
 * Replaces the reference's per-call weight preparation: rocket_weight_to_fp16
 * (ggml-rocket.cpp:3853-3931) and the NPU's packB of the resident route
 * (ggml_backend_rocket_mul_mat_prepacked, ggml-rocket.cpp:4306-4528). Nothing is expanded to
 * fp16: the packed form holds the same quantized bytes, re-laid so that every device load is
 * 16-byte aligned (Q4_K and F16 are copied unchanged).
 */
size_t b200_weight_packed_size(int type, int64_t N, int64_t K);
int    b200_weight_pack(int type, const void * src_native, int64_t N, int64_t K, void * dst_packed, void * stream);

/* Decode N native ggml rows of K weights to f32 (f16_out = 0) or fp16 (f16_out = 1), as
 * ggml's to_float does (bit-exact), the way the reference decodes a quantized weight row at
 * ggml-rocket.cpp:3894-3907. */
int    b200_dequantize(int type, const void * src_native, int64_t N, int64_t K, int f16_out, void * dst, void * stream);

/* ---- MUL_MAT ------------------------------------------------------------------------------
 * Replaces ggml_backend_rocket_mul_mat's device route (ggml-rocket.cpp:4548-4871): the
 * activation pack rocket_pack_activations_scratch (:1477-1502), the NPU GEMM
 * rocket_matmul_fp16_stream/_mt/_prepacked (:4834, :4844, :4449) and the unpack
 * rocket_unpack_output (:1520-1532), for one 2-D slice:
 *
 *     dst[m * ldd + n] = sum_k src1[m * lda + k] * W[n, k]     m < M, n < N
 *
 * src1 is F32 (row stride lda elements), W is `wtype` in the packed layout above, dst is F32
 * (row stride ldd elements). Each activation row is scaled by its max |value| into fp16 (the
 * reference's "sandwich", :1451-1475); the products accumulate in fp32 in tensor memory and
 * the row scale is applied to the fp32 result. Requires K % 32 == 0, N % 16 == 0, and
 * K % 256 == 0 for Q4_K / Q6_K. The workspace (device, 256-byte aligned) must hold
 * b200_mul_mat_workspace_size(wtype, M, N, K) bytes.
 */
size_t b200_mul_mat_workspace_size(int wtype, int64_t M, int64_t N, int64_t K);
int    b200_mul_mat(int wtype, const void * w_packed, int64_t N, int64_t K,
                    const float * src1, int64_t lda, int64_t M,
                    float * dst, int64_t ldd,
                    void * workspace, size_t workspace_bytes, int * dev_err, void * stream);

/* The two halves of b200_mul_mat, for a caller that reuses one packed activation across
 * several weights (the reference's fused QKV / gate-up group shares one pack,
 * ggml-rocket.cpp:4956-5020) or times them apart:
 *   b200_act_pack     src1 F32 [M, lda] -> a16 fp16 [M, K] (dense) + scales F32 [M]
 *   b200_gemm_packed  dst = scales[m] * (a16 . W^T); the workspace (256-byte aligned) holds
 *                     the partial tiles of output tiles whose K range several CTAs share
 *                     (b200_gemm_packed_workspace_size bytes; 0 when no tile is shared). */
int    b200_act_pack(const float * src1, int64_t lda, int64_t M, int64_t K, void * a16, float * scales, void * stream);
/* A dense FFN's GLU SWIGLU fused into the pack of the down projection that reads it: h =
 * silu(gate) * up per element (ggml_swiglu_split), then b200_act_pack of h's [M, F] rows -- a16 and
 * scales equal b200_swiglu followed by b200_act_pack bit for bit; h is never written. The reference
 * leaves SWIGLU to the host and packs the down projection's activations there (rk_pack_act_row,
 * ggml-rocket.cpp:1451-1475). gate / up rows: F floats at row strides ldg / ldu, 16-byte aligned;
 * F % 4 == 0 and F <= 16384, else B200_E_UNSUPPORTED. */
int    b200_swiglu_act_pack(const float * gate, int64_t ldg, const float * up, int64_t ldu, int64_t M, int64_t F,
                            void * a16, float * scales, void * stream);
size_t b200_gemm_packed_workspace_size(int wtype, int64_t M, int64_t N, int64_t K);
int    b200_gemm_packed(int wtype, const void * w_packed, int64_t N, int64_t K, const void * a16, const float * scales,
                        int64_t M, float * dst, int64_t ldd, void * workspace, size_t workspace_bytes, int * dev_err,
                        void * stream);

/* The combined-N GEMM of a fused group (the reference's _mul_mat_group / _group_resident,
 * ggml-rocket.cpp:4956-5020, 5040-5160: one GEMM over the members' weights side by side, each
 * member's columns unpacked into its own dst): n_members (1..4) weights of one type and one K
 * against the same packed activation, in ONE kernel launch whose schedule covers every member's
 * tiles. dst[m][t * ldd[m] + n] = scales[t] * (a16 . W_m^T)[t, n] for n < N[m]. Each member's
 * rules are b200_gemm_packed's; the workspace (256-byte aligned) holds
 * b200_gemm_packed_group_workspace_size bytes. The plan call reports the token tile, the most CTAs
 * sharing one tile's K range and the grid of that launch. */
size_t b200_gemm_packed_group_workspace_size(int n_members, int wtype, int64_t M, const int64_t * N, int64_t K);
int    b200_gemm_packed_group(int n_members, int wtype, const void * const * w_packed, const int64_t * N, int64_t K,
                              const void * a16, const float * scales, int64_t M, float * const * dst,
                              const int64_t * ldd, void * workspace, size_t workspace_bytes, int * dev_err,
                              void * stream);
int    b200_gemm_packed_group_plan(int n_members, int wtype, int64_t M, const int64_t * N, int64_t K,
                                   int * token_tile, int * splits, int * grid);

/* The launch plan b200_mul_mat uses on the current device: the token tile (tcgen05 N), the
 * most CTAs that share one output tile's K range (1 = every CTA owns whole tiles), the
 * persistent grid and the number of kernel launches one call makes. */
int    b200_mul_mat_plan(int wtype, int64_t M, int64_t N, int64_t K, int * token_tile, int * splits, int * grid,
                         int * launches);

/* ---- MUL_MAT without allocation ------------------------------------------------------------
 * No counterpart in the reference. For callers that cannot call cudaMalloc (a plugin inside a
 * process whose allocator owns the device, code that must not change the device memory map, a
 * fixed memory budget): the same MUL_MAT as b200_mul_mat, with its workspace taken from a 32 MiB
 * file-scope device array that every GPU loading this library holds until exit. The caller
 * passes only inputs and outputs. An op whose workspace (b200_mul_mat_workspace_size) exceeds
 * b200_mul_mat_noalloc_max_workspace() returns B200_E_TOO_LARGE. The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress), a set-up step, so make that first
 * call before any stream capture begins. dev_err may be NULL: the device error word then lives in
 * the array, keeps the first error any call records, and b200_mul_mat_noalloc_error()
 * synchronises the stream, returns it and clears it. Every call clears the part of the array that
 * would otherwise carry state into it (the flags CTAs use to hand partial tiles to each other)
 * before its kernels run. Calls share the array, so calls that overlap on the GPU race; the caller
 * must order them. */
size_t b200_mul_mat_noalloc_max_workspace(void);
int    b200_mul_mat_noalloc(int wtype, const void * w_packed, int64_t N, int64_t K,
                            const float * src1, int64_t lda, int64_t M, float * dst, int64_t ldd,
                            int * dev_err, void * stream);
int    b200_mul_mat_noalloc_error(void * stream, int * host_err);

/* ---- FLASH_ATTN_EXT ------------------------------------------------------------------------
 * Replaces ggml_backend_rocket_flash_attn (ggml-rocket.cpp:5444-5691): its gathers (:5487-5577),
 * the NPU per-head QK -> mask -> softmax -> PV (rocket_flash_attn_fp16_ctx, :5590) and its
 * scatter (:5644-5655), in one pass over the op's own strided tensors (ggml layouts, strides in
 * bytes, innermost stride = element size):
 *   q    F32 [D, T, H]        k F16 [D, KV, HK]       v F16 [DV, KV, HK]
 *   mask F16 [KV, >=T] (row t at mask + t*m_nb1) or NULL for an unmasked op
 *   dst  F32 [DV, H, T] contiguous
 *   dst[c, h, t] = sum_j softmax_j(S[t,j]) v[c, j, h/(H/HK)],
 *   S[t,j] = softcap*tanh(scale*q.k/softcap) (or scale*q.k when softcap == 0) + mask[t, j]
 * Q is scaled and narrowed to fp16 (a row whose scaled values leave fp16's range is divided by a
 * power of two that the score multiplies back, so no range fallback exists); q.k and P.v
 * accumulate in fp32 in tensor memory, the softmax runs in fp32, P is fp16. A fully masked row
 * is written as zeros. Requires D and DV in {64, 128}, H % HK == 0, 16-byte-aligned bases and
 * row strides, max_bias == 0.
 */
size_t b200_flash_attn_workspace_size(int D, int DV, int T, int H, int KV, int HK);
int    b200_flash_attn_ext(const float * q, int64_t q_nb1, int64_t q_nb2,
                           const void * k, int64_t k_nb1, int64_t k_nb2,
                           const void * v, int64_t v_nb1, int64_t v_nb2,
                           const void * mask, int64_t m_nb1,
                           float * dst, int D, int DV, int T, int H, int KV, int HK,
                           float scale, float max_bias, float softcap,
                           void * workspace, size_t workspace_bytes, int * dev_err, void * stream);
/* A quantized KV-cache view (ggml's -ctk / -ctv q8_0 or q4_0: type 8 or 2) as the fp16 tiles the
 * attention kernel reads: [HK][KV][D] of the view whose rows are nb1 bytes apart and heads nb2,
 * each value ggml's dequantized f32 rounded to fp16, written contiguous to dst (16-byte aligned,
 * HK * KV * D * 2 bytes). The reference declines FLASH_ATTN_EXT on a quantized cache (its handler
 * takes F16 K / V only, ggml-rocket.cpp:7654-7700); the backend runs such ops as this conversion
 * followed by b200_flash_attn_ext when B200_FA_QUANT_KV=1. */
int    b200_kv_to_f16(int type, const void * src, int64_t D, int64_t KV, int64_t HK, int64_t nb1, int64_t nb2,
                      void * dst, void * stream);

/* ---- decode-size MUL_MAT (M = 1..32) over Q4_K, Q6_K and Q8_0 weights ----------------------
 * The reference leaves decode (M below its ROCKET_MIN_M) on the CPU (ggml-rocket.cpp:7424-7496);
 * this is MUL_MAT for those M on the GPU: dst[m, n] = sum_k src1[m, k] * W[n, k] with W the
 * weight as b200_weight_pack packs it (16-byte aligned; K a multiple of 256, of 32 for Q8_0),
 * src1 f32 [M][lda], dst f32 [M][ldd]. Two launches: an activation prep (fp16 of src1 / s per
 * 256-value block, s the block's absmax, with the per-block sums the arithmetic needs) and a
 * weight-streaming kernel that decodes the weights into warp-level tensor-core MMA fragments as
 * exact integers and accumulates in fp32. Q4_K at M <= 8 streams 16-row blocks per CTA; every
 * other case takes 128-row x 256-weight tiles by TMA, one persistent CTA per SM over equal
 * contiguous ranges of tiles, 8-token column tiles sharing each decoded fragment. Rows split
 * between CTAs are added by the last to finish, in a fixed order (results do not depend on
 * timing). The workspace (b200_mul_mat_vec_workspace_size bytes, 256-byte aligned, a bound for
 * every weight type) holds the prepared activations, the partial sums and their counters; calls
 * sharing one must not overlap on the GPU. Returns B200_E_UNSUPPORTED for other weight types,
 * M > 32 or a K the type does not tile. */
size_t b200_mul_mat_vec_workspace_size(int64_t M, int64_t N, int64_t K);
int    b200_mul_mat_vec(int wtype, const void * w_packed, int64_t N, int64_t K, const float * src1, int64_t lda,
                        int64_t M, float * dst, int64_t ldd, void * workspace, size_t workspace_bytes,
                        int * dev_err, void * stream);

/* ---- the glue ops of a layer (RMS_NORM, ADD, MUL, SILU, SWIGLU, ROPE, GET_ROWS, CPY) ----------
 * The reference leaves these to the host's CPU backend (its supports_op claims only MUL_MAT,
 * MUL_MAT_ID and FLASH_ATTN_EXT, ggml-rocket.cpp:7410-7772); each follows ggml's CPU definition
 * element by element. Shapes are ggml's ne[4] (ne[0] innermost) with byte strides nb[4]; f32
 * outputs are contiguous. All run on `stream` and return B200_OK or a B200_E_* code. */
enum { B200_BIN_ADD = 0, B200_BIN_MUL = 1, B200_BIN_DIV = 2 };
/* every row of x scaled by 1 / sqrtf(mean(x^2) + eps) (ggml rms_norm) */
int b200_rms_norm(const float * x, const int64_t ne[4], const size_t nb[4], float eps, float * dst, void * stream);
/* RMS_NORM fused with the MUL by one weight row that follows it in a transformer graph
 * (dst = rms_norm(x) * w, w a dense f32 row of ne[0]); norm_dst, when not null, also receives the
 * normalised rows. Both outputs are bit-identical to b200_rms_norm then b200_binary(MUL); the fusion
 * saves one launch and a re-read of the normalised rows. */
int b200_rms_norm_mul(const float * x, const int64_t ne[4], const size_t nb[4], float eps, const float * w,
                      float * norm_dst, float * dst, void * stream);
/* The residual ADD in front of such a norm fused in as well: sum_dst = a + b (dense f32 of shape
 * ne, 16-byte aligned, as are w, norm_dst and dst), then dst = rms_norm(sum) * w and, when not
 * null, norm_dst = rms_norm(sum). Bit-identical to b200_binary(ADD), b200_rms_norm, b200_binary(MUL);
 * returns B200_E_UNSUPPORTED for operands that are not dense and aligned. */
int b200_add_rms_norm_mul(const float * a, const float * b, const int64_t ne[4], float eps, const float * w,
                          float * sum_dst, float * norm_dst, float * dst, void * stream);
/* The same norm (with the residual sum = x + res in front when res is not null) fused with the
 * activation pack of its product for the MUL_MATs that read it: a16 [rows, ne[0]] fp16 and scales
 * [rows] equal b200_act_pack of dst, bit for bit (the reference's rk_pack_act_row,
 * ggml-rocket.cpp:1451-1475); sum_dst (required with res), norm_dst and dst (the f32 product) are
 * written only when not null. Dense 16-byte aligned rows of ne[0] % 4 == 0 values, ne[0] <= 16384,
 * else B200_E_UNSUPPORTED. */
int b200_rms_norm_mul_act_pack(const float * x, const float * res, const int64_t ne[4], float eps, const float * w,
                               float * sum_dst, float * norm_dst, float * dst, void * a16, float * scales,
                               void * stream);
/* A MUL_MAT whose src0 carries ggml's Walsh-Hadamard hint (GGML_HINT_SRC0_IS_HADAMARD), which the
 * reference declines (ggml-rocket.cpp:7392-7403) because the CPU evaluates it as the fast
 * transform: dst row = scale * H_n row for every row of x, H_n the Sylvester-ordered Hadamard
 * matrix (H[i][k] = (-1)^popcount(i & k)), n = ne[0] a power of two from 32 to 1024, by log2(n)
 * butterfly rounds in f32 and one multiply by scale; dst contiguous f32. */
int b200_hadamard(const float * x, const int64_t ne[4], const size_t nb[4], float scale, float * dst, void * stream);
/* dst = a + b, a * b or a / b, b repeated over a (ggml_can_repeat: ane[i] % bne[i] == 0); dst has
 * a's shape */
int b200_binary(int op, const float * a, const int64_t ane[4], const size_t anb[4],
                const float * b, const int64_t bne[4], const size_t bnb[4], float * dst, void * stream);
/* dst = x / (1 + exp(-x)) */
int b200_silu(const float * x, const int64_t ne[4], const size_t nb[4], float * dst, void * stream);
/* dst = silu(a) * g, a and g of shape ne */
int b200_swiglu(const float * a, const size_t anb[4], const float * g, const size_t gnb[4], const int64_t ne[4],
                float * dst, void * stream);
/* ggml ROPE of x [head_dim, n_head, n_tokens, 1] at positions pos[n_tokens], mode 0 (normal) or 2
 * (neox), without YaRN extrapolation (ext_factor 0) and without frequency factors; dimensions
 * past n_dims are copied */
int b200_rope(const float * x, const int64_t ne[4], const size_t nb[4], const int32_t * pos, int n_dims, int mode,
              float freq_base, float freq_scale, float attn_factor, float * dst, void * stream);
/* The same ROPE (mode 0) with its output rounded to fp16 and stored at dst with byte strides dnb
 * (dnb[0] == 2): the ROPE of K and the f32 -> f16 CPY of its result into the KV-cache view in one
 * pass, bit-identical to b200_rope then b200_cpy. No counterpart in the reference (its host does
 * both). Rows of 8-byte aligned pairs, head_dim a power of two, head_dim / 2 * n_head <= 2048, else
 * B200_E_UNSUPPORTED. */
int b200_rope_f16(const float * x, const int64_t ne[4], const size_t nb[4], const int32_t * pos, int n_dims, int mode,
                  float freq_base, float freq_scale, float attn_factor, void * dst, const size_t dnb[4], void * stream);
/* dst[:, i, j, k] = src[:, idx[i, j, k], j, k]; src f32 (0) or f16 (1), dst f32 [sne[0], ine[0],
 * ine[1], ine[2]]; an index outside src's rows records a device error and yields a zero row */
int b200_get_rows(int src_type, const void * src, const int64_t sne[4], const size_t snb[4], const int32_t * idx,
                  const int64_t ine[4], const size_t inb[4], float * dst, int * dev_err, void * stream);
/* element k of src (ne[0] fastest) to element k of dst, converting between f32 (0) and f16 (1)
 * (round to nearest even); dst has src's shape (any strides) or is contiguous */
int b200_cpy(int src_type, const void * src, const int64_t sne[4], const size_t snb[4], int dst_type, void * dst,
             const int64_t dne[4], const size_t dnb[4], void * stream);

/* The MoE router's ops. SOFT_MAX without mask, ALiBi or sinks: w = x * scale, y = expf(w - max)
 * / sum(exp), the sum in double; dst f32 contiguous. */
int b200_soft_max(const float * x, const int64_t ne[4], const size_t nb[4], float scale, float * dst, void * stream);
/* ARGSORT of every row (ne[0] <= 1024): dst i32 [ne] holds the column indices in ascending or
 * descending order of value, ties in index order */
int b200_argsort(const float * x, const int64_t ne[4], const size_t nb[4], int descending, int32_t * dst,
                 void * stream);
/* SUM_ROWS: dst f32 [1, ne[1], ne[2], ne[3]] = the sum of every row, accumulated in double */
int b200_sum_rows(const float * x, const int64_t ne[4], const size_t nb[4], float * dst, void * stream);

/* ---- MUL_MAT_ID ----------------------------------------------------------------------------
 * Replaces ggml_backend_rocket_mul_mat_id (ggml-rocket.cpp:6692-6944): the counting sort of
 * (slot, token) rows by expert (:6706-6732), the per-expert gather (:6790-6800), the expert
 * GEMMs and the scatter (:6742-6754), as three kernels with no host round trip:
 *   as   [K, N, n_expert] expert weights, the whole stack packed by b200_weight_pack as one
 *        [n_expert * N, K] matrix (expert e's row n is row e*N + n)
 *   b    F32 [K, ne11, n_tokens]  (row (slot, t) at b + t*b_nb2 + (slot % ne11)*b_nb1)
 *   ids  I32 [n_used, n_tokens]   (ids + t*ids_nb1 + slot*ids_nb0)
 *   dst  F32 [N, n_used, n_tokens] (row (slot, t) at dst + t*d_nb2 + slot*d_nb1)
 *   dst[:, slot, t] = as[:, :, ids[slot, t]] . b[:, slot % ne11, t]
 * An id outside [0, n_expert) makes the kernels write nothing and set *dev_err to
 * B200_DEV_BAD_IDS (the reference returns 1 there, ggml-rocket.cpp:6719). The per-expert row
 * offsets, slots and tokens of the sort are left in the workspace
 * (b200_mul_mat_id_route_view gives their offsets) so a test can compare them with the CPU sort.
 */
#define B200_DEV_BAD_IDS 100
size_t b200_mul_mat_id_workspace_size(int64_t K, int64_t N, int64_t n_expert, int64_t n_used, int64_t n_tokens);
int    b200_mul_mat_id(int wtype, const void * as_packed, int64_t K, int64_t N, int64_t n_expert,
                       const float * b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                       const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                       float * dst, int64_t d_nb1, int64_t d_nb2,
                       void * workspace, size_t workspace_bytes, int * dev_err, void * stream);
/* n_members MUL_MAT_IDs that read the same b and the same ids (a MoE layer's gate and up
 * projections, ggml nodes sharing src1 and src2): the route and the gather-pack run once, then
 * one grouped GEMM per member (its stack as_packed[m], N[m] output rows, dst[m] with strides
 * d_nb1[m], d_nb2[m]). Host arrays of n_members entries (at most 16); the workspace is
 * b200_mul_mat_id_workspace_size's. Each dst equals the member's own b200_mul_mat_id. */
int    b200_mul_mat_id_group(int n_members, int wtype, const void * const * as_packed, const int64_t * N,
                             int64_t K, int64_t n_expert, const float * b, int64_t b_nb1, int64_t b_nb2,
                             int64_t ne11, const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used,
                             int64_t n_tokens, float * const * dst, const int64_t * d_nb1, const int64_t * d_nb2,
                             void * workspace, size_t workspace_bytes, int * dev_err, void * stream);
/* A MoE block's expert FFN in one call: the node chain gate = MUL_MAT_ID(gate_exps, x, ids),
 * up = MUL_MAT_ID(up_exps, x, ids), h = GLU SWIGLU(gate, up), dst = MUL_MAT_ID(down_exps, h, ids)
 * that llama.cpp's MoE FFN builds (the reference claims each MUL_MAT_ID on its own,
 * ggml-rocket.cpp:7497-7653, and leaves the GLU to the host). gate / up stacks: n_expert experts
 * of [F, H] in wtype_gate_up; down: n_expert of [H, F] in wtype_down; x rows as b200_mul_mat_id's
 * b with K = H; dst [n_tokens][n_used][H] with strides d_nb1 / d_nb2. The pairs are routed and x
 * gathered once for all three projections, gate / up / h stay in the workspace
 * (b200_mul_mat_id_ffn_workspace_size bytes), and SWIGLU is fused into the packing of the down
 * projection's rows. dst equals, bit for bit, b200_mul_mat_id_group(gate, up), b200_swiglu,
 * b200_mul_mat_id(down). H and F multiples of 32 and of the weight types' blocks; F <= 8192. */
size_t b200_mul_mat_id_ffn_workspace_size(int64_t H, int64_t F, int64_t n_expert, int64_t n_used, int64_t n_tokens);
int    b200_mul_mat_id_ffn(int wtype_gate_up, const void * gate_packed, const void * up_packed, int wtype_down,
                           const void * down_packed, int64_t H, int64_t F, int64_t n_expert, const float * x,
                           int64_t x_nb1, int64_t x_nb2, int64_t ne11, const int32_t * ids, int64_t ids_nb0,
                           int64_t ids_nb1, int64_t n_used, int64_t n_tokens, float * dst, int64_t d_nb1,
                           int64_t d_nb2, void * workspace, size_t workspace_bytes, int * dev_err, void * stream);
/* Byte offsets, inside the workspace, of the route arrays the last b200_mul_mat_id call wrote:
 * off int32 [n_expert + 1], row_slot int32 [n_used*n_tokens], row_tok int32 [n_used*n_tokens]. */
int    b200_mul_mat_id_route_view(int64_t K, int64_t n_expert, int64_t n_used, int64_t n_tokens,
                                  size_t * off_offset, size_t * slot_offset, size_t * tok_offset);

/* ---- MUL_MAT_ID with the experts split across GPUs (expert parallelism) -------------------
 * No counterpart in the reference, whose MUL_MAT_ID (ggml-rocket.cpp:6692-6944) runs on one
 * device; these are its per-rank halves around two all-to-all exchanges the caller runs
 * (ggml_b200.ep does them with NCCL). Rank r of n_ranks owns experts
 * [r*E/n_ranks, (r+1)*E/n_ranks) as one packed stack and its own tokens. Per op:
 *
 *  1. b200_moe_ep_dispatch (home rank): one send row per (token, b row j, destination rank),
 *     grouped by destination; its header is {slot mask, ids[0..n_used-1] of the token} (int32
 *     [n_used+1]); rows are packed fp16 with a per-row scale like MUL_MAT's activations.
 *     Buffers hold up to n_tokens*n_used rows. counts (device int32 [2*n_ranks+2]) receives
 *     rows per destination, return rows (slot-mask bits) per destination, total rows, total
 *     return rows. row_tok / row_slot / row_ret are the home rank's bookkeeping for step 3.
 *     scratch: b200_moe_ep_dispatch_scratch_size bytes of device memory, 256-byte aligned.
 *  2. b200_moe_ep_expert (owner rank): over the n_rows received rows (any number of sources,
 *     concatenated), writes one f32 row of N per (row, slot in its mask) into ret, in received
 *     order with each row's slots ascending -- the order the home rank expects back.
 *     n_pairs_hint (host, may be 0) sizes the token tile.
 *  3. b200_moe_ep_combine (home rank): the returned rows (in destination order, as step 1
 *     laid them out) -> dst[:, slot, token] with dst strides d_nb1 / d_nb2 in bytes.
 * An id outside [0, n_expert) (dispatch) or a header naming an expert this rank does not own
 * (expert) sets *dev_err to B200_DEV_BAD_IDS and produces no rows. */
size_t b200_moe_ep_dispatch_scratch_size(int64_t n_tokens, int64_t ne11, int64_t n_ranks);
int    b200_moe_ep_dispatch(const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used,
                            int64_t n_tokens, int64_t n_expert, int64_t n_ranks,
                            const float * b, int64_t b_nb1, int64_t b_nb2, int64_t ne11, int64_t K,
                            void * send_a16, float * send_scale, int32_t * send_hdr,
                            int32_t * row_tok, int32_t * row_slot, int32_t * row_ret, int32_t * counts,
                            void * scratch, size_t scratch_bytes, int * dev_err, void * stream);
size_t b200_moe_ep_expert_workspace_size(int64_t K, int64_t n_local, int64_t n_used, int64_t n_rows);
int    b200_moe_ep_expert(int wtype, const void * local_stack, int64_t K, int64_t N, int64_t n_local,
                          int64_t expert0, const void * recv_a16, const float * recv_scale,
                          const int32_t * recv_hdr, int64_t n_rows, int64_t n_used, int64_t n_pairs_hint,
                          float * ret, void * workspace, size_t workspace_bytes, int * dev_err, void * stream);
int    b200_moe_ep_combine(const float * ret, int64_t N, const int32_t * send_hdr, int64_t n_used,
                           const int32_t * row_tok, const int32_t * row_ret, const int32_t * counts,
                           int64_t n_ranks, int64_t max_rows, float * dst, int64_t d_nb1, int64_t d_nb2,
                           void * stream);

/* ---- MUL_MAT_ID expert parallelism over NVLink peer memory ----------------------------------
 * No counterpart in the reference. The same op as the per-rank halves above, with the two
 * exchanges done by the kernels' own stores into the other GPUs' buffers (no collective call, no
 * host synchronisation). Each rank allocates, with the same sizes on every rank:
 *   recv_a16  fp16 [n_ranks][cap][K]            rows other ranks push to it (cap = max rows one
 *                                                source sends one owner, e.g. n_tokens*n_used)
 *   recv_meta int32 [n_ranks][cap][n_used + 3]   {scale bits, slot mask, home token, ids}
 *   ret       f32 [n_tokens][n_used][N]          its own op output (dst's layout, strides given)
 *   flags     int32 [2 * n_ranks][4], zeroed once
 * and maps the other ranks' ones (b200_ep_shared_export on the owner, _open on the others).
 * peer_* arguments are device arrays of n_ranks device pointers (entry r = rank r's buffer as
 * mapped in this process). Per op, with an epoch that grows by one per op on every rank:
 *   home   b200_moe_ep_dispatch, then b200_moe_ep_p2p_push (rows into their owners' recv_a16 /
 *          recv_meta, counts into their flags)
 *   owner  b200_moe_ep_p2p_expert (waits for every source, runs the grouped GEMM whose
 *          epilogue stores each output row into its home rank's ret, then flags every home)
 *   home   b200_moe_ep_p2p_finish (waits for every owner): ret holds the op's dst.
 * Every wait is bounded (a rank that never arrives ends the op with a device error). */
#define B200_IPC_HANDLE_BYTES 64
int    b200_ep_shared_export(const void * ptr, void * handle, size_t * offset);
int    b200_ep_shared_open(const void * handle, void ** base);
int    b200_ep_shared_close(void * base);
int    b200_moe_ep_p2p_push(const void * send_a16, const float * send_scale, const int32_t * send_hdr,
                            const int32_t * row_tok, const int32_t * counts, int64_t n_ranks, int64_t rank,
                            int64_t n_used, int64_t K, int64_t cap, void * const * peer_recv_a16,
                            int32_t * const * peer_recv_meta, int * const * peer_flags, int epoch,
                            int64_t max_rows, void * stream);
size_t b200_moe_ep_p2p_expert_workspace_size(int64_t n_ranks, int64_t cap, int64_t K, int64_t n_local,
                                             int64_t n_used);
int    b200_moe_ep_p2p_expert(int wtype, const void * local_stack, int64_t K, int64_t N, int64_t n_local,
                              int64_t expert0, const void * recv_a16, const int32_t * recv_meta,
                              const int * flags, int64_t n_ranks, int64_t rank, int64_t n_used, int64_t cap,
                              int64_t pairs_hint, float * const * peer_ret, int64_t ret_nb1, int64_t ret_nb2,
                              int * const * peer_flags, int epoch, void * workspace, size_t workspace_bytes,
                              int * dev_err, void * stream);
int    b200_moe_ep_p2p_finish(const int * flags, int64_t n_ranks, int epoch, int * dev_err, void * stream);
/* The owner step for n_members expert stacks that read the same pushed rows (a layer's gate and
 * up): one wait, route and gather, then one grouped GEMM per member storing into its own return
 * buffers (peer_rets[m]: a host array of n_members DEVICE arrays of n_ranks pointers), then one
 * flag to every home. b200_moe_ep_p2p_expert is the one-member case. */
int    b200_moe_ep_p2p_expert_group(int n_members, int wtype, const void * const * local_stacks,
                                    const int64_t * N, int64_t K, int64_t n_local, int64_t expert0,
                                    const void * recv_a16, const int32_t * recv_meta, const int * flags,
                                    int64_t n_ranks, int64_t rank, int64_t n_used, int64_t cap, int64_t pairs_hint,
                                    float * const * const * peer_rets, const int64_t * ret_nb1,
                                    const int64_t * ret_nb2, int * const * peer_flags, int epoch, void * workspace,
                                    size_t workspace_bytes, int * dev_err, void * stream);
/* The owner step for a whole expert FFN, the MoE block's three MUL_MAT_IDs and the GLU between
 * them (gate = MUL_MAT_ID(gate_exps, x), up = MUL_MAT_ID(up_exps, x), h = SWIGLU(gate, up),
 * out = MUL_MAT_ID(down_exps, h): the order llama.cpp's MoE FFN builds its graph in) run where
 * the experts are. The home pushes x ([n_tokens][1][H], ne11 = 1) once with
 * b200_moe_ep_p2p_push; the owner waits, routes and gathers the rows once, keeps gate and up in
 * its own workspace, applies SWIGLU and packs h there, runs the down projection over the same
 * route and stores each [H] output row into its home rank's ret; then flags every home
 * (b200_moe_ep_p2p_finish on the home as for one op). Only x crosses NVLink out and only the
 * down projection's rows come back: the gate / up results and h never leave the owner. The
 * result equals, bit for bit, the single-GPU chain b200_mul_mat_id_group(gate, up),
 * b200_swiglu, b200_mul_mat_id(down). H and F multiples of 32 and of the weight types' blocks;
 * F <= 8192. */
size_t b200_moe_ep_p2p_ffn_workspace_size(int64_t n_ranks, int64_t cap, int64_t H, int64_t F, int64_t n_local,
                                          int64_t n_used);
int    b200_moe_ep_p2p_expert_ffn(int wtype_gate_up, const void * gate_stack, const void * up_stack, int wtype_down,
                                  const void * down_stack, int64_t H, int64_t F, int64_t n_local, int64_t expert0,
                                  const void * recv_a16, const int32_t * recv_meta, const int * flags,
                                  int64_t n_ranks, int64_t rank, int64_t n_used, int64_t cap, int64_t pairs_hint,
                                  float * const * peer_ret, int64_t ret_nb1, int64_t ret_nb2,
                                  int * const * peer_flags, int epoch, void * workspace, size_t workspace_bytes,
                                  int * dev_err, void * stream);

/* ---- the give-up limit of cross-GPU waits -------------------------------------------------------
 * The reference's fault policy (ggml-rocket.cpp:263-307) turns a device route that fails into an
 * error status instead of a hang. Here every kernel that waits for another GPU's flag (the
 * N-sharded and expert-parallel finish and owner waits below) gives up after this many nanoseconds
 * of %globaltimer, records B200_DEV_WAIT_PEER in its error word and returns, so the context stays
 * usable and the caller sees the failure. Process-wide; 0 restores the default of 2 s. */
#define B200_DEV_WAIT_PEER 7
void     b200_set_peer_wait_limit_ns(uint64_t ns);
uint64_t b200_peer_wait_limit_ns(void);

/* ---- MUL_MAT with the weight rows split across GPUs (N-sharded), all-gather by the epilogue ----
 * No counterpart in the reference (its MUL_MAT, ggml-rocket.cpp:4548-4871, runs on one device):
 * the same op with an [N, K] weight cut into n_ranks row blocks, one per GPU. Rank r calls
 *   b200_mul_mat_tp       its GEMM over w_shard (packed rows [col0, col0 + N_shard)) writes
 *                         every output box into every rank's dst (peer_dst: a DEVICE array of
 *                         n_ranks pointers to [M][ldd] f32 buffers, this rank's own included,
 *                         the others mapped with b200_ep_shared_open) at column col0, then puts
 *                         epoch into slot `rank` of every rank's flags (peer_flags, device array)
 *   b200_mul_mat_tp_finish waits (bounded) until every slot of this rank's flags ([n_ranks][4]
 *                         int32) holds epoch: then this rank's dst holds all N columns.
 * epoch must differ from the flags' previous contents (count calls from 1). col0 % 16 == 0,
 * N_shard % 16 == 0, ldd % 4 == 0; the workspace is b200_mul_mat_tp_workspace_size bytes. */
size_t b200_mul_mat_tp_workspace_size(int wtype, int64_t M, int64_t N_shard, int64_t K);
int    b200_mul_mat_tp(int wtype, const void * w_shard, int64_t N_shard, int64_t col0, int64_t K,
                       const float * src1, int64_t lda, int64_t M, float * const * peer_dst, int64_t ldd,
                       int64_t n_ranks, int64_t rank, int * const * peer_flags, int epoch, void * workspace,
                       size_t workspace_bytes, int * dev_err, void * stream);
int    b200_mul_mat_tp_finish(const int * flags, int64_t n_ranks, int epoch, int * dev_err, void * stream);

#ifdef __cplusplus
}
#endif

#endif /* GGML_B200_KERNELS_H */
