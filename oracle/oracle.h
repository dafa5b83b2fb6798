/*
 * CPU oracle for the ggml B200 backend's hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This library restates, in plain C, the arithmetic of the three prefill ops that
 * gregordinary/ggml-rocket offloads (MUL_MAT, FLASH_ATTN_EXT, MUL_MAT_ID) and of the
 * ggml block formats they read (Q8_0, Q4_K, Q6_K). It exists so that tests, the smoke
 * check and the bench's CPU-baseline leg can check the CUDA path against an independent
 * computation. Nothing in the product links or calls it.
 *
 * Parity pins: the dequantizers are checked bit-for-bit against the `gguf` 0.19.0
 * Python package's numpy restatement of ggml's dequantize_row_* (fixtures under
 * tests/golden/, made by tests/golden/make_golden.py). ggml itself is not present in
 * the build container, so the CPU-backend parity rows are pinned only through that
 * package and through the reference's own test constructions.
 */
#ifndef B200_ORACLE_H
#define B200_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type numbering (stable in GGUF files). */
enum {
    ORC_TYPE_F32  = 0,
    ORC_TYPE_F16  = 1,
    ORC_TYPE_Q8_0 = 8,
    ORC_TYPE_Q4_K = 12,
    ORC_TYPE_Q6_K = 14,
    ORC_TYPE_I32  = 26,
    ORC_TYPE_BF16 = 30,
};

uint16_t orc_fp32_to_fp16(float f);
float    orc_fp16_to_fp32(uint16_t h);
void     orc_fp32_to_fp16_row(const float * x, uint16_t * y, int64_t n);
void     orc_fp16_to_fp32_row(const uint16_t * x, float * y, int64_t n);

/* Elements per block and bytes per block of a weight type (1 / element size for plain types). */
int64_t orc_blck_size(int type);
size_t  orc_type_size(int type);
size_t  orc_row_size(int type, int64_t k);

/* One [k] row of `type` decoded to f32, as ggml's to_float does. 0 on success. */
int orc_dequantize_row(int type, const void * src, float * dst, int64_t k);

/* One [k] row of f32 encoded to `type`. Q8_0 follows ggml's reference rounding; the
 * Q4_K / Q6_K encoders are this oracle's own (any valid block is a valid test input,
 * since both sides decode identical bytes). 0 on success. */
int orc_quantize_row(int type, const float * src, void * dst, int64_t k);

/* The reference's activation "sandwich": per row s = max|A[m,:]| (1 when 0),
 * A16 = fp16(A * (1/s)). lda in elements. */
void orc_pack_act(const float * A, int64_t M, int64_t K, int64_t lda, uint16_t * A16, float * scales);

/* C[m*ldc + n] = sum_k A[m*lda + k] * W_n[k] in double, W_n the decoded row n of W
 * (row size orc_row_size(wtype, K)). nthreads <= 0 uses every core. */
int orc_mul_mat_f64(int wtype, const void * W, int64_t N, int64_t K,
                    const float * A, int64_t lda, int64_t M, float * C, int64_t ldc, int nthreads);

/* FLASH_ATTN_EXT in double. Strides are in BYTES, ggml style:
 *   q   F32 [D, T, H]       at q + t*q_nb1 + h*q_nb2 + d*q_nb0
 *   k   F16 [D, KV, HK]     at k + j*k_nb1 + hk*k_nb2 + d*k_nb0
 *   v   F16 [DV, KV, HK]    at v + j*v_nb1 + hk*v_nb2 + c*v_nb0
 *   mask F16 [KV, >=T] or NULL, at mask + t*m_nb1 + j*2
 *   dst F32 [DV, H, T] contiguous
 * q_mode: 0 reads Q as F32; 1 rounds Q to fp16 and applies the scale after the dot;
 * 2 rounds (scale*Q) to fp16 and applies no further scale. A fully masked row is zero. */
int orc_flash_attn_f64(const float * q, int64_t q_nb0, int64_t q_nb1, int64_t q_nb2,
                       const uint16_t * k, int64_t k_nb0, int64_t k_nb1, int64_t k_nb2,
                       const uint16_t * v, int64_t v_nb0, int64_t v_nb1, int64_t v_nb2,
                       const uint16_t * mask, int64_t m_nb1,
                       float * dst, int D, int DV, int T, int H, int KV, int HK,
                       float scale, float softcap, int q_mode, int nthreads);

/* The MUL_MAT_ID bucketing: a stable counting sort of the (slot, token) pairs by expert.
 * ids I32 [n_used, n_tokens] with byte strides ids_nb0/ids_nb1. Writes off[n_expert+1],
 * row_slot[n_used*n_tokens], row_tok[...]. Returns 1 on an id outside [0, n_expert). */
int orc_moe_route(const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1,
                  int64_t n_used, int64_t n_tokens, int64_t n_expert,
                  int32_t * off, int32_t * row_slot, int32_t * row_tok);

/* MUL_MAT_ID in double. as [K, N, n_expert] (expert e at as + e*as_nb2, rows of
 * orc_row_size(wtype, K)); b F32 [K, ne11, n_tokens] (byte strides b_nb1, b_nb2);
 * dst F32 [N, n_used, n_tokens] (byte strides d_nb1, d_nb2). Returns 1 on a bad id. */
int orc_mul_mat_id_f64(int wtype, const void * as, int64_t as_nb2, int64_t K, int64_t N, int64_t n_expert,
                       const float * b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                       const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                       float * dst, int64_t d_nb1, int64_t d_nb2, int nthreads);

/* The glue ops of a layer (RMS_NORM, SILU, SWIGLU, ROPE), restated from ggml's CPU backend
 * (ggml-cpu ops.cpp / vec.h; ggml is not in this container, so these are unpinned: the product's
 * kernels follow the same definitions, and the tests compare the two). Contiguous f32 arrays. */
/* per row of n: squares summed in double in index order, mean = (float)(sum / n),
 * y = x * (1.0f / sqrtf(mean + eps)) */
void orc_rms_norm(const float * x, int64_t rows, int64_t n, float eps, float * y);
/* y = x / (1 + expf(-x)) and y = silu(a) * g */
void orc_silu(const float * x, int64_t n, float * y);
void orc_swiglu(const float * a, const float * g, int64_t n, float * y);
/* ROPE of x [n_tokens][n_head][head_dim], mode 0 (normal) or 2 (neox), ext_factor 0, no
 * frequency factors: theta_0 = pos, theta_{j+1} = theta_j * powf(freq_base, -2 / n_dims);
 * cos / sin of freq_scale * theta_j, times attn_factor; dimensions past n_dims copied */
void orc_rope(const float * x, int64_t head_dim, int64_t n_head, int64_t n_tokens, const int32_t * pos,
              int n_dims, int mode, float freq_base, float freq_scale, float attn_factor, float * y);
/* ggml soft_max without mask: per row of n, w = x * scale, e = expf(w - max(w)) summed in double
 * in index order, y = e * (float)(1 / sum) */
void orc_soft_max(const float * x, int64_t rows, int64_t n, float scale, float * y);

#ifdef __cplusplus
}
#endif

#endif
