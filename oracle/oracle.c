/*
 * CPU oracle for the ggml B200 backend -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Every function here is a plain restatement of the arithmetic the reference performs or
 * calls, written for clarity; each cites the reference file:line it follows. Compiled with
 * -ffp-contract=off so that a multiply followed by an add stays two roundings, as ggml's
 * scalar dequantizers are written.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------------------ */
/* IEEE binary16 conversion, round to nearest even (what ggml_fp32_to_fp16 does on every  */
/* host the reference supports: the F16C / NEON instructions and the portable fallback). */
/* ------------------------------------------------------------------------------------ */

uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                       /* inf / nan */
        if (ax == 0x7f800000u) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    }
    if (ax >= 0x47800000u) return (uint16_t)(sign | 0x7c00u);   /* >= 65536: inf */
    const uint32_t e = ax >> 23;
    if (e < 113) {                                 /* result is fp16-subnormal or zero */
        if (e == 0) return (uint16_t)sign;         /* f32 subnormal: far below 2^-25 */
        const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
        const uint32_t shift = 126 - e;            /* value = mant * 2^(e-150); unit 2^-24 */
        if (shift > 24) return (uint16_t)sign;     /* < 2^-25, rounds to zero (tie goes even) */
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t h = ((e - 112) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;   /* may carry into inf: correct */
    return (uint16_t)(sign | h);
}

float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {                                   /* subnormal: normalise */
            e = 113;
            while (!(m & 0x400u)) { m <<= 1; e--; }
            m &= 0x3ffu;
            x = sign | (e << 23) | (m << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void orc_fp32_to_fp16_row(const float * x, uint16_t * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_fp32_to_fp16(x[i]);
}
void orc_fp16_to_fp32_row(const uint16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_fp16_to_fp32(x[i]);
}

static float bf16_to_fp32(uint16_t b) {
    const uint32_t x = (uint32_t)b << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------------------ */
/* ggml block formats. The layouts are the GGUF on-disk formats (sizes as listed by the   */
/* gguf package's constants: Q8_0 34 B / 32, Q4_K 144 B / 256, Q6_K 210 B / 256). The     */
/* reference decodes them through ggml's to_float at ggml-rocket.cpp:3894-3907 and        */
/* :4060-4064; these decoders restate that published algorithm.                           */
/* ------------------------------------------------------------------------------------ */

#define QK8_0 32
#define QK_K 256

int64_t orc_blck_size(int type) {
    switch (type) {
        case ORC_TYPE_Q8_0: return QK8_0;
        case ORC_TYPE_Q4_K: return QK_K;
        case ORC_TYPE_Q6_K: return QK_K;
        default: return 1;
    }
}

size_t orc_type_size(int type) {
    switch (type) {
        case ORC_TYPE_F32:  return 4;
        case ORC_TYPE_F16:  return 2;
        case ORC_TYPE_BF16: return 2;
        case ORC_TYPE_I32:  return 4;
        case ORC_TYPE_Q8_0: return 34;
        case ORC_TYPE_Q4_K: return 144;
        case ORC_TYPE_Q6_K: return 210;
        default: return 0;
    }
}

size_t orc_row_size(int type, int64_t k) {
    return orc_type_size(type) * (size_t)(k / orc_blck_size(type));
}

static uint16_t rd16(const uint8_t * p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t * p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }

/* Q8_0: { fp16 d; int8 qs[32] }; y = qs * d. */
static void dequant_q8_0(const uint8_t * x, float * y, int64_t k) {
    for (int64_t i = 0; i < k / QK8_0; i++) {
        const uint8_t * b = x + (size_t)i * 34;
        const float d = orc_fp16_to_fp32(rd16(b));
        for (int j = 0; j < QK8_0; j++) y[i * QK8_0 + j] = (float)(int8_t)b[2 + j] * d;
    }
}

/* The 6-bit (scale, min) pair j of a Q4_K super-block, from its 12 packed bytes. */
static void q4k_scale_min(int j, const uint8_t * q, uint8_t * sc, uint8_t * m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m  = q[j + 4] & 63;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
        *m  = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Q4_K: { fp16 d; fp16 dmin; u8 scales[12]; u8 qs[128] }. Eight sub-blocks of 32; the
 * 64 weights of sub-block pair (2c, 2c+1) take the low and high nibbles of qs[32c..32c+31]:
 * y = (d*sc) * q - (dmin*m). */
static void dequant_q4_k(const uint8_t * x, float * y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++) {
        const uint8_t * b = x + (size_t)i * 144;
        const float d = orc_fp16_to_fp32(rd16(b));
        const float dmin = orc_fp16_to_fp32(rd16(b + 2));
        const uint8_t * scales = b + 4;
        const uint8_t * q = b + 16;
        float * out = y + i * QK_K;
        for (int c = 0; c < 4; c++) {
            uint8_t sc, m;
            q4k_scale_min(2 * c, scales, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            q4k_scale_min(2 * c + 1, scales, &sc, &m);
            const float d2 = d * (float)sc, m2 = dmin * (float)m;
            for (int l = 0; l < 32; l++) out[64 * c + l]      = d1 * (float)(q[32 * c + l] & 0xf) - m1;
            for (int l = 0; l < 32; l++) out[64 * c + 32 + l] = d2 * (float)(q[32 * c + l] >> 4) - m2;
        }
    }
}

/* Q6_K: { u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d }. 6-bit codes, offset 32; each
 * 16-weight group w/16 has its own int8 scale: y = (d*scale) * (q - 32). */
static void dequant_q6_k(const uint8_t * x, float * y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++) {
        const uint8_t * b = x + (size_t)i * 210;
        const float d = orc_fp16_to_fp32(rd16(b + 208));
        float * out = y + i * QK_K;
        for (int h = 0; h < 2; h++) {
            const uint8_t * ql = b + 64 * h;
            const uint8_t * qh = b + 128 + 32 * h;
            const int8_t * sc = (const int8_t *)(b + 192 + 8 * h);
            for (int l = 0; l < 32; l++) {
                const int is = l / 16;
                const int q1 = (int)((ql[l] & 0xf) | (((qh[l] >> 0) & 3) << 4)) - 32;
                const int q2 = (int)((ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4)) - 32;
                const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                out[128 * h + l]      = d * (float)sc[is + 0] * (float)q1;
                out[128 * h + l + 32] = d * (float)sc[is + 2] * (float)q2;
                out[128 * h + l + 64] = d * (float)sc[is + 4] * (float)q3;
                out[128 * h + l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
        }
    }
}

int orc_dequantize_row(int type, const void * src, float * dst, int64_t k) {
    switch (type) {
        case ORC_TYPE_F32:  memcpy(dst, src, (size_t)k * 4); return 0;
        case ORC_TYPE_F16:  orc_fp16_to_fp32_row((const uint16_t *)src, dst, k); return 0;
        case ORC_TYPE_BF16: for (int64_t i = 0; i < k; i++) dst[i] = bf16_to_fp32(((const uint16_t *)src)[i]); return 0;
        case ORC_TYPE_Q8_0: if (k % QK8_0) return 1; dequant_q8_0((const uint8_t *)src, dst, k); return 0;
        case ORC_TYPE_Q4_K: if (k % QK_K) return 1; dequant_q4_k((const uint8_t *)src, dst, k); return 0;
        case ORC_TYPE_Q6_K: if (k % QK_K) return 1; dequant_q6_k((const uint8_t *)src, dst, k); return 0;
        default: return 1;
    }
}

/* ------------------------------------------------------------------------------------ */
/* Encoders (test-input generators).                                                     */
/* ------------------------------------------------------------------------------------ */

/* ggml's reference Q8_0 rounding: d = amax/127, q = roundf(x / d). */
static void quant_q8_0(const float * x, uint8_t * y, int64_t k) {
    for (int64_t i = 0; i < k / QK8_0; i++) {
        const float * v = x + i * QK8_0;
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) { const float a = fabsf(v[j]); if (a > amax) amax = a; }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t * b = y + (size_t)i * 34;
        wr16(b, orc_fp32_to_fp16(d));
        for (int j = 0; j < QK8_0; j++) b[2 + j] = (uint8_t)(int8_t)roundf(v[j] * id);
    }
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* A plain min/max Q4_K encoder: per 32-sub-block affine range, 6-bit scales and mins
 * relative to the super-block's d and dmin. */
static void quant_q4_k(const float * x, uint8_t * y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++) {
        const float * v = x + i * QK_K;
        float scl[8], mns[8], max_s = 0.0f, max_m = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = -INFINITY;
            for (int l = 0; l < 32; l++) {
                const float a = v[32 * j + l];
                if (a < lo) lo = a;
                if (a > hi) hi = a;
            }
            if (hi < lo) hi = lo;
            scl[j] = (hi - lo) / 15.0f;
            mns[j] = -lo;
            if (scl[j] > max_s) max_s = scl[j];
            if (mns[j] > max_m) max_m = mns[j];
        }
        uint8_t * b = y + (size_t)i * 144;
        const uint16_t dh = orc_fp32_to_fp16(max_s / 63.0f), mh = orc_fp32_to_fp16(max_m / 63.0f);
        wr16(b, dh);
        wr16(b + 2, mh);
        const float d = orc_fp16_to_fp32(dh), dmin = orc_fp16_to_fp32(mh);
        uint8_t sc[8], mq[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = (uint8_t)(d > 0.0f ? clampi((int)lroundf(scl[j] / d), 0, 63) : 0);
            mq[j] = (uint8_t)(dmin > 0.0f ? clampi((int)lroundf(mns[j] / dmin), 0, 63) : 0);
        }
        uint8_t * s = b + 4;
        for (int j = 0; j < 4; j++) {
            s[j]     = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
            s[j + 4] = (uint8_t)(mq[j] | ((mq[j + 4] >> 4) << 6));
            s[j + 8] = (uint8_t)((sc[j + 4] & 0x0f) | ((mq[j + 4] & 0x0f) << 4));
        }
        uint8_t q[QK_K];
        for (int j = 0; j < 8; j++) {
            const float d1 = d * (float)sc[j], m1 = dmin * (float)mq[j];
            for (int l = 0; l < 32; l++)
                q[32 * j + l] = (uint8_t)(d1 > 0.0f ? clampi((int)lroundf((v[32 * j + l] + m1) / d1), 0, 15) : 0);
        }
        uint8_t * qs = b + 16;
        for (int c = 0; c < 4; c++)
            for (int l = 0; l < 32; l++)
                qs[32 * c + l] = (uint8_t)(q[64 * c + l] | (q[64 * c + 32 + l] << 4));
    }
}

/* A plain symmetric Q6_K encoder: per 16-group scale amax/31, int8 scales relative to d. */
static void quant_q6_k(const float * x, uint8_t * y, int64_t k) {
    for (int64_t i = 0; i < k / QK_K; i++) {
        const float * v = x + i * QK_K;
        float scl[16], max_s = 0.0f;
        for (int j = 0; j < 16; j++) {
            float amax = 0.0f;
            for (int l = 0; l < 16; l++) { const float a = fabsf(v[16 * j + l]); if (a > amax) amax = a; }
            scl[j] = amax / 31.0f;
            if (scl[j] > max_s) max_s = scl[j];
        }
        uint8_t * b = y + (size_t)i * 210;
        const uint16_t dh = orc_fp32_to_fp16(max_s / 127.0f);
        wr16(b + 208, dh);
        const float d = orc_fp16_to_fp32(dh);
        int8_t sc[16];
        for (int j = 0; j < 16; j++) sc[j] = (int8_t)(d > 0.0f ? clampi((int)lroundf(scl[j] / d), -128, 127) : 0);
        memcpy(b + 192, sc, 16);
        uint8_t q[QK_K];
        for (int w = 0; w < QK_K; w++) {
            const float ds = d * (float)sc[w / 16];
            q[w] = (uint8_t)(clampi(ds != 0.0f ? (int)lroundf(v[w] / ds) : 0, -32, 31) + 32);
        }
        for (int h = 0; h < 2; h++) {
            uint8_t * ql = b + 64 * h;
            uint8_t * qh = b + 128 + 32 * h;
            const uint8_t * qq = q + 128 * h;
            for (int l = 0; l < 32; l++) {
                const uint8_t q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
                ql[l]      = (uint8_t)((q1 & 0xf) | ((q3 & 0xf) << 4));
                ql[l + 32] = (uint8_t)((q2 & 0xf) | ((q4 & 0xf) << 4));
                qh[l]      = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
            }
        }
    }
}

int orc_quantize_row(int type, const float * src, void * dst, int64_t k) {
    switch (type) {
        case ORC_TYPE_F32:  memcpy(dst, src, (size_t)k * 4); return 0;
        case ORC_TYPE_F16:  orc_fp32_to_fp16_row(src, (uint16_t *)dst, k); return 0;
        case ORC_TYPE_Q8_0: if (k % QK8_0) return 1; quant_q8_0(src, (uint8_t *)dst, k); return 0;
        case ORC_TYPE_Q4_K: if (k % QK_K) return 1; quant_q4_k(src, (uint8_t *)dst, k); return 0;
        case ORC_TYPE_Q6_K: if (k % QK_K) return 1; quant_q6_k(src, (uint8_t *)dst, k); return 0;
        default: return 1;
    }
}

/* ------------------------------------------------------------------------------------ */
/* MUL_MAT                                                                               */
/* ------------------------------------------------------------------------------------ */

/* rk_pack_act_row (ggml-rocket.cpp:1451-1475): s = max|row| (1 when 0); d = fp16(row * (1/s)). */
void orc_pack_act(const float * A, int64_t M, int64_t K, int64_t lda, uint16_t * A16, float * scales) {
    for (int64_t m = 0; m < M; m++) {
        const float * row = A + m * lda;
        float amax = 0.0f;
        for (int64_t k = 0; k < K; k++) { const float v = fabsf(row[k]); if (v > amax) amax = v; }
        const float s = amax > 0.0f ? amax : 1.0f;
        const float inv = 1.0f / s;
        for (int64_t k = 0; k < K; k++) A16[m * K + k] = orc_fp32_to_fp16(row[k] * inv);
        scales[m] = s;
    }
}

static int set_threads(int nthreads) {
#ifdef _OPENMP
    return nthreads > 0 ? nthreads : omp_get_max_threads();
#else
    (void)nthreads;
    return 1;
#endif
}

/* rocket_cpu_matmul_slice (ggml-rocket.cpp:4053-4084): each weight row decoded through
 * to_float, then an fp64 dot with each activation row, rounded once to f32. */
int orc_mul_mat_f64(int wtype, const void * W, int64_t N, int64_t K,
                    const float * A, int64_t lda, int64_t M, float * C, int64_t ldc, int nthreads) {
    if (orc_type_size(wtype) == 0 || K % orc_blck_size(wtype)) return 1;
    const size_t rbytes = orc_row_size(wtype, K);
    const int nt = set_threads(nthreads);
    int bad = 0;
#pragma omp parallel num_threads(nt)
    {
        float * wrow = (float *)malloc((size_t)K * sizeof(float));
        double * wd = (double *)malloc((size_t)K * sizeof(double));
#pragma omp for schedule(dynamic, 4)
        for (int64_t n = 0; n < N; n++) {
            if (orc_dequantize_row(wtype, (const uint8_t *)W + (size_t)n * rbytes, wrow, K)) { bad = 1; continue; }
            for (int64_t k = 0; k < K; k++) wd[k] = (double)wrow[k];
            for (int64_t m = 0; m < M; m++) {
                const float * a = A + m * lda;
                double acc = 0.0;
                for (int64_t k = 0; k < K; k++) acc += (double)a[k] * wd[k];
                C[m * ldc + n] = (float)acc;
            }
        }
        free(wrow);
        free(wd);
    }
    return bad;
}

/* ------------------------------------------------------------------------------------ */
/* FLASH_ATTN_EXT                                                                        */
/* ------------------------------------------------------------------------------------ */

/* rocket_fa_ref_f32 (ggml-rocket.cpp:5398-5442) and the test oracle ref_fa
 * (test-rocket-fa.cpp:101-135): scores, soft-cap, mask and softmax in double; a fully
 * masked row is written as zeros. */
int orc_flash_attn_f64(const float * q, int64_t q_nb0, int64_t q_nb1, int64_t q_nb2,
                       const uint16_t * k, int64_t k_nb0, int64_t k_nb1, int64_t k_nb2,
                       const uint16_t * v, int64_t v_nb0, int64_t v_nb1, int64_t v_nb2,
                       const uint16_t * mask, int64_t m_nb1,
                       float * dst, int D, int DV, int T, int H, int KV, int HK,
                       float scale, float softcap, int q_mode, int nthreads) {
    if (HK <= 0 || H % HK) return 1;
    const int gqa = H / HK;
    const int nt = set_threads(nthreads);
#pragma omp parallel num_threads(nt)
    {
        double * qd = (double *)malloc((size_t)D * sizeof(double));
        double * sc = (double *)malloc((size_t)KV * sizeof(double));
        double * acc = (double *)malloc((size_t)DV * sizeof(double));
#pragma omp for schedule(dynamic, 1)
        for (int64_t r = 0; r < (int64_t)H * T; r++) {
            const int h = (int)(r / T), t = (int)(r % T), hk = h / gqa;
            const char * qs = (const char *)q + t * q_nb1 + h * q_nb2;
            double post = (double)scale;
            for (int c = 0; c < D; c++) {
                const float x = *(const float *)(qs + c * q_nb0);
                if (q_mode == 1) qd[c] = (double)orc_fp16_to_fp32(orc_fp32_to_fp16(x));
                else if (q_mode == 2) qd[c] = (double)orc_fp16_to_fp32(orc_fp32_to_fp16(x * scale));
                else qd[c] = (double)x;
            }
            if (q_mode == 2) post = 1.0;
            double mx = -INFINITY;
            for (int j = 0; j < KV; j++) {
                const double mv = mask ? (double)orc_fp16_to_fp32(*(const uint16_t *)((const char *)mask + t * m_nb1 + (int64_t)j * 2)) : 0.0;
                if (mv == -INFINITY) { sc[j] = -INFINITY; continue; }
                const char * kr = (const char *)k + j * k_nb1 + hk * k_nb2;
                double d = 0.0;
                for (int c = 0; c < D; c++) d += qd[c] * (double)orc_fp16_to_fp32(*(const uint16_t *)(kr + c * k_nb0));
                double s = d * post;
                if (softcap != 0.0f) s = (double)softcap * tanh(s / (double)softcap);
                s += mv;
                sc[j] = s;
                if (s > mx) mx = s;
            }
            double sum = 0.0;
            for (int j = 0; j < KV; j++) {
                sc[j] = (mx == -INFINITY || sc[j] == -INFINITY) ? 0.0 : exp(sc[j] - mx);
                sum += sc[j];
            }
            for (int c = 0; c < DV; c++) acc[c] = 0.0;
            for (int j = 0; j < KV; j++) {
                if (sc[j] == 0.0) continue;
                const char * vr = (const char *)v + j * v_nb1 + hk * v_nb2;
                for (int c = 0; c < DV; c++) acc[c] += sc[j] * (double)orc_fp16_to_fp32(*(const uint16_t *)(vr + c * v_nb0));
            }
            const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
            float * dr = dst + ((int64_t)t * H + h) * DV;
            for (int c = 0; c < DV; c++) dr[c] = (float)(acc[c] * inv);
        }
        free(qd);
        free(sc);
        free(acc);
    }
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* MUL_MAT_ID                                                                            */
/* ------------------------------------------------------------------------------------ */

/* The bucketing of ggml_backend_rocket_mul_mat_id (ggml-rocket.cpp:6706-6732): count rows
 * per expert, prefix-sum the offsets, then place (slot, token) pairs in token-major order. */
int orc_moe_route(const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1,
                  int64_t n_used, int64_t n_tokens, int64_t n_expert,
                  int32_t * off, int32_t * row_slot, int32_t * row_tok) {
    for (int64_t e = 0; e <= n_expert; e++) off[e] = 0;
    for (int64_t t = 0; t < n_tokens; t++)
        for (int64_t e = 0; e < n_used; e++) {
            const int32_t x = *(const int32_t *)((const char *)ids + t * ids_nb1 + e * ids_nb0);
            if (x < 0 || x >= n_expert) return 1;
            off[x + 1]++;
        }
    for (int64_t e = 0; e < n_expert; e++) off[e + 1] += off[e];
    int32_t * cur = (int32_t *)malloc((size_t)n_expert * sizeof(int32_t));
    for (int64_t e = 0; e < n_expert; e++) cur[e] = off[e];
    for (int64_t t = 0; t < n_tokens; t++)
        for (int64_t e = 0; e < n_used; e++) {
            const int32_t x = *(const int32_t *)((const char *)ids + t * ids_nb1 + e * ids_nb0);
            const int32_t p = cur[x]++;
            row_slot[p] = (int32_t)e;
            row_tok[p] = (int32_t)t;
        }
    free(cur);
    return 0;
}

/* The op layout of ggml-rocket.cpp:6654-6663: dst[:, e, t] = as[:, :, ids[e,t]] . b[:, e % ne11, t].
 * Rows are visited per expert through the bucketing above, as the reference handler does. */
int orc_mul_mat_id_f64(int wtype, const void * as, int64_t as_nb2, int64_t K, int64_t N, int64_t n_expert,
                       const float * b, int64_t b_nb1, int64_t b_nb2, int64_t ne11,
                       const int32_t * ids, int64_t ids_nb0, int64_t ids_nb1, int64_t n_used, int64_t n_tokens,
                       float * dst, int64_t d_nb1, int64_t d_nb2, int nthreads) {
    if (orc_type_size(wtype) == 0 || K % orc_blck_size(wtype)) return 1;
    const int64_t rows = n_used * n_tokens;
    int32_t * off = (int32_t *)malloc((size_t)(n_expert + 1) * sizeof(int32_t));
    int32_t * slot = (int32_t *)malloc((size_t)(rows > 0 ? rows : 1) * sizeof(int32_t));
    int32_t * tok = (int32_t *)malloc((size_t)(rows > 0 ? rows : 1) * sizeof(int32_t));
    if (orc_moe_route(ids, ids_nb0, ids_nb1, n_used, n_tokens, n_expert, off, slot, tok)) {
        free(off); free(slot); free(tok);
        return 1;
    }
    const size_t rbytes = orc_row_size(wtype, K);
    const int nt = set_threads(nthreads);
#pragma omp parallel num_threads(nt)
    {
        float * wrow = (float *)malloc((size_t)K * sizeof(float));
#pragma omp for schedule(dynamic, 1) collapse(2)
        for (int64_t x = 0; x < n_expert; x++) {
            for (int64_t n = 0; n < N; n++) {
                if (off[x + 1] == off[x]) continue;
                orc_dequantize_row(wtype, (const uint8_t *)as + x * as_nb2 + (size_t)n * rbytes, wrow, K);
                for (int64_t r = off[x]; r < off[x + 1]; r++) {
                    const int64_t e = slot[r], t = tok[r];
                    const float * a = (const float *)((const char *)b + t * b_nb2 + (e % ne11) * b_nb1);
                    double acc = 0.0;
                    for (int64_t k = 0; k < K; k++) acc += (double)a[k] * (double)wrow[k];
                    *(float *)((char *)dst + t * d_nb2 + e * d_nb1 + n * 4) = (float)acc;
                }
            }
        }
        free(wrow);
    }
    free(off); free(slot); free(tok);
    return 0;
}

/* ------------------------------------------------------------------------------------ */
/* Glue ops, restated from ggml's CPU definitions (ggml_compute_forward_rms_norm_f32,       */
/* ggml_silu_f32, the swiglu vec op, ggml_compute_forward_rope_f32 with its rope cache).    */
/* ------------------------------------------------------------------------------------ */

void orc_rms_norm(const float * x, int64_t rows, int64_t n, float eps, float * y) {
    for (int64_t r = 0; r < rows; r++) {
        const float * xr = x + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; i++) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / (double)n);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < n; i++) y[r * n + i] = xr[i] * scale;
    }
}

static float orc_silu1(float x) { return x / (1.0f + expf(-x)); }

void orc_silu(const float * x, int64_t n, float * y) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_silu1(x[i]);
}

void orc_swiglu(const float * a, const float * g, int64_t n, float * y) {
    for (int64_t i = 0; i < n; i++) y[i] = orc_silu1(a[i]) * g[i];
}

void orc_rope(const float * x, int64_t head_dim, int64_t n_head, int64_t n_tokens, const int32_t * pos,
              int n_dims, int mode, float freq_base, float freq_scale, float attn_factor, float * y) {
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);
    float * cache = (float *)malloc((size_t)head_dim * sizeof(float));
    for (int64_t t = 0; t < n_tokens; t++) {
        float theta = (float)pos[t];
        for (int64_t i0 = 0; i0 < head_dim; i0 += 2) {
            const float th = freq_scale * theta;
            cache[i0 + 0] = cosf(th) * attn_factor;
            cache[i0 + 1] = sinf(th) * attn_factor;
            theta *= theta_scale;
        }
        for (int64_t h = 0; h < n_head; h++) {
            const float * src = x + (t * n_head + h) * head_dim;
            float * dst = y + (t * n_head + h) * head_dim;
            for (int64_t i0 = 0; i0 < n_dims; i0 += 2) {
                const float c = cache[i0], s = cache[i0 + 1];
                const int64_t e0 = mode == 2 ? i0 / 2 : i0;
                const int64_t e1 = mode == 2 ? i0 / 2 + n_dims / 2 : i0 + 1;
                const float x0 = src[e0], x1 = src[e1];
                dst[e0] = x0 * c - x1 * s;
                dst[e1] = x0 * s + x1 * c;
            }
            for (int64_t i0 = n_dims; i0 < head_dim; i0++) dst[i0] = src[i0];
        }
    }
    free(cache);
}

void orc_soft_max(const float * x, int64_t rows, int64_t n, float scale, float * y) {
    for (int64_t r = 0; r < rows; r++) {
        const float * xr = x + r * n;
        float * yr = y + r * n;
        float mx = -INFINITY;
        for (int64_t i = 0; i < n; i++) {
            const float w = xr[i] * scale;
            if (w > mx) mx = w;
        }
        double sum = 0.0;
        for (int64_t i = 0; i < n; i++) {
            const float e = expf(xr[i] * scale - mx);
            yr[i] = e;
            sum += (double)e;
        }
        const float inv = (float)(1.0 / sum);
        for (int64_t i = 0; i < n; i++) yr[i] *= inv;
    }
}
