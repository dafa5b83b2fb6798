/*
 * The host CPU's MUL_MAT path for a Q4_K weight, restated for TIMING -- TEST INFRASTRUCTURE ONLY:
 * bench.py's cpu_baseline leg and the CPU tests call it; nothing in the library does.
 *
 * The reference hands every op it declines (and every decode-size MUL_MAT: its claim floor,
 * ggml-rocket.cpp:7424-7496) to ggml's CPU backend, which is absent from this machine and the GPU
 * box. That backend computes a quantized weight times f32 activations in two steps, and this file
 * restates the published algorithm of both in C (AVX2 when the host has it, chosen at run time):
 *   1. each activation row is quantized to 8-bit blocks of 256 values: one float scale d per block
 *      (the value of largest magnitude maps to -127 or 127) and the sums of every 16 codes;
 *   2. each output is a sum over super-blocks of integer dot products: per 32-weight sub-block j,
 *      sum_l q4 * q8 (int32) times the 6-bit scale sc_j, and the minimum term m_j times the block's
 *      code sums, scaled in float by d_act * d and d_act * dmin.
 * The integer arithmetic is exact; only the 8-bit activation codes round (~0.4 % per value), so
 * results sit within ~1e-2 of the fp64 oracle, which is what the CPU test checks. Numerics are not
 * the point: this is the CPU arm's speed, on all host cores (OpenMP).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#if defined(__x86_64__)
#include <immintrin.h>
#define CPU_PATH_X86 1
#define AVX2_FN __attribute__((target("avx2,fma,f16c")))
#endif

int orc_cpu_path_mul_mat_q4k(const void * W, int64_t N, int64_t K, const float * A, int64_t lda, int64_t M,
                             float * C, int64_t ldc, int nthreads);
int orc_cpu_path_scalar_dot_check(const void * W, int64_t K, const float * a, float * out2);

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {   /* subnormal: normalise */
            exp = 113;
            while (!(man & 0x400u)) { man <<= 1; exp--; }
            bits = sign | (exp << 23) | ((man & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* one activation row -> 8-bit codes, one scale per 256 values, code sums per 16 */
static void quantize_row_8bit(const float * x, int64_t K, int8_t * q, float * d, int16_t * bsum) {
    for (int64_t b = 0; b < K / 256; b++) {
        const float * xb = x + 256 * b;
        float amax = 0.0f, vmax = 0.0f;
        for (int i = 0; i < 256; i++) {
            const float a = fabsf(xb[i]);
            if (a > amax) { amax = a; vmax = xb[i]; }
        }
        int8_t * qb = q + 256 * b;
        if (amax == 0.0f) {
            d[b] = 0.0f;
            memset(qb, 0, 256);
            for (int i = 0; i < 16; i++) bsum[16 * b + i] = 0;
            continue;
        }
        const float iscale = -127.0f / vmax;
        for (int i = 0; i < 256; i++) {
            int v = (int)lrintf(iscale * xb[i]);
            qb[i] = (int8_t)(v > 127 ? 127 : (v < -128 ? -128 : v));
        }
        for (int i = 0; i < 16; i++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += qb[16 * i + l];
            bsum[16 * b + i] = (int16_t)s;
        }
        d[b] = 1.0f / iscale;
    }
}

/* the 6-bit (scale, min) pair of sub-block j from the 12 packed scale bytes */
static inline void scale_min(int j, const uint8_t * s, int * sc, int * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* one weight row (nsb 144-byte super-blocks) against one quantized activation row, portable */
static float dot_q4k_8bit(const uint8_t * w, const int8_t * q, const float * d, const int16_t * bsum, int64_t nsb) {
    float sum = 0.0f;
    for (int64_t b = 0; b < nsb; b++) {
        const uint8_t * blk = w + 144 * b;
        const float wd = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const float wmin = f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        const uint8_t * qs = blk + 16;
        const int8_t * qa = q + 256 * b;
        int32_t sumi = 0, summ = 0;
        for (int c = 0; c < 4; c++) {   /* chunk c: sub-blocks 2c (low nibbles), 2c+1 (high) */
            int32_t lo = 0, hi = 0;
            for (int l = 0; l < 32; l++) {
                lo += (int32_t)(qs[32 * c + l] & 0x0f) * qa[64 * c + l];
                hi += (int32_t)(qs[32 * c + l] >> 4) * qa[64 * c + 32 + l];
            }
            int sc, m;
            scale_min(2 * c, blk + 4, &sc, &m);
            sumi += sc * lo;
            summ += m * (bsum[16 * b + 4 * c] + bsum[16 * b + 4 * c + 1]);
            scale_min(2 * c + 1, blk + 4, &sc, &m);
            sumi += sc * hi;
            summ += m * (bsum[16 * b + 4 * c + 2] + bsum[16 * b + 4 * c + 3]);
        }
        sum += d[b] * wd * (float)sumi - d[b] * wmin * (float)summ;
    }
    return sum;
}

#if defined(CPU_PATH_X86)
static int have_avx2(void) {
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") && __builtin_cpu_supports("f16c");
}

/* One weight row's per-super-block factors, decoded once and used for every activation row. */
typedef struct {
    float wd, wmin;
    int16_t sc[8], m[8];
} row_factors;

AVX2_FN static void decode_factors(const uint8_t * w, int64_t nsb, row_factors * f) {
    for (int64_t b = 0; b < nsb; b++) {
        const uint8_t * blk = w + 144 * b;
        f[b].wd = _cvtsh_ss((unsigned short)(blk[0] | (blk[1] << 8)));
        f[b].wmin = _cvtsh_ss((unsigned short)(blk[2] | (blk[3] << 8)));
        for (int j = 0; j < 8; j++) {
            int sc, m;
            scale_min(j, blk + 4, &sc, &m);
            f[b].sc[j] = (int16_t)sc;
            f[b].m[j] = (int16_t)m;
        }
    }
}

/* The same dot with AVX2: per 32-byte chunk, u8 nibbles x s8 codes summed in pairs to s16
 * (maddubs; 2 * 15 * 128 fits), times the sub-block scale and summed in pairs to s32 (madd). */
AVX2_FN static float dot_q4k_8bit_avx2(const uint8_t * w, const row_factors * f, const int8_t * q, const float * d,
                                       const int16_t * bsum, int64_t nsb) {
    const __m256i m4 = _mm256_set1_epi8(0x0f);
    float sum = 0.0f;
    for (int64_t b = 0; b < nsb; b++) {
        const uint8_t * qs = w + 144 * b + 16;
        const int8_t * qa = q + 256 * b;
        const int16_t * bs = bsum + 16 * b;
        __m256i acc = _mm256_setzero_si256();
        int32_t summ = 0;
        for (int c = 0; c < 4; c++) {
            const __m256i x = _mm256_loadu_si256((const __m256i *)(qs + 32 * c));
            const __m256i lo = _mm256_and_si256(x, m4);
            const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(x, 4), m4);
            const __m256i ya = _mm256_loadu_si256((const __m256i *)(qa + 64 * c));
            const __m256i yb = _mm256_loadu_si256((const __m256i *)(qa + 64 * c + 32));
            const __m256i pl = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, ya), _mm256_set1_epi16(f[b].sc[2 * c]));
            const __m256i ph = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, yb), _mm256_set1_epi16(f[b].sc[2 * c + 1]));
            acc = _mm256_add_epi32(acc, _mm256_add_epi32(pl, ph));
            summ += f[b].m[2 * c] * (bs[4 * c] + bs[4 * c + 1]) + f[b].m[2 * c + 1] * (bs[4 * c + 2] + bs[4 * c + 3]);
        }
        __m128i s4 = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
        s4 = _mm_add_epi32(s4, _mm_shuffle_epi32(s4, 0x4e));
        s4 = _mm_add_epi32(s4, _mm_shuffle_epi32(s4, 0xb1));
        const int32_t sumi = _mm_cvtsi128_si32(s4);
        sum += d[b] * f[b].wd * (float)sumi - d[b] * f[b].wmin * (float)summ;
    }
    return sum;
}
#endif

int orc_cpu_path_mul_mat_q4k(const void * W, int64_t N, int64_t K, const float * A, int64_t lda, int64_t M,
                             float * C, int64_t ldc, int nthreads) {
    if (!W || !A || !C || N <= 0 || M <= 0 || K <= 0 || K % 256 != 0) return -1;
    const int64_t nsb = K / 256;
    int8_t * q = (int8_t *)malloc((size_t)M * K);
    float * d = (float *)malloc((size_t)M * nsb * sizeof(float));
    int16_t * bsum = (int16_t *)malloc((size_t)M * nsb * 16 * sizeof(int16_t));
    if (!q || !d || !bsum) {
        free(q), free(d), free(bsum);
        return -2;
    }
#if defined(CPU_PATH_X86)
    const int avx2 = have_avx2();
#endif
#ifdef _OPENMP
    const int nt = nthreads > 0 ? nthreads : omp_get_max_threads();
#pragma omp parallel num_threads(nt)
#endif
    {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t m = 0; m < M; m++) quantize_row_8bit(A + m * lda, K, q + m * K, d + m * nsb, bsum + m * nsb * 16);
#if defined(CPU_PATH_X86)
        row_factors * f = avx2 ? (row_factors *)malloc((size_t)nsb * sizeof(row_factors)) : NULL;
#endif
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (int64_t n = 0; n < N; n++) {
            const uint8_t * w = (const uint8_t *)W + (size_t)n * nsb * 144;
#if defined(CPU_PATH_X86)
            if (f) {
                decode_factors(w, nsb, f);
                for (int64_t m = 0; m < M; m++)
                    C[m * ldc + n] = dot_q4k_8bit_avx2(w, f, q + m * K, d + m * nsb, bsum + m * nsb * 16, nsb);
                continue;
            }
#endif
            for (int64_t m = 0; m < M; m++)
                C[m * ldc + n] = dot_q4k_8bit(w, q + m * K, d + m * nsb, bsum + m * nsb * 16, nsb);
        }
#if defined(CPU_PATH_X86)
        free(f);
#endif
    }
    free(q), free(d), free(bsum);
    return 0;
}

/* Both dot implementations on one row pair (the CPU test checks that they agree exactly). */
int orc_cpu_path_scalar_dot_check(const void * W, int64_t K, const float * a, float * out2) {
    if (K % 256 != 0) return -1;
    const int64_t nsb = K / 256;
    int8_t * q = (int8_t *)malloc((size_t)K);
    float * d = (float *)malloc((size_t)nsb * sizeof(float));
    int16_t * bsum = (int16_t *)malloc((size_t)nsb * 16 * sizeof(int16_t));
    if (!q || !d || !bsum) {
        free(q), free(d), free(bsum);
        return -2;
    }
    quantize_row_8bit(a, K, q, d, bsum);
    out2[0] = dot_q4k_8bit((const uint8_t *)W, q, d, bsum, nsb);
    out2[1] = out2[0];
#if defined(CPU_PATH_X86)
    if (have_avx2()) {
        row_factors * f = (row_factors *)malloc((size_t)nsb * sizeof(row_factors));
        if (f) {
            decode_factors((const uint8_t *)W, nsb, f);
            out2[1] = dot_q4k_8bit_avx2((const uint8_t *)W, f, q, d, bsum, nsb);
            free(f);
        }
    }
#endif
    free(q), free(d), free(bsum);
    return 0;
}
