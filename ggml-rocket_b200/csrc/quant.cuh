// Device decoders for the ggml block formats the backend accepts as MUL_MAT / MUL_MAT_ID
// weights: Q8_0, Q4_K and Q6_K.
//
// The arithmetic is ggml's to_float (the decode the reference performs through type traits
// at ggml-rocket.cpp:3894-3907), with every product and difference rounded exactly as that
// scalar C code rounds it, so a decoded f32 value is bit-identical to dequantize_row_*:
//   Q8_0  y = q * d
//   Q4_K  y = (d * sc) * q - (dmin * m)      (d*sc*q is exact in f32, so one rounding)
//   Q6_K  y = (d * sc) * (q - 32)
// The fp16 a tensor core consumes is that f32 value rounded to nearest even, which is what
// the reference's rocket_weight_to_fp16 (ggml-rocket.cpp:3853-3931) produces.
//
// Two layouts are read:
//   native  the GGUF block rows, as ggml stores them (row n at n * row_size(K));
//   packed  the device-resident layout the weight cache keeps, laid out for TMA tiles and
//           conflict-free shared-memory reads; same bytes as native:
//             Q4_K  native rows (144-byte super-blocks are already 16-byte multiples)
//             Q6_K  plane A [rows][K/256][208 B] = {ql, qh, scales}; plane D [K/256][rows] fp16
//                   d, transposed so that one 256-byte TMA box holds a 128-row tile's d values
//             Q8_0  rows of 272-byte groups of 8 blocks {d[8], qs[256]}, K padded to 256 with
//                   zero blocks
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace b200 {

enum WeightType : int {
    WT_F32 = 0,
    WT_F16 = 1,
    WT_Q8_0 = 8,
    WT_Q4_K = 12,
    WT_Q6_K = 14,
    WT_BF16 = 30,
};

__host__ __device__ constexpr int wt_block_elems(int t) {
    return t == WT_Q8_0 ? 32 : (t == WT_Q4_K || t == WT_Q6_K) ? 256 : 1;
}
__host__ __device__ constexpr int wt_block_bytes(int t) {
    return t == WT_Q8_0 ? 34 : t == WT_Q4_K ? 144 : t == WT_Q6_K ? 210 : t == WT_F32 ? 4 : 2;
}

__device__ __forceinline__ float h2f_bits(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }

// Q4_K (scale, min) pair of sub-block i (0..7) from the 12 scale bytes held in s0..s2.
__device__ __forceinline__ void q4k_sm(int i, uint32_t s0, uint32_t s1, uint32_t s2,
                                       uint32_t& sc, uint32_t& m) {
    const int sh = 8 * (i & 3);
    const uint32_t a = (s0 >> sh) & 0xffu, b = (s1 >> sh) & 0xffu, c = (s2 >> sh) & 0xffu;
    if (i < 4) {
        sc = a & 63u;
        m = b & 63u;
    } else {
        sc = (c & 0x0fu) | ((a >> 6) << 4);
        m = (c >> 4) | ((b >> 6) << 4);
    }
}

// ---- packed-layout decoders (fused GEMM): one 32-weight half of a 64-weight chunk of one
// row, read from the raw tile the TMA placed in shared memory, -> 16 half2 words ----------
//
// Integer codes become floats without a conversion instruction: a code c in [0, 255] placed in
// the low byte of 0x4B000000 is the float 2^23 + c, and one exact subtraction yields c. The
// arithmetic after that is the scalar formula's, two floats at a time (sm_100 f32x2 ops).

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// Bytes 2i and 2i+1 of x as the floats 2^23 + byte.
__device__ __forceinline__ uint64_t magic_pair(uint32_t x, int i) {
    const uint32_t lo = __byte_perm(x, 0x4B000000u, 0x7540u + 2u * i);
    const uint32_t hi = __byte_perm(x, 0x4B000000u, 0x7541u + 2u * i);
    return f2_pack(__uint_as_float(lo), __uint_as_float(hi));
}
__device__ __forceinline__ uint32_t f2_to_half2(uint64_t v) {
    float lo, hi;
    f2_unpack(v, lo, hi);
    return pack_half2(lo, hi);
}

// Q4_K: raw row = native 144-byte super-blocks. Chunk j of super-block sb, half h: the low (h=0)
// or high (h=1) nibbles of qs[32j .. 32j+31], sub-block 2j+h: y = (d*sc)*q - dmin*m.
// The factors d*sc and dmin*m of the four sub-blocks 2j+h (j = 0..3) one thread decodes from a
// super-block, taken once per super-block; pick(j) selects chunk j's pair.
struct Q4kFactors {
    float d0, d1, d2, d3, m0, m1, m2, m3;
    __device__ __forceinline__ void pick(int j, float& d, float& m) const {
        d = j == 0 ? d0 : j == 1 ? d1 : j == 2 ? d2 : d3;
        m = j == 0 ? m0 : j == 1 ? m1 : j == 2 ? m2 : m3;
    }
};
__device__ __forceinline__ Q4kFactors q4k_factors(const uint8_t* blk, int h) {
    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
    const float d = h2f_bits(hdr.x), dmin = h2f_bits(hdr.x >> 16);
    uint32_t sc[4], m[4];
#pragma unroll
    for (int j = 0; j < 4; j++) q4k_sm(2 * j + h, hdr.y, hdr.z, hdr.w, sc[j], m[j]);
    Q4kFactors f;
    f.d0 = __fmul_rn(d, (float)sc[0]); f.m0 = __fmul_rn(dmin, (float)m[0]);
    f.d1 = __fmul_rn(d, (float)sc[1]); f.m1 = __fmul_rn(dmin, (float)m[1]);
    f.d2 = __fmul_rn(d, (float)sc[2]); f.m2 = __fmul_rn(dmin, (float)m[2]);
    f.d3 = __fmul_rn(d, (float)sc[3]); f.m3 = __fmul_rn(dmin, (float)m[3]);
    return f;
}
__device__ __forceinline__ void decode_q4k_half(const uint8_t* blk, int j, int h, float d1, float m1,
                                                uint32_t (&o)[16]) {
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * j);
    const uint64_t D1 = f2_pack(d1, d1), NM1 = f2_pack(-m1, -m1);
    const uint64_t MAG = f2_pack(-8388608.0f, -8388608.0f);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t x = (h ? (q[w] >> 4) : q[w]) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const uint64_t qf = f2_add(magic_pair(x, i), MAG);          // exact codes
            o[2 * w + i] = f2_to_half2(f2_fma(D1, qf, NM1));            // d1*q exact: one rounding
        }
    }
}

// Both 32-weight halves of chunk j of a Q4_K super-block: the low nibbles of qs[32j .. 32j+31]
// (sub-block 2j, factors d0/m0) into o0 and the high nibbles (sub-block 2j+1, d1/m1) into o1, from
// one read of the 32 bytes.
__device__ __forceinline__ void decode_q4k_both(const uint8_t* blk, int j, float d0, float m0, float d1, float m1,
                                                uint32_t (&o0)[16], uint32_t (&o1)[16]) {
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * j);
    const uint64_t D0 = f2_pack(d0, d0), NM0 = f2_pack(-m0, -m0);
    const uint64_t D1 = f2_pack(d1, d1), NM1 = f2_pack(-m1, -m1);
    const uint64_t MAG = f2_pack(-8388608.0f, -8388608.0f);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t lo = q[w] & 0x0F0F0F0Fu, hi = (q[w] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            o0[2 * w + i] = f2_to_half2(f2_fma(D0, f2_add(magic_pair(lo, i), MAG), NM0));
            o1[2 * w + i] = f2_to_half2(f2_fma(D1, f2_add(magic_pair(hi, i), MAG), NM1));
        }
    }
}

// Q6_K: raw row = 208-byte {ql, qh, scales} super-blocks, d from the transposed d plane.
// Chunk j (hh = j>>1 selects the 128-weight half, s = j&1 the nibble), half h selects
// ql[l] (h=0) or ql[l+32] (h=1); y = (d*sc) * (q - 32).
__device__ __forceinline__ void decode_q6k_half(const uint8_t* blk, float d, int j, int h, uint32_t (&o)[16]) {
    const int hh = j >> 1, s = j & 1;
    const uint4 la = *reinterpret_cast<const uint4*>(blk + 64 * hh + 32 * h);
    const uint4 lb = *reinterpret_cast<const uint4*>(blk + 64 * hh + 32 * h + 16);
    const uint4 ga = *reinterpret_cast<const uint4*>(blk + 128 + 32 * hh);
    const uint4 gb = *reinterpret_cast<const uint4*>(blk + 128 + 32 * hh + 16);
    const int si = 8 * hh + 4 * s + 2 * h;
    const float ds0 = __fmul_rn(d, (float)(int8_t)blk[192 + si]);
    const float ds1 = __fmul_rn(d, (float)(int8_t)blk[192 + si + 1]);
    const uint64_t MAG = f2_pack(-8388640.0f, -8388640.0f);             // -(2^23 + 32)
    const uint32_t ql[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
    const uint32_t qh[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
    const int hs = 4 * s + 2 * h;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t x = ((ql[w] >> (4 * s)) & 0x0F0F0F0Fu) | (((qh[w] >> hs) & 0x03030303u) << 4);
        const uint64_t DS = w < 4 ? f2_pack(ds0, ds0) : f2_pack(ds1, ds1);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const uint64_t qf = f2_add(magic_pair(x, i), MAG);          // exact q - 32
            o[2 * w + i] = f2_to_half2(f2_mul(DS, qf));
        }
    }
}

// Q8_0: raw row = 272-byte groups of 8 blocks {d[8] fp16, qs[256] int8}. Chunk c4 (0..3) of
// the group, half h: block 2*c4 + h; y = q * d.
__device__ __forceinline__ void decode_q8_0_half(const uint8_t* grp, int c4, int h, uint32_t (&o)[16]) {
    const int blk = 2 * c4 + h;
    const float d = __half2float(*reinterpret_cast<const __half*>(grp + 2 * blk));
    const uint4 qa = *reinterpret_cast<const uint4*>(grp + 16 + 32 * blk);
    const uint4 qb = *reinterpret_cast<const uint4*>(grp + 32 + 32 * blk);
    const uint64_t D = f2_pack(d, d);
    const uint64_t MAG = f2_pack(-8388736.0f, -8388736.0f);             // -(2^23 + 128)
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t x = q[w] ^ 0x80808080u;                             // int8 -> q + 128
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const uint64_t qf = f2_add(magic_pair(x, i), MAG);
            o[2 * w + i] = f2_to_half2(f2_mul(qf, D));
        }
    }
}

// ---- native-layout decoders (standalone dequant kernel): one 32-weight group -> f32 ----
// Reads bytes one at a time, since native Q6_K / Q8_0 blocks are only 2-byte aligned.

__device__ __forceinline__ float decode_native_elem_q8_0(const uint8_t* row, int k) {
    const uint8_t* b = row + (size_t)(k >> 5) * 34;
    const float d = h2f_bits((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    return __fmul_rn((float)(int8_t)b[2 + (k & 31)], d);
}

__device__ __forceinline__ float decode_native_elem_q4k(const uint8_t* row, int k) {
    const uint8_t* b = row + (size_t)(k >> 8) * 144;
    const int w = k & 255, c = w >> 6, hi = (w >> 5) & 1, l = w & 31;
    const float d = h2f_bits((uint32_t)b[0] | ((uint32_t)b[1] << 8));
    const float dmin = h2f_bits((uint32_t)b[2] | ((uint32_t)b[3] << 8));
    const uint8_t* s = b + 4;
    const int i = 2 * c + hi;
    uint32_t sc, m;
    if (i < 4) { sc = s[i] & 63u; m = s[i + 4] & 63u; }
    else { sc = (s[i + 4] & 0x0fu) | ((uint32_t)(s[i - 4] >> 6) << 4); m = (s[i + 4] >> 4) | ((uint32_t)(s[i] >> 6) << 4); }
    const uint32_t qb = b[16 + 32 * c + l];
    const uint32_t q = hi ? (qb >> 4) : (qb & 15u);
    return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
}

__device__ __forceinline__ float decode_native_elem_q6k(const uint8_t* row, int k) {
    const uint8_t* b = row + (size_t)(k >> 8) * 210;
    const int w = k & 255, hh = w >> 7, r = w & 127, g = r >> 5, l = r & 31;
    const float d = h2f_bits((uint32_t)b[208] | ((uint32_t)b[209] << 8));
    const uint8_t* ql = b + 64 * hh;
    const uint8_t* qh = b + 128 + 32 * hh;
    const int8_t sc = (int8_t)b[192 + 8 * hh + 2 * g + (l >> 4)];
    const uint32_t lb = ql[l + 32 * (g & 1)];
    const uint32_t nib = (g >= 2) ? (lb >> 4) : (lb & 15u);
    const int q = (int)(nib | (((uint32_t)(qh[l] >> (2 * g)) & 3u) << 4)) - 32;
    return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

}  // namespace b200
