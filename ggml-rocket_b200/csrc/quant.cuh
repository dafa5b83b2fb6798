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
//   packed  the device-resident layout the weight cache keeps, with every load 16-byte
//           aligned: Q4_K is native; Q6_K keeps {ql, qh, scales} (208 B per super-block)
//           in one plane and d in a second plane of fp16; Q8_0 keeps the int8 codes of 256
//           weights (256 B) in one plane and the 32-weight d values in a second plane, K
//           padded to a multiple of 256 with zero blocks.
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
    const uint32_t w[3] = {s0, s1, s2};
    auto B = [&](int b) { return byte_of(w[b >> 2], b & 3); };
    if (i < 4) {
        sc = B(i) & 63u;
        m = B(i + 4) & 63u;
    } else {
        sc = (B(i + 4) & 0x0fu) | ((B(i - 4) >> 6) << 4);
        m = (B(i + 4) >> 4) | ((B(i) >> 6) << 4);
    }
}

// ---- packed-layout decoders: one 64-weight chunk of one row -> 32 half2 words ------------
// `row` points at the row's first byte in plane A; `drow` at its first fp16 in plane D.

__device__ __forceinline__ void decode_q4k_chunk(const uint8_t* row, int kc, uint32_t (&h)[32]) {
    const uint8_t* blk = row + (size_t)(kc >> 2) * 144;
    const int j = kc & 3;
    const uint4 hdr = ld_nc_v4(blk);
    const uint4 qa = ld_nc_v4(blk + 16 + 32 * j);
    const uint4 qb = ld_nc_v4(blk + 32 + 32 * j);
    const float d = h2f_bits(hdr.x), dmin = h2f_bits(hdr.x >> 16);
    uint32_t sc0, m0, sc1, m1;
    q4k_sm(2 * j, hdr.y, hdr.z, hdr.w, sc0, m0);
    q4k_sm(2 * j + 1, hdr.y, hdr.z, hdr.w, sc1, m1);
    const float d1 = __fmul_rn(d, (float)sc0), mm1 = __fmul_rn(dmin, (float)m0);
    const float d2 = __fmul_rn(d, (float)sc1), mm2 = __fmul_rn(dmin, (float)m1);
    const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int i = 0; i < 16; i++) {   // weights 2i, 2i+1: low nibbles of bytes 2i, 2i+1
        const uint32_t b0 = byte_of(q[i >> 1], (2 * i) & 3), b1 = byte_of(q[i >> 1], (2 * i + 1) & 3);
        h[i] = pack_half2(__fsub_rn(__fmul_rn(d1, (float)(b0 & 15u)), mm1),
                          __fsub_rn(__fmul_rn(d1, (float)(b1 & 15u)), mm1));
        h[16 + i] = pack_half2(__fsub_rn(__fmul_rn(d2, (float)(b0 >> 4)), mm2),
                               __fsub_rn(__fmul_rn(d2, (float)(b1 >> 4)), mm2));
    }
}

__device__ __forceinline__ void decode_q6k_chunk(const uint8_t* row, const uint16_t* drow, int kc,
                                                 uint32_t (&h)[32]) {
    const int sb = kc >> 2, j = kc & 3, hh = j >> 1, s = j & 1;
    const uint8_t* blk = row + (size_t)sb * 208;
    const float d = __half2float(__ushort_as_half(__ldg(drow + sb)));
    const uint4 l0 = ld_nc_v4(blk + 64 * hh), l1 = ld_nc_v4(blk + 64 * hh + 16);
    const uint4 l2 = ld_nc_v4(blk + 64 * hh + 32), l3 = ld_nc_v4(blk + 64 * hh + 48);
    const uint4 g0 = ld_nc_v4(blk + 128 + 32 * hh), g1 = ld_nc_v4(blk + 128 + 32 * hh + 16);
    const uint4 sv = ld_nc_v4(blk + 192);
    const uint32_t ql[16] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w,
                             l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
    const uint32_t qh[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
    const int sbase = 8 * hh + 4 * s;
    float ds[4];
#pragma unroll
    for (int g = 0; g < 4; g++) {
        const int si = sbase + g;
        const int8_t scv = static_cast<int8_t>(byte_of(sw[si >> 2], si & 3));
        ds[g] = __fmul_rn(d, (float)scv);
    }
    const int ns = 4 * s;
#pragma unroll
    for (int i = 0; i < 32; i++) {
        float v[2];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int w = 2 * i + e;             // 0..63 within the chunk
            const int second = w >> 5;           // 0: ql[l], 1: ql[l+32]
            const int l = w & 31;
            const uint32_t lb = byte_of(ql[(l + 32 * second) >> 2], (l + 32 * second) & 3);
            const uint32_t hb = byte_of(qh[l >> 2], l & 3);
            const int q = (int)(((lb >> ns) & 15u) | (((hb >> (ns + 2 * second)) & 3u) << 4)) - 32;
            v[e] = __fmul_rn(ds[2 * second + (l >> 4)], (float)q);
        }
        h[i] = pack_half2(v[0], v[1]);
    }
}

__device__ __forceinline__ void decode_q8_0_chunk(const uint8_t* row, const uint16_t* drow, int kc,
                                                  uint32_t (&h)[32]) {
    const uint8_t* qs = row + (size_t)kc * 64;
    const uint32_t dd = __ldg(reinterpret_cast<const uint32_t*>(drow) + kc);
    const float d0 = h2f_bits(dd), d1 = h2f_bits(dd >> 16);
    uint32_t q[16];
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const uint4 v = ld_nc_v4(qs + 16 * c);
        q[4 * c] = v.x; q[4 * c + 1] = v.y; q[4 * c + 2] = v.z; q[4 * c + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 32; i++) {
        const float d = i < 16 ? d0 : d1;
        const int8_t a = static_cast<int8_t>(byte_of(q[i >> 1], (2 * i) & 3));
        const int8_t b = static_cast<int8_t>(byte_of(q[i >> 1], (2 * i + 1) & 3));
        h[i] = pack_half2(__fmul_rn((float)a, d), __fmul_rn((float)b, d));
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
