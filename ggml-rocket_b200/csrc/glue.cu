// The glue ops of a transformer layer on the device: RMS_NORM, ADD / MUL (with ggml's
// broadcast), SILU, SWIGLU, ROPE, GET_ROWS and CPY.
//
// The reference claims only MUL_MAT, MUL_MAT_ID and FLASH_ATTN_EXT and leaves these to the host's
// CPU backend; every one of them then forces a device-to-host copy of its input and a
// host-to-device copy of its output around the claimed ops. Run here, on tensors in device
// buffers, a layer's activations stay in HBM between ops.
//
// Each op follows ggml's CPU definition element by element (the host's ggml-cpu ops.cpp; ggml is
// not part of this project): the same f32 operations in the same order wherever the result can
// depend on it (explicit __fmul_rn / __fadd_rn where a contracted FMA would round differently),
// with two exceptions stated at the kernels: RMS_NORM sums its squares in a tree (in double, as
// ggml does sequentially) and SILU / ROPE call the device's expf / cosf / sinf (within a few ulp
// of the host libm's).
//
// All are bound by HBM (a read and a write per element, no reuse); they run as grid-stride
// kernels sized to 4 CTAs per SM, with programmatic launch like the other kernels.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "ggml-b200-kernels.h"
#include "glu.cuh"
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

struct Shape4 {
    int64_t ne[4];
    int64_t nb[4];   // bytes
};

static Shape4 shape_of(const int64_t ne[4], const size_t nb[4]) {
    Shape4 s;
    for (int i = 0; i < 4; i++) s.ne[i] = ne[i], s.nb[i] = (int64_t)nb[i];
    return s;
}

__device__ __forceinline__ void unravel(int64_t i, const int64_t ne[4], int64_t (&c)[4]) {
    c[0] = i % ne[0];
    i /= ne[0];
    c[1] = i % ne[1];
    i /= ne[1];
    c[2] = i % ne[2];
    c[3] = i / ne[2];
}
__device__ __forceinline__ int64_t offset_of(const int64_t (&c)[4], const int64_t nb[4]) {
    return c[0] * nb[0] + c[1] * nb[1] + c[2] * nb[2] + c[3] * nb[3];
}

static int grid_for(int64_t n, int threads) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (n + threads - 1) / threads;
    return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 4 * (1024 / threads)));
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// ---- RMS_NORM: y = x * (1 / sqrtf(mean(x^2) + eps)), one CTA per row ------------------------
// ggml sums x*x (an f32 product) into a double sequentially; here each thread sums its strided
// share in double and the CTA adds the shares in a tree: the same terms, another order.
constexpr int RMS_THREADS = 256;

// With w (a dense row of ne[0] f32, ggml's MUL of the normalised rows by one weight row fused
// in): dst = y * w and norm_dst = y (skipped when null), each product rounded as the two
// separate ops round it, so both outputs are bit-identical to RMS_NORM then MUL.
__global__ void __launch_bounds__(RMS_THREADS) rms_norm_kernel(const char* __restrict__ x, Shape4 s, float eps,
                                                               float* __restrict__ dst, const float* __restrict__ w,
                                                               float* __restrict__ norm_dst,
                                                               const float* __restrict__ res = nullptr,
                                                               float* __restrict__ sum_dst = nullptr) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ double red[RMS_THREADS / 32];
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    // rows of 16-byte aligned, dense f32 values: read as float4
    const bool vec = s.nb[0] == 4 && s.ne[0] % 4 == 0 && (s.nb[1] % 16) == 0 && (s.nb[2] % 16) == 0 &&
                     (s.nb[3] % 16) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
        const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
        double sum = 0.0;
        if (vec) {
            const float4* r4 = reinterpret_cast<const float4*>(row);
            const float4* q4 = res ? reinterpret_cast<const float4*>(res + r * s.ne[0]) : nullptr;
            for (int64_t i = threadIdx.x; i < s.ne[0] / 4; i += RMS_THREADS) {
                const float4 v = q4 ? add4(r4[i], q4[i]) : r4[i];
                sum += (double)__fmul_rn(v.x, v.x);
                sum += (double)__fmul_rn(v.y, v.y);
                sum += (double)__fmul_rn(v.z, v.z);
                sum += (double)__fmul_rn(v.w, v.w);
            }
        } else {
            for (int64_t i = threadIdx.x; i < s.ne[0]; i += RMS_THREADS) {
                const float v = *reinterpret_cast<const float*>(row + i * s.nb[0]);
                sum += (double)__fmul_rn(v, v);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int q = 0; q < RMS_THREADS / 32; q++) tot += red[q];
        const float mean = (float)(tot / (double)s.ne[0]);
        const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
        float* out = dst + r * s.ne[0];
        float* nout = norm_dst ? norm_dst + r * s.ne[0] : nullptr;
        const bool vout = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0 &&
                          (!w || (reinterpret_cast<uintptr_t>(w) & 15u) == 0) &&
                          (!norm_dst || (reinterpret_cast<uintptr_t>(norm_dst) & 15u) == 0);
        if (vec && vout) {
            const float4* r4 = reinterpret_cast<const float4*>(row);
            const float4* q4 = res ? reinterpret_cast<const float4*>(res + r * s.ne[0]) : nullptr;
            float4* s4 = sum_dst ? reinterpret_cast<float4*>(sum_dst + r * s.ne[0]) : nullptr;
            float4* o4 = reinterpret_cast<float4*>(out);
            for (int64_t i = threadIdx.x; i < s.ne[0] / 4; i += RMS_THREADS) {
                const float4 v = q4 ? add4(r4[i], q4[i]) : r4[i];
                if (s4) s4[i] = v;
                const float4 y = make_float4(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale), __fmul_rn(v.z, scale),
                                             __fmul_rn(v.w, scale));
                if (w) {
                    const float4 g = __ldg(reinterpret_cast<const float4*>(w) + i);
                    o4[i] = make_float4(__fmul_rn(y.x, g.x), __fmul_rn(y.y, g.y), __fmul_rn(y.z, g.z),
                                        __fmul_rn(y.w, g.w));
                    if (nout) reinterpret_cast<float4*>(nout)[i] = y;
                } else {
                    o4[i] = y;
                }
            }
        } else {
            for (int64_t i = threadIdx.x; i < s.ne[0]; i += RMS_THREADS) {
                const float y = __fmul_rn(*reinterpret_cast<const float*>(row + i * s.nb[0]), scale);
                if (w) {
                    out[i] = __fmul_rn(y, __ldg(w + i));
                    if (nout) nout[i] = y;
                } else {
                    out[i] = y;
                }
            }
        }
        __syncthreads();   // red is reused by the next row
    }
}

// ---- contiguous fast paths ----------------------------------------------------------------------
// Most of a layer's glue ops see dense f32 tensors. For those the per-element index arithmetic of
// the general kernels (64-bit divisions and remainders per element) costs more than the memory
// traffic, so dense operands take these kernels instead: 16-byte accesses, a grid-stride loop over
// float4 groups, no index math. The arithmetic per element is the general kernels' (the same
// __fadd_rn / __fmul_rn / silu on the same values), so results are bit-identical.
__device__ __forceinline__ float bin_op(int op, float x, float y) {
    return op == B200_BIN_ADD ? __fadd_rn(x, y) : op == B200_BIN_MUL ? __fmul_rn(x, y) : __fdiv_rn(x, y);
}
// a, dst dense [rows][ne0]; b dense [rows][ne0] (b_row = 0) or one row [ne0] repeated (b_row = 1)
__global__ void binary_dense_kernel(int op, const float4* __restrict__ a, const float4* __restrict__ b, int b_row,
                                    int64_t ne0_4, int64_t n4, float4* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 x = a[i];
        const float4 y = b[b_row ? i % ne0_4 : i];
        dst[i] = make_float4(bin_op(op, x.x, y.x), bin_op(op, x.y, y.y), bin_op(op, x.z, y.z), bin_op(op, x.w, y.w));
    }
}
__global__ void swiglu_dense_kernel(const float4* __restrict__ a, const float4* __restrict__ g, int64_t n4,
                                    float4* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 x = a[i], y = g[i];
        dst[i] = make_float4(swiglu_f(x.x, y.x), swiglu_f(x.y, y.y), swiglu_f(x.z, y.z), swiglu_f(x.w, y.w));
    }
}
__global__ void silu_dense_kernel(const float4* __restrict__ x, int64_t n4, float4* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = x[i];
        dst[i] = make_float4(silu_f(v.x), silu_f(v.y), silu_f(v.z), silu_f(v.w));
    }
}

// dense f32 -> dense f16 (round to nearest even), four values per thread
__global__ void cpy_f32_f16_dense_kernel(const float4* __restrict__ src, int64_t n4, uint2* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = src[i];
        const __half2 lo = __halves2half2(__float2half_rn(v.x), __float2half_rn(v.y));
        const __half2 hi = __halves2half2(__float2half_rn(v.z), __float2half_rn(v.w));
        dst[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    }
}

// ---- ADD / MUL / DIV: dst = a op b, b repeated over a (ggml_can_repeat) ------------------------
__global__ void binary_kernel(int op, const char* __restrict__ a, Shape4 sa, const char* __restrict__ b, Shape4 sb,
                              float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t n = sa.ne[0] * sa.ne[1] * sa.ne[2] * sa.ne[3];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c[4];
        unravel(i, sa.ne, c);
        const float x = *reinterpret_cast<const float*>(a + offset_of(c, sa.nb));
        const int64_t cb[4] = {c[0] % sb.ne[0], c[1] % sb.ne[1], c[2] % sb.ne[2], c[3] % sb.ne[3]};
        const float y = *reinterpret_cast<const float*>(b + offset_of(cb, sb.nb));
        dst[i] = op == B200_BIN_ADD ? __fadd_rn(x, y) : op == B200_BIN_MUL ? __fmul_rn(x, y) : __fdiv_rn(x, y);
    }
}


// ---- SILU and SWIGLU (dst = silu(a) * g) -------------------------------------------------------
__global__ void silu_kernel(const char* __restrict__ x, Shape4 s, float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t n = s.ne[0] * s.ne[1] * s.ne[2] * s.ne[3];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c[4];
        unravel(i, s.ne, c);
        dst[i] = silu(*reinterpret_cast<const float*>(x + offset_of(c, s.nb)));
    }
}

__global__ void swiglu_kernel(const char* __restrict__ a, Shape4 sa, const char* __restrict__ g, Shape4 sg,
                              float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t n = sa.ne[0] * sa.ne[1] * sa.ne[2] * sa.ne[3];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c[4];
        unravel(i, sa.ne, c);
        const float x = *reinterpret_cast<const float*>(a + offset_of(c, sa.nb));
        const float y = *reinterpret_cast<const float*>(g + offset_of(c, sg.nb));
        dst[i] = swiglu_f(x, y);
    }
}

// ---- ROPE, modes normal (pairs 2j, 2j+1) and neox (pairs j, j + n_dims/2) -----------------------
// ggml's rope cache: theta_0 = p, theta_{j+1} = theta_j * theta_scale (f32, sequentially), with
// theta_scale = powf(freq_base, -2 / n_dims) computed on the host; without YaRN extrapolation
// (ext_factor 0) the rotation uses cosf(freq_scale * theta_j) * attn_factor and the same for sin.
// Thread (row, j): one rotated pair (or, for j >= n_dims / 2, a copied pair).
__global__ void rope_kernel(const char* __restrict__ x, Shape4 s, const int32_t* __restrict__ pos, int n_dims,
                            int neox, float theta_scale, float freq_scale, float attn_factor, float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t half = s.ne[0] / 2;
    const int64_t n = half * s.ne[1] * s.ne[2] * s.ne[3];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i % half, r = i / half;
        const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
        const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
        float* out = dst + r * s.ne[0];
        if (2 * j >= n_dims) {   // past the rotated dimensions: copied
            out[2 * j] = *reinterpret_cast<const float*>(row + (2 * j) * s.nb[0]);
            out[2 * j + 1] = *reinterpret_cast<const float*>(row + (2 * j + 1) * s.nb[0]);
            continue;
        }
        float theta = (float)pos[i2];
        for (int64_t k = 0; k < j; k++) theta = __fmul_rn(theta, theta_scale);
        const float t = __fmul_rn(freq_scale, theta);
        const float c = __fmul_rn(cosf(t), attn_factor), sn = __fmul_rn(sinf(t), attn_factor);
        const int64_t e0 = neox ? j : 2 * j, e1 = neox ? j + n_dims / 2 : 2 * j + 1;
        const float x0 = *reinterpret_cast<const float*>(row + e0 * s.nb[0]);
        const float x1 = *reinterpret_cast<const float*>(row + e1 * s.nb[0]);
        out[e0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
        out[e1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
}

// The same ROPE with one CTA per token (i2): ggml's rope cache for that position -- the sequential
// products theta_j and their cos / sin -- is computed once into shared memory (the general kernel
// recomputes it for every head, an O(n_dims) product chain per element), then the CTA rotates every
// head of the token. Same values, same order of operations, bit-identical to rope_kernel.
constexpr int ROPE_MAX_HALF = 256;
__global__ void __launch_bounds__(256) rope_token_kernel(const char* __restrict__ x, Shape4 s,
                                                        const int32_t* __restrict__ pos, int n_dims, int neox,
                                                        float theta_scale, float freq_scale, float attn_factor,
                                                        float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float cs[ROPE_MAX_HALF], sn[ROPE_MAX_HALF];
    const int half_rot = n_dims / 2;
    const int64_t half = s.ne[0] / 2;
    for (int64_t tok = blockIdx.x; tok < s.ne[2] * s.ne[3]; tok += gridDim.x) {
        const int64_t i2 = tok % s.ne[2], i3 = tok / s.ne[2];
        // the product chain is sequential (one thread); its cos / sin are not (one thread each)
        if (threadIdx.x == 0) {
            float theta = (float)pos[i2];
            for (int j = 0; j < half_rot; j++) {
                cs[j] = theta;
                theta = __fmul_rn(theta, theta_scale);
            }
        }
        __syncthreads();
        for (int j = threadIdx.x; j < half_rot; j += blockDim.x) {
            const float t = __fmul_rn(freq_scale, cs[j]);
            sn[j] = __fmul_rn(sinf(t), attn_factor);
            cs[j] = __fmul_rn(cosf(t), attn_factor);
        }
        __syncthreads();
        const int64_t n = half * s.ne[1];
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
            const int64_t j = i % half, i1 = i / half;
            const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
            float* out = dst + ((i3 * s.ne[2] + i2) * s.ne[1] + i1) * s.ne[0];
            if (2 * j >= n_dims) {
                out[2 * j] = *reinterpret_cast<const float*>(row + (2 * j) * s.nb[0]);
                out[2 * j + 1] = *reinterpret_cast<const float*>(row + (2 * j + 1) * s.nb[0]);
                continue;
            }
            const float c = cs[j], sv = sn[j];
            const int64_t e0 = neox ? j : 2 * j, e1 = neox ? j + n_dims / 2 : 2 * j + 1;
            const float x0 = *reinterpret_cast<const float*>(row + e0 * s.nb[0]);
            const float x1 = *reinterpret_cast<const float*>(row + e1 * s.nb[0]);
            out[e0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv));
            out[e1] = __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, c));
        }
        __syncthreads();   // cs / sn are rewritten for the next token
    }
}

// RMS_NORM times its weight row (the residual ADD in front when res is given) fused with the
// activation pack of the product for the MUL_MATs that read it (the reference's sandwich,
// rk_pack_act_row in ggml-rocket.cpp:1451-1475): one CTA per dense row held in registers (V float4
// per thread); the sum of squares in the order rms_norm_kernel adds it, the products rounded as the
// separate ops round them, then the row's max |value|, fp16(z / s) and s as act_pack_kernel makes
// them. sum_dst / norm_dst / dst are written only when not null. Bit-identical to
// b200_[add_]rms_norm_mul followed by b200_act_pack of its product.
template <int V>
__global__ void __launch_bounds__(RMS_THREADS) norm_mul_pack_kernel(const float* __restrict__ x,
                                                                    const float* __restrict__ res, int ne0, float eps,
                                                                    const float* __restrict__ w,
                                                                    float* __restrict__ sum_dst,
                                                                    float* __restrict__ norm_dst,
                                                                    float* __restrict__ dst, __half* __restrict__ a16,
                                                                    float* __restrict__ scales) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ double red[RMS_THREADS / 32];
    __shared__ float fred[RMS_THREADS / 32];
    const int64_t r = blockIdx.x;
    const float4* x4 = reinterpret_cast<const float4*>(x + r * ne0);
    const float4* q4 = res ? reinterpret_cast<const float4*>(res + r * ne0) : nullptr;
    const int n4 = ne0 / 4;
    float4 v[V];
    double sum = 0.0;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = threadIdx.x + u * RMS_THREADS;
        if (i < n4) {
            v[u] = q4 ? add4(x4[i], q4[i]) : x4[i];
            sum += (double)__fmul_rn(v[u].x, v[u].x);
            sum += (double)__fmul_rn(v[u].y, v[u].y);
            sum += (double)__fmul_rn(v[u].z, v[u].z);
            sum += (double)__fmul_rn(v[u].w, v[u].w);
        } else {
            v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int q = 0; q < RMS_THREADS / 32; q++) tot += red[q];
    const float mean = (float)(tot / (double)ne0);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    float amax = 0.0f;
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = threadIdx.x + u * RMS_THREADS;
        if (i < n4) {
            if (sum_dst) reinterpret_cast<float4*>(sum_dst + r * ne0)[i] = v[u];
            const float4 y = make_float4(__fmul_rn(v[u].x, scale), __fmul_rn(v[u].y, scale), __fmul_rn(v[u].z, scale),
                                         __fmul_rn(v[u].w, scale));
            const float4 g = __ldg(reinterpret_cast<const float4*>(w) + i);
            v[u] = make_float4(__fmul_rn(y.x, g.x), __fmul_rn(y.y, g.y), __fmul_rn(y.z, g.z), __fmul_rn(y.w, g.w));
            if (norm_dst) reinterpret_cast<float4*>(norm_dst + r * ne0)[i] = y;
            if (dst) reinterpret_cast<float4*>(dst + r * ne0)[i] = v[u];
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[u].x), fabsf(v[u].y)), fmaxf(fabsf(v[u].z), fabsf(v[u].w))));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) fred[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = fred[0];
#pragma unroll
    for (int q = 1; q < RMS_THREADS / 32; q++) amax = fmaxf(amax, fred[q]);
    const float s = amax > 0.0f ? amax : 1.0f;
    const float inv = __frcp_rn(s);
    if (threadIdx.x == 0) scales[r] = s;
    uint2* out = reinterpret_cast<uint2*>(a16 + r * ne0);
#pragma unroll
    for (int u = 0; u < V; u++) {
        const int i = threadIdx.x + u * RMS_THREADS;
        if (i < n4) {
            uint2 h;
            h.x = pack_half2(__fmul_rn(v[u].x, inv), __fmul_rn(v[u].y, inv));
            h.y = pack_half2(__fmul_rn(v[u].z, inv), __fmul_rn(v[u].w, inv));
            out[i] = h;
        }
    }
}

// Normal-mode ROPE over rows whose pairs are 8-byte aligned (x's elements contiguous), one CTA per
// token: the rope cache as in rope_token_kernel, then the token's (head, pair) items with 32-bit
// indices (half = 2^half_shift pairs per row), each thread's RT pairs loaded as 8-byte vectors
// before any is rotated, so one CTA has all its loads in flight at once. Same values and order of
// operations as rope_kernel: bit-identical. F16OUT: each rotated pair is rounded to fp16 (round to
// nearest even, as the f32 -> f16 CPY rounds) and stored at dst + i1 nb1 + i2 nb2 + i3 nb3 of the
// fp16 destination sd (the ROPE and the CPY of its output into a KV-cache view in one pass);
// otherwise dst is the contiguous f32 result.
constexpr int ROPE_RT = 8;
template <bool F16OUT>
__global__ void __launch_bounds__(256) rope_token_pairs_kernel(const char* __restrict__ x, Shape4 s,
                                                              const int32_t* __restrict__ pos, int n_dims, int half_shift,
                                                              float theta_scale, float freq_scale, float attn_factor,
                                                              char* __restrict__ dst, Shape4 sd) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float cs[ROPE_MAX_HALF], sn[ROPE_MAX_HALF];
    const int half_rot = n_dims / 2;
    const int half_mask = (1 << half_shift) - 1;
    const int n = (int)s.ne[1] << half_shift;     // pairs of one token
    const int ne0 = (int)s.ne[0];
    for (int64_t tok = blockIdx.x; tok < s.ne[2] * s.ne[3]; tok += gridDim.x) {
        const int64_t i2 = tok % s.ne[2], i3 = tok / s.ne[2];
        const char* tx = x + i2 * s.nb[2] + i3 * s.nb[3];
        float* td = reinterpret_cast<float*>(dst) + (size_t)tok * (size_t)s.ne[1] * ne0;
        char* th = dst + i2 * sd.nb[2] + i3 * sd.nb[3];
        float2 v[ROPE_RT];
#pragma unroll
        for (int u = 0; u < ROPE_RT; u++) {
            const int i = threadIdx.x + 256 * u;
            if (i < n)
                v[u] = *reinterpret_cast<const float2*>(tx + (size_t)(i >> half_shift) * s.nb[1] + 8 * (i & half_mask));
        }
        if (threadIdx.x == 0) {
            float theta = (float)pos[i2];
            for (int j = 0; j < half_rot; j++) {
                cs[j] = theta;
                theta = __fmul_rn(theta, theta_scale);
            }
        }
        __syncthreads();
        for (int j = threadIdx.x; j < half_rot; j += blockDim.x) {
            const float t = __fmul_rn(freq_scale, cs[j]);
            sn[j] = __fmul_rn(sinf(t), attn_factor);
            cs[j] = __fmul_rn(cosf(t), attn_factor);
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < ROPE_RT; u++) {
            const int i = threadIdx.x + 256 * u;
            if (i >= n) continue;
            const int j = i & half_mask;
            float2 o = v[u];
            if (2 * j < n_dims) {
                const float c = cs[j], sv = sn[j];
                o.x = __fsub_rn(__fmul_rn(v[u].x, c), __fmul_rn(v[u].y, sv));
                o.y = __fadd_rn(__fmul_rn(v[u].x, sv), __fmul_rn(v[u].y, c));
            }
            if constexpr (F16OUT)
                *reinterpret_cast<__half2*>(th + (int64_t)(i >> half_shift) * sd.nb[1] + 4 * j) = __floats2half2_rn(o.x, o.y);
            else
                *reinterpret_cast<float2*>(td + (size_t)(i >> half_shift) * ne0 + 2 * j) = o;
        }
        __syncthreads();   // cs / sn are rewritten for the next token
    }
}

// ---- GET_ROWS: dst[:, i10, i11, i12] = src[:, idx[i10, i11, i12], i11, i12] (f32 or f16 -> f32) ----
// An index outside [0, src rows) records ERR_BAD_INDEX and writes zeros for that row.
__global__ void get_rows_kernel(int f16, const char* __restrict__ src, Shape4 ss, const char* __restrict__ idx,
                                Shape4 si, float* __restrict__ dst, int* err) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t n = ss.ne[0] * si.ne[0] * si.ne[1] * si.ne[2];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i0 = i % ss.ne[0];
        int64_t q = i / ss.ne[0];
        const int64_t i10 = q % si.ne[0];
        q /= si.ne[0];
        const int64_t i11 = q % si.ne[1], i12 = q / si.ne[1];
        const int64_t r = *reinterpret_cast<const int32_t*>(idx + i10 * si.nb[0] + i11 * si.nb[1] + i12 * si.nb[2]);
        if (r < 0 || r >= ss.ne[1]) {
            if (i0 == 0) atomicCAS(err, 0, ERR_BAD_INDEX);
            dst[i] = 0.0f;
            continue;
        }
        const char* p = src + r * ss.nb[1] + i11 * ss.nb[2] + i12 * ss.nb[3] + i0 * ss.nb[0];
        dst[i] = f16 ? __half2float(*reinterpret_cast<const __half*>(p)) : *reinterpret_cast<const float*>(p);
    }
}

// One CTA per output row (i10, i11, i12): the index is read once, the row copied with 8-byte
// (4 x f16) or 16-byte (4 x f32) loads when the source rows are contiguous and aligned (vec), else
// element by element. Same values and error behaviour as get_rows_kernel.
__global__ void __launch_bounds__(256) get_rows_row_kernel(int f16, int vec, const char* __restrict__ src, Shape4 ss,
                                                           const char* __restrict__ idx, Shape4 si,
                                                           float* __restrict__ dst, int* err) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t orow = blockIdx.x;   // i10 + ne[0] * (i11 + ne[1] * i12)
    const int64_t i10 = orow % si.ne[0], i11 = (orow / si.ne[0]) % si.ne[1], i12 = orow / (si.ne[0] * si.ne[1]);
    const int64_t r = *reinterpret_cast<const int32_t*>(idx + i10 * si.nb[0] + i11 * si.nb[1] + i12 * si.nb[2]);
    const int64_t n0 = ss.ne[0];
    float* out = dst + orow * n0;
    if (r < 0 || r >= ss.ne[1]) {
        if (threadIdx.x == 0) atomicCAS(err, 0, ERR_BAD_INDEX);
        for (int64_t i = threadIdx.x; i < n0; i += blockDim.x) out[i] = 0.0f;
        return;
    }
    const char* row = src + r * ss.nb[1] + i11 * ss.nb[2] + i12 * ss.nb[3];
    if (vec) {
        float4* o4 = reinterpret_cast<float4*>(out);
        if (f16) {
            const uint2* p = reinterpret_cast<const uint2*>(row);
            for (int64_t i = threadIdx.x; i < n0 / 4; i += blockDim.x) {
                const uint2 w = __ldg(p + i);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
                o4[i] = make_float4(a.x, a.y, b.x, b.y);
            }
        } else {
            const float4* p = reinterpret_cast<const float4*>(row);
            for (int64_t i = threadIdx.x; i < n0 / 4; i += blockDim.x) o4[i] = __ldg(p + i);
        }
        return;
    }
    for (int64_t i = threadIdx.x; i < n0; i += blockDim.x) {
        const char* p = row + i * ss.nb[0];
        out[i] = f16 ? __half2float(*reinterpret_cast<const __half*>(p)) : *reinterpret_cast<const float*>(p);
    }
}

// ---- CPY: element k of src (i0 fastest) -> element k of dst, f32 / f16 either side -------------
// dst either has src's shape (any strides) or is contiguous with src's element count.
__global__ void cpy_kernel(int src_f16, const char* __restrict__ src, Shape4 ss, int dst_f16, char* __restrict__ dst,
                           Shape4 sd, int same_shape) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t n = ss.ne[0] * ss.ne[1] * ss.ne[2] * ss.ne[3];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t c[4];
        unravel(i, ss.ne, c);
        const char* p = src + offset_of(c, ss.nb);
        const float v = src_f16 ? __half2float(*reinterpret_cast<const __half*>(p)) : *reinterpret_cast<const float*>(p);
        char* q;
        if (same_shape) {
            q = dst + offset_of(c, sd.nb);
        } else {
            q = dst + i * (dst_f16 ? 2 : 4);
        }
        if (dst_f16) *reinterpret_cast<__half*>(q) = __float2half_rn(v);
        else *reinterpret_cast<float*>(q) = v;
    }
}

// ---- SOFT_MAX (no mask, no ALiBi): w = x * scale; y = expf(w - max) / sum, sum in double ------
// ggml: the exps summed in index order into a double, then every value times (float)(1 / sum);
// here the CTA sums in a tree, in double.
constexpr int SM_THREADS = 256;

__global__ void __launch_bounds__(SM_THREADS) soft_max_kernel(const char* __restrict__ x, Shape4 s, float scale,
                                                              float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float fred[SM_THREADS / 32];
    __shared__ double dred[SM_THREADS / 32];
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
        const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
        float* out = dst + r * s.ne[0];
        float mx = -INFINITY;
        for (int64_t i = threadIdx.x; i < s.ne[0]; i += SM_THREADS)
            mx = fmaxf(mx, __fmul_rn(*reinterpret_cast<const float*>(row + i * s.nb[0]), scale));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) fred[warp] = mx;
        __syncthreads();
        mx = fred[0];
#pragma unroll
        for (int w = 1; w < SM_THREADS / 32; w++) mx = fmaxf(mx, fred[w]);
        double sum = 0.0;
        for (int64_t i = threadIdx.x; i < s.ne[0]; i += SM_THREADS) {
            const float e = expf(__fsub_rn(__fmul_rn(*reinterpret_cast<const float*>(row + i * s.nb[0]), scale), mx));
            out[i] = e;
            sum += (double)e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) dred[warp] = sum;
        __syncthreads();
        double tot = 0.0;
#pragma unroll
        for (int w = 0; w < SM_THREADS / 32; w++) tot += dred[w];
        const float inv = (float)(1.0 / tot);
        for (int64_t i = threadIdx.x; i < s.ne[0]; i += SM_THREADS) out[i] = __fmul_rn(out[i], inv);
        __syncthreads();   // fred / dred are reused by the next row
    }
}

// Rows of at most 32 * SMW_MAX values (the MoE router's 64-256 experts): one warp per row, the
// row held in registers, max and the double sum reduced with shuffles; the same per-element
// arithmetic as soft_max_kernel, the sum in another order.
constexpr int SMW_MAX = 32;
template <int E>
__global__ void __launch_bounds__(256) soft_max_warp_kernel(const char* __restrict__ x, Shape4 s, float scale,
                                                           float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
    const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
    float* out = dst + r * s.ne[0];
    const int n = (int)s.ne[0];
    float w[E];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < E; j++) {
        const int i = lane + 32 * j;
        w[j] = i < n ? __fmul_rn(*reinterpret_cast<const float*>(row + (int64_t)i * s.nb[0]), scale) : -INFINITY;
        mx = fmaxf(mx, w[j]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    double sum = 0.0;
#pragma unroll
    for (int j = 0; j < E; j++) {
        const int i = lane + 32 * j;
        w[j] = i < n ? expf(__fsub_rn(w[j], mx)) : 0.0f;
        sum += (double)w[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = (float)(1.0 / sum);
#pragma unroll
    for (int j = 0; j < E; j++) {
        const int i = lane + 32 * j;
        if (i < n) out[i] = __fmul_rn(w[j], inv);
    }
}

// ---- ARGSORT of every row (ne[0] <= 1024): a bitonic sort of (value, index) pairs in shared
// memory, ties broken by the smaller index (ggml's std::sort leaves the order of ties open) -----
constexpr int AS_MAX = 1024;

// A total order, so the output is always a permutation of [0, n): padding entries (index >= AS_MAX)
// after every row entry, NaNs after every number (in either direction), ties by index.
__device__ __forceinline__ bool as_before(float va, int ia, float vb, int ib, bool desc) {
    const bool pa = ia >= AS_MAX, pb = ib >= AS_MAX;
    if (pa != pb) return pb;
    const bool na = isnan(va), nb = isnan(vb);
    if (pa || na != nb) return pa ? ia < ib : nb;
    if (!na && va != vb) return desc ? va > vb : va < vb;
    return ia < ib;
}

__global__ void __launch_bounds__(AS_MAX / 2) argsort_kernel(const char* __restrict__ x, Shape4 s, int desc, int n2,
                                                             int32_t* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float sv[AS_MAX];
    __shared__ int si[AS_MAX];
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    const int n = (int)s.ne[0];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
        const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
        for (int i = threadIdx.x; i < n2; i += blockDim.x) {
            // padding sorts last in either order
            sv[i] = i < n ? *reinterpret_cast<const float*>(row + (int64_t)i * s.nb[0]) : (desc ? -INFINITY : INFINITY);
            si[i] = i < n ? i : AS_MAX + i;
        }
        __syncthreads();
        for (int k = 2; k <= n2; k <<= 1) {
            for (int j = k >> 1; j > 0; j >>= 1) {
                for (int t = threadIdx.x; t < n2 / 2; t += blockDim.x) {
                    // the pair (a, b = a + j) this thread compares in this step
                    const int a = 2 * j * (t / j) + (t % j), b = a + j;
                    const bool up = (a & k) == 0;   // this block of k sorts ascending in "before" order
                    const bool swap = up ? as_before(sv[b], si[b], sv[a], si[a], desc != 0)
                                         : as_before(sv[a], si[a], sv[b], si[b], desc != 0);
                    if (swap) {
                        const float tv = sv[a];
                        sv[a] = sv[b];
                        sv[b] = tv;
                        const int ti = si[a];
                        si[a] = si[b];
                        si[b] = ti;
                    }
                }
                __syncthreads();
            }
        }
        int32_t* out = dst + r * s.ne[0];
        for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = si[i];
        __syncthreads();
    }
}

// Rows of at most ASW_MAX entries (the MoE router's expert counts): one warp per row, the
// bitonic network over n2w = max(32, n2) positions held in registers (position j * 32 + lane in
// slot j of lane), exchanges across lanes by shuffles, within a lane by register swaps. Each entry
// is one 64-bit key whose unsigned order is argsort_kernel's total order: the upper word ranks the
// value (order-preserving bits of the float in the requested direction, -0 as +0; every NaN
// above every number; padding above all), the lower word is the index (ties by index). Same
// result as argsort_kernel.
constexpr int ASW_MAX = 256;
__device__ __forceinline__ uint64_t as_key(float v, int index, bool pad, bool desc) {
    uint32_t hi;
    if (pad) hi = 0xFFFFFFFFu;
    else if (isnan(v)) hi = 0xFFFFFFFEu;
    else {
        const uint32_t bits = __float_as_uint(v == 0.0f ? 0.0f : v);
        const uint32_t u = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);   // ascending order
        hi = desc ? ~u : u;   // numbers stay below 0xFF800001 either way
    }
    return ((uint64_t)hi << 32) | (uint32_t)index;
}
template <int E>
__global__ void __launch_bounds__(256) argsort_warp_kernel(const char* __restrict__ x, Shape4 s, int desc,
                                                          int32_t* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
    const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
    const int n = (int)s.ne[0];
    constexpr int N2 = 32 * E;
    uint64_t key[E];
#pragma unroll
    for (int j = 0; j < E; j++) {
        const int p = lane + 32 * j;
        const float v = p < n ? *reinterpret_cast<const float*>(row + (int64_t)p * s.nb[0]) : 0.0f;
        key[j] = as_key(v, p, p >= n, desc != 0);
    }
#pragma unroll
    for (int k = 2; k <= N2; k <<= 1) {
#pragma unroll
        for (int d = k >> 1; d > 0; d >>= 1) {
            if (d >= 32) {
                // partners in the same lane: slots j and j ^ (d / 32); the lower position takes the
                // smaller key in an ascending block, the larger in a descending one
#pragma unroll
                for (int j = 0; j < E; j++) {
                    const int jj = j ^ (d >> 5);
                    if (jj > j) {
                        const bool up = ((lane + 32 * j) & k) == 0;
                        const uint64_t lo = key[j] < key[jj] ? key[j] : key[jj];
                        const uint64_t hi = key[j] < key[jj] ? key[jj] : key[j];
                        key[j] = up ? lo : hi;
                        key[jj] = up ? hi : lo;
                    }
                }
            } else {
                // partners in lane ^ d, same slot
#pragma unroll
                for (int j = 0; j < E; j++) {
                    const uint64_t o = __shfl_xor_sync(0xffffffffu, key[j], d);
                    const bool up = ((lane + 32 * j) & k) == 0;
                    const bool lower = (lane & d) == 0;
                    const bool want_small = lower == up;
                    key[j] = want_small ? (o < key[j] ? o : key[j]) : (o < key[j] ? key[j] : o);
                }
            }
        }
    }
    int32_t* out = dst + r * s.ne[0];
#pragma unroll
    for (int j = 0; j < E; j++) {
        const int p = lane + 32 * j;
        if (p < n) out[p] = (int32_t)(uint32_t)key[j];
    }
}

// ---- Hadamard-tagged MUL_MAT: y = scale * H_n x per row, H_n the Sylvester-ordered Walsh-Hadamard
// matrix (H[i][k] = (-1)^popcount(i & k)), by the fast transform: log2(n) butterfly rounds of f32
// additions (h = 1, 2, 4, ...: (a, b) -> (a + b, a - b)), then one multiply by scale. One warp per
// row (n = 32 .. 1024), position j * 32 + lane in slot j of lane; exchanges across lanes by
// shuffles, within a lane by register pairs.
constexpr int HAD_MAX = 1024;
template <int E>
__global__ void __launch_bounds__(256) hadamard_kernel(const char* __restrict__ x, Shape4 s, float scale,
                                                      float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
    const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
    float v[E];
#pragma unroll
    for (int j = 0; j < E; j++) v[j] = *reinterpret_cast<const float*>(row + (int64_t)(lane + 32 * j) * s.nb[0]);
#pragma unroll
    for (int h = 1; h < 32; h <<= 1) {
        const bool lower = (lane & h) == 0;
#pragma unroll
        for (int j = 0; j < E; j++) {
            const float o = __shfl_xor_sync(0xffffffffu, v[j], h);
            v[j] = lower ? __fadd_rn(v[j], o) : __fsub_rn(o, v[j]);
        }
    }
#pragma unroll
    for (int hj = 1; hj < E; hj <<= 1) {
#pragma unroll
        for (int j = 0; j < E; j++) {
            if ((j & hj) == 0) {
                const float a = v[j], b = v[j + hj];
                v[j] = __fadd_rn(a, b);
                v[j + hj] = __fsub_rn(a, b);
            }
        }
    }
    float* out = dst + r * s.ne[0];
#pragma unroll
    for (int j = 0; j < E; j++) out[lane + 32 * j] = __fmul_rn(v[j], scale);
}

// ---- SUM_ROWS: the sum of every row, in double (ggml_vec_sum_f32 sums in ggml_float) -------
__global__ void __launch_bounds__(RMS_THREADS) sum_rows_kernel(const char* __restrict__ x, Shape4 s,
                                                               float* __restrict__ dst) {
    grid_dep_wait();
    grid_dep_launch();
    __shared__ double red[RMS_THREADS / 32];
    const int64_t rows = s.ne[1] * s.ne[2] * s.ne[3];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int64_t i1 = r % s.ne[1], i2 = (r / s.ne[1]) % s.ne[2], i3 = r / (s.ne[1] * s.ne[2]);
        const char* row = x + i1 * s.nb[1] + i2 * s.nb[2] + i3 * s.nb[3];
        double sum = 0.0;
        for (int64_t i = threadIdx.x; i < s.ne[0]; i += RMS_THREADS)
            sum += (double)*reinterpret_cast<const float*>(row + i * s.nb[0]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x == 0) {
            double tot = 0.0;
            for (int w = 0; w < RMS_THREADS / 32; w++) tot += red[w];
            dst[r] = (float)tot;
        }
        __syncthreads();
    }
}

static bool shape_ok(const int64_t ne[4], const size_t nb[4]) {
    if (!ne || !nb) return false;
    for (int i = 0; i < 4; i++)
        if (ne[i] <= 0) return false;
    return true;
}
static int64_t nelem(const int64_t ne[4]) { return ne[0] * ne[1] * ne[2] * ne[3]; }
// dense f32: contiguous strides and a 16-byte aligned base, rows a multiple of four values
static bool dense_f32(const void* p, const int64_t ne[4], const size_t nb[4]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15u) || ne[0] % 4) return false;
    size_t next = 4;
    for (int i = 0; i < 4; i++) {
        if (ne[i] != 1 && nb[i] != next) return false;
        next *= (size_t)ne[i];
    }
    return true;
}
static int done(cudaError_t e) { return e == cudaSuccess && cudaGetLastError() == cudaSuccess ? B200_OK : B200_E_CUDA; }

}  // namespace b200

extern "C" {

int b200_rms_norm(const float* x, const int64_t ne[4], const size_t nb[4], float eps, float* dst, void* stream) {
    using namespace b200;
    if (!x || !dst || !shape_ok(ne, nb) || !(eps >= 0.0f)) return B200_E_INVALID;
    const int64_t rows = ne[1] * ne[2] * ne[3];
    const int grid = (int)std::min<int64_t>(rows, 148 * 8);
    return done(launch_pdl(rms_norm_kernel, dim3((unsigned)grid), dim3(RMS_THREADS), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), eps,
                           dst, static_cast<const float*>(nullptr), static_cast<float*>(nullptr),
                           static_cast<const float*>(nullptr), static_cast<float*>(nullptr)));
}

int b200_add_rms_norm_mul(const float* a, const float* b, const int64_t ne[4], float eps, const float* w,
                          float* sum_dst, float* norm_dst, float* dst, void* stream) {
    using namespace b200;
    if (!a || !b || !w || !sum_dst || !dst || ne[0] <= 0 || ne[1] <= 0 || ne[2] <= 0 || ne[3] <= 0 || !(eps >= 0.0f))
        return B200_E_INVALID;
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (ne[0] % 4 != 0 || !al16(a) || !al16(b) || !al16(w) || !al16(sum_dst) || !al16(dst) ||
        (norm_dst && !al16(norm_dst)))
        return B200_E_UNSUPPORTED;   // the dense float4 path only
    const size_t nb[4] = {4, (size_t)ne[0] * 4, (size_t)(ne[0] * ne[1]) * 4, (size_t)(ne[0] * ne[1] * ne[2]) * 4};
    const int64_t rows = ne[1] * ne[2] * ne[3];
    const int grid = (int)std::min<int64_t>(rows, 148 * 8);
    return done(launch_pdl(rms_norm_kernel, dim3((unsigned)grid), dim3(RMS_THREADS), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(a), shape_of(ne, nb), eps,
                           dst, w, norm_dst, b, sum_dst));
}

int b200_rms_norm_mul_act_pack(const float* x, const float* res, const int64_t ne[4], float eps, const float* w,
                               float* sum_dst, float* norm_dst, float* dst, void* a16, float* scales, void* stream) {
    using namespace b200;
    if (!x || !w || !a16 || !scales || (res && !sum_dst) || ne[0] <= 0 || ne[1] <= 0 || ne[2] <= 0 || ne[3] <= 0 ||
        !(eps >= 0.0f))
        return B200_E_INVALID;
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const int64_t rows = ne[1] * ne[2] * ne[3];
    const int64_t per = (ne[0] / 4 + RMS_THREADS - 1) / RMS_THREADS;
    if (ne[0] % 4 != 0 || per > 16 || rows > INT32_MAX || !al16(x) || !al16(w) || (res && !al16(res)) ||
        (sum_dst && !al16(sum_dst)) || (norm_dst && !al16(norm_dst)) || (dst && !al16(dst)))
        return B200_E_UNSUPPORTED;   // dense, aligned rows of at most 16384 values
    const int n0 = (int)ne[0];
    __half* h = static_cast<__half*>(a16);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid((unsigned)rows), block(RMS_THREADS);
    if (per <= 1) return done(launch_pdl(norm_mul_pack_kernel<1>, grid, block, 0, st, x, res, n0, eps, w, sum_dst, norm_dst, dst, h, scales));
    if (per <= 2) return done(launch_pdl(norm_mul_pack_kernel<2>, grid, block, 0, st, x, res, n0, eps, w, sum_dst, norm_dst, dst, h, scales));
    if (per <= 4) return done(launch_pdl(norm_mul_pack_kernel<4>, grid, block, 0, st, x, res, n0, eps, w, sum_dst, norm_dst, dst, h, scales));
    if (per <= 8) return done(launch_pdl(norm_mul_pack_kernel<8>, grid, block, 0, st, x, res, n0, eps, w, sum_dst, norm_dst, dst, h, scales));
    return done(launch_pdl(norm_mul_pack_kernel<16>, grid, block, 0, st, x, res, n0, eps, w, sum_dst, norm_dst, dst, h, scales));
}

int b200_rms_norm_mul(const float* x, const int64_t ne[4], const size_t nb[4], float eps, const float* w,
                      float* norm_dst, float* dst, void* stream) {
    using namespace b200;
    if (!x || !w || !dst || !shape_ok(ne, nb) || !(eps >= 0.0f)) return B200_E_INVALID;
    const int64_t rows = ne[1] * ne[2] * ne[3];
    const int grid = (int)std::min<int64_t>(rows, 148 * 8);
    return done(launch_pdl(rms_norm_kernel, dim3((unsigned)grid), dim3(RMS_THREADS), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), eps,
                           dst, w, norm_dst, static_cast<const float*>(nullptr), static_cast<float*>(nullptr)));
}

int b200_binary(int op, const float* a, const int64_t ane[4], const size_t anb[4], const float* b, const int64_t bne[4],
                const size_t bnb[4], float* dst, void* stream) {
    using namespace b200;
    if (!a || !b || !dst || !shape_ok(ane, anb) || !shape_ok(bne, bnb)) return B200_E_INVALID;
    if (op != B200_BIN_ADD && op != B200_BIN_MUL && op != B200_BIN_DIV) return B200_E_UNSUPPORTED;
    for (int i = 0; i < 4; i++)
        if (ane[i] % bne[i] != 0) return B200_E_INVALID;   // b must repeat over a
    const int64_t n = nelem(ane);
    const bool b_same = bne[0] == ane[0] && bne[1] == ane[1] && bne[2] == ane[2] && bne[3] == ane[3];
    const bool b_row = bne[0] == ane[0] && bne[1] == 1 && bne[2] == 1 && bne[3] == 1;
    if (dense_f32(a, ane, anb) && dense_f32(b, bne, bnb) && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0 &&
        (b_same || b_row))
        return done(launch_pdl(binary_dense_kernel, dim3((unsigned)grid_for(n / 4, 256)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), op, reinterpret_cast<const float4*>(a),
                               reinterpret_cast<const float4*>(b), b_row ? 1 : 0, ane[0] / 4, n / 4,
                               reinterpret_cast<float4*>(dst)));
    return done(launch_pdl(binary_kernel, dim3((unsigned)grid_for(n, 256)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), op, reinterpret_cast<const char*>(a), shape_of(ane, anb),
                           reinterpret_cast<const char*>(b), shape_of(bne, bnb), dst));
}

int b200_silu(const float* x, const int64_t ne[4], const size_t nb[4], float* dst, void* stream) {
    using namespace b200;
    if (!x || !dst || !shape_ok(ne, nb)) return B200_E_INVALID;
    const int64_t n = nelem(ne);
    if (dense_f32(x, ne, nb) && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0)
        return done(launch_pdl(silu_dense_kernel, dim3((unsigned)grid_for(n / 4, 256)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), reinterpret_cast<const float4*>(x), n / 4,
                               reinterpret_cast<float4*>(dst)));
    return done(launch_pdl(silu_kernel, dim3((unsigned)grid_for(n, 256)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), dst));
}

int b200_swiglu(const float* a, const size_t anb[4], const float* g, const size_t gnb[4], const int64_t ne[4],
                float* dst, void* stream) {
    using namespace b200;
    if (!a || !g || !dst || !shape_ok(ne, anb) || !shape_ok(ne, gnb)) return B200_E_INVALID;
    const int64_t n = nelem(ne);
    if (dense_f32(a, ne, anb) && dense_f32(g, ne, gnb) && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0)
        return done(launch_pdl(swiglu_dense_kernel, dim3((unsigned)grid_for(n / 4, 256)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), reinterpret_cast<const float4*>(a),
                               reinterpret_cast<const float4*>(g), n / 4, reinterpret_cast<float4*>(dst)));
    return done(launch_pdl(swiglu_kernel, dim3((unsigned)grid_for(n, 256)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(a), shape_of(ne, anb),
                           reinterpret_cast<const char*>(g), shape_of(ne, gnb), dst));
}

int b200_rope(const float* x, const int64_t ne[4], const size_t nb[4], const int32_t* pos, int n_dims, int mode,
              float freq_base, float freq_scale, float attn_factor, float* dst, void* stream) {
    using namespace b200;
    if (!x || !pos || !dst || !shape_ok(ne, nb) || ne[0] % 2 != 0 || n_dims <= 0 || n_dims % 2 != 0 ||
        n_dims > ne[0] || !(freq_base > 0.0f))
        return B200_E_INVALID;
    if (mode != 0 && mode != 2) return B200_E_UNSUPPORTED;
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);   // the host libm's, as ggml's
    const int64_t n = (ne[0] / 2) * ne[1] * ne[2] * ne[3];
    const int64_t half = ne[0] / 2;
    const bool pow2 = half > 0 && (half & (half - 1)) == 0;
    const bool pairs8 = nb[0] == 4 && ne[0] % 2 == 0 && nb[1] % 8 == 0 && nb[2] % 8 == 0 && nb[3] % 8 == 0 &&
                        (reinterpret_cast<uintptr_t>(x) & 7u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0;
    if (mode == 0 && n_dims / 2 <= ROPE_MAX_HALF && pow2 && pairs8 && half * ne[1] <= 256 * ROPE_RT) {
        int shift = 0;
        while ((int64_t(1) << shift) < half) shift++;
        return done(launch_pdl(rope_token_pairs_kernel<false>, dim3((unsigned)std::min<int64_t>(ne[2] * ne[3], 148 * 8)),
                               dim3(256), 0, static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x),
                               shape_of(ne, nb), pos, n_dims, shift, theta_scale, freq_scale, attn_factor,
                               reinterpret_cast<char*>(dst), shape_of(ne, nb)));
    }
    if (n_dims / 2 <= ROPE_MAX_HALF)
        return done(launch_pdl(rope_token_kernel, dim3((unsigned)std::min<int64_t>(ne[2] * ne[3], 148 * 8)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), pos,
                               n_dims, mode == 2 ? 1 : 0, theta_scale, freq_scale, attn_factor, dst));
    return done(launch_pdl(rope_kernel, dim3((unsigned)grid_for(n, 256)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), pos,
                           n_dims, mode == 2 ? 1 : 0, theta_scale, freq_scale, attn_factor, dst));
}

int b200_rope_f16(const float* x, const int64_t ne[4], const size_t nb[4], const int32_t* pos, int n_dims, int mode,
                  float freq_base, float freq_scale, float attn_factor, void* dst, const size_t dnb[4], void* stream) {
    using namespace b200;
    if (!x || !pos || !dst || !shape_ok(ne, nb) || ne[0] % 2 != 0 || n_dims <= 0 || n_dims % 2 != 0 ||
        n_dims > ne[0] || !(freq_base > 0.0f))
        return B200_E_INVALID;
    const int64_t half = ne[0] / 2;
    const bool pow2 = half > 0 && (half & (half - 1)) == 0;
    const bool pairs8 = nb[0] == 4 && nb[1] % 8 == 0 && nb[2] % 8 == 0 && nb[3] % 8 == 0 &&
                        (reinterpret_cast<uintptr_t>(x) & 7u) == 0;
    const bool out4 = dnb[0] == 2 && dnb[1] % 4 == 0 && dnb[2] % 4 == 0 && dnb[3] % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(dst) & 3u) == 0;
    if (mode != 0 || n_dims / 2 > ROPE_MAX_HALF || !pow2 || !pairs8 || !out4 || half * ne[1] > 256 * ROPE_RT)
        return B200_E_UNSUPPORTED;   // the normal-mode pair kernel only
    const float theta_scale = powf(freq_base, -2.0f / (float)n_dims);   // the host libm's, as ggml's
    int shift = 0;
    while ((int64_t(1) << shift) < half) shift++;
    return done(launch_pdl(rope_token_pairs_kernel<true>, dim3((unsigned)std::min<int64_t>(ne[2] * ne[3], 148 * 8)),
                           dim3(256), 0, static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x),
                           shape_of(ne, nb), pos, n_dims, shift, theta_scale, freq_scale, attn_factor,
                           static_cast<char*>(dst), shape_of(ne, dnb)));
}

int b200_get_rows(int src_type, const void* src, const int64_t sne[4], const size_t snb[4], const int32_t* idx,
                  const int64_t ine[4], const size_t inb[4], float* dst, int* dev_err, void* stream) {
    using namespace b200;
    if (!src || !idx || !dst || !dev_err || !shape_ok(sne, snb) || !shape_ok(ine, inb) || ine[3] != 1)
        return B200_E_INVALID;
    if (src_type != 0 && src_type != 1) return B200_E_UNSUPPORTED;   // F32, F16
    if (ine[1] > sne[2] || ine[2] > sne[3]) return B200_E_INVALID;
    const int64_t n = sne[0] * ine[0] * ine[1] * ine[2];
    const int64_t rows = ine[0] * ine[1] * ine[2];
    if (rows > 0 && rows < (1ll << 31) && sne[0] >= 64) {
        // rows long enough for a CTA each: the index is read once per row
        const size_t esz = src_type == 1 ? 2 : 4;
        const bool vec = snb[0] == esz && sne[0] % 4 == 0 && snb[1] % (4 * esz) == 0 && snb[2] % (4 * esz) == 0 &&
                         snb[3] % (4 * esz) == 0 && (reinterpret_cast<uintptr_t>(src) & (4 * esz - 1)) == 0 &&
                         (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
        return done(launch_pdl(get_rows_row_kernel, dim3((unsigned)rows), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), src_type, vec ? 1 : 0, static_cast<const char*>(src),
                               shape_of(sne, snb), reinterpret_cast<const char*>(idx), shape_of(ine, inb), dst,
                               dev_err));
    }
    return done(launch_pdl(get_rows_kernel, dim3((unsigned)grid_for(n, 256)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), src_type, static_cast<const char*>(src),
                           shape_of(sne, snb), reinterpret_cast<const char*>(idx), shape_of(ine, inb), dst, dev_err));
}

int b200_cpy(int src_type, const void* src, const int64_t sne[4], const size_t snb[4], int dst_type, void* dst,
             const int64_t dne[4], const size_t dnb[4], void* stream) {
    using namespace b200;
    if (!src || !dst || !shape_ok(sne, snb) || !shape_ok(dne, dnb)) return B200_E_INVALID;
    if ((src_type != 0 && src_type != 1) || (dst_type != 0 && dst_type != 1)) return B200_E_UNSUPPORTED;
    const bool same = sne[0] == dne[0] && sne[1] == dne[1] && sne[2] == dne[2] && sne[3] == dne[3];
    if (!same) {
        const size_t es = dst_type ? 2 : 4;
        const bool contiguous = dnb[0] == es && dnb[1] == dnb[0] * (size_t)dne[0] &&
                                dnb[2] == dnb[1] * (size_t)dne[1] && dnb[3] == dnb[2] * (size_t)dne[2];
        if (!contiguous || nelem(sne) != nelem(dne)) return B200_E_INVALID;
    }
    const int64_t n = nelem(sne);
    if (src_type == 0 && dst_type == 1 && dense_f32(src, sne, snb) && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
        // the destination dense f16 with src's element order (same shape and contiguous, or contiguous)
        bool d_dense = true;
        size_t next = 2;
        for (int i = 0; i < 4; i++) {
            if (dne[i] != 1 && dnb[i] != next) d_dense = false;
            next *= (size_t)dne[i];
        }
        if (d_dense)
            return done(launch_pdl(cpy_f32_f16_dense_kernel, dim3((unsigned)grid_for(n / 4, 256)), dim3(256), 0,
                                   static_cast<cudaStream_t>(stream), static_cast<const float4*>(src), n / 4,
                                   static_cast<uint2*>(dst)));
    }
    return done(launch_pdl(cpy_kernel, dim3((unsigned)grid_for(n, 256)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), src_type, static_cast<const char*>(src),
                           shape_of(sne, snb), dst_type, static_cast<char*>(dst), shape_of(dne, dnb), same ? 1 : 0));
}

int b200_soft_max(const float* x, const int64_t ne[4], const size_t nb[4], float scale, float* dst, void* stream) {
    using namespace b200;
    if (!x || !dst || !shape_ok(ne, nb)) return B200_E_INVALID;
    const int64_t rows = ne[1] * ne[2] * ne[3];
    if (ne[0] <= 32 * SMW_MAX && rows < (1ll << 34)) {
        const dim3 grid((unsigned)((rows + 7) / 8)), block(256);
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        const char* xp = reinterpret_cast<const char*>(x);
        const Shape4 sh = shape_of(ne, nb);
        const int64_t e = (ne[0] + 31) / 32;
        if (e <= 1) return done(launch_pdl(soft_max_warp_kernel<1>, grid, block, 0, st, xp, sh, scale, dst));
        if (e <= 2) return done(launch_pdl(soft_max_warp_kernel<2>, grid, block, 0, st, xp, sh, scale, dst));
        if (e <= 4) return done(launch_pdl(soft_max_warp_kernel<4>, grid, block, 0, st, xp, sh, scale, dst));
        if (e <= 8) return done(launch_pdl(soft_max_warp_kernel<8>, grid, block, 0, st, xp, sh, scale, dst));
        if (e <= 16) return done(launch_pdl(soft_max_warp_kernel<16>, grid, block, 0, st, xp, sh, scale, dst));
        return done(launch_pdl(soft_max_warp_kernel<32>, grid, block, 0, st, xp, sh, scale, dst));
    }
    return done(launch_pdl(soft_max_kernel, dim3((unsigned)std::min<int64_t>(rows, 148 * 8)), dim3(SM_THREADS), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), scale,
                           dst));
}

int b200_argsort(const float* x, const int64_t ne[4], const size_t nb[4], int descending, int32_t* dst, void* stream) {
    using namespace b200;
    if (!x || !dst || !shape_ok(ne, nb)) return B200_E_INVALID;
    if (ne[0] > AS_MAX) return B200_E_UNSUPPORTED;
    int n2 = 2;
    while (n2 < ne[0]) n2 <<= 1;
    const int64_t rows = ne[1] * ne[2] * ne[3];
    if (n2 <= ASW_MAX && rows < (1ll << 34)) {
        const dim3 grid((unsigned)((rows + 7) / 8)), block(256);
        const cudaStream_t st = static_cast<cudaStream_t>(stream);
        const char* xp = reinterpret_cast<const char*>(x);
        const Shape4 sh = shape_of(ne, nb);
        const int d = descending ? 1 : 0;
        if (n2 <= 32) return done(launch_pdl(argsort_warp_kernel<1>, grid, block, 0, st, xp, sh, d, dst));
        if (n2 <= 64) return done(launch_pdl(argsort_warp_kernel<2>, grid, block, 0, st, xp, sh, d, dst));
        if (n2 <= 128) return done(launch_pdl(argsort_warp_kernel<4>, grid, block, 0, st, xp, sh, d, dst));
        return done(launch_pdl(argsort_warp_kernel<8>, grid, block, 0, st, xp, sh, d, dst));
    }
    const int threads = std::max(32, std::min(AS_MAX / 2, n2 / 2));
    return done(launch_pdl(argsort_kernel, dim3((unsigned)std::min<int64_t>(rows, 148 * 8)), dim3(threads), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb),
                           descending ? 1 : 0, n2, dst));
}

int b200_hadamard(const float* x, const int64_t ne[4], const size_t nb[4], float scale, float* dst, void* stream) {
    using namespace b200;
    if (!x || !dst || !shape_ok(ne, nb)) return B200_E_INVALID;
    const int64_t n = ne[0];
    if (n < 32 || n > HAD_MAX || (n & (n - 1)) != 0) return B200_E_UNSUPPORTED;
    const int64_t rows = ne[1] * ne[2] * ne[3];
    if (rows >= (1ll << 34)) return B200_E_UNSUPPORTED;
    const dim3 grid((unsigned)((rows + 7) / 8)), block(256);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const char* xp = reinterpret_cast<const char*>(x);
    const Shape4 sh = shape_of(ne, nb);
    switch (n) {
        case 32: return done(launch_pdl(hadamard_kernel<1>, grid, block, 0, st, xp, sh, scale, dst));
        case 64: return done(launch_pdl(hadamard_kernel<2>, grid, block, 0, st, xp, sh, scale, dst));
        case 128: return done(launch_pdl(hadamard_kernel<4>, grid, block, 0, st, xp, sh, scale, dst));
        case 256: return done(launch_pdl(hadamard_kernel<8>, grid, block, 0, st, xp, sh, scale, dst));
        case 512: return done(launch_pdl(hadamard_kernel<16>, grid, block, 0, st, xp, sh, scale, dst));
        default: return done(launch_pdl(hadamard_kernel<32>, grid, block, 0, st, xp, sh, scale, dst));
    }
}

int b200_sum_rows(const float* x, const int64_t ne[4], const size_t nb[4], float* dst, void* stream) {
    using namespace b200;
    if (!x || !dst || !shape_ok(ne, nb)) return B200_E_INVALID;
    const int64_t rows = ne[1] * ne[2] * ne[3];
    return done(launch_pdl(sum_rows_kernel, dim3((unsigned)std::min<int64_t>(rows, 148 * 8)), dim3(RMS_THREADS), 0,
                           static_cast<cudaStream_t>(stream), reinterpret_cast<const char*>(x), shape_of(ne, nb), dst));
}

}  // extern "C"
