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
 * b200_mul_mat_workspace_size(M, N, K) bytes.
 */
size_t b200_mul_mat_workspace_size(int64_t M, int64_t N, int64_t K);
int    b200_mul_mat(int wtype, const void * w_packed, int64_t N, int64_t K,
                    const float * src1, int64_t lda, int64_t M,
                    float * dst, int64_t ldd,
                    void * workspace, size_t workspace_bytes, int * dev_err, void * stream);

#ifdef __cplusplus
}
#endif

#endif /* GGML_B200_KERNELS_H */
