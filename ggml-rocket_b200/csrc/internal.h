// Declarations shared between the backend's translation units (not part of the C ABI).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <utility>

namespace b200 {

// Launch with programmatic stream serialization: the kernel may be scheduled while the previous
// kernel of the stream drains (its prologue overlaps that tail; it waits with grid_dep_wait()).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int device_sm_count();
// The give-up limit of waits on another GPU's flags (b200_set_peer_wait_limit_ns), nanoseconds.
uint64_t peer_wait_limit_ns();
bool make_tmap_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                      uint32_t box_rows, uint32_t box_cols);
// A 2-D uint16 tensor map [rows, cols] (cols innermost, row pitch in bytes), box [box_rows,
// box_cols], no swizzle; rows past the end read as zero.
bool make_tmap_2d_u16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_bytes,
                      uint32_t box_rows, uint32_t box_cols);
size_t packed_weight_bytes(int type, int64_t N, int64_t K, size_t* plane_d_off);
// The raw-tile tensor maps of a packed Q4_K / Q6_K / Q8_0 weight of `wrows` rows: boxes of 128
// rows x one 256-weight super-block column (tmW, uint16 elements) and, for Q6_K, the transposed
// d plane's 128-row box (tmD; unused otherwise).
bool make_weight_tile_maps(int wtype, const void* w_packed, int64_t wrows, int64_t K, CUtensorMap* tmW,
                           CUtensorMap* tmD);
// Decode-size MUL_MAT on the tiled weight-streaming kernel (gemv_tiles.cu): Q4_K / Q6_K / Q8_0,
// M <= 32. Same arguments and return codes as b200_mul_mat_vec.
size_t mul_mat_vec_tiles_workspace(int64_t M, int64_t N, int64_t K);
int mul_mat_vec_tiles(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda,
                      int64_t M, float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err,
                      cudaStream_t st);
bool weight_type_supported(int type, int64_t K);
// dst_bases / n_dst / col0: the output columns [col0, col0 + N) of every one of n_dst [M][ldd]
// buffers (a device array of pointers, other GPUs' included) instead of dst
int mul_mat_impl(int wtype, const void* w_packed, int64_t N, int64_t K, const float* src1, int64_t lda, int64_t M,
                 float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err, cudaStream_t st,
                 float* const* dst_bases = nullptr, int n_dst = 0, int64_t col0 = 0);
int gemm_packed_impl(int wtype, const void* w_packed, int64_t N, int64_t K, const __half* a16, const float* scales,
                     int64_t M, float* dst, int64_t ldd, void* workspace, size_t workspace_bytes, int* dev_err,
                     cudaStream_t st, float* const* dst_bases = nullptr, int n_dst = 0, int64_t col0 = 0);
size_t mul_mat_workspace(int wtype, int64_t M, int64_t N, int64_t K);
// Where, inside mul_mat_impl's workspace, the stream-K flags of that op live (byte offset and
// length; length 0 when the plan shares no output tile between CTAs).
void mul_mat_flags_range(int wtype, int64_t M, int64_t N, int64_t K, size_t* offset, size_t* bytes);
int act_pack_impl(const float* src1, int64_t lda, int64_t M, int64_t K, __half* a16, float* scales, cudaStream_t st);
int gemm_grouped_impl(int wtype, const void* w_stack, int64_t N, int64_t K, int64_t n_expert, const __half* a16,
                      const float* scales, int64_t rows, int bt, const int32_t* off, const int32_t* tile_start,
                      const int32_t* slot, const int32_t* tok, float* dst, int64_t d_nb1, int64_t d_nb2, int* dev_err,
                      cudaStream_t st, const int32_t* src = nullptr, float* const* dst_bases = nullptr);
// Gather b[:, slot[r] % ne11, tok[r]] for r < *n_rows (device count; max_rows bounds the grid)
// and pack each row to fp16 with its per-row scale (moe.cu).
// self (optional): self[r] = r for every row, the token / slot index of an output in row order.
int launch_gather_pack(const float* b, int64_t b_nb1, int64_t b_nb2, int64_t ne11, int64_t K, const int32_t* slot,
                       const int32_t* tok, const int32_t* n_rows, int64_t max_rows, __half* a16, float* scales,
                       cudaStream_t st, int32_t* self = nullptr);
// The expert FFN between its projections: h16[r] / hscale[r] = the packed row swiglu(gate[r],
// up[r]) for r < *n_rows (f32 rows of F; max_rows bounds the grid), moe.cu.
int launch_swiglu_pack(const float* gate, const float* up, int64_t F, const int32_t* n_rows, int64_t max_rows,
                       __half* h16, float* hscale, cudaStream_t st);

// expert parallelism helpers shared by the NCCL and peer-memory paths (moe_ep.cu)
int ep_token_tile_public(int64_t pairs, int64_t e_loc);
void ep_route_scan_public(const int32_t* ecnt, int32_t* bsum, int32_t* bad, int nb, int e_loc, int bt, int32_t* off,
                          int32_t* tile_start, int32_t* cursor, int* err, cudaStream_t st);

}  // namespace b200
