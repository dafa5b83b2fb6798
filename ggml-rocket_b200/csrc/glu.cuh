// The gated-linear-unit arithmetic shared by the glue kernels (SILU, SWIGLU) and the owner-side
// expert FFN of the expert-parallel path, so that both round every value the same way.
#pragma once

#include <cuda_runtime.h>

namespace b200 {

// ggml_silu_f32: x / (1 + expf(-x)), expf being the device's (within 2 ulp of the host libm's)
__device__ __forceinline__ float silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }
__device__ __forceinline__ float silu_f(float x) { return silu(x); }
// SWIGLU (ggml_swiglu_split): silu(gate) * up
__device__ __forceinline__ float swiglu_f(float gate, float up) { return __fmul_rn(silu(gate), up); }

}  // namespace b200
