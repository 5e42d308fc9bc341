// Gate and activation functions of the DGDA feature path and the SwiGLU FFN
// (maba_sparse/layers/dgda.py:190-197, model.py:37): SiLU, sigmoid and
// max(-softplus(x), -14), in float32 on the SFU exponent / logarithm / divide
// intrinsics (a few ulp; the features are stored in 16 bits or compared at 1e-5).
#pragma once
#include <cuda_runtime.h>

namespace maba {

__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
// softplus(x) = x above 20 (torch's threshold), log(1 + e^x) below
__device__ __forceinline__ float neg_softplus_clamped(float x) {
    const float sp = x > 20.f ? x : __logf(1.f + __expf(x));
    return fmaxf(-sp, -14.f);
}

}  // namespace maba
