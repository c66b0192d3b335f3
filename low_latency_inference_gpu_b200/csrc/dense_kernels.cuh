// Declarations shared by the launch-per-layer kernels and the chained-MLP paths.
#pragma once
#include <cuda_runtime.h>

#include "ll_b200.h"

namespace llk {

__device__ __forceinline__ float dense_act(float v, int act)
{
    if (act == LL_ACT_RELU)
        return v > 0.0f ? v : 0.0f;
    if (act == LL_ACT_GELU)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
    return v;
}

void launch_dense_warp_rm(const float *W, const float *b, const float *x, float *y, int M, int K, int act,
                          cudaStream_t s);

}  // namespace llk
