// Header-only launch-per-layer kernels with the reference's template names
// (include/ll/dense_warp.cuh:9-90 and include/ll/dense_mbyv_packed.cuh:15-63),
// re-implemented for sm_100a: 128-bit weight loads with four independent
// accumulators per lane, x staged in shared memory, butterfly shuffles, and no
// shuffle after an early exit (the whole warp leaves together).
//
// Same launch contract as the reference: dense_warp_rm_kernel<M, K, BLOCK_WARPS, Act>
// with grid ceil(M / BLOCK_WARPS), block BLOCK_WARPS * 32, dynamic shared memory
// K * sizeof(float).  W row-major [M x K].
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace ll {

struct ActIdentity {
    __device__ __forceinline__ float operator()(float x) const { return x; }
};

struct ActRelu {
    __device__ __forceinline__ float operator()(float x) const { return x > 0.0f ? x : 0.0f; }
};

// New: exact GELU, 0.5 x (1 + erf(x / sqrt 2)).
struct ActGelu {
    __device__ __forceinline__ float operator()(float x) const
    {
        return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
    }
};

template <int M, int K, int BLOCK_WARPS, class Act>
__global__ void __launch_bounds__(BLOCK_WARPS * 32) dense_warp_rm_kernel(const float *__restrict__ W_rm,
                                                                          const float *__restrict__ b,
                                                                          const float *__restrict__ x,
                                                                          float *__restrict__ y, Act act)
{
    static_assert(BLOCK_WARPS >= 1, "BLOCK_WARPS must be >= 1");
    extern __shared__ float4 ll_sx4[];
    float *sx = reinterpret_cast<float *>(ll_sx4);
    for (int i = threadIdx.x; i < K; i += BLOCK_WARPS * 32)
        sx[i] = x[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * BLOCK_WARPS + (threadIdx.x >> 5);
    if (row >= M)
        return;
    const float *wr = W_rm + (size_t)row * K;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    if constexpr (K % 4 == 0) {
        const float4 *w4 = reinterpret_cast<const float4 *>(wr);
        const float4 *x4 = reinterpret_cast<const float4 *>(sx);
#pragma unroll 4
        for (int j = lane; j < K / 4; j += 32) {
            const float4 w = __ldg(w4 + j);
            const float4 v = x4[j];
            a0 = fmaf(w.x, v.x, a0);
            a1 = fmaf(w.y, v.y, a1);
            a2 = fmaf(w.z, v.z, a2);
            a3 = fmaf(w.w, v.w, a3);
        }
    } else {
        for (int j = lane; j < K; j += 32)
            a0 = fmaf(__ldg(wr + j), sx[j], a0);
    }
    float acc = (a0 + a1) + (a2 + a3);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
        acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0)
        y[row] = act(acc + b[row]);
}

// Thread per output row over K-major padded weights W_cm[k * Mpad + row].
template <int M, int K, int Mpad, class Act>
__global__ void dense_mbyv_packed_kernel(const float *__restrict__ W_cm, const float *__restrict__ b_pad,
                                         const float *__restrict__ x, float *__restrict__ y, Act act)
{
    __shared__ float sx[K];
    for (int i = threadIdx.x; i < K; i += blockDim.x)
        sx[i] = x[i];
    __syncthreads();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= M)
        return;
    float acc = b_pad[row];
#pragma unroll 8
    for (int k = 0; k < K; ++k)
        acc = fmaf(__ldg(W_cm + (size_t)k * Mpad + row), sx[k], acc);
    y[row] = act(acc);
}

// Same signature as the reference's launcher (include/ll/dense_mbyv_packed.cuh:53-63);
// spreads the rows over 128-thread blocks instead of one block of Mpad threads.
template <int M, int K, class Act>
inline void launch_dense_mbyv_packed(cudaStream_t stream, const float *W_cm, const float *b_pad, const float *x,
                                     float *y, Act act)
{
    constexpr int Mpad = (M + 31) / 32 * 32;
    constexpr int threads = 128;
    dense_mbyv_packed_kernel<M, K, Mpad, Act><<<(Mpad + threads - 1) / threads, threads, 0, stream>>>(W_cm, b_pad, x,
                                                                                                       y, act);
}

}  // namespace ll
