// Launch-per-layer GEMV kernels for sm_100a.
//
// ll_dense_warp_rm replaces ll::dense_warp_rm_kernel (include/ll/dense_warp.cuh:33-90):
// one warp per output row, x staged in shared memory, 128-bit weight loads
// (4 independent accumulators) instead of the reference's strided scalar loop,
// butterfly shuffle reduction, fused bias + activation.
//
// ll_dense_mbyv_packed replaces ll::dense_mbyv_packed_kernel / launch_dense_mbyv_packed
// (include/ll/dense_mbyv_packed.cuh:15-63): one thread per output row over the
// K-major padded layout W_cm[k*Mpad + row].  x comes from shared memory, so
// there is no shuffle after the early exit (the reference returns for
// row >= M and then calls __shfl_sync with a full mask, :20-21 and :43).
#include <cuda_runtime.h>

#include "common.h"
#include "dense_kernels.cuh"

namespace llk {

__global__ void __launch_bounds__(256) dense_warp_rm_kernel_rt(const float *__restrict__ W, const float *__restrict__ b,
                                                               const float *__restrict__ x, float *__restrict__ y,
                                                               int M, int K, int act)
{
    extern __shared__ float4 sx4[];
    float *sx = reinterpret_cast<float *>(sx4);
    for (int i = threadIdx.x; i < K; i += blockDim.x)
        sx[i] = x[i];
    __syncthreads();
    const int warps = blockDim.x >> 5;
    const int row = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M)
        return;  // whole warp leaves together: no shuffle is left half-populated
    const float *wr = W + (size_t)row * K;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    const bool vec = ((K & 3) == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
    if (vec) {
        const int K4 = K >> 2;
        const float4 *w4 = reinterpret_cast<const float4 *>(wr);
        const float4 *x4 = reinterpret_cast<const float4 *>(sx);
        for (int j = lane; j < K4; j += 32) {
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
        y[row] = dense_act(acc + (b ? b[row] : 0.0f), act);
}

__global__ void __launch_bounds__(128) dense_mbyv_packed_kernel_rt(const float *__restrict__ W_cm,
                                                                   const float *__restrict__ b_pad,
                                                                   const float *__restrict__ x, float *__restrict__ y,
                                                                   int M, int K, int Mpad, int act)
{
    extern __shared__ float4 sx4[];
    float *sx = reinterpret_cast<float *>(sx4);
    for (int i = threadIdx.x; i < K; i += blockDim.x)
        sx[i] = x[i];
    __syncthreads();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= M)
        return;
    float acc = b_pad ? b_pad[row] : 0.0f;
    for (int k = 0; k < K; ++k)
        acc = fmaf(__ldg(W_cm + (size_t)k * Mpad + row), sx[k], acc);
    y[row] = dense_act(acc, act);
}

}  // namespace llk

extern "C" {

int ll_dense_warp_rm(const float *W, const float *b, const float *x, float *y, int M, int K, int act, void *stream)
{
    if (!W || !x || !y || M < 1 || K < 1 || K > 12288) {
        llh::set_error("ll_dense_warp_rm: invalid arguments (M=%d K=%d)", M, K);
        return LL_ERR_INVALID_ARG;
    }
    llk::launch_dense_warp_rm(W, b, x, y, M, K, act, static_cast<cudaStream_t>(stream));
    LL_CUDA_TRY(cudaGetLastError());
    return LL_OK;
}

int ll_dense_mbyv_packed(const float *W_cm, const float *b_pad, const float *x, float *y, int M, int K, int act,
                         void *stream)
{
    if (!W_cm || !x || !y || M < 1 || K < 1 || K > 12288) {
        llh::set_error("ll_dense_mbyv_packed: invalid arguments (M=%d K=%d)", M, K);
        return LL_ERR_INVALID_ARG;
    }
    const int Mpad = (M + 31) / 32 * 32;
    const int threads = 128;
    const int blocks = (Mpad + threads - 1) / threads;
    llk::dense_mbyv_packed_kernel_rt<<<blocks, threads, sizeof(float) * (size_t)K, static_cast<cudaStream_t>(stream)>>>(
        W_cm, b_pad, x, y, M, K, Mpad, act);
    LL_CUDA_TRY(cudaGetLastError());
    return LL_OK;
}

}  // extern "C"

namespace llk {

void launch_dense_warp_rm(const float *W, const float *b, const float *x, float *y, int M, int K, int act,
                          cudaStream_t s)
{
    // 8 warps per block for tall layers, fewer for short ones so more SMs take part
    const int warps = M >= 256 ? 8 : (M >= 64 ? 4 : 1);
    const int blocks = (M + warps - 1) / warps;
    dense_warp_rm_kernel_rt<<<blocks, warps * 32, sizeof(float) * (size_t)((K + 3) / 4 * 4), s>>>(W, b, x, y, M, K,
                                                                                                 act);
}

}  // namespace llk
