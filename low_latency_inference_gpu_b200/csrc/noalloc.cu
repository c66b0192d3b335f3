// Launch-per-layer MLP forward that allocates nothing.
//
// Who needs it: callers that must not enter the CUDA allocator on their request
// path -- a cudaMalloc can implicitly synchronise the device and take
// milliseconds, which a microsecond-budget serving loop cannot absorb -- and
// callers whose device memory is entirely owned by another allocator (a
// framework's pool, a fixed budget reserved at start-up).  They pass weights,
// input and output; the activations between layers live in one statically
// sized device array that belongs to this library.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds it (2 x LL_NOALLOC_MAX_WIDTH floats, 64 KB) until the process
// exits.  Host code cannot use its name as a device address, so its address is
// looked up once per device with cudaGetSymbolAddress and cached.
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"
#include "dense_kernels.cuh"

namespace {

// Ping-pong buffers for the hidden activations of one batch-1 request.
static __device__ __align__(256) float g_noalloc_act[2 * LL_NOALLOC_MAX_WIDTH];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float *g_act_ptr[kMaxDevices] = {};

// Device address of g_noalloc_act on the current device; looked up on the first call per device.
int scratch_on_current_device(float **out)
{
    int dev = 0;
    LL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        llh::set_error("ll_mlp_forward_noalloc: device index %d out of range", dev);
        return LL_ERR_INVALID_ARG;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_act_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_act);
        if (e != cudaSuccess || !p) {
            llh::set_error("ll_mlp_forward_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                           cudaGetErrorString(e));
            return LL_ERR_CUDA;
        }
        g_act_ptr[dev] = static_cast<float *>(p);
    }
    *out = g_act_ptr[dev];
    return LL_OK;
}

}  // namespace

extern "C" int ll_mlp_forward_noalloc(const ll_net_desc *net, const float *const *d_W, const float *const *d_b,
                                      const float *d_x, float *d_y, void *stream)
{
    if (!net || !net->layers || net->n_layers < 1 || net->n_layers > 64 || !d_W || !d_x || !d_y) {
        llh::set_error("ll_mlp_forward_noalloc: null or empty arguments");
        return LL_ERR_INVALID_ARG;
    }
    if (net->max_batch != 1) {
        llh::set_error("ll_mlp_forward_noalloc: batch-1 only (max_batch = %d)", net->max_batch);
        return LL_ERR_INVALID_ARG;
    }
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        if (d.wtype != LL_W_F32 || d.in_dim < 1 || d.out_dim < 1 || d.in_dim > 12288 || !d_W[l] ||
            (l > 0 && net->layers[l - 1].out_dim != d.in_dim)) {
            llh::set_error("ll_mlp_forward_noalloc: layer %d must be fp32 with consistent dims (in <= 12288)", l);
            return LL_ERR_INVALID_ARG;
        }
        if (l + 1 < net->n_layers && d.out_dim > LL_NOALLOC_MAX_WIDTH) {
            llh::set_error("ll_mlp_forward_noalloc: hidden width %d of layer %d exceeds the static scratch "
                           "limit LL_NOALLOC_MAX_WIDTH = %d",
                           d.out_dim, l, LL_NOALLOC_MAX_WIDTH);
            return LL_ERR_INVALID_ARG;
        }
    }
    float *act = nullptr;
    int rc = scratch_on_current_device(&act);
    if (rc)
        return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const float *in = d_x;
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        float *out = (l + 1 == net->n_layers) ? d_y : act + (size_t)(l & 1) * LL_NOALLOC_MAX_WIDTH;
        llk::launch_dense_warp_rm(d_W[l], d_b ? d_b[l] : nullptr, in, out, d.out_dim, d.in_dim, d.act, s);
        in = out;
    }
    LL_CUDA_TRY(cudaGetLastError());
    return LL_OK;
}
