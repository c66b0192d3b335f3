// Launch-per-inference comparison paths, kept as measured baselines:
//   ll_layered_mlp : one ll_dense_warp_rm launch per layer (the reference's
//                    fastest kernel path, src/bench_custom_warp_mlp_graph.cu:96-152);
//   ll_cublas_mlp  : cublasSgemm(OP_T, OP_N, M, 1, K) + bias/activation kernel per
//                    layer (src/bench_cublas_mlp_graph.cu:119-137).
// Both run direct or captured in a CUDA graph, kernel-only (CUDA events around
// each inference, include/bench_utils.h:93-128) or end to end (pinned H2D +
// kernels + D2H, host clock; src/bench_custom_warp_e2e.cu:165-194), and in the
// mailbox-per-tick structure of src/bench_persistent_cublas_mlp.cu:226-271
// (stage x from the mapped mailbox, layers, write y back, publish seq_out,
// stream synchronize, host spin on seq_out).
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <vector>

#include "common.h"
#include "dense_kernels.cuh"
#include "ptx.cuh"

namespace llk {

__global__ void bias_act_kernel(float *__restrict__ y, const float *__restrict__ b, int n, int act)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        y[i] = dense_act(y[i] + b[i], act);
}

__global__ void stage_x_from_mapped(float *__restrict__ d_x, const float *__restrict__ mb_x, int n)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        d_x[i] = ld_relaxed_sys_f32(mb_x + i);
}

__global__ void write_y_to_mapped(float *__restrict__ mb_y, const float *__restrict__ d_y, int n)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        st_relaxed_sys_f32(mb_y + i, d_y[i]);
}

__global__ void publish_seq_out(ll_tick_header *mb, uint32_t s)
{
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys_u32(&mb->seq_out, s);
    }
}

}  // namespace llk

namespace {

struct Chain {
    int device = 0;
    cudaStream_t stream = nullptr;
    int n = 0;
    std::vector<int> dims, acts;
    std::vector<float *> dW, db, dact;  // dact[0] = x, dact[n] = y
    float *h_x = nullptr, *h_y = nullptr;  // pinned
    void *mb_host = nullptr;
    ll_tick_header *mb_dev = nullptr;
    uint32_t seq = 0;
    cudaGraphExec_t g_kernel = nullptr, g_e2e = nullptr;
    virtual ~Chain() = default;
    virtual int enqueue_layers(cudaStream_t s) = 0;

    int setup(const ll_net_desc *net, const float *const *W, const float *const *b, int dev)
    {
        device = dev;
        LL_CUDA_TRY(cudaSetDevice(dev));
        n = net->n_layers;
        dims.resize(n + 1);
        acts.resize(n);
        dims[0] = net->layers[0].in_dim;
        for (int l = 0; l < n; ++l) {
            dims[l + 1] = net->layers[l].out_dim;
            acts[l] = net->layers[l].act;
        }
        LL_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        dW.assign(n, nullptr);
        db.assign(n, nullptr);
        dact.assign(n + 1, nullptr);
        for (int l = 0; l < n; ++l) {
            const size_t wn = (size_t)dims[l] * dims[l + 1];
            LL_CUDA_TRY(cudaMalloc(&dW[l], wn * 4));
            LL_CUDA_TRY(cudaMemcpy(dW[l], W[l], wn * 4, cudaMemcpyHostToDevice));
            LL_CUDA_TRY(cudaMalloc(&db[l], (size_t)dims[l + 1] * 4));
            if (b && b[l])
                LL_CUDA_TRY(cudaMemcpy(db[l], b[l], (size_t)dims[l + 1] * 4, cudaMemcpyHostToDevice));
            else
                LL_CUDA_TRY(cudaMemset(db[l], 0, (size_t)dims[l + 1] * 4));
        }
        for (int l = 0; l <= n; ++l) {
            LL_CUDA_TRY(cudaMalloc(&dact[l], (size_t)llh::round_up((size_t)dims[l], 4) * 4));
            LL_CUDA_TRY(cudaMemset(dact[l], 0, (size_t)llh::round_up((size_t)dims[l], 4) * 4));
        }
        LL_CUDA_TRY(cudaHostAlloc((void **)&h_x, (size_t)dims[0] * 4, cudaHostAllocDefault));
        LL_CUDA_TRY(cudaHostAlloc((void **)&h_y, (size_t)dims[n] * 4, cudaHostAllocDefault));
        const size_t mbb = ll_mailbox_bytes(dims[0], dims[n], 1);
        LL_CUDA_TRY(cudaHostAlloc(&mb_host, mbb, cudaHostAllocMapped | cudaHostAllocPortable));
        std::memset(mb_host, 0, mbb);
        LL_CUDA_TRY(cudaHostGetDevicePointer((void **)&mb_dev, mb_host, 0));
        return LL_OK;
    }

    void release()
    {
        cudaSetDevice(device);
        if (g_kernel)
            cudaGraphExecDestroy(g_kernel);
        if (g_e2e)
            cudaGraphExecDestroy(g_e2e);
        for (auto p : dW)
            if (p)
                cudaFree(p);
        for (auto p : db)
            if (p)
                cudaFree(p);
        for (auto p : dact)
            if (p)
                cudaFree(p);
        if (h_x)
            cudaFreeHost(h_x);
        if (h_y)
            cudaFreeHost(h_y);
        if (mb_host)
            cudaFreeHost(mb_host);
        if (stream)
            cudaStreamDestroy(stream);
    }

    int enqueue_e2e(cudaStream_t s)
    {
        LL_CUDA_TRY(cudaMemcpyAsync(dact[0], h_x, (size_t)dims[0] * 4, cudaMemcpyHostToDevice, s));
        int rc = enqueue_layers(s);
        if (rc)
            return rc;
        LL_CUDA_TRY(cudaMemcpyAsync(h_y, dact[n], (size_t)dims[n] * 4, cudaMemcpyDeviceToHost, s));
        return LL_OK;
    }

    int enqueue_tick(cudaStream_t s, uint32_t sq)
    {
        const float *mbx = reinterpret_cast<const float *>(reinterpret_cast<const char *>(mb_dev) + 16);
        float *mby = reinterpret_cast<float *>(reinterpret_cast<char *>(mb_dev) + 16 + 4 * (size_t)dims[0]);
        llk::stage_x_from_mapped<<<(dims[0] + 255) / 256, 256, 0, s>>>(dact[0], mbx, dims[0]);
        int rc = enqueue_layers(s);
        if (rc)
            return rc;
        llk::write_y_to_mapped<<<(dims[n] + 255) / 256, 256, 0, s>>>(mby, dact[n], dims[n]);
        llk::publish_seq_out<<<1, 32, 0, s>>>(mb_dev, sq);
        LL_CUDA_TRY(cudaGetLastError());
        return LL_OK;
    }

    int capture(bool e2e, cudaGraphExec_t *out)
    {
        if (*out)
            return LL_OK;
        cudaGraph_t g = nullptr;
        LL_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        int rc = e2e ? enqueue_e2e(stream) : enqueue_layers(stream);
        cudaError_t ce = cudaStreamEndCapture(stream, &g);
        if (rc)
            return rc;
        if (ce != cudaSuccess) {
            llh::set_error("graph capture failed: %s", cudaGetErrorString(ce));
            return LL_ERR_CUDA;
        }
        ce = cudaGraphInstantiate(out, g, 0);
        cudaGraphDestroy(g);
        if (ce != cudaSuccess) {
            llh::set_error("graph instantiate failed: %s", cudaGetErrorString(ce));
            return LL_ERR_CUDA;
        }
        return LL_OK;
    }

    int bench(int mode, const float *xs, int n_x, int n_req, float *y_last, double *lat_us)
    {
        LL_CUDA_TRY(cudaSetDevice(device));
        const size_t in = (size_t)dims[0], out = (size_t)dims[n];
        int rc = LL_OK;
        if (mode == LL_RUN_GRAPH_KERNEL)
            rc = capture(false, &g_kernel);
        else if (mode == LL_RUN_GRAPH_E2E)
            rc = capture(true, &g_e2e);
        if (rc)
            return rc;
        cudaEvent_t ea, eb;
        LL_CUDA_TRY(cudaEventCreate(&ea));
        LL_CUDA_TRY(cudaEventCreate(&eb));
        for (int r = 0; r < n_req && rc == LL_OK; ++r) {
            const float *x = xs + (size_t)(r % n_x) * in;
            if (mode == LL_RUN_DIRECT_KERNEL || mode == LL_RUN_GRAPH_KERNEL) {
                // inputs resident on the device: the copy is outside the timed span
                cudaMemcpyAsync(dact[0], x, in * 4, cudaMemcpyHostToDevice, stream);
                cudaEventRecord(ea, stream);
                if (mode == LL_RUN_DIRECT_KERNEL)
                    rc = enqueue_layers(stream);
                else if (cudaGraphLaunch(g_kernel, stream) != cudaSuccess)
                    rc = LL_ERR_CUDA;
                cudaEventRecord(eb, stream);
                if (cudaEventSynchronize(eb) != cudaSuccess) {
                    rc = LL_ERR_CUDA;
                    break;
                }
                float ms = 0;
                cudaEventElapsedTime(&ms, ea, eb);
                if (lat_us)
                    lat_us[r] = ms * 1000.0;
                if (y_last && r == n_req - 1)
                    cudaMemcpy(y_last, dact[n], out * 4, cudaMemcpyDeviceToHost);
            } else if (mode == LL_RUN_GRAPH_E2E || mode == LL_RUN_DIRECT_E2E) {
                const auto t0 = std::chrono::steady_clock::now();
                std::memcpy(h_x, x, in * 4);
                if (mode == LL_RUN_GRAPH_E2E) {
                    if (cudaGraphLaunch(g_e2e, stream) != cudaSuccess)
                        rc = LL_ERR_CUDA;
                } else {
                    rc = enqueue_e2e(stream);
                }
                if (cudaStreamSynchronize(stream) != cudaSuccess)
                    rc = LL_ERR_CUDA;
                if (y_last && r == n_req - 1)
                    std::memcpy(y_last, h_y, out * 4);
                const auto t1 = std::chrono::steady_clock::now();
                if (lat_us)
                    lat_us[r] = std::chrono::duration<double, std::micro>(t1 - t0).count();
            } else if (mode == LL_RUN_MAILBOX_TICK) {
                const auto t0 = std::chrono::steady_clock::now();
                seq = ll_next_seq(seq);
                ll_mailbox_post(mb_host, dims[0], x, 1, seq, 0);
                rc = enqueue_tick(stream, seq);
                if (cudaStreamSynchronize(stream) != cudaSuccess)
                    rc = LL_ERR_CUDA;
                if (rc == LL_OK)
                    rc = ll_mailbox_wait(mb_host, dims[0], dims[n], 1, seq, (y_last && r == n_req - 1) ? y_last : nullptr,
                                         1, 1000ull * 1000 * 1000);
                const auto t1 = std::chrono::steady_clock::now();
                if (lat_us)
                    lat_us[r] = std::chrono::duration<double, std::micro>(t1 - t0).count();
            } else {
                llh::set_error("unknown run mode %d", mode);
                rc = LL_ERR_INVALID_ARG;
            }
        }
        cudaEventDestroy(ea);
        cudaEventDestroy(eb);
        if (rc == LL_OK) {
            cudaError_t ce = cudaGetLastError();
            if (ce != cudaSuccess) {
                llh::set_error("CUDA error during bench: %s", cudaGetErrorString(ce));
                rc = LL_ERR_CUDA;
            }
        } else if (rc == LL_ERR_CUDA) {
            llh::set_error("CUDA error during bench: %s", cudaGetErrorString(cudaGetLastError()));
        }
        return rc;
    }
};

struct LayeredChain : Chain {
    int enqueue_layers(cudaStream_t s) override
    {
        for (int l = 0; l < n; ++l)
            llk::launch_dense_warp_rm(dW[l], db[l], dact[l], dact[l + 1], dims[l + 1], dims[l], acts[l], s);
        return LL_OK;
    }
};

struct CublasChain : Chain {
    cublasHandle_t h = nullptr;
    void *ws = nullptr;
    ~CublasChain() override
    {
        if (h)
            cublasDestroy(h);
        if (ws)
            cudaFree(ws);
    }
    int init_blas()
    {
        if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) {
            llh::set_error("cublasCreate failed");
            return LL_ERR_CUDA;
        }
        cublasSetStream(h, stream);
        cublasSetMathMode(h, CUBLAS_DEFAULT_MATH);  // fp32, as src/bench_cublas_mlp_graph.cu:117
        LL_CUDA_TRY(cudaMalloc(&ws, 4 << 20));
        cublasSetWorkspace(h, ws, 4 << 20);  // no allocation during graph capture
        return LL_OK;
    }
    int enqueue_layers(cudaStream_t s) override
    {
        cublasSetStream(h, s);
        const float one = 1.0f, zero = 0.0f;
        for (int l = 0; l < n; ++l) {
            const int M = dims[l + 1], K = dims[l];
            if (cublasSgemm(h, CUBLAS_OP_T, CUBLAS_OP_N, M, 1, K, &one, dW[l], K, dact[l], K, &zero, dact[l + 1], M) !=
                CUBLAS_STATUS_SUCCESS) {
                llh::set_error("cublasSgemm failed at layer %d", l);
                return LL_ERR_CUDA;
            }
            llk::bias_act_kernel<<<(M + 255) / 256, 256, 0, s>>>(dact[l + 1], db[l], M, acts[l]);
        }
        return LL_OK;
    }
};

int check_fp32_net(const ll_net_desc *net, const float *const *W)
{
    if (!net || !W || net->n_layers < 1 || net->n_layers > 64 || !net->layers) {
        llh::set_error("invalid net descriptor");
        return LL_ERR_BAD_DESC;
    }
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        if (d.wtype != LL_W_F32 || d.in_dim < 1 || d.out_dim < 1 || !W[l] ||
            (l > 0 && net->layers[l - 1].out_dim != d.in_dim)) {
            llh::set_error("layer %d: fp32 weights and consistent dims required", l);
            return LL_ERR_BAD_DESC;
        }
    }
    return LL_OK;
}

}  // namespace

struct ll_layered_mlp {
    LayeredChain c;
};
struct ll_cublas_mlp {
    CublasChain c;
};

extern "C" {

int ll_layered_mlp_create(const ll_net_desc *net, const float *const *W, const float *const *b, int device,
                          ll_layered_mlp **out)
{
    if (!out)
        return LL_ERR_INVALID_ARG;
    *out = nullptr;
    int rc = check_fp32_net(net, W);
    if (rc)
        return rc;
    auto *m = new ll_layered_mlp();
    rc = m->c.setup(net, W, b, device);
    if (rc) {
        m->c.release();
        delete m;
        return rc;
    }
    *out = m;
    return LL_OK;
}

int ll_layered_mlp_bench(ll_layered_mlp *m, int mode, const float *xs, int n_x, int n_req, float *y_last,
                         double *lat_us)
{
    if (!m || !xs || n_x < 1 || n_req < 0)
        return LL_ERR_INVALID_ARG;
    return m->c.bench(mode, xs, n_x, n_req, y_last, lat_us);
}

int ll_layered_mlp_destroy(ll_layered_mlp *m)
{
    if (m) {
        m->c.release();
        delete m;
    }
    return LL_OK;
}

int ll_cublas_mlp_create(const ll_net_desc *net, const float *const *W, const float *const *b, int device,
                         ll_cublas_mlp **out)
{
    if (!out)
        return LL_ERR_INVALID_ARG;
    *out = nullptr;
    int rc = check_fp32_net(net, W);
    if (rc)
        return rc;
    auto *m = new ll_cublas_mlp();
    rc = m->c.setup(net, W, b, device);
    if (rc == LL_OK)
        rc = m->c.init_blas();
    if (rc) {
        m->c.release();
        delete m;
        return rc;
    }
    *out = m;
    return LL_OK;
}

int ll_cublas_mlp_bench(ll_cublas_mlp *m, int mode, const float *xs, int n_x, int n_req, float *y_last,
                        double *lat_us)
{
    if (!m || !xs || n_x < 1 || n_req < 0)
        return LL_ERR_INVALID_ARG;
    return m->c.bench(mode, xs, n_x, n_req, y_last, lat_us);
}

int ll_cublas_mlp_destroy(ll_cublas_mlp *m)
{
    if (m) {
        m->c.release();
        delete m;
    }
    return LL_OK;
}

}  // extern "C"
