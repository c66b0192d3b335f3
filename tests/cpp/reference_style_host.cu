// A host program written the way the reference's benches are
// (src/bench_persistent_mbyv_mlp.cu:386-559, src/bench_custom_warp_mlp_graph.cu:96-121,
// src/bench_custom_mbyv_mlp.cu:83-160), compiled against this library's headers only:
// netcfg:: dims, host_init-style seeded weights, the TickBuffer mailbox driven by hand
// (write x, bump seq_in, spin on seq_out, stop = 1 + bump), and the launch-per-layer
// template kernels ll::dense_warp_rm_kernel<M, K, BW, Act>, ll::launch_dense_mbyv_packed<M, K>
// and ll::dense_mbyv_kernel<ROWS, COLS, BLOCKS, WARPS, REG_N, SHMEM_N, GLOB_N> (padded
// row-major weights, per-layer scratch, the reference bench's block / warp / storage split).
//
// Usage: reference_style_host <out.bin>
// Writes, as float32: y_engine[OUT], y_warp[OUT], y_packed[OUT], y_mbyv[OUT], then x[IN], W1, b1, W2,
// b2, W3, b3.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <vector>

#include "ll/dense_mbyv.cuh"
#include "ll/dense_warp.cuh"
#include "ll/engine.hpp"
#include "ll/pack_weights.h"
#include "ll/tick_buffer.h"
#include "net_config.h"

using namespace netcfg;

#define CK(call)                                                                                 \
    do {                                                                                         \
        cudaError_t e_ = (call);                                                                 \
        if (e_ != cudaSuccess) {                                                                 \
            std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            return 1;                                                                            \
        }                                                                                        \
    } while (0)

static void host_init(std::vector<float> &v, float scale, uint32_t seed)
{
    ll::check_or_exit(ll_fill_normal(v.data(), v.size(), 0.0f, scale, seed), "ll_fill_normal");
}

// Row-major weights with the columns padded to ll::PaddedCols<K, WARPS> (the layout
// ll::dense_mbyv_kernel reads; the reference bench defines the same helper locally).
template <int M, int K, int WARPS>
static std::vector<float> pack_weights_padded_rm(const std::vector<float> &W_rm)
{
    constexpr size_t P = ll::PaddedCols<K, WARPS>::padded_cols;
    std::vector<float> out((size_t)M * P, 0.0f);
    for (int r = 0; r < M; ++r)
        std::memcpy(&out[(size_t)r * P], &W_rm[(size_t)r * K], sizeof(float) * K);
    return out;
}

int main(int argc, char **argv)
{
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s out.bin\n", argv[0]);
        return 2;
    }
    std::vector<float> h_x(IN_DIM), h_W1(H1_DIM * IN_DIM), h_b1(H1_DIM), h_W2(H2_DIM * H1_DIM), h_b2(H2_DIM),
        h_W3(OUT_DIM * H2_DIM), h_b3(OUT_DIM);
    host_init(h_x, 1.0f, 1);
    host_init(h_W1, 0.02f, 2);
    host_init(h_b1, 0.01f, 3);
    host_init(h_W2, 0.02f, 4);
    host_init(h_b2, 0.01f, 5);
    host_init(h_W3, 0.02f, 6);
    host_init(h_b3, 0.01f, 7);

    // ---- resident engine + hand-driven TickBuffer ----
    const ll_net_desc net = ll::nets::make_net(ll::nets::reference_mlp, 3);
    std::vector<float> y_engine(OUT_DIM);
    {
        ll::Engine eng(net, {h_W1.data(), h_W2.data(), h_W3.data()}, {h_b1.data(), h_b2.data(), h_b3.data()});
        eng.start();
        auto *tb = eng.mailbox<ll::cfg::IN, ll::cfg::OUT>();
        uint32_t seq = tb->seq_out;
        for (int rep = 0; rep < 3; ++rep) {
            for (size_t i = 0; i < IN_DIM; ++i)
                tb->x[i] = h_x[i];
            __atomic_thread_fence(__ATOMIC_RELEASE);
            tb->seq_in = ++seq;
            ll::host_sfence();
            long spins = 0;
            while (tb->seq_out != seq) {
                ll::cpu_pause();
                if (++spins > 2000000000L) {
                    std::fprintf(stderr, "no answer\n");
                    return 1;
                }
            }
        }
        for (size_t i = 0; i < OUT_DIM; ++i)
            y_engine[i] = tb->y[i];
        eng.stop();
    }

    // ---- launch-per-layer template kernels ----
    float *d_x, *d_y1, *d_y2, *d_y3, *d_W1, *d_b1, *d_W2, *d_b2, *d_W3, *d_b3;
    CK(cudaMalloc(&d_x, IN_DIM * 4));
    CK(cudaMalloc(&d_y1, H1_DIM * 4));
    CK(cudaMalloc(&d_y2, H2_DIM * 4));
    CK(cudaMalloc(&d_y3, OUT_DIM * 4));
    CK(cudaMalloc(&d_W1, h_W1.size() * 4));
    CK(cudaMalloc(&d_b1, h_b1.size() * 4));
    CK(cudaMalloc(&d_W2, h_W2.size() * 4));
    CK(cudaMalloc(&d_b2, h_b2.size() * 4));
    CK(cudaMalloc(&d_W3, h_W3.size() * 4));
    CK(cudaMalloc(&d_b3, h_b3.size() * 4));
    CK(cudaMemcpy(d_x, h_x.data(), IN_DIM * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_W1, h_W1.data(), h_W1.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_b1, h_b1.data(), h_b1.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_W2, h_W2.data(), h_W2.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_b2, h_b2.data(), h_b2.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_W3, h_W3.data(), h_W3.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_b3, h_b3.data(), h_b3.size() * 4, cudaMemcpyHostToDevice));
    cudaStream_t s;
    CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    constexpr int BW1 = 8, BW2 = 4, BW3 = 1;  // src/bench_custom_warp_mlp_graph.cu:94-96
    ll::dense_warp_rm_kernel<(int)H1_DIM, (int)IN_DIM, BW1>
        <<<(H1_DIM + BW1 - 1) / BW1, BW1 * 32, IN_DIM * 4, s>>>(d_W1, d_b1, d_x, d_y1, ll::ActRelu{});
    ll::dense_warp_rm_kernel<(int)H2_DIM, (int)H1_DIM, BW2>
        <<<(H2_DIM + BW2 - 1) / BW2, BW2 * 32, H1_DIM * 4, s>>>(d_W2, d_b2, d_y1, d_y2, ll::ActRelu{});
    ll::dense_warp_rm_kernel<(int)OUT_DIM, (int)H2_DIM, BW3>
        <<<(OUT_DIM + BW3 - 1) / BW3, BW3 * 32, H2_DIM * 4, s>>>(d_W3, d_b3, d_y2, d_y3, ll::ActIdentity{});
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(s));
    std::vector<float> y_warp(OUT_DIM);
    CK(cudaMemcpy(y_warp.data(), d_y3, OUT_DIM * 4, cudaMemcpyDeviceToHost));

    // packed K-major path, last layer only re-run through dense_mbyv_packed on the same h2
    constexpr size_t Mpad3 = (OUT_DIM + 31) / 32 * 32;
    std::vector<float> W3cm(H2_DIM * Mpad3), b3p(Mpad3);
    ll::pack_rm_to_kmajor_padded(h_W3.data(), OUT_DIM, H2_DIM, W3cm.data(), Mpad3);
    ll::pack_bias_padded(h_b3.data(), OUT_DIM, b3p.data(), Mpad3);
    float *d_W3cm, *d_b3p, *d_y3p;
    CK(cudaMalloc(&d_W3cm, W3cm.size() * 4));
    CK(cudaMalloc(&d_b3p, b3p.size() * 4));
    CK(cudaMalloc(&d_y3p, OUT_DIM * 4));
    CK(cudaMemcpy(d_W3cm, W3cm.data(), W3cm.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_b3p, b3p.data(), b3p.size() * 4, cudaMemcpyHostToDevice));
    ll::launch_dense_mbyv_packed<(int)OUT_DIM, (int)H2_DIM>(s, d_W3cm, d_b3p, d_y2, d_y3p, ll::ActIdentity{});
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(s));
    std::vector<float> y_packed(OUT_DIM);
    CK(cudaMemcpy(y_packed.data(), d_y3p, OUT_DIM * 4, cudaMemcpyDeviceToHost));

    // ---- ll::dense_mbyv_kernel, launched as src/bench_custom_mbyv_mlp.cu:83-160 does ----
    constexpr size_t L1_BLOCKS = 4, L1_WARPS = 8, L1_REG_N = 16, L1_SHMEM_N = 16, L1_GLOB_N = 128 - 16 - 16;
    constexpr size_t L2_BLOCKS = 2, L2_WARPS = 8, L2_REG_N = 16, L2_SHMEM_N = 8, L2_GLOB_N = 32 - 16 - 8;
    constexpr size_t L3_BLOCKS = 1, L3_WARPS = 2, L3_REG_N = 16, L3_SHMEM_N = 0, L3_GLOB_N = 32 - 16;
    auto h_W1pad = pack_weights_padded_rm<(int)H1_DIM, (int)IN_DIM, (int)L1_WARPS>(h_W1);
    auto h_W2pad = pack_weights_padded_rm<(int)H2_DIM, (int)H1_DIM, (int)L2_WARPS>(h_W2);
    auto h_W3pad = pack_weights_padded_rm<(int)OUT_DIM, (int)H2_DIM, (int)L3_WARPS>(h_W3);
    float *d_W1p, *d_W2p, *d_W3p, *d_m1, *d_m2, *d_m3, *d_s1, *d_s2, *d_s3;
    CK(cudaMalloc(&d_W1p, h_W1pad.size() * 4));
    CK(cudaMalloc(&d_W2p, h_W2pad.size() * 4));
    CK(cudaMalloc(&d_W3p, h_W3pad.size() * 4));
    CK(cudaMalloc(&d_m1, H1_DIM * 4));
    CK(cudaMalloc(&d_m2, H2_DIM * 4));
    CK(cudaMalloc(&d_m3, OUT_DIM * 4));
    CK(cudaMalloc(&d_s1, L1_BLOCKS * L1_WARPS * 32 * L1_GLOB_N * 4));
    CK(cudaMalloc(&d_s2, L2_BLOCKS * L2_WARPS * 32 * L2_GLOB_N * 4));
    CK(cudaMalloc(&d_s3, L3_BLOCKS * L3_WARPS * 32 * L3_GLOB_N * 4));
    CK(cudaMemcpy(d_W1p, h_W1pad.data(), h_W1pad.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_W2p, h_W2pad.data(), h_W2pad.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_W3p, h_W3pad.data(), h_W3pad.size() * 4, cudaMemcpyHostToDevice));
    dim3 b1(32, (unsigned)L1_WARPS, 1), b2(32, (unsigned)L2_WARPS, 1), b3(32, (unsigned)L3_WARPS, 1);
    ll::dense_mbyv_kernel<H1_DIM, IN_DIM, L1_BLOCKS, L1_WARPS, L1_REG_N, L1_SHMEM_N, L1_GLOB_N>
        <<<L1_BLOCKS, b1, 0, s>>>(d_W1p, d_b1, d_x, d_m1, d_s1, ll::ActRelu{});
    ll::dense_mbyv_kernel<H2_DIM, H1_DIM, L2_BLOCKS, L2_WARPS, L2_REG_N, L2_SHMEM_N, L2_GLOB_N>
        <<<L2_BLOCKS, b2, 0, s>>>(d_W2p, d_b2, d_m1, d_m2, d_s2, ll::ActRelu{});
    ll::dense_mbyv_kernel<OUT_DIM, H2_DIM, L3_BLOCKS, L3_WARPS, L3_REG_N, L3_SHMEM_N, L3_GLOB_N>
        <<<L3_BLOCKS, b3, 0, s>>>(d_W3p, d_b3, d_m2, d_m3, d_s3, ll::ActIdentity{});
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(s));
    std::vector<float> y_mbyv(OUT_DIM);
    CK(cudaMemcpy(y_mbyv.data(), d_m3, OUT_DIM * 4, cudaMemcpyDeviceToHost));

    FILE *f = std::fopen(argv[1], "wb");
    if (!f)
        return 1;
    for (auto *v : {&y_engine, &y_warp, &y_packed, &y_mbyv, &h_x, &h_W1, &h_b1, &h_W2, &h_b2, &h_W3, &h_b3})
        std::fwrite(v->data(), 4, v->size(), f);
    std::fclose(f);
    std::printf("engine %.8f warp %.8f packed %.8f mbyv %.8f\n", y_engine[0], y_warp[0], y_packed[0], y_mbyv[0]);
    for (auto p : {d_x, d_y1, d_y2, d_y3, d_W1, d_b1, d_W2, d_b2, d_W3, d_b3, d_W3cm, d_b3p, d_y3p, d_W1p, d_W2p,
                   d_W3p, d_m1, d_m2, d_m3, d_s1, d_s2, d_s3})
        cudaFree(p);
    cudaStreamDestroy(s);
    return 0;
}
