// Synthetic workload generators and host-side weight conversions.
//
// The reference seeds every tensor with its own std::mt19937 and draws
// std::normal_distribution<float> (host_init, src/bench_cublas_mlp.cu:37-43);
// ll_fill_normal is that exact procedure, so with the same libstdc++ it
// reproduces the reference's bytes.  ll_init_params draws a whole net from one
// stream (W1, b1, W2, b2, ...) for the Xavier-uniform / N(0, 1/fan_in) nets.
#include <cmath>
#include <cstring>
#include <random>

#include "common.h"

extern "C" {

int ll_fill_normal(float *out, size_t n, float mean, float stddev, uint32_t seed)
{
    if (!out && n) {
        llh::set_error("ll_fill_normal: out is NULL");
        return LL_ERR_INVALID_ARG;
    }
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(mean, stddev);
    for (size_t i = 0; i < n; ++i)
        out[i] = nd(rng);
    return LL_OK;
}

int ll_fill_uniform(float *out, size_t n, float lo, float hi, uint32_t seed)
{
    if (!out && n) {
        llh::set_error("ll_fill_uniform: out is NULL");
        return LL_ERR_INVALID_ARG;
    }
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> ud(lo, hi);
    for (size_t i = 0; i < n; ++i)
        out[i] = ud(rng);
    return LL_OK;
}

int ll_init_params(const ll_net_desc *net, int init, uint32_t seed, float *const *W, float *const *b)
{
    if (!net || !W || net->n_layers < 1) {
        llh::set_error("ll_init_params: invalid arguments");
        return LL_ERR_INVALID_ARG;
    }
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> bias(-0.01f, 0.01f);
    for (int l = 0; l < net->n_layers; ++l) {
        const int in = net->layers[l].in_dim, out = net->layers[l].out_dim;
        const size_t n = (size_t)in * out;
        if (init == LL_INIT_XAVIER_UNIFORM) {
            const float lim = std::sqrt(6.0f / (float)(in + out));
            std::uniform_real_distribution<float> ud(-lim, lim);
            for (size_t i = 0; i < n; ++i)
                W[l][i] = ud(rng);
        } else if (init == LL_INIT_NORMAL_FANIN) {
            std::normal_distribution<float> nd(0.0f, 1.0f / std::sqrt((float)in));
            for (size_t i = 0; i < n; ++i)
                W[l][i] = nd(rng);
        } else {
            llh::set_error("ll_init_params: unknown init %d", init);
            return LL_ERR_INVALID_ARG;
        }
        if (b && b[l]) {
            for (int i = 0; i < out; ++i)
                b[l][i] = bias(rng);
        }
    }
    return LL_OK;
}

void ll_f32_to_bf16(const float *in, uint16_t *out, size_t n)
{
    for (size_t i = 0; i < n; ++i) {
        uint32_t u;
        std::memcpy(&u, &in[i], 4);
        if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
            out[i] = (uint16_t)((u >> 16) | 0x40u);
            continue;
        }
        u += 0x7fffu + ((u >> 16) & 1u);
        out[i] = (uint16_t)(u >> 16);
    }
}

void ll_quantize_int8_rows(const float *W, int m, int k, int8_t *q, float *s)
{
    for (int i = 0; i < m; ++i) {
        const float *row = W + (size_t)i * k;
        float amax = 0.0f;
        for (int j = 0; j < k; ++j)
            amax = std::fmax(amax, std::fabs(row[j]));
        const float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
        s[i] = sc;
        for (int j = 0; j < k; ++j) {
            float v = std::rint(row[j] / sc);
            v = std::fmin(127.0f, std::fmax(-127.0f, v));
            q[(size_t)i * k + j] = (int8_t)v;
        }
    }
}

void ll_pack_rm_to_kmajor_padded(const float *W_rm, size_t M, size_t K, float *W_cm, size_t Mpad)
{
    std::memset(W_cm, 0, sizeof(float) * K * Mpad);
    for (size_t k = 0; k < K; ++k)
        for (size_t m = 0; m < M; ++m)
            W_cm[k * Mpad + m] = W_rm[m * K + k];
}

void ll_pack_bias_padded(const float *b, size_t M, float *b_pad, size_t Mpad)
{
    std::memset(b_pad, 0, sizeof(float) * Mpad);
    std::memcpy(b_pad, b, sizeof(float) * M);
}

}  // extern "C"
