// Seeded workload generators of the oracle -- TEST INFRASTRUCTURE ONLY.
//
// bench.py's reference arm and the tests draw the benchmark workloads from here, so
// that the process timing the reference's CPU forward loads nothing but oracle/
// libraries.  The draws are the workload definitions themselves (no reference
// code is involved): one std::mt19937 stream per net, W1, b1, W2, b2, ... in
// layer order; weights Xavier-uniform U(+-sqrt(6 / (fan_in + fan_out))) or
// N(0, 1 / sqrt(fan_in)), biases U[-0.01, 0.01]; inputs from their own seed,
// U[lo, hi] or N(mean, sd), request-major.  std::normal_distribution<float> on
// an mt19937 is also the reference's host_init (src/bench_cublas_mlp.cu:37-43).
// tests/test_oracle.py checks every function here against the product library's
// generators bit for bit (same libstdc++ on both sides).
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <random>

extern "C" {

void oracle_fill_uniform(float *out, size_t n, float lo, float hi, uint32_t seed)
{
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> ud(lo, hi);
    for (size_t i = 0; i < n; ++i)
        out[i] = ud(rng);
}

void oracle_fill_normal(float *out, size_t n, float mean, float sd, uint32_t seed)
{
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(mean, sd);
    for (size_t i = 0; i < n; ++i)
        out[i] = nd(rng);
}

// normal_fanin = 0: Xavier-uniform weights; 1: N(0, 1/sqrt(fan_in)).  W[l] is [dims[l+1] x dims[l]].
void oracle_init_params(int n_layers, const int *dims, int normal_fanin, uint32_t seed, float *const *W,
                        float *const *b)
{
    std::mt19937 rng(seed);
    std::uniform_real_distribution<float> bias(-0.01f, 0.01f);
    for (int l = 0; l < n_layers; ++l) {
        const int in = dims[l], out = dims[l + 1];
        const size_t n = (size_t)in * (size_t)out;
        if (normal_fanin) {
            std::normal_distribution<float> nd(0.0f, 1.0f / std::sqrt((float)in));
            for (size_t i = 0; i < n; ++i)
                W[l][i] = nd(rng);
        } else {
            const float lim = std::sqrt(6.0f / (float)(in + out));
            std::uniform_real_distribution<float> ud(-lim, lim);
            for (size_t i = 0; i < n; ++i)
                W[l][i] = ud(rng);
        }
        for (int i = 0; i < out; ++i)
            b[l][i] = bias(rng);
    }
}

}  // extern "C"
