/*
 * CPU oracle for the resident MLP engine -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load this library, and only as the checker (or the timed CPU baseline),
 * never as the thing measured or shipped.  The product path lives in
 * low_latency_inference_gpu_b200/ and fails loudly without its CUDA library.
 *
 * What it restates (reference = mamedov-ma/low_latency_inference_gpu):
 *   - oracle_gemv_bias_act(): the reference CPU forward `cpu_gemv_bias_relu`
 *     (src/bench_persistent_mbyv_mlp.cu:50-67, identical copies at
 *     src/bench_cublas_mlp.cu:45-62 and src/bench_persistent_cublas_mlp.cu:58-75):
 *     acc = 0; acc += W[i*k + j] * x[j] for j = 0..k-1 in order; acc += b[i];
 *     optional ReLU.  Compiled with -ffp-contract=off so every product and sum
 *     rounds separately, exactly like the reference at -O3 on x86-64.
 *   - oracle_mlp_f32(): the layer chain of src/bench_persistent_mbyv_mlp.cu:408-410
 *     generalised to N layers with a per-layer activation.
 *   - GELU, bf16 and int8 handling have NO counterpart in the reference; they
 *     are this project's definitions (parity for them is unpinned):
 *       GELU(v)  = 0.5 v (1 + erf(v / sqrt(2)))           (fp32, erff)
 *       bf16(v)  = round-to-nearest-even of the fp32 bit pattern to 16 bits
 *       int8     : s[m] = max_k |W[m,k]| / 127, q = clamp(rint(W/s), -127, 127)
 *     The linear part of every layer still runs the reference loop order.
 *
 * Pinning: tests/test_oracle.py checks oracle_gemv_bias_act bit-for-bit
 * against the reference's own cpu_gemv_bias_relu built from the reference
 * sources into oracle/_ref (see oracle/Makefile), and against the committed
 * golden vectors in tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ORACLE_ACT_IDENTITY = 0, ORACLE_ACT_RELU = 1, ORACLE_ACT_GELU = 2 };

static float apply_act(float v, int act)
{
    if (act == ORACLE_ACT_RELU)
        return v > 0.0f ? v : 0.0f; /* src/bench_persistent_mbyv_mlp.cu:62-63 */
    if (act == ORACLE_ACT_GELU)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
    return v;
}

/* fp32 -> bf16 bits, round to nearest even (NaN kept quiet). */
uint16_t oracle_f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))
        return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h)
{
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float oracle_round_bf16(float f)
{
    return oracle_bf16_to_f32(oracle_f32_to_bf16(f));
}

void oracle_round_bf16_array(const float *in, float *out, size_t n)
{
    for (size_t i = 0; i < n; ++i)
        out[i] = oracle_round_bf16(in[i]);
}

/*
 * y[i] = act(sum_j W[i*k+j] * x[j] + b[i]) with the reference's summation
 * order (src/bench_persistent_mbyv_mlp.cu:56-64).  b may be NULL (treated as 0,
 * still added so the rounding sequence matches).
 */
void oracle_gemv_bias_act(const float *W, const float *b, const float *x, float *y, int m, int k, int act)
{
    for (int i = 0; i < m; i++) {
        float acc = 0.0f;
        const float *row = W + (size_t)i * (size_t)k;
        for (int j = 0; j < k; j++)
            acc += row[j] * x[j];
        acc += b ? b[i] : 0.0f;
        y[i] = apply_act(acc, act);
    }
}

/*
 * fp32 MLP, batch of n_rows independent rows (row-major [n_rows x dims[0]]).
 * dims has n_layers+1 entries; acts has n_layers entries.
 */
void oracle_mlp_f32(int n_layers, const int *dims, const int *acts, const float *const *W, const float *const *b,
                    const float *x, float *y, int n_rows)
{
    int maxd = 0;
    for (int l = 0; l <= n_layers; ++l)
        if (dims[l] > maxd)
            maxd = dims[l];
    float *h0 = (float *)malloc(sizeof(float) * (size_t)maxd);
    float *h1 = (float *)malloc(sizeof(float) * (size_t)maxd);
    for (int r = 0; r < n_rows; ++r) {
        memcpy(h0, x + (size_t)r * dims[0], sizeof(float) * (size_t)dims[0]);
        for (int l = 0; l < n_layers; ++l) {
            oracle_gemv_bias_act(W[l], b[l], h0, h1, dims[l + 1], dims[l], acts[l]);
            float *t = h0;
            h0 = h1;
            h1 = t;
        }
        memcpy(y + (size_t)r * dims[n_layers], h0, sizeof(float) * (size_t)dims[n_layers]);
    }
    free(h0);
    free(h1);
}

/*
 * bf16-weight MLP (config family "bf16 weights, fp32 accumulate"): W holds bf16
 * bit patterns.  The input and every hidden activation are rounded to bf16;
 * products and sums are fp32 in the reference order; the last layer's output
 * stays fp32.
 */
void oracle_mlp_bf16(int n_layers, const int *dims, const int *acts, const uint16_t *const *W,
                     const float *const *b, const float *x, float *y, int n_rows)
{
    int maxd = 0;
    for (int l = 0; l <= n_layers; ++l)
        if (dims[l] > maxd)
            maxd = dims[l];
    float *h0 = (float *)malloc(sizeof(float) * (size_t)maxd);
    float *h1 = (float *)malloc(sizeof(float) * (size_t)maxd);
    for (int r = 0; r < n_rows; ++r) {
        for (int j = 0; j < dims[0]; ++j)
            h0[j] = oracle_round_bf16(x[(size_t)r * dims[0] + j]);
        for (int l = 0; l < n_layers; ++l) {
            const int m = dims[l + 1], k = dims[l];
            for (int i = 0; i < m; ++i) {
                float acc = 0.0f;
                const uint16_t *row = W[l] + (size_t)i * (size_t)k;
                for (int j = 0; j < k; ++j)
                    acc += oracle_bf16_to_f32(row[j]) * h0[j];
                acc += b[l] ? b[l][i] : 0.0f;
                float v = apply_act(acc, acts[l]);
                h1[i] = (l + 1 < n_layers) ? oracle_round_bf16(v) : v;
            }
            float *t = h0;
            h0 = h1;
            h1 = t;
        }
        memcpy(y + (size_t)r * dims[n_layers], h0, sizeof(float) * (size_t)dims[n_layers]);
    }
    free(h0);
    free(h1);
}

/* Symmetric per-output-channel int8 quantisation of a row-major [m x k] matrix. */
void oracle_quantize_int8_rows(const float *W, int m, int k, int8_t *q, float *s)
{
    for (int i = 0; i < m; ++i) {
        const float *row = W + (size_t)i * (size_t)k;
        float amax = 0.0f;
        for (int j = 0; j < k; ++j) {
            float a = fabsf(row[j]);
            if (a > amax)
                amax = a;
        }
        float sc = amax > 0.0f ? amax / 127.0f : 1.0f;
        s[i] = sc;
        for (int j = 0; j < k; ++j) {
            float v = rintf(row[j] / sc);
            if (v > 127.0f)
                v = 127.0f;
            if (v < -127.0f)
                v = -127.0f;
            q[(size_t)i * (size_t)k + j] = (int8_t)v;
        }
    }
}

/*
 * int8-weight MLP with per-output-channel fp32 scales and bf16 activations:
 * acc = sum_j q[i,j] * h[j] (fp32, reference order); v = s[i]*acc + b[i];
 * activation; hidden outputs rounded to bf16, last layer fp32.
 */
void oracle_mlp_int8(int n_layers, const int *dims, const int *acts, const int8_t *const *Q,
                     const float *const *S, const float *const *b, const float *x, float *y, int n_rows)
{
    int maxd = 0;
    for (int l = 0; l <= n_layers; ++l)
        if (dims[l] > maxd)
            maxd = dims[l];
    float *h0 = (float *)malloc(sizeof(float) * (size_t)maxd);
    float *h1 = (float *)malloc(sizeof(float) * (size_t)maxd);
    for (int r = 0; r < n_rows; ++r) {
        for (int j = 0; j < dims[0]; ++j)
            h0[j] = oracle_round_bf16(x[(size_t)r * dims[0] + j]);
        for (int l = 0; l < n_layers; ++l) {
            const int m = dims[l + 1], k = dims[l];
            for (int i = 0; i < m; ++i) {
                float acc = 0.0f;
                const int8_t *row = Q[l] + (size_t)i * (size_t)k;
                for (int j = 0; j < k; ++j)
                    acc += (float)row[j] * h0[j];
                float v = S[l][i] * acc + (b[l] ? b[l][i] : 0.0f);
                v = apply_act(v, acts[l]);
                h1[i] = (l + 1 < n_layers) ? oracle_round_bf16(v) : v;
            }
            float *t = h0;
            h0 = h1;
            h1 = t;
        }
        memcpy(y + (size_t)r * dims[n_layers], h0, sizeof(float) * (size_t)dims[n_layers]);
    }
    free(h0);
    free(h1);
}

/*
 * K-major padded packing, restating include/ll/pack_weights.cuh:16-26:
 * W_cm[k*Mpad + m] = (m < M) ? W_rm[m*K + k] : 0.
 */
void oracle_pack_rm_to_kmajor_padded(const float *W_rm, size_t M, size_t K, float *W_cm, size_t Mpad)
{
    memset(W_cm, 0, sizeof(float) * K * Mpad);
    for (size_t m = 0; m < M; ++m)
        for (size_t k = 0; k < K; ++k)
            W_cm[k * Mpad + m] = W_rm[m * K + k];
}

/* Percentiles with linear interpolation, restating include/bench_utils.h:144-158 on sorted input. */
double oracle_percentile_linear(const double *sorted, size_t n, double p)
{
    if (n == 0)
        return 0.0;
    if (n == 1)
        return sorted[0];
    double idx = p * (double)(n - 1);
    size_t i = (size_t)floor(idx);
    size_t j = i + 1 < n ? i + 1 : n - 1;
    double t = idx - (double)i;
    return sorted[i] * (1.0 - t) + sorted[j] * t;
}

/* Percentile, nearest-rank convention of include/bench_utils.h:39-46 on sorted input. */
double oracle_percentile_nearest(const double *sorted, size_t n, double p)
{
    if (n == 0)
        return 0.0;
    double idx = p * (double)(n - 1);
    size_t i = (size_t)(idx + 0.5);
    if (i >= n)
        i = n - 1;
    return sorted[i];
}
