// Exposes the reference's OWN host-side CPU forward as a C ABI -- TEST
// INFRASTRUCTURE ONLY (the oracle pin and the "reference" CPU baseline).
//
// Built by oracle/Makefile (target `ref`) into oracle/_ref/libref.so.  The
// reference translation unit is compiled from where it lies (REF_TU, set by
// the Makefile) with its `main` renamed, so the functions called below are
// the reference's own code, not a copy:
//   host_init           src/bench_cublas_mlp.cu:37-43   (mt19937 + normal_distribution<float>)
//   cpu_gemv_bias_relu  src/bench_cublas_mlp.cu:45-62   (same body as src/bench_persistent_mbyv_mlp.cu:50-67)
// and the layer chain of src/bench_persistent_mbyv_mlp.cu:408-410.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>
#include <pthread.h>
#include <sched.h>

#define main reference_bench_main
#include REF_TU
#undef main

extern "C" {

void ref_host_init(float *out, size_t n, float scale, uint32_t seed)
{
    std::vector<float> v(n);
    host_init(v, scale, seed);
    std::memcpy(out, v.data(), n * sizeof(float));
}

void ref_cpu_gemv_bias_relu(const float *W, const float *b, const float *x, float *y, int m, int k, int relu)
{
    std::vector<float> Wv(W, W + (size_t)m * k), bv(b, b + m), xv(x, x + k);
    std::vector<float> r = cpu_gemv_bias_relu(Wv, bv, xv, m, k, relu != 0);
    std::memcpy(y, r.data(), (size_t)m * sizeof(float));
}

struct RefNet {
    int n_layers;
    std::vector<int> dims;
    std::vector<int> relu;
    std::vector<std::vector<float>> W, b;
};

static RefNet make_net(int n_layers, const int *dims, const int *relu, const float *const *W, const float *const *b)
{
    RefNet n;
    n.n_layers = n_layers;
    n.dims.assign(dims, dims + n_layers + 1);
    n.relu.assign(relu, relu + n_layers);
    for (int l = 0; l < n_layers; ++l) {
        n.W.emplace_back(W[l], W[l] + (size_t)dims[l] * dims[l + 1]);
        n.b.emplace_back(b[l], b[l] + dims[l + 1]);
    }
    return n;
}

// One request through the reference chain: vectors in, vector out, exactly as
// the reference benches call it.
static std::vector<float> ref_forward(const RefNet &n, const std::vector<float> &x)
{
    std::vector<float> h = cpu_gemv_bias_relu(n.W[0], n.b[0], x, n.dims[1], n.dims[0], n.relu[0] != 0);
    for (int l = 1; l < n.n_layers; ++l)
        h = cpu_gemv_bias_relu(n.W[l], n.b[l], h, n.dims[l + 1], n.dims[l], n.relu[l] != 0);
    return h;
}

// Batch of independent rows through the chain (outputs row-major).
void ref_mlp_forward(int n_layers, const int *dims, const int *relu, const float *const *W, const float *const *b,
                     const float *x, float *y, int n_rows)
{
    RefNet n = make_net(n_layers, dims, relu, W, b);
    for (int r = 0; r < n_rows; ++r) {
        std::vector<float> xv(x + (size_t)r * dims[0], x + (size_t)(r + 1) * dims[0]);
        std::vector<float> h = ref_forward(n, xv);
        std::memcpy(y + (size_t)r * dims[n_layers], h.data(), sizeof(float) * dims[n_layers]);
    }
}

// Sequential timed requests (steady_clock, like src/bench_persistent_mbyv_mlp.cu:536-548).
// Returns total ns; lat_ns may be null.
double ref_bench_mlp(int n_layers, const int *dims, const int *relu, const float *const *W, const float *const *b,
                     const float *xs, int n_x, long n_req, double *lat_ns, float *y_last)
{
    RefNet n = make_net(n_layers, dims, relu, W, b);
    std::vector<float> xv(dims[0]), h;
    auto t_start = std::chrono::steady_clock::now();
    for (long r = 0; r < n_req; ++r) {
        auto t0 = std::chrono::steady_clock::now();
        std::memcpy(xv.data(), xs + (size_t)(r % n_x) * dims[0], sizeof(float) * dims[0]);
        h = ref_forward(n, xv);
        auto t1 = std::chrono::steady_clock::now();
        if (lat_ns)
            lat_ns[r] = std::chrono::duration<double, std::nano>(t1 - t0).count();
    }
    double total = std::chrono::duration<double, std::nano>(std::chrono::steady_clock::now() - t_start).count();
    if (y_last)
        std::memcpy(y_last, h.data(), sizeof(float) * dims[n_layers]);
    return total;
}

// n_threads independent streams of n_req sequential requests; returns the
// slowest thread's ns.
double ref_bench_mlp_mt(int n_layers, const int *dims, const int *relu, const float *const *W, const float *const *b,
                        const float *xs, int n_x, long n_req, int n_threads, const int *cpus)
{
    std::vector<double> ns(n_threads, 0.0);
    std::vector<std::thread> th;
    for (int t = 0; t < n_threads; ++t) {
        th.emplace_back([&, t]() {
            if (cpus && cpus[t] >= 0) {
                cpu_set_t set;
                CPU_ZERO(&set);
                CPU_SET(cpus[t], &set);
                pthread_setaffinity_np(pthread_self(), sizeof(set), &set);
            }
            ns[t] = ref_bench_mlp(n_layers, dims, relu, W, b, xs, n_x, n_req, nullptr, nullptr);
        });
    }
    double worst = 0.0;
    for (int t = 0; t < n_threads; ++t) {
        th[t].join();
        if (ns[t] > worst)
            worst = ns[t];
    }
    return worst;
}

}  // extern "C"
