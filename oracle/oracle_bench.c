/*
 * Timed loops over the CPU oracle -- test infrastructure and the timed CPU baseline only.
 *
 * Used by bench.py's cpu_baseline leg (kind "port") when the reference's own
 * CPU forward (oracle/_ref) is not available.  It restates the reference's
 * host-side measurement: sequential batch-1 requests through the fp32 layer
 * chain (src/bench_persistent_mbyv_mlp.cu:408-410), per-request latency from a
 * monotonic clock like std::chrono::steady_clock (src/bench_persistent_mbyv_mlp.cu:536-548).
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

void oracle_mlp_f32(int n_layers, const int *dims, const int *acts, const float *const *W, const float *const *b,
                    const float *x, float *y, int n_rows);

static double now_ns(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e9 + (double)ts.tv_nsec;
}

/*
 * n_req sequential requests; request r reads xs[(r % n_x) * dims[0] ...].
 * lat_ns (may be NULL) receives each request's latency; y_last receives the
 * last output.  Returns total wall time in ns.
 */
double oracle_bench_mlp_f32(int n_layers, const int *dims, const int *acts, const float *const *W,
                            const float *const *b, const float *xs, int n_x, long n_req, double *lat_ns,
                            float *y_last)
{
    float *y = (float *)malloc(sizeof(float) * (size_t)dims[n_layers]);
    double t_start = now_ns();
    for (long r = 0; r < n_req; ++r) {
        double t0 = now_ns();
        oracle_mlp_f32(n_layers, dims, acts, W, b, xs + (size_t)(r % n_x) * dims[0], y, 1);
        double t1 = now_ns();
        if (lat_ns)
            lat_ns[r] = t1 - t0;
    }
    double total = now_ns() - t_start;
    if (y_last)
        memcpy(y_last, y, sizeof(float) * (size_t)dims[n_layers]);
    free(y);
    return total;
}

typedef struct {
    int n_layers;
    const int *dims;
    const int *acts;
    const float *const *W;
    const float *const *b;
    const float *xs;
    int n_x;
    long n_req;
    int cpu;
    double ns;
} oracle_thread_arg;

static void *oracle_thread_main(void *p)
{
    oracle_thread_arg *a = (oracle_thread_arg *)p;
    if (a->cpu >= 0) {
        cpu_set_t set;
        CPU_ZERO(&set);
        CPU_SET(a->cpu, &set);
        pthread_setaffinity_np(pthread_self(), sizeof(set), &set);
    }
    a->ns = oracle_bench_mlp_f32(a->n_layers, a->dims, a->acts, a->W, a->b, a->xs, a->n_x, a->n_req, NULL, NULL);
    return NULL;
}

/*
 * n_threads independent request streams, n_req each; returns the slowest
 * thread's wall time in ns (aggregate rate = n_threads * n_req / that).
 */
double oracle_bench_mlp_f32_mt(int n_layers, const int *dims, const int *acts, const float *const *W,
                               const float *const *b, const float *xs, int n_x, long n_req, int n_threads,
                               const int *cpus)
{
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    oracle_thread_arg *args = (oracle_thread_arg *)malloc(sizeof(oracle_thread_arg) * (size_t)n_threads);
    for (int t = 0; t < n_threads; ++t) {
        oracle_thread_arg a = {n_layers, dims, acts, W, b, xs, n_x, n_req, cpus ? cpus[t] : -1, 0.0};
        args[t] = a;
        pthread_create(&th[t], NULL, oracle_thread_main, &args[t]);
    }
    double worst = 0.0;
    for (int t = 0; t < n_threads; ++t) {
        pthread_join(th[t], NULL);
        if (args[t].ns > worst)
            worst = args[t].ns;
    }
    free(th);
    free(args);
    return worst;
}
