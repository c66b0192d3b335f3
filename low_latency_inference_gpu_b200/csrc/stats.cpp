// Latency statistics.  Same definitions as the reference's ll::compute_stats
// (include/bench_utils.h:144-171): sort, percentiles by linear interpolation
// between neighbouring samples, population standard deviation.
#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>

#include "common.h"

extern "C" void ll_compute_stats(const double *xs, size_t n, ll_stats *out)
{
    *out = ll_stats{0, 0, 0, 0, 0, 0, 0};
    if (n == 0 || !xs)
        return;
    std::vector<double> v(xs, xs + n);
    std::sort(v.begin(), v.end());
    auto pct = [&](double p) {
        if (v.size() == 1)
            return v[0];
        const double idx = p * (double)(v.size() - 1);
        const size_t i = (size_t)std::floor(idx);
        const size_t j = std::min(i + 1, v.size() - 1);
        const double t = idx - (double)i;
        return v[i] * (1.0 - t) + v[j] * t;
    };
    out->p50 = pct(0.50);
    out->p90 = pct(0.90);
    out->p99 = pct(0.99);
    out->min = v.front();
    out->max = v.back();
    out->mean = std::accumulate(v.begin(), v.end(), 0.0) / (double)v.size();
    double var = 0.0;
    for (double x : v)
        var += (x - out->mean) * (x - out->mean);
    out->sd = std::sqrt(var / (double)v.size());
}
