// C++ host wrapper over the C ABI (include/ll_b200.h).
//
// ll::Engine owns one resident engine on one GPU: it replaces the setup, launch
// and stop code of the reference's persistent benches
// (src/bench_persistent_mbyv_mlp.cu:386-491, 553-559) with RAII.  Errors throw
// ll::Error (or, with ll::ExitOnError, print and exit like the reference's
// CUDA_CHECK, include/bench_utils.h:14-22).
#pragma once
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include "ll/tick_buffer.h"
#include "ll_b200.h"

namespace ll {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

inline void check(int rc, const char *what)
{
    if (rc != LL_OK)
        throw Error(rc, std::string(what) + ": " + ll_last_error());
}

// Reference-style error handling: print and exit(1).
inline void check_or_exit(int rc, const char *what)
{
    if (rc != LL_OK) {
        std::fprintf(stderr, "%s failed (%d): %s\n", what, rc, ll_last_error());
        std::exit(1);
    }
}

class Engine {
public:
    Engine(const ll_net_desc &net, const std::vector<const void *> &W, const std::vector<const float *> &b,
           const std::vector<const float *> &scales = {}, int device = 0, const ll_engine_opts *opts = nullptr)
        : in_(net.layers[0].in_dim), out_(net.layers[net.n_layers - 1].out_dim)
    {
        check(ll_engine_create_ex(&net, W.data(), b.empty() ? nullptr : b.data(),
                                  scales.empty() ? nullptr : scales.data(), device, opts, &e_),
              "ll_engine_create");
    }
    Engine(const Engine &) = delete;
    Engine &operator=(const Engine &) = delete;
    ~Engine()
    {
        if (e_)
            ll_engine_destroy(e_);
    }

    // The mailbox, typed like the reference's TickBuffer (batch-1 nets).
    template <int IN, int OUT>
    TickBuffer<IN, OUT> *mailbox()
    {
        if (IN != in_ || OUT != out_)
            throw Error(LL_ERR_INVALID_ARG, "TickBuffer dims do not match the net");
        return static_cast<TickBuffer<IN, OUT> *>(ll_engine_mailbox(e_));
    }

    void start() { check(ll_engine_start(e_), "ll_engine_start"); }
    uint32_t submit(const float *x, int n_rows = 1)
    {
        uint32_t s = 0;
        check(ll_submit(e_, x, n_rows, &s), "ll_submit");
        return s;
    }
    void poll(uint32_t seq, float *y, uint64_t timeout_ns = 2000000000ull)
    {
        check(ll_poll(e_, seq, y, timeout_ns), "ll_poll");
    }
    void infer(const float *x, float *y, int n_rows = 1, uint64_t timeout_ns = 2000000000ull)
    {
        check(ll_infer(e_, x, n_rows, y, timeout_ns), "ll_infer");
    }
    void stop() { check(ll_engine_stop(e_), "ll_engine_stop"); }
    ll_engine_info info()
    {
        ll_engine_info i{};
        check(ll_engine_get_info(e_, &i), "ll_engine_get_info");
        return i;
    }
    ll_engine *handle() { return e_; }

private:
    ll_engine *e_ = nullptr;
    int in_, out_;
};

// Latency statistics, include/bench_utils.h:140-177.
struct Stats {
    double p50 = 0, p90 = 0, p99 = 0, min = 0, max = 0, mean = 0, sd = 0;
};

inline Stats compute_stats(const std::vector<double> &xs)
{
    ll_stats s{};
    ll_compute_stats(xs.data(), xs.size(), &s);
    return Stats{s.p50, s.p90, s.p99, s.min, s.max, s.mean, s.sd};
}

inline void print_stats(const char *name, const Stats &s, const char *unit = "us")
{
    std::printf("%s [%s] p50=%.3f p90=%.3f p99=%.3f min=%.3f max=%.3f mean=%.3f sd=%.3f\n", name, unit, s.p50, s.p90,
                s.p99, s.min, s.max, s.mean, s.sd);
}

}  // namespace ll
