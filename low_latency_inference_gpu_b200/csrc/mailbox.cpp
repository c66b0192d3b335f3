// Host half of the mailbox protocol, on plain memory (no CUDA): the engine
// uses it on host-mapped pinned memory; tests drive it against a CPU thread
// that plays the device.
//
// Protocol (reference: src/bench_persistent_mbyv_mlp.cu:23-40, 536-548):
//   post: write x and n_rows, then release-store seq_in (x86 TSO orders the
//         plain stores before it; with write-combined memory an sfence flushes
//         the payload before the doorbell and the doorbell itself afterwards);
//   wait: spin with `pause` on an acquire load of seq_out, then read y.
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstring>
#include <thread>

#include "common.h"

#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace llh {

static thread_local std::string g_last_error;

void set_error(const char *fmt, ...)
{
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

const char *last_error()
{
    return g_last_error.c_str();
}

}  // namespace llh

static inline void cpu_relax()
{
#if defined(__x86_64__)
    _mm_pause();
#else
    std::this_thread::yield();
#endif
}

static inline void store_fence()
{
#if defined(__x86_64__)
    _mm_sfence();
#else
    std::atomic_thread_fence(std::memory_order_seq_cst);
#endif
}

extern "C" {

const char *ll_last_error(void)
{
    return llh::last_error();
}

const char *ll_version(void)
{
    return "ll_b200 0.1 (sm_100a)";
}

size_t ll_mailbox_bytes(int in_dim, int out_dim, int max_batch)
{
    const size_t b = max_batch < 1 ? 1 : (size_t)max_batch;
    return llh::round_up(sizeof(ll_tick_header) + 4 * b * (size_t)in_dim + 4 * b * (size_t)out_dim, 64);
}

size_t ll_tagged_y_offset(int in_dim)
{
    return llh::round_up(sizeof(ll_tick_header) + 16 * (size_t)((in_dim + 2) / 3), 64);
}

size_t ll_tagged_mailbox_bytes(int in_dim, int out_dim)
{
    return llh::round_up(ll_tagged_y_offset(in_dim) + 16 * (size_t)((out_dim + 2) / 3), 64);
}

void ll_tagged_post(void *mailbox, int in_dim, const float *x, uint32_t seq)
{
    const int xc = (in_dim + 2) / 3;
    char *base = static_cast<char *>(mailbox) + sizeof(ll_tick_header);
    for (int c = 0; c < xc; ++c) {
        float v[3];
        for (int e = 0; e < 3; ++e)
            v[e] = 3 * c + e < in_dim ? x[3 * c + e] : 0.0f;
        uint32_t w[4];
        std::memcpy(w, v, 12);
        w[3] = seq;
        llh::store16(base + 16 * c, w);  // one aligned 16-byte store: the device never sees half a chunk
    }
    auto *h = static_cast<ll_tick_header *>(mailbox);
    h->n_rows = 1;
    // seq_in keeps its meaning for hosts and tools that watch it; the device polls the chunks
    __atomic_store_n(const_cast<uint32_t *>(&h->seq_in), seq, __ATOMIC_RELEASE);
}

int ll_tagged_wait(const void *mailbox, int in_dim, int out_dim, uint32_t seq, float *y, uint64_t timeout_ns)
{
    const int yc = (out_dim + 2) / 3;
    const char *base = static_cast<const char *>(mailbox) + ll_tagged_y_offset(in_dim);
    const auto t0 = std::chrono::steady_clock::now();
    uint32_t spins = 0;
    uint32_t w[4];
    for (;;) {
        int c = 0;
        for (; c < yc; ++c) {
            llh::load16(base + 16 * c, w);  // the whole chunk in one load: tag and values together
            if (w[3] != seq)
                break;
            if (y) {
                float v[3];
                std::memcpy(v, w, 12);
                for (int e = 0; e < 3 && 3 * c + e < out_dim; ++e)
                    y[3 * c + e] = v[e];
            }
        }
        if (c == yc)
            return LL_OK;
        cpu_relax();
        if ((++spins & 1023u) == 0) {
            const auto dt = std::chrono::steady_clock::now() - t0;
            if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(dt).count() > timeout_ns) {
                llh::set_error("tagged mailbox wait for seq %u timed out", seq);
                return LL_ERR_TIMEOUT;
            }
        }
    }
}

uint32_t ll_next_seq(uint32_t seq)
{
    uint32_t n = seq + 1u;
    if (n == 0u || n == LL_STOP_SEQ)
        n = 1u;
    return n;
}

void ll_mailbox_post(void *mailbox, int in_dim, const float *x, int n_rows, uint32_t seq, int write_combined)
{
    auto *h = static_cast<ll_tick_header *>(mailbox);
    float *xd = reinterpret_cast<float *>(static_cast<char *>(mailbox) + sizeof(ll_tick_header));
    if (x)
        std::memcpy(xd, x, sizeof(float) * (size_t)in_dim * (size_t)n_rows);
    h->n_rows = (uint32_t)n_rows;
    if (write_combined)
        store_fence();
    __atomic_store_n(const_cast<uint32_t *>(&h->seq_in), seq, __ATOMIC_RELEASE);
    if (write_combined)
        store_fence();
}

int ll_mailbox_wait(const void *mailbox, int in_dim, int out_dim, int max_batch, uint32_t seq, float *y, int n_rows,
                    uint64_t timeout_ns)
{
    const auto *h = static_cast<const ll_tick_header *>(mailbox);
    const auto t0 = std::chrono::steady_clock::now();
    uint32_t spins = 0;
    while (__atomic_load_n(const_cast<const uint32_t *>(&h->seq_out), __ATOMIC_ACQUIRE) != seq) {
        cpu_relax();
        if ((++spins & 1023u) == 0) {
            const auto dt = std::chrono::steady_clock::now() - t0;
            if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(dt).count() > timeout_ns) {
                llh::set_error("mailbox wait for seq %u timed out (seq_out=%u)", seq, h->seq_out);
                return LL_ERR_TIMEOUT;
            }
        }
    }
    if (y) {
        const float *yd = reinterpret_cast<const float *>(static_cast<const char *>(mailbox) +
                                                          sizeof(ll_tick_header) +
                                                          sizeof(float) * (size_t)in_dim * (size_t)max_batch);
        std::memcpy(y, yd, sizeof(float) * (size_t)out_dim * (size_t)n_rows);
    }
    return LL_OK;
}

}  // extern "C"
