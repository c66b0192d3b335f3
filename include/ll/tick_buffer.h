// The request/response mailbox, field for field the reference's TickBuffer
// (src/bench_persistent_mbyv_mlp.cu:88-95, src/bench_persistent_mlp.cu:65-72):
// seq_in (0 = idle, host bumps per request), seq_out (device echoes the
// finished seq), stop, a 32-bit word (the reference's `pad`, here the request's
// row count, 0 meaning 1), then x[IN] and y[OUT].  ll_engine_mailbox() returns
// memory with exactly this layout for batch-1 nets, so reference host code can
// keep writing h_tb->x[...] and spinning on h_tb->seq_out.
#pragma once
#include <cstddef>
#include <cstdint>

#include "ll_b200.h"

namespace ll {

inline constexpr uint32_t kStopSeq = LL_STOP_SEQ;  // src/bench_persistent_mbyv_mlp.cu:157

template <int IN, int OUT>
struct alignas(64) TickBuffer {
    volatile uint32_t seq_in;
    volatile uint32_t seq_out;
    volatile uint32_t stop;
    uint32_t pad;
    float x[IN];
    float y[OUT];
};

template <int IN, int OUT>
constexpr bool tick_buffer_layout_ok()
{
    using T = TickBuffer<IN, OUT>;
    return offsetof(T, seq_in) == 0 && offsetof(T, seq_out) == 4 && offsetof(T, stop) == 8 && offsetof(T, pad) == 12 &&
           offsetof(T, x) == sizeof(ll_tick_header) && offsetof(T, y) == sizeof(ll_tick_header) + sizeof(float) * IN;
}

static_assert(sizeof(ll_tick_header) == 16, "mailbox header is four 32-bit words");
static_assert(tick_buffer_layout_ok<512, 1>(), "reference TickBuffer layout");
static_assert(tick_buffer_layout_ok<64, 16>(), "config-0 TickBuffer layout");

// Host doorbell helpers with the reference's semantics (src/bench_persistent_mbyv_mlp.cu:23-40).
inline void cpu_pause()
{
#if defined(__x86_64__) || defined(_M_X64)
    __asm__ __volatile__("pause" ::: "memory");
#endif
}

inline void host_sfence()
{
#if defined(__x86_64__) || defined(_M_X64)
    __asm__ __volatile__("sfence" ::: "memory");
#else
    __atomic_thread_fence(__ATOMIC_SEQ_CST);
#endif
}

}  // namespace ll
