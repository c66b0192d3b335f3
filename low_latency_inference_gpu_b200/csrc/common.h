// Host-side helpers shared by the library's translation units.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "ll_b200.h"

namespace llh {

// Thread-local message behind ll_last_error().
void set_error(const char *fmt, ...);

inline size_t round_up(size_t x, size_t m)
{
    return (x + m - 1) / m * m;
}

inline int ceil_div(int a, int b)
{
    return (a + b - 1) / b;
}

// One 16-byte load / store instruction on an aligned address.  Written in asm so
// the compiler can neither split the access nor reorder it: a tagged chunk
// {v0, v1, v2, tag} must be read and written as a whole (aligned 16-byte SSE
// accesses are atomic on x86 CPUs with AVX).
inline void load16(const void *src, uint32_t out[4])
{
#if defined(__x86_64__)
    __attribute__((aligned(16))) uint32_t tmp[4];
    asm volatile("movdqa (%1), %%xmm15\n\tmovdqa %%xmm15, (%0)" ::"r"(tmp), "r"(src) : "xmm15", "memory");
    out[0] = tmp[0];
    out[1] = tmp[1];
    out[2] = tmp[2];
    out[3] = tmp[3];
#else
    __atomic_load(reinterpret_cast<const __int128 *>(src), reinterpret_cast<__int128 *>(out), __ATOMIC_ACQUIRE);
#endif
}

inline void store16(void *dst, const uint32_t in[4])
{
#if defined(__x86_64__)
    __attribute__((aligned(16))) uint32_t tmp[4] = {in[0], in[1], in[2], in[3]};
    asm volatile("movdqa (%1), %%xmm15\n\tmovdqa %%xmm15, (%0)" ::"r"(dst), "r"(tmp) : "xmm15", "memory");
#else
    __atomic_store(reinterpret_cast<__int128 *>(dst), reinterpret_cast<const __int128 *>(in), __ATOMIC_RELEASE);
#endif
}

}  // namespace llh

#define LL_CUDA_TRY(call)                                                                                   \
    do {                                                                                                    \
        cudaError_t _e = (call);                                                                            \
        if (_e != cudaSuccess) {                                                                            \
            llh::set_error("%s failed: %s (%d) at %s:%d", #call, cudaGetErrorString(_e), (int)_e, __FILE__, \
                           __LINE__);                                                                       \
            return LL_ERR_CUDA;                                                                             \
        }                                                                                                   \
    } while (0)
