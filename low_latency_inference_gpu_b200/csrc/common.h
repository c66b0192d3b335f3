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
