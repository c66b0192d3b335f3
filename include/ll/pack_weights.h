// Host weight packing with the reference's names (include/ll/pack_weights.cuh:9-32),
// forwarding to the library, plus the padded-column helper of
// include/ll/dense_mbyv.cuh:101-105.
#pragma once
#include <cstddef>

#include "ll_b200.h"

namespace ll {

static inline size_t round_up(size_t x, size_t m)
{
    return ((x + m - 1) / m) * m;
}

// W_cm[k*Mpad + m] = (m < M) ? W_rm[m*K + k] : 0
inline void pack_rm_to_kmajor_padded(const float *W_rm, size_t M, size_t K, float *W_cm, size_t Mpad)
{
    ll_pack_rm_to_kmajor_padded(W_rm, M, K, W_cm, Mpad);
}

inline void pack_bias_padded(const float *b, size_t M, float *b_pad, size_t Mpad)
{
    ll_pack_bias_padded(b, M, b_pad, Mpad);
}

constexpr size_t ceil_div(size_t a, size_t b)
{
    return (a + b - 1) / b;
}

template <size_t COLS, size_t WARPS>
struct PaddedCols {
    static constexpr size_t cols_per_warp = ceil_div(COLS, WARPS);
    static constexpr size_t padded_cols = WARPS * cols_per_warp;
};

}  // namespace ll
