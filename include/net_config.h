// Network configuration, same names and values as the reference's
// include/net_config.h:6-26 (netcfg::* and ll::cfg::* for its 512->256->64->1
// MLP), so host code written against the reference compiles unchanged.  The
// runtime layer descriptors (ll_layer_desc, include/ll_b200.h) generalise these
// compile-time constants; ll::nets lists the benchmarked workloads.
#pragma once
#include <cstddef>

#include "ll_b200.h"

namespace netcfg {
static constexpr std::size_t IN_DIM = 512;
static constexpr std::size_t H1_DIM = 256;
static constexpr std::size_t H2_DIM = 64;
static constexpr std::size_t OUT_DIM = 1;
static constexpr std::size_t BATCH = 1;
}  // namespace netcfg

namespace ll::cfg {
constexpr int IN = 512;
constexpr int H1 = 256;
constexpr int H2 = 64;
constexpr int OUT = 1;
constexpr int WARPS_PER_BLOCK = 8;
}  // namespace ll::cfg

namespace ll::nets {

// The reference's own MLP as a descriptor list (ReLU, ReLU, identity).
inline constexpr ll_layer_desc reference_mlp[] = {
    {512, 256, LL_ACT_RELU, LL_W_F32}, {256, 64, LL_ACT_RELU, LL_W_F32}, {64, 1, LL_ACT_IDENTITY, LL_W_F32}};

// fp32 64->256->256->16, ReLU hidden, identity out, batch 1.
inline constexpr ll_layer_desc config0[] = {
    {64, 256, LL_ACT_RELU, LL_W_F32}, {256, 256, LL_ACT_RELU, LL_W_F32}, {256, 16, LL_ACT_IDENTITY, LL_W_F32}};

// fp32 128 -> 512 (x8 square layers) -> 32, ReLU hidden: 10 layers.
inline constexpr ll_layer_desc config1[] = {
    {128, 512, LL_ACT_RELU, LL_W_F32}, {512, 512, LL_ACT_RELU, LL_W_F32}, {512, 512, LL_ACT_RELU, LL_W_F32},
    {512, 512, LL_ACT_RELU, LL_W_F32}, {512, 512, LL_ACT_RELU, LL_W_F32}, {512, 512, LL_ACT_RELU, LL_W_F32},
    {512, 512, LL_ACT_RELU, LL_W_F32}, {512, 512, LL_ACT_RELU, LL_W_F32}, {512, 512, LL_ACT_RELU, LL_W_F32},
    {512, 32, LL_ACT_IDENTITY, LL_W_F32}};

inline constexpr ll_net_desc make_net(const ll_layer_desc *layers, int n, int max_batch = 1)
{
    return ll_net_desc{n, layers, max_batch, 0};
}

}  // namespace ll::nets
