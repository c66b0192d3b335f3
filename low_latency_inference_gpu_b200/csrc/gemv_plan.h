// Host-side plan of the small-batch kernel (gemv_net.cuh), shared by the batched
// forward (batched.cu: one cooperative launch per forward) and the engine's resident
// variant (engine.cu): the shared-memory layout, the per-CTA weight images, and the
// parameter fields that do not change between forwards.
#pragma once
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.h"
#include "gemv_net.cuh"

namespace llk {

// Dynamic shared memory per CTA the plan may use (232 448 B per block opt-in on B200;
// 1 KB is left for the kernel's static shared memory).
constexpr size_t kGvSmemLimit = 232448 - 1024;

// Shared-memory layout of the small-batch kernel for G CTAs: the per-CTA image
// (biases and scales of every layer's slice, then each layer's weight slice of
// ceil(N/G) rows), the per-warp partial sums, two mbarriers, then the staged input
// rows (fp32, largest in_dim + 4 floats apart).
struct GemvLayout {
    int rmax[LL_MAX_LAYERS] = {};
    uint32_t woff[LL_MAX_LAYERS] = {}, boff[LL_MAX_LAYERS] = {};
    uint32_t img_bytes = 0, img_a_bytes = 0;
    uint32_t off_part = 0, off_bar = 0, off_x = 0;
    int xstride = 0;
    size_t smem(int bp) const { return off_x + (size_t)bp * (size_t)xstride * sizeof(float); }
};

// Batch rows of the instantiation that serves `rows` rows.
inline int gemv_bp(int rows)
{
    return rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : rows <= 8 ? 8 : rows <= 16 ? 16 : 32;
}

inline void gemv_layout(const ll_net_desc *net, int G, GemvLayout &g)
{
    const bool i8 = net->layers[0].wtype == LL_W_I8;
    size_t fl = 0;
    int kmax = 0;
    for (int l = 0; l < net->n_layers; ++l) {
        g.rmax[l] = (net->layers[l].out_dim + G - 1) / G;
        g.boff[l] = (uint32_t)fl;
        fl += (size_t)g.rmax[l] * (i8 ? 2 : 1);
        kmax = std::max(kmax, net->layers[l].in_dim);
    }
    size_t off = llh::round_up(fl * sizeof(float), 16);
    for (int l = 0; l < net->n_layers; ++l) {
        g.woff[l] = (uint32_t)std::min<size_t>(off, 1u << 30);
        off += llh::round_up((size_t)g.rmax[l] * net->layers[l].in_dim * (i8 ? 1 : 2), 16);
        if (l == 0)
            g.img_a_bytes = (uint32_t)std::min<size_t>(off, 1u << 30);
    }
    g.img_bytes = (uint32_t)std::min<size_t>(off, 1u << 30);
    off = llh::round_up(off, 128);
    g.off_part = (uint32_t)std::min<size_t>(off, 1u << 30);
    off += (size_t)kGvWarps * kGvRowGroup * kGvMaxRows * sizeof(float);
    g.off_bar = (uint32_t)std::min<size_t>(off, 1u << 30);
    off += 16;  // two mbarriers: image copy A (biases + layer 0) and B (the other layers)
    g.off_x = (uint32_t)std::min<size_t>(llh::round_up(off, 128), 1u << 30);
    g.xstride = kmax + 4;
}

// The small-batch kernel takes nets of <= 32 rows whose slices and staged rows fit one SM.
inline bool gemv_fits(const ll_net_desc *net, int G)
{
    if (net->max_batch > kGvMaxRows)
        return false;
    GemvLayout g;
    gemv_layout(net, G, g);
    return g.smem(gemv_bp(net->max_batch)) <= kGvSmemLimit;
}

// Per-CTA images, img_bytes apart: CTA c's bias (+ scale) slices and weight slices of
// every layer (output rows [c*N/G, (c+1)*N/G)), laid out exactly as the front of its
// shared memory, so two bulk copies load them.  W: host row-major [N][K] in the layer's
// type (bf16 or int8); scales: int8 only.
inline std::vector<uint8_t> gemv_pack_images(const ll_net_desc *net, const void *const *W, const float *const *b,
                                             const float *const *scales, int G, const GemvLayout &gl)
{
    const bool i8 = net->layers[0].wtype == LL_W_I8;
    const size_t es = i8 ? 1 : 2;
    std::vector<uint8_t> img((size_t)G * gl.img_bytes, 0);
    for (int c = 0; c < G; ++c) {
        uint8_t *base = img.data() + (size_t)c * gl.img_bytes;
        for (int l = 0; l < net->n_layers; ++l) {
            const int K = net->layers[l].in_dim, N = net->layers[l].out_dim;
            const int r0 = (int)((unsigned)c * (unsigned)N / (unsigned)G);
            const int R = (int)((unsigned)(c + 1) * (unsigned)N / (unsigned)G) - r0;
            float *bd = reinterpret_cast<float *>(base) + gl.boff[l];
            for (int i = 0; i < R; ++i) {
                bd[i] = (b && b[l]) ? b[l][r0 + i] : 0.0f;
                if (i8)
                    bd[gl.rmax[l] + i] = scales[l][r0 + i];
            }
            std::memcpy(base + gl.woff[l], static_cast<const uint8_t *>(W[l]) + (size_t)r0 * K * es, (size_t)R * K * es);
        }
    }
    return img;
}

// The fields of GemvNetParams fixed by the net and the layout (the rest is per forward,
// or the caller's buffers).
inline void gemv_static_params(const ll_net_desc *net, const GemvLayout &gl, const uint8_t *d_img, GemvNetParams &g)
{
    std::memset(&g, 0, sizeof(g));
    g.img = d_img;
    g.img_bytes = gl.img_bytes;
    g.img_a_bytes = gl.img_a_bytes;
    for (int l = 0; l < net->n_layers; ++l) {
        g.dims[l] = net->layers[l].in_dim;
        g.acts[l] = net->layers[l].act;
        g.rmax[l] = gl.rmax[l];
        g.woff[l] = gl.woff[l];
        g.boff[l] = gl.boff[l];
    }
    g.dims[net->n_layers] = net->layers[net->n_layers - 1].out_dim;
    g.n_layers = net->n_layers;
    g.xstride = gl.xstride;
    g.off_part = gl.off_part;
    g.off_bar = gl.off_bar;
    g.off_x = gl.off_x;
}

}  // namespace llk
