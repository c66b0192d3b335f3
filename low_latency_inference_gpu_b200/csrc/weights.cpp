// Weight files: a network's descriptor and its row-major weights, biases and
// int8 scales in one little-endian file, so real models load instead of the
// in-process generators (the reference fills its weights with host_init,
// src/bench_cublas_mlp.cu:37-43, and has no file format).
//
// Layout ("LLWB", version 1):
//   header   32 bytes: magic "LLWB", version, n_layers, wtype, max_batch, flags
//            (bit 0 biases present, bit 1 scales present), 2 reserved words;
//   layers   n_layers x 16 bytes: in_dim, out_dim, act, reserved;
//   payload  per layer: W [out x in] in the net's weight type, then the biases
//            [out] fp32 (if present), then the scales [out] fp32 (int8 nets);
//            every section starts on a 64-byte boundary (zero padding);
//   trailer  8 bytes: FNV-1a 64 of every payload byte (padding included).
#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include "common.h"

struct ll_weights {
    std::vector<ll_layer_desc> layers;
    ll_net_desc net{};
    std::vector<std::vector<uint8_t>> W;
    std::vector<std::vector<float>> b, s;
    bool has_b = false, has_s = false;
};

namespace {

constexpr uint32_t kMagic = 0x42574c4cu;  // "LLWB" little-endian
constexpr uint32_t kVersion = 1;

size_t esize(int wtype)
{
    return wtype == LL_W_F32 ? 4 : wtype == LL_W_BF16 ? 2 : 1;
}

struct Fnv {
    uint64_t h = 1469598103934665603ull;
    void add(const void *p, size_t n)
    {
        const uint8_t *c = static_cast<const uint8_t *>(p);
        for (size_t i = 0; i < n; ++i) {
            h ^= c[i];
            h *= 1099511628211ull;
        }
    }
};

struct File {
    FILE *f = nullptr;
    ~File()
    {
        if (f)
            fclose(f);
    }
};

int check_desc(const ll_net_desc *net)
{
    if (!net || net->n_layers < 1 || net->n_layers > 1024 || !net->layers) {
        llh::set_error("weights: bad net descriptor");
        return LL_ERR_BAD_DESC;
    }
    const int wt = net->layers[0].wtype;
    if (wt < LL_W_F32 || wt > LL_W_I8) {
        llh::set_error("weights: unknown weight type %d", wt);
        return LL_ERR_BAD_DESC;
    }
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        if (d.in_dim < 1 || d.out_dim < 1 || d.in_dim > (1 << 20) || d.out_dim > (1 << 20) || d.wtype != wt ||
            d.act < LL_ACT_IDENTITY || d.act > LL_ACT_GELU || (l > 0 && net->layers[l - 1].out_dim != d.in_dim)) {
            llh::set_error("weights: layer %d descriptor is invalid or does not chain", l);
            return LL_ERR_BAD_DESC;
        }
    }
    return LL_OK;
}

}  // namespace

extern "C" {

int ll_weights_save(const char *path, const ll_net_desc *net, const void *const *W, const float *const *b,
                    const float *const *scales)
{
    int rc = check_desc(net);
    if (rc)
        return rc;
    if (!path || !W) {
        llh::set_error("weights: path and W are required");
        return LL_ERR_INVALID_ARG;
    }
    const int wt = net->layers[0].wtype;
    if (wt == LL_W_I8 && !scales) {
        llh::set_error("weights: an int8 net needs its scales");
        return LL_ERR_INVALID_ARG;
    }
    File file;
    file.f = fopen(path, "wb");
    if (!file.f) {
        llh::set_error("weights: cannot open %s for writing", path);
        return LL_ERR_INVALID_ARG;
    }
    const uint32_t flags = (b ? 1u : 0u) | (wt == LL_W_I8 ? 2u : 0u);
    const uint32_t hdr[8] = {kMagic, kVersion, (uint32_t)net->n_layers, (uint32_t)wt, (uint32_t)net->max_batch,
                             flags, 0u, 0u};
    bool ok = fwrite(hdr, sizeof(hdr), 1, file.f) == 1;
    for (int l = 0; l < net->n_layers && ok; ++l) {
        const uint32_t ld[4] = {(uint32_t)net->layers[l].in_dim, (uint32_t)net->layers[l].out_dim,
                                (uint32_t)net->layers[l].act, 0u};
        ok = fwrite(ld, sizeof(ld), 1, file.f) == 1;
    }
    Fnv fnv;
    static const uint8_t zeros[64] = {0};
    auto section = [&](const void *p, size_t n) {
        if (!ok)
            return;
        if (n && (!p || fwrite(p, n, 1, file.f) != 1)) {
            ok = false;
            return;
        }
        fnv.add(p, n);
        const size_t pad = llh::round_up(n, 64) - n;
        if (pad) {
            ok = fwrite(zeros, pad, 1, file.f) == 1;
            fnv.add(zeros, pad);
        }
    };
    for (int l = 0; l < net->n_layers && ok; ++l) {
        const ll_layer_desc &d = net->layers[l];
        if (!W[l]) {
            llh::set_error("weights: layer %d weights are NULL", l);
            return LL_ERR_INVALID_ARG;
        }
        section(W[l], (size_t)d.out_dim * d.in_dim * esize(wt));
        if (b) {
            std::vector<float> zb;
            const float *bl = b[l];
            if (!bl) {
                zb.assign((size_t)d.out_dim, 0.0f);
                bl = zb.data();
            }
            section(bl, sizeof(float) * (size_t)d.out_dim);
        }
        if (wt == LL_W_I8) {
            if (!scales[l]) {
                llh::set_error("weights: layer %d scales are NULL", l);
                return LL_ERR_INVALID_ARG;
            }
            section(scales[l], sizeof(float) * (size_t)d.out_dim);
        }
    }
    if (ok)
        ok = fwrite(&fnv.h, sizeof(fnv.h), 1, file.f) == 1;
    if (!ok) {
        llh::set_error("weights: write to %s failed", path);
        return LL_ERR_INVALID_ARG;
    }
    return LL_OK;
}

int ll_weights_load(const char *path, ll_weights **out)
{
    if (!path || !out) {
        llh::set_error("weights: path and out are required");
        return LL_ERR_INVALID_ARG;
    }
    *out = nullptr;
    File file;
    file.f = fopen(path, "rb");
    if (!file.f) {
        llh::set_error("weights: cannot open %s", path);
        return LL_ERR_INVALID_ARG;
    }
    uint32_t hdr[8];
    if (fread(hdr, sizeof(hdr), 1, file.f) != 1 || hdr[0] != kMagic) {
        llh::set_error("weights: %s is not a weight file", path);
        return LL_ERR_BAD_DESC;
    }
    if (hdr[1] != kVersion) {
        llh::set_error("weights: %s has version %u (this library reads %u)", path, hdr[1], kVersion);
        return LL_ERR_UNSUPPORTED;
    }
    auto w = std::make_unique<ll_weights>();
    const int n = (int)hdr[2], wt = (int)hdr[3];
    if (n < 1 || n > 1024) {
        llh::set_error("weights: %s declares %d layers", path, n);
        return LL_ERR_BAD_DESC;
    }
    w->layers.resize((size_t)n);
    for (int l = 0; l < n; ++l) {
        uint32_t ld[4];
        if (fread(ld, sizeof(ld), 1, file.f) != 1) {
            llh::set_error("weights: %s is truncated (layer table)", path);
            return LL_ERR_BAD_DESC;
        }
        w->layers[l] = ll_layer_desc{(int32_t)ld[0], (int32_t)ld[1], (int32_t)ld[2], wt};
    }
    w->net = ll_net_desc{n, w->layers.data(), (int32_t)hdr[4], 0};
    int rc = check_desc(&w->net);
    if (rc)
        return rc;
    w->has_b = (hdr[5] & 1u) != 0;
    w->has_s = (hdr[5] & 2u) != 0;
    if (w->has_s != (wt == LL_W_I8)) {
        llh::set_error("weights: %s: scales flag does not match the weight type", path);
        return LL_ERR_BAD_DESC;
    }
    Fnv fnv;
    bool ok = true;
    auto section = [&](void *p, size_t nbytes) {
        if (!ok)
            return;
        const size_t total = llh::round_up(nbytes, 64);
        std::vector<uint8_t> buf(total);
        if (total && fread(buf.data(), total, 1, file.f) != 1) {
            ok = false;
            return;
        }
        fnv.add(buf.data(), total);
        std::memcpy(p, buf.data(), nbytes);
    };
    w->W.resize((size_t)n);
    w->b.resize((size_t)n);
    w->s.resize((size_t)n);
    for (int l = 0; l < n && ok; ++l) {
        const ll_layer_desc &d = w->layers[l];
        w->W[l].resize((size_t)d.out_dim * d.in_dim * esize(wt));
        section(w->W[l].data(), w->W[l].size());
        if (w->has_b) {
            w->b[l].resize((size_t)d.out_dim);
            section(w->b[l].data(), sizeof(float) * w->b[l].size());
        }
        if (w->has_s) {
            w->s[l].resize((size_t)d.out_dim);
            section(w->s[l].data(), sizeof(float) * w->s[l].size());
        }
    }
    uint64_t sum = 0;
    if (!ok || fread(&sum, sizeof(sum), 1, file.f) != 1) {
        llh::set_error("weights: %s is truncated", path);
        return LL_ERR_BAD_DESC;
    }
    if (sum != fnv.h) {
        llh::set_error("weights: %s is corrupt (checksum mismatch)", path);
        return LL_ERR_BAD_DESC;
    }
    *out = w.release();
    return LL_OK;
}

const ll_net_desc *ll_weights_net(const ll_weights *w)
{
    return w ? &w->net : nullptr;
}

int ll_weights_arrays(const ll_weights *w, const void **W, const float **b, const float **scales)
{
    if (!w || !W) {
        llh::set_error("weights: handle and W are required");
        return LL_ERR_INVALID_ARG;
    }
    for (int l = 0; l < w->net.n_layers; ++l) {
        W[l] = w->W[l].data();
        if (b)
            b[l] = w->has_b ? w->b[l].data() : nullptr;
        if (scales)
            scales[l] = w->has_s ? w->s[l].data() : nullptr;
    }
    return LL_OK;
}

void ll_weights_free(ll_weights *w)
{
    delete w;
}

}  // extern "C"
