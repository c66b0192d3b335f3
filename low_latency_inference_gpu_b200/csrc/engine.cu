// Resident MLP engine: planner, weight-image packing, launch and the C ABI
// around ll_resident_mlp_kernel (see resident_kernel.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <pthread.h>
#include <sched.h>
#include <chrono>
#include <cstring>
#include <deque>
#include <random>
#include <thread>
#include <utility>
#include <vector>

#include "common.h"
#include "engine_types.h"
#include "fast3_kernel.cuh"
#include "gemv_plan.h"
#include "resident_kernel.cuh"
#include "ring_kernel.cuh"
#include "deep_kernel.cuh"

#if defined(__x86_64__)
#include <immintrin.h>
#endif

using namespace llk;

namespace {

constexpr int kSmemLimit = 227 * 1024 - 4096;  // dynamic smem budget per CTA (static Shared + Params copy use the rest)

inline void cpu_relax()
{
#if defined(__x86_64__)
    _mm_pause();
#endif
}

int elems_per_unit(int wtype)
{
    return wtype == LL_W_F32 ? 4 : (wtype == LL_W_BF16 ? 8 : 16);
}

int wbytes(int wtype)
{
    return wtype == LL_W_F32 ? 4 : (wtype == LL_W_BF16 ? 2 : 1);
}

int pow2_floor(int v)
{
    int p = 1;
    while (p * 2 <= v)
        p *= 2;
    return p;
}

int log2i(int v)
{
    int l = 0;
    while ((1 << (l + 1)) <= v)
        ++l;
    return l;
}

// lanes per row: each lane gets >= 2 weight units when the row is long enough.
int choose_lpr_log2(int K, int wtype)
{
    const int U = K / elems_per_unit(wtype);
    const int want = std::max(1, std::min(32, U / 2));
    return log2i(pow2_floor(want));
}

struct LayerPlan {
    int mode = 0;
    int in = 0, out = 0, act = 0, wtype = 0;
    int K = 0;   // padded dot length
    int R = 0;   // rows per CTA (or OUTp for K-split)
    int Mp = 0;  // padded full width
    int in_buf = BUF_X, in_ld = 0, out_buf = BUF_X, out_ld = 0;
    int stage = 0;
};

struct PlanResult {
    int S = 1, C = 1;
    std::vector<LayerPlan> L;
    std::vector<int> stage_first, stage_last, stage_in_ld;
    std::vector<size_t> stage_image;  // bytes per CTA image of each stage
    size_t buf_floats[BUF_COUNT] = {0, 0, 0, 0, 0, 0};
    size_t smem = 0;
    std::string why;
};

size_t layer_image_bytes(const LayerPlan &l)
{
    size_t w = llh::round_up((size_t)l.R * (size_t)l.K * wbytes(l.wtype), 16);
    size_t b = llh::round_up((size_t)l.R * 4, 16);
    size_t s = l.wtype == LL_W_I8 ? b : 0;
    return w + b + s;
}

// Assign modes / buffers to layers of a stage partition and size everything.
bool build_plan(const ll_net_desc &net, int C, const std::vector<int> &bounds, bool replicate_first, PlanResult &pr)
{
    const int n = net.n_layers;
    const int S = (int)bounds.size() - 1;
    const int wt = net.layers[0].wtype;
    const int E = elems_per_unit(wt);
    const int Rq = std::max(4, E);
    const int bmax4 = (int)llh::round_up((size_t)std::max(1, net.max_batch), 4);
    pr = PlanResult();
    pr.S = S;
    pr.C = C;
    pr.L.resize(n);
    size_t x_ld_max = 0, ab_w = 0, l_w = 0, g_f = 0, st_w = 4;
    for (int s = 0; s < S; ++s) {
        const int f = bounds[s], e = bounds[s + 1] - 1;
        pr.stage_first.push_back(f);
        pr.stage_last.push_back(e);
        int cur_buf = BUF_X;
        int cur_ld = (s == 0) ? (int)llh::round_up((size_t)net.layers[0].in_dim, (size_t)E) : pr.L[f - 1].Mp;
        pr.stage_in_ld.push_back(cur_ld);
        x_ld_max = std::max(x_ld_max, (size_t)cur_ld);
        int next_ab = BUF_A;
        int local_R = 0;
        size_t img = 0;
        for (int l = f; l <= e; ++l) {
            LayerPlan &lp = pr.L[l];
            const ll_layer_desc &d = net.layers[l];
            lp.in = d.in_dim;
            lp.out = d.out_dim;
            lp.act = d.act;
            lp.wtype = wt;
            lp.stage = s;
            const bool last_stage = (s == S - 1);
            int mode;
            if (last_stage && l == e)
                mode = (e > f) ? LM_KSPLIT_GATHER : LM_ROWSPLIT_GATHER;
            else if (last_stage && l == e - 1)
                mode = LM_ROWSPLIT_LOCAL;
            else if (!last_stage && l == e)
                mode = LM_ROWSPLIT_GLOBAL;
            else if (s == 0 && l == f && replicate_first)
                mode = LM_REPLICATED;
            else
                mode = LM_ROWSPLIT_ALLGATHER;
            lp.mode = mode;
            if (mode == LM_KSPLIT_GATHER) {
                lp.K = local_R;
                lp.R = (int)llh::round_up((size_t)d.out_dim, 4);
                lp.Mp = lp.R;
                lp.in_buf = BUF_L;
                lp.in_ld = local_R;
                lp.out_buf = BUF_G;
                lp.out_ld = lp.R;
                g_f = std::max(g_f, (size_t)C * bmax4 * lp.R);
                st_w = std::max(st_w, (size_t)lp.R);
            } else {
                lp.K = cur_ld;
                lp.in_buf = cur_buf;
                lp.in_ld = cur_ld;
                if (mode == LM_REPLICATED) {
                    lp.R = (int)llh::round_up((size_t)d.out_dim, (size_t)Rq);
                    lp.Mp = lp.R;
                } else {
                    lp.R = (int)llh::round_up((size_t)llh::ceil_div(d.out_dim, C), (size_t)Rq);
                    lp.Mp = lp.R * C;
                }
                st_w = std::max(st_w, (size_t)lp.R);
                if (mode == LM_REPLICATED || mode == LM_ROWSPLIT_ALLGATHER) {
                    lp.out_buf = next_ab;
                    lp.out_ld = lp.Mp;
                    ab_w = std::max(ab_w, (size_t)lp.Mp);
                    next_ab = next_ab == BUF_A ? BUF_B : BUF_A;
                    cur_buf = lp.out_buf;
                    cur_ld = lp.Mp;
                } else if (mode == LM_ROWSPLIT_LOCAL) {
                    lp.out_buf = BUF_L;
                    lp.out_ld = lp.R;
                    local_R = lp.R;
                    l_w = std::max(l_w, (size_t)lp.R);
                } else if (mode == LM_ROWSPLIT_GATHER) {
                    lp.out_buf = BUF_G;
                    lp.out_ld = lp.Mp;
                    g_f = std::max(g_f, (size_t)bmax4 * lp.Mp);
                } else {  // GLOBAL
                    lp.out_buf = BUF_X;
                    lp.out_ld = lp.Mp;
                }
            }
            img += layer_image_bytes(lp);
        }
        pr.stage_image.push_back(img);
    }
    size_t max_img = 0;
    for (size_t v : pr.stage_image)
        max_img = std::max(max_img, v);
    // activation rows: a batch-1 net's kernel has no 4-row product path, so one row is all it
    // reads or writes (the gather buffer keeps the padded row count: its layout uses it)
    const size_t arows = net.max_batch > 1 ? (size_t)bmax4 : 1;
    pr.buf_floats[BUF_X] = arows * x_ld_max;
    pr.buf_floats[BUF_A] = arows * ab_w;
    pr.buf_floats[BUF_B] = arows * ab_w;
    pr.buf_floats[BUF_L] = arows * l_w;
    pr.buf_floats[BUF_G] = g_f;
    pr.buf_floats[BUF_STAGE] = arows * st_w;
    size_t total = llh::round_up(max_img, 128);
    for (int i = 0; i < BUF_COUNT; ++i)
        total += llh::round_up(std::max<size_t>(pr.buf_floats[i], 4) * 4, 128);
    pr.smem = total;
    return total <= (size_t)kSmemLimit;
}

// Greedy partition of layers into stages so each CTA image fits.
bool plan_net(const ll_net_desc &net, int C, int replicate_opt, int min_stages, int max_stages, PlanResult &out)
{
    const int n = net.n_layers;
    for (int S = std::max(1, min_stages); S <= std::min(max_stages, n); ++S) {
        // balanced contiguous split by weight bytes
        std::vector<double> wsz(n);
        double tot = 0;
        for (int l = 0; l < n; ++l) {
            wsz[l] = (double)net.layers[l].in_dim * net.layers[l].out_dim * wbytes(net.layers[l].wtype);
            tot += wsz[l];
        }
        std::vector<int> bounds = {0};
        double acc = 0;
        int s = 1;
        for (int l = 0; l < n && s < S; ++l) {
            acc += wsz[l];
            const int remaining_layers = n - (l + 1);
            const int remaining_stages = S - s;
            if ((acc >= tot * s / S && remaining_layers >= remaining_stages) || remaining_layers == remaining_stages) {
                bounds.push_back(l + 1);
                ++s;
            }
        }
        bounds.push_back(n);
        if ((int)bounds.size() != S + 1)
            continue;
        // the last stage needs >= 1 layer; a K-split tail needs 2 (else row-split gather)
        const int n0 = bounds[1] - bounds[0];
        bool rep;
        if (replicate_opt == 1)
            rep = n0 >= 3 || (S > 1 && n0 >= 2);
        else if (replicate_opt == 0)
            rep = false;
        else {
            const double first_bytes = (double)net.layers[0].in_dim * net.layers[0].out_dim * wbytes(net.layers[0].wtype);
            rep = (n0 >= 3) && first_bytes <= 72.0 * 1024;
        }
        PlanResult pr;
        if (build_plan(net, C, bounds, rep, pr)) {
            out = pr;
            return true;
        }
        if (rep && build_plan(net, C, bounds, false, pr)) {
            out = pr;
            return true;
        }
    }
    return false;
}

// Pack the shared-memory image of CTA `rank` of stage `s` (dst == nullptr: offsets only).
void pack_image(const ll_net_desc &net, const PlanResult &pr, int s, int rank, const void *const *W,
                const float *const *b, const float *const *scales, uint8_t *dst, std::vector<uint32_t> &w_off,
                std::vector<uint32_t> &b_off, std::vector<uint32_t> &s_off)
{
    (void)net;
    size_t off = 0;
    for (int l = pr.stage_first[s]; l <= pr.stage_last[s]; ++l) {
        const LayerPlan &lp = pr.L[l];
        const int wb = wbytes(lp.wtype);
        const size_t wsz = llh::round_up((size_t)lp.R * lp.K * wb, 16);
        const size_t bsz = llh::round_up((size_t)lp.R * 4, 16);
        const bool has_s = lp.wtype == LL_W_I8;
        w_off[l] = (uint32_t)off;
        b_off[l] = (uint32_t)(off + wsz);
        s_off[l] = has_s ? (uint32_t)(off + wsz + bsz) : 0xffffffffu;
        if (dst) {
            uint8_t *wdst = dst + off;
            std::memset(wdst, 0, wsz);
            float *bdst = reinterpret_cast<float *>(dst + off + wsz);
            std::memset(bdst, 0, bsz);
            float *sdst = has_s ? reinterpret_cast<float *>(dst + off + wsz + bsz) : nullptr;
            if (sdst)
                std::memset(sdst, 0, bsz);
            const uint8_t *src = static_cast<const uint8_t *>(W[l]);
            for (int r = 0; r < lp.R; ++r) {
                int grow;  // global output row
                int col0;  // first global input column of this slice
                if (lp.mode == LM_KSPLIT_GATHER) {
                    grow = r;
                    col0 = rank * lp.K;
                } else if (lp.mode == LM_REPLICATED) {
                    grow = r;
                    col0 = 0;
                } else {
                    grow = rank * lp.R + r;
                    col0 = 0;
                }
                if (grow >= lp.out)
                    continue;
                for (int k = 0; k < lp.K; ++k) {
                    const int gk = col0 + k;
                    if (gk >= lp.in)
                        break;
                    std::memcpy(wdst + ((size_t)r * lp.K + k) * wb, src + ((size_t)grow * lp.in + gk) * wb, wb);
                }
                bdst[r] = b && b[l] ? b[l][grow] : 0.0f;
                if (sdst)
                    sdst[r] = scales && scales[l] ? scales[l][grow] : 1.0f;
            }
        }
        off += wsz + bsz + (has_s ? bsz : 0);
    }
}

// Register-resident kernels compiled for specific 3-layer shapes.
struct Fast3Entry {
    int in, h1, h2, out, C;
    const void *fn;
    int K1, K2, K3, NB;
    int S1, S2, R2;
    int rows;  // rows one pass carries (micro-batching)
    const void *ring_fn;  // pipelined ring kernel of the shape (variant 4), or null
    int ring_smem;        // its dynamic shared memory (bytes)
};

template <int IN, int H1, int H2, int OUT, int C>
Fast3Entry fast3_entry()
{
    using S = Fast3Shape<IN, H1, H2, OUT, C>;
    const void *ring = nullptr;
    int ring_smem = 0;
    if constexpr (S::MaxRows == kFast3Rows) {
        ring = reinterpret_cast<const void *>(&ll_ring_kernel<IN, H1, H2, OUT, C>);
        ring_smem = RingPool<IN, H1, H2, OUT, C>::BYTES;
    }
    return Fast3Entry{IN, H1, H2, OUT, C, reinterpret_cast<const void *>(&ll_fast3_kernel<IN, H1, H2, OUT, C>),
                      S::K1, S::K2, S::K3, S::NB, S::S1, S::S2, S::R2, S::MaxRows, ring, ring_smem};
}

const Fast3Entry *find_fast3(const ll_net_desc &net, int C)
{
    // first match wins when the cluster size is automatic: 8 CTAs (fewer weights per
    // thread, measured ~0.1 us lower p50 than 4 on B200), 4 when asked for
    static const Fast3Entry table[] = {
        fast3_entry<64, 256, 256, 16, 8>(),  // fp32 64->256->256->16 (the batch-1 latency workload)
        fast3_entry<64, 256, 256, 16, 4>(),
    };
    if (net.n_layers != 3 || net.max_batch != 1 || net.layers[0].wtype != LL_W_F32)
        return nullptr;
    for (const Fast3Entry &e : table) {
        if (e.in == net.layers[0].in_dim && e.h1 == net.layers[0].out_dim && e.h2 == net.layers[1].out_dim &&
            e.out == net.layers[2].out_dim && (C == 0 || C == e.C))
            return &e;
    }
    return nullptr;
}

// Per-CTA image of the register-resident kernel: [NW][kThreads] weights (thread-minor, so the
// one-time load is coalesced), then biases b1[H1], this CTA's b2 rows, b3[OUT].
std::vector<uint8_t> pack_fast3(const Fast3Entry &f, const void *const *W, const float *const *b, size_t &stride)
{
    const int T = kThreads, NW = f.K1 + f.K2 + f.K3;
    stride = llh::round_up(((size_t)NW * T + f.NB) * 4, 256);
    std::vector<uint8_t> img((size_t)f.C * stride, 0);
    const float *W1 = static_cast<const float *>(W[0]);
    const float *W2 = static_cast<const float *>(W[1]);
    const float *W3 = static_cast<const float *>(W[2]);
    for (int c = 0; c < f.C; ++c) {
        float *o = reinterpret_cast<float *>(img.data() + (size_t)c * stride);
        // weight j of a thread pairs with input element 4*(s + S*(j/4)) + j%4 (16-byte pieces
        // interleaved across the S lanes of a row group); layer 3: local row lane + 32*j
        for (int t = 0; t < T; ++t) {
            const int r1 = t / f.S1, s1 = t % f.S1;
            for (int j = 0; j < f.K1; ++j)
                o[(size_t)j * T + t] = W1[(size_t)r1 * f.in + 4 * (s1 + f.S1 * (j / 4)) + j % 4];
            const int g2 = c * f.R2 + t / f.S2, s2 = t % f.S2;
            for (int j = 0; j < f.K2; ++j)
                o[(size_t)(f.K1 + j) * T + t] = W2[(size_t)g2 * f.h1 + 4 * (s2 + f.S2 * (j / 4)) + j % 4];
            const int w = t / 32, lane = t % 32;
            for (int j = 0; j < f.K3; ++j)
                o[(size_t)(f.K1 + f.K2 + j) * T + t] =
                    w < f.out ? W3[(size_t)w * f.h2 + c * f.R2 + lane + 32 * j] : 0.0f;
        }
        float *bo = o + (size_t)NW * T;
        for (int i = 0; i < f.h1; ++i)
            bo[i] = b && b[0] ? b[0][i] : 0.0f;
        for (int i = 0; i < f.R2; ++i)
            bo[f.h1 + i] = b && b[1] ? b[1][c * f.R2 + i] : 0.0f;
        for (int i = 0; i < f.out; ++i)
            bo[f.h1 + f.R2 + i] = b && b[2] ? b[2][i] : 0.0f;
    }
    return img;
}

// Per-CTA image of the pipelined ring kernel (CTA c), [NW][kThreads] weights then the register-
// resident image's biases (b1[H1], this CTA's b2 rows, b3[OUT]); thread t = (warp w, lane l):
//   layer 1, one-row pass: 4 q + e  ->  W1[32 q + 2 w + (l >> 4)][4 (l & 15) + e], q < H1 / 32;
//   layer 1, split pass:   4 i + e  ->  W1[c R1 + 2 w + i][4 (l & 15) + e], i < 2;
//   layer 2: 2 local rows x the h1 pieces l, l + 32, ... (one row pair per warp), as ring_layers.cuh
//            reads them;
//   layer 3: as in the register-resident image (warp w = output w, local rows l + 32 j).
std::vector<uint8_t> pack_ring(const Fast3Entry &f, const void *const *W, const float *const *b, size_t &stride)
{
    constexpr int RB2 = 2;
    const int T = kThreads;
    const int Q1 = f.h1 / 32, K1 = 4 * Q1, K1S = 8, R1 = f.h1 / f.C;
    const int L2 = 32, P2 = f.h1 / 4 / L2, K2 = RB2 * 4 * P2;
    const int NW = K1 + K1S + K2 + f.K3;
    if (f.in != 64 || T != 512 || f.h1 % 32 != 0 || R1 != 2 * (T / 32) || f.R2 != RB2 * (T / 32) || K2 != f.K2) {
        llh::set_error("ring image: the shape does not fit the blocked layers");
        return {};
    }
    stride = llh::round_up(((size_t)NW * T + f.NB) * 4, 256);
    std::vector<uint8_t> img((size_t)f.C * stride, 0);
    const float *W1 = static_cast<const float *>(W[0]);
    const float *W2 = static_cast<const float *>(W[1]);
    const float *W3 = static_cast<const float *>(W[2]);
    for (int c = 0; c < f.C; ++c) {
        float *o = reinterpret_cast<float *>(img.data() + (size_t)c * stride);
        for (int t = 0; t < T; ++t) {
            const int w = t / 32, l = t % 32, s = l & 15;
            for (int q = 0; q < Q1; ++q)
                for (int e = 0; e < 4; ++e)
                    o[(size_t)(4 * q + e) * T + t] = W1[(size_t)(32 * q + 2 * w + (l >> 4)) * f.in + 4 * s + e];
            for (int i = 0; i < 2; ++i)
                for (int e = 0; e < 4; ++e)
                    o[(size_t)(K1 + 4 * i + e) * T + t] = W1[(size_t)(c * R1 + 2 * w + i) * f.in + 4 * s + e];
            for (int r = 0; r < RB2; ++r)
                for (int p = 0; p < P2; ++p)
                    for (int e = 0; e < 4; ++e)
                        o[(size_t)(K1 + K1S + r * 4 * P2 + 4 * p + e) * T + t] =
                            W2[(size_t)(c * f.R2 + RB2 * w + r) * f.h1 + 4 * (l + L2 * p) + e];
            for (int j = 0; j < f.K3; ++j)
                o[(size_t)(K1 + K1S + K2 + j) * T + t] = w < f.out ? W3[(size_t)w * f.h2 + c * f.R2 + l + 32 * j] : 0.0f;
        }
        float *bo = o + (size_t)NW * T;
        for (int i = 0; i < f.h1; ++i)
            bo[i] = b && b[0] ? b[0][i] : 0.0f;
        for (int i = 0; i < f.R2; ++i)
            bo[f.h1 + i] = b && b[1] ? b[1][c * f.R2 + i] : 0.0f;
        for (int i = 0; i < f.out; ++i)
            bo[f.h1 + f.R2 + i] = b && b[2] ? b[2][i] : 0.0f;
    }
    return img;
}

// Register-resident kernels compiled for deep nets of one hidden width (IN -> H x (NL-1) -> OUT).
struct DeepEntry {
    int wt, in, h, out, nl, C, lps;
    const void *fn;
    int NW, NB, NS, RPW, RL, OPW;
};

template <int WT, int IN, int H, int OUT, int NL, int C, int LPS>
DeepEntry deep_entry()
{
    using D = DeepShape<WT, IN, H, OUT, NL, C, LPS>;
    return DeepEntry{WT,   IN,   H,    OUT,   NL,    C,     LPS,  reinterpret_cast<const void *>(&ll_deep_kernel<WT, IN, H, OUT, NL, C, LPS>),
                     D::NW, D::NB, D::NS, D::RPW, D::RL, D::OPW};
}

const DeepEntry *find_deep(const ll_net_desc &net, int C)
{
    static const DeepEntry table[] = {
        deep_entry<LL_W_F32, 128, 512, 32, 10, 16, 2>(),   // 128 -> 512 x 9 -> 32 on 5 clusters of 16
        deep_entry<LL_W_BF16, 256, 1024, 64, 6, 16, 1>(),  // 256 -> 1024 x 5 -> 64 on 5 clusters of 16
    };
    if (net.max_batch != 1)
        return nullptr;
    for (const DeepEntry &e : table) {
        if (net.n_layers != e.nl || (C != 0 && C != e.C))
            continue;
        bool match = true;
        for (int l = 0; l < e.nl && match; ++l) {
            const ll_layer_desc &d = net.layers[l];
            match = d.wtype == e.wt && d.in_dim == (l == 0 ? e.in : e.h) && d.out_dim == (l == e.nl - 1 ? e.out : e.h);
        }
        if (match)
            return &e;
    }
    return nullptr;
}

// Per-CTA image of the deep kernel (CTA = stage * C + rank): [NW][kThreads] 32-bit weight
// registers (thread-minor; fp32, or two bf16 per register: logical weight 2m in the low half of
// register m) then NB fp32 biases.  Hidden layer (KP = kin / 128 pieces per lane): warp w, lane
// l holds rows RPW w + r (global rank * R + RPW w + r), logical weight (r KP + j) 4 + e pairing
// with input element 4 (l + 32 j) + e; the last layer: logical weight o RL + j of warp w, lane l
// is W[OPW w + o][rank * R + l + 32 j].
std::vector<uint8_t> pack_deep(const DeepEntry &d, const void *const *W, const float *const *b, size_t &stride)
{
    const int T = kThreads, R = d.h / d.C, EPR = d.wt == LL_W_BF16 ? 2 : 1;
    stride = llh::round_up(((size_t)d.NW * T + d.NB) * 4, 256);
    std::vector<uint8_t> img((size_t)d.NS * d.C * stride, 0);
    // logical weight i of thread t's slice at register `off` (bf16: bit patterns, two per register)
    auto put = [&](uint32_t *o, int off, int i, int t, const void *Wl, size_t idx) {
        uint32_t &reg = o[(size_t)(off + i / EPR) * T + t];
        if (EPR == 1) {
            std::memcpy(&reg, static_cast<const float *>(Wl) + idx, 4);
        } else {
            const uint32_t h = static_cast<const uint16_t *>(Wl)[idx];
            reg |= (i & 1) ? h << 16 : h;
        }
    };
    for (int st = 0; st < d.NS; ++st) {
        const int l0 = st * d.lps, l1 = st == d.NS - 1 ? d.nl - 1 : (st + 1) * d.lps - 1;
        for (int c = 0; c < d.C; ++c) {
            uint32_t *o = reinterpret_cast<uint32_t *>(img.data() + ((size_t)st * d.C + c) * stride);
            float *bo = reinterpret_cast<float *>(o + (size_t)d.NW * T);
            int woff = 0, boff = 0;
            for (int l = l0; l <= l1; ++l) {
                const int kin = l == 0 ? d.in : d.h;
                if (l == d.nl - 1) {
                    for (int t = 0; t < T; ++t)
                        for (int q = 0; q < d.OPW; ++q)
                            for (int j = 0; j < d.RL; ++j)
                                put(o, woff, q * d.RL + j, t, W[l],
                                    (size_t)(d.OPW * (t / 32) + q) * kin + c * R + t % 32 + 32 * j);
                    for (int i = 0; i < d.out; ++i)
                        bo[boff + i] = b && b[l] ? b[l][i] : 0.0f;
                    woff += d.OPW * d.RL / EPR;
                    boff += d.out;
                } else {
                    const int KP = kin / 128;
                    if (R != d.RPW * (T / 32) || kin % 128 != 0) {
                        llh::set_error("deep kernel image: %d rows per warp and 16-byte pieces per lane", d.RPW);
                        return {};
                    }
                    for (int t = 0; t < T; ++t) {
                        const int wp = t / 32, ln = t % 32;
                        for (int r = 0; r < d.RPW; ++r)
                            for (int j = 0; j < KP; ++j)
                                for (int e = 0; e < 4; ++e)
                                    put(o, woff, (r * KP + j) * 4 + e, t, W[l],
                                        (size_t)(c * R + d.RPW * wp + r) * kin + 4 * (ln + 32 * j) + e);
                    }
                    for (int i = 0; i < R; ++i)
                        bo[boff + i] = b && b[l] ? b[l][c * R + i] : 0.0f;
                    woff += d.RPW * KP * 4 / EPR;
                    boff += R;
                }
            }
            if (woff > d.NW || boff > d.NB) {
                llh::set_error("deep kernel image: stage %d needs %d weight registers / %d biases per thread / CTA",
                               st, woff, boff);
                return {};
            }
        }
    }
    return img;
}

}  // namespace

struct ll_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    Params base{};
    bool echo = false;
    int in_dim = 0, out_dim = 0, max_batch = 1;
    int grid = 1;
    PlanResult plan;
    void *mb_host = nullptr;
    ll_tick_header *mb_dev = nullptr;
    size_t mb_bytes = 0;
    int wc = 0;
    EngineCtrl *ctrl_host = nullptr;
    EngineCtrl *ctrl_dev = nullptr;
    uint8_t *d_image = nullptr;
    float *d_xfer = nullptr;
    unsigned *d_words = nullptr;  // [kMaxStages] cnt, [2*kMaxStages] hdr, abort, q_done
    uint32_t seq = 0;
    // requests posted and not yet collected, oldest first: (seq, ring index); the
    // tagged ring holds up to `ring` of them, the TickBuffer one
    std::deque<std::pair<uint32_t, uint64_t>> inflight;
    int ring = 1;           // tagged ring slots
    size_t ring_xstride = 0; // bytes between the x chunks of consecutive slots (contiguous)
    size_t ring_ystride = 0; // bytes between the y chunks of consecutive slots (64-byte aligned)
    size_t ring_ybase = 0;   // byte offset of slot 0's y chunks
    uint64_t ring_next = 0; // ring index of the next request to post
    uint32_t last_served = 0;
    bool running = false;
    int launches = 0;
    int last_status = LL_OK;
    ll_engine_opts opts{};
    bool attrs_set = false;
    const void *kfn = nullptr;  // kernel launched (generic or register-resident)
    int variant = 1;
    int micro = 1;      // ring slots the device may take together
    int micro_max = 1;  // rows the kernel can carry in one pass
    // kernel variant 3 (resident small-batch kernel, one CTA per SM, weights in shared memory)
    GemvNetParams gv{};            // fields fixed at create time
    GemvLayout gl;
    int gv_bp = 1;                 // batch rows of the instantiation (gemv_bp(max_batch))
    int gv_smem = 0;               // dynamic shared memory per CTA
    uint8_t *gv_img = nullptr;     // per-CTA images
    uint32_t *gv_hand[2] = {};     // tagged hand-off words [4][widest layer]
    __nv_bfloat16 *gv_act[2] = {}; // counted hand-off rows [32][widest layer]
    unsigned *gv_cnt = nullptr;    // arrival counters, one 128-byte line per layer
    float *gv_relay = nullptr;     // x rows of the current request [32][in]
    float *gv_gather = nullptr;    // last layer's outputs [32][out]
    unsigned long long *gv_req = nullptr;  // request word
    unsigned *gv_status = nullptr;
    size_t gv_hand_bytes = 0, gv_act_bytes = 0;
    uint32_t passes = 0, rows = 0;  // summed over exited launches
    int weight_regs = 0;
};

extern "C" void ll_engine_opts_default(ll_engine_opts *o)
{
    std::memset(o, 0, sizeof(*o));
    o->cluster_size = 0;
    o->replicate_first = -1;
    o->write_combined = 0;
    o->mailbox_format = 0;
    o->idle_timeout_ns = 30ull * 1000 * 1000 * 1000;
    o->step_timeout_ns = 200ull * 1000 * 1000;
    o->max_stages = 0;
}

namespace {

int validate_net(const ll_net_desc *net, const void *const *W)
{
    if (!net || net->n_layers < 1 || net->n_layers > kMaxLayers || !net->layers) {
        llh::set_error("net descriptor: n_layers must be in [1, %d]", kMaxLayers);
        return LL_ERR_BAD_DESC;
    }
    if (net->max_batch < 1 || net->max_batch > 64) {
        llh::set_error("net descriptor: max_batch must be in [1, 64]");
        return LL_ERR_BAD_DESC;
    }
    const int wt = net->layers[0].wtype;
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        if (d.in_dim < 1 || d.out_dim < 1 || d.in_dim > 16384 || d.out_dim > 16384) {
            llh::set_error("layer %d: dims out of range", l);
            return LL_ERR_BAD_DESC;
        }
        if (l > 0 && net->layers[l - 1].out_dim != d.in_dim) {
            llh::set_error("layer %d: in_dim %d != previous out_dim %d", l, d.in_dim, net->layers[l - 1].out_dim);
            return LL_ERR_BAD_DESC;
        }
        if (d.act < LL_ACT_IDENTITY || d.act > LL_ACT_GELU) {
            llh::set_error("layer %d: unknown activation %d", l, d.act);
            return LL_ERR_BAD_DESC;
        }
        if (d.wtype != wt || wt < LL_W_F32 || wt > LL_W_I8) {
            llh::set_error("layer %d: all layers must share one valid weight type", l);
            return LL_ERR_BAD_DESC;
        }
        if (W && !W[l]) {
            llh::set_error("layer %d: weight pointer is NULL", l);
            return LL_ERR_INVALID_ARG;
        }
    }
    return LL_OK;
}

int alloc_mailbox(ll_engine *e)
{
    if (e->opts.mailbox_format == 1) {
        if (e->max_batch != 1 || e->in_dim > 384 || e->out_dim > 96 || e->in_dim < 1 || e->out_dim < 1) {
            llh::set_error("tagged mailbox (format 1) needs batch 1, 1 <= in_dim <= 384, 1 <= out_dim <= 96");
            return LL_ERR_UNSUPPORTED;
        }
    } else if (e->opts.mailbox_format != 0) {
        llh::set_error("unknown mailbox format %d", e->opts.mailbox_format);
        return LL_ERR_INVALID_ARG;
    }
    e->ring = e->opts.ring_slots < 1 ? 1 : e->opts.ring_slots;
    if (e->ring > 1 && (e->opts.mailbox_format != 1 || e->ring > 64)) {
        llh::set_error("a request ring (ring_slots %d) needs the tagged mailbox and at most 64 slots", e->ring);
        return LL_ERR_UNSUPPORTED;
    }
    e->micro = e->opts.micro_batch < 1 ? 1 : e->opts.micro_batch;
    if (e->micro > 1) {
        // the multi-slot read holds whole slots in the registers of up to kTagReadWarpsMax warps
        const int nxc = (e->in_dim + 2) / 3;
        const int rpw = tag_rows_per_warp(nxc);
        const int warps = rpw > 0 ? (e->micro + rpw - 1) / rpw : kTagReadWarpsMax + 1;
        if (e->opts.mailbox_format != 1 || e->micro > e->ring || e->micro > e->micro_max ||
            warps > kTagReadWarpsMax) {
            llh::set_error("micro_batch %d needs the tagged mailbox, at most ring_slots (%d), at most the rows "
                           "the kernel carries (%d: the register-resident kernel of a shape with room for "
                           "%d), and whole slots in at most %d reading warps (%d slot(s) per warp here)",
                           e->micro, e->ring, e->micro_max, kFast3Rows, kTagReadWarpsMax, rpw);
            return LL_ERR_UNSUPPORTED;
        }
    }
    if (e->opts.mailbox_format == 1) {
        // header, the x chunks of every slot back to back (a pass that takes several waiting
        // requests reads one contiguous run: measured ~2x faster over PCIe than slots 512 bytes
        // apart), then from a 64-byte boundary the y chunks, each slot's on its own lines.
        // One slot is exactly the single tagged mailbox (ll_tagged_mailbox_bytes).
        e->ring_xstride = 16 * (size_t)((e->in_dim + 2) / 3);
        e->ring_ystride = llh::round_up(16 * (size_t)((e->out_dim + 2) / 3), 64);
        e->ring_ybase = llh::round_up(sizeof(ll_tick_header) + e->ring_xstride * (size_t)e->ring, 64);
        e->mb_bytes = llh::round_up(e->ring_ybase + e->ring_ystride * (size_t)e->ring, 64);
    } else {
        e->mb_bytes = ll_mailbox_bytes(e->in_dim, e->out_dim, e->max_batch);
    }
    unsigned flags = cudaHostAllocMapped | cudaHostAllocPortable;
    if (e->wc)
        flags |= cudaHostAllocWriteCombined;
    LL_CUDA_TRY(cudaHostAlloc(&e->mb_host, e->mb_bytes, flags));
    std::memset(e->mb_host, 0, e->mb_bytes);
    LL_CUDA_TRY(cudaHostGetDevicePointer((void **)&e->mb_dev, e->mb_host, 0));
    LL_CUDA_TRY(cudaHostAlloc((void **)&e->ctrl_host, sizeof(EngineCtrl), cudaHostAllocMapped | cudaHostAllocPortable));
    std::memset((void *)e->ctrl_host, 0, sizeof(EngineCtrl));
    LL_CUDA_TRY(cudaHostGetDevicePointer((void **)&e->ctrl_dev, (void *)e->ctrl_host, 0));
    return LL_OK;
}

// Shared-memory layout and per-stage tables (no CUDA).
void layout_buffers(Params &p, const PlanResult &pr, int in_dim, int out_dim, int max_batch)
{
    p.C = pr.C;
    p.n_stages = pr.S;
    p.in_dim = in_dim;
    p.out_dim = out_dim;
    p.max_batch = max_batch;
    p.bmax4 = (int)llh::round_up((size_t)max_batch, 4);
    p.in_ld = pr.stage_in_ld.empty() ? (int)llh::round_up((size_t)std::max(in_dim, 1), 4) : pr.stage_in_ld[0];
    for (int s = 0; s < kMaxStages; ++s) {
        p.stage_first[s] = s < pr.S && !pr.stage_first.empty() ? pr.stage_first[s] : 0;
        p.stage_last[s] = s < pr.S && !pr.stage_last.empty() ? pr.stage_last[s] : -1;
        p.stage_in_ld[s] = s < (int)pr.stage_in_ld.size() ? pr.stage_in_ld[s] : p.in_ld;
        p.image_bytes[s] = s < (int)pr.stage_image.size() ? (uint32_t)pr.stage_image[s] : 0u;
    }
    size_t max_img = 0;
    for (size_t v : pr.stage_image)
        max_img = std::max(max_img, v);
    size_t off = llh::round_up(max_img, 128);
    for (int i = 0; i < BUF_COUNT; ++i) {
        p.buf_off[i] = (uint32_t)off;
        off += llh::round_up(std::max<size_t>(pr.buf_floats[i], 4) * 4, 128);
    }
    p.smem_bytes = (uint32_t)off;
}

int finish_setup(ll_engine *e)
{
    const PlanResult &pr = e->plan;
    Params &p = e->base;
    e->grid = pr.S * pr.C;
    p.mb = e->mb_dev;
    p.mb_x = reinterpret_cast<const float *>(reinterpret_cast<const char *>(e->mb_dev) + sizeof(ll_tick_header));
    if (e->opts.mailbox_format == 1)
        p.mb_y = reinterpret_cast<float *>(reinterpret_cast<char *>(e->mb_dev) + e->ring_ybase);
    else
        p.mb_y = reinterpret_cast<float *>(reinterpret_cast<char *>(e->mb_dev) + sizeof(ll_tick_header) +
                                       sizeof(float) * (size_t)e->in_dim * e->max_batch);
    p.ctrl = e->ctrl_dev;
    p.mailbox_format = e->opts.mailbox_format;
    p.ring_slots = e->ring;
    p.ring_xstride_f = (uint32_t)(e->ring_xstride / 4);
    p.ring_ystride_f = (uint32_t)(e->ring_ystride / 4);
    p.ring_base = 0;
    p.micro_batch = e->micro;
    p.idle_ns = e->opts.idle_timeout_ns;
    p.step_ns = e->opts.step_timeout_ns;
    p.peer_margin_ns = 2ull * 1000 * 1000 * 1000;
    p.diag_wait_never = e->opts.diag_wait_never;
    // device words
    LL_CUDA_TRY(cudaMalloc((void **)&e->d_words, sizeof(unsigned) * (4 * kMaxStages + 8)));
    p.xfer_cnt = e->d_words;
    p.xfer_hdr = e->d_words + kMaxStages;
    p.abort_flag = e->d_words + 3 * kMaxStages;
    p.q_done = e->d_words + 3 * kMaxStages + 1;
    if (pr.S > 1) {
        size_t stride = 0;
        for (int l = 0; l < (int)pr.L.size(); ++l)
            if (pr.L[l].mode == LM_ROWSPLIT_GLOBAL)
                stride = std::max(stride, (size_t)p.bmax4 * pr.L[l].Mp);
        stride = llh::round_up(stride, 64);
        LL_CUDA_TRY(cudaMalloc((void **)&e->d_xfer, sizeof(float) * stride * pr.S));
        LL_CUDA_TRY(cudaMemset(e->d_xfer, 0, sizeof(float) * stride * pr.S));
        p.xfer = e->d_xfer;
        p.xfer_stride = (uint32_t)stride;
        // batch 1: 64-bit tagged words (Mp of them fit: the region holds bmax4 = 4 rows of floats)
        p.xfer_tagged = e->max_batch == 1 ? 1 : 0;
    }
    LL_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    return LL_OK;
}

// The generic kernel's instantiation for a plan: by the net's weight type, and without the
// 4-row product path for batch-1 nets.
const void *generic_kernel_for(const Params &p)
{
    const bool batched = p.max_batch > 1;
    const int wt = p.n_layers > 0 ? p.L[0].wtype : LL_W_F32;
    if (wt == LL_W_BF16)
        return batched ? reinterpret_cast<const void *>(&ll_resident_mlp_kernel<LL_W_BF16, true>)
                       : reinterpret_cast<const void *>(&ll_resident_mlp_kernel<LL_W_BF16, false>);
    if (wt == LL_W_I8)
        return batched ? reinterpret_cast<const void *>(&ll_resident_mlp_kernel<LL_W_I8, true>)
                       : reinterpret_cast<const void *>(&ll_resident_mlp_kernel<LL_W_I8, false>);
    return batched ? reinterpret_cast<const void *>(&ll_resident_mlp_kernel<LL_W_F32, true>)
                   : reinterpret_cast<const void *>(&ll_resident_mlp_kernel<LL_W_F32, false>);
}

int set_kernel_attrs(ll_engine *e)
{
    if (e->attrs_set)
        return LL_OK;
    if (!e->kfn)
        e->kfn = generic_kernel_for(e->base);
    if (e->base.smem_bytes > 0)
        LL_CUDA_TRY(cudaFuncSetAttribute(e->kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)e->base.smem_bytes));
    if (e->base.C > 8)
        LL_CUDA_TRY(cudaFuncSetAttribute(e->kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    e->attrs_set = true;
    return LL_OK;
}

// Kernel variant 3: one cooperative launch of the resident small-batch kernel over every
// SM; its tags, counters and request word restart from zero at each launch.
int launch_gemv(ll_engine *e, const Params &p)
{
    if (p.mode == MODE_QUEUE &&
        (reinterpret_cast<uintptr_t>(p.q_x) % 16 != 0 || reinterpret_cast<uintptr_t>(p.q_y) % 16 != 0)) {
        llh::set_error("queue buffers must be 16-byte aligned");
        return LL_ERR_INVALID_ARG;
    }
    for (int i = 0; i < 2; ++i)
        LL_CUDA_TRY(cudaMemsetAsync(e->gv_hand[i], 0, e->gv_hand_bytes, e->stream));
    LL_CUDA_TRY(cudaMemsetAsync(e->gv_cnt, 0, sizeof(unsigned) * kGvCntStride * (size_t)e->gv.n_layers, e->stream));
    LL_CUDA_TRY(cudaMemsetAsync(e->gv_req, 0, sizeof(unsigned long long), e->stream));
    LL_CUDA_TRY(cudaMemsetAsync(e->gv_status, 0, sizeof(unsigned), e->stream));
    GemvNetParams g = e->gv;
    g.n_rows = 1;
    GemvResident &r = g.res;
    r.mb = p.mb;
    r.mb_x = p.mb_x;
    r.mb_y = p.mb_y;
    r.ctrl = p.ctrl;
    r.mode = p.mode;
    r.tagged = e->opts.mailbox_format == 1 ? 1 : 0;
    r.max_rows = e->max_batch;
    r.last_seq = p.last_seq;
    r.idle_ns = p.idle_ns;
    r.peer_margin_ns = p.peer_margin_ns;
    r.q_x = p.q_x;
    r.q_y = p.q_y;
    r.q_n = p.q_n;
    r.q_rows = p.q_rows;
    r.q_stamp = p.q_stamp;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)e->grid, 1, 1);
    cfg.blockDim = dim3(kGvThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)e->gv_smem;
    cfg.stream = e->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the layers hand off across all of them
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[] = {&g};
    LL_CUDA_TRY(cudaLaunchKernelExC(&cfg, e->kfn, args));
    ++e->launches;
    return LL_OK;
}

int launch(ll_engine *e, const Params &p)
{
    int rc = set_kernel_attrs(e);
    if (rc)
        return rc;
    LL_CUDA_TRY(cudaMemsetAsync(e->d_words, 0, sizeof(unsigned) * (4 * kMaxStages + 8), e->stream));
    if (p.xfer_tagged && e->d_xfer)  // tags restart with the launch (queue mode numbers from 1)
        LL_CUDA_TRY(cudaMemsetAsync(e->d_xfer, 0, sizeof(float) * p.xfer_stride * (size_t)e->plan.S, e->stream));
    e->ctrl_host->state = ST_IDLE;
    e->ctrl_host->status = LL_OK;
    e->ctrl_host->err_where = 0;
    e->ctrl_host->exit_reason = EXIT_NONE;
    e->ctrl_host->served = p.last_seq;
    e->ctrl_host->passes = 0;
    e->ctrl_host->rows = 0;
    if (e->variant == 3)
        return launch_gemv(e, p);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)e->grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = e->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int max_clusters = 0;
    cudaError_t oe = cudaOccupancyMaxActiveClusters(&max_clusters, e->kfn, &cfg);
    if (oe != cudaSuccess || max_clusters < p.n_stages) {
        llh::set_error("resident kernel needs %d co-resident clusters of %d CTAs (%u B smem); device fits %d (%s)",
                       p.n_stages, p.C, p.smem_bytes, max_clusters, cudaGetErrorString(oe));
        cudaGetLastError();
        return LL_ERR_BAD_DESC;
    }
    void *args[] = {const_cast<Params *>(&p)};
    LL_CUDA_TRY(cudaLaunchKernelExC(&cfg, e->kfn, args));
    ++e->launches;
    return LL_OK;
}

// Collect a finished launch: returns LL_OK or LL_ERR_DEVICE_FAULT / LL_ERR_CUDA.
int reap(ll_engine *e)
{
    cudaError_t ce = cudaStreamSynchronize(e->stream);
    e->running = false;
    if (ce != cudaSuccess) {
        llh::set_error("resident kernel failed: %s", cudaGetErrorString(ce));
        e->last_status = LL_ERR_CUDA;
        return LL_ERR_CUDA;
    }
    e->last_served = static_cast<ll_tick_header *>(e->mb_host)->seq_out;
    e->passes += e->ctrl_host->passes;
    e->rows += e->ctrl_host->rows;
    if (e->ctrl_host->status != LL_OK) {
        llh::set_error("resident kernel reported status %u at location 0x%x", e->ctrl_host->status,
                       e->ctrl_host->err_where);
        e->last_status = (int)e->ctrl_host->status;
        return LL_ERR_DEVICE_FAULT;
    }
    return LL_OK;
}

int ensure_running(ll_engine *e)
{
    if (e->running) {
        if (e->ctrl_host->state != ST_EXITED)
            return LL_OK;
        int rc = reap(e);
        if (rc)
            return rc;
    }
    LL_CUDA_TRY(cudaSetDevice(e->device));
    Params p = e->base;
    p.mode = MODE_MAILBOX;
    p.last_seq = e->last_served;
    // ring position of the first request the device has not taken: just after the
    // last one it answered, else the oldest one still in flight
    p.ring_base = (uint32_t)(e->ring_next % (uint64_t)e->ring);
    if (!e->inflight.empty()) {
        uint64_t idx = e->inflight.front().second;
        for (const auto &f : e->inflight)
            if (f.first == e->last_served)
                idx = f.second + 1;
        p.ring_base = (uint32_t)(idx % (uint64_t)e->ring);
    }
    // make sure the doorbell state is consistent: seq_out == last served
    int rc = launch(e, p);
    if (rc)
        return rc;
    e->running = true;
    // wait until the weights are resident (bounded)
    const auto t0 = std::chrono::steady_clock::now();
    while (e->ctrl_host->state < ST_RUNNING) {
        cpu_relax();
        if (cudaStreamQuery(e->stream) != cudaErrorNotReady) {
            int r2 = reap(e);
            if (r2 == LL_OK) {
                llh::set_error("resident kernel exited during start-up (exit reason %u)", e->ctrl_host->exit_reason);
                return LL_ERR_DEVICE_FAULT;
            }
            return r2;
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) {
            llh::set_error("resident kernel did not report ready within 10 s");
            return LL_ERR_TIMEOUT;
        }
    }
    return LL_OK;
}

int engine_common_create(ll_engine *e, const ll_engine_opts *opts)
{
    if (opts)
        e->opts = *opts;
    else
        ll_engine_opts_default(&e->opts);
    if (e->opts.idle_timeout_ns == 0)
        e->opts.idle_timeout_ns = 30ull * 1000 * 1000 * 1000;
    if (e->opts.step_timeout_ns == 0)
        e->opts.step_timeout_ns = 200ull * 1000 * 1000;
    e->wc = e->opts.write_combined;
    LL_CUDA_TRY(cudaSetDevice(e->device));
    return alloc_mailbox(e);
}

// Spin on seq_out with liveness checks; copies y.
// Format 1: true once every y chunk carries `seq` (then y is copied out).
size_t ring_slot_of(const ll_engine *e, uint32_t seq)
{
    for (const auto &f : e->inflight)
        if (f.first == seq)
            return (size_t)(f.second % (uint64_t)e->ring);
    return 0;
}

bool tagged_done(ll_engine *e, uint32_t seq, float *y)
{
    const int yc = (e->out_dim + 2) / 3;
    const char *base = static_cast<const char *>(e->mb_host) + e->ring_ybase + ring_slot_of(e, seq) * e->ring_ystride;
    uint32_t w[4];
    for (int c = 0; c < yc; ++c) {
        llh::load16(base + 16 * c, w);  // the whole chunk in one load: tag and values together
        if (w[3] != seq)
            return false;
        if (y) {
            float v[3];
            std::memcpy(v, w, 12);
            for (int k = 0; k < 3 && 3 * c + k < e->out_dim; ++k)
                y[3 * c + k] = v[k];
        }
    }
    return true;
}

int engine_wait(ll_engine *e, uint32_t seq, float *y, int n_rows, uint64_t timeout_ns)
{
    const ll_tick_header *h = static_cast<const ll_tick_header *>(e->mb_host);
    const bool tagged = e->opts.mailbox_format == 1;
    const auto t0 = std::chrono::steady_clock::now();
    uint32_t spins = 0;
    auto done = [&]() {
        return tagged ? tagged_done(e, seq, y)
                      : __atomic_load_n(const_cast<const uint32_t *>(&h->seq_out), __ATOMIC_ACQUIRE) == seq;
    };
    while (!done()) {
        cpu_relax();
        if ((++spins & 4095u) == 0) {
            if (e->ctrl_host->state == ST_EXITED && !done()) {
                // kernel left (idle exit raced this request, or a fault): relaunch picks the request up
                int rc = ensure_running(e);
                if (rc)
                    return rc;
            }
            const auto dt = std::chrono::steady_clock::now() - t0;
            if ((uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(dt).count() > timeout_ns) {
                llh::set_error("request seq %u not answered within %llu ns (device state %u, status %u)", seq,
                               (unsigned long long)timeout_ns, e->ctrl_host->state, e->ctrl_host->status);
                return LL_ERR_TIMEOUT;
            }
        }
    }
    if (y && !tagged) {
        const float *yd = reinterpret_cast<const float *>(static_cast<const char *>(e->mb_host) +
                                                          sizeof(ll_tick_header) +
                                                          sizeof(float) * (size_t)e->in_dim * e->max_batch);
        std::memcpy(y, yd, sizeof(float) * (size_t)e->out_dim * n_rows);
    }
    // a ring's device position comes from seq_out alone (reap): replies may be collected
    // out of order, so a collected seq says nothing about what the device took last
    if (e->ring == 1)
        e->last_served = seq;
    for (auto it = e->inflight.begin(); it != e->inflight.end(); ++it)
        if (it->first == seq) {
            e->inflight.erase(it);
            break;
        }
    return LL_OK;
}

// Write x into one slot of the tagged ring as chunks stamped with seq (no doorbell).
void write_tagged_slot(ll_engine *e, size_t slot, const float *x, uint32_t seq)
{
    char *base = static_cast<char *>(e->mb_host) + sizeof(ll_tick_header) + slot * e->ring_xstride;
    const int xc = (e->in_dim + 2) / 3;
    for (int c = 0; c < xc; ++c) {
        uint32_t w[4] = {0u, 0u, 0u, seq};
        for (int k = 0; k < 3 && 3 * c + k < e->in_dim; ++k)
            std::memcpy(&w[k], &x[3 * c + k], 4);
        llh::store16(base + 16 * c, w);  // one aligned 16-byte store per chunk
    }
}

inline void host_store_fence()
{
#if defined(__x86_64__)
    _mm_sfence();
#else
    std::atomic_thread_fence(std::memory_order_seq_cst);
#endif
}

// Post one request in the engine's mailbox format (tagged: into the next ring slot).
void engine_post(ll_engine *e, const float *x, int n_rows, uint32_t seq)
{
    if (e->opts.mailbox_format == 1) {
        write_tagged_slot(e, (size_t)(e->ring_next % (uint64_t)e->ring), x, seq);
        auto *h = static_cast<ll_tick_header *>(e->mb_host);
        h->n_rows = 1;
        __atomic_store_n(const_cast<uint32_t *>(&h->seq_in), seq, __ATOMIC_RELEASE);  // bookkeeping only
    } else {
        ll_mailbox_post(e->mb_host, e->in_dim, x, n_rows, seq, e->wc);
    }
    e->inflight.emplace_back(seq, e->ring_next++);
    e->seq = seq;
}

int engine_stop_kernel(ll_engine *e)
{
    if (!e->running)
        return LL_OK;
    while (!e->inflight.empty()) {
        const uint32_t s = e->inflight.front().first;
        if (engine_wait(e, s, nullptr, 1, 1000ull * 1000 * 1000) != LL_OK) {
            e->inflight.clear();
            break;
        }
    }
    ll_tick_header *h = static_cast<ll_tick_header *>(e->mb_host);
    __atomic_store_n(const_cast<uint32_t *>(&h->stop), 1u, __ATOMIC_RELEASE);
    const auto t0 = std::chrono::steady_clock::now();
    while (cudaStreamQuery(e->stream) == cudaErrorNotReady) {
        std::this_thread::sleep_for(std::chrono::microseconds(50));
        if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(10)) {
            llh::set_error("resident kernel did not stop within 10 s");
            return LL_ERR_TIMEOUT;
        }
    }
    int rc = reap(e);
    __atomic_store_n(const_cast<uint32_t *>(&h->stop), 0u, __ATOMIC_RELEASE);
    e->last_served = h->seq_out;
    return rc;
}

struct Packed {
    PlanResult pr;
    Params p{};
    std::vector<uint8_t> images;
};

// Plan, pack and lay out a net; touches no CUDA state.
int plan_and_pack(const ll_net_desc *net, const void *const *W, const float *const *b, const float *const *scales,
                  const ll_engine_opts &o, bool want_images, Packed &pk)
{
    int rc = validate_net(net, want_images ? W : nullptr);
    if (rc)
        return rc;
    if (want_images && !W) {
        llh::set_error("W is NULL");
        return LL_ERR_INVALID_ARG;
    }
    if (want_images && net->layers[0].wtype == LL_W_I8 && !scales) {
        llh::set_error("int8 weights need per-channel scales");
        return LL_ERR_INVALID_ARG;
    }
    int C = o.cluster_size == 0 ? 16 : o.cluster_size;
    if (C != 1 && C != 2 && C != 4 && C != 8 && C != 16) {
        llh::set_error("cluster_size must be 1, 2, 4, 8 or 16");
        return LL_ERR_INVALID_ARG;
    }
    const int max_stages = o.max_stages > 0 ? std::min(o.max_stages, kMaxStages) : kMaxStages;
    if (!plan_net(*net, C, o.replicate_first, o.min_stages, max_stages, pk.pr)) {
        llh::set_error("network does not fit %d stages of %d CTAs in shared memory", max_stages, C);
        return LL_ERR_BAD_DESC;
    }
    const PlanResult &pr = pk.pr;
    Params &p = pk.p;
    p.n_layers = net->n_layers;
    p.act_bf16 = net->layers[0].wtype != LL_W_F32;
    layout_buffers(p, pr, net->layers[0].in_dim, net->layers[net->n_layers - 1].out_dim, net->max_batch);
    size_t stride = 16;
    for (size_t v : pr.stage_image)
        stride = std::max(stride, llh::round_up(v, 16));
    p.image_stride = (uint32_t)stride;
    std::vector<uint32_t> w_off(net->n_layers), b_off(net->n_layers), s_off(net->n_layers);
    if (want_images)
        pk.images.assign((size_t)pr.S * pr.C * stride, 0);
    for (int s = 0; s < pr.S; ++s)
        for (int r = 0; r < pr.C; ++r) {
            if (want_images)
                pack_image(*net, pr, s, r, W, b, scales, pk.images.data() + ((size_t)s * pr.C + r) * stride, w_off,
                           b_off, s_off);
            else if (r == 0)
                pack_image(*net, pr, s, r, nullptr, nullptr, nullptr, nullptr, w_off, b_off, s_off);
        }
    for (int l = 0; l < net->n_layers; ++l) {
        const LayerPlan &lp = pr.L[l];
        LayerDev &d = p.L[l];
        d.mode = lp.mode;
        d.act = lp.act;
        d.wtype = lp.wtype;
        d.lpr_log2 = choose_lpr_log2(lp.K, lp.wtype);
        d.K = lp.K;
        d.M = lp.out;
        d.Mp = lp.Mp;
        d.R = lp.R;
        d.in_buf = lp.in_buf;
        d.in_ld = lp.in_ld;
        d.out_buf = lp.out_buf;
        d.out_ld = lp.out_ld;
        d.w_off = w_off[l];
        d.b_off = b_off[l];
        d.s_off = s_off[l];
        d.round_out = (p.act_bf16 && l + 1 < net->n_layers) ? 1 : 0;
    }
    return LL_OK;
}

void export_plan(const Params &p, ll_plan *out)
{
    std::memset(out, 0, sizeof(*out));
    out->n_layers = p.n_layers;
    out->n_stages = p.n_stages;
    out->cluster_size = p.C;
    out->threads = kThreads;
    out->bmax4 = p.bmax4;
    out->in_ld = p.in_ld;
    out->act_bf16 = p.act_bf16;
    for (int s = 0; s < kMaxStages; ++s) {
        out->stage_first[s] = p.stage_first[s];
        out->stage_last[s] = p.stage_last[s];
        out->stage_in_ld[s] = p.stage_in_ld[s];
        out->image_bytes[s] = p.image_bytes[s];
    }
    for (int i = 0; i < BUF_COUNT; ++i)
        out->buf_off[i] = p.buf_off[i];
    out->smem_bytes = p.smem_bytes;
    out->image_stride = p.image_stride;
    for (int l = 0; l < p.n_layers && l < 24; ++l) {
        const LayerDev &d = p.L[l];
        ll_plan_layer &o = out->layers[l];
        o.mode = d.mode;
        o.act = d.act;
        o.wtype = d.wtype;
        o.lpr_log2 = d.lpr_log2;
        o.K = d.K;
        o.M = d.M;
        o.Mp = d.Mp;
        o.R = d.R;
        o.in_buf = d.in_buf;
        o.in_ld = d.in_ld;
        o.out_buf = d.out_buf;
        o.out_ld = d.out_ld;
        o.w_off = d.w_off;
        o.b_off = d.b_off;
        o.s_off = d.s_off;
        o.round_out = d.round_out;
    }
}

// Register-resident kernel (variant 2) or, with `ring`, the pipelined ring kernel (variant 4:
// the same C compute CTAs plus one I/O CTA per cluster; tagged mailbox only).
int create_fast3(const ll_net_desc *net, const void *const *W, const float *const *b, int device,
                 const ll_engine_opts &o, const Fast3Entry &f, bool ring, ll_engine **out)
{
    if (ring && (!f.ring_fn || o.mailbox_format != 1)) {
        llh::set_error("the pipelined ring kernel (variant 4) needs the tagged mailbox (mailbox_format 1) and a "
                       "register-resident shape with room for multi-row passes (8 CTAs per cluster)");
        return LL_ERR_UNSUPPORTED;
    }
    size_t stride = 0;
    std::vector<uint8_t> img = ring ? pack_ring(f, W, b, stride) : pack_fast3(f, W, b, stride);
    if (img.empty())
        return LL_ERR_UNSUPPORTED;
    ll_engine *e = new ll_engine();
    e->device = device;
    e->in_dim = f.in;
    e->out_dim = f.out;
    e->max_batch = 1;
    e->kfn = ring ? f.ring_fn : f.fn;
    e->variant = ring ? 4 : 2;
    e->micro_max = f.rows;
    e->weight_regs = ring ? 4 * (f.h1 / 32) + 8 + f.K2 + f.K3 : f.K1 + f.K2 + f.K3;
    int rc = engine_common_create(e, &o);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    PlanResult &pr = e->plan;
    pr.S = 1;
    pr.C = f.C;
    pr.stage_first = {0};
    pr.stage_last = {2};
    pr.stage_in_ld = {f.in};
    pr.stage_image = {img.size() / f.C};
    Params &p = e->base;
    p.n_layers = 3;
    p.act_bf16 = 0;
    for (int l = 0; l < 3; ++l) {
        p.L[l] = LayerDev{};
        p.L[l].act = net->layers[l].act;
        p.L[l].M = net->layers[l].out_dim;
    }
    layout_buffers(p, pr, f.in, f.out, 1);
    p.smem_bytes = ring ? (uint32_t)f.ring_smem : 0u;  // the ring kernel's pool is dynamic; the rest static
    p.image_stride = (uint32_t)stride;
    cudaError_t ce = cudaMalloc((void **)&e->d_image, img.size());
    if (ce == cudaSuccess)
        ce = cudaMemcpy(e->d_image, img.data(), img.size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        llh::set_error("uploading register images: %s", cudaGetErrorString(ce));
        ll_engine_destroy(e);
        return LL_ERR_CUDA;
    }
    p.image = e->d_image;
    rc = finish_setup(e);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    if (ring) {  // the I/O CTA is the cluster's last rank (its abort broadcast covers every rank)
        e->grid = f.C + 1;
        e->base.C = f.C + 1;
    }
    *out = e;
    return LL_OK;
}

// Register-resident kernel for a deep net (variant 2, several clusters): one request at a time,
// TickBuffer or tagged mailbox (ring slots, no micro-batching), or the device queue.
int create_deep(const ll_net_desc *net, const void *const *W, const float *const *b, int device,
                const ll_engine_opts &o, const DeepEntry &d, ll_engine **out)
{
    size_t stride = 0;
    std::vector<uint8_t> img = pack_deep(d, W, b, stride);
    if (img.empty())
        return LL_ERR_UNSUPPORTED;
    ll_engine *e = new ll_engine();
    e->device = device;
    e->in_dim = d.in;
    e->out_dim = d.out;
    e->max_batch = 1;
    e->kfn = d.fn;
    e->variant = 2;
    e->micro_max = 1;
    e->weight_regs = d.NW;
    int rc = engine_common_create(e, &o);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    PlanResult &pr = e->plan;
    pr.S = d.NS;
    pr.C = d.C;
    pr.L.assign(d.nl, LayerPlan{});
    Params &p = e->base;
    p.n_layers = d.nl;
    p.act_bf16 = d.wt == LL_W_BF16 ? 1 : 0;  // the tagged poll rounds x to bf16 for a bf16 net
    for (int st = 0; st < d.NS; ++st) {
        const int l0 = st * d.lps, l1 = st == d.NS - 1 ? d.nl - 1 : (st + 1) * d.lps - 1;
        pr.stage_first.push_back(l0);
        pr.stage_last.push_back(l1);
        pr.stage_in_ld.push_back(l0 == 0 ? d.in : d.h);
        pr.stage_image.push_back(stride);
        for (int l = l0; l <= l1; ++l) {
            LayerPlan &lp = pr.L[l];
            lp.in = net->layers[l].in_dim;
            lp.out = net->layers[l].out_dim;
            lp.act = net->layers[l].act;
            lp.wtype = d.wt;
            lp.K = lp.in;
            lp.stage = st;
            lp.Mp = l == d.nl - 1 ? d.out : d.h;
            lp.R = l == d.nl - 1 ? d.out : d.h / d.C;
            // how the layer's outputs leave the CTA
            lp.mode = l == d.nl - 1                        ? LM_KSPLIT_GATHER
                      : l + 1 == d.nl - 1 && l + 1 <= l1    ? LM_ROWSPLIT_LOCAL
                      : l == l1                             ? LM_ROWSPLIT_GLOBAL
                                                            : LM_ROWSPLIT_ALLGATHER;
            p.L[l] = LayerDev{};
            p.L[l].mode = lp.mode;
            p.L[l].act = lp.act;
            p.L[l].wtype = d.wt;
            p.L[l].round_out = d.wt == LL_W_BF16 && l < d.nl - 1 ? 1 : 0;
            p.L[l].K = lp.K;
            p.L[l].M = lp.out;
            p.L[l].Mp = lp.Mp;
            p.L[l].R = lp.R;
        }
    }
    layout_buffers(p, pr, d.in, d.out, 1);
    p.smem_bytes = 0;  // all shared memory of this kernel is static
    p.image_stride = (uint32_t)stride;
    cudaError_t ce = cudaMalloc((void **)&e->d_image, img.size());
    if (ce == cudaSuccess)
        ce = cudaMemcpy(e->d_image, img.data(), img.size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        llh::set_error("uploading register images: %s", cudaGetErrorString(ce));
        ll_engine_destroy(e);
        return LL_ERR_CUDA;
    }
    p.image = e->d_image;
    rc = finish_setup(e);  // grid S * C; the L2 hand-off buffers of the ROWSPLIT_GLOBAL layers
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    if (!p.xfer_tagged || (size_t)p.xfer_stride < 2 * (size_t)d.h) {
        llh::set_error("deep kernel: the hand-off buffers hold %u floats per stage, %d needed", p.xfer_stride, 2 * d.h);
        ll_engine_destroy(e);
        return LL_ERR_UNSUPPORTED;
    }
    *out = e;
    return LL_OK;
}

// Kernel variant 3 (resident small-batch kernel): bf16 or int8 weights of one type, up to
// 32 rows, the TickBuffer mailbox (or the tagged one at batch 1), in and out widths
// multiples of 4, slices that fit one SM.
// Returns an empty string when the net can run on it, else the reason.
const char *gemv_engine_refusal(const ll_net_desc *net, const float *const *scales, const ll_engine_opts &o, int sms)
{
    const int t = net->layers[0].wtype;
    if (t != LL_W_BF16 && t != LL_W_I8)
        return "bf16 or int8 weights";
    for (int l = 0; l < net->n_layers; ++l)
        if (net->layers[l].wtype != t)
            return "one weight type for every layer";
    if (t == LL_W_I8 && !scales)
        return "per-channel scales for int8 weights";
    if (net->max_batch < 1 || net->max_batch > kGvMaxRows)
        return "max_batch <= 32";
    if (net->layers[0].in_dim % 4 != 0 || net->layers[net->n_layers - 1].out_dim % 4 != 0)
        return "in_dim and out_dim multiples of 4";
    if (o.ring_slots > 1 || o.micro_batch > 1 || (o.mailbox_format != 0 && o.mailbox_format != 1) ||
        (o.mailbox_format == 1 && net->max_batch != 1))
        return "the TickBuffer mailbox, or the tagged one at max_batch 1 (one slot, no micro-batching)";
    if (!gemv_fits(net, sms))
        return "every layer's row slice plus the staged rows in one SM's shared memory";
    return "";
}

int create_gemv(const ll_net_desc *net, const void *const *W, const float *const *b, const float *const *scales,
                int device, const ll_engine_opts &o, int sms, ll_engine **out)
{
    const int L = net->n_layers;
    const bool i8 = net->layers[0].wtype == LL_W_I8;
    ll_engine *e = new ll_engine();
    auto fail = [&](int code) {
        ll_engine_destroy(e);
        return code;
    };
    e->device = device;
    e->in_dim = net->layers[0].in_dim;
    e->out_dim = net->layers[L - 1].out_dim;
    e->max_batch = net->max_batch;
    e->variant = 3;
    e->gv_bp = gemv_bp(net->max_batch);
    static const void *const k8[6] = {
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 1, 1, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 1, 2, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 1, 4, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 2, 4, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 4, 4, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 8, 4, true>)};
    static const void *const k16[6] = {
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 1, 1, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 1, 2, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 1, 4, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 2, 4, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 4, 4, true>),
        reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 8, 4, true>)};
    const int idx = 31 - __builtin_clz((unsigned)e->gv_bp);
    e->kfn = i8 ? k8[idx] : k16[idx];
    int rc = engine_common_create(e, &o);
    if (rc)
        return fail(rc);
    gemv_layout(net, sms, e->gl);
    e->gv_smem = (int)e->gl.smem(e->gv_bp);
    int max_w = 0;
    for (int l = 0; l < L; ++l)
        max_w = std::max(max_w, net->layers[l].out_dim);
    const std::vector<uint8_t> img = gemv_pack_images(net, W, b, scales, sms, e->gl);
    e->gv_hand_bytes = sizeof(uint32_t) * kGvTagRows * (size_t)max_w;
    e->gv_act_bytes = sizeof(__nv_bfloat16) * kGvMaxRows * (size_t)max_w;
    cudaError_t ce = cudaMalloc((void **)&e->gv_img, img.size());
    if (ce == cudaSuccess)
        ce = cudaMemcpy(e->gv_img, img.data(), img.size(), cudaMemcpyHostToDevice);
    for (int i = 0; i < 2 && ce == cudaSuccess; ++i) {
        ce = cudaMalloc((void **)&e->gv_hand[i], e->gv_hand_bytes);
        if (ce == cudaSuccess)
            ce = cudaMalloc((void **)&e->gv_act[i], e->gv_act_bytes);
    }
    if (ce == cudaSuccess)
        ce = cudaMalloc((void **)&e->gv_cnt, sizeof(unsigned) * kGvCntStride * (size_t)L);
    if (ce == cudaSuccess)
        ce = cudaMalloc((void **)&e->gv_relay, sizeof(float) * kGvMaxRows * (size_t)e->in_dim);
    if (ce == cudaSuccess)
        ce = cudaMalloc((void **)&e->gv_gather, sizeof(float) * kGvMaxRows * (size_t)e->out_dim);
    if (ce == cudaSuccess)
        ce = cudaMalloc((void **)&e->gv_req, sizeof(unsigned long long));
    if (ce == cudaSuccess)
        ce = cudaMalloc((void **)&e->gv_status, sizeof(unsigned));
    if (ce == cudaSuccess)
        ce = cudaFuncSetAttribute(e->kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, e->gv_smem);
    int per_sm = 0;
    if (ce == cudaSuccess)
        ce = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, e->kfn, kGvThreads, (size_t)e->gv_smem);
    if (ce != cudaSuccess) {
        llh::set_error("resident small-batch kernel set-up: %s", cudaGetErrorString(ce));
        return fail(LL_ERR_CUDA);
    }
    if (per_sm < 1) {
        llh::set_error("resident small-batch kernel: a CTA does not fit one SM");
        return fail(LL_ERR_BAD_DESC);
    }
    e->attrs_set = true;
    GemvNetParams &g = e->gv;
    gemv_static_params(net, e->gl, e->gv_img, g);
    g.hand[0] = e->gv_hand[0];
    g.hand[1] = e->gv_hand[1];
    g.act[0] = e->gv_act[0];
    g.act[1] = e->gv_act[1];
    g.cnt = e->gv_cnt;
    g.status = e->gv_status;
    g.wait_ns = e->opts.step_timeout_ns;
    g.res.relay_x = e->gv_relay;
    g.res.gather_y = e->gv_gather;
    g.res.req = e->gv_req;
    PlanResult &pr = e->plan;
    pr.S = 1;
    pr.C = 1;
    Params &p = e->base;
    p.n_layers = L;
    p.max_batch = net->max_batch;
    rc = finish_setup(e);
    if (rc)
        return fail(rc);
    e->grid = sms;  // one CTA per SM
    *out = e;
    return LL_OK;
}

}  // namespace

extern "C" {

int ll_engine_create_ex(const ll_net_desc *net, const void *const *W, const float *const *b,
                        const float *const *scales, int device, const ll_engine_opts *opts, ll_engine **out)
{
    if (!out) {
        llh::set_error("out is NULL");
        return LL_ERR_INVALID_ARG;
    }
    *out = nullptr;
    ll_engine_opts o;
    if (opts)
        o = *opts;
    else
        ll_engine_opts_default(&o);
    int rc = validate_net(net, W);
    if (rc)
        return rc;
    if (!W) {
        llh::set_error("W is NULL");
        return LL_ERR_INVALID_ARG;
    }
    const Fast3Entry *f3 = (o.kernel_variant == 1 || o.kernel_variant == 3) ? nullptr : find_fast3(*net, o.cluster_size);
    if (((o.kernel_variant == 2 && (o.micro_batch > 1 || !find_deep(*net, o.cluster_size))) || o.kernel_variant == 4) &&
        !f3) {
        llh::set_error("no register-resident kernel is compiled for this net shape / cluster size");
        return LL_ERR_UNSUPPORTED;
    }
    if (f3)
        return create_fast3(net, W, b, device, o, *f3, o.kernel_variant == 4, out);
    // deep nets of one hidden width: the multi-cluster register-resident kernel, unless a plan
    // is forced (cluster size aside) or requests are to be taken several at a time
    const DeepEntry *dp = (o.kernel_variant == 0 || o.kernel_variant == 2) && !o.min_stages && !o.max_stages &&
                                  o.replicate_first < 0 && o.micro_batch <= 1
                              ? find_deep(*net, o.cluster_size)
                              : nullptr;
    if (dp)
        return create_deep(net, W, b, device, o, *dp, out);
    if (o.kernel_variant == 3 || o.kernel_variant == 0) {
        int sms = 0;
        LL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        const char *why = gemv_engine_refusal(net, scales, o, sms);
        if (o.kernel_variant == 3 && *why) {
            llh::set_error("the resident small-batch kernel (variant 3) needs %s", why);
            return LL_ERR_UNSUPPORTED;
        }
        // automatic: when the weights exceed what one 16-CTA cluster holds in shared memory
        // (the generic kernel would then pipeline several clusters through L2 anyway)
        size_t wbytes = 0;
        for (int l = 0; l < net->n_layers; ++l)
            wbytes += (size_t)net->layers[l].in_dim * net->layers[l].out_dim *
                      (net->layers[l].wtype == LL_W_I8 ? 1 : net->layers[l].wtype == LL_W_BF16 ? 2 : 4);
        const bool forced_plan = o.cluster_size || o.min_stages || o.max_stages;
        if (o.kernel_variant == 3 || (!*why && !forced_plan && wbytes > 16 * (size_t)227 * 1024))
            return create_gemv(net, W, b, scales, device, o, sms, out);
    }
    Packed pk;
    rc = plan_and_pack(net, W, b, scales, o, true, pk);
    if (rc)
        return rc;
    ll_engine *e = new ll_engine();
    e->device = device;
    e->in_dim = net->layers[0].in_dim;
    e->out_dim = net->layers[net->n_layers - 1].out_dim;
    e->max_batch = net->max_batch;
    rc = engine_common_create(e, &o);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    e->plan = pk.pr;
    e->base = pk.p;
    cudaError_t ce = cudaMalloc((void **)&e->d_image, pk.images.size());
    if (ce == cudaSuccess)
        ce = cudaMemcpy(e->d_image, pk.images.data(), pk.images.size(), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
        llh::set_error("uploading weight images: %s", cudaGetErrorString(ce));
        ll_engine_destroy(e);
        return LL_ERR_CUDA;
    }
    e->base.image = e->d_image;
    rc = finish_setup(e);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    *out = e;
    return LL_OK;
}

int ll_plan_net(const ll_net_desc *net, const void *const *W, const float *const *b, const float *const *scales,
                const ll_engine_opts *opts, ll_plan *plan, uint8_t *images, size_t images_cap, size_t *images_bytes)
{
    ll_engine_opts o;
    if (opts)
        o = *opts;
    else
        ll_engine_opts_default(&o);
    Packed pk;
    int rc = plan_and_pack(net, W, b, scales, o, images != nullptr, pk);
    if (rc)
        return rc;
    const size_t need = (size_t)pk.pr.S * pk.pr.C * pk.p.image_stride;
    if (images_bytes)
        *images_bytes = need;
    if (plan)
        export_plan(pk.p, plan);
    if (images) {
        if (images_cap < need) {
            llh::set_error("images buffer too small: %zu < %zu", images_cap, need);
            return LL_ERR_INVALID_ARG;
        }
        std::memcpy(images, pk.images.data(), need);
    }
    return LL_OK;
}

int ll_engine_create(const ll_net_desc *net, const void *const *W, const float *const *b, const float *const *scales,
                     int device, ll_engine **out)
{
    return ll_engine_create_ex(net, W, b, scales, device, nullptr, out);
}

int ll_echo_engine_create(int device, int in_dim, int out_dim, const ll_engine_opts *opts, ll_engine **out)
{
    if (!out || in_dim < 0 || out_dim < 0 || in_dim > 16384 || out_dim > 16384) {
        llh::set_error("invalid echo engine arguments");
        return LL_ERR_INVALID_ARG;
    }
    *out = nullptr;
    ll_engine *e = new ll_engine();
    e->device = device;
    e->echo = true;
    e->in_dim = in_dim;
    e->out_dim = out_dim;
    e->max_batch = 1;
    int rc = engine_common_create(e, opts);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    PlanResult &pr = e->plan;
    pr.S = 1;
    pr.C = 1;
    pr.stage_first = {0};
    pr.stage_last = {-1};
    pr.stage_in_ld = {(int)llh::round_up((size_t)std::max(in_dim, 4), 4)};
    pr.stage_image = {0};
    pr.buf_floats[BUF_X] = 4 * (size_t)pr.stage_in_ld[0];
    e->base.n_layers = 0;
    layout_buffers(e->base, pr, in_dim, out_dim, 1);
    rc = finish_setup(e);
    if (rc) {
        ll_engine_destroy(e);
        return rc;
    }
    *out = e;
    return LL_OK;
}

void *ll_engine_mailbox(ll_engine *e)
{
    return e ? e->mb_host : nullptr;
}

float *ll_engine_mailbox_x(ll_engine *e)
{
    return e ? reinterpret_cast<float *>(static_cast<char *>(e->mb_host) + sizeof(ll_tick_header)) : nullptr;
}

float *ll_engine_mailbox_y(ll_engine *e)
{
    if (!e)
        return nullptr;
    if (e->opts.mailbox_format == 1)  // slot 0's first y chunk (ll_tagged_y_offset for one slot)
        return reinterpret_cast<float *>(static_cast<char *>(e->mb_host) + e->ring_ybase);
    return reinterpret_cast<float *>(static_cast<char *>(e->mb_host) + sizeof(ll_tick_header) +
                                     sizeof(float) * (size_t)e->in_dim * e->max_batch);
}

int ll_engine_start(ll_engine *e)
{
    if (!e) {
        llh::set_error("engine is NULL");
        return LL_ERR_INVALID_ARG;
    }
    return ensure_running(e);
}

int ll_submit(ll_engine *e, const float *x, int n_rows, uint32_t *seq)
{
    if (!e || n_rows < 1 || n_rows > e->max_batch) {
        llh::set_error("ll_submit: bad engine or n_rows %d (max %d)", n_rows, e ? e->max_batch : 0);
        return LL_ERR_INVALID_ARG;
    }
    const size_t cap = e->opts.mailbox_format == 1 ? (size_t)e->ring : 1u;
    if (e->inflight.size() >= cap) {
        llh::set_error("ll_submit: %zu request(s) outstanding (the mailbox holds %zu)", e->inflight.size(), cap);
        return LL_ERR_BUSY;
    }
    int rc = ensure_running(e);
    if (rc)
        return rc;
    const uint32_t s = ll_next_seq(e->last_served > e->seq ? e->last_served : e->seq);
    if (e->opts.mailbox_format == 1 && !x) {
        llh::set_error("ll_submit: the tagged mailbox needs x (the chunks carry the sequence number)");
        return LL_ERR_INVALID_ARG;
    }
    engine_post(e, x, n_rows, s);
    if (seq)
        *seq = s;
    return LL_OK;
}

int ll_submit_many(ll_engine *e, const float *xs, int k, uint32_t *seqs)
{
    if (!e || !xs || k < 1 || !seqs) {
        llh::set_error("ll_submit_many: null engine, x or seqs, or k %d < 1", k);
        return LL_ERR_INVALID_ARG;
    }
    if (e->opts.mailbox_format != 1) {
        if (k != 1) {
            llh::set_error("ll_submit_many: the TickBuffer holds one request (k = %d)", k);
            return LL_ERR_INVALID_ARG;
        }
        return ll_submit(e, xs, 1, seqs);
    }
    if (e->inflight.size() + (size_t)k > (size_t)e->ring) {
        llh::set_error("ll_submit_many: %zu request(s) outstanding, %d more do not fit the %d-slot ring",
                       e->inflight.size(), k, e->ring);
        return LL_ERR_BUSY;
    }
    int rc = ensure_running(e);
    if (rc)
        return rc;
    uint32_t s = e->last_served > e->seq ? e->last_served : e->seq;
    for (int i = 0; i < k; ++i)
        seqs[i] = s = ll_next_seq(s);
    // Slots 1..k-1 first, then the doorbell word, then slot 0.  The device takes the slots
    // strictly in order, so it can start on the burst only once slot 0 is visible, and x86
    // stores become visible in program order: the rest of the burst is there by then.
    const uint64_t base = e->ring_next;
    for (int i = 1; i < k; ++i)
        write_tagged_slot(e, (size_t)((base + (uint64_t)i) % (uint64_t)e->ring), xs + (size_t)i * e->in_dim, seqs[i]);
    auto *h = static_cast<ll_tick_header *>(e->mb_host);
    h->n_rows = 1;
    if (e->wc)
        host_store_fence();
    __atomic_store_n(const_cast<uint32_t *>(&h->seq_in), seqs[k - 1], __ATOMIC_RELEASE);
    if (e->wc)
        host_store_fence();
    write_tagged_slot(e, (size_t)(base % (uint64_t)e->ring), xs, seqs[0]);
    if (e->wc)
        host_store_fence();
    for (int i = 0; i < k; ++i)
        e->inflight.emplace_back(seqs[i], e->ring_next++);
    e->seq = seqs[k - 1];
    return LL_OK;
}

int ll_poll(ll_engine *e, uint32_t seq, float *y, uint64_t timeout_ns)
{
    if (!e) {
        llh::set_error("engine is NULL");
        return LL_ERR_INVALID_ARG;
    }
    const ll_tick_header *h = static_cast<const ll_tick_header *>(e->mb_host);
    const int n_rows = h->n_rows == 0 ? 1 : (int)h->n_rows;
    return engine_wait(e, seq, y, n_rows, timeout_ns);
}

int ll_infer(ll_engine *e, const float *x, int n_rows, float *y, uint64_t timeout_ns)
{
    uint32_t s = 0;
    int rc = ll_submit(e, x, n_rows, &s);
    if (rc)
        return rc;
    return ll_poll(e, s, y, timeout_ns);
}

int ll_engine_stop(ll_engine *e)
{
    if (!e) {
        llh::set_error("engine is NULL");
        return LL_ERR_INVALID_ARG;
    }
    cudaSetDevice(e->device);
    return engine_stop_kernel(e);
}

int ll_engine_destroy(ll_engine *e)
{
    if (!e)
        return LL_OK;
    cudaSetDevice(e->device);
    int rc = LL_OK;
    if (e->running)
        rc = engine_stop_kernel(e);
    if (e->stream)
        cudaStreamDestroy(e->stream);
    if (e->d_image)
        cudaFree(e->d_image);
    if (e->d_xfer)
        cudaFree(e->d_xfer);
    if (e->d_words)
        cudaFree(e->d_words);
    for (void *q : {(void *)e->gv_img, (void *)e->gv_hand[0], (void *)e->gv_hand[1], (void *)e->gv_act[0],
                    (void *)e->gv_act[1], (void *)e->gv_cnt, (void *)e->gv_relay, (void *)e->gv_gather,
                    (void *)e->gv_req, (void *)e->gv_status})
        if (q)
            cudaFree(q);
    if (e->mb_host)
        cudaFreeHost(e->mb_host);
    if (e->ctrl_host)
        cudaFreeHost((void *)e->ctrl_host);
    delete e;
    return rc;
}

int ll_engine_set_trace(ll_engine *e, unsigned long long *d_trace, int n)
{
    if (!e || n < 0 || (n > 0 && !d_trace)) {
        llh::set_error("ll_engine_set_trace: invalid arguments");
        return LL_ERR_INVALID_ARG;
    }
    e->base.trace = n > 0 ? d_trace : nullptr;
    e->base.trace_n = n;
    return LL_OK;
}

int ll_engine_get_info(ll_engine *e, ll_engine_info *info)
{
    if (!e || !info) {
        llh::set_error("NULL argument");
        return LL_ERR_INVALID_ARG;
    }
    std::memset(info, 0, sizeof(*info));
    info->n_stages = e->plan.S;
    info->cluster_size = e->plan.C;
    info->threads = e->variant == 3 ? kGvThreads : kThreads;
    info->smem_bytes = e->variant == 3 ? (int32_t)e->gv_smem : (int32_t)e->base.smem_bytes;
    size_t mi = 0;
    for (size_t v : e->plan.stage_image)
        mi = std::max(mi, v);
    info->image_bytes = e->variant == 3 ? (int32_t)e->gl.img_bytes : (int32_t)mi;
    info->launches = e->launches;
    info->state = (int32_t)e->ctrl_host->state;
    info->status = (int32_t)e->ctrl_host->status;
    info->err_where = (int32_t)e->ctrl_host->err_where;
    info->served = static_cast<ll_tick_header *>(e->mb_host)->seq_out;
    for (int l = 0; l < e->base.n_layers && l < 24; ++l)
        info->layer_modes[l] = e->base.L[l].mode;
    info->kernel_variant = e->variant;
    info->weight_regs = e->weight_regs;
    info->passes = e->passes;
    info->rows = e->rows;
    return LL_OK;
}

int ll_engine_bench_closed_loop(ll_engine *e, const float *xs, int n_x, int n_req, int n_rows, float *ys,
                                double *lat_us)
{
    if (!e || !xs || n_x < 1 || n_req < 0 || n_rows < 1 || n_rows > e->max_batch) {
        llh::set_error("ll_engine_bench_closed_loop: invalid arguments");
        return LL_ERR_INVALID_ARG;
    }
    if (!e->inflight.empty()) {
        llh::set_error("request outstanding");
        return LL_ERR_BUSY;
    }
    int rc = ensure_running(e);
    if (rc)
        return rc;
    const size_t xin = (size_t)e->in_dim * n_rows;
    const size_t yout = (size_t)e->out_dim * n_rows;
    std::vector<float> ybuf(yout);
    for (int r = 0; r < n_req; ++r) {
        const auto t0 = std::chrono::steady_clock::now();
        const uint32_t s = ll_next_seq(e->last_served > e->seq ? e->last_served : e->seq);
        engine_post(e, xs + (size_t)(r % n_x) * xin, n_rows, s);
        rc = engine_wait(e, s, ys ? ys + (size_t)r * yout : ybuf.data(), n_rows, 2000ull * 1000 * 1000);
        const auto t1 = std::chrono::steady_clock::now();
        if (rc)
            return rc;
        if (lat_us)
            lat_us[r] = std::chrono::duration<double, std::micro>(t1 - t0).count();
    }
    return LL_OK;
}

int ll_engine_bench_ring(ll_engine *e, const float *xs, int n_x, int n_req, int depth, float *ys, double *lat_us,
                         double *elapsed_s)
{
    if (!e || !xs || n_x < 1 || n_req < 0 || depth < 1 || e->max_batch != 1 || e->opts.mailbox_format != 1 ||
        depth > e->ring) {
        llh::set_error("ll_engine_bench_ring: invalid arguments (needs the tagged mailbox, 1 <= depth <= ring_slots)");
        return LL_ERR_INVALID_ARG;
    }
    if (!e->inflight.empty()) {
        llh::set_error("request outstanding");
        return LL_ERR_BUSY;
    }
    int rc = ensure_running(e);
    if (rc)
        return rc;
    using clk = std::chrono::steady_clock;
    const size_t xin = (size_t)e->in_dim, yout = (size_t)e->out_dim;
    std::vector<clk::time_point> posted_at((size_t)depth);  // by request index mod depth
    std::vector<float> ybuf(yout);
    const auto t0 = clk::now();
    auto last_progress = t0;
    int posted = 0, done = 0;
    while (done < n_req) {
        // keep the ring full: every free slot takes the next request at once
        while (posted < n_req && posted - done < depth) {
            const uint32_t s = ll_next_seq(e->last_served > e->seq ? e->last_served : e->seq);
            posted_at[(size_t)(posted % depth)] = clk::now();
            engine_post(e, xs + (size_t)(posted % n_x) * xin, 1, s);
            ++posted;
        }
        const uint32_t s = e->inflight.front().first;
        float *y = ys ? ys + (size_t)done * yout : ybuf.data();
        if (tagged_done(e, s, y)) {
            rc = engine_wait(e, s, nullptr, 1, 0);  // bookkeeping: the reply is there and copied
            if (rc)
                return rc;
            const auto t1 = clk::now();
            if (lat_us)
                lat_us[done] = std::chrono::duration<double, std::micro>(t1 - posted_at[(size_t)(done % depth)]).count();
            ++done;
            last_progress = t1;
            continue;
        }
        cpu_relax();
        if (clk::now() - last_progress > std::chrono::seconds(2)) {
            if (e->ctrl_host->state == ST_EXITED) {
                rc = ensure_running(e);
                if (rc)
                    return rc;
                last_progress = clk::now();
                continue;
            }
            llh::set_error("ring bench: request seq %u not answered within 2 s", s);
            return LL_ERR_TIMEOUT;
        }
    }
    if (elapsed_s)
        *elapsed_s = std::chrono::duration<double>(clk::now() - t0).count();
    return LL_OK;
}

int ll_engine_bench_ring_mt(ll_engine *e, const float *xs, int n_x, int n_req, int depth, float *ys, double *lat_us,
                            double *elapsed_s, int poster_cpu)
{
    if (!e || !xs || n_x < 1 || n_req < 1 || depth < 1 || e->max_batch != 1 || e->opts.mailbox_format != 1 ||
        depth > e->ring) {
        llh::set_error("ll_engine_bench_ring_mt: invalid arguments (needs the tagged mailbox, 1 <= depth <= ring_slots)");
        return LL_ERR_INVALID_ARG;
    }
    if (!e->inflight.empty()) {
        llh::set_error("request outstanding");
        return LL_ERR_BUSY;
    }
    int rc = ensure_running(e);
    if (rc)
        return rc;
    using clk = std::chrono::steady_clock;
    const size_t xin = (size_t)e->in_dim, yout = (size_t)e->out_dim;
    const int yc = (e->out_dim + 2) / 3;
    // every request's sequence number and ring slot are fixed up front (the rule engine_post
    // follows: consecutive numbers after the last one posted or served)
    std::vector<uint32_t> seqs((size_t)n_req);
    uint32_t s = e->last_served > e->seq ? e->last_served : e->seq;
    for (int k = 0; k < n_req; ++k)
        seqs[(size_t)k] = s = ll_next_seq(s);
    const uint64_t base = e->ring_next;
    std::vector<int64_t> posted_at((size_t)n_req);  // steady_clock ns, written by the poster
    std::atomic<int> posted{0}, done{0};
    std::atomic<bool> quit{false};
    auto *h = static_cast<ll_tick_header *>(e->mb_host);
    auto now_ns = []() { return std::chrono::duration_cast<std::chrono::nanoseconds>(clk::now().time_since_epoch()).count(); };
    const auto t0 = clk::now();
    std::thread poster([&] {
        if (poster_cpu >= 0) {
            cpu_set_t set;
            CPU_ZERO(&set);
            CPU_SET(poster_cpu, &set);
            pthread_setaffinity_np(pthread_self(), sizeof(set), &set);  // best effort
        }
        int k = 0;
        while (k < n_req && !quit.load(std::memory_order_relaxed)) {
            const int lim = std::min(n_req, done.load(std::memory_order_acquire) + depth);
            if (k >= lim) {
                cpu_relax();
                continue;
            }
            for (; k < lim; ++k) {
                posted_at[(size_t)k] = now_ns();
                write_tagged_slot(e, (size_t)((base + (uint64_t)k) % (uint64_t)e->ring), xs + (size_t)(k % n_x) * xin,
                                  seqs[(size_t)k]);
            }
            h->n_rows = 1;
            __atomic_store_n(const_cast<uint32_t *>(&h->seq_in), seqs[(size_t)k - 1], __ATOMIC_RELEASE);
            posted.store(k, std::memory_order_release);
        }
    });
    std::vector<float> ybuf(yout);
    const char *ybase = static_cast<const char *>(e->mb_host) + e->ring_ybase;
    auto last_progress = clk::now();
    rc = LL_OK;
    for (int k = 0; k < n_req && rc == LL_OK; ++k) {
        const char *yl = ybase + (size_t)((base + (uint64_t)k) % (uint64_t)e->ring) * e->ring_ystride;
        float *y = ys ? ys + (size_t)k * yout : ybuf.data();
        for (uint32_t spins = 0;; ++spins) {
            bool ok = true;
            uint32_t w[4];
            for (int c = 0; c < yc && ok; ++c) {
                llh::load16(yl + 16 * c, w);  // the whole chunk in one load: tag and values together
                if (w[3] != seqs[(size_t)k]) {
                    ok = false;
                } else {
                    float v[3];
                    std::memcpy(v, w, 12);
                    for (int j = 0; j < 3 && 3 * c + j < e->out_dim; ++j)
                        y[3 * c + j] = v[j];
                }
            }
            if (ok)
                break;
            cpu_relax();
            if ((spins & 1023u) == 1023u && clk::now() - last_progress > std::chrono::seconds(2)) {
                llh::set_error("ring bench: request seq %u not answered within 2 s (device state %u, status %u)",
                               seqs[(size_t)k], e->ctrl_host->state, e->ctrl_host->status);
                rc = LL_ERR_TIMEOUT;
                break;
            }
        }
        if (rc != LL_OK)
            break;
        const int64_t t1 = now_ns();
        last_progress = clk::now();
        while (posted.load(std::memory_order_acquire) <= k) {
        }  // orders the poster's posted_at[k] before this read (the reply already implies the post)
        if (lat_us)
            lat_us[k] = (double)(t1 - posted_at[(size_t)k]) / 1000.0;
        done.store(k + 1, std::memory_order_release);
    }
    quit.store(true, std::memory_order_relaxed);
    poster.join();
    // the engine's host-side position: every request posted was answered (or the run failed:
    // the caller stops the engine)
    const int n_posted = posted.load(std::memory_order_acquire);
    if (n_posted > 0) {
        e->seq = seqs[(size_t)n_posted - 1];
        e->ring_next = base + (uint64_t)n_posted;
    }
    if (elapsed_s)
        *elapsed_s = std::chrono::duration<double>(clk::now() - t0).count();
    return rc;
}

int ll_engine_serve_poisson(ll_engine *e, const float *xs, int n_x, int n_total, double rate_per_s, uint64_t seed,
                            int rank, int world, double *lat_us, int *n_served, double *elapsed_s, float *ys,
                            int *req_idx)
{
    if (!e || !xs || n_x < 1 || n_total < 0 || !(rate_per_s > 0) || world < 1 || rank < 0 || rank >= world ||
        !lat_us || e->max_batch != 1) {
        llh::set_error("ll_engine_serve_poisson: invalid arguments");
        return LL_ERR_INVALID_ARG;
    }
    if (!e->inflight.empty()) {
        llh::set_error("request outstanding");
        return LL_ERR_BUSY;
    }
    // the whole stream, identical on every rank: exponential gaps, then a uniform GPU per request
    std::mt19937_64 rng(seed);
    std::exponential_distribution<double> gap(rate_per_s);
    std::uniform_int_distribution<int> gpu(0, world - 1);
    std::vector<double> arrive;  // seconds from the start, this rank's requests
    std::vector<int> which;      // global request index (selects the input row)
    double t = 0.0;
    for (int i = 0; i < n_total; ++i) {
        t += gap(rng);
        if (gpu(rng) == rank) {
            arrive.push_back(t);
            which.push_back(i);
        }
    }
    int rc = ensure_running(e);
    if (rc)
        return rc;
    const size_t cap = e->opts.mailbox_format == 1 ? (size_t)e->ring : 1u;
    const size_t n = arrive.size();
    const size_t xin = (size_t)e->in_dim;
    using clk = std::chrono::steady_clock;
    const auto t0 = clk::now() + std::chrono::microseconds(200);
    auto at = [&](size_t j) { return t0 + std::chrono::nanoseconds((int64_t)(arrive[j] * 1e9)); };
    size_t posted = 0, done = 0;
    auto last_progress = clk::now();
    while (done < n) {
        const auto now = clk::now();
        while (posted < n && e->inflight.size() < cap && now >= at(posted)) {
            const uint32_t s = ll_next_seq(e->last_served > e->seq ? e->last_served : e->seq);
            engine_post(e, xs + (size_t)(which[posted] % n_x) * xin, 1, s);
            ++posted;
        }
        if (!e->inflight.empty()) {
            const uint32_t s = e->inflight.front().first;
            const bool ok = e->opts.mailbox_format == 1
                                ? tagged_done(e, s, nullptr)
                                : __atomic_load_n(const_cast<const uint32_t *>(&static_cast<ll_tick_header *>(
                                                      e->mb_host)->seq_out),
                                                  __ATOMIC_ACQUIRE) == s;
            if (ok) {
                // bookkeeping (the reply is there); copies y out when asked
                rc = engine_wait(e, s, ys ? ys + done * (size_t)e->out_dim : nullptr, 1, 0);
                if (rc)
                    return rc;
                const auto tdone = clk::now();
                lat_us[done] = std::chrono::duration<double, std::micro>(tdone - at(done)).count();
                if (req_idx)
                    req_idx[done] = which[done];
                ++done;
                last_progress = tdone;
                continue;
            }
            if (now - last_progress > std::chrono::seconds(2)) {
                if (e->ctrl_host->state == ST_EXITED) {
                    rc = ensure_running(e);
                    if (rc)
                        return rc;
                    last_progress = clk::now();
                    continue;
                }
                llh::set_error("serve: request seq %u not answered within 2 s", s);
                return LL_ERR_TIMEOUT;
            }
        }
        cpu_relax();
    }
    if (n_served)
        *n_served = (int)n;
    if (elapsed_s)
        *elapsed_s = std::chrono::duration<double>(clk::now() - t0).count();
    return LL_OK;
}

int ll_engine_run_queue(ll_engine *e, const float *d_x, float *d_y, int n_req, int n_rows, float *ms,
                        unsigned long long *d_stamps)
{
    if (!e || !d_x || !d_y || n_req < 1 || n_rows < 1 || n_rows > e->max_batch) {
        llh::set_error("ll_engine_run_queue: invalid arguments");
        return LL_ERR_INVALID_ARG;
    }
    if (e->variant == 4 && reinterpret_cast<uintptr_t>(d_x) % 16 != 0) {
        llh::set_error("ll_engine_run_queue: the pipelined ring kernel reads the queue by bulk copies: d_x must be "
                       "16-byte aligned");
        return LL_ERR_INVALID_ARG;
    }
    LL_CUDA_TRY(cudaSetDevice(e->device));
    int rc = engine_stop_kernel(e);
    if (rc)
        return rc;
    // the resident small-batch kernel hands off in 16-bit tags up to 4 rows: a launch serves
    // at most 65534 / n_layers requests before they run out, so longer queues take several
    int cap = n_req;
    if (e->variant == 3 && e->gv_bp <= kGvTagRows)
        cap = (int)((kGvTagLimit - 1u) / (unsigned)e->gv.n_layers);
    float total = 0.0f;
    for (int done = 0; done < n_req && rc == LL_OK;) {
        const int n = std::min(n_req - done, cap);
        Params p = e->base;
        p.mode = MODE_QUEUE;
        p.q_x = d_x + (size_t)done * n_rows * e->in_dim;
        p.q_y = d_y + (size_t)done * n_rows * e->out_dim;
        p.q_n = n;
        p.q_rows = n_rows;
        p.q_stamp = d_stamps ? d_stamps + done : nullptr;
        cudaEvent_t a, b;
        LL_CUDA_TRY(cudaEventCreate(&a));
        LL_CUDA_TRY(cudaEventCreate(&b));
        LL_CUDA_TRY(cudaEventRecord(a, e->stream));
        rc = launch(e, p);
        if (rc) {
            cudaEventDestroy(a);
            cudaEventDestroy(b);
            return rc;
        }
        LL_CUDA_TRY(cudaEventRecord(b, e->stream));
        e->running = true;
        rc = reap(e);
        float t = 0;
        cudaEventElapsedTime(&t, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        total += t;
        done += n;
    }
    if (ms)
        *ms = total;
    // the mailbox kernel is relaunched lazily; its doorbell baseline is unchanged
    e->last_served = static_cast<ll_tick_header *>(e->mb_host)->seq_out;
    return rc;
}

}  // extern "C"
