// Register-resident kernel for deep batch-1 nets of one hidden width
// (IN -> H -> ... -> H -> OUT, NL layers; fp32 or bf16 weights), compiled per shape.
//
// The weights do not fit one cluster's register files, so the net's NL - 1 hidden layers are
// cut into NS stages of LPS consecutive layers (the last layer joins the last stage), one
// 16-CTA cluster per stage, and every weight lives in a register of its stage's CTAs for the
// whole launch: the 8.7 MB of the fp32 128 -> 512 x 9 -> 32 net take 64 registers per thread
// on 5 clusters (2 layers each), the 9 MB of the bf16 256 -> 1024 x 5 -> 64 net (two weights
// per register) 64 on 5 clusters (1 layer each).  A bf16 net computes in fp32 on bf16 inputs:
// x and every hidden output are rounded to bf16, the last layer's output is not.  Per request
// only x and the activations move:
//   stage 0  : on the mailbox rank 0 takes the request and sends it to the other CTAs' shared
//              memory (st.async, one mbarrier): a tagged slot's chunks straight from the polling
//              lanes' registers, the TickBuffer's {seq} + x from shared memory; from a
//              device queue every CTA of the stage loads x from HBM itself (no push);
//   a layer  : rows split over the cluster, R = H / C rows per CTA, RPW = R / 16 per warp:
//              lane l takes the 16-byte input pieces l, l + 32, ... for all RPW rows (a
//              quarter-warp reads 128 consecutive bytes), then a transpose-reduce over the warp
//              (deep_dot); the CTA's R outputs are staged in its shared memory and sent to
//              every CTA of the cluster by C bulk copies of 4 R bytes (alternating buffers, one
//              mbarrier each: C messages per CTA instead of one small store per warp and CTA);
//   between stages: the stage's last layer writes every output as a 64-bit word {seq, fp32}
//              (single-copy atomic) into an L2 hand-off buffer, and the next stage's threads
//              poll those words until each carries the request's number;
//   last layer: K-split over the local rows of the layer before it (no all-gather): warp w
//              owns outputs OPW w .. OPW w + OPW - 1, lane l takes local rows l, l + 32, ...;
//              the CTA's OUT partials go to rank 0 as one bulk copy, and rank 0 adds the C
//              partials in rank order, writes y and publishes.
// One request is in flight at a time: stage 0 takes request n once the last stage has
// published request n-1 (a counter), so every hand-off buffer holds one request.
// Measured (config 1, device queue): 12.4 us per request against 19.5 for the generic
// kernel's shared-memory weights on 3 clusters.  Three layers per stage (3 clusters, 98
// weights per thread) spill registers and were slower (14.1 us).
// The reference keeps layer 1 resident per thread and re-reads the rest every tick
// (src/bench_persistent_mbyv_mlp.cu:159-221), with global atomics between layers (:308-377).
#pragma once
#include <type_traits>
#include "engine_types.h"
#include "fast3_kernel.cuh"
#include "ptx.cuh"
#include "resident_kernel.cuh"
#include "ring_layers.cuh"

namespace llk {

template <int B, int E, class F>
__device__ __forceinline__ void static_for(F &&f)
{
    if constexpr (B < E) {
        f(std::integral_constant<int, B>{});
        static_for<B + 1, E>(f);
    }
}

template <int WT, int IN, int H, int OUT, int NL, int C, int LPS>
struct DeepShape {
    static constexpr int T = kThreads;
    static constexpr int NS = (NL - 1 + LPS - 1) / LPS;  // stages (clusters) over the hidden layers
    static constexpr int R = H / C;                      // rows of a hidden layer per CTA
    static constexpr int RPW = R / (T / 32);             // rows per warp
    static constexpr int S = T / R;                      // lanes holding one row's sum
    static constexpr int RL = R / 32;                    // last layer: local rows per lane
    static constexpr int OPW = OUT / (T / 32);           // last layer: outputs per warp
    static constexpr int EPR = WT == LL_W_BF16 ? 2 : 1;  // weights per 32-bit register
    static_assert(WT == LL_W_F32 || WT == LL_W_BF16, "fp32 or bf16 weights");
    static_assert(NL >= 2 && NS >= 2 && NS <= kMaxStages, "2 .. kMaxStages stages");
    static_assert(H % C == 0 && R % 32 == 0 && (RPW == 2 || RPW == 4), "2 or 4 rows per warp");
    static_assert(IN % 128 == 0 && H % 128 == 0 && H % T == 0, "16-byte pieces over a warp's 32 lanes");
    static_assert(OUT % (T / 32) == 0 && OPW >= 1 && (OPW * RL) % EPR == 0, "last-layer split");
    static_assert(C <= 32, "one lane per destination CTA");
    static_assert(IN % 4 == 0 && OUT % 4 == 0, "16-byte x and y pieces");

    static constexpr int first(int s) { return s * LPS; }
    static constexpr int last(int s) { return s == NS - 1 ? NL - 1 : (s + 1) * LPS - 1; }
    static constexpr int stage_of(int l) { return l / LPS < NS - 1 ? l / LPS : NS - 1; }
    static constexpr int kin(int l) { return l == 0 ? IN : H; }
    static constexpr int kp(int l) { return kin(l) / 128; }  // 16-byte input pieces per lane
    // weight registers per thread of layer l, and their offset in the thread's register array
    static constexpr int nw(int l) { return (l == NL - 1 ? OPW * RL : RPW * kp(l) * 4) / EPR; }
    static constexpr int woff(int l)
    {
        int o = 0;
        for (int j = first(stage_of(l)); j < l; ++j)
            o += nw(j);
        return o;
    }
    // biases of layer l held by a CTA (its rows, or all outputs of the last layer)
    static constexpr int nb(int l) { return l == NL - 1 ? OUT : R; }
    static constexpr int boff(int l)
    {
        int o = 0;
        for (int j = first(stage_of(l)); j < l; ++j)
            o += nb(j);
        return o;
    }
    static constexpr int stage_nw(int s) { return woff(last(s)) + nw(last(s)); }
    static constexpr int max_nw()
    {
        int m = 0;
        for (int s = 0; s < NS; ++s)
            m = woff(last(s)) + nw(last(s)) > m ? woff(last(s)) + nw(last(s)) : m;
        return m;
    }
    static constexpr int max_nb()
    {
        int m = 0;
        for (int s = 0; s < NS; ++s)
            m = boff(last(s)) + nb(last(s)) > m ? boff(last(s)) + nb(last(s)) : m;
        return m;
    }
    static constexpr int NW = max_nw();  // weights per thread (registers)
    static constexpr int NB = max_nb();  // biases per CTA image
    static_assert(NW <= 72, "weights per thread: 512 threads have 128 registers each");
};

// Logical weight i of a thread's register array (i must fold to a constant: the loops around
// every use are unrolled): the register itself (fp32), or half of it (bf16 pairs: element 2m
// in the low 16 bits of register m, 2m + 1 in the high).
template <int WT, int NW>
__device__ __forceinline__ float deep_w(const float (&w)[NW], int i)
{
    if constexpr (WT == LL_W_BF16) {
        const uint32_t u = __float_as_uint(w[i >> 1]);
        return __uint_as_float((i & 1) ? (u & 0xffff0000u) : (u << 16));
    } else {
        return w[i];
    }
}

// The RPW output rows of warp w (local rows RPW w .. RPW w + RPW - 1) of a row-split layer:
// lane l takes the 16-byte input pieces l, l + 32, ... (KP of them) for all RPW rows (so each
// piece read from shared memory serves every row of the warp and a warp reads the input vector
// once: 4 wavefronts per 512 bytes), with accumulators per element of a piece (NA below,
// added pairwise); then transpose-reduce rounds over masks 16 .. 32 / RPW (each lane
// keeps one row: row (lane / (32 / RPW)) of the warp) and a butterfly over the remaining masks.
// Logical weight I0 + (r KP + j) 4 + e pairs row r with piece j, element e.
template <int WT, int I0, int KP, int RPW, int NW>
__device__ __forceinline__ float deep_dot(const float (&w)[NW], const float *in, int lane)
{
    static_assert(RPW == 2 || RPW == 4, "rows per warp");
    static_assert((I0 + RPW * KP * 4 - 1) / (WT == LL_W_BF16 ? 2 : 1) < NW, "weights in the stage's array");
    // four accumulators per row for 2 rows; for 4 rows two (elements 0, 2 and 1, 3), which
    // keeps the sums and a 64-register weight slice within 128 registers
    constexpr int NA = RPW == 2 ? 4 : 2;
    const float4 *x4 = reinterpret_cast<const float4 *>(in) + lane;
    float a[RPW][4];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
        a[r][0] = a[r][1] = a[r][2] = a[r][3] = 0.f;
#pragma unroll
    for (int j = 0; j < KP; ++j) {
        const float4 v = x4[32 * j];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int i = I0 + (r * KP + j) * 4;
            a[r][0] = fmaf(deep_w<WT>(w, i), v.x, a[r][0]);
            a[r][1] = fmaf(deep_w<WT>(w, i + 1), v.y, a[r][1]);
            a[r][2 % NA] = fmaf(deep_w<WT>(w, i + 2), v.z, a[r][2 % NA]);
            a[r][3 % NA] = fmaf(deep_w<WT>(w, i + 3), v.w, a[r][3 % NA]);
        }
    }
    float t[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
        t[r] = NA == 4 ? (a[r][0] + a[r][1]) + (a[r][2] + a[r][3]) : a[r][0] + a[r][1];
    rx_round<RPW, 16>(t, lane);
    if constexpr (RPW == 4)
        rx_round<2, 8>(t, lane);
    float acc = t[0];
#pragma unroll
    for (int o = 16 / RPW; o > 0; o >>= 1)
        acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

// Stages after the first: thread t polls hand-off words t, t + kThreads, ..., its warp
// accepting its words once all are current; then the CTA barrier.  (Several loads in flight per
// word, issued a fraction of an L2 round trip apart, were measured slower: 14.0 against 13.3
// us per request.)  Returns false (the same for every thread) on abort or when the idle bound
// ran out (reported); sh.cmd is the CTA's quit flag.
template <int H>
__device__ bool deep_poll_words(const KernelCtx &k, const unsigned long long *src, float *xs, bool queue,
                                uint32_t want, uint32_t last)
{
    static_assert(H % kThreads == 0, "whole hand-off words per thread");
    constexpr int NWD = H / kThreads;
    const Params &p = *k.p;
    const int tid = threadIdx.x, lane = tid & 31;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        unsigned long long wd[NWD];
        bool cur = true;
#pragma unroll
        for (int i = 0; i < NWD; ++i)
            wd[i] = ld_relaxed_gpu_u64(src + tid + i * kThreads);
#pragma unroll
        for (int i = 0; i < NWD; ++i) {
            const uint32_t tag = (uint32_t)(wd[i] >> 32);
            cur = cur && (queue ? tag == want : (tag != 0u && tag != last));
        }
        if (__all_sync(0xffffffffu, cur)) {
#pragma unroll
            for (int i = 0; i < NWD; ++i)
                xs[tid + i * kThreads] = __uint_as_float((uint32_t)wd[i]);
            if (tid == 0)
                k.sh->xtag = (uint32_t)(wd[0] >> 32);
            break;
        }
        if ((it & 31u) == 31u) {
            int v = 0;
            if (lane == 0) {
                if (*reinterpret_cast<volatile uint32_t *>(&k.sh->abort) || global_abort(k) ||
                    *reinterpret_cast<volatile uint32_t *>(&k.sh->cmd))
                    v = 1;
                else if (globaltimer() - t0 > p.idle_ns + 2 * p.peer_margin_ns)
                    v = 2;
            }
            v = __shfl_sync(0xffffffffu, v, 0);
            if (v) {
                if (lane == 0) {
                    if (v == 2) {
                        report_error(k, LL_ERR_DEVICE_FAULT, EW_XFER);
                        broadcast_abort(k);
                    }
                    atomicOr(&k.sh->cmd, 1u);
                }
                break;
            }
        }
    }
    __syncthreads();
    return *reinterpret_cast<volatile uint32_t *>(&k.sh->cmd) == 0u;
}

template <int WT, int IN, int H, int OUT, int NL, int C, int LPS>
__global__ void __launch_bounds__(kThreads, 1) ll_deep_kernel(const __grid_constant__ Params pg)
{
    using D = DeepShape<WT, IN, H, OUT, NL, C, LPS>;
    constexpr bool kBf16 = WT == LL_W_BF16;  // x and hidden outputs rounded to bf16
    constexpr int XW = IN > H ? IN : H;
    constexpr int NYC = (OUT + 2) / 3;  // tagged y chunks
    __shared__ __align__(16) float xs[XW];      // the stage's input: x (stage 0) or the previous stage's outputs
    constexpr int NXC = (IN + 2) / 3;           // tagged chunks of x
    __shared__ __align__(16) uint4 xch[NXC];    // stage 0 peers: x's tagged chunks, forwarded by rank 0
    __shared__ __align__(16) float hb[2][H];    // all-gathered hidden vectors, alternating by layer
    __shared__ __align__(16) float hloc[D::R];  // this CTA's rows of the layer before a K-split last layer
    __shared__ __align__(16) float gath[C * OUT];  // last stage, rank 0: partials [rank][output]
    __shared__ __align__(16) float hst[D::R > OUT ? D::R : OUT];  // this CTA's outputs (or partials) to send
    __shared__ __align__(16) float yo[3 * NYC + 4];
    __shared__ __align__(16) float bias[D::NB];
    __shared__ __align__(16) Shared sh;
    __shared__ __align__(16) Params sp;
    {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&pg);
        uint32_t *dst = reinterpret_cast<uint32_t *>(&sp);
        for (int i = threadIdx.x; i < (int)(sizeof(Params) / 4); i += kThreads)
            dst[i] = src[i];
    }
    __syncthreads();
    const Params &p = sp;
    KernelCtx k;
    k.p = &p;
    k.sh = &sh;
    k.smem = nullptr;
    k.rank = cluster_ctarank();
    k.stage = (int)(blockIdx.x / (unsigned)C);
    const int stage = k.stage;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // a row-split layer: warp w computes local rows RPW w .. RPW w + RPW - 1; lane l holds row
    // g's sum, and lane sl == 0 of each group of S lanes stores it
    const int g = tid / D::S, sl = tid % D::S;
    const bool leader = stage == 0 && k.rank == 0;
    const uint32_t bar_h[2] = {smem_u32(&sh.bar[1]), smem_u32(&sh.bar[2])};
    const uint32_t bar_g = smem_u32(&sh.bar[3]);
    const uint32_t bar_diag = smem_u32(&sh.bar[4]);
    const uint32_t bar_req = smem_u32(&sh.bar[5]);

    if (tid == 0) {
        for (int i = 0; i < 7; ++i)
            mbar_init(smem_u32(&sh.bar[i]), 1);
        sh.cmd = 0;
        sh.fail = 0;
        sh.abort = 0;
        sh.hstop = 0;
        sh.xtag = 0;
        fence_mbar_init_cluster();
        if (leader)
            st_relaxed_sys_u32(&p.ctrl->state, ST_LOADING);
    }
    // ---- biases into SMEM (the weights go to registers in the stage's own loop below) ----
    const float *img = reinterpret_cast<const float *>(p.image + (size_t)blockIdx.x * p.image_stride);
    for (int i = tid; i < D::NB; i += kThreads)
        bias[i] = __ldg(img + (size_t)D::NW * kThreads + i);
    for (int i = tid; i < C * OUT; i += kThreads)
        gath[i] = 0.0f;
    for (int i = tid; i < 3 * NYC + 4; i += kThreads)
        yo[i] = 0.0f;
    // The request loop is compiled once per stage (stage s as a constant): only the stage's own
    // weights are live in registers, and each stage carries only the code it runs.
    uint32_t n_done = 0;
    auto serve = [&](auto sc) {
        constexpr int s = decltype(sc)::value;
        // ---- the stage's weights into registers (image [NW][T] per CTA, coalesced) ----
        float w[D::stage_nw(s)];
#pragma unroll
        for (int j = 0; j < D::stage_nw(s); ++j)
            w[j] = ld_once_f32(img + (size_t)j * kThreads + tid);  // volatile: never re-issued later
        __syncthreads();
        cluster_sync();
        if (leader && tid == 0)
            st_relaxed_sys_u32(&p.ctrl->state, ST_RUNNING);

        bool ok = true;
        if (p.diag_wait_never && leader)
            ok = cta_wait_bar(k, bar_diag, 0, EW_DIAG, p.step_ns);

        uint32_t last = p.last_seq, ph_req = 0, ph_g = 0;
        uint32_t ph_h[2] = {0, 0};
        const uint32_t x_addr = smem_u32(xs), h_addr = smem_u32(sh.hdr);

        while (ok) {
            if (p.mode == MODE_QUEUE && (int)n_done >= p.q_n)
                break;  // every stage knows the queue length
            uint32_t seq;
            // ---------------- 1. the stage's input ----------------
            // Device queue: every CTA of stage 0 takes the request itself (x from HBM), so x
            // needs no push between them; on the mailbox rank 0 takes it and pushes x.
            if (s == 0 && (k.rank == 0 || p.mode == MODE_QUEUE)) {
                if (n_done > 0) {
                    // the last stage has published request n_done - 1 (bounded wait)
                    if (tid == 0) {
                        const uint64_t deadline = globaltimer() + p.step_ns;
                        uint32_t it = 0;
                        while (ld_acquire_gpu(p.q_done) < n_done) {
                            if ((++it & 31u) == 0 && (global_abort(k) || globaltimer() > deadline)) {
                                if (!global_abort(k)) {
                                    report_error(k, LL_ERR_DEVICE_FAULT, EW_QUEUE_GO);
                                    broadcast_abort(k);
                                }
                                sh.fail = 1;
                                break;
                            }
                        }
                    }
                    __syncthreads();
                    if (*reinterpret_cast<volatile uint32_t *>(&sh.fail))
                        break;
                }
                if (p.mode == MODE_QUEUE) {
                    if (tid == 0) {
                        sh.cmd = n_done + 1u;
                        if (k.rank == 0)
                            trace(k, n_done, 0);
                    }
                    if (tid < IN / 4) {
                        float4 v = __ldg(reinterpret_cast<const float4 *>(p.q_x + (size_t)n_done * IN) + tid);
                        if constexpr (kBf16)
                            v = make_float4(round_bf16(v.x), round_bf16(v.y), round_bf16(v.z), round_bf16(v.w));
                        reinterpret_cast<float4 *>(xs)[tid] = v;
                    }
                } else if (p.mailbox_format == 1) {
                    if (warp == 0) {
                        // the polling lanes forward the chunks to the peers straight from registers
                        // (with the header {seq, 1}, on the peers' request barrier)
                        const ChunkFwd fwd{smem_u32(xch), h_addr, bar_req, bar_req, 1, C - 1, 0};
                        const uint32_t c = poll_tagged(k, last, xs, ring_slot(p, n_done), nullptr, &fwd);
                        if (lane == 0) {
                            if (c == kCmdExit)
                                broadcast_abort(k);
                            sh.cmd = c;
                            trace(k, n_done, 0);
                        }
                    }
                } else {
                    if (tid == 0) {
                        const uint32_t c = poll_mailbox(k, last);
                        if (c == kCmdExit)
                            broadcast_abort(k);
                        sh.cmd = c;
                        trace(k, n_done, 0);
                    }
                    __syncthreads();
                    // batch 1: no header fetch (n_rows is 1; stop is seen on the idle cadence)
                    if (*reinterpret_cast<volatile uint32_t *>(&sh.cmd) != kCmdExit && tid < IN / 4) {
                        float4 v = ld_relaxed_sys_v4(p.mb_x + 4 * tid);
                        if constexpr (kBf16)
                            v = make_float4(round_bf16(v.x), round_bf16(v.y), round_bf16(v.z), round_bf16(v.w));
                        reinterpret_cast<float4 *>(xs)[tid] = v;
                    }
                }
                __syncthreads();
                seq = *reinterpret_cast<volatile uint32_t *>(&sh.cmd);
                if (seq == kCmdExit)
                    break;
                if (tid == 0 && k.rank == 0)
                    trace(k, n_done, 1);
                // {seq} + x into the other CTAs of the stage: (C - 1) (1 + IN / 4) stores of 16 bytes
                constexpr int per = 1 + IN / 4;
                const bool push = p.mode == MODE_MAILBOX && p.mailbox_format == 0;  // (tagged: forwarded)
                for (int i = tid; push && i < (C - 1) * per; i += kThreads) {
                    const uint32_t d = 1u + (uint32_t)(i / per);
                    const int j = i % per;
                    if (j == 0)
                        st_async_v4(mapa(h_addr, d), make_float4(__uint_as_float(seq), __uint_as_float(1u), 0.f, 0.f),
                                    mapa(bar_req, d));
                    else
                        st_async_v4(mapa(x_addr + (uint32_t)(j - 1) * 16u, d), reinterpret_cast<const float4 *>(xs)[j - 1],
                                    mapa(bar_req, d));
                }
                if (tid == 0 && k.rank == 0)
                    trace(k, n_done, 2);
            } else if (s == 0) {
                if (tid == 0)
                    mbar_arrive_expect_tx(bar_req, 16u + (p.mailbox_format == 1 ? 16u * NXC : 4u * IN));
                if (!cta_wait_bar(k, bar_req, ph_req & 1u, EW_PEER_POLL, p.idle_ns + p.peer_margin_ns))
                    break;
                ++ph_req;
                seq = *reinterpret_cast<volatile uint32_t *>(&sh.hdr[0]);
                if (p.mailbox_format == 1) {
                    // unpack the forwarded {v0, v1, v2, tag} chunks into x (rounded to bf16 for a
                    // bf16 net, as rank 0's poll does)
                    for (int ch = tid; ch < NXC; ch += kThreads) {
                        const uint4 v = xch[ch];
                        const float f[3] = {__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z)};
#pragma unroll
                        for (int e = 0; e < 3; ++e)
                            if (3 * ch + e < IN)
                                xs[3 * ch + e] = kBf16 ? round_bf16(f[e]) : f[e];
                    }
                }
            } else {
                // The previous stage's outputs arrive as words {seq, fp32} (deep_poll_words).
                // Queue mode numbers requests 1, 2, ... per launch (the words are cleared at every
                // launch).  On the mailbox the number is the host's sequence number, which a
                // hand-driven host may advance by more than one: a word is current when its tag is
                // neither 0 nor `last` (the request this stage served before); with one request in
                // flight, once every word is current they all carry the same number, read from
                // word 0.
                const bool queue = p.mode == MODE_QUEUE;
                const unsigned long long *src =
                    reinterpret_cast<const unsigned long long *>(p.xfer + (size_t)(stage - 1) * p.xfer_stride);
                if (!deep_poll_words<H>(k, src, xs, queue, n_done + 1u, last))
                    break;
                seq = *reinterpret_cast<volatile uint32_t *>(&sh.xtag);  // written before the barrier above
            }
            __syncthreads();

            // ---------------- 2. this stage's layers ----------------
            {
                static_for<D::first(s), D::last(s) + 1>([&](auto lc) {
                    constexpr int l = decltype(lc)::value;
                    if (!ok)
                        return;
                    constexpr bool head = l == D::first(s);  // reads the stage's input
                    const float *in = head ? xs : hb[(l - 1) & 1];
                    if constexpr (l == NL - 1) {
                        // K-split over this CTA's local rows of the previous layer's output: lane l
                        // takes local rows l, l + 32, ... (logical weight o RL + j: output
                        // OPW w + o, local row l + 32 j), then a butterfly per output
                        const float *hin = head ? xs + k.rank * D::R : hloc;
                        float t[D::OPW];
#pragma unroll
                        for (int o = 0; o < D::OPW; ++o) {
                            t[o] = 0.f;
#pragma unroll
                            for (int j = 0; j < D::RL; ++j)
                                t[o] = fmaf(deep_w<WT>(w, D::woff(l) * D::EPR + o * D::RL + j), hin[lane + 32 * j],
                                            t[o]);
                        }
#pragma unroll
                        for (int m = 16; m > 0; m >>= 1)
#pragma unroll
                            for (int o = 0; o < D::OPW; ++o)
                                t[o] += __shfl_xor_sync(0xffffffffu, t[o], m);
                        // the CTA's OUT partials, staged, then one bulk copy to rank 0 (hst is free: its
                        // last copy was read before the issuing thread passed a CTA barrier since)
                        if (lane == 0) {
#pragma unroll
                            for (int o = 0; o < D::OPW; ++o)
                                hst[D::OPW * warp + o] = t[o];
                            fence_proxy_async_shared();  // visible to the bulk copy
                        }
                        __syncthreads();
                        if (tid == 0) {
                            bulk_s2peer(mapa(smem_u32(&gath[k.rank * OUT]), 0u), smem_u32(hst), (uint32_t)(OUT * 4),
                                        mapa(bar_g, 0u));
                            bulk_commit_group();
                            bulk_wait_group_read<0>();  // hst may be written again after the next barrier
                        }
                        if (k.rank == 0 && tid == 0 && l < 10)
                            trace(k, n_done, 3 + l);
                    } else {
                        const float acc = deep_dot<WT, D::woff(l) * D::EPR, D::kp(l), D::RPW>(w, in, lane);
                        float v = relu_or(acc + bias[D::boff(l) + g], p.L[l].act);
                        if constexpr (kBf16)
                            v = round_bf16(v);  // a hidden output
                        if constexpr (l + 1 == NL - 1 && l + 1 <= D::last(s)) {
                            // the last layer follows in this stage: it reads this CTA's rows only
                            if (sl == 0)
                                hloc[g] = v;
                            __syncthreads();
                        } else if constexpr (l == D::last(s)) {
                            // to the next stage through L2: one word {seq, value} per row
                            if (sl == 0) {
                                unsigned long long *dw =
                                    reinterpret_cast<unsigned long long *>(p.xfer + (size_t)s * p.xfer_stride);
                                st_relaxed_gpu_u64(dw + k.rank * D::R + g,
                                                   ((unsigned long long)seq << 32) | __float_as_uint(v));
                            }
                        } else {
                            // all-gather: the CTA's R outputs, staged, then one bulk copy of 4 R bytes
                            // into every CTA of the cluster (lane d of warp 0 serves CTA d)
                            constexpr int b = l & 1;
                            if (sl == 0) {
                                hst[g] = v;
                                fence_proxy_async_shared();  // visible to the bulk copies
                            }
                            if (tid == 0)
                                mbar_arrive_expect_tx(bar_h[b], (uint32_t)(H * 4));
                            __syncthreads();
                            if (tid < C) {
                                bulk_s2peer(mapa(smem_u32(&hb[b][k.rank * D::R]), (uint32_t)tid), smem_u32(hst),
                                            (uint32_t)(D::R * 4), mapa(bar_h[b], (uint32_t)tid));
                                bulk_commit_group();
                                bulk_wait_group_read<0>();  // hst is free again once the wait below has
                                                            // passed its CTA barrier
                            }
                            ok = cta_wait_bar(k, bar_h[b], ph_h[b] & 1u, EW_LAYER_BASE + (uint32_t)l, p.step_ns);
                            ++ph_h[b];
                        }
                        if (k.rank == 0 && tid == 0 && l < 10)
                            trace(k, n_done, 3 + l);
                    }
                });
            }
            if (!ok)
                break;

            // ---------------- 3. rank 0 of the last stage publishes ----------------
            if (s == D::NS - 1 && k.rank == 0) {
                if (tid == 0)
                    mbar_arrive_expect_tx(bar_g, (uint32_t)(C * OUT * 4));
                ok = cta_wait_bar(k, bar_g, ph_g & 1u, EW_GATHER, p.step_ns);
                ++ph_g;
                if (!ok)
                    break;
                if (warp == 0) {
                    constexpr int lb = D::boff(NL - 1);
                    const int act = p.L[NL - 1].act;
                    for (int o = lane; o < OUT; o += 32) {
                        float v = 0.f;
#pragma unroll
                        for (int c = 0; c < C; ++c)
                            v += gath[c * OUT + o];
                        yo[o] = relu_or(v + bias[lb + o], act);
                    }
                    __syncwarp();
                    if (p.mode == MODE_MAILBOX && p.mailbox_format == 1) {
                        // tagged output: chunk c = {y[3c], y[3c+1], y[3c+2], seq}, relaxed stores, no fence
                        float *dst = p.mb_y + (size_t)ring_slot(p, n_done) * p.ring_ystride_f;
                        for (int c = lane; c < NYC; c += 32)
                            st_relaxed_sys_v4(dst + 4 * c,
                                              make_float4(yo[3 * c], yo[3 * c + 1], yo[3 * c + 2], __uint_as_float(seq)));
                    } else {
                        for (int c = lane; c < OUT / 4; c += 32) {
                            const float4 q = reinterpret_cast<const float4 *>(yo)[c];
                            if (p.mode == MODE_QUEUE)
                                reinterpret_cast<float4 *>(p.q_y + (size_t)n_done * OUT)[c] = q;
                            else
                                st_relaxed_sys_v4(p.mb_y + 4 * c, q);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) {
                        trace(k, n_done, 13);
                        if (p.mode == MODE_QUEUE) {
                            if (p.q_stamp)
                                p.q_stamp[n_done] = globaltimer();
                        } else if (p.mailbox_format == 1) {
                            st_relaxed_sys_u32(&p.mb->seq_out, seq);  // bookkeeping only: the host waits on the tags
                        } else {
                            // release: y reaches the host before seq_out (src/bench_persistent_mbyv_mlp.cu:365-370)
                            st_release_sys_u32(&p.mb->seq_out, seq);
                        }
                        // stage 0 may take the next request: a plain counter (stage 0 reads nothing this
                        // stage wrote; every CTA of the pipeline is past request n_done by now)
                        atomicAdd(p.q_done, 1u);
                        trace(k, n_done, 14);
                    }
                }
            }
            last = seq;
            ++n_done;
        }
    };
    static_for<0, D::NS>([&](auto sc) {
        if (stage == decltype(sc)::value)
            serve(sc);
    });

    // Leave together: no CTA may exit while a peer can still write its shared memory (and no
    // bulk copy of this CTA is still in flight).
    if (warp == 0)
        bulk_wait_group_all();
    __syncthreads();
    cluster_sync();
    if (leader && tid == 0) {
        st_relaxed_sys_u32(&p.ctrl->passes, n_done);
        st_relaxed_sys_u32(&p.ctrl->rows, n_done);
        if (p.mode == MODE_QUEUE)
            st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_QUEUE_DONE);
        st_release_sys_u32(&p.ctrl->state, ST_EXITED);
    }
}

}  // namespace llk
