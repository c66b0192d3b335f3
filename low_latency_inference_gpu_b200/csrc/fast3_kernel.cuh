// Register-resident resident kernel for 3-layer fp32 nets (IN -> H1 -> H2 -> OUT),
// batch 1, compiled per shape.
//
// Every weight lives in a register for the whole launch (the register file is
// 256 KB per SM; a cluster of C CTAs holds the net), so per request only x and
// the activations move, through shared memory and DSMEM:
//   request : rank 0 polls the mailbox (the header with one 16-byte acquire load, or
//             the tagged slot, whose chunks carry x), reads x once and pushes {seq, x}
//             into every peer's shared memory (st.async, one mbarrier); in queue mode
//             every CTA loads x from HBM and rank 0 sends each peer a 16-byte go {seq}
//             that the peer waits for before its layer-3 partial;
//   layer 1 : replicated in every CTA, S1 = T/H1 threads per row, K1 = IN/S1 weights
//             per thread, butterfly over the S1 lanes;
//   layer 2 : rows split over the cluster (R2 = H2/C per CTA), S2 = T/R2 threads per
//             row, K2 = H1/S2 weights per thread;
//   (lane s of a row group takes the 16-byte input pieces s, s+S, s+2S, ... so the
//   eight lanes of a quarter-warp read 128 consecutive bytes: no bank conflicts)
//   layer 3 : K-split over the local R2 rows: warp w owns output w, lane l takes local
//             rows l, l+32, ...; one partial per output is pushed to rank 0, which adds the C
//             partials in rank order, writes y and release-stores seq_out.
// The reference's closest kernel keeps only layer 1 resident (registers / SMEM /
// global scratch per thread, src/bench_persistent_mbyv_mlp.cu:159-221) and re-reads
// the rest every tick; its layer barriers are global atomics (:308-377).
#pragma once
#include <type_traits>
#include "engine_types.h"
#include "ptx.cuh"
#include "resident_kernel.cuh"

namespace llk {

// Rows one pass of the register-resident kernel can carry: requests taken together from
// the ring (micro-batching).  A pass over 2..16 rows runs the 4-row code over groups of 4
// rows, each weight held in a register used once per row in the same FMA order as for a
// request alone (so replies are bit-identical to single requests).  Shapes whose weights
// leave fewer than ~70 registers free (more than 56 weights per thread) carry one row: the
// 4-row accumulators would spill.
constexpr int kFast3Rows = 16;
constexpr int kFast3Group = 4;

template <int IN, int H1, int H2, int OUT, int C>
struct Fast3Shape {
    static constexpr int T = kThreads;
    static constexpr int S1 = T / H1;
    static constexpr int K1 = IN / S1;
    static constexpr int R2 = H2 / C;
    static constexpr int S2 = T / R2;
    static constexpr int K2 = H1 / S2;
    static constexpr int K3 = R2 / 32;
    static constexpr int NW = K1 + K2 + K3;  // weights per thread
    static_assert(T % H1 == 0 && IN % S1 == 0 && K1 % 4 == 0, "layer-1 split");
    static_assert(H2 % C == 0 && T % R2 == 0 && H1 % S2 == 0 && K2 % 4 == 0, "layer-2 split");
    static_assert(R2 % 32 == 0 && K3 >= 1, "layer-3 split");
    static_assert(OUT >= 1 && OUT <= T / 32 && OUT % 4 == 0, "one warp per output, float4 stores");
    static_assert(S1 <= 32 && S2 <= 32 && (S1 & (S1 - 1)) == 0 && (S2 & (S2 - 1)) == 0, "butterfly groups");
    static_assert(IN % 4 == 0, "x is moved in 16-byte pieces");
    static constexpr int NB = H1 + R2 + OUT;  // biases per CTA image
    static constexpr int MaxRows = NW <= 56 ? kFast3Rows : 1;
    static_assert(MaxRows <= T / 32, "rank 0 finishes one row per warp");
    static_assert(MaxRows == 1 || MaxRows % kFast3Group == 0, "rows come in groups");
};

__device__ __forceinline__ float relu_or(float v, int act)
{
    return act == LL_ACT_RELU ? fmaxf(v, 0.0f) : (act == LL_ACT_GELU ? act_apply(v, LL_ACT_GELU) : v);
}

// The three layers of one pass, shared by the register-resident kernel and the pipelined
// ring kernel (ring_kernel.cuh).  Rows are walked in ng groups of GR (rows past the last
// request of the pass compute on stale inputs inside the buffers and are never sent or
// stored); per row the FMA order is the same for every GR, so a request's reply does not
// depend on how many rows its pass carried.
//
// Layer 1, replicated in every CTA: h1[row][r1] = act(W1[r1] . x[row] + b1[r1]); S1 threads
// per output row, lane s1 of a row group takes the 16-byte input pieces s1, s1 + S1, ...
// (a0, a1) += (w.x * v.x, w.y * v.y): one packed instruction of two independent IEEE fp32 FMAs
// when PACKED, else two scalar FMAs; each accumulator sees the same rounding either way.
template <bool PACKED>
__device__ __forceinline__ void fma_pair(float &a0, float &a1, float w0, float w1, float v0, float v1)
{
    if constexpr (PACKED) {
        const float2 r = __ffma2_rn(make_float2(w0, w1), make_float2(v0, v1), make_float2(a0, a1));
        a0 = r.x;
        a1 = r.y;
    } else {
        a0 = fmaf(w0, v0, a0);
        a1 = fmaf(w1, v1, a1);
    }
}

template <class S, int GR, int IN, int H1, bool PACKED = false>
__device__ __forceinline__ void f3_layer1(const float (&w1)[S::K1], const float *xs, float *h1, const float *b1,
                                          int ng, int r1, int s1, int act)
{
    for (int g = 0; g < ng; ++g) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xs + g * GR * IN) + s1;
        float a0[GR], a1[GR];
#pragma unroll
        for (int r = 0; r < GR; ++r)
            a0[r] = a1[r] = 0.f;
#pragma unroll
        for (int j = 0; j < S::K1 / 4; ++j) {
#pragma unroll
            for (int r = 0; r < GR; ++r) {
                const float4 v = x4[r * (IN / 4) + j * S::S1];
                if constexpr (PACKED) {
                    fma_pair<true>(a0[r], a1[r], w1[4 * j], w1[4 * j + 1], v.x, v.y);
                    fma_pair<true>(a0[r], a1[r], w1[4 * j + 2], w1[4 * j + 3], v.z, v.w);
                } else {
                    a0[r] = fmaf(w1[4 * j], v.x, a0[r]);
                    a1[r] = fmaf(w1[4 * j + 1], v.y, a1[r]);
                    a0[r] = fmaf(w1[4 * j + 2], v.z, a0[r]);
                    a1[r] = fmaf(w1[4 * j + 3], v.w, a1[r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < GR; ++r) {
            float acc = a0[r] + a1[r];
#pragma unroll
            for (int o = S::S1 / 2; o > 0; o >>= 1)
                acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (s1 == 0)
                h1[(g * GR + r) * H1 + r1] = relu_or(acc + b1[r1], act);
        }
    }
}

// Layer 2, rows split over the cluster: h2[row][r2] = act(W2[local row r2] . h1[row] + b2[r2]).
template <class S, int GR, int H1, bool PACKED = false>
__device__ __forceinline__ void f3_layer2(const float (&w2)[S::K2], const float *h1, float *h2, const float *b2,
                                          int ng, int r2, int s2, int act)
{
    for (int g = 0; g < ng; ++g) {
        const float4 *v4 = reinterpret_cast<const float4 *>(h1 + g * GR * H1) + s2;
        float a0[GR], a1[GR];
#pragma unroll
        for (int r = 0; r < GR; ++r)
            a0[r] = a1[r] = 0.f;
#pragma unroll
        for (int j = 0; j < S::K2 / 4; ++j) {
#pragma unroll
            for (int r = 0; r < GR; ++r) {
                const float4 v = v4[r * (H1 / 4) + j * S::S2];
                if constexpr (PACKED) {
                    fma_pair<true>(a0[r], a1[r], w2[4 * j], w2[4 * j + 1], v.x, v.y);
                    fma_pair<true>(a0[r], a1[r], w2[4 * j + 2], w2[4 * j + 3], v.z, v.w);
                } else {
                    a0[r] = fmaf(w2[4 * j], v.x, a0[r]);
                    a1[r] = fmaf(w2[4 * j + 1], v.y, a1[r]);
                    a0[r] = fmaf(w2[4 * j + 2], v.z, a0[r]);
                    a1[r] = fmaf(w2[4 * j + 3], v.w, a1[r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < GR; ++r) {
            float acc = a0[r] + a1[r];
#pragma unroll
            for (int o = S::S2 / 2; o > 0; o >>= 1)
                acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (s2 == 0)
                h2[(g * GR + r) * S::R2 + r2] = relu_or(acc + b2[r2], act);
        }
    }
}

// One round of a transpose-reduce: N values per lane become N/2, summed with the lane's
// partner l ^ M; the lane whose bit M is clear keeps values [0, N/2), the other [N/2, N).
// Each kept value is own + partner, exactly the pair a butterfly step with mask M adds, so
// after the rounds of masks S/2, S/4, ..., 1 over N = S values every lane holds the same
// sum a butterfly would have given for its row: bit-identical, with N - 1 shuffles instead
// of N log2(S).
template <int N, int M>
__device__ __forceinline__ void xreduce_round(float (&t)[16], int lane)
{
    const bool upper = (lane & M) != 0;
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        const float give = upper ? t[i] : t[i + N / 2];
        const float keep = upper ? t[i + N / 2] : t[i];
        t[i] = keep + __shfl_xor_sync(0xffffffffu, give, M);
    }
}

// Layer 2 over 16 batch rows at once (S2 = 16 lanes per output row): the products as in
// f3_layer2, then a transpose-reduce over the row's 16 lanes, after which lane s2 holds batch
// row s2's sum.  Bit-identical to f3_layer2.
template <class S, int H1, bool PACKED>
__device__ __forceinline__ void f3_layer2_x16(const float (&w2)[S::K2], const float *h1, float *h2, const float *b2,
                                              int r2, int s2, int act)
{
    static_assert(S::S2 == 16, "one batch row per lane of the row group");
    const float4 *v4 = reinterpret_cast<const float4 *>(h1) + s2;
    float t[16];
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // 8 rows at a time: fewer accumulators live
        float a0[8], a1[8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
            a0[r] = a1[r] = 0.f;
#pragma unroll
        for (int j = 0; j < S::K2 / 4; ++j) {
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const float4 v = v4[(8 * half + r) * (H1 / 4) + j * S::S2];
                if constexpr (PACKED) {
                    fma_pair<true>(a0[r], a1[r], w2[4 * j], w2[4 * j + 1], v.x, v.y);
                    fma_pair<true>(a0[r], a1[r], w2[4 * j + 2], w2[4 * j + 3], v.z, v.w);
                } else {
                    a0[r] = fmaf(w2[4 * j], v.x, a0[r]);
                    a1[r] = fmaf(w2[4 * j + 1], v.y, a1[r]);
                    a0[r] = fmaf(w2[4 * j + 2], v.z, a0[r]);
                    a1[r] = fmaf(w2[4 * j + 3], v.w, a1[r]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r)
            t[8 * half + r] = a0[r] + a1[r];
    }
    const int lane = threadIdx.x & 31;
    xreduce_round<16, 8>(t, lane);
    xreduce_round<8, 4>(t, lane);
    xreduce_round<4, 2>(t, lane);
    xreduce_round<2, 1>(t, lane);
    h2[s2 * S::R2 + r2] = relu_or(t[0] + b2[r2], act);  // lane s2 holds batch row s2
}

// Layer 3 over 16 batch rows at once: after the transpose-reduce over 32 lanes (masks 16, 8,
// 4, 2, then a last butterfly step with mask 1) lanes 2r and 2r + 1 hold batch row r's
// partial; lane r returns row r's (bit-identical to f3_layer3).
template <class S>
__device__ __forceinline__ float f3_layer3_x16(const float (&w3)[S::K3], const float *h2, int lane)
{
    float t[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < S::K3; ++j)
            acc = fmaf(w3[j], h2[r * S::R2 + lane + 32 * j], acc);
        t[r] = acc;
    }
    xreduce_round<16, 16>(t, lane);
    xreduce_round<8, 8>(t, lane);
    xreduce_round<4, 4>(t, lane);
    xreduce_round<2, 2>(t, lane);
    t[0] += __shfl_xor_sync(0xffffffffu, t[0], 1);
    return __shfl_sync(0xffffffffu, t[0], (2 * lane) & 31);
}

// Layer 3, K-split over the CTA's R2 rows of h2: the warp that owns an output returns, in lane
// r < rows, row r's partial sum over this CTA's slice (lane l takes local rows l, l + 32, ...).
template <class S, int GR>
__device__ __forceinline__ float f3_layer3(const float (&w3)[S::K3], const float *h2, int rows, int lane)
{
    float mine = 0.f;
    for (int r = 0; r < (GR == 1 ? 1 : rows); ++r) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < S::K3; ++j)
            acc = fmaf(w3[j], h2[r * S::R2 + lane + 32 * j], acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == r)
            mine = acc;
    }
    return mine;
}

template <int IN, int H1, int H2, int OUT, int C>
__global__ void __launch_bounds__(kThreads, 1) ll_fast3_kernel(const __grid_constant__ Params pg)
{
    using S = Fast3Shape<IN, H1, H2, OUT, C>;
    constexpr int MB = S::MaxRows;
    constexpr int YO = 3 * ((OUT + 2) / 3) + 4;  // one output row, zero-padded
    __shared__ __align__(16) float xs[MB * IN];
    __shared__ __align__(16) float h1[MB * H1];
    __shared__ __align__(16) float h2[MB * S::R2];
    __shared__ __align__(16) float gath[MB * C * OUT];  // [row][rank][output]
    __shared__ __align__(16) float yo[MB * YO];
    __shared__ uint32_t rseq[MB];  // rank 0: sequence number of each row taken together
    __shared__ uint32_t bad_words[kTagReadWarpsMax];  // rank 0: incomplete-row masks of a multi-slot read
    // rank 0: the host had posted beyond the last request taken.  Indexed by pass parity: warp 0
    // sets the flag for the next pass while the other reading warps may still read this pass's.
    __shared__ uint32_t s_backlog[2];
    constexpr int NXC = (IN + 2) / 3;  // tagged chunks per row
    __shared__ __align__(16) uint4 xch[MB * NXC];  // peers: the tagged chunks rank 0 forwards
    __shared__ __align__(16) float bias[S::NB];
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
    k.stage = 0;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool leader = k.rank == 0;
    const uint32_t bar_req = smem_u32(&sh.bar[5]);
    const uint32_t bar_g = smem_u32(&sh.bar[3]);
    const uint32_t bar_diag = smem_u32(&sh.bar[4]);
    const uint32_t bar_x = smem_u32(&sh.bar[6]);
    const int act1 = p.L[0].act, act2 = p.L[1].act, act3 = p.L[2].act;

    if (tid == 0) {
        for (int i = 0; i < 7; ++i)
            mbar_init(smem_u32(&sh.bar[i]), 1);
        sh.cmd = 0;
        sh.fail = 0;
        sh.abort = 0;
        sh.hstop = 0;
        s_backlog[0] = s_backlog[1] = 0;
        fence_mbar_init_cluster();
        if (leader)
            st_relaxed_sys_u32(&p.ctrl->state, ST_LOADING);
    }
    // ---- weights into registers (coalesced: image is [NW][T] floats per CTA), biases into SMEM ----
    const float *img = reinterpret_cast<const float *>(p.image + (size_t)blockIdx.x * p.image_stride);
    // volatile loads: the compiler may not re-issue them later, so the weights stay in registers
    float w1[S::K1], w2[S::K2], w3[S::K3];
#pragma unroll
    for (int j = 0; j < S::K1; ++j)
        w1[j] = ld_once_f32(img + (size_t)j * kThreads + tid);
#pragma unroll
    for (int j = 0; j < S::K2; ++j)
        w2[j] = ld_once_f32(img + (size_t)(S::K1 + j) * kThreads + tid);
#pragma unroll
    for (int j = 0; j < S::K3; ++j)
        w3[j] = ld_once_f32(img + (size_t)(S::K1 + S::K2 + j) * kThreads + tid);
    for (int i = tid; i < S::NB; i += kThreads)
        bias[i] = __ldg(img + (size_t)S::NW * kThreads + i);
    for (int i = tid; i < MB * C * OUT; i += kThreads)
        gath[i] = 0.0f;
    for (int i = tid; i < MB * YO; i += kThreads)
        yo[i] = 0.0f;
    __syncthreads();
    cluster_sync();
    if (leader && tid == 0)
        st_relaxed_sys_u32(&p.ctrl->state, ST_RUNNING);

    bool ok = true;
    if (p.diag_wait_never && leader)
        ok = cta_wait_bar(k, bar_diag, 0, EW_DIAG, p.step_ns);

    const int r1 = tid / S::S1, s1 = tid % S::S1;
    const int r2 = tid / S::S2, s2 = tid % S::S2;
    const uint32_t x_addr = smem_u32(xs), h_addr = smem_u32(sh.hdr), g_addr = smem_u32(gath);
    uint32_t last = p.last_seq, n_done = 0, ph_req = 0, ph_g = 0, ph_x = 0, passes = 0;
    // warps of rank 0 that read a multi-slot batch (whole slots per warp)
    constexpr int NXC_ = (IN + 2) / 3;
    constexpr int RPW = tag_rows_per_warp(NXC_);
    static_assert(RPW >= 1, "a reading warp holds at least one slot");
    const int read_warps = p.micro_batch > 1 ? (p.micro_batch + RPW - 1) / RPW : 1;

    while (ok) {
        uint32_t seq, nb = 1;
        if (p.mode == MODE_QUEUE && (int)n_done >= p.q_n)
            break;
        // ---------------- request ----------------
        // Queue mode: every CTA loads x itself from HBM, so x is not pushed over DSMEM.  Rank 0
        // sends each peer a 16-byte go {seq} once it has started the request (and so has
        // finished the previous one); a peer waits for it before its layer-3 partial, so a
        // peer that runs ahead never overwrites partials rank 0 still reads.  (On the
        // mailbox every CTA polling host memory over PCIe made the requests 4x slower, so
        // there rank 0 alone polls and pushes x.)
        const bool own_x = p.mode == MODE_QUEUE;
        if (own_x) {
            seq = n_done + 1;
            if (tid == 0) {
                if (leader)
                    trace(k, n_done, 0);
                else
                    mbar_arrive_expect_tx(bar_req, 16u);
            }
            const float *src = p.q_x + (size_t)n_done * IN;
            if (tid < IN / 4)
                reinterpret_cast<float4 *>(xs)[tid] = __ldg(reinterpret_cast<const float4 *>(src) + tid);
            __syncthreads();
            if (leader && tid > 0 && tid < C)
                st_async_v4(mapa(h_addr, (uint32_t)tid), make_float4(__uint_as_float(seq), 0.f, 0.f, 0.f),
                            mapa(bar_req, (uint32_t)tid));
            if (leader && tid == 0)
                trace(k, n_done, 1);
        } else if (leader) {
            if (p.mailbox_format == 1) {
                if (warp < read_warps) {
                    // x arrives with the doorbell.  On a micro-batched ring the poll also reads
                    // the host's seq_in (the last sequence number posted); when it is ahead of
                    // the request just taken, requests are waiting, and the next pass takes up to
                    // micro_batch of them with one read of their slots (warps 0..read_warps-1,
                    // whole slots each).  Otherwise (and when that read finds nothing) warp 0's
                    // single-slot poll waits for the next request: a read spanning several slots
                    // was measured ~2 us slower to see a new request.
                    // The polling lanes forward the raw chunks to the peers from registers as
                    // soon as the tags match (header {seq, rows} + row 0 on the peers' request
                    // barrier, rows 1.. on their x barrier).
                    const ChunkFwd fwd{smem_u32(xch), h_addr, bar_req, bar_x, 1, C - 1, 0};
                    uint32_t c = 0, posted = 0;
                    int got = 0;
                    if constexpr (MB > 1) {
                        // written by warp 0 during the previous pass, before its barriers
                        if (*reinterpret_cast<volatile uint32_t *>(&s_backlog[passes & 1u]))
                            got = take_tagged_rows(k, last, xs, n_done, p.micro_batch, rseq, &posted, bad_words,
                                                   read_warps, &fwd);
                    }
                    if (warp == 0) {
                        if (got > 0) {
                            c = seq_after(last, got);
                        } else {
                            c = poll_tagged(k, last, xs, ring_slot(p, n_done), p.micro_batch > 1 ? &posted : nullptr,
                                            &fwd);
                            got = 1;
                        }
                        if (tid == 0) {
                            s_backlog[(passes + 1u) & 1u] =
                                (p.micro_batch > 1 && c != kCmdExit && (int32_t)(posted - c) > 0) ? 1u : 0u;
                            sh.nrows = (uint32_t)got;
                            if (c == kCmdExit)
                                broadcast_abort(k);
                            sh.cmd = c;
                            trace(k, n_done, 0);
                        }
                    }
                }
            } else if (tid == 0) {
                const uint32_t c = poll_mailbox(k, last);
                if (c == kCmdExit)
                    broadcast_abort(k);
                sh.cmd = c;
                trace(k, n_done, 0);
            }
            __syncthreads();
            seq = *reinterpret_cast<volatile uint32_t *>(&sh.cmd);
            if (seq == kCmdExit)
                break;
            if (p.mailbox_format == 1)
                nb = *reinterpret_cast<volatile uint32_t *>(&sh.nrows);
            // batch 1: no header fetch (n_rows is 1; stop is seen on the idle cadence, so a
            // stop that comes with a doorbell bump costs one extra, harmless reply)
            if (p.mailbox_format == 0) {
                if (tid < IN / 4)
                    reinterpret_cast<float4 *>(xs)[tid] = ld_relaxed_sys_v4(p.mb_x + tid * 4);
                __syncthreads();
            }
            if (tid == 0)
                trace(k, n_done, 1);
            if (p.mailbox_format == 0) {
                // the TickBuffer: push {seq, 1} + x to every peer, (C-1) * (1 + IN/4) st.async of
                // 16 bytes completing the peer's request barrier
                constexpr int per = 1 + IN / 4;
                if (tid < (C - 1) * per) {
                    const uint32_t d = 1u + (uint32_t)(tid / per);
                    const int j = tid % per;
                    if (j == 0)
                        st_async_v4(mapa(h_addr, d), make_float4(__uint_as_float(seq), __uint_as_float(1u), 0.f, 0.f),
                                    mapa(bar_req, d));
                    else
                        st_async_v4(mapa(x_addr + (uint32_t)(j - 1) * 16u, d),
                                    reinterpret_cast<const float4 *>(xs)[j - 1], mapa(bar_req, d));
                }
            }
            if (tid == 0)
                trace(k, n_done, 2);
        } else {
            // a peer: the header + row 0 (tagged chunks, or the TickBuffer's float rows), then
            // rows 1.. of a micro-batch
            const bool chunks = p.mailbox_format == 1;
            const uint32_t row_bytes = chunks ? 16u * NXC : 4u * IN;
            if (tid == 0)
                mbar_arrive_expect_tx(bar_req, 16u + row_bytes);
            if (!cta_wait_bar(k, bar_req, ph_req & 1u, EW_PEER_POLL, p.idle_ns + p.peer_margin_ns))
                break;
            ++ph_req;
            seq = *reinterpret_cast<volatile uint32_t *>(&sh.hdr[0]);
            nb = *reinterpret_cast<volatile uint32_t *>(&sh.hdr[1]);
            nb = nb < 1u ? 1u : (nb > (uint32_t)MB ? (uint32_t)MB : nb);
            if (nb > 1) {
                if (tid == 0)
                    mbar_arrive_expect_tx(bar_x, row_bytes * (nb - 1));
                if (!cta_wait_bar(k, bar_x, ph_x & 1u, EW_PEER_POLL, p.step_ns))
                    break;
                ++ph_x;
            }
            if (chunks) {
                // unpack {v0, v1, v2, tag} chunks into the x rows
                for (int t = tid; t < (int)nb * NXC; t += kThreads) {
                    const int r = t / NXC, ch = t - r * NXC;
                    const uint4 v = xch[t];
                    float *dst = xs + r * IN + 3 * ch;
                    dst[0] = __uint_as_float(v.x);
                    if (3 * ch + 1 < IN)
                        dst[1] = __uint_as_float(v.y);
                    if (3 * ch + 2 < IN)
                        dst[2] = __uint_as_float(v.z);
                }
                __syncthreads();
            }
            if (tid == 0 && k.rank == 1)
                trace(k, n_done, 15);
        }

        // ---------------- the layers, over nb rows (weights used once per row) ----------------
        // GR = rows computed together: 1 for a single request, kFast3Group for a micro-batch, whose
        // rows are walked in groups of GR (rows past nb in the last group compute on stale inputs
        // inside the buffers and are never sent or stored)
        auto pass = [&](auto group_rows) -> bool {
            constexpr int GR = decltype(group_rows)::value;
            const int ng = GR == 1 ? 1 : ((int)nb + GR - 1) / GR;
            // ---------------- layer 1 (replicated), layer 2 (rows split over the cluster) ----------------
            f3_layer1<S, GR, IN, H1>(w1, xs, h1, bias, ng, r1, s1, act1);
            __syncthreads();
            if (leader && tid == 0)
                trace(k, n_done, 3);
            f3_layer2<S, GR, H1>(w2, h1, h2, bias + H1, ng, r2, s2, act2);
            if (own_x && !leader) {
                // rank 0's go for this request (sent while layers 1-2 ran); ends on its abort
                if (!cta_wait_bar(k, bar_req, ph_req & 1u, EW_PEER_POLL, p.step_ns))
                    return false;
                ++ph_req;
            } else {
                __syncthreads();
            }
            if (leader && tid == 0)
                trace(k, n_done, 4);
            // ---------------- layer 3 (K-split partials -> rank 0) ----------------
            if (warp < OUT) {
                const float mine = f3_layer3<S, GR>(w3, h2, (int)nb, lane);  // lane r sends row r's partial
                if (lane < (int)nb)
                    st_async_u32(mapa(g_addr + (uint32_t)((lane * C + k.rank) * OUT + warp) * 4u, 0u),
                                 __float_as_uint(mine), mapa(bar_g, 0u));
            }
            if (leader && tid == 0)
                trace(k, n_done, 5);

            // ---------------- rank 0: sum partials, write y, publish ----------------
            if (leader) {
                if (tid == 0)
                    mbar_arrive_expect_tx(bar_g, (uint32_t)(C * OUT * 4) * nb);
                const bool got = cta_wait_bar(k, bar_g, ph_g & 1u, EW_GATHER, p.step_ns);
                ++ph_g;
                if (!got)
                    return false;
                if (tid == 0)
                    trace(k, n_done, 12);
                if (warp < (int)nb) {
                    // warp r finishes row r.  The output row goes through shared memory: lanes
                    // < OUT finish one output each, then the storing lanes pick up their 16-byte
                    // groups (full-warp shuffles here cost ~1650 cycles in this loop, the
                    // shared-memory round ~60)
                    const int r = GR == 1 ? 0 : warp;
                    float *yr = yo + r * YO;
                    if (lane < OUT) {
                        float v = 0.f;
#pragma unroll
                        for (int c = 0; c < C; ++c)
                            v += gath[(r * C + c) * OUT + lane];
                        yr[lane] = relu_or(v + bias[H1 + S::R2 + lane], act3);
                    }
                    __syncwarp();
                    const bool tagged = p.mode == MODE_MAILBOX && p.mailbox_format == 1;
                    // tagged output: lane c packs {y[3c], y[3c+1], y[3c+2], seq}
                    constexpr int NYC = (OUT + 2) / 3;
                    if (tagged) {
                        const uint32_t sq = GR == 1 ? seq : rseq[r];
                        if (lane < NYC)
                            st_relaxed_sys_v4(p.mb_y + (size_t)ring_slot(p, n_done + (uint32_t)r) * p.ring_ystride_f +
                                                  4 * lane,
                                              make_float4(yr[3 * lane], yr[3 * lane + 1], yr[3 * lane + 2],
                                                          __uint_as_float(sq)));
                    } else if (lane < OUT / 4) {
                        const float4 q = reinterpret_cast<const float4 *>(yr)[lane];
                        if (p.mode == MODE_QUEUE)
                            reinterpret_cast<float4 *>(p.q_y + (size_t)n_done * OUT)[lane] = q;
                        else
                            st_relaxed_sys_v4(p.mb_y + 4 * lane, q);
                    }
                    __syncwarp();
                    if (warp == 0 && lane == 0) {
                        trace(k, n_done, 13);
                        if (p.mode == MODE_QUEUE) {
                            if (p.q_stamp)
                                p.q_stamp[n_done] = globaltimer();
                        } else if (tagged) {
                            st_relaxed_sys_u32(&p.mb->seq_out, seq);  // bookkeeping only: the host waits on the tags
                        } else {
                            st_release_sys_u32(&p.mb->seq_out, seq);
                        }
                        trace(k, n_done, 14);
                    }
                }
            }
            return true;
        };
        if constexpr (MB == 1)
            ok = pass(std::integral_constant<int, 1>{});
        else
            ok = nb == 1 ? pass(std::integral_constant<int, 1>{}) : pass(std::integral_constant<int, kFast3Group>{});
        if (!ok)
            break;
        ++passes;
        last = seq;
        n_done += nb;
    }
    __syncthreads();
    cluster_sync();
    if (leader && tid == 0) {
        st_relaxed_sys_u32(&p.ctrl->passes, passes);
        st_relaxed_sys_u32(&p.ctrl->rows, n_done);
        if (p.mode == MODE_QUEUE)
            st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_QUEUE_DONE);
        st_release_sys_u32(&p.ctrl->state, ST_EXITED);
    }
}

}  // namespace llk
