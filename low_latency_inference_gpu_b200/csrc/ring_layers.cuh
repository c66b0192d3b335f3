// Layers 1 and 2 of the pipelined ring kernel's compute CTAs (ring_kernel.cuh), blocked so
// that every input value a thread reads from shared memory serves several output rows.
//
// A pass carries up to 16 requests.  With one output row per thread (the register-resident
// kernel's mapping) each loaded input value feeds one FMA, and the layers are bound by
// moving inputs from shared memory into registers (pass timeline: ~2.4 us per layer for 16
// rows against ~0.5 us of FMA issue).  Here a thread holds its
// weights as RB rows x a K slice:
//   layer 1 (IN -> H1, replicated in every compute CTA): RB1 = 4 rows x 8 inputs per thread,
//     8 lanes (one row group) share the K range of 4 rows; a loaded 16-byte input piece
//     feeds 16 FMAs;
//   layer 2 (H1 -> R2 local rows): RB2 = 2 rows x 8 inputs per thread, a warp (32 lanes) per
//     row group; a loaded piece feeds 8 FMAs.
// The K slices are reduced across a row group's lanes by a transpose-reduce (one
// xor-shuffle round per mask, each round halving the values a lane holds), so a pass of
// 16 rows ends with every lane holding whole sums; a pass of one row uses a plain butterfly
// over the same masks.  Per (output row, request) the products are summed in the same
// order either way (each lane's FMA chain over its K slice, then the same pairwise
// additions, which commute), so a request's reply does not depend on the size of its pass.
// Weight j of thread t (image [NW][kThreads], thread-minor):
//   layer 1: j = r * (4 P1) + 4 p + e  ->  W1[4 g1 + r][4 (s1 + L1 p) + e],  g1 = t / L1, s1 = t % L1
//   layer 2: j = r * (4 P2) + 4 p + e  ->  W2[c R2 + 2 g2 + r][4 (s2 + 32 p) + e],  g2 = warp, s2 = lane
//   layer 3: as in the register-resident kernel (warp w = output w, local rows lane + 32 j).
#pragma once
#include "fast3_kernel.cuh"

namespace llk {

template <int IN, int H1, int H2, int OUT, int C>
struct RingShape {
    static constexpr int T = kThreads;
    static constexpr int RB1 = 4;            // layer-1 rows per thread
    static constexpr int G1 = H1 / RB1;      // layer-1 row groups
    static constexpr int L1 = T / G1;        // lanes (K slices) per layer-1 row group
    static constexpr int P1 = IN / 4 / L1;   // 16-byte input pieces per lane
    static constexpr int K1 = RB1 * 4 * P1;  // layer-1 weights per thread
    static constexpr int R2 = H2 / C;        // layer-2 rows of this CTA
    static constexpr int RB2 = 2;            // layer-2 rows per thread
    static constexpr int G2 = R2 / RB2;      // layer-2 row groups: one per warp
    static constexpr int L2 = T / G2;        // lanes per layer-2 row group
    static constexpr int P2 = H1 / 4 / L2;   // 16-byte h1 pieces per lane
    static constexpr int K2 = RB2 * 4 * P2;  // layer-2 weights per thread
    static constexpr int K3 = R2 / 32;       // layer 3, as in the register-resident kernel
    static constexpr int NW = K1 + K2 + K3;
    static constexpr int NB = H1 + R2 + OUT;
    static_assert(H1 % RB1 == 0 && T % G1 == 0 && L1 == 8 && IN % (4 * L1) == 0 && P1 >= 1, "layer-1 blocking");
    static_assert(R2 % RB2 == 0 && G2 == T / 32 && L2 == 32 && H1 % (4 * L2) == 0 && P2 >= 1, "layer-2 blocking");
    static_assert(R2 % 32 == 0 && K3 >= 1, "layer-3 split");
    static_assert(RB1 * 8 == 32 && RB2 * 16 == 32, "32 sums per lane before a 16-row transpose-reduce");
};

// One transpose-reduce round over an array of N sums: lanes with `M` set keep the upper
// half, the others the lower half, each adding its partner's copy of the half it keeps.
template <int N, int M, int A>
__device__ __forceinline__ void rx_round(float (&t)[A], int lane)
{
    static_assert(N <= A && N % 2 == 0, "round size");
    const bool upper = (lane & M) != 0;
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        const float give = upper ? t[i] : t[i + N / 2];
        const float keep = upper ? t[i + N / 2] : t[i];
        t[i] = keep + __shfl_xor_sync(0xffffffffu, give, M);
    }
}

// Layer 1 for a pass of up to 16 rows (rows past the pass's requests compute on stale inputs
// and are never sent): `halves` halves of 8 rows, 4 x 8 sums per lane, reduced over the 8
// lanes of the row group (masks 4, 2, 1).  Lane s1 then holds output row 4 g1 + 2 (s1 >> 2 & 1) +
// (s1 >> 1 & 1) for the 4 requests 8 h + 4 (s1 & 1) + j.
template <class S, int IN, int H1>
__device__ __forceinline__ void ring_layer1_x16(const float (&w1)[S::K1], const float *xs, float *h1,
                                                const float *b1, int g1, int s1, int act, int halves)
{
    const int lane = threadIdx.x & 31;
    const int r = 2 * ((s1 >> 2) & 1) + ((s1 >> 1) & 1);
    const int row = S::RB1 * g1 + r;
    const float bias = b1[row];
#pragma unroll 1
    for (int half = 0; half < halves; ++half) {
        float t[32];
#pragma unroll
        for (int i = 0; i < 32; ++i)
            t[i] = 0.f;
#pragma unroll
        for (int p = 0; p < S::P1; ++p) {
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const float4 v = reinterpret_cast<const float4 *>(xs + (8 * half + b) * IN)[s1 + S::L1 * p];
#pragma unroll
                for (int rr = 0; rr < S::RB1; ++rr) {
                    const float *w = w1 + rr * 4 * S::P1 + 4 * p;
                    float a = t[rr * 8 + b];
                    a = fmaf(w[0], v.x, a);
                    a = fmaf(w[1], v.y, a);
                    a = fmaf(w[2], v.z, a);
                    a = fmaf(w[3], v.w, a);
                    t[rr * 8 + b] = a;
                }
            }
        }
        rx_round<32, 4>(t, lane);
        rx_round<16, 2>(t, lane);
        rx_round<8, 1>(t, lane);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            h1[(8 * half + 4 * (s1 & 1) + j) * H1 + row] = relu_or(t[j] + bias, act);
    }
}

// Layer 1 for a pass of one row: the same FMA chains, then a butterfly over the same masks;
// lane s1 < RB1 writes output row 4 g1 + s1.
template <class S, int IN, int H1>
__device__ __forceinline__ void ring_layer1_x1(const float (&w1)[S::K1], const float *xs, float *h1,
                                               const float *b1, int g1, int s1, int act)
{
    float a[S::RB1];
#pragma unroll
    for (int rr = 0; rr < S::RB1; ++rr)
        a[rr] = 0.f;
#pragma unroll
    for (int p = 0; p < S::P1; ++p) {
        const float4 v = reinterpret_cast<const float4 *>(xs)[s1 + S::L1 * p];
#pragma unroll
        for (int rr = 0; rr < S::RB1; ++rr) {
            const float *w = w1 + rr * 4 * S::P1 + 4 * p;
            a[rr] = fmaf(w[0], v.x, a[rr]);
            a[rr] = fmaf(w[1], v.y, a[rr]);
            a[rr] = fmaf(w[2], v.z, a[rr]);
            a[rr] = fmaf(w[3], v.w, a[rr]);
        }
    }
#pragma unroll
    for (int m = 4; m > 0; m >>= 1)
#pragma unroll
        for (int rr = 0; rr < S::RB1; ++rr)
            a[rr] += __shfl_xor_sync(0xffffffffu, a[rr], m);
    float mine = a[0];
#pragma unroll
    for (int rr = 1; rr < S::RB1; ++rr)
        if (s1 == rr)
            mine = a[rr];
    if (s1 < S::RB1)
        h1[S::RB1 * g1 + s1] = relu_or(mine + b1[S::RB1 * g1 + s1], act);
}

// Layer 2 for a pass of 16 rows: 2 x 16 sums per lane, reduced over the warp (masks 16, 8,
// 4, 2, 1); lane l then holds local row 2 g2 + (l >> 4) for request l & 15.
template <class S, int H1>
__device__ __forceinline__ void ring_layer2_x16(const float (&w2)[S::K2], const float *h1, float *h2,
                                                const float *b2, int g2, int act)
{
    const int lane = threadIdx.x & 31;
    float t[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        t[i] = 0.f;
#pragma unroll
    for (int p = 0; p < S::P2; ++p) {
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            const float4 v = reinterpret_cast<const float4 *>(h1 + b * H1)[lane + 32 * p];
#pragma unroll
            for (int rr = 0; rr < S::RB2; ++rr) {
                const float *w = w2 + rr * 4 * S::P2 + 4 * p;
                float a = t[rr * 16 + b];
                a = fmaf(w[0], v.x, a);
                a = fmaf(w[1], v.y, a);
                a = fmaf(w[2], v.z, a);
                a = fmaf(w[3], v.w, a);
                t[rr * 16 + b] = a;
            }
        }
    }
    rx_round<32, 16>(t, lane);
    rx_round<16, 8>(t, lane);
    rx_round<8, 4>(t, lane);
    rx_round<4, 2>(t, lane);
    rx_round<2, 1>(t, lane);
    const int row = S::RB2 * g2 + (lane >> 4);
    h2[(lane & 15) * S::R2 + row] = relu_or(t[0] + b2[row], act);
}

// Layer 2 for a pass of one row: the same chains, a butterfly over the warp; lane rr < RB2
// writes local row 2 g2 + rr.
template <class S, int H1>
__device__ __forceinline__ void ring_layer2_x1(const float (&w2)[S::K2], const float *h1, float *h2,
                                               const float *b2, int g2, int act)
{
    const int lane = threadIdx.x & 31;
    float a[S::RB2];
#pragma unroll
    for (int rr = 0; rr < S::RB2; ++rr)
        a[rr] = 0.f;
#pragma unroll
    for (int p = 0; p < S::P2; ++p) {
        const float4 v = reinterpret_cast<const float4 *>(h1)[lane + 32 * p];
#pragma unroll
        for (int rr = 0; rr < S::RB2; ++rr) {
            const float *w = w2 + rr * 4 * S::P2 + 4 * p;
            a[rr] = fmaf(w[0], v.x, a[rr]);
            a[rr] = fmaf(w[1], v.y, a[rr]);
            a[rr] = fmaf(w[2], v.z, a[rr]);
            a[rr] = fmaf(w[3], v.w, a[rr]);
        }
    }
#pragma unroll
    for (int m = 16; m > 0; m >>= 1)
#pragma unroll
        for (int rr = 0; rr < S::RB2; ++rr)
            a[rr] += __shfl_xor_sync(0xffffffffu, a[rr], m);
    const float mine = lane == 1 ? a[1] : a[0];
    if (lane < S::RB2)
        h2[S::RB2 * g2 + lane] = relu_or(mine + b2[S::RB2 * g2 + lane], act);
}

}  // namespace llk
