// Layers 1 and 2 of the pipelined ring kernel's compute CTAs (ring_kernel.cuh), blocked so
// that every input value a thread reads from shared memory serves several output rows.
//
// A pass carries up to 16 requests.  With one output row per thread (the register-resident
// kernel's mapping) each loaded input value feeds one FMA, and the layers are bound by
// moving inputs from shared memory into registers.  Here:
//   layer 1 (IN -> H1): a pass of several rows splits the layer over the C compute CTAs (R1 =
//     H1 / C rows each, 2 per warp: lane l takes input piece l % 16 of both rows for the 8
//     batch rows of its half-warp; ring_layer1_split) and the CTAs exchange their slices;
//     a pass of one row computes all H1 rows in every CTA (8 rows per thread, the same
//     per-piece products and the same reduction tree: ring_layer1_x1), so a request's h1
//     is bit-identical either way.  h1 is kept slice-major: block c (the rows of CTA c),
//     then batch row, then local row;
//   layer 2 (H1 -> R2 local rows): RB2 = 2 rows x 8 inputs per thread, a warp (32 lanes) per
//     row group; a loaded piece feeds 8 FMAs.
// The K slices are reduced across a row group's lanes by a transpose-reduce (one
// xor-shuffle round per mask, each round halving the values a lane holds), so a pass of
// 16 rows ends with every lane holding whole sums; a pass of one row uses a plain butterfly
// over the same masks.  Per (output row, request) the products are summed in the same
// order either way (each lane's FMA chain over its K slice, then the same pairwise
// additions, which commute), so a request's reply does not depend on the size of its pass.
// Weight j of thread t (warp w, lane l; image [NW][kThreads], thread-minor), in this order:
//   layer 1, one row (K1): j = 4 q + e  ->  W1[32 q + 2 w + (l >> 4)][4 (l & 15) + e],  q < H1 / 32
//   layer 1, split (K1S):  j = 4 i + e  ->  W1[c R1 + 2 w + i][4 (l & 15) + e],  i < 2 (CTA c)
//   layer 2: j = r * (4 P2) + 4 p + e  ->  W2[c R2 + 2 g2 + r][4 (s2 + 32 p) + e],  g2 = warp, s2 = lane
//   layer 3: as in the register-resident kernel (warp w = output w, local rows lane + 32 j).
#pragma once
#include "fast3_kernel.cuh"

namespace llk {

template <int IN, int H1, int H2, int OUT, int C>
struct RingShape {
    static constexpr int T = kThreads;
    static constexpr int R1 = H1 / C;        // layer-1 rows of this CTA in a split pass
    static constexpr int Q1 = H1 / 32;       // layer-1 rows per thread in a one-row pass
    static constexpr int K1 = 4 * Q1;        // layer-1 weights per thread, one-row pass
    static constexpr int K1S = 8;            // layer-1 weights per thread, split pass (2 rows x 4)
    static constexpr int R2 = H2 / C;        // layer-2 rows of this CTA
    static constexpr int RB2 = 2;            // layer-2 rows per thread
    static constexpr int G2 = R2 / RB2;      // layer-2 row groups: one per warp
    static constexpr int L2 = T / G2;        // lanes per layer-2 row group
    static constexpr int P2 = H1 / 4 / L2;   // 16-byte h1 pieces per lane
    static constexpr int K2 = RB2 * 4 * P2;  // layer-2 weights per thread
    static constexpr int K3 = R2 / 32;       // layer 3, as in the register-resident kernel
    static constexpr int NW = K1 + K1S + K2 + K3;
    static constexpr int NB = H1 + R2 + OUT;
    static_assert(IN == 64 && T == 512 && H1 % 32 == 0 && R1 == 2 * (T / 32),
                  "layer 1: 16 input pieces over a half-warp, 2 rows per warp in a split pass");
    static_assert(R2 % RB2 == 0 && G2 == T / 32 && L2 == 32 && H1 % (4 * L2) == 0 && P2 >= 1, "layer-2 blocking");
    static_assert(R2 % 32 == 0 && K3 >= 1, "layer-3 split");
    static_assert(RB2 * 16 == 32, "32 sums per lane before a 16-row transpose-reduce");
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

// Partial product of one 16-byte input piece and four weights, the order both layer-1
// variants use.
__device__ __forceinline__ float l1_piece(const float *w, float4 v)
{
    float a = 0.f;
    a = fmaf(w[0], v.x, a);
    a = fmaf(w[1], v.y, a);
    a = fmaf(w[2], v.z, a);
    a = fmaf(w[3], v.w, a);
    return a;
}

// Layer 1 of a pass of up to 16 rows, split over the C compute CTAs: this CTA's R1 rows (warp
// w: local rows 2w, 2w + 1) for batch rows 8 h .. 8 h + 7 in half-warp h, lane s = l % 16 taking
// input piece s; a transpose-reduce over the 16 lanes of each half (masks 8, 4, 2, 1: the same
// pairs as a butterfly) leaves lane s with local row 2w + (s >> 3), batch row 8 h + (s & 7), which
// it writes into this CTA's slice block `h1s` [batch row][R1] (rows past the pass's requests
// compute on stale inputs and are never sent).
template <class S, int IN, int H1>
__device__ __forceinline__ void ring_layer1_split(const float (&w1s)[S::K1S], const float *xs, float *h1s,
                                                  const float *b1, int rank, int act)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int s = lane & 15, half = lane >> 4;
    float t[16];  // t[8 i + bb]: local row 2w + i, batch row 8 half + bb
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) {
        const float4 v = reinterpret_cast<const float4 *>(xs + (8 * half + bb) * IN)[s];
        t[bb] = l1_piece(w1s, v);
        t[8 + bb] = l1_piece(w1s + 4, v);
    }
    rx_round<16, 8>(t, lane);
    rx_round<8, 4>(t, lane);
    rx_round<4, 2>(t, lane);
    rx_round<2, 1>(t, lane);
    const int r = 2 * warp + (s >> 3);
    h1s[(8 * half + (s & 7)) * S::R1 + r] = relu_or(t[0] + b1[rank * S::R1 + r], act);
}

// Layer 1 of a pass of one row, every row in every CTA: thread (w, l) takes rows 32 q + 2 w +
// (l >> 4), q < H1 / 32, input piece l % 16, with the products of ring_layer1_split and a
// butterfly over the same masks, so each h1 value is bit-identical to the split pass's; lane
// s = 0 of each half-warp writes its rows into their blocks of `h1` (block q: the rows of CTA
// q, batch row 0).
template <class S, int IN, int H1>
__device__ __forceinline__ void ring_layer1_x1(const float (&w1)[S::K1], const float *xs, float *h1,
                                               const float *b1, int act)
{
    constexpr int MB = 16;  // batch rows per slice block
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int s = lane & 15;
    const float4 v = reinterpret_cast<const float4 *>(xs)[s];
    float a[S::Q1];
#pragma unroll
    for (int q = 0; q < S::Q1; ++q)
        a[q] = l1_piece(w1 + 4 * q, v);
#pragma unroll
    for (int m = 8; m > 0; m >>= 1)
#pragma unroll
        for (int q = 0; q < S::Q1; ++q)
            a[q] += __shfl_xor_sync(0xffffffffu, a[q], m);
    if (s == 0) {
        const int r = 2 * warp + (lane >> 4);
#pragma unroll
        for (int q = 0; q < S::Q1; ++q)
            h1[q * MB * S::R1 + r] = relu_or(a[q] + b1[32 * q + r], act);
    }
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
            const int q = lane + 32 * p;  // piece q: block q / 8 (R1 = 32 rows), row b, offset q % 8
            const float4 v = reinterpret_cast<const float4 *>(h1 + (q >> 3) * 16 * S::R1 + b * S::R1)[q & 7];
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
        const int q = lane + 32 * p;  // piece q: block q / 8, batch row 0, offset q % 8
        const float4 v = reinterpret_cast<const float4 *>(h1 + (q >> 3) * 16 * S::R1)[q & 7];
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
