// Batched dense layer for many rows on SM pairs: the weights-in-TMEM tile of
// tc_swap.cuh run by two CTAs of a cluster as one 2-SM MMA (cta_group::2).
//
//   D[256 channels x 256 rows] = W[n0:n0+256, :] . X[m0:m0+256, :]^T     (fp32, TMEM)
//
// CTA r of the pair (r = 0, 1) owns channels n0 + 128 r .. + 127 (its TMEM lanes, as in the
// one-SM tile) and loads rows m0 + 128 r .. + 127 of X; the MMA, issued by CTA 0 alone, reads
// A (the weights) from both CTAs' tensor memory and B (the rows) from both CTAs' shared
// memory, and writes each CTA's 128 channels x 256 rows of D into that CTA's tensor memory.
// So X crosses the L2-to-SM crossbar once per pair instead of once per CTA: per 64-deep K
// step an SM receives 16 KB of rows + 8 KB of int8 weights instead of 32 + 8 KB.
// Synchronisation across the pair:
//   * both CTAs' row loads complete their bytes on CTA 0's `xfull` (the 2-SM form of the
//     tensor load names CTA 0's barrier); CTA 0 expects the bytes of both halves;
//   * each CTA's converter warps arrive on CTA 0's `afull` once their weight stage is in
//     their own tensor memory (8 arrivals: 4 warps per CTA);
//   * CTA 0's MMA thread commits to the `xempty` / `aempty` / `accf` barriers of both CTAs
//     (tcgen05.commit to the pair; no data moves by multicast);
//   * tensor memory is allocated and freed by warp 1 of both CTAs (2-SM allocation), after a
//     cluster barrier, so no MMA of the pair can touch a CTA's tensor memory after it is freed.
// Every wait is bounded (globaltimer); a CTA that gives up records the error, and the pair
// drains the MMAs already issued before tensor memory is freed.  Every load is a plain
// (non-multicast) tensor load of this GPU's memory.
//
// No counterpart in the reference (its batched GEMMs are cuBLAS calls,
// src/bench_cublas_mlp.cu); the layer contract is y = act(W x + b).
#pragma once
#include "tc_swap.cuh"

namespace llk {

constexpr int kSw2Half = kSwRows / 2;   // rows of X per CTA
constexpr int kSw2XG = 2;               // 64-deep K blocks of X per tensor load (one box: 32 KB)
constexpr int kSw2XStages = 4;          // X ring in shared memory (one box each)

template <bool WINT8>
struct TcSwap2Smem {
    static constexpr int XB = kSw2Half * kTcK * 2;                 // 16 KB: this CTA's half of a K step's rows
    static constexpr int XSB = kSw2XG * XB;                        // X stage (one box): kSw2XG K blocks
    static constexpr int WB = kSwChan * kTcK * (WINT8 ? 1 : 2);    // one K block of weights
    static constexpr int WG = sw_wgroup<WINT8>();
    static constexpr int WSB = WG * WB;                            // weight stage (one box): 32 KB
    static constexpr int WSTAGES = 2;
    static constexpr int OFF_X = 0;
    static constexpr int OFF_W = kSw2XStages * XSB;
    // xfull[S], xempty[S], wfull[W], wempty[W], afull[A], aempty[A], accf
    static constexpr int OFF_BAR = OFF_W + WSTAGES * WSB;
    static constexpr int N_BAR = 2 * kSw2XStages + 2 * WSTAGES + 2 * kSwAStages + 1;
    static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;  // tmem base, fail flag
    static constexpr int OFF_BIAS = OFF_MISC + 16;        // bias[128], scale[128]
    static constexpr int BYTES = OFF_BIAS + 8 * kSwChan;
    static constexpr int ALLOC = BYTES + 1024;
    static_assert(XB % 1024 == 0 && WB % 1024 == 0 && WSB % 1024 == 0, "1024-byte aligned tiles");
    static_assert(ALLOC <= 227 * 1024, "shared memory");
    static_assert(kSwRows * kSwChan * 4 <= kSw2XStages * XSB, "the fp32 output tile fits the X ring");
};

// Instruction descriptor, kind::f16 on a pair: A = B = bf16, D = fp32, both K-major,
// M = 256 (128 per CTA), N = n.
__host__ __device__ constexpr uint32_t tc_idesc_bf16_pair(int n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// 3-D tensor load {x, y, z} of this CTA's tile (x = K within a 64-wide block, y = row, z =
// 64-wide K block) whose completion bytes go to an mbarrier of the pair (cluster address:
// CTA 0's barrier), cta_group::2 form; no multicast.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *tm, int x, int y, int z,
                                                 uint32_t cluster_bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(cluster_bar)
        : "memory");
}

__device__ __forceinline__ void tc_mma_bf16_ts_pair(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                    uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on the mbarrier at this shared-memory offset in both CTAs of the pair (cluster ranks
// 0 and 1) when every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit_both(uint32_t bar)
{
    const uint16_t pair_mask = 0x3;
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(bar), "h"(pair_mask)
                 : "memory");
}

template <bool WINT8>
__global__ void __launch_bounds__(kSwThreads, 1) ll_tc_swap2_kernel(const __grid_constant__ TcLayerParams p)
{
    using L = TcSwap2Smem<WINT8>;
    constexpr int WS = L::WSTAGES;
    constexpr int XS = kSw2XStages;
    extern __shared__ uint8_t sw_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sw_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t *misc = reinterpret_cast<uint32_t *>(smem + L::OFF_MISC);
    volatile uint32_t *fail = misc + 1;
    float *s_bias = reinterpret_cast<float *>(smem + L::OFF_BIAS);
    float *s_scale = s_bias + kSwChan;
    auto bar = [&](int i) { return sbase + (uint32_t)L::OFF_BAR + 8u * (uint32_t)i; };
    auto b_xfull = [&](int s) { return bar(s); };
    auto b_xempty = [&](int s) { return bar(XS + s); };
    auto b_wfull = [&](int s) { return bar(2 * XS + s); };
    auto b_wempty = [&](int s) { return bar(2 * XS + WS + s); };
    auto b_afull = [&](int s) { return bar(2 * XS + 2 * WS + s); };
    auto b_aempty = [&](int s) { return bar(2 * XS + 2 * WS + kSwAStages + s); };
    const uint32_t b_accf = bar(2 * XS + 2 * WS + 2 * kSwAStages);

    const uint32_t rank = cluster_ctarank();  // 0 or 1: the pair is the cluster
    const bool lead = rank == 0u;
    auto at_lead = [&](uint32_t a) { return mapa(a, 0u); };

    const uint32_t cta_lin = blockIdx.x + gridDim.x * blockIdx.y;
    auto stamp = [&](int k) {
        if (p.trace)
            p.trace[cta_lin * (uint32_t)kTcTraceSlots + (uint32_t)k] = globaltimer();
    };
    if (tid == 0)
        stamp(kTcTraceEntry);
    const int n0 = blockIdx.x * kSwChan;            // this CTA's first channel
    const int m0 = blockIdx.y * kSwRows;            // the pair's first row
    const int mx = m0 + (int)rank * kSw2Half;       // this CTA's first row of X
    const int nk = p.K / kTcK;

    if (tid == 0) {
        for (int s = 0; s < XS; ++s) {
            mbar_init(b_xfull(s), 1);   // CTA 0's: its producer's arrive + both halves' bytes
            mbar_init(b_xempty(s), 1);  // the MMA thread's commit
        }
        for (int s = 0; s < WS; ++s) {
            mbar_init(b_wfull(s), 1);
            mbar_init(b_wempty(s), 4 * kSwConvGroups);  // each converter warp, after its last K block of the stage
        }
        for (int s = 0; s < kSwAStages; ++s) {
            mbar_init(b_afull(s), 8);   // CTA 0's: four converter warps of each CTA
            mbar_init(b_aempty(s), 1);  // the MMA thread's commit
        }
        mbar_init(b_accf, 1);
        misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&p.tm_x);
        prefetch_tmap(&p.tm_w);
    }
    if (warp == 1) {  // both CTAs, the same warp: one 2-SM allocation
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         sbase + (uint32_t)L::OFF_MISC),
                     "r"(kSwTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised and their tensor memory allocated
    tc_fence_after();
    const uint32_t tmem = misc[0];
    griddep_launch_dependents();

    const bool conv = warp >= 4;               // converters: warps 4.. in groups of 4
    const int cgrp = conv ? (warp - 4) >> 2 : 0;  // converter group (its K steps: kb = cgrp mod kSwConvGroups)
    const bool epi = warp >= 4 && warp < 8;      // epilogue: the first converter group
    const int q = warp & 3;
    const int chan = 32 * q + lane;  // this thread's TMEM lane = output channel within the CTA's 128
    if (warp == 3) {
        // ---------------- TMA producer: this CTA's weight tiles (independent of the previous layer) ----------------
        if (lane == 0) {
            const int ng = (nk + L::WG - 1) / L::WG;
            for (int g = 0; g < ng; ++g) {
                const int s = g % WS;
                if (g >= WS && !tc_wait(b_wempty(s), ((g / WS) - 1) & 1, p.wait_ns, fail, p.status, 6))
                    break;
                mbar_arrive_expect_tx(b_wfull(s), L::WSB);
                tma_load_3d(sbase + L::OFF_W + s * L::WSB, &p.tm_w, 0, n0, g * L::WG, b_wfull(s));
            }
        }
    } else if (epi && q == 0) {
        for (int i = lane; i < kSwChan; i += 32) {
            s_bias[i] = __ldg(p.bias + n0 + i);
            s_scale[i] = p.scale ? __ldg(p.scale + n0 + i) : 1.0f;
        }
    }
    if (warp != 3)
        griddep_wait();  // X belongs to the previous layer (and Y to the one before it) until here
    if (tid == 0)
        stamp(kTcTraceDepDone);

    if (warp == 0 || warp == 2) {
        // ---------------- TMA producers: this CTA's half of the rows, kSw2XG K blocks per load, ----------------
        // ---------------- even / odd loads from warps 0 / 2 (a box past K is zero-filled and     ----------------
        // ---------------- still counts its bytes)                                                ----------------
        if (lane == 0) {
            const int ngx = (nk + kSw2XG - 1) / kSw2XG;
            for (int gx = warp >> 1; gx < ngx; gx += 2) {
                const int s = gx % XS;
                if (gx >= XS && !tc_wait(b_xempty(s), ((gx / XS) - 1) & 1, p.wait_ns, fail, p.status, 1))
                    break;
                if (lead)
                    mbar_arrive_expect_tx(b_xfull(s), 2u * L::XSB);  // both halves land on this barrier
                tma_load_3d_pair(sbase + L::OFF_X + s * L::XSB, &p.tm_x, 0, mx, gx * kSw2XG, at_lead(b_xfull(s)));
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (CTA 0 of the pair) ----------------
        if (lead && lane == 0) {
            constexpr uint32_t idesc = tc_idesc_bf16_pair(kSwRows);  // M = 256 channels, N = 256 rows
            bool ok = true;
            for (int kb = 0; kb < nk && ok; ++kb) {
                const int gx = kb / kSw2XG, xsub = kb - gx * kSw2XG, s = gx % XS, sa = kb % kSwAStages;
                if (xsub == 0)
                    ok = tc_wait(b_xfull(s), (gx / XS) & 1, p.wait_ns, fail, p.status, 2);
                ok = ok && tc_wait(b_afull(sa), (kb / kSwAStages) & 1, p.wait_ns, fail, p.status, 2);
                if (!ok)
                    break;
                if (kb == 0)
                    stamp(kTcTraceFirstData);
                if (kb < 4)
                    stamp(kTcTraceStageReady + kb);
                tc_fence_after();
                const uint32_t xa = sbase + L::OFF_X + s * L::XSB + xsub * L::XB;
                const uint32_t aa = tmem + 256u + (uint32_t)sa * 32u;
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; ++kk)
                    tc_mma_bf16_ts_pair(tmem, aa + (uint32_t)kk * 8u, sw128_kmajor_desc(xa + kk * 32), idesc,
                                        (kb | kk) != 0);
                // the stages of both CTAs are free when these MMAs complete
                if (xsub == kSw2XG - 1 || kb == nk - 1)
                    tc_commit_both(b_xempty(s));
                tc_commit_both(b_aempty(sa));
            }
            stamp(kTcTraceMmaIssued);
            // accumulators complete (also arrives when nothing was issued)
            tc_commit_both(b_accf);
        }
    } else if (conv) {
        // ---------------- weights: shared memory -> registers -> bf16 -> this CTA's TMEM ----------------
        for (int kb = cgrp; kb < nk; kb += kSwConvGroups) {
            const int sa = kb % kSwAStages, g = kb / L::WG, sub = kb - g * L::WG, sw = g % WS;
            if (kb >= kSwAStages &&
                !tc_wait_warp(b_aempty(sa), ((kb / kSwAStages) - 1) & 1, p.wait_ns, fail, p.status, 3))
                break;
            // this group's first K block of the stage: wait for the stage
            if (sub < kSwConvGroups && !tc_wait_warp(b_wfull(sw), (g / WS) & 1, p.wait_ns, fail, p.status, 3))
                break;
            const uint8_t *wr = smem + L::OFF_W + sw * L::WSB + sub * L::WB + chan * (kTcK * (WINT8 ? 1 : 2));
            uint32_t o[32];
            if constexpr (WINT8) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(wr + 16 * (j ^ ((chan >> 1) & 3)));
                    uint32_t t[8];
                    i8x16_to_bf16(v, t);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        o[8 * j + e] = t[e];
                }
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 v = *reinterpret_cast<const uint4 *>(wr + 16 * (j ^ (chan & 7)));
                    o[4 * j] = v.x;
                    o[4 * j + 1] = v.y;
                    o[4 * j + 2] = v.z;
                    o[4 * j + 3] = v.w;
                }
            }
            __syncwarp();
            // this group's last K block of the stage: the stage is read as far as this warp goes
            if (lane == 0 && (sub + kSwConvGroups >= L::WG || kb + kSwConvGroups >= nk))
                mbar_arrive_local(b_wempty(sw));
            tc_st_32cols(tmem + ((uint32_t)(32 * q) << 16) + 256u + (uint32_t)sa * 32u, o);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                // release at CTA scope (a cluster-scope release held the warp ~0.5 us per K step);
                // the tensor-memory writes it covers are ordered by tcgen05.wait::st and
                // tcgen05.fence::before_thread_sync before it
                mbar_arrive_remote_cta(at_lead(b_afull(sa)));
            if (kb == 0 && lane == 0 && q == 0)
                stamp(kTcTraceConvDone);
        }
    }

    // ---------------- epilogue: warps 4..7, lane = channel, columns = rows ----------------
    if (epi) {
        tc_wait_warp(b_accf, 0, p.wait_ns, fail, p.status, 4);
        tc_fence_after();
        if (tid == 128)
            stamp(kTcTraceAccum);
    }
    __syncthreads();
    const bool go = *fail == 0u;
    if (epi && go) {
        const float sc = s_scale[chan], bi = s_bias[chan];
        const int esz = p.out_f32 ? 4 : 2;
        const int row_bytes = kSwChan * esz;
        uint8_t *stage = smem + L::OFF_X;  // the X ring is idle: every MMA of the pair has completed
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        if (p.out_f32) {
            if (p.act == 1)
                sw_stage_tile<1, true>(tq, stage, chan, sc, bi);
            else if (p.act == 2)
                sw_stage_tile<2, true>(tq, stage, chan, sc, bi);
            else
                sw_stage_tile<0, true>(tq, stage, chan, sc, bi);
        } else {
            if (p.act == 1)
                sw_stage_tile<1, false>(tq, stage, chan, sc, bi);
            else if (p.act == 2)
                sw_stage_tile<2, false>(tq, stage, chan, sc, bi);
            else
                sw_stage_tile<0, false>(tq, stage, chan, sc, bi);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int cpr = row_bytes / 16;
        uint8_t *out = static_cast<uint8_t *>(p.out);
        for (int idx = tid - 128; idx < kSwRows * cpr; idx += 128) {
            const int r = idx / cpr, ch = idx - r * cpr;
            *reinterpret_cast<uint4 *>(out + ((size_t)(m0 + r) * p.N + n0) * esz + (size_t)ch * 16) =
                *reinterpret_cast<const uint4 *>(stage + (size_t)r * row_bytes + (size_t)ch * 16);
        }
    }

    // ---------------- drain and free ----------------
    // Both CTAs wait (bounded) for the accumulator barrier, which completes only when every
    // MMA issued for the pair has, then meet at a cluster barrier before either frees its
    // tensor memory (the pair's MMAs read and write both).
    tc_fence_before();
    __syncthreads();
    if (tid == 0)
        stamp(kTcTraceEnd);
    if (warp == 1 && *fail && lane == 0) {
        const uint64_t t0 = globaltimer();
        while (!mbar_try_wait(b_accf, 0) && globaltimer() - t0 < p.wait_ns) {
        }
    }
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kSwTmemCols)
                     : "memory");
    }
}

}  // namespace llk
