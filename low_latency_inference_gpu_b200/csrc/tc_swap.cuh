// Batched dense layer for many rows (stacked batches): weights as the MMA's A
// operand in tensor memory, rows as N.
//
//   D[128 channels x 256 rows] = W[n0:n0+128, :] . X[m0:m0+256, :]^T     (fp32, TMEM)
//   Y[row][channel] = act(D * scale[channel] + bias[channel])
//
// Per 64-deep K step X passes through shared memory once (TMA, 128-byte swizzle,
// read by the MMA as the B operand); the weight tile arrives by TMA too (int8 with
// 64-byte swizzle, bf16 with 128-byte swizzle, so that the 32 lanes of a warp,
// one channel row each, read it without bank conflicts), is read once into
// registers, converted (int8: exact bf16) and stored to tensor memory with
// tcgen05.st, where tcgen05.mma reads it as A.  The weight loads start before the
// dependency on the previous layer resolves.  K is not split: one CTA owns a
// 128 x 256 output tile.  Roles (256 threads): warps 0 and 2 TMA for X; warp 1
// TMEM allocation + the MMA thread; warp 3 TMA for the weights; warps 4..7 convert
// the weight stages into their TMEM lane quarter and run the epilogue for the same
// lanes (= channels).  Every wait is bounded.
#pragma once
#include "tc_layer.cuh"

namespace llk {

constexpr int kSwRows = 256;      // rows per tile (MMA N)
constexpr int kSwChan = 128;      // channels per tile (MMA M)
constexpr int kSwConvGroups = 2;  // converter warp groups: group g converts the K steps kb = g mod 2
constexpr int kSwThreads = 128 + 128 * kSwConvGroups;
constexpr int kSwXStages = 4;     // X ring in shared memory (32 KB each)
constexpr int kSwAStages = 8;     // weight stages in TMEM (32 columns each)
constexpr uint32_t kSwTmemCols = 512;  // D: columns [0, 256); A stages: [256, 512)

// An SM's TMA engine completes roughly one box per ~400-600 cycles almost whatever its size
// (up to 32 KB), so a K step's 8 KB int8 weight tile as its own box cost as much as the 32 KB
// row tile: one box carries WGROUP consecutive 64-deep K blocks (a 3-D view of W), 32 KB.
template <bool WINT8>
constexpr int sw_wgroup()
{
    return WINT8 ? 4 : 2;
}

template <bool WINT8>
struct TcSwapSmem {
    static constexpr int XB = kSwRows * kTcK * 2;                // 32 KB
    static constexpr int WB = kSwChan * kTcK * (WINT8 ? 1 : 2);  // one K block of weights: 8 KB int8, 16 KB bf16
    static constexpr int WG = sw_wgroup<WINT8>();                // K blocks per weight box
    static constexpr int WSB = WG * WB;                          // weight stage (one box): 32 KB
    static constexpr int WSTAGES = 2;                            // weight ring in shared memory
    static constexpr int OFF_X = 0;
    static constexpr int OFF_W = kSwXStages * XB;
    static constexpr int OFF_BAR = OFF_W + WSTAGES * WSB;  // xfull[S], xempty[S], wfull[W], wempty[W], afull[A], aempty[A], accf
    static constexpr int N_BAR = 2 * kSwXStages + 2 * WSTAGES + 2 * kSwAStages + 1;
    static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;  // tmem base, fail flag
    static constexpr int OFF_BIAS = OFF_MISC + 16;        // bias[128], scale[128]
    static constexpr int BYTES = OFF_BIAS + 8 * kSwChan;
    static constexpr int ALLOC = BYTES + 1024;
    static_assert(XB % 1024 == 0 && WB % 1024 == 0 && WSB % 1024 == 0, "1024-byte aligned tiles");
    static_assert(ALLOC <= 227 * 1024, "shared memory");
};

// Store 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (one row each).
__device__ __forceinline__ void tc_st_32cols(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tc_mma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Epilogue of one lane quarter: this lane's channel over the tile's 256 rows (TMEM columns),
// act(D * scale + bias), into the row-major staging tile.
template <int ACT, bool F32>
__device__ __forceinline__ void sw_stage_tile(uint32_t tq, uint8_t *stage, int chan, float sc, float bi)
{
    constexpr int ESZ = F32 ? 4 : 2, ROW = kSwChan * ESZ;
#pragma unroll 1
    for (int c0 = 0; c0 < kSwRows; c0 += 64) {
        float v[64];
        tc_ld_64cols(tq + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            const float y = tc_act_t<ACT>(fmaf(v[i], sc, bi));
            uint8_t *d = stage + (size_t)(c0 + i) * ROW + (size_t)chan * ESZ;
            if constexpr (F32)
                *reinterpret_cast<float *>(d) = y;
            else
                *reinterpret_cast<__nv_bfloat16 *>(d) = __float2bfloat16_rn(y);
        }
    }
}

template <bool WINT8>
__global__ void __launch_bounds__(kSwThreads, 1) ll_tc_swap_kernel(const __grid_constant__ TcLayerParams p)
{
    using L = TcSwapSmem<WINT8>;
    constexpr int WS = L::WSTAGES;
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
    auto b_xempty = [&](int s) { return bar(kSwXStages + s); };
    auto b_wfull = [&](int s) { return bar(2 * kSwXStages + s); };
    auto b_wempty = [&](int s) { return bar(2 * kSwXStages + WS + s); };
    auto b_afull = [&](int s) { return bar(2 * kSwXStages + 2 * WS + s); };
    auto b_aempty = [&](int s) { return bar(2 * kSwXStages + 2 * WS + kSwAStages + s); };
    const uint32_t b_accf = bar(2 * kSwXStages + 2 * WS + 2 * kSwAStages);

    const uint32_t cta_lin = blockIdx.x + gridDim.x * blockIdx.y;
    auto stamp = [&](int k) {
        if (p.trace)
            p.trace[cta_lin * (uint32_t)kTcTraceSlots + (uint32_t)k] = globaltimer();
    };
    if (tid == 0)
        stamp(kTcTraceEntry);
    const int n0 = blockIdx.x * kSwChan;   // first channel
    const int m0 = blockIdx.y * kSwRows;   // first row
    const int nk = p.K / kTcK;

    if (tid == 0) {
        for (int s = 0; s < kSwXStages; ++s) {
            mbar_init(b_xfull(s), 1);
            mbar_init(b_xempty(s), 1);
        }
        for (int s = 0; s < WS; ++s) {
            mbar_init(b_wfull(s), 1);
            mbar_init(b_wempty(s), 4 * kSwConvGroups);  // each converter warp, after its last K block of the stage
        }
        for (int s = 0; s < kSwAStages; ++s) {
            mbar_init(b_afull(s), 4);  // one arrive per converter warp
            mbar_init(b_aempty(s), 1);
        }
        mbar_init(b_accf, 1);
        misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&p.tm_x);
        prefetch_tmap(&p.tm_w);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         sbase + (uint32_t)L::OFF_MISC),
                     "r"(kSwTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    griddep_launch_dependents();

    const bool conv = warp >= 4;               // converters: warps 4.. in groups of 4
    const int cgrp = conv ? (warp - 4) >> 2 : 0;  // converter group (its K steps: kb = cgrp mod kSwConvGroups)
    const bool epi = warp >= 4 && warp < 8;      // epilogue: the first converter group
    const int q = warp & 3;
    const int chan = 32 * q + lane;  // this thread's TMEM lane = output channel within the tile
    if (warp == 3) {
        // ---------------- TMA producer: weight tiles (independent of the previous layer) ----------------
        if (lane == 0) {
            // one box per WG K blocks (a box past K is filled with zeros and still counts its bytes)
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
        // biases and scales do not depend on the previous layer either
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
        // ---------------- TMA producers: X tiles, even K steps from warp 0, odd from warp 2 ----------------
        // (a thread issuing back-to-back tensor loads holds each for hundreds of cycles;
        // two issuers raise the SM's TMA throughput ~1.6x)
        if (lane == 0) {
            for (int kb = warp >> 1; kb < nk; kb += 2) {
                const int s = kb % kSwXStages;
                if (kb >= kSwXStages &&
                    !tc_wait(b_xempty(s), ((kb / kSwXStages) - 1) & 1, p.wait_ns, fail, p.status, 1))
                    break;
                mbar_arrive_expect_tx(b_xfull(s), L::XB);
                tma_load_2d(sbase + L::OFF_X + s * L::XB, &p.tm_x, kb * kTcK, m0, b_xfull(s));
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc_bf16(kSwRows);  // M = 128 channels, N = 256 rows
            bool ok = true;
            for (int kb = 0; kb < nk && ok; ++kb) {
                const int s = kb % kSwXStages, sa = kb % kSwAStages;
                ok = tc_wait(b_xfull(s), (kb / kSwXStages) & 1, p.wait_ns, fail, p.status, 2) &&
                     tc_wait(b_afull(sa), (kb / kSwAStages) & 1, p.wait_ns, fail, p.status, 2);
                if (!ok)
                    break;
                if (kb == 0)
                    stamp(kTcTraceFirstData);
                if (kb < 4)
                    stamp(kTcTraceStageReady + kb);
                tc_fence_after();
                const uint32_t xa = sbase + L::OFF_X + s * L::XB;
                const uint32_t aa = tmem + 256u + (uint32_t)sa * 32u;
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; ++kk)
                    tc_mma_bf16_ts(tmem, aa + (uint32_t)kk * 8u, sw128_kmajor_desc(xa + kk * 32), idesc,
                                   (kb | kk) != 0);
                tc_commit(b_xempty(s));   // X stage free when these MMAs complete
                tc_commit(b_aempty(sa));  // and the weight stage in TMEM
            }
            stamp(kTcTraceMmaIssued);
            tc_commit(b_accf);
        }
    } else if (conv) {
        // ---------------- weights: shared memory -> registers -> bf16 -> TMEM (lanes of quarter q) ----------------
        for (int kb = cgrp; kb < nk; kb += kSwConvGroups) {
            const int sa = kb % kSwAStages, g = kb / L::WG, sub = kb - g * L::WG, sw = g % WS;
            if (kb >= kSwAStages &&
                !tc_wait_warp(b_aempty(sa), ((kb / kSwAStages) - 1) & 1, p.wait_ns, fail, p.status, 3))
                break;
            // this group's first K block of the stage: wait for the stage
            if (sub < kSwConvGroups && !tc_wait_warp(b_wfull(sw), (g / WS) & 1, p.wait_ns, fail, p.status, 3))
                break;
            // this lane's channel row of K block `sub` of the stage; the TMA swizzle moved 16-byte
            // chunk j of row r to chunk j ^ (r / 2 % 4) (int8, 64-byte rows) or j ^ (r % 8) (bf16,
            // 128-byte rows), so the warp's 32 rows spread over all banks
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
                mbar_arrive_local(b_wempty(sw));  // the stage is read: the producer may refill it
            tc_st_32cols(tmem + ((uint32_t)(32 * q) << 16) + 256u + (uint32_t)sa * 32u, o);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive_local(b_afull(sa));
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
    __syncthreads();  // every role is done; bias and scale are in shared memory
    const bool go = *fail == 0u;
    if (epi && go) {
        // The accumulator holds a channel per lane and a row per column; Y is row-major.
        // Stage the tile row-major in the X ring (idle: every MMA has completed), then
        // write whole rows with 16-byte stores.  (Storing straight from the lanes gives
        // 64-byte pieces 4 KB apart; draining 8 MB of those kept a layer's grid alive
        // ~18 us after its last CTA had finished.)
        const float sc = s_scale[chan], bi = s_bias[chan];
        const int esz = p.out_f32 ? 4 : 2;
        const int row_bytes = kSwChan * esz;  // one tile row: 256 (bf16) or 512 (fp32) bytes
        uint8_t *stage = smem + L::OFF_X;
        static_assert(kSwRows * kSwChan * 4 <= kSwXStages * L::XB, "fp32 tile fits the X ring");
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        // one instantiation per (activation, output type), chosen once (see tc_finish_64)
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
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps: the tile is staged
        const int cpr = row_bytes / 16;  // 16-byte chunks per row
        uint8_t *out = static_cast<uint8_t *>(p.out);
        for (int idx = tid - 128; idx < kSwRows * cpr; idx += 128) {
            const int r = idx / cpr, ch = idx - r * cpr;
            *reinterpret_cast<uint4 *>(out + ((size_t)(m0 + r) * p.N + n0) * esz + (size_t)ch * 16) =
                *reinterpret_cast<const uint4 *>(stage + (size_t)r * row_bytes + (size_t)ch * 16);
        }
    }

    // ---------------- drain and free ----------------
    tc_fence_before();
    __syncthreads();
    if (tid == 0)
        stamp(kTcTraceEnd);
    if (warp == 1) {
        if (*fail && lane == 0) {
            const uint64_t t0 = globaltimer();
            while (!mbar_try_wait(b_accf, 0) && globaltimer() - t0 < p.wait_ns) {
            }
        }
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kSwTmemCols)
                     : "memory");
    }
}

}  // namespace llk
