// Batched dense layer on the 5th-generation tensor cores (tcgen05 + TMEM), one
// launch per layer:
//
//   Y[rows x N] = act( (X[rows x K] . Wd[N x K]^T) * scale[N] + bias[N] )
//
// X is bf16 (row-major), W is bf16 or int8 (row-major, per-output-channel fp32
// scale applied after accumulation; int8 -> bf16 is exact), accumulation fp32 in
// TMEM, Y bf16 (hidden layers) or fp32 (last layer).
//
// CTA tile: 128 rows x BN output channels, K walked in 64-element steps through a
// STAGES-deep shared-memory ring; the grid's z dimension splits K, and the S
// splits of a tile form one thread-block cluster that adds its partials through L2:
// each CTA stores its partial tile to a scratch buffer, the cluster synchronises,
// and each CTA sums the S partials of its 128/S rows in rank order (deterministic).
// Roles (one CTA per SM):
//   warp 0        TMA producer: X tile [128 x 64] bf16 and W tile [BN x 64]
//                 (bf16 straight into the 128-byte-swizzled operand layout; int8
//                 into a staging buffer);
//   warp 1        TMEM allocation + the single thread that issues tcgen05.mma
//                 (M=128, N=BN, K=16, bf16 x bf16 -> fp32) and tcgen05.commit;
//   warps 4..11   int8 only: convert the staged int8 tile into the swizzled bf16
//                 operand (exact), fence the async proxy, arrive;
//   warps 4..7    epilogue: tcgen05.ld of their 32 TMEM lanes (= tile rows), then
//                 the rows go out (no split) or to the scratch buffer (split-K);
//   all threads   split-K: sum of the cluster's S partials for this CTA's rows.
// Every wait is bounded (globaltimer); a wait that runs out records the error
// and the CTA drains and frees its TMEM before returning.
//
// Reference: the batched configurations have no counterpart kernel in the
// reference (its batched GEMMs are cuBLAS SGEMM calls, src/bench_cublas_mlp.cu);
// the arithmetic follows its layer contract y = act(W x + b).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>

#include "ptx.cuh"

namespace llk {

constexpr int kTcRows = 128;      // tile rows (MMA M)
constexpr int kTcK = 64;          // K per pipeline stage (128 bytes of bf16: one swizzle row)
constexpr int kTcThreads = 384;   // 12 warps
constexpr int kTcEpiWarp0 = 4;    // epilogue warps 4..7
constexpr int kTcConvWarp0 = 4;   // converter warps 4..11
constexpr int kTcConvThreads = 256;

struct TcLayerParams {
    CUtensorMap tm_x;   // bf16 [rows_pad][K], box {64, 128}, 128-byte swizzle
    CUtensorMap tm_w;   // bf16 [N][K] box {64, BN} swizzled, or int8 [N][K] box {64, BN} unswizzled
    const float *bias;  // [N]
    const float *scale; // [N] or nullptr
    void *out;          // bf16 or fp32 [rows_pad][N]
    unsigned *status;   // device error word: bit 0 wait ran out; the failing role in bits 8..15
    int K, N;
    int k_chunk;        // K per split (multiple of 64)
    int splits;         // = cluster size along z: 1, 2, 4, 8 or 16
    int act;            // LL_ACT_*
    int out_f32;
    unsigned long long wait_ns;
    unsigned long long *trace;  // optional: kTcTraceSlots globaltimer stamps per CTA (see kTcTrace*), or null
    float *scratch;             // split-K partials: [tile][split][BN/4][128] float4 (L2-resident)
};

// Trace stamps per CTA (CTA id = x + gridDim.x * (y + gridDim.y * z)).
enum {
    kTcTraceEntry = 0,     // kernel entry
    kTcTraceDepDone = 1,   // previous layer complete (griddepcontrol.wait returned)
    kTcTraceFirstData = 2, // MMA thread: first stage landed (and converted)
    kTcTraceMmaIssued = 3, // MMA thread: last MMA issued
    kTcTraceAccum = 4,     // epilogue: accumulator complete
    kTcTraceClusterA = 5,  // after the first cluster barrier
    kTcTraceClusterB = 6,  // after the partial rows were exchanged
    kTcTraceEnd = 7,       // rows written
    kTcTraceStaged = 8,    // split-K: this CTA's partial tile stored
    kTcTraceStageReady = 9,   // 9..12: MMA thread, K steps 0..3 ready (landed and converted)
    kTcTraceReissue = 13,     // producer: first stage re-issued (after the MMAs freed it)
    kTcTraceReissueReady = 14,// MMA thread: that re-issued stage ready
    kTcTraceConvDone = 15,    // converter warp: K step 0 converted
    kTcTraceSlots = 16
};

// ---- PTX wrappers used only by this kernel ----
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// 3-D tiled load {x, y, z} (the grouped weight boxes: x = K within a 64-wide block,
// y = row, z = 64-wide K block).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *tm, int x, int y, int z, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *tm)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

// Add expected transaction bytes to the current phase without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Bulk copy of this CTA's shared memory into a peer's (cluster address), completing
// the byte count on the peer's mbarrier (cluster address).
__device__ __forceinline__ void mbar_arrive_local(uint32_t bar)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle layout
// (rows of 128 bytes, 8-row atoms of 1024 bytes; leading offset unused = 1,
// stride offset = 1024 bytes between 8-row groups; version 1; layout 2 = 128B swizzle).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr)
{
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: A = B = bf16, D = fp32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t tc_idesc_bf16(int n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 lanes x 64 consecutive fp32 columns: two 32-column loads and one wait in a single
// asm block, so no use of the registers can be scheduled before the wait.
__device__ __forceinline__ void tc_ld_64cols(uint32_t taddr, float (&v)[64])
{
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr), "r"(taddr + 32u)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i)
        v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float tc_act(float v, int act)
{
    if (act == 1)  // LL_ACT_RELU
        return fmaxf(v, 0.0f);
    if (act == 2)  // LL_ACT_GELU: 0.5 x (1 + erf(x / sqrt 2))
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    return v;
}

template <int ACT>
__device__ __forceinline__ float tc_act_t(float v)
{
    if constexpr (ACT == 1)
        return fmaxf(v, 0.0f);
    else if constexpr (ACT == 2)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    else
        return v;
}

// v = act(v * scale + bias) over 64 accumulator columns.  The activation is a template
// argument, chosen once per tile: unrolled 64 times with the run-time switch (GELU's erf
// inlined into every element) the epilogue was ~50 KB of straight-line code that ran once
// per launch, and streaming it through the instruction cache cost ~14 us per tile.
template <int ACT>
__device__ __forceinline__ void tc_finish_64(float (&v)[64], const float *scale, const float *bias)
{
#pragma unroll
    for (int i = 0; i < 64; ++i)
        v[i] = tc_act_t<ACT>(fmaf(v[i], scale[i], bias[i]));
}

// One tile row (this thread's TMEM lane) finished into its row of the staging tile.
template <int BN, int ACT>
__device__ __forceinline__ void tc_stage_rows(uint32_t tq, uint8_t *srow, const float *scale, const float *bias,
                                              bool out_f32)
{
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 64) {
        float v[64];
        tc_ld_64cols(tq + (uint32_t)c0, v);
        tc_finish_64<ACT>(v, scale + c0, bias + c0);
        if (out_f32) {
            float4 *dst = reinterpret_cast<float4 *>(srow + (size_t)c0 * 4);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
            uint4 *dst = reinterpret_cast<uint4 *>(srow + (size_t)c0 * 2);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                uint32_t u[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * i + 2 * e], v[8 * i + 2 * e + 1]);
                    u[e] = *reinterpret_cast<const uint32_t *>(&h);
                }
                dst[i] = make_uint4(u[0], u[1], u[2], u[3]);
            }
        }
    }
}

// Bounded mbarrier wait; false when the bound ran out (or another role already failed).
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, unsigned long long bound_ns,
                                        volatile uint32_t *fail, unsigned *status, uint32_t role)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity))
            return true;
        if ((it & 63u) == 0) {
            if (*fail)
                return false;
            if (globaltimer() - t0 > bound_ns) {
                *fail = 1u;
                atomicOr(status, 1u | (role << 8));
                return false;
            }
        }
    }
}

// Warp-collective bounded wait: every lane observes the phase itself (so the
// data the phase guards is visible to each of them) and the verdict is uniform
// across the warp, so the warp never splits at a later __syncwarp or bar.sync.
__device__ __forceinline__ bool tc_wait_warp(uint32_t bar, uint32_t parity, unsigned long long bound_ns,
                                             volatile uint32_t *fail, unsigned *status, uint32_t role)
{
    const int lane = threadIdx.x & 31;
    const uint64_t t0 = lane == 0 ? globaltimer() : 0;
    bool done = mbar_try_wait(bar, parity);
    for (uint32_t it = 1;; ++it) {
        if (__all_sync(0xffffffffu, done))
            return true;
        if ((it & 63u) == 0) {
            uint32_t give_up = 0;
            if (lane == 0) {
                if (*fail) {
                    give_up = 1;
                } else if (globaltimer() - t0 > bound_ns) {
                    *fail = 1u;
                    atomicOr(status, 1u | (role << 8));
                    give_up = 1;
                }
            }
            if (__shfl_sync(0xffffffffu, give_up, 0))
                return false;
        }
        if (!done)
            done = mbar_try_wait(bar, parity);
    }
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b)
{
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// 4 int8 (k order) -> 2 bf16x2 words, exact for every int8 value: the bf16 with bits
// 0x43mm is 128 + mm for a magnitude mm in [0, 128] (7 stored mantissa bits; 0x4380 is
// 256), so 0x43|mm minus 128 is the exact magnitude; the sign bit of each source byte
// is then copied to bit 15 of its half (prmt's sign-replicating selector nibbles 8..b).
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t &lo, uint32_t &hi)
{
    const uint32_t mag = __vabs4(w);  // per-byte |v|, -128 -> 0x80 = 128
    const uint32_t c128 = 0x43004300u;
    lo = bf16x2_sub(prmt(mag, 0x43434343u, 0x4140u), c128);
    hi = bf16x2_sub(prmt(mag, 0x43434343u, 0x4342u), c128);
    lo |= prmt(w, 0u, 0x9484u) & 0x80008000u;
    hi |= prmt(w, 0u, 0xB4A4u) & 0x80008000u;
}

// 16 int8 -> 16 bf16 (exact), packed as 8 bf16x2 words in k order.
__device__ __forceinline__ void i8x16_to_bf16(uint4 q, uint32_t (&o)[8])
{
    i8x4_to_bf16x4(q.x, o[0], o[1]);
    i8x4_to_bf16x4(q.y, o[2], o[3]);
    i8x4_to_bf16x4(q.z, o[4], o[5]);
    i8x4_to_bf16x4(q.w, o[6], o[7]);
}

template <int BN, bool WINT8, int STAGES>
struct TcSmem {
    static constexpr int XB = kTcRows * kTcK * 2;   // X tile bytes (16 KB)
    static constexpr int WB = BN * kTcK * 2;        // W bf16 tile bytes
    static constexpr int QB = WINT8 ? BN * kTcK : 0; // W int8 staging bytes
    static constexpr int OFF_X = 0;
    static constexpr int OFF_W = STAGES * XB;
    static constexpr int OFF_Q = OFF_W + STAGES * WB;
    static constexpr int PIPE_END = OFF_Q + STAGES * QB;
    // without a split: the finished tile, row-major (RSO bytes per row, padded), at offset 0
    static constexpr int RSO = BN * 4 + 16;
    // split-K for the 64- and 128-wide tiles (a split 256-wide tile would move 128 KB of
    // fp32 partials per CTA)
    static constexpr bool CAN_SPLIT = BN <= 128;
    static constexpr int OFF_BAR = (PIPE_END + 1023) / 1024 * 1024;  // full[S], qfull[S], conv[S], empty[S], accf
    static constexpr int N_BAR = 4 * STAGES + 1;
    static constexpr int OFF_MISC = OFF_BAR + 8 * N_BAR;          // tmem base, fail flag
    static constexpr int OFF_BIAS = OFF_MISC + 16;                // bias[BN], scale[BN]
    static constexpr int BYTES = OFF_BIAS + 8 * BN;
    static constexpr int ALLOC = BYTES + 1024;                    // slack to align the base to 1024
    static_assert(XB % 1024 == 0 && WB % 1024 == 0 && QB % 1024 == 0, "1024-byte aligned tiles");
    static_assert(BN == 64 || BN == 128 || BN == 256, "N tile");
    static_assert(ALLOC <= 227 * 1024, "shared memory");
    static_assert(kTcRows * RSO <= PIPE_END, "the finished tile fits the idle pipeline buffers");
    static_assert(kTcRows / 2 * (BN + 4) * 4 <= PIPE_END, "split-K sums (at most 64 rows) fit them too");
};

template <int BN, bool WINT8, int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1) ll_tc_layer_kernel(const __grid_constant__ TcLayerParams p)
{
    using L = TcSmem<BN, WINT8, STAGES>;
    extern __shared__ uint8_t tc_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint32_t *misc = reinterpret_cast<uint32_t *>(smem + L::OFF_MISC);
    volatile uint32_t *fail = misc + 1;
    float *s_bias = reinterpret_cast<float *>(smem + L::OFF_BIAS);
    float *s_scale = s_bias + BN;
    auto bar = [&](int i) { return sbase + (uint32_t)L::OFF_BAR + 8u * (uint32_t)i; };
    // barrier indices
    auto b_full = [&](int s) { return bar(s); };
    auto b_qfull = [&](int s) { return bar(STAGES + s); };
    auto b_conv = [&](int s) { return bar(2 * STAGES + s); };
    auto b_empty = [&](int s) { return bar(3 * STAGES + s); };
    const uint32_t b_accf = bar(4 * STAGES);

    const uint32_t cta_lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    auto stamp = [&](int k) {
        if (p.trace)
            p.trace[cta_lin * (uint32_t)kTcTraceSlots + (uint32_t)k] = globaltimer();
    };
    if (tid == 0)
        stamp(kTcTraceEntry);
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * kTcRows;
    const int k0 = blockIdx.z * p.k_chunk;
    const int nk = p.k_chunk / kTcK;
    const int S = p.splits;
    const int R = kTcRows / S;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(b_full(s), WINT8 ? 1 : 2);  // bf16: the X and the W producer each arrive
            mbar_init(b_qfull(s), 1);
            mbar_init(b_conv(s), kTcConvThreads / 32);
            mbar_init(b_empty(s), 1);
        }
        mbar_init(b_accf, 1);
        misc[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        prefetch_tmap(&p.tm_x);
        prefetch_tmap(&p.tm_w);
    }
    if (warp == 1) {  // whole warp: allocate BN TMEM columns (power of two >= 32)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         sbase + (uint32_t)L::OFF_MISC),
                     "r"((uint32_t)BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];
    griddep_launch_dependents();  // the next layer may start its own set-up on free SMs

    // Two TMA issuers: one thread issuing back-to-back tensor loads holds each for
    // hundreds of cycles, so X and W come from different threads (measured on B200:
    // 52 -> 83 B/clock per SM for 32 KB boxes with a second issuer).  Weights, biases
    // and scales do not depend on the previous layer: their issuer and loaders start
    // before (and never wait for) the dependency, hiding behind the previous layer's tail.
    if (warp == 2) {
        // ---------------- W producer ----------------
        if (lane == 0) {
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                if (kb >= STAGES && !tc_wait(b_empty(s), ((kb / STAGES) - 1) & 1, p.wait_ns, fail, p.status, 1))
                    break;
                const int kx = k0 + kb * kTcK;
                if (WINT8) {
                    mbar_arrive_expect_tx(b_qfull(s), L::QB);
                    tma_load_2d(sbase + L::OFF_Q + s * L::QB, &p.tm_w, kx, n0, b_qfull(s));
                } else {
                    mbar_arrive_expect_tx(b_full(s), L::WB);
                    tma_load_2d(sbase + L::OFF_W + s * L::WB, &p.tm_w, kx, n0, b_full(s));
                }
            }
        }
    } else if (warp == 3) {
        for (int i = lane; i < BN; i += 32) {
            s_bias[i] = __ldg(p.bias + n0 + i);
            s_scale[i] = p.scale ? __ldg(p.scale + n0 + i) : 1.0f;
        }
    } else {
        griddep_wait();  // X belongs to the previous layer (and Y to the one before it) until here
    }
    if (tid == 0)
        stamp(kTcTraceDepDone);

    if (warp == 0) {
        // ---------------- X producer ----------------
        if (lane == 0) {
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                if (kb >= STAGES && !tc_wait(b_empty(s), ((kb / STAGES) - 1) & 1, p.wait_ns, fail, p.status, 1))
                    break;
                if (kb == STAGES)
                    stamp(kTcTraceReissue);
                mbar_arrive_expect_tx(b_full(s), L::XB);
                tma_load_2d(sbase + L::OFF_X + s * L::XB, &p.tm_x, k0 + kb * kTcK, m0, b_full(s));
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc_bf16(BN);
            bool ok = true;
            for (int kb = 0; kb < nk && ok; ++kb) {
                const int s = kb % STAGES;
                const uint32_t ph = (kb / STAGES) & 1;
                ok = tc_wait(b_full(s), ph, p.wait_ns, fail, p.status, 2);
                if (ok && WINT8)
                    ok = tc_wait(b_conv(s), ph, p.wait_ns, fail, p.status, 2);
                if (!ok)
                    break;
                if (kb == 0)
                    stamp(kTcTraceFirstData);
                if (kb < 4)
                    stamp(kTcTraceStageReady + kb);
                if (kb == STAGES)
                    stamp(kTcTraceReissueReady);
                tc_fence_after();
                const uint32_t xa = sbase + L::OFF_X + s * L::XB, wa = sbase + L::OFF_W + s * L::WB;
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; ++kk)
                    tc_mma_bf16(tmem, sw128_kmajor_desc(xa + kk * 32), sw128_kmajor_desc(wa + kk * 32), idesc,
                                (kb | kk) != 0);
                tc_commit(b_empty(s));  // frees stage s when these MMAs complete
            }
            stamp(kTcTraceMmaIssued);
            tc_commit(b_accf);  // accumulator complete (also arrives when nothing was issued)
        }
    } else if (WINT8 && warp >= kTcConvWarp0) {
        // ---------------- int8 -> bf16 operand conversion ----------------
        const int ct = tid - kTcConvWarp0 * 32;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            if (!tc_wait_warp(b_qfull(s), (kb / STAGES) & 1, p.wait_ns, fail, p.status, 3))
                break;
            const uint8_t *q = smem + L::OFF_Q + s * L::QB;
            uint8_t *w = smem + L::OFF_W + s * L::WB;
            for (int c = ct; c < BN * 4; c += kTcConvThreads) {
                const int r = c >> 2, j = c & 3;  // row, 16-byte piece of the 64-byte int8 row
                const uint4 v = *reinterpret_cast<const uint4 *>(q + r * 64 + j * 16);
                uint32_t o[8];
                i8x16_to_bf16(v, o);
                uint8_t *row = w + r * 128;
                *reinterpret_cast<uint4 *>(row + (((2 * j) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
                *reinterpret_cast<uint4 *>(row + (((2 * j + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
            }
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core (async proxy)
            __syncwarp();
            if (lane == 0)
                mbar_arrive_local(b_conv(s));
            if (kb == 0 && tid == kTcConvWarp0 * 32)
                stamp(kTcTraceConvDone);
        }
    }

    // ---------------- epilogue ----------------
    // Warps 4..7 read the accumulator (warp w owns TMEM lanes 32*(w%4)..+31 = tile rows).
    // Without a K split they finish their rows (through a row-major staging tile).  With a
    // split, every CTA stores its whole partial tile to the scratch buffer in L2
    // ([BN/4][128] float4: a warp's 32 rows of one 4-column group are 512 consecutive
    // bytes), the cluster synchronises (release/acquire at cluster scope), and each CTA
    // adds the S partials of its R = 128/S rows in rank order (deterministic) and
    // finishes them.  The stores and the cluster barrier run on every path, failed or
    // not; only the final writes depend on success.  (Measured: 4 % faster per forward
    // than sending the rows to their owners through distributed shared memory.)
    const bool epi = warp >= kTcEpiWarp0 && warp < kTcEpiWarp0 + 4;
    const int q = warp & 3;
    const int trow = 32 * q + lane;  // tile row of this epilogue thread
    if (epi) {
        tc_wait_warp(b_accf, 0, p.wait_ns, fail, p.status, 4);
        tc_fence_after();
        if (tid == kTcEpiWarp0 * 32)
            stamp(kTcTraceAccum);
    }
    const uint32_t rank = S > 1 ? cluster_ctarank() : 0u;
    __syncthreads();
    if (tid == 0)
        stamp(kTcTraceClusterA);
    const bool go = *fail == 0u;  // the roles have all finished: stable from here on
    if (epi && (go || S > 1)) {
        const uint32_t tq = tmem + ((uint32_t)(32 * q) << 16);
        if (S == 1) {
            // finished rows go to a row-major staging tile in the (idle) pipeline buffers,
            // written out below with whole-row stores; one instantiation per activation
            uint8_t *srow = smem + (size_t)trow * L::RSO;
            if (p.act == 1)
                tc_stage_rows<BN, 1>(tq, srow, s_scale, s_bias, p.out_f32 != 0);
            else if (p.act == 2)
                tc_stage_rows<BN, 2>(tq, srow, s_scale, s_bias, p.out_f32 != 0);
            else
                tc_stage_rows<BN, 0>(tq, srow, s_scale, s_bias, p.out_f32 != 0);
        }
        float4 *part = S > 1 ? reinterpret_cast<float4 *>(p.scratch) +
                                   ((size_t)(blockIdx.x + gridDim.x * blockIdx.y) * S + rank) * (kTcRows * (BN / 4))
                             : nullptr;
#pragma unroll 1
        for (int c0 = 0; S > 1 && c0 < BN; c0 += 64) {
            float v[64];
            tc_ld_64cols(tq + (uint32_t)c0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i)
                part[(size_t)(c0 / 4 + i) * kTcRows + trow] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    }
    if (S == 1 && epi && go) {
        // Whole rows out of the staging tile: consecutive threads write consecutive 16-byte
        // pieces of one row.  (Each thread storing its own row gives 32 rows' 16-byte
        // pieces per warp store; draining those kept a stacked layer's grid alive for
        // ~12 us after its last CTA had finished.)
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps: tile staged
        const int esz = p.out_f32 ? 4 : 2;
        const int cpr = BN * esz / 16;  // 16-byte pieces per row
        uint8_t *out = static_cast<uint8_t *>(p.out);
        for (int idx = tid - kTcEpiWarp0 * 32; idx < kTcRows * cpr; idx += 128) {
            const int r = idx / cpr, ch = idx - r * cpr;
            *reinterpret_cast<uint4 *>(out + ((size_t)(m0 + r) * p.N + n0) * esz + (size_t)ch * 16) =
                *reinterpret_cast<const uint4 *>(smem + (size_t)r * L::RSO + (size_t)ch * 16);
        }
    }
    if (S > 1) {
        if (tid == kTcEpiWarp0 * 32)
            stamp(kTcTraceStaged);
        // every CTA of the cluster has stored its partial tile (release/acquire at cluster
        // scope orders those global stores before the reads below)
        __syncwarp();
        cluster_sync();
        if (tid == 0)
            stamp(kTcTraceClusterB);
        if (go && *fail == 0u) {
            constexpr int C4 = BN / 4;
            const float4 *tile_parts = reinterpret_cast<const float4 *>(p.scratch) +
                                       (size_t)(blockIdx.x + gridDim.x * blockIdx.y) * S * (kTcRows * C4);
            // (1) sums, row-fastest so the L2 loads are coalesced: a thread issues the loads of
            // up to 3 items x 4 partials before adding (rank order kept), into a padded
            // row-major tile in the idle pipeline buffers
            constexpr int SR = BN + 4;  // staged row stride in floats (16-byte pad: no bank conflicts)
            float *sums = reinterpret_cast<float *>(smem);
            const int n_items = R * C4;
            for (int base = tid; base < n_items; base += 3 * kTcThreads) {
                float4 acc[3];
#pragma unroll
                for (int u = 0; u < 3; ++u)
                    acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int s0 = 0; s0 < S; s0 += 4) {
                    float4 v[3][4];
#pragma unroll
                    for (int u = 0; u < 3; ++u) {
                        const int idx = base + u * kTcThreads, r = idx % R, c4 = idx / R;
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (idx < n_items && s0 + j < S)
                                v[u][j] = __ldcg(tile_parts + (size_t)(s0 + j) * (kTcRows * C4) +
                                                 (size_t)c4 * kTcRows + (int)rank * R + r);
                    }
#pragma unroll
                    for (int u = 0; u < 3; ++u)
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (base + u * kTcThreads < n_items && s0 + j < S) {
                                acc[u].x += v[u][j].x;
                                acc[u].y += v[u][j].y;
                                acc[u].z += v[u][j].z;
                                acc[u].w += v[u][j].w;
                            }
                }
#pragma unroll
                for (int u = 0; u < 3; ++u) {
                    const int idx = base + u * kTcThreads;
                    if (idx < n_items)
                        *reinterpret_cast<float4 *>(sums + (idx % R) * SR + (idx / R) * 4) = acc[u];
                }
            }
            __syncthreads();
            // (2) finish and write whole rows: consecutive threads, consecutive columns
            for (int idx = tid; idx < n_items; idx += kTcThreads) {
                const int r = idx / C4, c = (idx % C4) * 4;
                const float4 a = *reinterpret_cast<const float4 *>(sums + r * SR + c);
                float o4[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    o4[e] = tc_act(fmaf(o4[e], s_scale[c + e], s_bias[c + e]), p.act);
                const size_t off = (size_t)(m0 + (int)rank * R + r) * p.N + n0 + c;
                if (p.out_f32) {
                    *reinterpret_cast<float4 *>(static_cast<float *>(p.out) + off) =
                        make_float4(o4[0], o4[1], o4[2], o4[3]);
                } else {
                    const __nv_bfloat162 h0 = __floats2bfloat162_rn(o4[0], o4[1]);
                    const __nv_bfloat162 h1 = __floats2bfloat162_rn(o4[2], o4[3]);
                    *reinterpret_cast<uint2 *>(static_cast<__nv_bfloat16 *>(p.out) + off) =
                        make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
                }
            }
        }
    }

    // ---------------- drain and free ----------------
    // A role that gave up leaves copies or MMAs in flight: wait (bounded) until the
    // accumulator barrier shows every issued MMA finished before TMEM is freed.
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
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN)
                     : "memory");
    }
}

}  // namespace llk
