// Small-batch MLP forward (1..32 rows) as ONE cooperative launch over every SM:
// matrix-by-vector per layer with a grid-wide layer barrier, for the batch sweep
// of bf16 / int8 nets whose rows are too few for the tensor-core tiles.
//
// Mapping (one CTA per SM, G CTAs):
//   * layer l's output channels are split into G contiguous row slices; CTA c owns
//     rows [c*N/G, (c+1)*N/G).  At entry the CTA bulk-copies its slice of EVERY
//     layer's weights, with its biases and scales, into shared memory from a
//     per-CTA image packed at create time: two copies (biases + layer 0, then the
//     other layers), since each bulk copy costs its issuing thread ~0.3 us.
//     Weights do not depend on activations, so the whole net streams from HBM at
//     once while layer 0 runs, and no weight byte is read twice;
//   * layers hand off through L2, by one of two protocols chosen by batch size:
//     - up to 4 rows (latency-bound): self-validating words.  A hidden output is
//       one 32-bit word {bf16 value in the high half, 16-bit tag in the low half},
//       tag = (forward, layer) number, written with a relaxed store and no fence;
//       a consumer polls the words it needs (16-byte loads, several in flight,
//       stale ones re-read together, bounded) until every tag is the expected one.
//       A 32-bit access is single-copy atomic, so a matching tag vouches for its
//       value: the layer barrier costs one L2 trip instead of a release fence, a
//       counter and a second read.  The host clears the words before the 16-bit
//       tags wrap, so a stale word never carries a current tag;
//     - 8 rows and more (volume-bound: every CTA reads rows x in_dim values):
//       plain bf16 outputs (half the bytes) and an arrival counter per layer; a
//       producer adds 1 with release semantics after its stores, a consumer's
//       thread 0 waits (acquire, bounded) for all producers and the CTA then reads
//       the rows once with L2-coherent loads, all in flight;
//     every CTA reads the same rows, so each starts at its own offset to spread the
//     reads over the L2 slices;
//   * inside a CTA the 8 warps split K; a lane owns one K chunk (16 weight bytes)
//     and BPL batch rows at a time (lane = k-lane * BG + batch group, rows
//     b = bg + BG*i), weight chunks are broadcast reads, the K lanes reduce with
//     shuffles and the warps through shared memory; the epilogue applies the
//     int8 scale, the bias and the activation and rounds hidden outputs to bf16.
// Every wait is bounded by wait_ns; a CTA that gives up records the failing
// layer in the status word, lets its own bulk copies land and returns, so the
// others time out too and the host reads the error (no trap, no endless spin).
//
// Resident mode (RES = true: the engine's kernel variant 3): the same CTAs stay up
// and serve requests, the weight slices loaded once and kept in shared memory.
//   * CTA 0 polls the host-mapped TickBuffer (seq_in, acquire; stop and the idle
//     bound on a cadence) or takes the next request of a device queue, copies the
//     request's x rows into an L2 relay buffer and publishes a 64-bit request word
//     {seq, rows, cmd} with release; the other CTAs poll it (acquire, bounded by the
//     idle bound + a margin) and read x from the relay like a hidden layer;
//   * the last layer's outputs go to an L2 gather buffer behind an arrival counter;
//     CTA 0 copies them into the mailbox's y rows and release-stores seq_out;
//   * tags and counters restart at every launch (the host clears them); before the
//     16-bit tags would wrap, the kernel leaves (exit reason "tags") and the host
//     relaunches it on the next request, as after an idle exit.
//
// Reference: the per-layer contract y = act(W x + b) over row-major W is
// cpu_gemv_bias_relu (src/bench_persistent_mbyv_mlp.cu:50-67); the grid-wide
// layer barrier replaces the reference's global-atomic layer barrier of the
// persistent MByV kernel (src/bench_persistent_mbyv_mlp.cu:308-377).
#pragma once
#include <cuda_bf16.h>

#include <cstdint>

#include "engine_types.h"
#include "ll_b200.h"
#include "ptx.cuh"

namespace llk {

constexpr int kGvThreads = 256;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kGvRowGroup = 8;   // output rows per pass (accumulators per lane: 8 x BPL)
constexpr int kGvMaxRows = 32;   // batch rows per launch
constexpr int kGvTagRows = 4;     // batch rows up to which layers hand off in tagged words
constexpr int kGvCntStride = 32;  // one arrival counter per 128-byte line
constexpr int kGvUnroll = 16;     // 16-byte loads in flight per thread while staging
// Tags are 1..kGvTagLimit; before a forward whose tags would pass it the host clears
// the hand-off words (tag 0 = never written) and starts again from 1.
constexpr uint32_t kGvTagLimit = 0xffffu;
// A CTA leaving after a failed wait first lets its weight copies land; a copy from
// HBM takes microseconds, so this bound only matters if the device is broken.
constexpr unsigned long long kGvDrainNs = 1000ull * 1000 * 1000;

// Per-CTA trace slots (within the 16-slot per-layer trace of the batched path):
// per layer 0..2; layer 0's record also holds the prologue stamps 3..7.
enum {
    kGvTraceInput = 0,      // the layer's input rows are staged (all tags seen)
    kGvTraceReady = 1,      // ... and its weight slice has landed
    kGvTracePublished = 2,  // outputs stored
    kGvTraceEntry = 3,      // kernel entry (barriers initialised)
    kGvTraceCopy0 = 4,      // first image copy issued (biases + layer 0)
    kGvTraceCopies = 5,     // second image copy issued
    kGvTraceMath = 8,       // per layer, first row group: products summed within the warps
    kGvTraceReduced = 9,    // ... partial sums in shared memory
    kGvTraceStored = 10     // ... outputs stored
};

// Resident mode: the engine's mailbox / queue and the L2 buffers between CTA 0 and the rest.
struct GemvResident {
    ll_tick_header *mb;        // the TickBuffer (device view of the mapped host memory)
    const float *mb_x;         // its x rows [max_batch][in]
    float *mb_y;               // its y rows [max_batch][out]
    EngineCtrl *ctrl;          // state, status, exit reason, counters (mapped host memory)
    float *relay_x;            // [32][in] fp32: the current request's rows, for every CTA
    float *gather_y;           // [32][out] fp32: the last layer's outputs, for CTA 0
    unsigned long long *req;   // request word: seq | rows << 32 | cmd << 48 (0 at launch)
    int mode;                  // MODE_MAILBOX or MODE_QUEUE
    int tagged;                // the tagged mailbox (batch 1): x and y in chunks {v0, v1, v2, seq}
    int max_rows;              // the mailbox's rows (max_batch <= the instantiation's rows)
    uint32_t last_seq;         // the last request answered before this launch
    unsigned long long idle_ns, peer_margin_ns;
    const float *q_x;          // queue mode: q_n requests of q_rows rows, back to back
    float *q_y;
    int q_n, q_rows;
    unsigned long long *q_stamp;  // queue mode: globaltimer when each request's y is stored
};

struct GemvNetParams {
    unsigned long long *trace[LL_MAX_LAYERS];  // per layer: 16 slots per CTA, or null
    const uint8_t *img;                 // per-CTA images, img_bytes apart: the CTA's shared-memory
                                        // prefix (biases / scales at boff, weight slices at woff)
    int dims[LL_MAX_LAYERS + 1];
    int acts[LL_MAX_LAYERS];
    int rmax[LL_MAX_LAYERS];            // ceil(N_l / G): rows of the largest slice
    uint32_t woff[LL_MAX_LAYERS];       // byte offset of the layer's weight slice in shared memory
    uint32_t boff[LL_MAX_LAYERS];       // float offset of the layer's bias (+ scale) slice
    int n_layers;
    int n_rows;                         // batch rows of this launch, 1..32
    int xstride;                        // floats per staged input row (largest in_dim + 4)
    uint32_t img_bytes;                 // per-CTA image (a multiple of 16)
    uint32_t img_a_bytes;               // its first copy: biases + layer 0 (the second: the rest)
    uint32_t off_part, off_bar, off_x;  // shared-memory layout, bytes (the image starts at 0)
    const float *x;                     // [n_rows][dims[0]] fp32, 16-byte aligned
    float *y;                           // [n_rows][dims[L]] fp32
    uint32_t *hand[2];                  // tagged hand-off words [4][widest layer]: bf16 << 16 | tag
    uint32_t tag_base;                  // tag of layer l's outputs = tag_base + l (1..65535)
    __nv_bfloat16 *act[2];              // counted hand-off rows [32][widest layer] bf16
    unsigned *cnt;                      // arrival counters, layer l at cnt[l * kGvCntStride]
    unsigned epoch;                     // forward number: layer l's counter reaches epoch * producers
    unsigned *status;                   // bit 0: a wait ran out; bits 8..15: 16 + failing layer
    unsigned long long wait_ns;
    GemvResident res;                   // resident mode only
};

// Resident mode, tagged mailbox (warp 0 of CTA 0): waits for the request after `last`, whose
// x chunks {v0, v1, v2, seq} carry the new sequence number in every chunk, and writes x into
// `relay` -- detection and the x read are one PCIe round trip.  Stop and the idle bound are
// checked every 64 polls.  Returns 0 with *seq set, or 1 (leave) with *reason set.
__device__ __forceinline__ uint32_t gv_poll_tagged(const GemvResident &rs, uint32_t last, float *relay, int in_dim,
                                                   uint32_t *seq, uint32_t *reason)
{
    constexpr int kChunks = 4;  // 128 chunks per warp: in_dim <= 384 (the tagged format's limit)
    const int lane = threadIdx.x & 31;
    const int nxc = (in_dim + 2) / 3;
    const uint4 *chunks = reinterpret_cast<const uint4 *>(rs.mb_x);
    uint32_t want = last + 1u;
    if (want == 0u || want == LL_STOP_SEQ)
        want = 1u;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        uint4 v[kChunks];
        bool ok = true;
#pragma unroll
        for (int j = 0; j < kChunks; ++j)
            if (lane + 32 * j < nxc)
                v[j] = ld_relaxed_sys_v4_u32(reinterpret_cast<const unsigned *>(chunks + lane + 32 * j));
#pragma unroll
        for (int j = 0; j < kChunks; ++j)
            if (lane + 32 * j < nxc && v[j].w != want)
                ok = false;
        if (__all_sync(0xffffffffu, ok)) {
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
                const int ch = lane + 32 * j;
                if (ch < nxc) {
                    const float f[3] = {__uint_as_float(v[j].x), __uint_as_float(v[j].y), __uint_as_float(v[j].z)};
#pragma unroll
                    for (int e = 0; e < 3; ++e)
                        if (3 * ch + e < in_dim)
                            relay[3 * ch + e] = f[e];
                }
            }
            *seq = want;
            return 0u;
        }
        if ((it & 63u) == 63u) {
            uint32_t verdict = 0u;
            if (lane == 0) {
                if (ld_relaxed_sys(&rs.mb->stop))
                    verdict = EXIT_STOP;
                else if (globaltimer() - t0 > rs.idle_ns)
                    verdict = EXIT_IDLE;
            }
            verdict = __shfl_sync(0xffffffffu, verdict, 0);
            if (verdict) {
                *reason = verdict;
                return 1u;
            }
        }
    }
}

__device__ __forceinline__ void gv_st_release_u64(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long gv_ld_acquire_u64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float gv_bf16_lo(uint32_t u)
{
    return __uint_as_float(u << 16);
}

__device__ __forceinline__ float gv_bf16_hi(uint32_t u)
{
    return __uint_as_float(u & 0xffff0000u);
}

__device__ __forceinline__ float gv_round_bf16(float v)
{
    return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float gv_act(float v, int act)
{
    if (act == LL_ACT_RELU)
        return fmaxf(v, 0.0f);
    if (act == LL_ACT_GELU)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
    return v;
}

__device__ __forceinline__ void gv_st_word(uint32_t *p, uint32_t v)
{
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint4 gv_ld_words(const uint4 *p)
{
    uint4 v;
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Wrap-safe: the counter of layer l grows by (producers of l) per forward.
__device__ __forceinline__ bool gv_wait_count(const unsigned *cnt, unsigned target, unsigned long long bound_ns)
{
    if ((int)(ld_acquire_gpu(cnt) - target) >= 0)
        return true;
    const uint64_t t0 = globaltimer();
    for (;;) {
        if ((int)(ld_acquire_gpu(cnt) - target) >= 0)
            return true;
        if (globaltimer() - t0 > bound_ns)
            return false;
    }
}

__device__ __forceinline__ bool gv_tags_are(uint4 v, uint32_t tag)
{
    return ((v.x & 0xffffu) == tag) & ((v.y & 0xffffu) == tag) & ((v.z & 0xffffu) == tag) &
           ((v.w & 0xffffu) == tag);
}

__device__ __forceinline__ bool gv_wait_bar(uint32_t bar, unsigned long long bound_ns)
{
    if (mbar_try_wait(bar, 0))
        return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, 0))
        if (globaltimer() - t0 > bound_ns)
            return false;
    return true;
}

__device__ __forceinline__ void gv_stamp(unsigned long long *tr, int slot)
{
    if (tr)
        tr[slot] = globaltimer();
}

// 16 weight bytes -> CH floats (bf16: 8 values, exact; int8: 16 values, exact).
template <bool WINT8>
__device__ __forceinline__ void gv_weights(uint4 q, float (&w)[WINT8 ? 16 : 8])
{
    const uint32_t u[4] = {q.x, q.y, q.z, q.w};
    if constexpr (WINT8) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                w[4 * j + e] = (float)(int8_t)(u[j] >> (8 * e));
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w[2 * j] = gv_bf16_lo(u[j]);
            w[2 * j + 1] = gv_bf16_hi(u[j]);
        }
    }
}

template <bool WINT8, int BG, int BPL, bool RES = false>
__global__ void __launch_bounds__(kGvThreads, 1) ll_gemv_net_kernel(const __grid_constant__ GemvNetParams p)
{
    extern __shared__ __align__(128) uint8_t gv_dynamic_smem[];
    uint8_t *const smem = gv_dynamic_smem;
    constexpr int BP = BG * BPL;         // batch rows this instantiation covers
    constexpr int KL = 32 / BG;          // lanes along K in a warp
    constexpr int CH = WINT8 ? 16 : 8;   // K elements per 16-byte weight chunk
    constexpr int ES = WINT8 ? 1 : 2;    // weight element size
    constexpr bool kTagged = BP <= kGvTagRows;  // hand-off protocol (see the top of this file)
    static_assert(BP <= kGvMaxRows && (32 % BG) == 0, "batch mapping");
    static_assert(sizeof(GemvNetParams) % 4 == 0, "parameter copy");

    // The per-layer tables are indexed at run time; read from the parameter space
    // every such access is a constant-cache miss, so the CTA copies them once, all
    // threads in parallel, and reads the shared-memory copy.
    __shared__ GemvNetParams sp;
    __shared__ uint32_t s_fail;
    __shared__ uint32_t s_req[3];  // resident mode: seq, rows, cmd of the request being served
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kl = lane / BG, bg = lane - kl * BG;
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    const uint32_t sbase = smem_u32(smem);
    {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&p);
        uint32_t *dst = reinterpret_cast<uint32_t *>(&sp);
        for (int i = tid; i < (int)(sizeof(GemvNetParams) / 4); i += kGvThreads)
            dst[i] = src[i];
    }
    if (tid == 0) {
        s_fail = 0u;
        mbar_init(sbase + p.off_bar, 1);       // image copy A: biases + layer 0
        mbar_init(sbase + p.off_bar + 8u, 1);  // image copy B: layers 1..
        fence_mbar_init_cluster();
    }
    __syncthreads();
    const int L = sp.n_layers, XS = sp.xstride;
    int nr = sp.n_rows;
    float *xs = reinterpret_cast<float *>(smem + sp.off_x);
    float *part = reinterpret_cast<float *>(smem + sp.off_part);
    const float *sbias = reinterpret_cast<const float *>(smem);
    const uint32_t bar_a = sbase + sp.off_bar, bar_b = bar_a + 8u;
    const bool has_b = sp.img_bytes > sp.img_a_bytes;

    auto slice = [&](int l, int &r0) {
        const unsigned N = (unsigned)sp.dims[l + 1];
        r0 = (int)((unsigned)c * N / (unsigned)G);
        return (int)((unsigned)(c + 1) * N / (unsigned)G) - r0;
    };

    unsigned long long *tr0 = sp.trace[0] ? sp.trace[0] + (size_t)c * 16 : nullptr;
    if (tid == 0) {
        gv_stamp(tr0, kGvTraceEntry);
        const uint8_t *img = sp.img + (size_t)c * sp.img_bytes;
        mbar_arrive_expect_tx(bar_a, sp.img_a_bytes);
        bulk_g2s(sbase, img, sp.img_a_bytes, bar_a);
        gv_stamp(tr0, kGvTraceCopy0);
        if (has_b) {
            mbar_arrive_expect_tx(bar_b, sp.img_bytes - sp.img_a_bytes);
            bulk_g2s(sbase + sp.img_a_bytes, img + sp.img_a_bytes, sp.img_bytes - sp.img_a_bytes, bar_b);
        }
        gv_stamp(tr0, kGvTraceCopies);
    }
    bool a_ready = false, b_ready = false;
    if constexpr (!RES) {
        // batch rows past n_rows stay zero in the staged input for the whole launch
        for (int i = tid; i < (BP - nr) * XS; i += kGvThreads)
            xs[(size_t)nr * XS + i] = 0.0f;
    } else {
        // the weight slices stay for the whole launch: wait for both copies once
        bool ok = gv_wait_bar(bar_a, sp.wait_ns) && (!has_b || gv_wait_bar(bar_b, sp.wait_ns));
        if (!ok && tid == 0) {
            s_fail = 1u;
            atomicOr(sp.status, 1u | (15u << 8));
        }
        a_ready = b_ready = true;
        __syncthreads();
        if (c == 0 && tid == 0 && !s_fail)
            st_relaxed_sys_u32(&sp.res.ctrl->state, ST_RUNNING);
    }
    uint32_t last = RES ? sp.res.last_seq : 0u, tag = 1u, served = 0u, rows_served = 0u;
    unsigned long long last_word = 0ull;  // resident mode: the request word last seen

    for (uint32_t n_req = 0; !s_fail; ++n_req) {
        uint32_t seq = 0;
        if constexpr (RES) {
            // ---------------- request: CTA 0 takes it, the others read the request word ----------------
            const GemvResident &rs = sp.res;
            if (c == 0) {
                // the tagged mailbox (batch 1, so only the 1-row instantiations carry it)
                if (BP == 1 && rs.tagged && rs.mode == MODE_MAILBOX) {
                    // warp 0 polls the chunks, x arrives with the doorbell
                    if (warp == 0) {
                        uint32_t cmd = 0, sq = 0, reason = EXIT_NONE;
                        if (kTagged && tag + (uint32_t)L > kGvTagLimit) {
                            cmd = 1u;
                            reason = EXIT_TAGS;
                        } else if constexpr (BP == 1) {
                            cmd = gv_poll_tagged(rs, last, rs.relay_x, sp.dims[0], &sq, &reason);
                        }
                        if (lane == 0) {
                            if (cmd)
                                st_relaxed_sys_u32(&rs.ctrl->exit_reason, reason);
                            s_req[0] = sq;
                            s_req[1] = cmd ? 0u : 1u;
                            s_req[2] = cmd;
                        }
                    }
                    __syncthreads();  // warp 0's relay stores before thread 0's release
                } else {
                    if (tid == 0) {
                        uint32_t cmd = 0, rows = 0, reason = EXIT_NONE;
                        if (kTagged && tag + (uint32_t)L > kGvTagLimit) {
                            cmd = 1u;
                            reason = EXIT_TAGS;
                        } else if (rs.mode == MODE_QUEUE) {
                            if ((int)n_req >= rs.q_n) {
                                cmd = 1u;
                                reason = EXIT_QUEUE_DONE;
                            } else {
                                seq = n_req + 1u;
                                rows = (uint32_t)rs.q_rows;
                            }
                        } else {
                            // the TickBuffer doorbell: seq_in alone (acquire); stop and the idle
                            // bound are checked every 64 polls
                            const uint64_t t0 = globaltimer();
                            for (uint32_t it = 0;; ++it) {
                                const uint32_t sq = ld_acquire_sys(&rs.mb->seq_in);
                                if (sq != last && sq != 0u) {
                                    seq = sq;
                                    break;
                                }
                                if ((it & 63u) == 63u) {
                                    if (ld_relaxed_sys(&rs.mb->stop)) {
                                        cmd = 1u;
                                        reason = EXIT_STOP;
                                        break;
                                    }
                                    if (globaltimer() - t0 > rs.idle_ns) {
                                        cmd = 1u;
                                        reason = EXIT_IDLE;
                                        break;
                                    }
                                }
                            }
                        }
                        if (cmd)
                            st_relaxed_sys_u32(&rs.ctrl->exit_reason, reason);
                        s_req[0] = seq;
                        s_req[1] = rows;
                        s_req[2] = cmd;
                    }
                    __syncthreads();
                    if (!s_req[2]) {
                        // x rows into the relay buffer (16-byte pieces; in_dim is a multiple of 4)
                        const int q = sp.dims[0] / 4;
                        float4 *dst = reinterpret_cast<float4 *>(rs.relay_x);
                        if (rs.mode == MODE_QUEUE) {
                            const int n4 = (int)s_req[1] * q;
                            const float4 *src =
                                reinterpret_cast<const float4 *>(rs.q_x + (size_t)n_req * rs.q_rows * sp.dims[0]);
                            for (int i = tid; i < n4; i += kGvThreads)
                                dst[i] = __ldg(src + i);
                        } else {
                            // the header's row count and the first rows of x in ONE PCIe round trip:
                            // up to 4 rows (4 loads a thread) are read before the count is known,
                            // rows past it are dropped; rows past those 4 take a second trip
                            constexpr int kSpec = 4;
                            const int spec = min(min(rs.max_rows, kGvTagRows) * q, kSpec * kGvThreads) / q * q;
                            float4 v[kSpec];
    #pragma unroll
                            for (int u = 0; u < kSpec; ++u)
                                if (tid + u * kGvThreads < spec)
                                    v[u] = ld_relaxed_sys_v4(rs.mb_x + (size_t)(tid + u * kGvThreads) * 4);
                            if (tid == 0) {
                                // clamped to the mailbox's rows: x and y are read and written there
                                const uint32_t hr = ld_relaxed_sys(&rs.mb->n_rows);
                                s_req[1] = hr == 0u ? 1u : (hr > (uint32_t)rs.max_rows ? (uint32_t)rs.max_rows : hr);
                            }
                            __syncthreads();
                            const int n4 = (int)s_req[1] * q;
    #pragma unroll
                            for (int u = 0; u < kSpec; ++u)
                                if (tid + u * kGvThreads < min(spec, n4))
                                    dst[tid + u * kGvThreads] = v[u];
                            // the other rows: 4 loads a thread in flight before any store (a load
                            // of mapped host memory is one PCIe round trip; one after another they
                            // cost a trip each)
                            constexpr int kRest = 4;
                            for (int i0 = spec + tid; i0 < n4; i0 += kRest * kGvThreads) {
                                float4 w[kRest];
    #pragma unroll
                                for (int u = 0; u < kRest; ++u)
                                    if (i0 + u * kGvThreads < n4)
                                        w[u] = ld_relaxed_sys_v4(rs.mb_x + (size_t)(i0 + u * kGvThreads) * 4);
    #pragma unroll
                                for (int u = 0; u < kRest; ++u)
                                    if (i0 + u * kGvThreads < n4)
                                        dst[i0 + u * kGvThreads] = w[u];
                            }
                        }
                        __syncthreads();  // every thread's relay stores before thread 0's release
                    }
                }
                if (tid == 0)
                    gv_st_release_u64(rs.req, (unsigned long long)s_req[0] | ((unsigned long long)s_req[1] << 32) |
                                                  ((unsigned long long)s_req[2] << 48));
            } else {
                if (tid == 0) {
                    // the next request word (bounded: CTA 0 leaves at the idle bound and says so)
                    unsigned long long w = gv_ld_acquire_u64(rs.req);
                    const uint64_t t0 = globaltimer();
                    while (w == last_word) {
                        if (globaltimer() - t0 > rs.idle_ns + rs.peer_margin_ns) {
                            w = 1ull << 48;
                            break;
                        }
                        w = gv_ld_acquire_u64(rs.req);
                    }
                    last_word = w;
                    s_req[0] = (uint32_t)w;
                    s_req[1] = (uint32_t)(w >> 32) & 0xffffu;
                    s_req[2] = (uint32_t)(w >> 48);
                }
                __syncthreads();
            }
            if (s_req[2])
                break;
            seq = s_req[0];
            nr = (int)s_req[1];
            __syncthreads();  // every thread has read s_req before thread 0 writes the request's fields
            if (tid == 0) {
                sp.n_rows = nr;
                sp.x = rs.relay_x;
                sp.y = rs.gather_y;
                sp.tag_base = tag;
                sp.epoch = n_req + 1u;
            }
            __syncthreads();
        }

        for (int l = 0; l < L; ++l) {
            int r0;
            const int R = slice(l, r0);
            if (R == 0)
                continue;  // no rows here: this CTA neither reads layer l's input nor writes its output
            const int K = sp.dims[l], N = sp.dims[l + 1];
            unsigned long long *tr = sp.trace[l] ? sp.trace[l] + (size_t)c * 16 : nullptr;

            // ---- input: layer 0 from the caller, later layers from the previous layer ----
            // A thread issues up to kGvUnroll 16-byte loads before it stores any of them, so
            // the L2 round trips overlap; every CTA starts at its own rotation of the rows.
            bool ok = true;
            if (l > 0 && !kTagged) {
                if (tid == 0) {
                    const unsigned producers = (unsigned)min(G, K);  // layer l-1 has K rows over G CTAs
                    if (!gv_wait_count(sp.cnt + (size_t)(l - 1) * kGvCntStride, sp.epoch * producers, sp.wait_ns)) {
                        s_fail = 1u;
                        atomicOr(sp.status, 1u | ((16u + (unsigned)l) << 8));
                    }
                }
                __syncthreads();
                if (s_fail)
                    break;
            }
            {
                // groups of 16 bytes: 4 fp32 inputs (layer 0), 4 tagged words, or 8 bf16 values
                const int per = (l == 0 || kTagged) ? 4 : 8;
                const int q = K / per, total = nr * q, rot = (int)((unsigned)c * (unsigned)total / (unsigned)G);
                const uint4 *src = l == 0 ? reinterpret_cast<const uint4 *>(sp.x)
                                   : kTagged ? reinterpret_cast<const uint4 *>(sp.hand[(l - 1) & 1])
                                             : reinterpret_cast<const uint4 *>(sp.act[(l - 1) & 1]);
                const uint32_t tag = sp.tag_base + (uint32_t)(l - 1);
                for (int i0 = tid; i0 < total && ok; i0 += kGvThreads * kGvUnroll) {
                    uint4 v[kGvUnroll];
                    int gi[kGvUnroll];
                    uint32_t pending = 0u;
    #pragma unroll
                    for (int u = 0; u < kGvUnroll; ++u) {
                        int i = i0 + u * kGvThreads + rot;
                        gi[u] = i - (i >= total ? total : 0);
                        if (i0 + u * kGvThreads < total) {
                            v[u] = (l > 0 && kTagged) ? gv_ld_words(src + gi[u]) : __ldcg(src + gi[u]);
                            pending |= 1u << u;
                        }
                    }
                    uint64_t t0 = 0;
                    for (;;) {
    #pragma unroll
                        for (int u = 0; u < kGvUnroll; ++u) {
                            if (!((pending >> u) & 1u))
                                continue;
                            const int b = gi[u] / q, e = per * (gi[u] - b * q);
                            float *d = xs + (size_t)b * XS + e;
                            if (l == 0) {
                                *reinterpret_cast<float4 *>(d) =
                                    make_float4(gv_round_bf16(__uint_as_float(v[u].x)), gv_round_bf16(__uint_as_float(v[u].y)),
                                                gv_round_bf16(__uint_as_float(v[u].z)), gv_round_bf16(__uint_as_float(v[u].w)));
                            } else if (kTagged) {
                                if (!gv_tags_are(v[u], tag))
                                    continue;
                                *reinterpret_cast<float4 *>(d) = make_float4(
                                    __uint_as_float(v[u].x & 0xffff0000u), __uint_as_float(v[u].y & 0xffff0000u),
                                    __uint_as_float(v[u].z & 0xffff0000u), __uint_as_float(v[u].w & 0xffff0000u));
                            } else {
                                *reinterpret_cast<float4 *>(d) = make_float4(gv_bf16_lo(v[u].x), gv_bf16_hi(v[u].x),
                                                                             gv_bf16_lo(v[u].y), gv_bf16_hi(v[u].y));
                                *reinterpret_cast<float4 *>(d + 4) = make_float4(gv_bf16_lo(v[u].z), gv_bf16_hi(v[u].z),
                                                                                 gv_bf16_lo(v[u].w), gv_bf16_hi(v[u].w));
                            }
                            pending &= ~(1u << u);
                        }
                        if (!pending)
                            break;
                        const uint64_t now = globaltimer();  // only tagged words can still be pending
                        if (!t0)
                            t0 = now;
                        else if (now - t0 > sp.wait_ns) {
                            ok = false;
                            break;
                        }
    #pragma unroll
                        for (int u = 0; u < kGvUnroll; ++u)
                            if ((pending >> u) & 1u)
                                v[u] = gv_ld_words(src + gi[u]);
                    }
                }
            }
            if (tid == 0)
                gv_stamp(tr, kGvTraceInput);
            // ---- the image copies: A (biases + layer 0) first, B (later layers) from layer 1 ----
            if (ok && !a_ready && !gv_wait_bar(bar_a, sp.wait_ns))
                ok = false;
            if (ok && l > 0 && !b_ready && !gv_wait_bar(bar_b, sp.wait_ns))
                ok = false;
            a_ready = true;
            b_ready = b_ready || l > 0;
            if (!ok) {
                s_fail = 1u;
                atomicOr(sp.status, 1u | ((16u + (unsigned)l) << 8));
            }
            __syncthreads();
            if (s_fail)
                break;
            if (tid == 0)
                gv_stamp(tr, kGvTraceReady);

            const uint8_t *ws = smem + sp.woff[l];
            const float *sb = sbias + sp.boff[l];
            const int rmax = sp.rmax[l], act = sp.acts[l];
            const int nch = K / CH;
            for (int rg = 0; rg < R; rg += kGvRowGroup) {
                float acc[kGvRowGroup][BPL];
    #pragma unroll
                for (int r = 0; r < kGvRowGroup; ++r)
    #pragma unroll
                    for (int i = 0; i < BPL; ++i)
                        acc[r][i] = 0.0f;
                for (int cc = warp * KL + kl; cc < nch; cc += kGvWarps * KL) {
                    const int k = cc * CH;
                    float xv[BPL][CH];
    #pragma unroll
                    for (int i = 0; i < BPL; ++i) {
                        const float4 *xp = reinterpret_cast<const float4 *>(xs + (size_t)(bg + BG * i) * XS + k);
    #pragma unroll
                        for (int j = 0; j < CH / 4; ++j) {
                            const float4 v = xp[j];
                            xv[i][4 * j] = v.x;
                            xv[i][4 * j + 1] = v.y;
                            xv[i][4 * j + 2] = v.z;
                            xv[i][4 * j + 3] = v.w;
                        }
                    }
                    // every row's chunk first, then the products j-outer: consecutive FMAs
                    // are independent (a lane keeps kGvRowGroup x BPL sums)
                    uint4 wq[kGvRowGroup];
    #pragma unroll
                    for (int r = 0; r < kGvRowGroup; ++r)
                        wq[r] = rg + r < R ? *reinterpret_cast<const uint4 *>(ws + ((size_t)(rg + r) * K + k) * ES)
                                           : make_uint4(0u, 0u, 0u, 0u);
    #pragma unroll
                    for (int h = 0; h < CH / 8; ++h) {  // 8 inputs at a time (int8 chunks hold 16)
                        float wf[kGvRowGroup][8];
    #pragma unroll
                        for (int r = 0; r < kGvRowGroup; ++r) {
                            float w16[CH];
                            gv_weights<WINT8>(wq[r], w16);
    #pragma unroll
                            for (int j = 0; j < 8; ++j)
                                wf[r][j] = w16[8 * h + j];
                        }
    #pragma unroll
                        for (int j = 0; j < 8; ++j)
    #pragma unroll
                            for (int r = 0; r < kGvRowGroup; ++r)
    #pragma unroll
                                for (int i = 0; i < BPL; ++i)
                                    acc[r][i] = fmaf(wf[r][j], xv[i][8 * h + j], acc[r][i]);
                    }
                }
                // the K lanes of a batch group hold partial sums of the same outputs
    #pragma unroll
                for (int r = 0; r < kGvRowGroup; ++r)
    #pragma unroll
                    for (int i = 0; i < BPL; ++i)
    #pragma unroll
                        for (int off = 16; off >= BG; off >>= 1)
                            acc[r][i] += __shfl_xor_sync(0xffffffffu, acc[r][i], off);
                if (tid == 0 && rg == 0)
                    gv_stamp(tr, kGvTraceMath);
                if (kl == 0) {
    #pragma unroll
                    for (int r = 0; r < kGvRowGroup; ++r)
    #pragma unroll
                        for (int i = 0; i < BPL; ++i)
                            part[(warp * kGvRowGroup + r) * kGvMaxRows + bg + BG * i] = acc[r][i];
                }
                __syncthreads();
                if (tid == 0 && rg == 0)
                    gv_stamp(tr, kGvTraceReduced);
                for (int t = tid; t < kGvRowGroup * BP; t += kGvThreads) {
                    const int r = t / BP, b = t - r * BP;
                    if (rg + r < R && b < nr) {
                        float s = 0.0f;
    #pragma unroll
                        for (int w = 0; w < kGvWarps; ++w)
                            s += part[(w * kGvRowGroup + r) * kGvMaxRows + b];
                        float v = WINT8 ? __fadd_rn(__fmul_rn(sb[rmax + rg + r], s), sb[rg + r]) : __fadd_rn(s, sb[rg + r]);
                        v = gv_act(v, act);
                        const size_t o = (size_t)b * N + r0 + rg + r;
                        if (l + 1 == L)
                            sp.y[o] = v;
                        else if (kTagged)
                            gv_st_word(sp.hand[l & 1] + o,
                                       ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v)) << 16) |
                                           (sp.tag_base + (uint32_t)l));
                        else
                            sp.act[l & 1][o] = __float2bfloat16_rn(v);
                    }
                }
                if (tid == 0 && rg == 0)
                    gv_stamp(tr, kGvTraceStored);
                __syncthreads();
            }
            // counted hand-off: the barrier above orders every thread's outputs before
            // thread 0's release (resident mode: the last layer's outputs too, for CTA 0)
            if (tid == 0 && ((!kTagged && l + 1 < L) || (RES && l + 1 == L)))
                red_release_gpu_add(sp.cnt + (size_t)l * kGvCntStride, 1u);
            if (tid == 0)
                gv_stamp(tr, kGvTracePublished);
        }

        if constexpr (!RES) {
            break;
        } else {
            if (s_fail)
                break;
            // ---------------- CTA 0: the outputs into the mailbox (or the queue), then seq_out ----------------
            const GemvResident &rs = sp.res;
            if (c == 0) {
                const int N = sp.dims[L];
                if (tid == 0) {
                    const unsigned producers = (unsigned)min(G, N);
                    if (!gv_wait_count(sp.cnt + (size_t)(L - 1) * kGvCntStride, sp.epoch * producers, sp.wait_ns)) {
                        s_fail = 1u;
                        atomicOr(sp.status, 1u | ((16u + (unsigned)L) << 8));
                    }
                }
                __syncthreads();
                if (s_fail)
                    break;
                const int n4 = nr * N / 4;  // out_dim is a multiple of 4
                const float4 *src = reinterpret_cast<const float4 *>(rs.gather_y);
                if (rs.mode == MODE_QUEUE) {
                    float4 *dst = reinterpret_cast<float4 *>(rs.q_y + (size_t)n_req * rs.q_rows * N);
                    for (int i = tid; i < n4; i += kGvThreads)
                        dst[i] = __ldcg(src + i);
                } else if (BP == 1 && rs.tagged) {
                    // tagged y chunks {y0, y1, y2, seq}: the host waits on the tags, so no release
                    for (int t = tid; t < (N + 2) / 3; t += kGvThreads) {
                        float v[3];
#pragma unroll
                        for (int e = 0; e < 3; ++e)
                            v[e] = 3 * t + e < N ? __ldcg(rs.gather_y + 3 * t + e) : 0.0f;
                        st_relaxed_sys_v4(rs.mb_y + (size_t)t * 4, make_float4(v[0], v[1], v[2], __uint_as_float(seq)));
                    }
                } else {
                    // every L2 load before the first store to the mailbox (the stores are
                    // ordered asm, so a load after one would wait for it)
                    constexpr int kY = 2;
                    for (int i0 = tid; i0 < n4; i0 += kY * kGvThreads) {
                        float4 v[kY];
#pragma unroll
                        for (int u = 0; u < kY; ++u)
                            if (i0 + u * kGvThreads < n4)
                                v[u] = __ldcg(src + i0 + u * kGvThreads);
#pragma unroll
                        for (int u = 0; u < kY; ++u)
                            if (i0 + u * kGvThreads < n4)
                                st_relaxed_sys_v4(rs.mb_y + (size_t)(i0 + u * kGvThreads) * 4, v[u]);
                    }
                }
                __syncthreads();  // every thread's y stores before thread 0's release
                if (tid == 0) {
                    if (rs.mode == MODE_QUEUE) {
                        if (rs.q_stamp)
                            rs.q_stamp[n_req] = globaltimer();
                    } else if (BP == 1 && rs.tagged) {
                        st_relaxed_sys_u32(&rs.mb->seq_out, seq);  // bookkeeping for a relaunch only
                    } else {
                        st_release_sys_u32(&rs.mb->seq_out, seq);
                    }
                }
            }
            last = seq;
            ++served;
            rows_served += (uint32_t)nr;
            if (kTagged)
                tag += (uint32_t)L;
        }
    }

    if constexpr (RES) {
        if (c == 0 && tid == 0) {
            // a CTA 0 that left on a failed wait still tells the others to leave
            if (s_fail)
                gv_st_release_u64(sp.res.req, (unsigned long long)last | (1ull << 48));
        }
        if (s_fail && tid == 0) {
            st_relaxed_sys_u32(&sp.res.ctrl->err_where, 0x200u + (unsigned)c);
            st_relaxed_sys_u32(&sp.res.ctrl->status, (uint32_t)LL_ERR_DEVICE_FAULT);
        }
        if (c == 0 && tid == 0) {
            st_relaxed_sys_u32(&sp.res.ctrl->passes, served);
            st_relaxed_sys_u32(&sp.res.ctrl->rows, rows_served);
            st_release_sys_u32(&sp.res.ctrl->state, ST_EXITED);
        }
    }

    // A CTA that gave up may still have copies in flight: let them land first.
    if (s_fail && tid == 0) {
        gv_wait_bar(bar_a, kGvDrainNs);
        if (has_b)
            gv_wait_bar(bar_b, kGvDrainNs);
    }
}

}  // namespace llk
