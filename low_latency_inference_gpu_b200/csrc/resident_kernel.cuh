// The resident (persistent) MLP kernel for sm_100a.
//
// One launch serves requests until told to stop.  The grid is n_stages
// thread-block clusters of C CTAs (one CTA per SM).  Each CTA holds a slice of
// its stage's layers in shared memory for the whole launch (the reference keeps
// weights "resident" in registers / SMEM / global scratch per thread,
// include/ll/weights_storage.cuh:7-240; here the slice is one bulk-copied SMEM
// image).  Per request:
//   stage 0  : rank 0 alone polls the mailbox header (host-mapped TickBuffer,
//              src/bench_persistent_mbyv_mlp.cu:229-281) with one 16-byte acquire
//              load, reads x once and pushes {seq, n_rows, x} into its peers'
//              shared memory (st.async + mbarrier tx), so PCIe sees one poller;
//   layers   : row-split GEMV from SMEM, outputs pushed to peer CTAs with
//              st.async + mbarrier complete_tx (DSMEM) instead of the
//              reference's global-atomic layer barriers (:308-377);
//   boundary : between clusters, rows go through L2 with a release counter;
//   output   : last layer as K-split partials gathered at rank 0, which writes
//              y and release-stores seq_out (:365-370).
// Every wait is bounded by %globaltimer and reports an error status instead of
// spinning forever (the reference spins unboundedly, :232-247).
#pragma once
#include <cuda_bf16.h>

#include "engine_types.h"
#include "ptx.cuh"

namespace llk {

constexpr uint32_t kCmdExit = 0u;  // 0 is never a live sequence number

struct Shared {
    uint32_t hdr[4];  // request header pushed by the dispatcher: seq, n_rows (16-byte aligned: first member)
    uint64_t bar[7];  // 0 image load, 1 buffer A, 2 buffer B, 3 gather G, 4 diagnostic, 5 header, 6 x rows
    uint32_t cmd;
    uint32_t nrows;
    uint32_t fail;
    uint32_t abort;
    uint32_t hstop;  // stop flag seen in the header that came with the current doorbell
    uint32_t xtag;   // later pipeline stages: the request number the hand-off words carry
};

__device__ __forceinline__ float act_apply(float v, int act)
{
    if (act == LL_ACT_RELU)
        return v > 0.0f ? v : 0.0f;
    if (act == LL_ACT_GELU)
        return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
    return v;
}

__device__ __forceinline__ float round_bf16(float v)
{
    return __bfloat162float(__float2bfloat16_rn(v));
}

// Load one 16-byte weight unit from shared memory as floats.
template <int WT>
__device__ __forceinline__ void load_unit(const uint8_t *p, float *w)
{
    if constexpr (WT == LL_W_F32) {
        float4 v = *reinterpret_cast<const float4 *>(p);
        w[0] = v.x;
        w[1] = v.y;
        w[2] = v.z;
        w[3] = v.w;
    } else if constexpr (WT == LL_W_BF16) {
        uint4 u = *reinterpret_cast<const uint4 *>(p);
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[2 * i] = __uint_as_float(q[i] << 16);
            w[2 * i + 1] = __uint_as_float(q[i] & 0xffff0000u);
        }
    } else {
        uint4 u = *reinterpret_cast<const uint4 *>(p);
        const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                w[4 * i + j] = static_cast<float>(static_cast<int8_t>((q[i] >> (8 * j)) & 0xffu));
        }
    }
}

template <int WT>
struct UnitInfo {
    static constexpr int elems = WT == LL_W_F32 ? 4 : (WT == LL_W_BF16 ? 8 : 16);
    static constexpr int wbytes = WT == LL_W_F32 ? 4 : (WT == LL_W_BF16 ? 2 : 1);
};

// dot(W[r, 0:K], in[b, 0:K]) for r < R, b < B, computed by `lpr` lanes per row
// with a butterfly reduction; epi(b, r, value) runs on the row's first lane.
// Batch-1 products (BB = 1) take two rows per lane where the warp has a second row
// (r and r + the rows one pass of the CTA covers): each x piece read from shared memory
// then serves two rows, which cuts the layer's shared-memory traffic by a quarter, and
// the two FMA chains overlap.  Each row's sum is formed exactly as with one row per lane
// (same K slices per lane, same FMA order, same butterfly), so results do not change.
template <int WT, int BB, class Epi>
__device__ __forceinline__ void rows_dot(const uint8_t *W, int R, int K, const float *in, int in_ld, int B,
                                         int lpr_log2, Epi &&epi)
{
    constexpr int E = UnitInfo<WT>::elems;
    const int U = K / E;
    const int lpr = 1 << lpr_log2;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int sub = lane & (lpr - 1);
    const int rpw = 32 >> lpr_log2;  // rows per warp pass
    const int step = (kThreads / 32) * rpw;  // rows one pass of the CTA covers
    const size_t row_bytes = (size_t)K * UnitInfo<WT>::wbytes;
    for (int b0 = 0; b0 < B; b0 += BB) {
        for (int rb = warp * rpw; rb < R;) {
            const int r = rb + (lane >> lpr_log2);
            const bool valid = r < R;
            const int rr = valid ? r : R - 1;
            const uint8_t *wrow = W + (size_t)rr * row_bytes;
            if (BB == 1 && rb + step < R) {
                const int r2 = r + step;
                const bool valid2 = r2 < R;
                const uint8_t *wrow2 = W + (size_t)(valid2 ? r2 : R - 1) * row_bytes;
                float acc = 0.0f, acc2 = 0.0f;
                for (int u = sub; u < U; u += lpr) {
                    float w[E], w2[E];
                    load_unit<WT>(wrow + (size_t)u * 16, w);
                    load_unit<WT>(wrow2 + (size_t)u * 16, w2);
                    const float *xr = in + (size_t)b0 * in_ld + u * E;
#pragma unroll
                    for (int e = 0; e < E; e += 4) {
                        const float4 x4 = *reinterpret_cast<const float4 *>(xr + e);
                        acc = fmaf(w[e], x4.x, acc);
                        acc = fmaf(w[e + 1], x4.y, acc);
                        acc = fmaf(w[e + 2], x4.z, acc);
                        acc = fmaf(w[e + 3], x4.w, acc);
                        acc2 = fmaf(w2[e], x4.x, acc2);
                        acc2 = fmaf(w2[e + 1], x4.y, acc2);
                        acc2 = fmaf(w2[e + 2], x4.z, acc2);
                        acc2 = fmaf(w2[e + 3], x4.w, acc2);
                    }
                }
                for (int off = lpr >> 1; off > 0; off >>= 1) {
                    acc += __shfl_xor_sync(0xffffffffu, acc, off);
                    acc2 += __shfl_xor_sync(0xffffffffu, acc2, off);
                }
                if (sub == 0) {
                    if (valid)
                        epi(b0, r, acc);
                    if (valid2)
                        epi(b0, r2, acc2);
                }
                rb += 2 * step;
                continue;
            }
            float acc[BB];
#pragma unroll
            for (int bb = 0; bb < BB; ++bb)
                acc[bb] = 0.0f;
            for (int u = sub; u < U; u += lpr) {
                float w[E];
                load_unit<WT>(wrow + (size_t)u * 16, w);
#pragma unroll
                for (int bb = 0; bb < BB; ++bb) {
                    const float *xr = in + (size_t)(b0 + bb) * in_ld + u * E;
#pragma unroll
                    for (int e = 0; e < E; e += 4) {
                        const float4 x4 = *reinterpret_cast<const float4 *>(xr + e);
                        acc[bb] = fmaf(w[e], x4.x, acc[bb]);
                        acc[bb] = fmaf(w[e + 1], x4.y, acc[bb]);
                        acc[bb] = fmaf(w[e + 2], x4.z, acc[bb]);
                        acc[bb] = fmaf(w[e + 3], x4.w, acc[bb]);
                    }
                }
            }
            for (int off = lpr >> 1; off > 0; off >>= 1) {
#pragma unroll
                for (int bb = 0; bb < BB; ++bb)
                    acc[bb] += __shfl_xor_sync(0xffffffffu, acc[bb], off);
            }
            if (valid && sub == 0) {
#pragma unroll
                for (int bb = 0; bb < BB; ++bb)
                    if (b0 + bb < B)
                        epi(b0 + bb, r, acc[bb]);
            }
            rb += step;
        }
    }
}

// One layer's products.  The kernel is instantiated per weight type and for batch-1 nets
// without the 4-row path: every layer of a net has the same weight type, and the code a
// request runs through stays small enough for the instruction cache.
template <int WT, bool BATCHED, class Epi>
__device__ __forceinline__ void layer_dot(const uint8_t *W, int R, int K, const float *in, int in_ld, int B,
                                          int lpr_log2, Epi &&epi)
{
    if constexpr (BATCHED) {
        if (B > 1) {
            rows_dot<WT, 4>(W, R, K, in, in_ld, B, lpr_log2, epi);
            return;
        }
    }
    rows_dot<WT, 1>(W, R, K, in, in_ld, B, lpr_log2, epi);
}

struct KernelCtx {
    const Params *p;
    Shared *sh;
    uint8_t *smem;
    uint32_t rank;
    int stage;
};

// Record a device error (status is sticky per launch).
__device__ __forceinline__ void report_error(const KernelCtx &k, uint32_t status, uint32_t where)
{
    st_relaxed_sys_u32(&k.p->ctrl->err_where, where);
    st_relaxed_sys_u32(&k.p->ctrl->status, status);
}

// Tell every CTA of this cluster, and the other clusters, to leave the loop.
__device__ __forceinline__ void broadcast_abort(const KernelCtx &k)
{
    const uint32_t a = smem_u32(&k.sh->abort);
    for (int r = 0; r < k.p->C; ++r)
        st_cluster_u32(mapa(a, (uint32_t)r), 1u);
    atomicExch(k.p->abort_flag, 1u);
}

__device__ __forceinline__ bool global_abort(const KernelCtx &k)
{
    return ld_relaxed_gpu_u32(k.p->abort_flag) != 0;
}

__device__ __forceinline__ void trace(const KernelCtx &k, uint32_t req, int slot)
{
    if (k.p->trace && req < (uint32_t)k.p->trace_n) {
        k.p->trace[(size_t)req * kTraceSlots + slot] = globaltimer();
        k.p->trace[(size_t)req * kTraceSlots + 16 + slot] = clock64();
    }
}

// All threads wait for an mbarrier phase; thread 0 alone watches the clock.
// Returns true when the phase completed; false on abort (quiet) or timeout
// (reported with `where`).  The verdict is the same for every thread.
__device__ __forceinline__ bool cta_wait_bar(const KernelCtx &k, uint32_t bar, uint32_t parity, uint32_t where,
                                             uint64_t bound_ns)
{
    volatile uint32_t *abort = &k.sh->abort;
    volatile uint32_t *fail = &k.sh->fail;
    const bool timer = threadIdx.x == 0;
    const uint64_t deadline = timer ? globaltimer() + bound_ns : 0;
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(bar, parity))
            break;
        if (*abort) {
            atomicOr(&k.sh->fail, 1u);
            break;
        }
        if (timer) {
            if ((it & 15u) == 15u && globaltimer() > deadline) {
                atomicOr(&k.sh->fail, 2u);
                break;
            }
        } else if (*fail) {
            break;
        }
    }
    __syncthreads();
    const uint32_t f = *fail;
    if (f != 0 && threadIdx.x == 0 && (f & 2u)) {
        report_error(k, LL_ERR_DEVICE_FAULT, where);
        broadcast_abort(k);
    }
    return f == 0;
}

// Thread 0 of the dispatcher (rank 0 of stage 0): wait for a new request.
// The poll reads seq_in alone: a wider load would cover seq_out, which this
// thread has just release-stored, and would wait behind that PCIe write.
// `stop` is checked on the idle cadence here; for batched nets a stop that
// arrives with a doorbell (src/bench_persistent_mbyv_mlp.cu:554-557) is also
// caught by read_header() before the request's rows are read.
// Returns the sequence number, or kCmdExit (stop, idle bound, abort).
__device__ uint32_t poll_mailbox(const KernelCtx &k, uint32_t last)
{
    const Params &p = *k.p;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        const uint32_t s = ld_acquire_sys(&p.mb->seq_in);
        if (s != last && s != 0)
            return s;
        if ((it & 63u) == 63u) {
            if (*reinterpret_cast<volatile uint32_t *>(&k.sh->abort) || global_abort(k))
                return kCmdExit;
            if (ld_relaxed_sys(&p.mb->stop)) {  // stop without a doorbell (src/bench_persistent_mlp.cu:409)
                st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_STOP);
                return kCmdExit;
            }
            if (globaltimer() - t0 > p.idle_ns) {
                st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_IDLE);
                return kCmdExit;
            }
        }
    }
}

// Tagged mailbox (format 1), warp 0 of the dispatcher: every lane loads up to
// kTagChunksPerLane 16-byte x chunks {v0, v1, v2, tag} per poll; the request is
// taken when every chunk carries exactly the next sequence number, and its floats
// go straight into X -- detection and the x read are one PCIe round trip.  (A
// slot's previous lap, or an older snapshot, holds an older number.)
constexpr int kTagChunksPerLane = 4;

__device__ __forceinline__ uint32_t next_seq_dev(uint32_t s)
{
    const uint32_t n = s + 1u;
    return (n == 0u || n == LL_STOP_SEQ) ? 1u : n;
}

// Slot of request n of this launch in the tagged ring (x and y bases).
__device__ __forceinline__ uint32_t ring_slot(const Params &p, uint32_t n)
{
    return p.ring_slots > 1 ? (p.ring_base + n) % (uint32_t)p.ring_slots : 0u;
}

// Forwarding of the raw tagged chunks to other CTAs of a cluster (register-resident and
// pipelined ring kernels): the polling lanes push the chunks they hold straight from
// registers, so the receivers' copy of x leaves the moment the tags match.  Chunk ch of row r
// goes to the shared address chunks + 16 * (r * nxc + ch) of ranks first .. first+peers-1 and
// completes their barrier bar_first (row 0) or bar_rest (rows 1..); lane 0 adds a 16-byte
// header {seq, rows} at hdr (on bar_first).  Every address is the same offset in each CTA
// (mapa).
// Where the chunks of a multi-row read go: chunk `ch` of row r lands at chunks + 16 (r nxc + ch)
// in CTAs first .. first + peers - 1 (the same shared-memory offset in each); row 0 and the
// header {seq, rows} complete bar_first there, rows 1.. bar_rest (row0_rest != 0: the header
// alone completes bar_first, every row bar_rest).
struct ChunkFwd {
    uint32_t chunks, hdr, bar_first, bar_rest;
    int first, peers;
    int row0_rest;
};

__device__ __forceinline__ void fwd_chunk(const ChunkFwd &f, int row, int ch, int nxc, uint4 c)
{
    const float4 v = make_float4(__uint_as_float(c.x), __uint_as_float(c.y), __uint_as_float(c.z), __uint_as_float(c.w));
    const uint32_t a = f.chunks + 16u * (uint32_t)(row * nxc + ch);
    const uint32_t b = (row == 0 && !f.row0_rest) ? f.bar_first : f.bar_rest;
    for (int d = f.first; d < f.first + f.peers; ++d)
        st_async_v4(mapa(a, (uint32_t)d), v, mapa(b, (uint32_t)d));
}

__device__ __forceinline__ void fwd_header(const ChunkFwd &f, uint32_t seq, uint32_t rows)
{
    for (int d = f.first; d < f.first + f.peers; ++d)
        st_async_v4(mapa(f.hdr, (uint32_t)d), make_float4(__uint_as_float(seq), __uint_as_float(rows), 0.f, 0.f),
                    mapa(f.bar_first, (uint32_t)d));
}

// Warp 0 waits for the next request in a tagged ring slot (the single-slot poll) and
// unpacks x into X (unless X is null).
// `posted` (optional, micro-batched rings): lane 31 also reads the host's seq_in word (the
// last sequence number it posted; bookkeeping in the tagged format) in the same round trip,
// and *posted gets the value seen with the request, so the caller knows whether more
// requests are waiting behind it.
// `fwd` (optional): forward the request's chunks to the cluster's other CTAs (ChunkFwd).
__device__ uint32_t poll_tagged(const KernelCtx &k, uint32_t last, float *X, uint32_t slot, uint32_t *posted = nullptr,
                                const ChunkFwd *fwd = nullptr)
{
    const Params &p = *k.p;
    const int lane = threadIdx.x & 31;
    const int nxc = (p.in_dim + 2) / 3;
    const uint4 *chunks = reinterpret_cast<const uint4 *>(p.mb_x + (size_t)slot * p.ring_xstride_f);
    const uint32_t want = next_seq_dev(last);
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
        uint4 c[kTagChunksPerLane];
#pragma unroll
        for (int j = 0; j < kTagChunksPerLane; ++j)
            if (lane + 32 * j < nxc)
                c[j] = ld_relaxed_sys_v4_u32(reinterpret_cast<const unsigned *>(chunks + lane + 32 * j));
        uint32_t seen = 0;
        if (posted && lane == 31)
            seen = ld_relaxed_sys(&p.mb->seq_in);
        const uint32_t tag = __shfl_sync(0xffffffffu, c[0].w, 0);
        bool same = true;
#pragma unroll
        for (int j = 0; j < kTagChunksPerLane; ++j)
            if (lane + 32 * j < nxc && c[j].w != tag)
                same = false;
        if (__all_sync(0xffffffffu, same) && tag == want) {
            if (fwd) {
#pragma unroll
                for (int j = 0; j < kTagChunksPerLane; ++j)
                    if (lane + 32 * j < nxc)
                        fwd_chunk(*fwd, 0, lane + 32 * j, nxc, c[j]);
                if (lane == 0)
                    fwd_header(*fwd, tag, 1u);
            }
#pragma unroll
            for (int j = 0; j < kTagChunksPerLane; ++j) {
                const int ch = lane + 32 * j;
                if (X && ch < nxc) {
                    const float v[3] = {__uint_as_float(c[j].x), __uint_as_float(c[j].y), __uint_as_float(c[j].z)};
#pragma unroll
                    for (int e = 0; e < 3; ++e)
                        if (3 * ch + e < p.in_dim)
                            X[3 * ch + e] = p.act_bf16 ? round_bf16(v[e]) : v[e];
                }
            }
            if (posted)
                *posted = __shfl_sync(0xffffffffu, seen, 31);
            return tag;
        }
        if ((it & 63u) == 63u) {
            uint32_t verdict = 0;
            if (lane == 0) {
                if (*reinterpret_cast<volatile uint32_t *>(&k.sh->abort) || global_abort(k)) {
                    verdict = 1;
                } else if (ld_relaxed_sys(&p.mb->stop)) {
                    st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_STOP);
                    verdict = 1;
                } else if (globaltimer() - t0 > p.idle_ns) {
                    st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_IDLE);
                    verdict = 1;
                }
            }
            if (__shfl_sync(0xffffffffu, verdict, 0))
                return kCmdExit;
        }
    }
}

// The sequence number m requests after `last` (0 <= m < 2^31): m steps of next_seq_dev in closed
// form.  The sequence cycles through 1 .. LL_STOP_SEQ - 1 (period 2^32 - 2); 0 and LL_STOP_SEQ
// step to 1, like LL_STOP_SEQ - 1 does.
__host__ __device__ __forceinline__ uint32_t seq_after(uint32_t last, int m)
{
    constexpr uint64_t kPeriod = 0xFFFFFFFEull;
    if (m == 0)
        return last;
    const uint64_t pos = (last == 0u || last == LL_STOP_SEQ) ? kPeriod - 1u : (uint64_t)last - 1u;
    uint64_t q = pos + (uint64_t)m;
    if (q >= kPeriod)
        q -= kPeriod;
    return (uint32_t)q + 1u;
}

// Rows of a tagged ring one reading warp holds in registers (whole slots: 32 lanes x
// kTagChunksPerLane chunks), and the most warps a multi-slot read may use.
__host__ __device__ constexpr int tag_rows_per_warp(int nxc)
{
    return (32 * kTagChunksPerLane) / nxc;
}
constexpr int kTagReadWarpsMax = 16;

// Tagged request ring, micro-batched (warps 0..nw-1 of the dispatcher): ONE read of the
// ring slots of requests n .. n+maxb-1 of this launch (slot ring_slot(n + i)), taking
// every request that is complete and follows without a gap: slot n+i is taken when each
// of its chunks carries the (i+1)-th sequence number after `last`.  Warp w reads the
// rows [w * rpw, (w + 1) * rpw) (rpw whole slots, by default tag_rows_per_warp(nxc), its
// chunks in registers); the warps' loads are all in flight at once, so one PCIe round trip reads
// all maxb slots (maxb <= nw * rpw <= kTagReadWarpsMax * rpw and maxb <= 32, checked on
// the host).  Each warp's mask of incomplete rows goes through bad_words[w] (shared
// memory) and a named barrier (id 2, nw warps), so every warp sees the same first gap.
// Row i of x goes to X + i * in_dim (unless X is null) and its sequence number to seqs[i]
// (warp 0 writes them); in warp 0, *posted = the host's seq_in word (the last sequence number it
// posted), read by lane 31 in the same round trip.
// Returns the rows taken, the same in every reading warp (0 when request n is not
// complete yet; then the caller waits on its slot alone with poll_tagged, whose
// single-slot round trips are shorter: a read that spans several slots was measured
// ~2 us slower to detect a new request).
__device__ int take_tagged_rows(const KernelCtx &k, uint32_t last, float *X, uint32_t n, int maxb, uint32_t *seqs,
                                uint32_t *posted, uint32_t *bad_words, int nw, const ChunkFwd *fwd = nullptr,
                                int rpw = 0)
{
    const Params &p = *k.p;
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nxc = (p.in_dim + 2) / 3;
    if (rpw <= 0)
        rpw = tag_rows_per_warp(nxc);  // rows per reading warp (at most what its registers hold)
    const int r0 = warp * rpw;
    const int rows_here = min(rpw, maxb - r0);
    const int total = rows_here > 0 ? rows_here * nxc : 0;
    uint4 c[kTagChunksPerLane];
    int row[kTagChunksPerLane], ch[kTagChunksPerLane];
#pragma unroll
    for (int j = 0; j < kTagChunksPerLane; ++j) {
        const int q = lane + 32 * j;
        const int rl = q < total ? q / nxc : 0;
        row[j] = r0 + rl;
        ch[j] = q - rl * nxc;
        if (q < total)
            c[j] = ld_relaxed_sys_v4_u32(reinterpret_cast<const unsigned *>(
                p.mb_x + (size_t)ring_slot(p, n + (uint32_t)row[j]) * p.ring_xstride_f + 4 * ch[j]));
    }
    const uint32_t seen = (warp == 0 && lane == 31) ? ld_relaxed_sys(&p.mb->seq_in) : 0u;
    if (warp == 0)
        *posted = __shfl_sync(0xffffffffu, seen, 31);
    uint32_t bad = 0;
#pragma unroll
    for (int j = 0; j < kTagChunksPerLane; ++j)
        if (lane + 32 * j < total && c[j].w != seq_after(last, row[j] + 1))
            bad |= 1u << row[j];
    bad = __reduce_or_sync(0xffffffffu, bad);
    if (warp == 0 && lane == 0)
        trace(k, n, 11);  // this warp's loads have landed
    if (nw > 1) {
        if (lane == 0)
            bad_words[warp] = bad;
        asm volatile("bar.sync 2, %0;" ::"r"(32 * nw) : "memory");
        bad = 0;
        for (int w = 0; w < nw; ++w)
            bad |= bad_words[w];
    }
    const uint32_t stop_bit = maxb < 32 ? (1u << maxb) : 0u;
    const int nb = (bad | stop_bit) ? __ffs(bad | stop_bit) - 1 : 32;  // complete slots before the first gap
    if (fwd && nb > 0) {
#pragma unroll
        for (int j = 0; j < kTagChunksPerLane; ++j)
            if (lane + 32 * j < total && row[j] < nb)
                fwd_chunk(*fwd, row[j], ch[j], nxc, c[j]);
        if (warp == 0 && lane == 0)
            fwd_header(*fwd, seq_after(last, nb), (uint32_t)nb);
    }
#pragma unroll
    for (int j = 0; j < kTagChunksPerLane; ++j) {
        if (X && lane + 32 * j < total && row[j] < nb) {
            const float v[3] = {__uint_as_float(c[j].x), __uint_as_float(c[j].y), __uint_as_float(c[j].z)};
#pragma unroll
            for (int e = 0; e < 3; ++e)
                if (3 * ch[j] + e < p.in_dim)
                    X[row[j] * p.in_dim + 3 * ch[j] + e] = p.act_bf16 ? round_bf16(v[e]) : v[e];
        }
    }
    if (warp == 0 && lane < nb)
        seqs[lane] = seq_after(last, lane + 1);
    return nb;
}

// One thread reads the 16-byte header after the doorbell: stop flag and row count.
__device__ __forceinline__ void read_header(const KernelCtx &k)
{
    const Params &p = *k.p;
    const uint4 h = ld_relaxed_sys_v4_u32(reinterpret_cast<const unsigned *>(p.mb));
    const uint32_t n = h.w == 0 ? 1u : h.w;
    k.sh->nrows = n > (uint32_t)p.max_batch ? (uint32_t)p.max_batch : n;
    k.sh->hstop = h.z;
}

__device__ __forceinline__ float *buf_ptr(const KernelCtx &k, int id)
{
    return reinterpret_cast<float *>(k.smem + k.p->buf_off[id]);
}

__device__ __forceinline__ uint32_t buf_addr(const KernelCtx &k, int id)
{
    return smem_u32(k.smem + k.p->buf_off[id]);
}

// Copy the request rows from the mailbox into X (row stride in_ld), rounding to bf16 if asked.
__device__ __forceinline__ void stage_input_mailbox(const KernelCtx &k, int nrows)
{
    const Params &p = *k.p;
    float *X = buf_ptr(k, BUF_X);
    const int in = p.in_dim;
    if ((in & 3) == 0) {
        const int q = in >> 2;
        for (int t = threadIdx.x; t < nrows * q; t += kThreads) {
            const int b = t / q, c = t - b * q;
            float4 v = ld_relaxed_sys_v4(p.mb_x + (size_t)b * in + c * 4);
            if (p.act_bf16) {
                v.x = round_bf16(v.x);
                v.y = round_bf16(v.y);
                v.z = round_bf16(v.z);
                v.w = round_bf16(v.w);
            }
            *reinterpret_cast<float4 *>(X + (size_t)b * p.in_ld + c * 4) = v;
        }
    } else {
        for (int t = threadIdx.x; t < nrows * in; t += kThreads) {
            const int b = t / in, c = t - b * in;
            float v = ld_relaxed_sys_f32(p.mb_x + (size_t)b * in + c);
            X[(size_t)b * p.in_ld + c] = p.act_bf16 ? round_bf16(v) : v;
        }
    }
}

__device__ __forceinline__ void stage_input_device(const KernelCtx &k, const float *src, int nrows)
{
    const Params &p = *k.p;
    float *X = buf_ptr(k, BUF_X);
    const int in = p.in_dim;
    for (int t = threadIdx.x; t < nrows * in; t += kThreads) {
        const int b = t / in, c = t - b * in;
        float v = __ldg(src + (size_t)b * in + c);
        X[(size_t)b * p.in_ld + c] = p.act_bf16 ? round_bf16(v) : v;
    }
}

// Dispatcher: push {seq, n_rows} and the staged x rows into every peer CTA of the cluster.
__device__ __forceinline__ void push_request(const KernelCtx &k, uint32_t seq, int nrows, uint32_t bar_hdr,
                                             uint32_t bar_x)
{
    const Params &p = *k.p;
    const int in4 = p.in_ld >> 2;
    const int per = nrows * in4;
    const int total = (p.C - 1) * (1 + per);
    const float *X = buf_ptr(k, BUF_X);
    const uint32_t x_addr = buf_addr(k, BUF_X);
    const uint32_t h_addr = smem_u32(k.sh->hdr);
    for (int t = threadIdx.x; t < total; t += kThreads) {
        const uint32_t d = 1u + (uint32_t)(t / (1 + per));
        const int j = t % (1 + per);
        if (j == 0) {
            st_async_v4(mapa(h_addr, d), make_float4(__uint_as_float(seq), __uint_as_float((uint32_t)nrows), 0.f, 0.f),
                        mapa(bar_hdr, d));
        } else {
            const int idx = j - 1;
            const int b = idx / in4, c4 = idx - b * in4;
            const uint32_t off = (uint32_t)(((size_t)b * p.in_ld + c4 * 4) * 4);
            st_async_v4(mapa(x_addr + off, d), *reinterpret_cast<const float4 *>(X + (size_t)b * p.in_ld + c4 * 4),
                        mapa(bar_x, d));
        }
    }
}

// Store helper for one finished output element of a row-split layer.
struct EpiRows {
    float *out;
    int ld;
    const float *bias;
    const float *scale;
    int act;
    int round_out;
    __device__ __forceinline__ void operator()(int b, int r, float acc) const
    {
        float v = scale ? acc * scale[r] : acc;
        v = act_apply(v + bias[r], act);
        out[(size_t)b * ld + r] = round_out ? round_bf16(v) : v;
    }
};

struct EpiRaw {
    float *out;
    int ld;
    __device__ __forceinline__ void operator()(int b, int r, float acc) const { out[(size_t)b * ld + r] = acc; }
};

// Push nrows x R floats from the staging buffer into `dst_buf` of cluster CTAs
// [r_lo, r_hi) at column offset col0, completing tx on their `bar`.
__device__ __forceinline__ void push_rows(const KernelCtx &k, const float *stage, int R, int nrows, uint32_t dst_base,
                                          int dst_ld, int col0, uint32_t bar, int r_lo, int r_hi)
{
    const int n4 = R >> 2;
    const int per = nrows * n4;
    const int total = per * (r_hi - r_lo);
    for (int t = threadIdx.x; t < total; t += kThreads) {
        const int d = r_lo + t / per;
        const int rem = t % per;
        const int b = rem / n4, c4 = rem - b * n4;
        const float4 v = *reinterpret_cast<const float4 *>(stage + (size_t)b * R + c4 * 4);
        const uint32_t off = (uint32_t)(((size_t)b * dst_ld + col0 + c4 * 4) * 4);
        st_async_v4(mapa(dst_base + off, (uint32_t)d), v, mapa(bar, (uint32_t)d));
    }
}

template <int WT, bool BATCHED>
__global__ void __launch_bounds__(kThreads, 1) ll_resident_mlp_kernel(const __grid_constant__ Params pg)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(16) Shared sh;
    __shared__ __align__(16) Params sp;  // plan copied once: every later read is a shared-memory load

    {
        static_assert(sizeof(Params) % 4 == 0, "Params is copied word by word");
        const uint32_t *src = reinterpret_cast<const uint32_t *>(&pg);
        uint32_t *dst = reinterpret_cast<uint32_t *>(&sp);
        for (int i = threadIdx.x; i < (int)(sizeof(Params) / 4); i += kThreads)
            dst[i] = src[i];
        __syncthreads();
    }
    const Params &p = sp;

    KernelCtx k;
    k.p = &p;
    k.sh = &sh;
    k.smem = smem;
    k.rank = cluster_ctarank();
    k.stage = (int)(blockIdx.x / (unsigned)p.C);
    const int tid = threadIdx.x;
    const bool leader = (k.stage == 0 && k.rank == 0);  // dispatcher
    const bool last_stage = (k.stage == p.n_stages - 1);
    const bool final_writer = last_stage && k.rank == 0;
    const uint32_t bar_load = smem_u32(&sh.bar[0]);
    const uint32_t bar_a = smem_u32(&sh.bar[1]);
    const uint32_t bar_b = smem_u32(&sh.bar[2]);
    const uint32_t bar_g = smem_u32(&sh.bar[3]);
    const uint32_t bar_diag = smem_u32(&sh.bar[4]);
    const uint32_t bar_hdr = smem_u32(&sh.bar[5]);
    const uint32_t bar_x = smem_u32(&sh.bar[6]);

    if (tid == 0) {
        for (int i = 0; i < 7; ++i)
            mbar_init(smem_u32(&sh.bar[i]), 1);
        sh.cmd = 0;
        sh.nrows = 1;
        sh.fail = 0;
        sh.abort = 0;
        sh.hstop = 0;
        fence_mbar_init_cluster();
        if (leader)
            st_relaxed_sys_u32(&p.ctrl->state, ST_LOADING);
    }
    // Zero all activation buffers once so padded columns are exact zeros.
    {
        uint4 *z = reinterpret_cast<uint4 *>(smem + p.buf_off[BUF_X]);
        const uint32_t n16 = (p.smem_bytes - p.buf_off[BUF_X]) / 16;
        for (uint32_t i = tid; i < n16; i += kThreads)
            z[i] = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();

    bool ok = true;
    const uint32_t img_bytes = p.image_bytes[k.stage];
    if (img_bytes > 0) {
        if (tid == 0) {
            mbar_arrive_expect_tx(bar_load, img_bytes);
            const uint8_t *src = p.image + (size_t)blockIdx.x * p.image_stride;
            const uint32_t dst = smem_u32(smem);
            for (uint32_t off = 0; off < img_bytes; off += 32768u) {
                const uint32_t n = img_bytes - off < 32768u ? img_bytes - off : 32768u;
                bulk_g2s(dst + off, src + off, n, bar_load);
            }
        }
        ok = cta_wait_bar(k, bar_load, 0, EW_LOAD, p.step_ns);
    }
    cluster_sync();  // barriers initialised and images resident in every CTA of the cluster
    if (leader && tid == 0)
        st_relaxed_sys_u32(&p.ctrl->state, ST_RUNNING);

    if (ok && p.diag_wait_never && leader) {
        // bar[4] is never arrived on: this bounded wait must run out
        ok = cta_wait_bar(k, bar_diag, 0, EW_DIAG, p.step_ns);
    }

    uint32_t last = p.last_seq;
    uint32_t n_done = 0;
    uint32_t ph_a = 0, ph_b = 0;
    uint32_t ph_g = 0, ph_hdr = 0, ph_x = 0;
    const int first_l = p.stage_first[k.stage];
    const int last_l = p.stage_last[k.stage];

    while (ok) {
        // ---------------- 1. obtain the next request ----------------
        uint32_t seq;
        int nrows;
        if (p.mode == MODE_QUEUE && (int)n_done >= p.q_n)
            break;  // every stage knows the queue length
        if (leader) {
            // A pipeline of clusters carries one request at a time: every stage hands off
            // through a single buffer, so the first stage takes request n only once the last
            // stage has published request n-1 (queue mode, and a mailbox ring with several
            // requests waiting; a closed-loop host never has two in flight).
            if (n_done > 0 && p.n_stages > 1) {
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
                seq = n_done + 1;
                nrows = p.q_rows;
                if (tid == 0)
                    trace(k, n_done, 0);
                stage_input_device(k, p.q_x + (size_t)n_done * p.q_rows * p.in_dim, nrows);
            } else {
                if (p.mailbox_format == 1) {
                    if (tid < 32) {
                        const uint32_t c = poll_tagged(k, last, buf_ptr(k, BUF_X), ring_slot(p, n_done));
                        if (tid == 0) {
                            if (c == kCmdExit)
                                broadcast_abort(k);
                            sh.cmd = c;
                            sh.nrows = 1;
                            sh.hstop = 0;
                            trace(k, n_done, 0);
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
                if (p.mailbox_format == 1) {
                    // x already in X
                } else if (p.max_batch == 1) {
                    // batch 1: no header fetch (n_rows is 1; stop is seen on the idle cadence, so a
                    // stop that comes with a doorbell bump costs one extra, harmless reply)
                    if (tid == 0) {
                        sh.nrows = 1;
                        sh.hstop = 0;
                    }
                    stage_input_mailbox(k, 1);
                    __syncthreads();
                } else {
                    if (tid == 0)
                        read_header(k);
                    __syncthreads();
                    stage_input_mailbox(k, (int)*reinterpret_cast<volatile uint32_t *>(&sh.nrows));
                }
                nrows = (int)*reinterpret_cast<volatile uint32_t *>(&sh.nrows);
                if (*reinterpret_cast<volatile uint32_t *>(&sh.hstop)) {
                    if (tid == 0) {
                        st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_STOP);
                        broadcast_abort(k);
                    }
                    break;
                }
            }
            __syncthreads();
            if (tid == 0)
                trace(k, n_done, 1);
            if (p.C > 1)
                push_request(k, seq, nrows, bar_hdr, bar_x);
            if (tid == 0)
                trace(k, n_done, 2);
        } else if (k.stage == 0) {
            // peer of the dispatcher: {seq, n_rows} then x arrive by DSMEM push
            if (tid == 0)
                mbar_arrive_expect_tx(bar_hdr, 16u);
            if (!cta_wait_bar(k, bar_hdr, ph_hdr & 1u, EW_PEER_POLL, p.idle_ns + p.peer_margin_ns))
                break;
            ++ph_hdr;
            seq = *reinterpret_cast<volatile uint32_t *>(&sh.hdr[0]);
            nrows = (int)*reinterpret_cast<volatile uint32_t *>(&sh.hdr[1]);
            if (nrows < 1 || nrows > p.max_batch)
                nrows = 1;  // never index past the buffers, whatever arrived
            if (tid == 0)
                mbar_arrive_expect_tx(bar_x, (uint32_t)(nrows * p.in_ld * 4));
            if (!cta_wait_bar(k, bar_x, ph_x & 1u, EW_PEER_POLL, p.step_ns))
                break;
            ++ph_x;
            if (tid == 0 && k.rank == 1)
                trace(k, n_done, 15);
        } else if (p.xfer_tagged) {
            // Batch 1: the previous cluster's values arrive as words {seq, fp32}; every thread
            // polls its words until each carries this request's number.  Queue mode numbers
            // requests 1, 2, ... per launch.  On the mailbox the number is the host's sequence
            // number, which a hand-driven host may advance by more than one: a word is current
            // when its tag is neither 0 (the words are cleared at every launch) nor `last` (the
            // request this stage served before).  Stage 0 hands over request n only after the
            // last stage has published request n-1, so the buffer holds words of `last` or of
            // the one new request: once every word is current they all carry the same number,
            // read from word 0.  Thread 0 watches the abort flag and the idle bound.
            const bool queue = p.mode == MODE_QUEUE;
            const uint32_t want = queue ? n_done + 1u : 0u;
            const unsigned long long *src =
                reinterpret_cast<const unsigned long long *>(p.xfer + (size_t)(k.stage - 1) * p.xfer_stride);
            float *X = buf_ptr(k, BUF_X);
            const int ld = p.stage_in_ld[k.stage];
            const uint64_t t0 = globaltimer();
            bool quit = false;
            for (uint32_t it = 0;; ++it) {
                bool got = true;
                for (int t = tid; t < ld; t += kThreads) {
                    const unsigned long long w = ld_relaxed_gpu_u64(src + t);
                    const uint32_t tag = (uint32_t)(w >> 32);
                    if (queue ? tag == want : (tag != 0u && tag != last)) {
                        X[t] = __uint_as_float((uint32_t)w);
                        if (t == 0)
                            sh.xtag = tag;
                    } else {
                        got = false;
                    }
                }
                if (__syncthreads_and(got))
                    break;
                if ((it & 31u) == 31u) {
                    if (tid == 0) {
                        uint32_t stop = (sh.abort || global_abort(k)) ? 1u : 0u;
                        if (!stop && globaltimer() - t0 > p.idle_ns + 2 * p.peer_margin_ns) {
                            report_error(k, LL_ERR_DEVICE_FAULT, EW_XFER);
                            broadcast_abort(k);
                            stop = 1u;
                        }
                        sh.cmd = stop;
                    }
                    __syncthreads();
                    quit = *reinterpret_cast<volatile uint32_t *>(&sh.cmd) != 0u;
                    __syncthreads();  // every thread has read sh.cmd before thread 0 writes it again
                    if (quit)
                        break;
                }
            }
            if (quit)
                break;
            seq = *reinterpret_cast<volatile uint32_t *>(&sh.xtag);  // written before the barrier above
            nrows = 1;
            if (tid == 0 && final_writer)
                trace(k, n_done, 11);
        } else {
            // Wait for the previous cluster's rows of this request (through L2).
            if (tid == 0) {
                const unsigned target = (unsigned)p.C * (n_done + 1u);
                const unsigned *cnt = p.xfer_cnt + (k.stage - 1);
                const uint64_t t0 = globaltimer();
                uint32_t c = kCmdExit;
                for (uint32_t it = 0;; ++it) {
                    if (ld_acquire_gpu(cnt) >= target) {
                        c = ld_relaxed_gpu_u32(p.xfer_hdr + 2 * (k.stage - 1));
                        sh.nrows = ld_relaxed_gpu_u32(p.xfer_hdr + 2 * (k.stage - 1) + 1);
                        break;
                    }
                    if ((it & 31u) == 31u) {
                        if (sh.abort || global_abort(k))
                            break;
                        if (globaltimer() - t0 > p.idle_ns + 2 * p.peer_margin_ns) {
                            report_error(k, LL_ERR_DEVICE_FAULT, EW_XFER);
                            broadcast_abort(k);
                            break;
                        }
                    }
                }
                sh.cmd = c;
                if (final_writer)
                    trace(k, n_done, 11);
            }
            __syncthreads();
            seq = *reinterpret_cast<volatile uint32_t *>(&sh.cmd);
            nrows = (int)*reinterpret_cast<volatile uint32_t *>(&sh.nrows);
            if (seq == kCmdExit)
                break;
            if (nrows < 1 || nrows > p.max_batch)
                nrows = 1;
            const float *src = p.xfer + (size_t)(k.stage - 1) * p.xfer_stride;
            float *X = buf_ptr(k, BUF_X);
            const int ld = p.stage_in_ld[k.stage];
            const int q = ld >> 2;
            for (int t = tid; t < nrows * q; t += kThreads) {
                const int b = t / q, c4 = t - b * q;
                *reinterpret_cast<float4 *>(X + (size_t)b * ld + c4 * 4) = ld_cg_v4(src + (size_t)b * ld + c4 * 4);
            }
        }
        __syncthreads();

        // ---------------- 2. this stage's layers ----------------
        for (int l = first_l; l <= last_l && ok; ++l) {
            const LayerDev &L = p.L[l];
            const uint8_t *W = smem + L.w_off;
            const float *bias = reinterpret_cast<const float *>(smem + L.b_off);
            const float *scale = L.s_off == 0xffffffffu ? nullptr : reinterpret_cast<const float *>(smem + L.s_off);
            const float *in = buf_ptr(k, L.in_buf);
            float *stg = buf_ptr(k, BUF_STAGE);
            switch (L.mode) {
            case LM_REPLICATED:
            case LM_ROWSPLIT_LOCAL: {
                EpiRows epi{buf_ptr(k, L.out_buf), L.out_ld, bias, scale, L.act, L.round_out};
                layer_dot<WT, BATCHED>(W, L.R, L.K, in, L.in_ld, nrows, L.lpr_log2, epi);
                __syncthreads();
                break;
            }
            case LM_ROWSPLIT_ALLGATHER: {
                EpiRows epi{stg, L.R, bias, scale, L.act, L.round_out};
                layer_dot<WT, BATCHED>(W, L.R, L.K, in, L.in_ld, nrows, L.lpr_log2, epi);
                __syncthreads();
                const bool use_a = L.out_buf == BUF_A;
                const uint32_t bar = use_a ? bar_a : bar_b;
                const uint32_t ph = use_a ? ph_a : ph_b;
                push_rows(k, stg, L.R, nrows, buf_addr(k, L.out_buf), L.out_ld, (int)k.rank * L.R, bar, 0, p.C);
                if (tid == 0)
                    mbar_arrive_expect_tx(bar, (uint32_t)(nrows * L.Mp * 4));
                ok = cta_wait_bar(k, bar, ph & 1u, EW_LAYER_BASE + (uint32_t)l, p.step_ns);
                if (use_a)
                    ++ph_a;
                else
                    ++ph_b;
                break;
            }
            case LM_KSPLIT_GATHER: {
                EpiRaw epi{stg, L.R};
                layer_dot<WT, BATCHED>(W, L.R, L.K, in, L.in_ld, nrows, L.lpr_log2, epi);
                __syncthreads();
                // partials -> G[rank][b][OUTp] of rank 0
                push_rows(k, stg, L.R, nrows, buf_addr(k, BUF_G) + k.rank * (uint32_t)(p.bmax4 * L.R * 4), L.R, 0,
                          bar_g, 0, 1);
                break;
            }
            case LM_ROWSPLIT_GATHER: {
                EpiRows epi{stg, L.R, bias, scale, L.act, 0};
                layer_dot<WT, BATCHED>(W, L.R, L.K, in, L.in_ld, nrows, L.lpr_log2, epi);
                __syncthreads();
                push_rows(k, stg, L.R, nrows, buf_addr(k, BUF_G), L.Mp, (int)k.rank * L.R, bar_g, 0, 1);
                break;
            }
            case LM_ROWSPLIT_GLOBAL: {
                EpiRows epi{stg, L.R, bias, scale, L.act, L.round_out};
                layer_dot<WT, BATCHED>(W, L.R, L.K, in, L.in_ld, nrows, L.lpr_log2, epi);
                __syncthreads();
                if (p.xfer_tagged) {
                    // batch 1: every value leaves as one 64-bit word {seq, fp32}; the next stage
                    // polls the words themselves (one L2 trip; no header, fence or counter)
                    unsigned long long *dw =
                        reinterpret_cast<unsigned long long *>(p.xfer + (size_t)k.stage * p.xfer_stride) + k.rank * L.R;
                    for (int t = tid; t < L.R; t += kThreads)
                        st_relaxed_gpu_u64(dw + t, ((unsigned long long)seq << 32) | __float_as_uint(stg[t]));
                    break;
                }
                float *dst = p.xfer + (size_t)k.stage * p.xfer_stride;
                const int n4 = L.R >> 2;
                for (int t = tid; t < nrows * n4; t += kThreads) {
                    const int b = t / n4, c4 = t - b * n4;
                    st_cg_v4(dst + (size_t)b * L.Mp + k.rank * L.R + c4 * 4,
                             *reinterpret_cast<const float4 *>(stg + (size_t)b * L.R + c4 * 4));
                }
                if (tid == 0 && k.rank == 0) {
                    st_relaxed_gpu_u32(p.xfer_hdr + 2 * k.stage, seq);
                    st_relaxed_gpu_u32(p.xfer_hdr + 2 * k.stage + 1, (uint32_t)nrows);
                }
                __syncthreads();
                if (tid == 0) {
                    __threadfence();
                    red_release_gpu_add(p.xfer_cnt + k.stage, 1u);
                }
                break;
            }
            default:
                break;
            }
            if (leader && tid == 0 && l - first_l < 8)
                trace(k, n_done, 3 + (l - first_l));
        }
        if (!ok)
            break;

        // ---------------- 3. rank 0 of the last stage publishes ----------------
        if (final_writer) {
            const float *G;
            bool ksplit = false;
            int ld_g = 0;
            const LayerDev *Lf = nullptr;
            if (p.n_layers > 0) {
                Lf = &p.L[p.n_layers - 1];
                ksplit = Lf->mode == LM_KSPLIT_GATHER;
                ld_g = Lf->mode == LM_KSPLIT_GATHER ? Lf->R : Lf->Mp;
                const uint32_t bytes = ksplit ? (uint32_t)(p.C * nrows * Lf->R * 4) : (uint32_t)(nrows * Lf->Mp * 4);
                if (tid == 0)
                    mbar_arrive_expect_tx(bar_g, bytes);
                ok = cta_wait_bar(k, bar_g, ph_g & 1u, EW_GATHER, p.step_ns);
                ++ph_g;
                if (!ok)
                    break;
                G = buf_ptr(k, BUF_G);
            } else {
                G = buf_ptr(k, BUF_X);  // echo: y = x
                ld_g = p.in_ld;
            }
            if (tid == 0)
                trace(k, n_done, 12);
            if (tid < 32 && p.mode == MODE_MAILBOX && p.mailbox_format == 1) {
                // tagged output: chunk c = {y[3c], y[3c+1], y[3c+2], seq}, relaxed stores, no fence
                const int out = p.out_dim, nyc = (out + 2) / 3;
                const float *fbias = Lf ? reinterpret_cast<const float *>(smem + Lf->b_off) : nullptr;
                const float *fscale =
                    (Lf && Lf->s_off != 0xffffffffu) ? reinterpret_cast<const float *>(smem + Lf->s_off) : nullptr;
                const int fact = Lf ? Lf->act : LL_ACT_IDENTITY;
                for (int ch = tid; ch < nyc; ch += 32) {
                    float v[3] = {0.f, 0.f, 0.f};
                    for (int e = 0; e < 3; ++e) {
                        const int o = 3 * ch + e;
                        if (o >= out)
                            break;
                        if (Lf == nullptr) {
                            v[e] = o < p.in_dim ? G[o] : 0.0f;
                        } else if (ksplit) {
                            float acc = 0.0f;
                            for (int c = 0; c < p.C; ++c)
                                acc += G[(size_t)c * p.bmax4 * ld_g + o];
                            if (fscale)
                                acc *= fscale[o];
                            v[e] = act_apply(acc + fbias[o], fact);
                        } else {
                            v[e] = G[o];
                        }
                    }
                    st_relaxed_sys_v4(p.mb_y + (size_t)ring_slot(p, n_done) * p.ring_ystride_f + 4 * ch,
                                      make_float4(v[0], v[1], v[2], __uint_as_float(seq)));
                }
                __syncwarp();
                if (tid == 0) {
                    trace(k, n_done, 13);
                    st_relaxed_sys_u32(&p.mb->seq_out, seq);  // bookkeeping only: the host waits on the tags
                    if (p.n_stages > 1) {  // the first stage may take the next request
                        __threadfence();
                        red_release_gpu_add(p.q_done, 1u);
                    }
                    trace(k, n_done, 14);
                }
            } else if (tid < 32) {
                const int out = p.out_dim;
                float *ydst = p.mode == MODE_QUEUE ? p.q_y + (size_t)n_done * p.q_rows * out : p.mb_y;
                const float *fbias = Lf ? reinterpret_cast<const float *>(smem + Lf->b_off) : nullptr;
                const float *fscale =
                    (Lf && Lf->s_off != 0xffffffffu) ? reinterpret_cast<const float *>(smem + Lf->s_off) : nullptr;
                const int fact = Lf ? Lf->act : LL_ACT_IDENTITY;
                for (int idx = tid; idx < nrows * out; idx += 32) {
                    const int b = idx / out, o = idx - b * out;
                    float v;
                    if (Lf == nullptr) {
                        v = o < p.in_dim ? G[(size_t)b * ld_g + o] : 0.0f;
                    } else if (ksplit) {
                        float acc = 0.0f;
                        for (int c = 0; c < p.C; ++c)
                            acc += G[((size_t)c * p.bmax4 + b) * ld_g + o];
                        if (fscale)
                            acc *= fscale[o];
                        v = act_apply(acc + fbias[o], fact);
                    } else {
                        v = G[(size_t)b * ld_g + o];
                    }
                    if (p.mode == MODE_QUEUE)
                        ydst[idx] = v;
                    else
                        st_relaxed_sys_f32(ydst + idx, v);
                }
                __syncwarp();
                if (tid == 0) {
                    trace(k, n_done, 13);
                    if (p.mode == MODE_QUEUE) {
                        if (p.q_stamp)
                            p.q_stamp[n_done] = globaltimer();
                    } else {
                        // release: y reaches the host before seq_out (src/bench_persistent_mbyv_mlp.cu:365-370)
                        st_release_sys_u32(&p.mb->seq_out, seq);
                    }
                    if (p.n_stages > 1) {  // the first stage may take the next request
                        __threadfence();
                        red_release_gpu_add(p.q_done, 1u);
                    }
                    trace(k, n_done, 14);
                }
            }
        }
        last = seq;
        ++n_done;
    }

    // Leave together: no CTA may exit while a peer can still write its shared memory.
    __syncthreads();
    cluster_sync();
    if (leader && tid == 0) {
        if (p.mode == MODE_QUEUE)
            st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_QUEUE_DONE);
        st_release_sys_u32(&p.ctrl->state, ST_EXITED);
    }
}

}  // namespace llk
