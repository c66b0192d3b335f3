// Pipelined ring kernel (engine kernel variant 4) for the 3-layer fp32 nets of the
// register-resident kernel, serving the tagged request ring at high request rates.
//
// The register-resident kernel (fast3_kernel.cuh) runs a pass strictly in sequence on rank 0:
// read the waiting ring slots over PCIe, forward x to the peers, compute, gather, reply,
// and only then read the next slots.  At 16 requests per pass that is ~6 us of reading and
// forwarding plus ~8 us of layers.  Here a cluster of C + 1 CTAs splits the roles, so the
// I/O of one pass overlaps the layers of the previous one:
//   ranks 0..C-1  compute CTAs: the register-resident kernel's weights, held in registers
//                 blocked for many rows per pass (ring_layers.cuh: each input value read from
//                 shared memory serves 4 or 2 output rows); a request's reply is the same
//                 bit for bit whatever the size of its pass;
//                 x arrives in one of two chunk buffers (by pass parity), the CTA unpacks it,
//                 tells the I/O CTA the buffer is free, runs the layers and sends its
//                 layer-3 partials into the I/O CTA's gather buffer of that parity;
//   rank C        the I/O CTA, no weights:
//                 warp 0       reader: poll the next ring slot (and push its chunks to the C
//                              compute CTAs from registers, the register-resident kernel's
//                              protocol), or read up to micro_batch waiting slots at once by
//                              bulk copies from host memory into this CTA's shared memory and
//                              forward them by bulk copies, one per compute CTA and part,
//                              which run on while the reader starts on the next pass
//                              (ring_take_rows);
//                 warps 8..15  gatherer: add the C partials per output in rank order, apply
//                              bias and activation, write each reply into its slot.
// Pass p uses x chunk buffer b = p & 1 and gather buffer g = p % 3 (partials and the
// pass's row metadata).  Before forwarding pass p the reader waits until every compute CTA
// has unpacked pass p-2 (mbarrier `xfree[b]`, C remote arrivals) and until the gatherer has
// finished pass p-3 (`gfree[g]`), so no buffer is overwritten while it is still read; the
// third gather buffer lets the reader start a pass while the replies of the pass two
// before it are still being written.  The reader hands each pass's row count, first
// request index and sequence numbers to the gatherer through `posted[g]`.  Requests are taken and replies
// written in ring order, so the host-side protocol is the register-resident kernel's.
// Every wait is bounded (step_timeout_ns inside a pass, idle_timeout_ns + a margin between
// passes); an exit (stop, idle bound, abort) is broadcast to the cluster, and the gatherer
// finishes the pass whose partials it is waiting for.  Mailbox only (tagged format); no
// device queue.
//
// No counterpart in the reference, whose persistent kernels serve one request at a time
// (src/bench_persistent_mbyv_mlp.cu:229-381).
#pragma once
#include "fast3_kernel.cuh"
#include "ring_layers.cuh"

namespace llk {

constexpr int kRingReadWarps = 8;    // I/O CTA warps 0..7
constexpr int kRingGatherWarp0 = 8;  // I/O CTA warps 8..15
constexpr int kRingGathBufs = 3;  // gather buffers: the reader may run NG - 1 passes ahead of the replies
constexpr int kRingGatherThreads = kThreads - 32 * kRingGatherWarp0;

// A warp waits for an mbarrier phase.  Lane 0 watches the clock and, when `abortable`, the
// abort flags.  Returns 1 when the phase completed, 0 on abort, -1 when the bound ran out;
// the verdict is the same in every lane.
__device__ __forceinline__ int warp_wait_bar(const KernelCtx &k, uint32_t bar, uint32_t parity, uint64_t bound_ns,
                                             bool abortable)
{
    const int lane = threadIdx.x & 31;
    const uint64_t t0 = lane == 0 ? globaltimer() : 0;
    for (uint32_t it = 0;; ++it) {
        const bool done = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, done))
            return 1;
        if ((it & 15u) == 15u) {
            int verdict = 1;
            if (lane == 0) {
                if (abortable && (*reinterpret_cast<volatile uint32_t *>(&k.sh->abort) || global_abort(k)))
                    verdict = 0;
                else if (globaltimer() - t0 > bound_ns)
                    verdict = -1;
            }
            verdict = __shfl_sync(0xffffffffu, verdict, 0);
            if (verdict != 1)
                return verdict;
        }
    }
}

// Reader warp: read up to maxb waiting ring slots (requests n, n + 1, ...) in one go.  Lane 0
// copies the slots from host memory into `stage` (this CTA's shared memory, slot layout kept)
// with one or two 1-D bulk copies (TMA; two when the slots wrap around the ring), which read
// host memory in large requests (measured on B200: 16 slots in 1.6 us against 2.6 us for 16-byte
// loads spread over 8 warps); lane 31 reads seq_in meanwhile.  After the copies land (bounded
// wait) the lanes check the tags.  Returns nb, the complete slots before the first gap (0: request
// n is not complete yet), or -1 when the copies did not land in time.  The forwarder warp sends
// the rows on (ring_forward).
template <int NXC, int MAXB>
__device__ int ring_take_rows(const KernelCtx &k, uint32_t last, uint32_t n, int maxb, uint32_t *seqs,
                              uint32_t *posted, const uint4 *stage_p, uint32_t stage, uint32_t rbar, uint32_t rpar)
{
    const Params &p = *k.p;
    const int lane = threadIdx.x & 31;
    constexpr uint32_t RB = 16u * NXC;  // bytes per slot
    if (lane == 0) {
        const uint32_t s0 = ring_slot(p, n);
        const int first = min(maxb, p.ring_slots - (int)s0);
        mbar_arrive_expect_tx(rbar, RB * (uint32_t)maxb);
        bulk_g2s(stage, p.mb_x + (size_t)s0 * p.ring_xstride_f, RB * (uint32_t)first, rbar);
        if (first < maxb)
            bulk_g2s(stage + RB * (uint32_t)first, p.mb_x, RB * (uint32_t)(maxb - first), rbar);
    }
    const uint32_t seen = lane == 31 ? ld_relaxed_sys(&p.mb->seq_in) : 0u;
    *posted = __shfl_sync(0xffffffffu, seen, 31);
    if (warp_wait_bar(k, rbar, rpar, p.step_ns, false) != 1)
        return -1;
    if (lane == 0)
        trace(k, n, 11);  // the slots have landed
    // lane r < maxb holds request r's sequence number; chunk i of row r must carry it.  The
    // loop has a fixed trip count (MAXB rows), so its shared loads and shuffles issue back to
    // back.
    const uint32_t want = seq_after(last, lane + 1);
    const uint32_t *tags = reinterpret_cast<const uint32_t *>(stage_p) + 3;  // word 3 of each chunk
    uint32_t bad = 0;
#pragma unroll
    for (int i0 = 0; i0 < MAXB * NXC; i0 += 32) {
        const int i = i0 + lane;
        const bool in = i < maxb * NXC;
        const int row = (in ? i : 0) / NXC;
        const uint32_t expect = __shfl_sync(0xffffffffu, want, row);
        if (in && tags[4 * i] != expect)
            bad |= 1u << row;
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    if (lane == 0)
        trace(k, n, 15);  // the tags are checked
    const uint32_t stop_bit = maxb < 32 ? (1u << maxb) : 0u;
    const int nb = (bad | stop_bit) ? __ffs(bad | stop_bit) - 1 : 32;
    if (lane < nb)
        seqs[lane] = want;
    return nb;
}

// Forwarder warp: send a pass's rows from `stage` to the C compute CTAs (lane d serves CTA d):
// the header {seq, rows} by st.async completing bar_first, the rows by one bulk copy per CTA
// completing bar_rest.  The copies move ~25 GB/s out of the SM, so a 16-row pass takes ~2 us
// of this warp while the reader goes on to the next pass.
template <int NXC, int C>
__device__ __forceinline__ void ring_forward(uint32_t seq, int nb, uint32_t stage, uint32_t chunks, uint32_t hdr,
                                             uint32_t bar_first, uint32_t bar_rest)
{
    const int lane = threadIdx.x & 31;
    constexpr uint32_t RB = 16u * NXC;
    if (lane < C) {
        const uint32_t d = (uint32_t)lane;
        st_async_v4(mapa(hdr, d), make_float4(__uint_as_float(seq), __uint_as_float((uint32_t)nb), 0.f, 0.f),
                    mapa(bar_first, d));
        bulk_s2peer(mapa(chunks, d), stage, RB * (uint32_t)nb, mapa(bar_rest, d));
    }
}

// Layout of the ring kernel's dynamic shared-memory pool (bytes).  Compute CTAs use [xs | h1[3]
// | h2 | xch[2]], the I/O CTA [gath[NG] | yo | stage[2] | qx] (stage: its copies of the rows it
// forwards; qx: a device-queue pass's rows as they are stored in HBM).  Remote writes go to the other role's region at the same offset in the receiving
// CTA.  h1 holds layer 1's outputs slice-major (ring_layers.cuh); a split pass's slices arrive
// from every compute CTA, so there are three buffers, used by pass % 3: the slowest compute CTA
// is at most two passes behind the fastest (the reader hands pass p + 2 over only when every
// compute CTA has unpacked pass p), so a slice never lands in a buffer still being read.
template <int IN, int H1, int H2, int OUT, int C>
struct RingPool {
    static constexpr int MB = kFast3Rows;
    static constexpr int NXC = (IN + 2) / 3;            // tagged chunks per row
    static constexpr int YO = 3 * ((OUT + 2) / 3) + 4;  // one output row, zero-padded
    static constexpr int R2 = H2 / C;
    static constexpr int NH1 = 3;
    static constexpr int OFF_XS = 0;
    static constexpr int H1_B = 4 * MB * H1;  // one h1 buffer
    static constexpr int OFF_H1 = OFF_XS + 4 * MB * IN;
    static constexpr int OFF_H2 = OFF_H1 + NH1 * H1_B;
    static constexpr int OFF_XCH = (OFF_H2 + 4 * MB * R2 + 15) / 16 * 16;
    static constexpr int XCH_B = 16 * MB * NXC;
    static constexpr int COMPUTE_END = OFF_XCH + 2 * XCH_B;
    static constexpr int GATH_F = MB * C * OUT;  // [row][rank][output]
    static constexpr int OFF_G = 0;
    static constexpr int OFF_YO = OFF_G + kRingGathBufs * 4 * GATH_F;
    static constexpr int OFF_STG = (OFF_YO + 4 * MB * YO + 15) / 16 * 16;
    static constexpr int OFF_QX = OFF_STG + 2 * XCH_B;  // device queue: a pass's rows as stored in HBM
    static constexpr int IO_END = OFF_QX + 4 * MB * IN;
    static constexpr int BYTES = COMPUTE_END > IO_END ? COMPUTE_END : IO_END;
};

template <int IN, int H1, int H2, int OUT, int C>
__global__ void __launch_bounds__(kThreads, 1) ll_ring_kernel(const __grid_constant__ Params pg)
{
    using S = Fast3Shape<IN, H1, H2, OUT, C>;    // layer 3 and the buffer shapes
    using RS = RingShape<IN, H1, H2, OUT, C>;    // the blocked weights of layers 1 and 2
    using PL = RingPool<IN, H1, H2, OUT, C>;
    static_assert(RS::NB == S::NB && RS::R2 == S::R2 && RS::K3 == S::K3 && RS::R1 == RS::R2,
                  "the ring image's biases and layer-3 slice are the register-resident image's; a layer-1 "
                  "slice block stages in h2's place");
    constexpr int MB = kFast3Rows;
    static_assert(S::MaxRows == kFast3Rows, "the shape leaves no room for multi-row passes");
    constexpr int NXC = PL::NXC;
    constexpr int YO = PL::YO;
    constexpr int IO = C;  // rank of the I/O CTA
    constexpr int OFF_XS = PL::OFF_XS, OFF_H1 = PL::OFF_H1, OFF_H2 = PL::OFF_H2, OFF_XCH = PL::OFF_XCH;
    constexpr int XCH_B = PL::XCH_B, GATH_F = PL::GATH_F, OFF_G = PL::OFF_G, OFF_YO = PL::OFF_YO;
    constexpr int OFF_STG = PL::OFF_STG, OFF_QX = PL::OFF_QX;
    extern __shared__ __align__(128) uint8_t pool[];  // PL::BYTES, dynamic
    __shared__ __align__(16) uint32_t hdr2[2][4];  // compute CTAs: {seq, rows} of the pass in buffer b
    __shared__ __align__(8) uint64_t rb[14 + 3 * kRingGathBufs];  // see the barrier indices below
    __shared__ uint32_t fq[2][4];                   // I/O: reader -> forwarder, per stage buffer: rows, seq, kind, n
    __shared__ __align__(16) float bias[S::NB];
    __shared__ uint32_t mseq[kRingGathBufs][MB];   // I/O: sequence number of each row of the pass in buffer g
    __shared__ uint32_t mrows[kRingGathBufs], mbase[kRingGathBufs];  // I/O: rows (0 = exit), first request index
    __shared__ uint32_t s_backlog[2];
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
    const bool io = k.rank == (uint32_t)IO;
    // barriers: compute CTAs 0,1 bar_req[b] (the header {seq, rows}), 2,3 bar_x[b] (the rows);
    // I/O CTA 4,5 xfree[b], then NG each of bar_g[g] (partials), gfree[g], posted[g]
    auto bar = [&](int i) { return smem_u32(&rb[i]); };
    constexpr int NG = kRingGathBufs;
    auto bar_g = [&](int g) { return bar(6 + g); };
    auto gfree = [&](int g) { return bar(6 + NG + g); };
    auto posted_bar = [&](int g) { return bar(6 + 2 * NG + g); };
    const uint32_t rbar = bar(6 + 3 * NG);  // I/O CTA: the reader's slot copies from host memory
    auto fready = [&](int b) { return bar(7 + 3 * NG + b); };  // I/O CTA: stage[b] handed to the forwarder
    auto sfree = [&](int b) { return bar(9 + 3 * NG + b); };   // I/O CTA: the forwarder is done with stage[b]
    auto h1bar = [&](int j) { return bar(11 + 3 * NG + j); };  // compute CTAs: layer-1 slices in h1[j]
    const uint32_t pool_a = smem_u32(pool);

    if (tid == 0) {
        for (int i = 0; i < 4; ++i)
            mbar_init(bar(i), 1);
        for (int i = 0; i < 2; ++i)
            mbar_init(bar(4 + i), C);
        for (int i = 0; i < NG; ++i) {
            mbar_init(bar_g(i), 1);
            mbar_init(gfree(i), 1);
            mbar_init(posted_bar(i), 1);
        }
        mbar_init(rbar, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(fready(i), 1);
            mbar_init(sfree(i), 1);
        }
        for (int j = 0; j < PL::NH1; ++j)
            mbar_init(h1bar(j), 1);
        sh.cmd = 0;
        sh.fail = 0;
        sh.abort = 0;
        sh.hstop = 0;
        s_backlog[0] = s_backlog[1] = 0;
        fence_mbar_init_cluster();
        if (io)
            st_relaxed_sys_u32(&p.ctrl->state, ST_LOADING);
    }
    // weights into registers (compute CTAs; the I/O CTA holds none), biases into shared memory
    // (the I/O CTA takes CTA 0's copy: it needs the layer-3 biases)
    const float *img = reinterpret_cast<const float *>(p.image + (size_t)(io ? 0u : k.rank) * p.image_stride);
    float w1[RS::K1], w1s[RS::K1S], w2[RS::K2], w3[S::K3];
    if (!io) {
#pragma unroll
        for (int j = 0; j < RS::K1; ++j)
            w1[j] = ld_once_f32(img + (size_t)j * kThreads + tid);
#pragma unroll
        for (int j = 0; j < RS::K1S; ++j)
            w1s[j] = ld_once_f32(img + (size_t)(RS::K1 + j) * kThreads + tid);
#pragma unroll
        for (int j = 0; j < RS::K2; ++j)
            w2[j] = ld_once_f32(img + (size_t)(RS::K1 + RS::K1S + j) * kThreads + tid);
#pragma unroll
        for (int j = 0; j < S::K3; ++j)
            w3[j] = ld_once_f32(img + (size_t)(RS::K1 + RS::K1S + RS::K2 + j) * kThreads + tid);
    }
    for (int i = tid; i < S::NB; i += kThreads)
        bias[i] = __ldg(img + (size_t)RS::NW * kThreads + i);
    if (io) {
        float *gz = reinterpret_cast<float *>(pool + OFF_G);
        for (int i = tid; i < NG * GATH_F + MB * YO; i += kThreads)
            gz[i] = 0.0f;  // gath[NG] and yo are contiguous
    }
    __syncthreads();
    cluster_sync();  // every barrier of the cluster is initialised before any remote operation
    if (io && tid == 0)
        st_relaxed_sys_u32(&p.ctrl->state, ST_RUNNING);

    uint32_t passes_done = 0, rows_done = 0, last_replied = 0;
    if (!io) {
        // ======================= compute CTA =======================
        const int g2 = warp;  // layer-2 row group
        float *xs = reinterpret_cast<float *>(pool + OFF_XS);
        float *h2 = reinterpret_cast<float *>(pool + OFF_H2);
        const int act1 = p.L[0].act, act2 = p.L[1].act;
        uint32_t ph_x[2] = {0u, 0u};
        uint32_t ph_h1 = 0u;  // bit j: the phase of h1bar(j)
        uint32_t n_req = 0;  // request index of the pass's first row (as counted by the reader)
        for (uint32_t pass = 0;; ++pass) {
            const int b = (int)(pass & 1u);
            const uint32_t par = (pass >> 1) & 1u;
            if (tid == 0)
                mbar_arrive_expect_tx(bar(b), 16u);  // the header {seq, rows} alone
            if (!cta_wait_bar(k, bar(b), par, EW_PEER_POLL, p.idle_ns + p.peer_margin_ns))
                break;
            if (k.rank == 0 && tid == 0)
                trace(k, n_req, 8);
            const uint32_t seq = *reinterpret_cast<volatile uint32_t *>(&hdr2[b][0]);
            if (seq == kCmdExit)
                break;  // the device queue is served (a live request never carries 0)
            uint32_t nb = *reinterpret_cast<volatile uint32_t *>(&hdr2[b][1]);
            nb = nb < 1u ? 1u : (nb > (uint32_t)MB ? (uint32_t)MB : nb);
            {  // the pass's rows, every one on bar_x
                if (tid == 0)
                    mbar_arrive_expect_tx(bar(2 + b), 16u * NXC * nb);
                const uint32_t px = b ? ph_x[1] : ph_x[0];
                if (!cta_wait_bar(k, bar(2 + b), px & 1u, EW_PEER_POLL, p.step_ns))
                    break;
                if (b)
                    ++ph_x[1];
                else
                    ++ph_x[0];
                if (k.rank == 0 && tid == 0)
                    trace(k, n_req, 9);
            }
            // unpack {v0, v1, v2, tag} chunks into the x rows, then release the chunk buffer
            const uint4 *xch = reinterpret_cast<const uint4 *>(pool + OFF_XCH + b * XCH_B);
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
            if (tid == 0)
                mbar_arrive_remote_cta(mapa(bar(4 + b), (uint32_t)IO));  // xfree[b]: x buffer b read
            if (k.rank == 0 && tid == 0)
                trace(k, n_req, 10);
            // layers 1 and 2 with the blocked weights (ring_layers.cuh): one row, or up to 16 at
            // once (the rows past nb compute on stale inputs inside the buffers and are never sent)
            const int hj = (int)(pass % (uint32_t)PL::NH1);
            float *h1 = reinterpret_cast<float *>(pool + OFF_H1 + hj * PL::H1_B);
            if (nb == 1) {
                ring_layer1_x1<RS, IN, H1>(w1, xs, h1, bias, act1);
                __syncthreads();
            } else {
                // this CTA's slice, staged in h2's place (free until layer 2), then one bulk copy
                // of it into every compute CTA's h1[hj] (thread d serves CTA d)
                ring_layer1_split<RS, IN, H1>(w1s, xs, h2, bias, (int)k.rank, act1);
                fence_proxy_async_shared();  // this thread's staging stores, visible to the copies
                __syncthreads();
                constexpr uint32_t SLICE_B = 4u * MB * RS::R1;
                if (tid < C) {
                    bulk_s2peer(mapa(pool_a + OFF_H1 + (uint32_t)hj * PL::H1_B + k.rank * SLICE_B, (uint32_t)tid),
                                smem_u32(h2), SLICE_B, mapa(h1bar(hj), (uint32_t)tid));
                    bulk_commit_group();
                    bulk_wait_group_read<0>();  // h2 is written by layer 2 after the barrier below
                }
                if (tid == 0)
                    mbar_arrive_expect_tx(h1bar(hj), C * SLICE_B);
                if (!cta_wait_bar(k, h1bar(hj), (ph_h1 >> hj) & 1u, EW_LAYER_BASE, p.step_ns))
                    break;
                ph_h1 ^= 1u << hj;
            }
            if (k.rank == 0 && tid == 0)
                trace(k, n_req, 3);
            if (nb == 1)
                ring_layer2_x1<RS, H1>(w2, h1, h2, bias + H1, g2, act2);
            else
                ring_layer2_x16<RS, H1>(w2, h1, h2, bias + H1, g2, act2);
            __syncthreads();
            if (k.rank == 0 && tid == 0)
                trace(k, n_req, 4);
            // layer 3: K-split partials into the I/O CTA's gather buffer of this parity
            if (warp < OUT) {
                const float mine = nb == 1 ? f3_layer3<S, 1>(w3, h2, 1, lane)
                                   : nb <= (uint32_t)kFast3Group ? f3_layer3<S, kFast3Group>(w3, h2, (int)nb, lane)
                                                                 : f3_layer3_x16<S>(w3, h2, lane);
                const uint32_t g = pass % (uint32_t)NG;
                const uint32_t g_addr = pool_a + OFF_G + g * 4u * GATH_F;
                if (lane < (int)nb)
                    st_async_u32(mapa(g_addr + (uint32_t)((lane * C + (int)k.rank) * OUT + warp) * 4u, (uint32_t)IO),
                                 __float_as_uint(mine), mapa(bar_g((int)g), (uint32_t)IO));
            }
            if (k.rank == 0 && tid == 0)
                trace(k, n_req, 5);
            n_req += nb;
        }
    } else if (warp < kRingReadWarps) {
        // ======================= I/O CTA: reader (warp 0) and forwarder (warp 1) =======================
        // The reader polls or reads the slots of each pass (a multi-slot read is one or two bulk
        // copies from host memory, ring_take_rows) and posts the pass to the gatherer; the
        // forwarder sends a multi-slot pass's rows to the compute CTAs (ring_forward), handed
        // over per stage buffer b through `fready[b]` and returned through `sfree[b]`.  Warps 2 ..
        // kRingReadWarps - 1 have no part.
        const int read_warps = 1;
        if (warp == 1) {
            for (uint32_t pass = 0;; ++pass) {
                const int b = (int)(pass & 1u);
                // abortable: every exit of the reader comes with the abort flag set
                if (warp_wait_bar(k, fready(b), (pass >> 1) & 1u, p.idle_ns + 2 * p.peer_margin_ns, true) != 1)
                    break;
                if (fq[b][2] == 1u) {
                    ring_forward<NXC, C>(fq[b][1], (int)fq[b][0], pool_a + OFF_STG + (uint32_t)b * XCH_B,
                                         pool_a + OFF_XCH + (uint32_t)b * XCH_B, smem_u32(&hdr2[b][0]), bar(b),
                                         bar(2 + b));
                    if (lane == 0)
                        trace(k, fq[b][3], 14);  // the copies are issued
                    bulk_commit_group();
                    bulk_wait_group_read<0>();  // the copies have read stage[b]
                }
                __syncwarp();
                if (lane == 0)
                    mbar_arrive_remote_cta(mapa(sfree(b), (uint32_t)IO));  // this CTA's own barrier
                if (fq[b][1] == kCmdExit)
                    break;  // the reader's last pass (the queue is served, or the mailbox closed)
            }
            bulk_wait_group_all();  // no copy into a compute CTA may be in flight when the cluster leaves
        } else if (warp < read_warps) {
            uint32_t last = p.last_seq, n_done = 0, rphase = 0;
            for (uint32_t pass = 0;; ++pass) {
                const int b = (int)(pass & 1u), g = (int)(pass % (uint32_t)NG);
                if (warp == 0) {
                    if (lane == 0)
                        trace(k, n_done, 7);
                    int w = 1;
                    // the compute CTAs have unpacked pass - 2 (x buffer b), and the gatherer has
                    // finished pass - NG (gather buffer g, row metadata g)
                    if (pass >= 2)
                        w = warp_wait_bar(k, bar(4 + b), ((pass - 2u) >> 1) & 1u, p.step_ns, true);
                    if (w == 1 && pass >= (uint32_t)NG)
                        w = warp_wait_bar(k, gfree(g), ((pass - NG) / NG) & 1u, p.step_ns, true);
                    if (lane == 0) {
                        if (w < 0) {
                            report_error(k, LL_ERR_DEVICE_FAULT, EW_GATHER);
                            broadcast_abort(k);
                        }
                        // on a failed wait the abort flag is (or gets) set: the gatherer leaves on it
                        // (no phase is posted here: pass p - NG may still be unfinished, and a second
                        // phase of posted[g] would look like none to the gatherer)
                        sh.cmd = w == 1 ? 1u : 0u;
                        trace(k, n_done, 6);
                    }
                }
                if (warp == 0 && pass >= 2 && *reinterpret_cast<volatile uint32_t *>(&sh.cmd) != 0u) {
                    // the forwarder is done with stage buffer b (pass p - 2)
                    const int w = warp_wait_bar(k, sfree(b), ((pass - 2u) >> 1) & 1u, p.step_ns, true);
                    if (lane == 0 && w != 1) {
                        if (w < 0)
                            report_error(k, LL_ERR_DEVICE_FAULT, EW_GATHER);
                        broadcast_abort(k);
                        sh.cmd = 0u;
                    }
                    __syncwarp();
                }
                if (read_warps > 1)
                    asm volatile("bar.sync 2, %0;" ::"r"(32 * read_warps) : "memory");
                else
                    __syncwarp();
                if (*reinterpret_cast<volatile uint32_t *>(&sh.cmd) == 0u)
                    break;
                // rows 1.. of a multi-slot read are staged in this CTA's stage[b] and bulk-copied
                // to the compute CTAs' chunk buffer b
                const uint32_t xch_b = pool_a + OFF_XCH + (uint32_t)b * XCH_B;
                const ChunkFwd fwd{xch_b, smem_u32(&hdr2[b][0]), bar(b), bar(2 + b), 0, C, 1};
                uint32_t posted = 0;
                int got = 0;
                bool staged = false;  // the pass's rows sit in stage[b] for the forwarder
                const bool queue = p.mode == MODE_QUEUE;
                if (queue) {
                    // device queue: the next up-to-micro_batch requests of q_x (rows in HBM), put
                    // into stage[b] in the ring's chunk format for the forwarder; none left: the
                    // exit pass below
                    const int left = p.q_n - (int)n_done;
                    got = left < p.micro_batch ? left : p.micro_batch;
                    uint4 *stg_p = reinterpret_cast<uint4 *>(pool + OFF_STG + b * XCH_B);
                    if (got > 0) {
                        // the rows, contiguous in HBM, by one bulk copy into qx (bounded wait),
                        // then into the chunk format from shared memory
                        __syncwarp();
                        if (lane == 0) {
                            fence_proxy_async_shared();  // the previous pass's reads of qx come first
                            mbar_arrive_expect_tx(rbar, 4u * IN * (uint32_t)got);
                            bulk_g2s(pool_a + OFF_QX, p.q_x + (size_t)n_done * IN, 4u * IN * (uint32_t)got, rbar);
                        }
                        const int w = warp_wait_bar(k, rbar, rphase & 1u, p.step_ns, false);
                        ++rphase;
                        if (w != 1) {
                            if (lane == 0) {
                                report_error(k, LL_ERR_DEVICE_FAULT, EW_PEER_POLL);
                                broadcast_abort(k);
                            }
                            got = 0;
                        }
                    }
                    const float *qrow = reinterpret_cast<const float *>(pool + OFF_QX);
                    for (int i = lane; i < got * NXC; i += 32) {
                        const int r = i / NXC, ch = i - r * NXC;
                        const float *src = qrow + r * IN + 3 * ch;
                        const float v0 = src[0];
                        const float v1 = 3 * ch + 1 < IN ? src[1] : 0.f;
                        const float v2 = 3 * ch + 2 < IN ? src[2] : 0.f;
                        stg_p[i] = make_uint4(__float_as_uint(v0), __float_as_uint(v1), __float_as_uint(v2),
                                              n_done + (uint32_t)r + 1u);
                    }
                    if (lane < got)
                        mseq[g][lane] = seq_after(last, lane + 1);
                    fence_proxy_async_shared();  // the forwarder's bulk copies read stage[b]
                    staged = got > 0;
                } else if (*reinterpret_cast<volatile uint32_t *>(&s_backlog[pass & 1u])) {
                    const uint32_t stg = pool_a + OFF_STG + (uint32_t)b * XCH_B;
                    got = ring_take_rows<NXC, MB>(k, last, n_done, p.micro_batch, mseq[g], &posted,
                                              reinterpret_cast<const uint4 *>(pool + OFF_STG + b * XCH_B), stg, rbar,
                                              rphase & 1u);
                    ++rphase;
                    staged = got > 0;
                    if (got < 0) {
                        // the slot copies did not land: leave (the final drain waits for them)
                        if (lane == 0) {
                            report_error(k, LL_ERR_DEVICE_FAULT, EW_PEER_POLL);
                            broadcast_abort(k);
                        }
                        got = 0;
                    }
                }
                if (warp == 0) {
                    uint32_t c;
                    if (got > 0) {
                        c = seq_after(last, got);
                    } else if (queue) {
                        // the queue is served: an exit header to every compute CTA (on this pass's
                        // buffer: they leave after the passes before it) and 0 rows to the gatherer
                        c = kCmdExit;
                        if (lane == 0)
                            fwd_header(fwd, kCmdExit, 0u);
                    } else {
                        c = poll_tagged(k, last, nullptr, ring_slot(p, n_done), p.micro_batch > 1 ? &posted : nullptr,
                                        &fwd);
                        got = 1;
                    }
                    bulk_commit_group();  // the slot reads (completion is awaited on rbar)
                    __syncwarp();  // the lanes' mseq writes come before lane 0's release below
                    if (lane == 0) {
                        trace(k, n_done, 1);
                        // hand stage[b] to the forwarder: the rows to send (a multi-slot pass), or
                        // nothing (a polled request, pushed above from registers)
                        fq[b][0] = (uint32_t)got;
                        fq[b][1] = c;
                        fq[b][2] = staged ? 1u : 0u;
                        fq[b][3] = n_done;
                        mbar_arrive_remote_cta(mapa(fready(b), (uint32_t)IO));  // this CTA's own barrier
                        if (got == 1)
                            mseq[g][0] = c;
                        s_backlog[(pass + 1u) & 1u] =
                            (p.micro_batch > 1 && c != kCmdExit && (int32_t)(posted - c) > 0) ? 1u : 0u;
                        if (c == kCmdExit && !queue)
                            broadcast_abort(k);
                        mrows[g] = c == kCmdExit ? 0u : (uint32_t)got;
                        mbase[g] = n_done;
                        trace(k, n_done, 0);
                        mbar_arrive_remote_cta(mapa(posted_bar(g), (uint32_t)IO));  // this CTA's own barrier
                    }
                }
                if (read_warps > 1)
                    asm volatile("bar.sync 2, %0;" ::"r"(32 * read_warps) : "memory");
                const uint32_t rows = *reinterpret_cast<volatile uint32_t *>(&mrows[g]);
                if (rows == 0u)
                    break;
                last = seq_after(last, (int)rows);
                n_done += rows;
            }
            // no bulk copy into a compute CTA may be in flight when the cluster leaves
            if (warp == 0)
                bulk_wait_group_all();
        }
    } else {
        // ======================= I/O CTA: gatherer =======================
        // Gatherer warp 0 waits for the pass and its partials and publishes the row count
        // (0 = leave); all gatherer warps then finish rows gw, gw + 8, ... of the pass.
        const int gt = tid - 32 * kRingGatherWarp0, gw = warp - kRingGatherWarp0;
        constexpr int NGW = kRingGatherThreads / 32;
        for (uint32_t pass = 0;; ++pass) {
            const int g = (int)(pass % (uint32_t)NG);
            const uint32_t par = (pass / NG) & 1u;
            if (gw == 0) {
                // the next pass (abortable: an exit is broadcast; every pass posted before it has
                // already been waited for in order), then its partials (not abortable: a pass that
                // was forwarded is finished, within the step bound)
                uint32_t nb = 0;
                int w = warp_wait_bar(k, posted_bar(g), par, p.idle_ns + 2 * p.peer_margin_ns, true);
                if (w == 1) {
                    nb = *reinterpret_cast<volatile uint32_t *>(&mrows[g]);
                    if (nb > 0u) {
                        if (lane == 0)
                            mbar_arrive_expect_tx(bar_g(g), (uint32_t)(C * OUT * 4) * nb);
                        w = warp_wait_bar(k, bar_g(g), par, p.step_ns, false);
                        if (w != 1)
                            nb = 0;
                    }
                }
                if (lane == 0) {
                    if (w < 0) {
                        report_error(k, LL_ERR_DEVICE_FAULT, nb == 0u && mrows[g] == 0u ? EW_PEER_POLL : EW_GATHER);
                        broadcast_abort(k);
                    }
                    sh.nrows = nb;
                    if (nb > 0u)
                        trace(k, mbase[g], 12);
                }
            }
            asm volatile("bar.sync 3, %0;" ::"r"(kRingGatherThreads) : "memory");
            const uint32_t nb = *reinterpret_cast<volatile uint32_t *>(&sh.nrows);
            if (nb == 0u)
                break;
            const uint32_t base = *reinterpret_cast<volatile uint32_t *>(&mbase[g]);
            const float *gath = reinterpret_cast<const float *>(pool + OFF_G) + (size_t)g * GATH_F;
            for (int r = gw; r < (int)nb; r += NGW) {
                float *yr = reinterpret_cast<float *>(pool + OFF_YO) + r * YO;
                if (lane < OUT) {
                    float v = 0.f;
#pragma unroll
                    for (int c = 0; c < C; ++c)
                        v += gath[(r * C + c) * OUT + lane];
                    yr[lane] = relu_or(v + bias[H1 + S::R2 + lane], p.L[2].act);
                }
                __syncwarp();
                constexpr int NYC = (OUT + 2) / 3;
                if (p.mode == MODE_QUEUE) {
                    if (lane < OUT)
                        p.q_y[(size_t)(base + (uint32_t)r) * OUT + lane] = yr[lane];
                    if (lane == 0 && p.q_stamp)
                        p.q_stamp[base + (uint32_t)r] = globaltimer();
                } else if (lane < NYC) {
                    st_relaxed_sys_v4(p.mb_y + (size_t)ring_slot(p, base + (uint32_t)r) * p.ring_ystride_f + 4 * lane,
                                      make_float4(yr[3 * lane], yr[3 * lane + 1], yr[3 * lane + 2],
                                                  __uint_as_float(mseq[g][r])));
                }
                __syncwarp();
            }
            asm volatile("bar.sync 3, %0;" ::"r"(kRingGatherThreads) : "memory");  // every row of the pass written
            if (gt == 0) {
                trace(k, base, 13);
                mbar_arrive_remote_cta(mapa(gfree(g), (uint32_t)IO));  // this CTA's own barrier
            }
            last_replied = mseq[g][nb - 1];
            ++passes_done;
            rows_done += nb;
        }
        // seq_out is bookkeeping on the tagged mailbox (the host waits on the y tags and reads
        // seq_out after an exit, to resume the ring): written once here, not per pass, because
        // it shares a line with seq_in, which the host writes for every request and the reader
        // polls; a device write per pass made that line travel between CPU and GPU
        if (gt == 0 && passes_done > 0 && p.mode != MODE_QUEUE)
            st_relaxed_sys_u32(&p.mb->seq_out, last_replied);
    }
    if (!io && tid < C)
        bulk_wait_group_all();  // this CTA's layer-1 slices have landed in every compute CTA
    __syncthreads();
    cluster_sync();
    if (io && tid == 32 * kRingGatherWarp0) {
        st_relaxed_sys_u32(&p.ctrl->passes, passes_done);
        st_relaxed_sys_u32(&p.ctrl->rows, rows_done);
    }
    __syncthreads();
    if (io && tid == 0) {
        if (p.mode == MODE_QUEUE)
            st_relaxed_sys_u32(&p.ctrl->exit_reason, EXIT_QUEUE_DONE);
        st_release_sys_u32(&p.ctrl->state, ST_EXITED);
    }
}

}  // namespace llk
