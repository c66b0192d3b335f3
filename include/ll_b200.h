/*
 * ll_b200.h -- C ABI of the B200 (sm_100a) low-latency MLP inference engine.
 *
 * The reference (mamedov-ma/low_latency_inference_gpu) has no library or FFI:
 * its host code launches header-only kernels with <<<>>> and drives a
 * TickBuffer mailbox by hand.  Every entry point below replaces one of those
 * host-side constructs; the reference interface each one stands in for is
 * cited beside it (paths are relative to the reference project root).
 *
 * Conventions: plain pointers and sizes only; every call returns an int status
 * (LL_OK on success) instead of the reference's print-and-exit CUDA_CHECK
 * (include/bench_utils.h:14-22); ll_last_error() gives the message of the
 * calling thread's last failure.  Weights are host row-major [out x in]
 * exactly as the reference's host vectors (src/bench_cublas_mlp.cu:69-80).
 */
#ifndef LL_B200_H
#define LL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (replace CUDA_CHECK -> std::exit(1), include/bench_utils.h:14-22) ---- */
enum {
    LL_OK = 0,
    LL_ERR_CUDA = 1,         /* a CUDA runtime / cuBLAS call failed */
    LL_ERR_TIMEOUT = 2,      /* host-side wait ran out (request not answered in time) */
    LL_ERR_BAD_DESC = 3,     /* network descriptor invalid or does not fit the device */
    LL_ERR_DEVICE_FAULT = 4, /* the resident kernel reported an error (see ll_engine_info) */
    LL_ERR_STOPPED = 5,      /* engine stopped */
    LL_ERR_INVALID_ARG = 6,
    LL_ERR_UNSUPPORTED = 7,
    LL_ERR_BUSY = 8          /* a request is still outstanding */
};

/* ---- activations (include/ll/dense_warp.cuh:9-21 ActIdentity/ActRelu; GELU is new) ---- */
enum { LL_ACT_IDENTITY = 0, LL_ACT_RELU = 1, LL_ACT_GELU = 2 };

/* ---- weight storage types ---- */
enum { LL_W_F32 = 0, LL_W_BF16 = 1, LL_W_I8 = 2 };

/* ---- initialisers for ll_init_params ---- */
enum { LL_INIT_XAVIER_UNIFORM = 0, LL_INIT_NORMAL_FANIN = 1 };

/*
 * Layer / network descriptors: the runtime form of include/net_config.h:6-26
 * (netcfg::IN_DIM/H1_DIM/H2_DIM/OUT_DIM, compile-time constants there).
 */
typedef struct ll_layer_desc {
    int32_t in_dim;
    int32_t out_dim;
    int32_t act;   /* LL_ACT_* applied after bias */
    int32_t wtype; /* LL_W_*; all layers of one net share it */
} ll_layer_desc;

typedef struct ll_net_desc {
    int32_t n_layers;
    const ll_layer_desc *layers;
    int32_t max_batch; /* rows per request the mailbox can carry (>= 1) */
    int32_t reserved;
} ll_net_desc;

/*
 * Mailbox header: field order and meaning of the reference's TickBuffer
 * (src/bench_persistent_mbyv_mlp.cu:88-95, src/bench_persistent_mlp.cu:65-72):
 * seq_in (0 = idle, host increments per request), seq_out (device echoes the
 * finished seq), stop, then one 32-bit word the reference calls `pad`, used
 * here as the request's row count (0 means 1).  The float x[] block follows at
 * byte 16 and y[] right after x[] (in_dim * max_batch floats), so for a batch-1
 * net the layout is byte-identical to the reference struct.
 */
typedef struct ll_tick_header {
    volatile uint32_t seq_in;
    volatile uint32_t seq_out;
    volatile uint32_t stop;
    uint32_t n_rows;
} ll_tick_header;

#define LL_STOP_SEQ 0xFFFFFFFFu /* src/bench_persistent_mbyv_mlp.cu:157 */

typedef struct ll_engine_opts {
    int32_t cluster_size;       /* CTAs per cluster: 1,2,4,8,16; 0 = automatic */
    int32_t replicate_first;    /* first layer computed by every CTA: -1 auto, 0 no, 1 yes */
    int32_t write_combined;     /* allocate the mailbox write-combined (reference default) */
    int32_t mailbox_format;     /* 0 = the reference's TickBuffer layout; 1 = tagged chunks (batch 1,
                                   see ll_tagged_post): no x read after the doorbell, no release fence */
    uint64_t idle_timeout_ns;   /* resident kernel exits after this long idle; relaunched on demand */
    uint64_t step_timeout_ns;   /* bound on every device wait inside one request */
    int32_t max_stages;         /* cap on pipeline stages (clusters); 0 = automatic */
    int32_t min_stages;         /* spread the layers over at least this many clusters; 0 = as few as fit */
    int32_t diag_wait_never;    /* test hook: rank 0 waits on a barrier nothing completes, so the bounded
                                   wait runs out after step_timeout_ns and the kernel reports
                                   LL_ERR_DEVICE_FAULT at location 6 and leaves (no fault is caused) */
    int32_t kernel_variant;     /* 0 = automatic, 1 = generic shared-memory kernel, 2 = register-resident
                                   kernel compiled for the net's shape (3-layer fp32, batch 1),
                                   3 = resident small-batch kernel: one CTA on every SM, each holding
                                   its row slice of every layer in shared memory for the whole launch,
                                   layers handed off through L2 (bf16 or int8 weights, up to 32 rows,
                                   the TickBuffer mailbox or the tagged one at max_batch 1, in / out
                                   widths multiples of 4; it takes every SM, so no other resident
                                   engine may run on the GPU),
                                   4 = pipelined ring kernel (no counterpart in the reference): the
                                   register-resident kernel's C compute CTAs plus one I/O CTA per
                                   cluster that reads the next waiting ring slots and writes the
                                   replies while the compute CTAs run the layers of the previous
                                   pass (tagged mailbox only; replies bit-identical to variant 2;
                                   no device queue).  For request rates above what one pass at a
                                   time sustains; asked for explicitly.
                                   Automatic picks 2 for the shapes it is compiled for, 3 for bf16 /
                                   int8 nets that qualify and whose weights exceed one 16-CTA
                                   cluster's shared memory (about 3.6 MB) unless cluster options are
                                   forced, else 1. */
    int32_t ring_slots;         /* tagged mailbox only: request slots (1..64; 0 = 1).  Up to ring_slots
                                   requests may be outstanding (ll_submit before the earlier ll_poll);
                                   the device serves them in order, slot after slot.  Layout: the
                                   16-byte header, the x chunks of slots 0..Q-1 back to back, then
                                   from the next 64-byte boundary the y chunks of each slot, each
                                   slot's starting on a fresh 64-byte line (one slot is exactly the
                                   single tagged mailbox) */
    int32_t micro_batch;        /* request ring on the register-resident kernel: the device takes up to
                                   this many waiting requests (consecutive slots, each complete) in one
                                   poll and runs them as one small batch (1..16, at most ring_slots;
                                   0 = 1).  Replies still go to each request's own slot and are
                                   bit-identical to the same requests served one at a time. */
    int32_t reserved[2];
} ll_engine_opts;

typedef struct ll_engine_info {
    int32_t n_stages;       /* clusters in the pipeline */
    int32_t cluster_size;   /* CTAs per cluster */
    int32_t threads;        /* threads per CTA */
    int32_t smem_bytes;     /* dynamic shared memory per CTA */
    int32_t image_bytes;    /* largest per-CTA resident weight image */
    int32_t launches;       /* resident-kernel launches since create */
    int32_t state;          /* 0 idle, 1 loading, 2 running, 3 exiting, 4 exited */
    int32_t status;         /* last device status (LL_OK or LL_ERR_*) */
    int32_t err_where;      /* device-side location code of the last error */
    uint32_t served;        /* last seq the device published */
    int32_t layer_modes[24];
    int32_t kernel_variant; /* 1 generic, 2 register-resident, 3 resident small-batch, 4 pipelined ring */
    int32_t weight_regs;    /* register-resident: weights held per thread */
    uint32_t passes;        /* register-resident: passes over the layers by the launches that have
                               exited (ll_engine_stop, idle exit, queue runs) */
    uint32_t rows;          /* ... and the requests those passes took: rows / passes is the mean
                               micro-batch */
} ll_engine_info;

/*
 * Placement of a net on the GPU, as computed by the planner (no GPU needed).
 * Each layer is split over the CTAs of one cluster ("stage"); the per-CTA
 * shared-memory images hold the weight slices.  Layer modes: 0 replicated,
 * 1 row-split + all-gather, 2 row-split kept local, 3 K-split gathered at
 * rank 0, 4 row-split gathered at rank 0, 5 row-split handed to the next
 * cluster through global memory.  The reference fixes this split at compile
 * time per kernel (BLOCKS / WARPS template arguments, include/ll/mbyv.cuh:8-35).
 */
typedef struct ll_plan_layer {
    int32_t mode, act, wtype, lpr_log2;
    int32_t K, M, Mp, R;
    int32_t in_buf, in_ld, out_buf, out_ld;
    uint32_t w_off, b_off, s_off;
    int32_t round_out;
} ll_plan_layer;

typedef struct ll_plan {
    int32_t n_layers, n_stages, cluster_size, threads, bmax4, in_ld, act_bf16, reserved;
    int32_t stage_first[9], stage_last[9], stage_in_ld[9];
    uint32_t image_bytes[9];
    uint32_t buf_off[6]; /* X, A, B, L, G, STAGE */
    uint32_t smem_bytes;
    uint32_t image_stride; /* bytes between consecutive CTA images (CTA = stage * cluster_size + rank) */
    ll_plan_layer layers[24];
} ll_plan;

/*
 * Plan a net without touching the GPU.  If images is non-NULL it receives the
 * packed per-CTA images (n_stages * cluster_size * image_stride bytes, which
 * must not exceed images_cap).  *images_bytes gets the required size.
 */
int ll_plan_net(const ll_net_desc *net, const void *const *W, const float *const *b, const float *const *scales,
                const ll_engine_opts *opts, ll_plan *plan, uint8_t *images, size_t images_cap,
                size_t *images_bytes);

typedef struct ll_engine ll_engine;

void ll_engine_opts_default(ll_engine_opts *opts);

/*
 * Create a resident engine: uploads the weights, plans the per-CTA shared-memory
 * images and allocates the host-mapped mailbox.  Replaces the setup half of the
 * reference's persistent benches (src/bench_persistent_mbyv_mlp.cu:386-491:
 * cudaSetDeviceFlags, cudaMalloc/cudaMemcpy of W/b, cudaHostAlloc(Mapped) of the
 * TickBuffer, kernel launch).  W[l] points to host data of the layer's wtype
 * (float / uint16 bf16 bits / int8); b[l] fp32 [out_dim] (NULL = zeros);
 * scales[l] fp32 [out_dim] for LL_W_I8 (ignored otherwise; scales may be NULL).
 */
int ll_engine_create(const ll_net_desc *net, const void *const *W, const float *const *b, const float *const *scales,
                     int device, ll_engine **out);
int ll_engine_create_ex(const ll_net_desc *net, const void *const *W, const float *const *b,
                        const float *const *scales, int device, const ll_engine_opts *opts, ll_engine **out);

/*
 * Ping-pong floor: the same resident kernel and mailbox with no layers.  It
 * waits for seq_in, reads in_dim floats of x, writes y[i] = x[i] (0 beyond
 * in_dim) for i < out_dim and publishes seq_out.  in_dim = out_dim = 0 echoes
 * only the sequence number.  The reference has no such kernel; its nearest is
 * the empty-launch bench src/bench_main.cu:9-34.
 */
int ll_echo_engine_create(int device, int in_dim, int out_dim, const ll_engine_opts *opts, ll_engine **out);

/* Host pointer of the mailbox (layout of ll_tick_header + x + y, see above; on a tagged
 * ring, _x and _y point at slot 0's x and y chunks). */
void *ll_engine_mailbox(ll_engine *e);
float *ll_engine_mailbox_x(ll_engine *e);
float *ll_engine_mailbox_y(ll_engine *e);

/* Launch the resident kernel (also done lazily by ll_submit). */
int ll_engine_start(ll_engine *e);

/*
 * Host doorbell, the reference's per-request host code
 * (src/bench_persistent_mbyv_mlp.cu:539-544): write x (skipped when x is
 * NULL: the caller already wrote the mailbox), release-store seq_in; poll
 * waits until seq_out == seq (or timeout_ns) and copies y out (y may be NULL).
 */
int ll_submit(ll_engine *e, const float *x, int n_rows, uint32_t *seq);
/*
 * Burst submit (no counterpart in the reference, whose mailbox holds one
 * request): posts k batch-1 requests, rows xs[k][in_dim], into the next k slots
 * of the tagged request ring and returns their sequence numbers in seqs[k]
 * (collect each with ll_poll).  Slots 1..k-1 are written first, then seq_in,
 * then slot 0: the device takes slots strictly in order, so when it sees the
 * burst's first request the whole burst is already waiting (a micro-batched
 * engine then takes several per pass).  LL_ERR_BUSY when fewer than k slots
 * are free; on the TickBuffer (one slot) k must be 1.
 */
int ll_submit_many(ll_engine *e, const float *xs, int k, uint32_t *seqs);
int ll_poll(ll_engine *e, uint32_t seq, float *y, uint64_t timeout_ns);
int ll_infer(ll_engine *e, const float *x, int n_rows, float *y, uint64_t timeout_ns);

/* Stop (src/bench_persistent_mbyv_mlp.cu:553-559: stop = 1, bump seq_in, wait). */
int ll_engine_stop(ll_engine *e);
int ll_engine_destroy(ll_engine *e);
int ll_engine_get_info(ll_engine *e, ll_engine_info *info);

/*
 * Closed-loop timing through the mailbox, in C++ so no interpreter sits in the
 * loop: n_req sequential requests, request r taking xs[(r % n_x)] (n_rows rows
 * each); lat_us[r] = host steady_clock time from writing x to reading y
 * (src/bench_persistent_mbyv_mlp.cu:536-548 times the same span minus the x/y
 * copies).  ys (may be NULL) receives every request's output, row-major.
 */
int ll_engine_bench_closed_loop(ll_engine *e, const float *xs, int n_x, int n_req, int n_rows, float *ys,
                                double *lat_us);

/*
 * Closed loop with the request ring kept full (throughput through the C ABI with
 * host buffers; no counterpart in the reference, whose host loop keeps one
 * request outstanding, src/bench_persistent_mbyv_mlp.cu:536-548): n_req batch-1
 * requests, request r taking xs[r % n_x]; a request is posted (x copied into its
 * slot) as soon as one of `depth` slots is free (1 <= depth <= ring_slots) and
 * its reply copied to ys[r] (may be NULL) as soon as it is there, in order.
 * lat_us[r] (may be NULL) = post to reply in microseconds; *elapsed_s = first
 * post to last reply.  Tagged mailbox only.
 */
int ll_engine_bench_ring(ll_engine *e, const float *xs, int n_x, int n_req, int depth, float *ys, double *lat_us,
                         double *elapsed_s);
/* The same closed loop on two host threads: a poster thread (pinned to poster_cpu when
 * >= 0) writes each request into its slot as soon as one of `depth` slots is free, while
 * the calling thread collects the replies in order; sequence numbers and slots follow the
 * same rule as ll_engine_bench_ring.  Needs the kernel to stay up during the run (a relaunch
 * in the middle is reported as a timeout). */
int ll_engine_bench_ring_mt(ll_engine *e, const float *xs, int n_x, int n_req, int depth, float *ys, double *lat_us,
                            double *elapsed_s, int poster_cpu);

/*
 * Device-resident queue: runs n_req sequential requests whose inputs d_x
 * [n_req][n_rows][in_dim] already sit in device memory, writing d_y
 * [n_req][n_rows][out_dim]; each request starts only after the previous one
 * finished (batch-1 latency semantics, no PCIe).  *ms = CUDA-event time of the
 * launch; d_stamps (device, may be NULL) gets a %globaltimer ns stamp per
 * finished request.  The resident mailbox kernel is stopped first.
 */
int ll_engine_run_queue(ll_engine *e, const float *d_x, float *d_y, int n_req, int n_rows, float *ms,
                        unsigned long long *d_stamps);

/*
 * Device timeline of the first n requests of every later launch: d_trace is a
 * device buffer of n * 32 uint64 per request: 16 %globaltimer ns stamps, then
 * the same 16 events as SM clock64 cycles (slot 0
 * request seen, 1 x staged, 2 pushed to peers, 3.. after each layer of the
 * first stage, 11 handoff received by the last stage, 12 gather complete,
 * 13 y written, 14 published, 15 x received by rank 1).  NULL turns it off.
 * The reference's only tracing is -lineinfo (CMakeLists.txt:9).
 */
int ll_engine_set_trace(ll_engine *e, unsigned long long *d_trace, int n);

const char *ll_last_error(void);

/* ---- launch-per-layer kernels (sm_100a), one inference per launch sequence ---- */

/* y = act(W x + b), W row-major [M x K]; replaces ll::dense_warp_rm_kernel (include/ll/dense_warp.cuh:33-90). */
int ll_dense_warp_rm(const float *W, const float *b, const float *x, float *y, int M, int K, int act,
                     void *stream);
/* y = act(W_cm^T x + b_pad), W_cm K-major [K x Mpad]; replaces ll::launch_dense_mbyv_packed
 * (include/ll/dense_mbyv_packed.cuh:53-63). */
int ll_dense_mbyv_packed(const float *W_cm, const float *b_pad, const float *x, float *y, int M, int K, int act,
                         void *stream);
/*
 * MLP forward that allocates nothing (no counterpart in the reference).
 * For callers that cannot call cudaMalloc on their request path -- it may
 * implicitly synchronise the device and take milliseconds -- or whose device
 * memory is owned by another allocator.  Same kernels as ll_layered_mlp's direct
 * path: one ll_dense_warp_rm launch per layer on `stream`, on the current device.
 * d_W / d_b are host arrays of device pointers (fp32, row-major [out x in];
 * d_b may be NULL), d_x / d_y device vectors; batch 1.
 * The hidden activations live in a library-owned static device array of
 * 2 x LL_NOALLOC_MAX_WIDTH floats (64 KB per GPU, held until the process
 * exits); a hidden width above LL_NOALLOC_MAX_WIDTH is rejected with
 * LL_ERR_INVALID_ARG.  The first call on a device looks the array up with
 * cudaGetSymbolAddress; make that first call before any stream capture.
 * All calls share the array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller.  Nothing in
 * the array needs to start at zero: every layer writes all the values the next
 * one reads.
 */
#define LL_NOALLOC_MAX_WIDTH 8192
int ll_mlp_forward_noalloc(const ll_net_desc *net, const float *const *d_W, const float *const *d_b,
                           const float *d_x, float *d_y, void *stream);

/*
 * Batched dense path on the tensor cores (tcgen05 + TMEM), for the batched
 * configurations: an MLP forward over up to max_batch rows as one tensor-core
 * layer kernel per layer (128-row x bn tiles; the K splits of a tile run as one
 * thread-block cluster and add their partials in rank order through an L2 scratch
 * buffer, so results are deterministic), chained with programmatic dependent
 * launch.  No counterpart
 * kernel in the reference, whose batched GEMMs are cuBLAS SGEMM calls
 * (src/bench_cublas_mlp.cu, src/bench_cublas_mlp_graph.cu:119-187); the layer
 * contract y = act(W x + b) and the row-major weight layout are the reference's.
 * Weights: bf16 (uint16 bit patterns) or int8 with per-output-channel fp32
 * scales (y = act(s * (q . x) + b)); every layer shares one type; in_dim and
 * out_dim multiples of 64.  x is fp32 and rounded to bf16; hidden activations
 * are bf16; y is fp32.
 */
#define LL_MAX_LAYERS 24
typedef struct ll_batched_mlp ll_batched_mlp;
typedef struct {
    int32_t bn;          /* output channels per CTA tile: 0 = auto, 64, 128 or 256 */
    int32_t splits;      /* K splits per tile (= cluster size): 0 = auto, else a power of two <= 16 dividing in_dim/64 */
    int32_t pdl;         /* 1 = chain layers with programmatic dependent launch (default) */
    int32_t kernel;      /* 0 = auto; 1 = split-K tiles (128 rows x bn, K split over a cluster);
                            2 = weights-in-TMEM tiles (128 channels x 256 rows, whole K; the weights
                            go global -> registers -> tensor memory as the MMA's A operand, only the
                            rows pass through shared memory);
                            3 = small-batch matrix-by-vector (max_batch <= 32): the whole forward
                            is ONE cooperative launch, one CTA per SM; each CTA holds its row slice
                            of every layer's weights in shared memory and the layers hand off
                            through L2 behind a grid-wide layer barrier (bounded waits).
                            Auto takes 3 when max_batch <= 32 and the slices fit (and bn / splits
                            are not forced), else per layer 2 for >= 96 weights-in-TMEM tiles
                            (stacked batches) and 1 otherwise. */
    uint64_t wait_ns;    /* bound on every device-side wait; 0 = 1 s */
    int32_t graph;       /* 1 = replay the per-layer launches of a forward from a CUDA graph captured
                            on first use (default; recaptured when the pointers or the row count
                            change), so the host enqueues one graph instead of one launch per layer;
                            0 = launch every layer from the host */
    int32_t sm_pairs;    /* kernel 2 tiles on SM pairs: 1 = a layer with an even number of 128-channel
                            tiles runs them as 256-channel tiles of two CTAs, one 2-SM MMA
                            (cta_group::2) reading each CTA's weights from its tensor memory and each
                            CTA's half of the rows from its shared memory, so the rows cross the
                            L2-to-SM crossbar once per pair (measured: 40 % fewer bytes, 3 % slower
                            on stacked config 3); 0 = one CTA per 128-channel tile (default) */
    int32_t reserved[2];
} ll_batched_opts;
typedef struct {
    int32_t n_layers;
    int32_t rows_pad;    /* max_batch rounded up to 256 */
    int32_t bn[LL_MAX_LAYERS];
    int32_t splits[LL_MAX_LAYERS];
    int32_t ctas[LL_MAX_LAYERS];       /* at max_batch rows */
    int32_t smem_bytes[LL_MAX_LAYERS];
    int32_t kind[LL_MAX_LAYERS];       /* 1 split-K tiles, 2 weights-in-TMEM tiles, 3 small-batch
                                          (then bn = output channels per CTA, ctas = SMs) */
} ll_batched_info;
void ll_batched_opts_default(ll_batched_opts *opts);
/* Host-only tiling estimate (no GPU needed): the most CTAs up to one per SM.  ll_batched_mlp_create
 * refines it with the device's cluster occupancy so that every layer runs in one wave;
 * ll_batched_mlp_info reports the tiling actually used. */
int ll_batched_plan(const ll_net_desc *net, const ll_batched_opts *opts, ll_batched_info *info);
int ll_batched_mlp_create(const ll_net_desc *net, const void *const *W, const float *const *b,
                          const float *const *scales, int device, const ll_batched_opts *opts,
                          ll_batched_mlp **out);
/* Enqueue one forward on `stream` (device pointers; x [n_rows x in], y [n_rows x out], fp32;
 * x 16-byte aligned).  Returns launch errors only; ll_batched_mlp_check reports device-side
 * ones.  Forwards of one object run one after another on one stream. */
int ll_batched_mlp_forward(ll_batched_mlp *m, const float *d_x, float *d_y, int n_rows, void *stream);
/* Synchronise `stream` and read the device status word: LL_OK, or LL_ERR_DEVICE_FAULT when a
 * bounded wait ran out (the workspace is then cleared so the next forward starts clean). */
int ll_batched_mlp_check(ll_batched_mlp *m, void *stream);
/* Host buffers: copy x in, forward, check, copy y out (on the object's own stream). */
int ll_batched_mlp_infer(ll_batched_mlp *m, const float *x, float *y, int n_rows);
int ll_batched_mlp_info(ll_batched_mlp *m, ll_batched_info *info);
/* Optional phase trace (device buffer of n >= n_layers * max_ctas * 16 entries, or NULL to stop):
 * every CTA of layer l writes globaltimer stamps at d_trace[(l * max_ctas + cta) * 16 + k],
 * max_ctas = the largest ctas[] of ll_batched_mlp_info; k = 0 entry, 1 previous layer done,
 * 2 first stage landed, 3 last MMA issued, 4 accumulator complete, 5 cluster barrier,
 * 6 partial rows exchanged, 7 end, 8 partial tile staged (split-K only), 9..12 K steps 0..3 ready
 * for the MMA, 13 first stage re-issued, 14 that stage ready, 15 K step 0 converted (int8). */
int ll_batched_mlp_set_trace(ll_batched_mlp *m, unsigned long long *d_trace, size_t n);
int ll_batched_mlp_destroy(ll_batched_mlp *m);

/* Host packing, include/ll/pack_weights.cuh:16-32. */
void ll_pack_rm_to_kmajor_padded(const float *W_rm, size_t M, size_t K, float *W_cm, size_t Mpad);
void ll_pack_bias_padded(const float *b, size_t M, float *b_pad, size_t Mpad);

/*
 * Launch-per-layer MLP object: one ll_dense_warp_rm launch per layer on
 * device-resident weights, optionally captured in a CUDA graph; the comparison
 * path of src/bench_custom_warp_mlp_graph.cu:96-152 and (with pinned copies
 * inside the graph) src/bench_custom_warp_e2e.cu:165-194.
 */
typedef struct ll_layered_mlp ll_layered_mlp;
enum { LL_RUN_DIRECT_KERNEL = 0, LL_RUN_GRAPH_KERNEL = 1, LL_RUN_GRAPH_E2E = 2, LL_RUN_DIRECT_E2E = 3,
       LL_RUN_MAILBOX_TICK = 4 };
int ll_layered_mlp_create(const ll_net_desc *net, const float *const *W, const float *const *b, int device,
                          ll_layered_mlp **out);
/* Times n_req requests in the given LL_RUN_* mode; lat_us[r] per request; y_last gets the last output. */
int ll_layered_mlp_bench(ll_layered_mlp *m, int mode, const float *xs, int n_x, int n_req, float *y_last,
                         double *lat_us);
int ll_layered_mlp_destroy(ll_layered_mlp *m);

/*
 * cuBLAS comparison path: per layer cublasSgemm(OP_T, OP_N, M, 1, K) plus a
 * bias(+ReLU) kernel, direct or captured in a CUDA graph
 * (src/bench_cublas_mlp.cu:119-137, src/bench_cublas_mlp_graph.cu:119-187),
 * e2e with pinned copies, or the mailbox-per-tick structure of
 * src/bench_persistent_cublas_mlp.cu:226-271.  fp32 nets only.
 */
typedef struct ll_cublas_mlp ll_cublas_mlp;
int ll_cublas_mlp_create(const ll_net_desc *net, const float *const *W, const float *const *b, int device,
                         ll_cublas_mlp **out);
int ll_cublas_mlp_bench(ll_cublas_mlp *m, int mode, const float *xs, int n_x, int n_req, float *y_last,
                        double *lat_us);
int ll_cublas_mlp_destroy(ll_cublas_mlp *m);

/* ---- synthetic workload generators (the reference's host_init, src/bench_cublas_mlp.cu:37-43) ---- */

/* std::mt19937(seed) + std::normal_distribution<float>(mean, stddev): bit-identical to host_init. */
int ll_fill_normal(float *out, size_t n, float mean, float stddev, uint32_t seed);
/* std::mt19937(seed) + std::uniform_real_distribution<float>(lo, hi). */
int ll_fill_uniform(float *out, size_t n, float lo, float hi, uint32_t seed);
/*
 * Parameters of a whole net from ONE std::mt19937(seed) stream, drawn in the
 * order W1, b1, W2, b2, ... (W row-major [out x in]); W Xavier-uniform
 * U(+-sqrt(6/(in+out))) or N(0, 1/in); biases U[-0.01, 0.01].
 */
int ll_init_params(const ll_net_desc *net, int init, uint32_t seed, float *const *W, float *const *b);
/* fp32 -> bf16 bit patterns, round to nearest even. */
void ll_f32_to_bf16(const float *in, uint16_t *out, size_t n);
/* Symmetric per-output-channel int8: s[m] = max|W[m,:]|/127, q = clamp(rint(W/s), -127, 127). */
void ll_quantize_int8_rows(const float *W, int m, int k, int8_t *q, float *s);

/* ---- statistics (include/bench_utils.h:140-171, linear-interpolated percentiles) ---- */
typedef struct ll_stats {
    double p50, p90, p99, min, max, mean, sd;
} ll_stats;
void ll_compute_stats(const double *xs, size_t n, ll_stats *out);

/* ---- host-side mailbox protocol on any memory (used by the engine; testable without a GPU) ---- */
/* Bytes of a mailbox for the given dims (header + x + y, rounded to 64). */
size_t ll_mailbox_bytes(int in_dim, int out_dim, int max_batch);
/* Write x (if non-NULL) and n_rows, then release-store seq_in = seq.  On the TickBuffer any
 * seq that differs from the last one posted and from 0 starts a request (the reference's hosts
 * use ++seq; ll_submit uses ll_next_seq). */
void ll_mailbox_post(void *mailbox, int in_dim, const float *x, int n_rows, uint32_t seq, int write_combined);
/* Spin until seq_out == seq (acquire) or timeout; copies n_rows*out_dim floats of y. LL_OK / LL_ERR_TIMEOUT. */
int ll_mailbox_wait(const void *mailbox, int in_dim, int out_dim, int max_batch, uint32_t seq, float *y,
                    int n_rows, uint64_t timeout_ns);
/*
 * Tagged mailbox (mailbox_format 1, batch-1 nets; no counterpart in the reference,
 * whose TickBuffer needs a second PCIe round trip to read x after seq_in and a
 * release fence before seq_out).  Layout: the 16-byte header, then
 * ceil(in_dim/3) x chunks, then ceil(out_dim/3) y chunks; a chunk is 16 bytes
 * {v0, v1, v2, tag} written with one aligned 16-byte store (atomic on x86 CPUs
 * with AVX and for one 16-byte GPU access), tag = the request's sequence number.
 * The device polls the x chunks themselves and takes the request when every tag
 * carries exactly the next sequence number after the last one it served
 * (ll_next_seq: a hand-driven host must number its requests that way; a slot's
 * previous lap holds an older number); it writes the y chunks with relaxed
 * stores and the host waits until every y tag equals its sequence number.
 * The y chunks start on a fresh 64-byte line (ll_tagged_y_offset): no cache
 * line holds both host-written x and device-written y.
 * Limits: in_dim <= 384, out_dim <= 96.
 */
size_t ll_tagged_mailbox_bytes(int in_dim, int out_dim);
/* Byte offset of the first y chunk: the x chunks' end rounded up to 64. */
size_t ll_tagged_y_offset(int in_dim);
void ll_tagged_post(void *mailbox, int in_dim, const float *x, uint32_t seq);
int ll_tagged_wait(const void *mailbox, int in_dim, int out_dim, uint32_t seq, float *y, uint64_t timeout_ns);

/* Next sequence number after seq: skips 0 (idle) and LL_STOP_SEQ. */
uint32_t ll_next_seq(uint32_t seq);

/*
 * Open-loop serving of a Poisson request stream (no counterpart in the reference,
 * whose benches are closed loops).  The stream has n_total requests with
 * exponential gaps of mean 1/rate_per_s (std::mt19937_64(seed)); after each gap
 * a GPU is drawn uniformly from [0, world) from the same generator, so every
 * rank sees the same stream and serves the requests drawn for `rank`, in
 * arrival order, input row (request index % n_x) of xs.  A request is posted
 * when its arrival time has come and a mailbox slot is free (up to ring_slots
 * outstanding on the tagged mailbox, one on the TickBuffer); lat_us[j] (capacity
 * n_total) receives the time from the scheduled arrival of this rank's j-th
 * request to the host seeing its reply, in microseconds.  *n_served = requests
 * of this rank, *elapsed_s = start to the last reply.  Optional outputs (NULL to
 * skip): ys[j][out_dim] = the reply to this rank's j-th request and req_idx[j] =
 * its index in the whole stream (its input row is req_idx[j] % n_x); both have
 * capacity n_total rows.  Batch-1 engines.
 */
int ll_engine_serve_poisson(ll_engine *e, const float *xs, int n_x, int n_total, double rate_per_s, uint64_t seed,
                            int rank, int world, double *lat_us, int *n_served, double *elapsed_s, float *ys,
                            int *req_idx);

/*
 * Weight files (no counterpart in the reference, which generates its weights in
 * process with host_init, src/bench_cublas_mlp.cu:37-43): the net descriptor and
 * its row-major weights (in the net's type), fp32 biases and int8 scales in one
 * little-endian file ("LLWB" v1: 32-byte header, 16-byte layer records, 64-byte
 * aligned sections, FNV-1a 64 checksum of the payload).  b may be NULL (no
 * biases stored); scales are required for int8 nets.  ll_weights_load validates
 * magic, version, dims, sizes and checksum (LL_ERR_BAD_DESC / LL_ERR_UNSUPPORTED);
 * ll_weights_arrays fills n_layers pointers for ll_engine_create and friends,
 * valid until ll_weights_free.
 */
typedef struct ll_weights ll_weights;
int ll_weights_save(const char *path, const ll_net_desc *net, const void *const *W, const float *const *b,
                    const float *const *scales);
int ll_weights_load(const char *path, ll_weights **out);
const ll_net_desc *ll_weights_net(const ll_weights *w);
int ll_weights_arrays(const ll_weights *w, const void **W, const float **b, const float **scales);
void ll_weights_free(ll_weights *w);

/* Library version string. */
const char *ll_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LL_B200_H */
