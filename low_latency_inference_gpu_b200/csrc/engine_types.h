// Plan and control structures shared by the resident-engine host code and
// its kernel.  Plain data only (no CUDA types) so host C++ can build them.
#pragma once
#include <cstdint>

#include "ll_b200.h"

namespace llk {

constexpr int kMaxLayers = 24;
constexpr int kMaxStages = 9;
constexpr int kThreads = 512;  // threads per CTA of the resident kernel
constexpr int kMaxCluster = 16;
constexpr int kTraceSlots = 32;  // per request: 16 %globaltimer ns stamps, then the same 16 events in SM clock64 cycles

// How one layer is spread over the CTAs of its stage's cluster.
enum LayerMode : int32_t {
    LM_REPLICATED = 0,        // every CTA computes all rows (input already local everywhere)
    LM_ROWSPLIT_ALLGATHER = 1, // CTA computes R rows, pushes them into every peer's buffer (DSMEM)
    LM_ROWSPLIT_LOCAL = 2,    // CTA computes R rows, keeps them (the next layer is K-split)
    LM_KSPLIT_GATHER = 3,     // last layer: partial sums over the local K slice, gathered at rank 0
    LM_ROWSPLIT_GATHER = 4,   // last layer: R finished rows per CTA gathered at rank 0
    LM_ROWSPLIT_GLOBAL = 5,   // stage boundary: R rows per CTA written to global memory for the next cluster
};

enum BufId : int32_t { BUF_X = 0, BUF_A = 1, BUF_B = 2, BUF_L = 3, BUF_G = 4, BUF_STAGE = 5, BUF_COUNT = 6 };

enum Mode : int32_t { MODE_MAILBOX = 0, MODE_QUEUE = 1 };

// EXIT_TAGS: a resident small-batch launch used up its 16-bit hand-off tags (relaunched on demand)
enum ExitReason : uint32_t {
    EXIT_NONE = 0, EXIT_STOP = 1, EXIT_IDLE = 2, EXIT_ABORT = 3, EXIT_QUEUE_DONE = 4, EXIT_TAGS = 5
};

enum EngineState : uint32_t { ST_IDLE = 0, ST_LOADING = 1, ST_RUNNING = 2, ST_EXITING = 3, ST_EXITED = 4 };

// Device-side error locations reported in EngineCtrl::err_where.
enum ErrWhere : uint32_t {
    EW_NONE = 0,
    EW_LOAD = 1,         // weight image bulk load
    EW_GATHER = 2,       // rank-0 gather of the last layer
    EW_XFER = 3,         // inter-stage handoff
    EW_QUEUE_GO = 4,     // pipeline sequencing (the first stage waits for the last)
    EW_PEER_POLL = 5,    // a non-leader CTA outlived the leader's idle bound
    EW_DIAG = 6,         // the diagnostic never-completing wait ran out (expected)
    EW_LAYER_BASE = 0x100 // + layer index: all-gather wait of that layer
};

struct LayerDev {
    int32_t mode, act, wtype, lpr_log2;
    int32_t K;      // dot length (padded)
    int32_t M;      // logical output rows of the layer
    int32_t Mp;     // padded output width of the layer's full vector (C*R), or OUTp for K-split
    int32_t R;      // rows computed by each CTA (OUTp for K-split)
    int32_t in_buf, in_ld, out_buf, out_ld;
    uint32_t w_off, b_off, s_off; // byte offsets inside the CTA image (s_off = 0xffffffff: no scales)
    int32_t round_out; // round outputs to bf16 (hidden layers of bf16/int8 nets)
    int32_t pad_;
};

// Host-mapped control block (one per engine).
struct EngineCtrl {
    volatile uint32_t state;
    volatile uint32_t status;
    volatile uint32_t err_where;
    volatile uint32_t served;
    volatile uint32_t exit_reason;
    volatile uint32_t launches;
    volatile uint32_t passes;  // register-resident kernel, at exit: passes over the layers this launch
    volatile uint32_t rows;    // ... and requests taken (more than passes when micro-batched)
    volatile uint32_t pad[8];
};

struct Params {
    ll_tick_header *mb;  // device view of the mailbox
    const float *mb_x;
    float *mb_y;
    EngineCtrl *ctrl;    // device view of the control block
    int32_t mode;
    int32_t mailbox_format;
    int32_t in_dim, out_dim, max_batch, bmax4; // bmax4 = max_batch rounded up to 4
    int32_t in_ld;       // stage-0 X row stride
    int32_t n_layers, n_stages, C;
    int32_t act_bf16;    // inputs / hidden activations are rounded to bf16
    int32_t out_ld_g;    // G row stride (OUTp) for K-split gathers
    LayerDev L[kMaxLayers];
    int32_t stage_first[kMaxStages], stage_last[kMaxStages];
    int32_t stage_in_ld[kMaxStages];
    const uint8_t *image; // per-CTA images, image_stride bytes apart, indexed by blockIdx.x
    uint32_t image_stride;
    uint32_t image_bytes[kMaxStages];
    uint32_t buf_off[BUF_COUNT];
    uint32_t smem_bytes;
    float *xfer;          // [n_stages][xfer_stride] floats; header in xfer_hdr
    uint32_t xfer_stride;
    int32_t xfer_tagged;  // batch-1 pipelines: values handed off as 64-bit words {seq, fp32}
    unsigned *xfer_cnt;   // [n_stages] monotone counters
    unsigned *xfer_hdr;   // [n_stages][2]: seq, n_rows
    unsigned *abort_flag; // global abort / exit signal
    unsigned *q_done;     // queue-mode completion counter (multi-stage)
    uint64_t idle_ns, step_ns, peer_margin_ns;
    uint32_t last_seq;
    // tagged request ring: request n of this launch uses slot (ring_base + n) % ring_slots; the
    // x chunks of consecutive slots are contiguous (ring_xstride_f floats apart, from mb_x), the
    // y chunks of a slot start ring_ystride_f floats after the previous slot's (from mb_y);
    // one slot is the single tagged mailbox
    int32_t ring_slots;
    uint32_t ring_xstride_f, ring_ystride_f;
    uint32_t ring_base;
    int32_t micro_batch;  // register-resident kernel: ring slots taken together (1 = one request)
    int32_t diag_wait_never;
    unsigned long long *trace;  // optional [trace_n][kTraceSlots] timeline of the first requests
    int32_t trace_n;
    // queue mode
    const float *q_x;
    float *q_y;
    int32_t q_n, q_rows;
    unsigned long long *q_stamp;
};

}  // namespace llk
