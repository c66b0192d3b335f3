// Batched dense path: an MLP forward over many rows as one tcgen05 layer kernel
// per layer (tc_layer.cuh), chained with programmatic dependent launch so each
// layer's set-up overlaps the previous layer's tail.  Weights stay resident in
// HBM in their own type (int8 + per-channel scales, or bf16); activations move
// between layers as bf16 row-major buffers padded to 128 rows.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.h"
#include "gemv_net.cuh"
#include "gemv_plan.h"
#include "tc_layer.cuh"
#include "tc_swap.cuh"
#include "tc_swap2.cuh"

using namespace llk;

namespace {

constexpr int kMaxSplitCTAs = 148;  // one CTA per SM

enum { kKindSplitK = 1, kKindWeightsInTmem = 2, kKindGemv = 3 };

constexpr int kGvPlanCtas = 148;                   // SMs assumed by the host-only plan (B200)

struct LayerRun {
    int kind = kKindSplitK;
    int bn = 256, splits = 1, ctas = 0, smem = 0;
    bool pair = false;  // weights-in-TMEM tiles on SM pairs (2-SM MMA; clusters of 2 along x)
    int K = 0, N = 0, act = 0, out_f32 = 0;
    const void *kfn = nullptr;
    const void *w = nullptr;  // device weights (weights-in-TMEM kernel)
    TcLayerParams p{};
};

// Weights-in-TMEM tiles (128 channels x 256 rows, K whole) for a layer when there are
// enough of them to fill most of the GPU; otherwise the split-K tiles.  The rule uses
// shapes only, so the host-side plan and the device agree.
int layer_kind(int N, int rows_pad, const ll_batched_opts *o)
{
    if (o && o->kernel)
        return (o->kernel == kKindWeightsInTmem && N % kSwChan == 0 && rows_pad % kSwRows == 0) ? kKindWeightsInTmem
                                                                                                : kKindSplitK;
    const int tiles = (N % kSwChan == 0 && rows_pad % kSwRows == 0) ? (N / kSwChan) * (rows_pad / kSwRows) : 0;
    return tiles >= 96 ? kKindWeightsInTmem : kKindSplitK;
}

// kKindGemv for the whole net (auto for <= 32 rows when it fits, or forced), else 0.
int net_kind(const ll_net_desc *net, const ll_batched_opts *o, int G)
{
    const int forced = o ? o->kernel : 0;
    const bool tiles_forced = o && (o->bn || o->splits);
    if (forced == kKindGemv || (forced == 0 && !tiles_forced && gemv_fits(net, G)))
        return kKindGemv;
    return 0;
}

template <int BN, bool I8>
constexpr int stages_for()
{
    // as many stages as fit beside the exchange region: more bytes in flight per SM
    return I8 ? (BN == 256 ? 3 : BN == 128 ? 5 : 6) : (BN == 256 ? 4 : BN == 128 ? 6 : 8);
}

template <int BN, bool I8>
const void *kernel_for(int &smem)
{
    constexpr int ST = stages_for<BN, I8>();
    smem = TcSmem<BN, I8, ST>::ALLOC;
    return reinterpret_cast<const void *>(&ll_tc_layer_kernel<BN, I8, ST>);
}

const void *pick_kernel(int bn, bool i8, int &smem)
{
    if (i8)
        return bn == 256 ? kernel_for<256, true>(smem) : bn == 128 ? kernel_for<128, true>(smem)
                                                                  : kernel_for<64, true>(smem);
    return bn == 256 ? kernel_for<256, false>(smem) : bn == 128 ? kernel_for<128, false>(smem)
                                                               : kernel_for<64, false>(smem);
}

// Largest power of two <= cap (and <= 16, the largest cluster) that divides n.
// The 256-wide tile has no shared memory left for the split-K exchange.
bool can_split(int bn, bool i8)
{
    if (bn == 256)
        return i8 ? TcSmem<256, true, stages_for<256, true>()>::CAN_SPLIT
                  : TcSmem<256, false, stages_for<256, false>()>::CAN_SPLIT;
    if (bn == 128)
        return i8 ? TcSmem<128, true, stages_for<128, true>()>::CAN_SPLIT
                  : TcSmem<128, false, stages_for<128, false>()>::CAN_SPLIT;
    return i8 ? TcSmem<64, true, stages_for<64, true>()>::CAN_SPLIT
              : TcSmem<64, false, stages_for<64, false>()>::CAN_SPLIT;
}

int split_at_most(int n, int cap)
{
    for (int d = 16; d >= 1; d >>= 1)
        if (d <= cap && n % d == 0)
            return d;
    return 1;
}

// Tile width and split count of one layer: the most CTAs up to one per SM, each
// with at least two 64-deep K steps; ties go to the wider tile (fewer X re-reads).
// The splits of a tile run as one cluster, so a split count is a power of two <= 16.
void plan_layer(int K, int N, int rows, bool i8, const ll_batched_opts *o, int &bn, int &splits)
{
    const int mt = (rows + kTcRows - 1) / kTcRows;
    int best_bn = 0, best_s = 1, best_ctas = -1;
    for (int cand : {256, 128, 64}) {
        if (N % cand != 0 || (o && o->bn && o->bn != cand))
            continue;
        const int tiles = (N / cand) * mt;
        int s;
        if (o && o->splits > 0)
            s = o->splits;
        else
            s = can_split(cand, i8)
                    ? split_at_most(K / kTcK, std::min(std::max(1, kMaxSplitCTAs / tiles), std::max(1, K / 128)))
                    : 1;
        const int ctas = tiles * s;
        if (ctas > best_ctas) {
            best_ctas = ctas;
            best_bn = cand;
            best_s = s;
        }
    }
    bn = best_bn;
    splits = best_s;
}

int validate(const ll_net_desc *net, const ll_batched_opts *o)
{
    if (!net || net->n_layers < 1 || net->n_layers > LL_MAX_LAYERS || !net->layers) {
        llh::set_error("batched net: n_layers must be in [1, %d]", LL_MAX_LAYERS);
        return LL_ERR_BAD_DESC;
    }
    if (net->max_batch < 1 || net->max_batch > 65536) {
        llh::set_error("batched net: max_batch must be in [1, 65536]");
        return LL_ERR_BAD_DESC;
    }
    const int wt = net->layers[0].wtype;
    if (wt != LL_W_BF16 && wt != LL_W_I8) {
        llh::set_error("batched net: weights must be bf16 or int8 (the tensor-core path)");
        return LL_ERR_BAD_DESC;
    }
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        if (d.wtype != wt) {
            llh::set_error("layer %d: all layers must share one weight type", l);
            return LL_ERR_BAD_DESC;
        }
        if (d.in_dim < kTcK || d.in_dim % kTcK != 0 || d.in_dim > 65536) {
            llh::set_error("layer %d: in_dim %d must be a positive multiple of 64", l, d.in_dim);
            return LL_ERR_BAD_DESC;
        }
        if (d.out_dim < 64 || d.out_dim % 64 != 0 || d.out_dim > 65536) {
            llh::set_error("layer %d: out_dim %d must be a positive multiple of 64", l, d.out_dim);
            return LL_ERR_BAD_DESC;
        }
        if (l > 0 && net->layers[l - 1].out_dim != d.in_dim) {
            llh::set_error("layer %d: in_dim %d != previous out_dim %d", l, d.in_dim, net->layers[l - 1].out_dim);
            return LL_ERR_BAD_DESC;
        }
        if (d.act < LL_ACT_IDENTITY || d.act > LL_ACT_GELU) {
            llh::set_error("layer %d: unknown activation %d", l, d.act);
            return LL_ERR_BAD_DESC;
        }
    }
    if (o && ((o->bn != 0 && o->bn != 64 && o->bn != 128 && o->bn != 256) || o->splits < 0 || o->splits > 16 ||
              (o->splits & (o->splits - 1)) != 0 || o->kernel < 0 || o->kernel > kKindGemv)) {
        llh::set_error("batched opts: bn must be 0/64/128/256, splits 0 (auto) or a power of two <= 16, kernel 0..3");
        return LL_ERR_INVALID_ARG;
    }
    if (o && o->kernel == kKindGemv && !gemv_fits(net, kGvPlanCtas)) {
        llh::set_error("batched opts: the small-batch kernel takes <= %d rows whose weight slices and staged "
                       "rows fit one SM's shared memory",
                       kGvMaxRows);
        return LL_ERR_INVALID_ARG;
    }
    if (o && o->splits > 0) {
        for (int l = 0; l < net->n_layers; ++l)
            if ((net->layers[l].in_dim / kTcK) % o->splits != 0) {
                llh::set_error("layer %d: splits %d must divide in_dim/64", l, o->splits);
                return LL_ERR_INVALID_ARG;
            }
    }
    if (o && o->bn && o->splits > 1 && !can_split(o->bn, wt == LL_W_I8)) {
        llh::set_error("batched opts: a %d-wide tile cannot be split (no shared memory for the exchange)", o->bn);
        return LL_ERR_INVALID_ARG;
    }
    if (o && o->bn) {
        for (int l = 0; l < net->n_layers; ++l)
            if (net->layers[l].out_dim % o->bn != 0) {
                llh::set_error("layer %d: out_dim %d is not a multiple of bn %d", l, net->layers[l].out_dim, o->bn);
                return LL_ERR_INVALID_ARG;
            }
    }
    return LL_OK;
}

void fill_info(const ll_net_desc *net, const ll_batched_opts *o, ll_batched_info *info, int G = kGvPlanCtas)
{
    std::memset(info, 0, sizeof(*info));
    const int rows_pad = (int)llh::round_up((size_t)net->max_batch, kSwRows);
    info->n_layers = net->n_layers;
    info->rows_pad = rows_pad;
    const bool i8 = net->layers[0].wtype == LL_W_I8;
    if (net_kind(net, o, G) == kKindGemv) {
        GemvLayout g;
        gemv_layout(net, G, g);
        for (int l = 0; l < net->n_layers; ++l) {
            info->kind[l] = kKindGemv;
            info->bn[l] = g.rmax[l];  // output channels per CTA
            info->splits[l] = 1;
            info->ctas[l] = G;
            info->smem_bytes[l] = (int)g.smem(gemv_bp(net->max_batch));
        }
        return;
    }
    for (int l = 0; l < net->n_layers; ++l) {
        int bn, s, smem;
        info->kind[l] = layer_kind(net->layers[l].out_dim, rows_pad, o);
        if (info->kind[l] == kKindWeightsInTmem) {
            info->bn[l] = kSwChan;
            info->splits[l] = 1;
            info->ctas[l] = (net->layers[l].out_dim / kSwChan) * (rows_pad / kSwRows);
            info->smem_bytes[l] = i8 ? TcSwapSmem<true>::ALLOC : TcSwapSmem<false>::ALLOC;
            continue;
        }
        plan_layer(net->layers[l].in_dim, net->layers[l].out_dim, net->max_batch, i8, o, bn, s);
        pick_kernel(bn, i8, smem);
        info->bn[l] = bn;
        info->splits[l] = s;
        info->ctas[l] = (net->layers[l].out_dim / bn) * ((net->max_batch + kTcRows - 1) / kTcRows) * s;
        info->smem_bytes[l] = smem;
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D row-major tensor map: inner dim `cols` elements, `rows` rows, box {64, box_rows}.
bool make_map(CUtensorMap *m, CUtensorMapDataType t, int esize, const void *base, int cols, int rows, int box_rows,
              CUtensorMapSwizzle swizzle)
{
    auto fn = encode_fn();
    if (!fn)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * (cuuint64_t)esize};
    cuuint32_t box[2] = {(cuuint32_t)kTcK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, t, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D view of a row-major [rows][cols] matrix as {64, rows, cols / 64} (x = position in a
// 64-wide column block, y = row, z = block), box {64, box_rows, group}: one load brings
// `group` consecutive column blocks of box_rows rows, each block's tile contiguous.
bool make_map_grouped(CUtensorMap *m, CUtensorMapDataType t, int esize, const void *base, int cols, int rows,
                      int box_rows, int group, CUtensorMapSwizzle swizzle)
{
    auto fn = encode_fn();
    if (!fn)
        return false;
    cuuint64_t dims[3] = {(cuuint64_t)kTcK, (cuuint64_t)rows, (cuuint64_t)(cols / kTcK)};
    cuuint64_t strides[2] = {(cuuint64_t)cols * (cuuint64_t)esize, (cuuint64_t)kTcK * (cuuint64_t)esize};
    cuuint32_t box[3] = {(cuuint32_t)kTcK, (cuuint32_t)box_rows, (cuuint32_t)group};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, t, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 rows -> bf16 (round to nearest even) into the padded layer-0 buffer, four values
// per thread and step (16-byte loads, 8-byte stores; n4 = n / 4, n a multiple of 64).
__global__ void to_bf16_kernel(const float4 *__restrict__ x, uint2 *__restrict__ out, size_t n4)
{
    griddep_wait();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = __ldg(x + i);
        const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        out[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
    }
    griddep_launch_dependents();
}

int max_active_clusters(const void *kfn, int smem, int S)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, (unsigned)S);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute ca[1];
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = 1;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = (unsigned)S;
    cfg.attrs = ca;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// On the device: the (bn, splits) with the most CTAs such that every cluster of
// the layer is resident at once (one wave; the occupancy query knows how many
// clusters of S CTAs the GPCs can hold), each split at least two 64-deep K steps.
// Ties go to the wider tile.  Forced options are taken as given.
bool choose_tiling(int K, int N, int rows, bool i8, const ll_batched_opts *o, LayerRun &r)
{
    const int mt = (rows + kTcRows - 1) / kTcRows;
    int best = -1;
    for (int bn : {256, 128, 64}) {
        if (N % bn != 0 || (o && o->bn && o->bn != bn))
            continue;
        int smem = 0;
        const void *kfn = pick_kernel(bn, i8, smem);
        if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
            cudaFuncSetAttribute(kfn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
            return false;
        const int tiles = (N / bn) * mt;
        for (int S = 16; S >= 1; S >>= 1) {
            if (o && o->splits && o->splits != S)
                continue;
            if ((K / kTcK) % S != 0 || (!(o && o->splits) && S > 1 && K / S < 128) || (S > 1 && !can_split(bn, i8)))
                continue;
            const int fit = max_active_clusters(kfn, smem, S);
            if (fit < 1)
                continue;
            if (!(o && (o->splits || o->bn)) && tiles > fit)
                continue;  // would need a second wave
            const int ctas = tiles * S;
            if (ctas > best) {
                best = ctas;
                r.bn = bn;
                r.splits = S;
                r.ctas = ctas;
                r.smem = smem;
                r.kfn = kfn;
            }
        }
    }
    if (best < 0 && !(o && (o->splits || o->bn))) {  // nothing fits one wave: smallest legal grid
        int smem = 0;
        const int bn = N % 256 == 0 ? 256 : N % 128 == 0 ? 128 : 64;
        r.kfn = pick_kernel(bn, i8, smem);
        r.bn = bn;
        r.splits = 1;
        r.ctas = (N / bn) * mt;
        r.smem = smem;
        best = r.ctas;
    }
    return best > 0;
}

}  // namespace

struct ll_batched_mlp {
    int device = 0;
    int n_layers = 0, in_dim = 0, out_dim = 0, max_rows = 0, rows_pad = 0, wtype = 0;
    std::vector<void *> d_w;
    std::vector<float *> d_b, d_s;
    __nv_bfloat16 *act[2] = {nullptr, nullptr};
    float *out_pad = nullptr;  // fp32 [rows_pad x out] for the last layer
    unsigned *status = nullptr;
    std::vector<LayerRun> runs;
    int max_ctas = 0;
    cudaStream_t own = nullptr;  // non-blocking stream for ll_batched_mlp_infer
    int pdl = 1;
    unsigned long long wait_ns = 1000ull * 1000 * 1000;
    // small-batch kernel (kKindGemv): one cooperative launch per forward
    bool gemv = false;
    int sms = 0;
    GemvLayout gl;
    GemvNetParams gp{};
    const void *gv_kfn[6] = {};   // by batch rows 1, 2, 4, 8, 16, 32
    uint32_t *hand[2] = {};       // hand-off words [32][widest layer]
    uint8_t *img = nullptr;       // per-CTA shared-memory images (biases, scales, weight slices)
    size_t hand_bytes = 0;
    uint32_t tag_next = 1;        // tag of the next tagged forward's layer 0
    float *scratch = nullptr;     // split-K partial tiles (exchange through L2)
    unsigned *cnt = nullptr;      // arrival counters of the counted hand-off
    unsigned epoch = 0;           // counted forwards since the counters were cleared
    // tensor-core path: the last forward's launches as a CUDA graph, and what it was captured for
    int use_graph = 1;
    cudaGraphExec_t gexec = nullptr;
    const float *g_x = nullptr;
    float *g_y = nullptr;
    int g_rows = 0;
};

namespace {

void destroy_all(ll_batched_mlp *m)
{
    if (!m)
        return;
    cudaSetDevice(m->device);
    for (void *p : m->d_w)
        cudaFree(p);
    for (float *p : m->d_b)
        cudaFree(p);
    for (float *p : m->d_s)
        cudaFree(p);
    cudaFree(m->act[0]);
    cudaFree(m->act[1]);
    cudaFree(m->out_pad);
    cudaFree(m->status);
    cudaFree(m->hand[0]);
    cudaFree(m->cnt);
    cudaFree(m->scratch);
    if (m->gexec)
        cudaGraphExecDestroy(m->gexec);
    cudaFree(m->img);
    cudaFree(m->hand[1]);
    if (m->own)
        cudaStreamDestroy(m->own);
    delete m;
}

}  // namespace

namespace {
int enqueue_tc(ll_batched_mlp *m, const float *d_x, float *d_y, int n_rows, cudaStream_t st);
}  // namespace

extern "C" {

void ll_batched_opts_default(ll_batched_opts *o)
{
    if (!o)
        return;
    std::memset(o, 0, sizeof(*o));
    o->pdl = 1;
    o->graph = 1;
}

int ll_batched_plan(const ll_net_desc *net, const ll_batched_opts *opts, ll_batched_info *info)
{
    if (!info)
        return LL_ERR_INVALID_ARG;
    int rc = validate(net, opts);
    if (rc)
        return rc;
    fill_info(net, opts, info);
    return LL_OK;
}

int ll_batched_mlp_create(const ll_net_desc *net, const void *const *W, const float *const *b,
                          const float *const *scales, int device, const ll_batched_opts *opts, ll_batched_mlp **out)
{
    if (!out || !W)
        return LL_ERR_INVALID_ARG;
    *out = nullptr;
    int rc = validate(net, opts);
    if (rc)
        return rc;
    const bool i8 = net->layers[0].wtype == LL_W_I8;
    for (int l = 0; l < net->n_layers; ++l) {
        if (!W[l] || (i8 && (!scales || !scales[l]))) {
            llh::set_error("layer %d: weights%s missing", l, i8 ? " or scales" : "");
            return LL_ERR_INVALID_ARG;
        }
    }
    if (!encode_fn()) {
        llh::set_error("cuTensorMapEncodeTiled is not available from the driver");
        return LL_ERR_CUDA;
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms < 1) {
        cudaGetLastError();
        llh::set_error("device %d: cannot read the SM count", device);
        return LL_ERR_CUDA;
    }
    ll_batched_info info;
    fill_info(net, opts, &info, sms);

    auto *m = new ll_batched_mlp();
    m->device = device;
    m->n_layers = net->n_layers;
    m->in_dim = net->layers[0].in_dim;
    m->out_dim = net->layers[net->n_layers - 1].out_dim;
    m->max_rows = net->max_batch;
    m->rows_pad = info.rows_pad;
    m->wtype = net->layers[0].wtype;
    m->pdl = opts ? opts->pdl : 1;
    if (opts && opts->wait_ns)
        m->wait_ns = opts->wait_ns;
    m->sms = sms;
    m->gemv = info.kind[0] == kKindGemv;
    m->use_graph = opts ? opts->graph : 1;
    auto fail = [&](int code) {
        destroy_all(m);
        return code;
    };
#define LLB_TRY(call)                                                                                        \
    do {                                                                                                     \
        cudaError_t _e = (call);                                                                             \
        if (_e != cudaSuccess) {                                                                             \
            llh::set_error("%s failed: %s", #call, cudaGetErrorString(_e));                                   \
            return fail(LL_ERR_CUDA);                                                                        \
        }                                                                                                    \
    } while (0)
    LLB_TRY(cudaSetDevice(device));
    LLB_TRY(cudaStreamCreateWithFlags(&m->own, cudaStreamNonBlocking));
    int max_w = m->in_dim;
    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        max_w = std::max(max_w, d.out_dim);
        const size_t welems = (size_t)d.in_dim * (size_t)d.out_dim;
        void *dw = nullptr;
        LLB_TRY(cudaMalloc(&dw, welems * (i8 ? 1 : 2)));
        m->d_w.push_back(dw);
        LLB_TRY(cudaMemcpy(dw, W[l], welems * (i8 ? 1 : 2), cudaMemcpyHostToDevice));
        float *db = nullptr;
        LLB_TRY(cudaMalloc(&db, sizeof(float) * d.out_dim));
        m->d_b.push_back(db);
        if (b && b[l])
            LLB_TRY(cudaMemcpy(db, b[l], sizeof(float) * d.out_dim, cudaMemcpyHostToDevice));
        else
            LLB_TRY(cudaMemset(db, 0, sizeof(float) * d.out_dim));
        float *ds = nullptr;
        if (i8) {
            LLB_TRY(cudaMalloc(&ds, sizeof(float) * d.out_dim));
            LLB_TRY(cudaMemcpy(ds, scales[l], sizeof(float) * d.out_dim, cudaMemcpyHostToDevice));
        }
        m->d_s.push_back(ds);
    }
    const size_t act_elems = (size_t)m->rows_pad * (size_t)max_w;
    for (int i = 0; i < 2; ++i) {
        LLB_TRY(cudaMalloc(&m->act[i], act_elems * 2));
        LLB_TRY(cudaMemset(m->act[i], 0, act_elems * 2));  // padded rows stay zero
    }
    LLB_TRY(cudaMalloc(&m->out_pad, sizeof(float) * (size_t)m->rows_pad * m->out_dim));
    LLB_TRY(cudaMalloc(&m->status, sizeof(unsigned)));
    LLB_TRY(cudaMemset(m->status, 0, sizeof(unsigned)));

    if (m->gemv) {
        gemv_layout(net, sms, m->gl);
        const size_t need = m->gl.smem(gemv_bp(m->max_rows));
        if (need > kGvSmemLimit) {
            llh::set_error("small-batch kernel: %zu bytes of shared memory per SM needed", need);
            return fail(LL_ERR_BAD_DESC);
        }
        m->hand_bytes = sizeof(uint32_t) * kGvTagRows * (size_t)max_w;
        for (int i = 0; i < 2; ++i) {
            LLB_TRY(cudaMalloc(&m->hand[i], m->hand_bytes));
            LLB_TRY(cudaMemset(m->hand[i], 0, m->hand_bytes));  // tag 0: never written
        }
        LLB_TRY(cudaMalloc(&m->cnt, sizeof(unsigned) * kGvCntStride * (size_t)net->n_layers));
        LLB_TRY(cudaMemset(m->cnt, 0, sizeof(unsigned) * kGvCntStride * (size_t)net->n_layers));
        // per-CTA images: the CTA's bias (+ scale) slices and weight slices, laid out
        // exactly as the front of its shared memory, so two bulk copies load them
        const std::vector<uint8_t> img = gemv_pack_images(net, W, b, scales, sms, m->gl);
        LLB_TRY(cudaMalloc(&m->img, img.size()));
        LLB_TRY(cudaMemcpy(m->img, img.data(), img.size(), cudaMemcpyHostToDevice));
        GemvNetParams &g = m->gp;
        gemv_static_params(net, m->gl, m->img, g);
        g.hand[0] = m->hand[0];
        g.hand[1] = m->hand[1];
        g.act[0] = m->act[0];
        g.act[1] = m->act[1];
        g.cnt = m->cnt;
        g.status = m->status;
        g.wait_ns = m->wait_ns;
        const void *k8[6] = {reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 1, 1>),
                             reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 1, 2>),
                             reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 1, 4>),
                             reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 2, 4>),
                             reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 4, 4>),
                             reinterpret_cast<const void *>(&ll_gemv_net_kernel<true, 8, 4>)};
        const void *k16[6] = {reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 1, 1>),
                              reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 1, 2>),
                              reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 1, 4>),
                              reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 2, 4>),
                              reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 4, 4>),
                              reinterpret_cast<const void *>(&ll_gemv_net_kernel<false, 8, 4>)};
        const int top = 31 - __builtin_clz((unsigned)gemv_bp(m->max_rows));
        for (int i = 0; i <= top; ++i) {  // the variants of up to max_batch rows
            m->gv_kfn[i] = i8 ? k8[i] : k16[i];
            LLB_TRY(cudaFuncSetAttribute(m->gv_kfn[i], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)m->gl.smem(1 << i)));
        }
        int per_sm = 0;
        LLB_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, m->gv_kfn[top], kGvThreads,
                                                              m->gl.smem(gemv_bp(m->max_rows))));
        if (per_sm < 1) {
            llh::set_error("small-batch kernel: a CTA does not fit one SM");
            return fail(LL_ERR_BAD_DESC);
        }
        for (int l = 0; l < net->n_layers; ++l) {
            LayerRun r;
            r.kind = kKindGemv;
            r.bn = info.bn[l];
            r.splits = 1;
            r.ctas = sms;
            r.smem = info.smem_bytes[l];
            r.K = net->layers[l].in_dim;
            r.N = net->layers[l].out_dim;
            r.act = net->layers[l].act;
            r.out_f32 = (l + 1 == net->n_layers);
            r.w = m->d_w[l];
            m->runs.push_back(r);
        }
        m->max_ctas = sms;
        *out = m;
        return LL_OK;
    }

    for (int l = 0; l < net->n_layers; ++l) {
        const ll_layer_desc &d = net->layers[l];
        LayerRun r;
        r.bn = info.bn[l];
        r.splits = info.splits[l];
        r.ctas = info.ctas[l];
        r.K = d.in_dim;
        r.N = d.out_dim;
        r.act = d.act;
        r.out_f32 = (l + 1 == net->n_layers);
        r.kind = info.kind[l];
        r.w = m->d_w[l];
        if (r.kind == kKindWeightsInTmem) {
            r.bn = kSwChan;
            r.splits = 1;
            r.ctas = info.ctas[l];
            r.pair = (d.out_dim / kSwChan) % 2 == 0 && opts && opts->sm_pairs > 0;
            if (r.pair) {
                r.smem = i8 ? TcSwap2Smem<true>::ALLOC : TcSwap2Smem<false>::ALLOC;
                r.kfn = i8 ? reinterpret_cast<const void *>(&ll_tc_swap2_kernel<true>)
                           : reinterpret_cast<const void *>(&ll_tc_swap2_kernel<false>);
            } else {
                r.smem = i8 ? TcSwapSmem<true>::ALLOC : TcSwapSmem<false>::ALLOC;
                r.kfn = i8 ? reinterpret_cast<const void *>(&ll_tc_swap_kernel<true>)
                           : reinterpret_cast<const void *>(&ll_tc_swap_kernel<false>);
            }
            LLB_TRY(cudaFuncSetAttribute(r.kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, r.smem));
        } else if (!choose_tiling(d.in_dim, d.out_dim, m->max_rows, i8, opts, r)) {
            llh::set_error("layer %d: no tile / cluster shape can be scheduled on this device", l);
            return fail(LL_ERR_BAD_DESC);
        }
        TcLayerParams &p = r.p;
        const bool swk = r.kind == kKindWeightsInTmem;
        const int x_box = swk ? (r.pair ? kSw2Half : kSwRows) : kTcRows;
        // weights: bf16 128-byte swizzled (the MMA operand layout, or conflict-free row reads);
        // int8 unswizzled for the split-K converters, 64-byte swizzled for the row reads of
        // the weights-in-TMEM converters
        const CUtensorMapSwizzle wsw = !i8 ? CU_TENSOR_MAP_SWIZZLE_128B
                                           : swk ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
        const CUtensorMapDataType wt = i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        const bool wmap_ok =
            swk ? make_map_grouped(&p.tm_w, wt, i8 ? 1 : 2, m->d_w[l], d.in_dim, d.out_dim, r.bn,
                                   i8 ? sw_wgroup<true>() : sw_wgroup<false>(), wsw)
                : make_map(&p.tm_w, wt, i8 ? 1 : 2, m->d_w[l], d.in_dim, d.out_dim, r.bn, wsw);
        // SM pairs load kSw2XG K blocks of their half of the rows per tensor load (a 3-D view of X)
        const bool xmap_ok =
            r.pair ? make_map_grouped(&p.tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m->act[l & 1], d.in_dim,
                                      m->rows_pad, x_box, kSw2XG, CU_TENSOR_MAP_SWIZZLE_128B)
                   : make_map(&p.tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m->act[l & 1], d.in_dim, m->rows_pad, x_box,
                              CU_TENSOR_MAP_SWIZZLE_128B);
        if (!xmap_ok || !wmap_ok) {
            llh::set_error("layer %d: tensor map encoding failed", l);
            return fail(LL_ERR_CUDA);
        }
        p.bias = m->d_b[l];
        p.scale = m->d_s[l];
        p.out = r.out_f32 ? static_cast<void *>(m->out_pad) : static_cast<void *>(m->act[(l + 1) & 1]);
        p.status = m->status;
        p.K = d.in_dim;
        p.N = d.out_dim;
        p.k_chunk = d.in_dim / r.splits;
        p.splits = r.splits;
        p.act = d.act;
        p.out_f32 = r.out_f32;
        p.wait_ns = m->wait_ns;
        p.trace = nullptr;
        p.scratch = nullptr;
        m->max_ctas = std::max(m->max_ctas, r.ctas);
        m->runs.push_back(r);
    }
    // split-K layers exchange their partial tiles through one L2 scratch buffer (layers run
    // one after another: a layer writes it only after the previous one completed)
    size_t scratch_bytes = 0;
    for (const LayerRun &r : m->runs)
        if (r.kind == kKindSplitK && r.splits > 1)
            scratch_bytes = std::max(scratch_bytes, (size_t)r.ctas * kTcRows * (size_t)r.bn * sizeof(float));
    if (scratch_bytes) {
        LLB_TRY(cudaMalloc(&m->scratch, scratch_bytes));
        for (LayerRun &r : m->runs)
            if (r.kind == kKindSplitK && r.splits > 1)
                r.p.scratch = m->scratch;
    }
#undef LLB_TRY
    *out = m;
    return LL_OK;
}

int ll_batched_mlp_forward(ll_batched_mlp *m, const float *d_x, float *d_y, int n_rows, void *stream)
{
    if (!m || !d_x || !d_y || n_rows < 1 || n_rows > m->max_rows) {
        llh::set_error("batched forward: bad arguments (n_rows must be in [1, max_batch])");
        return LL_ERR_INVALID_ARG;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    LL_CUDA_TRY(cudaSetDevice(m->device));
    if (reinterpret_cast<uintptr_t>(d_x) % 16 != 0) {  // both paths read x 16 bytes at a time
        llh::set_error("batched forward: x must be 16-byte aligned");
        return LL_ERR_INVALID_ARG;
    }
    if (m->gemv) {
        const int bp = gemv_bp(n_rows);
        const int idx = 31 - __builtin_clz((unsigned)bp);
        const bool tagged = bp <= kGvTagRows;
        if (tagged && m->tag_next + (uint32_t)m->n_layers > kGvTagLimit) {
            // the 16-bit tags would wrap: clear the words so no stale one can match again
            for (int i = 0; i < 2; ++i)
                LL_CUDA_TRY(cudaMemsetAsync(m->hand[i], 0, m->hand_bytes, st));
            m->tag_next = 1;
        }
        GemvNetParams g = m->gp;
        g.n_rows = n_rows;
        g.x = d_x;
        g.y = d_y;
        g.tag_base = m->tag_next;
        g.epoch = m->epoch + 1u;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)m->sms, 1, 1);
        cfg.blockDim = dim3(kGvThreads, 1, 1);
        cfg.dynamicSmemBytes = m->gl.smem(bp);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the layer barrier needs all of them
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        void *args[] = {&g};
        LL_CUDA_TRY(cudaLaunchKernelExC(&cfg, m->gv_kfn[idx], args));
        if (tagged)  // advanced only once the launch is in the stream
            m->tag_next += (uint32_t)m->n_layers;
        else
            m->epoch = g.epoch;
        return LL_OK;
    }
    if (m->use_graph) {
        if (!m->gexec || m->g_x != d_x || m->g_y != d_y || m->g_rows != n_rows) {
            // capture on the object's own stream (the caller's may be the legacy default
            // stream, which cannot be captured); the graph then runs on the caller's stream
            if (m->gexec) {
                cudaGraphExecDestroy(m->gexec);
                m->gexec = nullptr;
            }
            LL_CUDA_TRY(cudaStreamBeginCapture(m->own, cudaStreamCaptureModeThreadLocal));
            const int rc = enqueue_tc(m, d_x, d_y, n_rows, m->own);
            cudaGraph_t graph = nullptr;
            const cudaError_t ec = cudaStreamEndCapture(m->own, &graph);
            if (rc != LL_OK || ec != cudaSuccess) {
                if (graph)
                    cudaGraphDestroy(graph);
                if (rc == LL_OK)
                    llh::set_error("batched forward: graph capture failed: %s", cudaGetErrorString(ec));
                return rc != LL_OK ? rc : LL_ERR_CUDA;
            }
            const cudaError_t ei = cudaGraphInstantiate(&m->gexec, graph, 0);
            cudaGraphDestroy(graph);
            if (ei != cudaSuccess) {
                m->gexec = nullptr;
                llh::set_error("batched forward: graph instantiation failed: %s", cudaGetErrorString(ei));
                return LL_ERR_CUDA;
            }
            m->g_x = d_x;
            m->g_y = d_y;
            m->g_rows = n_rows;
        }
        LL_CUDA_TRY(cudaGraphLaunch(m->gexec, st));
        return LL_OK;
    }
    return enqueue_tc(m, d_x, d_y, n_rows, st);
}

}  // extern "C"

namespace {

// The tensor-core forward's launches: input rows to bf16, one kernel per layer (chained
// with programmatic dependent launch), the caller's rows out of the padded output.
int enqueue_tc(ll_batched_mlp *m, const float *d_x, float *d_y, int n_rows, cudaStream_t st)
{
    const size_t n4 = (size_t)n_rows * m->in_dim / 4;  // in_dim is a multiple of 64
    to_bf16_kernel<<<(unsigned)std::min<size_t>((n4 + 255) / 256, 1184), 256, 0, st>>>(
        reinterpret_cast<const float4 *>(d_x), reinterpret_cast<uint2 *>(m->act[0]), n4);
    LL_CUDA_TRY(cudaGetLastError());
    const int mt = (n_rows + kTcRows - 1) / kTcRows;
    const int mt_sw = (n_rows + kSwRows - 1) / kSwRows;
    for (LayerRun &r : m->runs) {
        cudaLaunchConfig_t cfg = {};
        const bool sw = r.kind == kKindWeightsInTmem;
        cfg.gridDim = sw ? dim3((unsigned)(r.N / kSwChan), (unsigned)mt_sw, 1u)
                         : dim3((unsigned)(r.N / r.bn), (unsigned)mt, (unsigned)r.splits);
        cfg.blockDim = dim3(sw ? kSwThreads : kTcThreads, 1, 1);
        cfg.dynamicSmemBytes = (size_t)r.smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = m->pdl ? 1 : 0;
        attr[1].id = cudaLaunchAttributeClusterDimension;  // the K splits of a tile form one cluster
        attr[1].val.clusterDim.x = r.pair ? 2u : 1u;       // an SM pair shares one 256-channel tile
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = (unsigned)r.splits;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        void *args[] = {&r.p};
        LL_CUDA_TRY(cudaLaunchKernelExC(&cfg, r.kfn, args));
    }
    // the last layer wrote [rows_pad x out] fp32; hand the caller its n_rows
    LL_CUDA_TRY(cudaMemcpyAsync(d_y, m->out_pad, sizeof(float) * (size_t)n_rows * m->out_dim,
                                cudaMemcpyDeviceToDevice, st));
    return LL_OK;
}

}  // namespace

extern "C" {

int ll_batched_mlp_check(ll_batched_mlp *m, void *stream)
{
    if (!m)
        return LL_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    LL_CUDA_TRY(cudaSetDevice(m->device));
    // stream-ordered only: a resident engine on the same GPU never finishes, so no device-wide sync
    unsigned s = 0;
    LL_CUDA_TRY(cudaMemcpyAsync(&s, m->status, sizeof(s), cudaMemcpyDeviceToHost, st));
    LL_CUDA_TRY(cudaStreamSynchronize(st));
    if (s) {
        cudaMemsetAsync(m->status, 0, sizeof(unsigned), st);
        if (m->gemv) {  // the failed forward left part of its words or counts: start over
            for (int i = 0; i < 2; ++i)
                cudaMemsetAsync(m->hand[i], 0, m->hand_bytes, st);
            cudaMemsetAsync(m->cnt, 0, sizeof(unsigned) * kGvCntStride * (size_t)m->n_layers, st);
            m->tag_next = 1;
            m->epoch = 0;
        }
        cudaStreamSynchronize(st);
        llh::set_error("batched forward: a device wait ran out (status 0x%x, role %u)", s, (s >> 8) & 0xffu);
        return LL_ERR_DEVICE_FAULT;
    }
    return LL_OK;
}

int ll_batched_mlp_infer(ll_batched_mlp *m, const float *x, float *y, int n_rows)
{
    if (!m || !x || !y || n_rows < 1 || n_rows > m->max_rows) {
        llh::set_error("batched infer: bad arguments");
        return LL_ERR_INVALID_ARG;
    }
    LL_CUDA_TRY(cudaSetDevice(m->device));
    float *dx = nullptr, *dy = nullptr;
    LL_CUDA_TRY(cudaMalloc(&dx, sizeof(float) * (size_t)n_rows * m->in_dim));
    if (cudaMalloc(&dy, sizeof(float) * (size_t)n_rows * m->out_dim) != cudaSuccess) {
        cudaFree(dx);
        llh::set_error("batched infer: cudaMalloc failed");
        return LL_ERR_CUDA;
    }
    int rc = LL_OK;
    if (cudaMemcpyAsync(dx, x, sizeof(float) * (size_t)n_rows * m->in_dim, cudaMemcpyHostToDevice, m->own) !=
        cudaSuccess)
        rc = LL_ERR_CUDA;
    if (rc == LL_OK)
        rc = ll_batched_mlp_forward(m, dx, dy, n_rows, m->own);
    if (rc == LL_OK)
        rc = ll_batched_mlp_check(m, m->own);
    if (rc == LL_OK && (cudaMemcpyAsync(y, dy, sizeof(float) * (size_t)n_rows * m->out_dim, cudaMemcpyDeviceToHost,
                                        m->own) != cudaSuccess ||
                        cudaStreamSynchronize(m->own) != cudaSuccess))
        rc = LL_ERR_CUDA;
    cudaFree(dx);
    cudaFree(dy);
    return rc;
}

int ll_batched_mlp_set_trace(ll_batched_mlp *m, unsigned long long *d_trace, size_t n)
{
    if (!m)
        return LL_ERR_INVALID_ARG;
    const size_t per_layer = (size_t)m->max_ctas * kTcTraceSlots;
    if (d_trace && n < per_layer * m->runs.size()) {
        llh::set_error("trace buffer needs %zu entries", per_layer * m->runs.size());
        return LL_ERR_INVALID_ARG;
    }
    for (size_t l = 0; l < m->runs.size(); ++l) {
        m->runs[l].p.trace = d_trace ? d_trace + l * per_layer : nullptr;
        m->gp.trace[l] = m->runs[l].p.trace;
    }
    if (m->gexec) {  // the captured launches carry the old trace pointers
        cudaGraphExecDestroy(m->gexec);
        m->gexec = nullptr;
    }
    return LL_OK;
}

int ll_batched_mlp_info(ll_batched_mlp *m, ll_batched_info *info)
{
    if (!m || !info)
        return LL_ERR_INVALID_ARG;
    std::memset(info, 0, sizeof(*info));
    info->n_layers = m->n_layers;
    info->rows_pad = m->rows_pad;
    for (int l = 0; l < m->n_layers; ++l) {
        info->kind[l] = m->runs[l].kind;
        info->bn[l] = m->runs[l].bn;
        info->splits[l] = m->runs[l].splits;
        info->ctas[l] = m->runs[l].ctas;
        info->smem_bytes[l] = m->runs[l].smem;
    }
    return LL_OK;
}

int ll_batched_mlp_destroy(ll_batched_mlp *m)
{
    if (!m)
        return LL_ERR_INVALID_ARG;
    destroy_all(m);
    return LL_OK;
}

}  // extern "C"
