"""B200-native low-latency MLP inference engine (Python mirror of the C ABI).

Everything here is a thin ctypes layer over ``_lib/libll_b200.so`` (sources in
``csrc/``, declarations in ``include/ll_b200.h``).  There is no Python or CPU
compute path: if the native library is missing, importing a handle raises.

Reference mapping (mamedov-ma/low_latency_inference_gpu):
  * ``Engine``      -- persistent mailbox kernel + TickBuffer protocol
                       (src/bench_persistent_mbyv_mlp.cu:88-95, 140-381, 536-559)
  * ``EchoEngine``  -- empty-mailbox ping-pong floor (no reference counterpart)
  * ``LayeredMLP``  -- launch-per-layer warp GEMV chain, direct / CUDA graph / e2e
                       (include/ll/dense_warp.cuh:33-90, src/bench_custom_warp_mlp_graph.cu,
                       src/bench_custom_warp_e2e.cu)
  * ``CublasMLP``   -- cuBLAS SGEMM chain (src/bench_cublas_mlp_graph.cu,
                       src/bench_persistent_cublas_mlp.cu)
  * ``fill_normal`` -- host_init (src/bench_cublas_mlp.cu:37-43)
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libll_b200.so")

# ---- constants (include/ll_b200.h) ----
LL_OK, LL_ERR_CUDA, LL_ERR_TIMEOUT, LL_ERR_BAD_DESC, LL_ERR_DEVICE_FAULT = 0, 1, 2, 3, 4
LL_ERR_STOPPED, LL_ERR_INVALID_ARG, LL_ERR_UNSUPPORTED, LL_ERR_BUSY = 5, 6, 7, 8
ACT_IDENTITY, ACT_RELU, ACT_GELU = 0, 1, 2
W_F32, W_BF16, W_I8 = 0, 1, 2
INIT_XAVIER_UNIFORM, INIT_NORMAL_FANIN = 0, 1
RUN_DIRECT_KERNEL, RUN_GRAPH_KERNEL, RUN_GRAPH_E2E, RUN_DIRECT_E2E, RUN_MAILBOX_TICK = 0, 1, 2, 3, 4
STOP_SEQ = 0xFFFFFFFF

ERROR_NAMES = {
    0: "LL_OK", 1: "LL_ERR_CUDA", 2: "LL_ERR_TIMEOUT", 3: "LL_ERR_BAD_DESC", 4: "LL_ERR_DEVICE_FAULT",
    5: "LL_ERR_STOPPED", 6: "LL_ERR_INVALID_ARG", 7: "LL_ERR_UNSUPPORTED", 8: "LL_ERR_BUSY",
}

# Exported symbols the C ABI header declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = [
    "ll_engine_opts_default", "ll_engine_create", "ll_engine_create_ex", "ll_echo_engine_create",
    "ll_engine_mailbox", "ll_engine_mailbox_x", "ll_engine_mailbox_y", "ll_engine_start", "ll_submit",
    "ll_poll", "ll_infer", "ll_engine_stop", "ll_engine_destroy", "ll_engine_get_info",
    "ll_engine_bench_closed_loop", "ll_engine_run_queue", "ll_last_error", "ll_dense_warp_rm",
    "ll_dense_mbyv_packed", "ll_pack_rm_to_kmajor_padded", "ll_pack_bias_padded", "ll_layered_mlp_create",
    "ll_layered_mlp_bench", "ll_layered_mlp_destroy", "ll_cublas_mlp_create", "ll_cublas_mlp_bench",
    "ll_cublas_mlp_destroy", "ll_fill_normal", "ll_fill_uniform", "ll_init_params", "ll_f32_to_bf16",
    "ll_quantize_int8_rows", "ll_compute_stats", "ll_mailbox_bytes", "ll_mailbox_post", "ll_mailbox_wait",
    "ll_next_seq", "ll_version", "ll_plan_net", "ll_engine_set_trace", "ll_mlp_forward_noalloc",
    "ll_tagged_mailbox_bytes", "ll_tagged_y_offset", "ll_tagged_post", "ll_tagged_wait",
    "ll_batched_opts_default", "ll_batched_plan", "ll_batched_mlp_create", "ll_batched_mlp_forward",
    "ll_batched_mlp_check", "ll_batched_mlp_infer", "ll_batched_mlp_info", "ll_batched_mlp_destroy",
    "ll_batched_mlp_set_trace", "ll_engine_serve_poisson",
    "ll_weights_save", "ll_weights_load", "ll_weights_net", "ll_weights_arrays", "ll_weights_free",
    "ll_submit_many", "ll_engine_bench_ring", "ll_engine_bench_ring_mt",
]
MAX_LAYERS = 24


class LLError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERROR_NAMES.get(code, code)}: {msg}")
        self.code = code


# ---- ctypes structs ----
class LayerDesc(ctypes.Structure):
    _fields_ = [("in_dim", ctypes.c_int32), ("out_dim", ctypes.c_int32), ("act", ctypes.c_int32),
                ("wtype", ctypes.c_int32)]


class NetDesc(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("layers", ctypes.POINTER(LayerDesc)), ("max_batch", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class EngineOpts(ctypes.Structure):
    _fields_ = [("cluster_size", ctypes.c_int32), ("replicate_first", ctypes.c_int32),
                ("write_combined", ctypes.c_int32), ("mailbox_format", ctypes.c_int32),
                ("idle_timeout_ns", ctypes.c_uint64), ("step_timeout_ns", ctypes.c_uint64),
                ("max_stages", ctypes.c_int32), ("min_stages", ctypes.c_int32), ("diag_wait_never", ctypes.c_int32),
                ("kernel_variant", ctypes.c_int32), ("ring_slots", ctypes.c_int32), ("micro_batch", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 2)]


# ll_engine_opts.kernel_variant
VARIANT_AUTO, VARIANT_GENERIC, VARIANT_REGISTER_RESIDENT, VARIANT_RESIDENT_SMALL_BATCH = 0, 1, 2, 3
VARIANT_PIPELINED_RING = 4


class EngineInfo(ctypes.Structure):
    _fields_ = [("n_stages", ctypes.c_int32), ("cluster_size", ctypes.c_int32), ("threads", ctypes.c_int32),
                ("smem_bytes", ctypes.c_int32), ("image_bytes", ctypes.c_int32), ("launches", ctypes.c_int32),
                ("state", ctypes.c_int32), ("status", ctypes.c_int32), ("err_where", ctypes.c_int32),
                ("served", ctypes.c_uint32), ("layer_modes", ctypes.c_int32 * 24), ("kernel_variant", ctypes.c_int32),
                ("weight_regs", ctypes.c_int32), ("passes", ctypes.c_uint32), ("rows", ctypes.c_uint32)]


class Stats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("p50", "p90", "p99", "min", "max", "mean", "sd")]


class TickHeader(ctypes.Structure):
    _fields_ = [("seq_in", ctypes.c_uint32), ("seq_out", ctypes.c_uint32), ("stop", ctypes.c_uint32),
                ("n_rows", ctypes.c_uint32)]


class PlanLayer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("mode", "act", "wtype", "lpr_log2", "K", "M", "Mp", "R", "in_buf",
                                               "in_ld", "out_buf", "out_ld")] + \
               [("w_off", ctypes.c_uint32), ("b_off", ctypes.c_uint32), ("s_off", ctypes.c_uint32),
                ("round_out", ctypes.c_int32)]


class Plan(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("n_layers", "n_stages", "cluster_size", "threads", "bmax4", "in_ld",
                                               "act_bf16", "reserved")] + \
               [("stage_first", ctypes.c_int32 * 9), ("stage_last", ctypes.c_int32 * 9),
                ("stage_in_ld", ctypes.c_int32 * 9), ("image_bytes", ctypes.c_uint32 * 9),
                ("buf_off", ctypes.c_uint32 * 6), ("smem_bytes", ctypes.c_uint32), ("image_stride", ctypes.c_uint32),
                ("layers", PlanLayer * 24)]


class BatchedOpts(ctypes.Structure):
    _fields_ = [("bn", ctypes.c_int32), ("splits", ctypes.c_int32), ("pdl", ctypes.c_int32),
                ("kernel", ctypes.c_int32), ("wait_ns", ctypes.c_uint64), ("graph", ctypes.c_int32),
                ("sm_pairs", ctypes.c_int32), ("reserved", ctypes.c_int32 * 2)]


class BatchedInfo(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("rows_pad", ctypes.c_int32), ("bn", ctypes.c_int32 * 24),
                ("splits", ctypes.c_int32 * 24), ("ctas", ctypes.c_int32 * 24), ("smem_bytes", ctypes.c_int32 * 24),
                ("kind", ctypes.c_int32 * 24)]


LAYER_MODE_NAMES = {0: "replicated", 1: "rowsplit_allgather", 2: "rowsplit_local", 3: "ksplit_gather",
                    4: "rowsplit_gather", 5: "rowsplit_global"}


_lib: Optional[ctypes.CDLL] = None

_fp = ctypes.POINTER(ctypes.c_float)
_dp = ctypes.POINTER(ctypes.c_double)
_vp = ctypes.c_void_p


def _sig(lib):
    P = ctypes.POINTER
    s = {
        "ll_engine_opts_default": (None, [P(EngineOpts)]),
        "ll_engine_create_ex": (ctypes.c_int, [P(NetDesc), P(_vp), P(_fp), P(_fp), ctypes.c_int, P(EngineOpts),
                                               P(_vp)]),
        "ll_echo_engine_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, P(EngineOpts), P(_vp)]),
        "ll_engine_mailbox": (_vp, [_vp]),
        "ll_engine_mailbox_x": (_vp, [_vp]),
        "ll_engine_mailbox_y": (_vp, [_vp]),
        "ll_engine_start": (ctypes.c_int, [_vp]),
        "ll_submit": (ctypes.c_int, [_vp, _fp, ctypes.c_int, P(ctypes.c_uint32)]),
        "ll_poll": (ctypes.c_int, [_vp, ctypes.c_uint32, _fp, ctypes.c_uint64]),
        "ll_infer": (ctypes.c_int, [_vp, _fp, ctypes.c_int, _fp, ctypes.c_uint64]),
        "ll_engine_stop": (ctypes.c_int, [_vp]),
        "ll_engine_destroy": (ctypes.c_int, [_vp]),
        "ll_engine_get_info": (ctypes.c_int, [_vp, P(EngineInfo)]),
        "ll_engine_bench_closed_loop": (ctypes.c_int, [_vp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, _dp]),
        "ll_engine_run_queue": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _fp, _vp]),
        "ll_engine_set_trace": (ctypes.c_int, [_vp, _vp, ctypes.c_int]),
        "ll_mlp_forward_noalloc": (ctypes.c_int, [P(NetDesc), P(_vp), P(_vp), _vp, _vp, _vp]),
        "ll_last_error": (ctypes.c_char_p, []),
        "ll_dense_warp_rm": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
        "ll_dense_mbyv_packed": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
        "ll_pack_rm_to_kmajor_padded": (None, [_fp, ctypes.c_size_t, ctypes.c_size_t, _fp, ctypes.c_size_t]),
        "ll_pack_bias_padded": (None, [_fp, ctypes.c_size_t, _fp, ctypes.c_size_t]),
        "ll_layered_mlp_create": (ctypes.c_int, [P(NetDesc), P(_fp), P(_fp), ctypes.c_int, P(_vp)]),
        "ll_layered_mlp_bench": (ctypes.c_int, [_vp, ctypes.c_int, _fp, ctypes.c_int, ctypes.c_int, _fp, _dp]),
        "ll_layered_mlp_destroy": (ctypes.c_int, [_vp]),
        "ll_cublas_mlp_create": (ctypes.c_int, [P(NetDesc), P(_fp), P(_fp), ctypes.c_int, P(_vp)]),
        "ll_cublas_mlp_bench": (ctypes.c_int, [_vp, ctypes.c_int, _fp, ctypes.c_int, ctypes.c_int, _fp, _dp]),
        "ll_cublas_mlp_destroy": (ctypes.c_int, [_vp]),
        "ll_fill_normal": (ctypes.c_int, [_fp, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]),
        "ll_fill_uniform": (ctypes.c_int, [_fp, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]),
        "ll_init_params": (ctypes.c_int, [P(NetDesc), ctypes.c_int, ctypes.c_uint32, P(_fp), P(_fp)]),
        "ll_f32_to_bf16": (None, [_fp, P(ctypes.c_uint16), ctypes.c_size_t]),
        "ll_quantize_int8_rows": (None, [_fp, ctypes.c_int, ctypes.c_int, P(ctypes.c_int8), _fp]),
        "ll_compute_stats": (None, [_dp, ctypes.c_size_t, P(Stats)]),
        "ll_mailbox_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "ll_mailbox_post": (None, [_vp, ctypes.c_int, _fp, ctypes.c_int, ctypes.c_uint32, ctypes.c_int]),
        "ll_mailbox_wait": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint32, _fp,
                                           ctypes.c_int, ctypes.c_uint64]),
        "ll_next_seq": (ctypes.c_uint32, [ctypes.c_uint32]),
        "ll_tagged_mailbox_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int]),
        "ll_tagged_y_offset": (ctypes.c_size_t, [ctypes.c_int]),
        "ll_tagged_post": (None, [_vp, ctypes.c_int, _fp, ctypes.c_uint32]),
        "ll_tagged_wait": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_uint32, _fp, ctypes.c_uint64]),
        "ll_version": (ctypes.c_char_p, []),
        "ll_plan_net": (ctypes.c_int, [P(NetDesc), P(_vp), P(_fp), P(_fp), P(EngineOpts), P(Plan), _vp,
                                       ctypes.c_size_t, P(ctypes.c_size_t)]),
        "ll_batched_opts_default": (None, [P(BatchedOpts)]),
        "ll_batched_plan": (ctypes.c_int, [P(NetDesc), P(BatchedOpts), P(BatchedInfo)]),
        "ll_batched_mlp_create": (ctypes.c_int, [P(NetDesc), P(_vp), P(_fp), P(_fp), ctypes.c_int, P(BatchedOpts),
                                                 P(_vp)]),
        "ll_batched_mlp_forward": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp]),
        "ll_batched_mlp_check": (ctypes.c_int, [_vp, _vp]),
        "ll_batched_mlp_infer": (ctypes.c_int, [_vp, _fp, _fp, ctypes.c_int]),
        "ll_batched_mlp_info": (ctypes.c_int, [_vp, P(BatchedInfo)]),
        "ll_batched_mlp_destroy": (ctypes.c_int, [_vp]),
        "ll_batched_mlp_set_trace": (ctypes.c_int, [_vp, _vp, ctypes.c_size_t]),
        "ll_weights_save": (ctypes.c_int, [ctypes.c_char_p, P(NetDesc), P(_vp), P(_fp), P(_fp)]),
        "ll_weights_load": (ctypes.c_int, [ctypes.c_char_p, P(_vp)]),
        "ll_weights_net": (P(NetDesc), [_vp]),
        "ll_weights_arrays": (ctypes.c_int, [_vp, P(_vp), P(_fp), P(_fp)]),
        "ll_weights_free": (None, [_vp]),
        "ll_engine_serve_poisson": (ctypes.c_int, [_vp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                                   ctypes.c_uint64, ctypes.c_int, ctypes.c_int, _dp,
                                                   ctypes.POINTER(ctypes.c_int), _dp, _fp,
                                                   ctypes.POINTER(ctypes.c_int)]),
        "ll_submit_many": (ctypes.c_int, [_vp, _fp, ctypes.c_int, P(ctypes.c_uint32)]),
        "ll_engine_bench_ring": (ctypes.c_int, [_vp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, _dp, _dp]),
        "ll_engine_bench_ring_mt": (ctypes.c_int, [_vp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, _dp, _dp,
                                                    ctypes.c_int]),
    }
    for name, (res, args) in s.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args


def lib() -> ctypes.CDLL:
    """The native library; raises (never falls back) when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"native library missing: {LIB_PATH} (run __graft_entry__.build())")
        l = ctypes.CDLL(LIB_PATH)
        _sig(l)
        _lib = l
    return _lib


def _check(rc: int):
    if rc != LL_OK:
        raise LLError(rc, lib().ll_last_error().decode(errors="replace"))


def _f(a: np.ndarray):
    return a.ctypes.data_as(_fp)


def _d(a: np.ndarray):
    return a.ctypes.data_as(_dp)


# ---- network description ----
@dataclass
class Net:
    dims: List[int]           # [in, h1, ..., out]
    acts: List[int]           # per layer
    wtype: int = W_F32
    max_batch: int = 1

    @property
    def n_layers(self) -> int:
        return len(self.dims) - 1

    def desc(self):
        arr = (LayerDesc * self.n_layers)()
        for l in range(self.n_layers):
            arr[l] = LayerDesc(self.dims[l], self.dims[l + 1], self.acts[l], self.wtype)
        d = NetDesc(self.n_layers, arr, self.max_batch, 0)
        d._keep = arr
        return d

    @property
    def n_params(self) -> int:
        return sum(self.dims[l] * self.dims[l + 1] for l in range(self.n_layers))

    @property
    def flops_per_row(self) -> int:
        return 2 * self.n_params


def mlp(dims: Sequence[int], hidden_act: int = ACT_RELU, out_act: int = ACT_IDENTITY, wtype: int = W_F32,
        max_batch: int = 1) -> Net:
    n = len(dims) - 1
    return Net(list(dims), [hidden_act] * (n - 1) + [out_act], wtype, max_batch)


# ---- generators ----
def fill_normal(n: int, mean: float, std: float, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(lib().ll_fill_normal(_f(out), n, mean, std, seed))
    return out


def fill_uniform(n: int, lo: float, hi: float, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(lib().ll_fill_uniform(_f(out), n, lo, hi, seed))
    return out


def init_params(net: Net, init: int, seed: int):
    """fp32 master weights [out x in] and biases of a net, one mt19937 stream (W1, b1, W2, b2, ...)."""
    Ws = [np.empty((net.dims[l + 1], net.dims[l]), np.float32) for l in range(net.n_layers)]
    bs = [np.empty(net.dims[l + 1], np.float32) for l in range(net.n_layers)]
    Wp = (_fp * net.n_layers)(*[_f(w) for w in Ws])
    bp = (_fp * net.n_layers)(*[_f(b) for b in bs])
    d = net.desc()
    _check(lib().ll_init_params(ctypes.byref(d), init, seed, Wp, bp))
    return Ws, bs


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty(a.shape, np.uint16)
    lib().ll_f32_to_bf16(_f(a), out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), a.size)
    return out


def quantize_int8_rows(W: np.ndarray):
    W = np.ascontiguousarray(W, np.float32)
    m, k = W.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().ll_quantize_int8_rows(_f(W), m, k, q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), _f(s))
    return q, s


def compute_stats(xs) -> dict:
    a = np.ascontiguousarray(xs, np.float64)
    st = Stats()
    lib().ll_compute_stats(_d(a), a.size, ctypes.byref(st))
    return {k: getattr(st, k) for k, _ in Stats._fields_}


def pack_rm_to_kmajor_padded(W: np.ndarray, Mpad: int) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    M, K = W.shape
    out = np.empty((K, Mpad), np.float32)
    lib().ll_pack_rm_to_kmajor_padded(_f(W), M, K, _f(out), Mpad)
    return out


def pack_bias_padded(b: np.ndarray, Mpad: int) -> np.ndarray:
    b = np.ascontiguousarray(b, np.float32)
    out = np.empty(Mpad, np.float32)
    lib().ll_pack_bias_padded(_f(b), b.size, _f(out), Mpad)
    return out


# ---- the workloads (synthetic inputs, seeded) ----
CONFIGS = {
    # fp32 MLP 64->256->256->16, ReLU hidden, identity out, batch 1; Xavier-U W, U[-0.01,0.01] b (seed 0); x U[-1,1] seed 1
    0: dict(dims=[64, 256, 256, 16], act=ACT_RELU, wtype=W_F32, init=INIT_XAVIER_UNIFORM, x="uniform", x_seed=1,
            max_batch=1),
    # fp32 MLP 128 -> 512 x 8 square layers -> 32 (10 GEMVs), ReLU; x N(0,1) seed 2
    1: dict(dims=[128] + [512] * 9 + [32], act=ACT_RELU, wtype=W_F32, init=INIT_XAVIER_UNIFORM, x="normal",
            x_seed=2, max_batch=1),
    # bf16 weights, fp32 accumulate, 256 -> 1024 x 4 square layers -> 64, GELU; W N(0,1/fan_in); x U[-1,1] seed 3
    2: dict(dims=[256] + [1024] * 5 + [64], act=ACT_GELU, wtype=W_BF16, init=INIT_NORMAL_FANIN, x="uniform",
            x_seed=3, max_batch=32),
    # int8 W + per-channel scales, bf16 activations: 1024 -> 2048 x 6 square -> 256, ReLU, batch 256; x N(0,1) seed 4
    3: dict(dims=[1024] + [2048] * 7 + [256], act=ACT_RELU, wtype=W_I8, init=INIT_NORMAL_FANIN, x="normal",
            x_seed=4, max_batch=256),
    # the reference's own MLP (include/net_config.h:6-14), used for golden parity
    "ref": dict(dims=[512, 256, 64, 1], act=ACT_RELU, wtype=W_F32, init=None, x="normal", x_seed=1, max_batch=1),
}


def config_net(cfg, max_batch: Optional[int] = None) -> Net:
    c = CONFIGS[cfg]
    return mlp(c["dims"], c["act"], ACT_IDENTITY, c["wtype"], max_batch or c["max_batch"])


def config_params(cfg):
    """(net, fp32 master W list, b list) for a workload; the reference MLP uses host_init seeds 2..7."""
    c = CONFIGS[cfg]
    net = config_net(cfg)
    if cfg == "ref":
        # src/bench_cublas_mlp.cu:74-80: W1 (0.02, 2), b1 (0.01, 3), W2 (0.02, 4), b2 (0.01, 5), W3 (0.02, 6), b3 (0.01, 7)
        Ws, bs = [], []
        for l in range(net.n_layers):
            Ws.append(fill_normal(net.dims[l] * net.dims[l + 1], 0.0, 0.02, 2 + 2 * l).reshape(net.dims[l + 1],
                                                                                              net.dims[l]))
            bs.append(fill_normal(net.dims[l + 1], 0.0, 0.01, 3 + 2 * l))
        return net, Ws, bs
    Ws, bs = init_params(net, c["init"], 0)
    return net, Ws, bs


def config_inputs(cfg, n_rows: int) -> np.ndarray:
    c = CONFIGS[cfg]
    n = n_rows * c["dims"][0]
    if c["x"] == "uniform":
        x = fill_uniform(n, -1.0, 1.0, c["x_seed"])
    else:
        x = fill_normal(n, 0.0, 1.0, c["x_seed"])
    return x.reshape(n_rows, c["dims"][0])


def device_weights(net: Net, Ws, bs):
    """Convert fp32 masters into what the engine takes for the net's weight type: (W list, b list, scales)."""
    if net.wtype == W_F32:
        return [np.ascontiguousarray(w, np.float32) for w in Ws], bs, None
    if net.wtype == W_BF16:
        return [f32_to_bf16(w) for w in Ws], bs, None
    qs, ss = zip(*[quantize_int8_rows(w) for w in Ws])
    return list(qs), bs, list(ss)


def default_opts() -> EngineOpts:
    o = EngineOpts()
    lib().ll_engine_opts_default(ctypes.byref(o))
    return o


class Engine:
    """Resident-kernel engine bound to one GPU; mirrors the reference's persistent bench host code."""

    def __init__(self, net: Net, W, b, scales=None, device: int = 0, opts: Optional[EngineOpts] = None,
                 _handle=None):
        self.net = net
        self.in_dim = net.dims[0] if net else 0
        self.out_dim = net.dims[-1] if net else 0
        self.h = ctypes.c_void_p()
        if _handle is not None:
            self.h = _handle
            return
        self._keep = [np.ascontiguousarray(w) for w in W]
        self._keepb = [np.ascontiguousarray(x, np.float32) for x in b] if b is not None else None
        self._keeps = [np.ascontiguousarray(x, np.float32) for x in scales] if scales is not None else None
        Wp = (_vp * net.n_layers)(*[w.ctypes.data for w in self._keep])
        bp = (_fp * net.n_layers)(*[_f(x) for x in self._keepb]) if self._keepb is not None else None
        sp = (_fp * net.n_layers)(*[_f(x) for x in self._keeps]) if self._keeps is not None else None
        d = net.desc()
        o = opts if opts is not None else default_opts()
        _check(lib().ll_engine_create_ex(ctypes.byref(d), Wp, bp, sp, device, ctypes.byref(o), ctypes.byref(self.h)))
        self.max_batch = net.max_batch

    def start(self):
        _check(lib().ll_engine_start(self.h))

    def submit(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.in_dim)
        seq = ctypes.c_uint32()
        _check(lib().ll_submit(self.h, _f(x), x.shape[0], ctypes.byref(seq)))
        self._rows = x.shape[0]
        return seq.value

    def submit_many(self, xs: np.ndarray) -> List[int]:
        """Post k batch-1 requests at once (ll_submit_many: the whole burst is written before
        the device can take its first request); returns their sequence numbers."""
        xs = np.ascontiguousarray(xs, np.float32).reshape(-1, self.in_dim)
        seqs = (ctypes.c_uint32 * xs.shape[0])()
        _check(lib().ll_submit_many(self.h, _f(xs), xs.shape[0], seqs))
        self._rows = 1
        return list(seqs)

    def poll(self, seq: int, timeout_s: float = 2.0) -> np.ndarray:
        y = np.empty((self._rows, self.out_dim), np.float32)
        _check(lib().ll_poll(self.h, seq, _f(y), int(timeout_s * 1e9)))
        return y

    def infer(self, x: np.ndarray, timeout_s: float = 2.0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.in_dim)
        y = np.empty((x.shape[0], self.out_dim), np.float32)
        _check(lib().ll_infer(self.h, _f(x), x.shape[0], _f(y), int(timeout_s * 1e9)))
        return y

    def bench_closed_loop(self, xs: np.ndarray, n_req: int, n_rows: int = 1, keep_outputs: bool = False):
        xs = np.ascontiguousarray(xs, np.float32).reshape(-1, n_rows * self.in_dim)
        lat = np.empty(n_req, np.float64)
        ys = np.empty((n_req, n_rows, self.out_dim), np.float32) if keep_outputs else None
        _check(lib().ll_engine_bench_closed_loop(self.h, _f(xs), xs.shape[0], n_req, n_rows,
                                                 _f(ys) if ys is not None else None, _d(lat)))
        return lat, ys

    def serve_poisson(self, xs: np.ndarray, n_total: int, rate_per_s: float, seed: int = 5, rank: int = 0,
                      world: int = 1, keep_outputs: bool = False):
        """Open-loop Poisson stream (see ll_engine_serve_poisson): (latencies in us of this rank's
        requests, from their scheduled arrival; seconds from the start to the last reply), plus
        (replies [n][out_dim], stream index of each request) when keep_outputs."""
        xs = np.ascontiguousarray(xs, np.float32).reshape(-1, self.in_dim)
        lat = np.empty(max(1, n_total), np.float64)
        n = ctypes.c_int()
        el = ctypes.c_double()
        ys = np.empty((max(1, n_total), self.out_dim), np.float32) if keep_outputs else None
        idx = np.empty(max(1, n_total), np.int32) if keep_outputs else None
        _check(lib().ll_engine_serve_poisson(self.h, _f(xs), xs.shape[0], n_total, rate_per_s, seed, rank, world,
                                             _d(lat), ctypes.byref(n), ctypes.byref(el),
                                             _f(ys) if keep_outputs else None,
                                             idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)) if keep_outputs
                                             else None))
        if keep_outputs:
            return lat[:n.value].copy(), el.value, ys[:n.value].copy(), idx[:n.value].copy()
        return lat[:n.value].copy(), el.value

    def bench_ring(self, xs: np.ndarray, n_req: int, depth: int, keep_outputs: bool = False):
        """Closed loop with `depth` requests kept in flight (ll_engine_bench_ring): (latencies in
        us from post to reply, elapsed seconds, replies [n_req][out_dim] or None)."""
        xs = np.ascontiguousarray(xs, np.float32).reshape(-1, self.in_dim)
        lat = np.empty(max(1, n_req), np.float64)
        ys = np.empty((max(1, n_req), self.out_dim), np.float32) if keep_outputs else None
        el = ctypes.c_double()
        _check(lib().ll_engine_bench_ring(self.h, _f(xs), xs.shape[0], n_req, depth,
                                          _f(ys) if keep_outputs else None, _d(lat), ctypes.byref(el)))
        return lat[:n_req].copy(), el.value, (ys[:n_req].copy() if keep_outputs else None)

    def bench_ring_mt(self, xs: np.ndarray, n_req: int, depth: int, poster_cpu: int = -1,
                      keep_outputs: bool = False):
        """bench_ring on two host threads (ll_engine_bench_ring_mt): a poster thread (pinned to
        poster_cpu when >= 0) and the calling thread collecting replies."""
        xs = np.ascontiguousarray(xs, np.float32).reshape(-1, self.in_dim)
        lat = np.empty(max(1, n_req), np.float64)
        ys = np.empty((max(1, n_req), self.out_dim), np.float32) if keep_outputs else None
        el = ctypes.c_double()
        _check(lib().ll_engine_bench_ring_mt(self.h, _f(xs), xs.shape[0], n_req, depth,
                                             _f(ys) if keep_outputs else None, _d(lat), ctypes.byref(el),
                                             int(poster_cpu)))
        return lat[:n_req].copy(), el.value, (ys[:n_req].copy() if keep_outputs else None)

    def run_queue(self, d_x_ptr: int, d_y_ptr: int, n_req: int, n_rows: int = 1, d_stamps_ptr: int = 0) -> float:
        ms = ctypes.c_float()
        _check(lib().ll_engine_run_queue(self.h, d_x_ptr, d_y_ptr, n_req, n_rows, ctypes.byref(ms),
                                         d_stamps_ptr or None))
        return ms.value

    def set_trace(self, d_trace_ptr: int, n: int):
        """Record a device timeline of the first n requests of later launches (32 uint64 per request)."""
        _check(lib().ll_engine_set_trace(self.h, d_trace_ptr or None, n))

    def info(self) -> EngineInfo:
        inf = EngineInfo()
        _check(lib().ll_engine_get_info(self.h, ctypes.byref(inf)))
        return inf

    def mailbox(self) -> int:
        return lib().ll_engine_mailbox(self.h)

    def stop(self):
        _check(lib().ll_engine_stop(self.h))

    def close(self):
        if self.h:
            rc = lib().ll_engine_destroy(self.h)
            self.h = ctypes.c_void_p()
            _check(rc)

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class EchoEngine(Engine):
    """Ping-pong floor: the resident kernel and mailbox with no layers."""

    def __init__(self, in_dim: int = 0, out_dim: int = 0, device: int = 0, opts: Optional[EngineOpts] = None):
        h = ctypes.c_void_p()
        o = opts if opts is not None else default_opts()
        _check(lib().ll_echo_engine_create(device, in_dim, out_dim, ctypes.byref(o), ctypes.byref(h)))
        super().__init__(None, None, None, _handle=h)
        self.in_dim = in_dim
        self.out_dim = out_dim
        self.max_batch = 1

    def submit(self, x: Optional[np.ndarray] = None) -> int:
        seq = ctypes.c_uint32()
        xa = None if x is None or self.in_dim == 0 else np.ascontiguousarray(x, np.float32)
        _check(lib().ll_submit(self.h, _f(xa) if xa is not None else None, 1, ctypes.byref(seq)))
        self._rows = 1
        return seq.value

    def bench_closed_loop(self, xs: Optional[np.ndarray], n_req: int, n_rows: int = 1, keep_outputs: bool = False):
        if xs is None or self.in_dim == 0:
            xs = np.zeros((1, max(self.in_dim, 1)), np.float32)
        xs = np.ascontiguousarray(xs, np.float32)
        lat = np.empty(n_req, np.float64)
        ys = np.empty((n_req, 1, max(self.out_dim, 1)), np.float32) if keep_outputs else None
        _check(lib().ll_engine_bench_closed_loop(self.h, _f(xs), xs.shape[0], n_req, 1,
                                                 _f(ys) if ys is not None else None, _d(lat)))
        return lat, ys


class _ChainMLP:
    _create = None
    _bench = None
    _destroy = None

    def __init__(self, net: Net, Ws, bs, device: int = 0):
        self.net = net
        self._keep = [np.ascontiguousarray(w, np.float32) for w in Ws]
        self._keepb = [np.ascontiguousarray(x, np.float32) for x in bs]
        Wp = (_fp * net.n_layers)(*[_f(w) for w in self._keep])
        bp = (_fp * net.n_layers)(*[_f(x) for x in self._keepb])
        self.h = ctypes.c_void_p()
        d = net.desc()
        _check(getattr(lib(), self._create)(ctypes.byref(d), Wp, bp, device, ctypes.byref(self.h)))

    def bench(self, mode: int, xs: np.ndarray, n_req: int):
        xs = np.ascontiguousarray(xs, np.float32).reshape(-1, self.net.dims[0])
        lat = np.empty(n_req, np.float64)
        y = np.empty(self.net.dims[-1], np.float32)
        _check(getattr(lib(), self._bench)(self.h, mode, _f(xs), xs.shape[0], n_req, _f(y), _d(lat)))
        return lat, y

    def close(self):
        if self.h:
            getattr(lib(), self._destroy)(self.h)
            self.h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


class LayeredMLP(_ChainMLP):
    _create, _bench, _destroy = "ll_layered_mlp_create", "ll_layered_mlp_bench", "ll_layered_mlp_destroy"


class CublasMLP(_ChainMLP):
    _create, _bench, _destroy = "ll_cublas_mlp_create", "ll_cublas_mlp_bench", "ll_cublas_mlp_destroy"


def dense_warp_rm(W_ptr: int, b_ptr: int, x_ptr: int, y_ptr: int, M: int, K: int, act: int, stream: int = 0):
    _check(lib().ll_dense_warp_rm(W_ptr, b_ptr, x_ptr, y_ptr, M, K, act, stream or None))


def dense_mbyv_packed(Wcm_ptr: int, bpad_ptr: int, x_ptr: int, y_ptr: int, M: int, K: int, act: int,
                      stream: int = 0):
    _check(lib().ll_dense_mbyv_packed(Wcm_ptr, bpad_ptr, x_ptr, y_ptr, M, K, act, stream or None))


def plan_net(net: Net, W=None, b=None, scales=None, opts: Optional[EngineOpts] = None, want_images: bool = False):
    """(Plan, images or None) for a net, computed on the host without a GPU."""
    o = opts if opts is not None else default_opts()
    d = net.desc()
    plan = Plan()
    need = ctypes.c_size_t()
    Wp = bp = sp = None
    keep = []
    if want_images:
        kw = [np.ascontiguousarray(w) for w in W]
        kb = [np.ascontiguousarray(x, np.float32) for x in b] if b is not None else None
        ks = [np.ascontiguousarray(x, np.float32) for x in scales] if scales is not None else None
        keep = [kw, kb, ks]
        Wp = (_vp * net.n_layers)(*[w.ctypes.data for w in kw])
        bp = (_fp * net.n_layers)(*[_f(x) for x in kb]) if kb is not None else None
        sp = (_fp * net.n_layers)(*[_f(x) for x in ks]) if ks is not None else None
    _check(lib().ll_plan_net(ctypes.byref(d), Wp, bp, sp, ctypes.byref(o), ctypes.byref(plan), None, 0,
                             ctypes.byref(need)))
    if not want_images:
        return plan, None
    img = np.zeros(need.value, np.uint8)
    _check(lib().ll_plan_net(ctypes.byref(d), Wp, bp, sp, ctypes.byref(o), ctypes.byref(plan),
                             img.ctypes.data, img.size, ctypes.byref(need)))
    del keep
    return plan, img


NOALLOC_MAX_WIDTH = 8192


def mlp_forward_noalloc(net: Net, d_W_ptrs, d_b_ptrs, d_x_ptr: int, d_y_ptr: int, stream: int = 0):
    """Forward pass that allocates nothing (see ll_mlp_forward_noalloc in include/ll_b200.h):
    device pointers in, device pointer out, hidden activations in a static library-owned array."""
    d = net.desc()
    Wp = (_vp * net.n_layers)(*d_W_ptrs)
    bp = (_vp * net.n_layers)(*d_b_ptrs) if d_b_ptrs is not None else None
    _check(lib().ll_mlp_forward_noalloc(ctypes.byref(d), Wp, bp, d_x_ptr, d_y_ptr, stream or None))


# ---- batched dense path (tensor cores) ----
KERNEL_SPLITK, KERNEL_WEIGHTS_IN_TMEM, KERNEL_GEMV = 1, 2, 3


def batched_opts(bn: int = 0, splits: int = 0, pdl: int = 1, wait_ns: int = 0, kernel: int = 0,
                 graph: int = 1, sm_pairs: int = 0) -> BatchedOpts:
    o = BatchedOpts()
    lib().ll_batched_opts_default(ctypes.byref(o))
    o.bn, o.splits, o.pdl, o.wait_ns, o.kernel, o.graph = bn, splits, pdl, wait_ns, kernel, graph
    o.sm_pairs = sm_pairs
    return o


def _batched_info_dict(info: BatchedInfo) -> dict:
    n = info.n_layers
    return {"rows_pad": info.rows_pad, "bn": list(info.bn[:n]), "splits": list(info.splits[:n]),
            "ctas": list(info.ctas[:n]), "smem_bytes": list(info.smem_bytes[:n]), "kind": list(info.kind[:n])}


def batched_plan(net: Net, opts: Optional[BatchedOpts] = None) -> dict:
    """Tiling the batched path would use for `net` at max_batch rows (host only)."""
    d = net.desc()
    info = BatchedInfo()
    _check(lib().ll_batched_plan(ctypes.byref(d), ctypes.byref(opts) if opts is not None else None,
                                 ctypes.byref(info)))
    return _batched_info_dict(info)


class BatchedMLP:
    """tcgen05 tensor-core MLP over many rows (bf16 or int8 + per-channel scales weights)."""

    def __init__(self, net: Net, W, b, scales=None, device: int = 0, opts: Optional[BatchedOpts] = None):
        self.net = net
        self.in_dim, self.out_dim = net.dims[0], net.dims[-1]
        self.h = ctypes.c_void_p()
        self._keep = [np.ascontiguousarray(w) for w in W]
        self._keepb = [np.ascontiguousarray(x, np.float32) for x in b] if b is not None else None
        self._keeps = [np.ascontiguousarray(x, np.float32) for x in scales] if scales is not None else None
        Wp = (_vp * net.n_layers)(*[w.ctypes.data for w in self._keep])
        bp = (_fp * net.n_layers)(*[_f(x) for x in self._keepb]) if self._keepb is not None else None
        sp = (_fp * net.n_layers)(*[_f(x) for x in self._keeps]) if self._keeps is not None else None
        d = net.desc()
        _check(lib().ll_batched_mlp_create(ctypes.byref(d), Wp, bp, sp, device,
                                           ctypes.byref(opts) if opts is not None else None, ctypes.byref(self.h)))
        self._keep = self._keepb = self._keeps = None  # copied to the device

    def forward(self, d_x_ptr: int, d_y_ptr: int, n_rows: int, stream: int = 0):
        _check(lib().ll_batched_mlp_forward(self.h, d_x_ptr, d_y_ptr, n_rows, stream or None))

    def check(self, stream: int = 0):
        _check(lib().ll_batched_mlp_check(self.h, stream or None))

    def infer(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.in_dim)
        y = np.empty((x.shape[0], self.out_dim), np.float32)
        _check(lib().ll_batched_mlp_infer(self.h, _f(x), _f(y), x.shape[0]))
        return y

    def info(self) -> dict:
        info = BatchedInfo()
        _check(lib().ll_batched_mlp_info(self.h, ctypes.byref(info)))
        return _batched_info_dict(info)

    def set_trace(self, d_trace_ptr: int, n: int):
        """Per-CTA phase stamps (see ll_batched_mlp_set_trace); d_trace_ptr = 0 turns tracing off."""
        _check(lib().ll_batched_mlp_set_trace(self.h, d_trace_ptr or None, n))

    TRACE_PHASES = ("entry", "prev_layer_done", "first_stage", "mma_issued", "accumulated", "cluster_barrier",
                    "exchanged", "end", "staged", "k0_ready", "k1_ready", "k2_ready", "k3_ready", "reissue",
                    "reissue_ready", "k0_converted")

    def phase_trace(self, x: np.ndarray, warm: int = 3) -> list:
        """One traced forward of x (after `warm` untraced ones): per layer, the median over
        its CTAs of each phase stamp in microseconds from the first CTA's entry into
        layer 0, plus the last CTA's end (needs torch for the device buffers)."""
        import torch

        info = self.info()
        n_layers, mx = len(info["ctas"]), max(info["ctas"])
        tr = torch.zeros(n_layers * mx * 16, dtype=torch.int64, device="cuda")
        dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        dy = torch.empty((x.shape[0], self.out_dim), dtype=torch.float32, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        for _ in range(warm):
            self.forward(dx.data_ptr(), dy.data_ptr(), x.shape[0], st)
        self.set_trace(tr.data_ptr(), tr.numel())
        self.forward(dx.data_ptr(), dy.data_ptr(), x.shape[0], st)
        self.set_trace(0, 0)
        self.check(st)
        t = tr.cpu().numpy().reshape(n_layers, mx, 16).astype(np.float64)
        t0 = min(t[l, :info["ctas"][l], 0].min() for l in range(n_layers))
        out = []
        for l in range(n_layers):
            c = (t[l, :info["ctas"][l]] - t0) / 1000.0
            row = {name: float(np.median(c[:, k])) for k, name in enumerate(self.TRACE_PHASES)
                   if (k != 8 or info["splits"][l] > 1) and np.all(c[:, k] > -1e6)}
            row["end_max"] = float(c[:, 7].max())
            out.append(row)
        return out

    def close(self):
        if self.h:
            lib().ll_batched_mlp_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- weight files ----
_W_DTYPE = {W_F32: np.float32, W_BF16: np.uint16, W_I8: np.int8}


def save_weights(path: str, net: Net, W, b=None, scales=None):
    """Write net + weights (in the net's type: fp32, bf16 bits as uint16, int8) + biases
    + int8 scales to one file (see ll_weights_save)."""
    d = net.desc()
    keep = [np.ascontiguousarray(w, _W_DTYPE[net.wtype]) for w in W]
    keepb = [np.ascontiguousarray(x, np.float32) for x in b] if b is not None else None
    keeps = [np.ascontiguousarray(x, np.float32) for x in scales] if scales is not None else None
    Wp = (_vp * net.n_layers)(*[w.ctypes.data for w in keep])
    bp = (_fp * net.n_layers)(*[_f(x) for x in keepb]) if keepb is not None else None
    sp = (_fp * net.n_layers)(*[_f(x) for x in keeps]) if keeps is not None else None
    _check(lib().ll_weights_save(os.fsencode(path), ctypes.byref(d), Wp, bp, sp))


def load_weights(path: str):
    """(net, W, b, scales) from a weight file; b / scales are None when the file has none."""
    h = ctypes.c_void_p()
    _check(lib().ll_weights_load(os.fsencode(path), ctypes.byref(h)))
    try:
        nd = lib().ll_weights_net(h).contents
        n = nd.n_layers
        layers = [nd.layers[i] for i in range(n)]
        wt = layers[0].wtype
        net = Net([layers[0].in_dim] + [x.out_dim for x in layers], [x.act for x in layers], wt, nd.max_batch)
        Wp, bp, sp = (_vp * n)(), (_fp * n)(), (_fp * n)()
        _check(lib().ll_weights_arrays(h, Wp, bp, sp))
        W, b, s = [], [], []
        for l, x in enumerate(layers):
            nel = x.out_dim * x.in_dim
            buf = (ctypes.c_uint8 * (nel * np.dtype(_W_DTYPE[wt]).itemsize)).from_address(Wp[l])
            W.append(np.frombuffer(buf, _W_DTYPE[wt]).reshape(x.out_dim, x.in_dim).copy())
            b.append(np.ctypeslib.as_array(bp[l], (x.out_dim,)).copy() if bp[l] else None)
            s.append(np.ctypeslib.as_array(sp[l], (x.out_dim,)).copy() if sp[l] else None)
        return net, W, (b if all(v is not None for v in b) else None), (s if wt == W_I8 else None)
    finally:
        lib().ll_weights_free(h)
