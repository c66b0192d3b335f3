"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline /
reference legs may import this package, and only as the checker or the timed
CPU baseline.  It wraps two shared libraries built by ``oracle/Makefile``:

* ``liboracle.so`` -- the C restatement in ``oracle.c`` (reference loop order
  of cpu_gemv_bias_relu, src/bench_persistent_mbyv_mlp.cu:50-67, plus this
  project's GELU / bf16 / int8 definitions);
* ``_ref/libref.so`` -- the reference's own host_init and cpu_gemv_bias_relu
  compiled from the reference sources (``make -C oracle ref``), used to pin the
  restatement and as the "reference" CPU baseline.  Optional: absent on a box
  that never saw the reference sources.
"""
from __future__ import annotations

import ctypes
import os
from typing import List, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(_HERE, "liboracle.so")
REF_LIB = os.path.join(_HERE, "_ref", "libref.so")

_fp = ctypes.POINTER(ctypes.c_float)
_dp = ctypes.POINTER(ctypes.c_double)
_ip = ctypes.POINTER(ctypes.c_int)

_o = None
_r = None


def _f(a):
    return a.ctypes.data_as(_fp)


def olib():
    global _o
    if _o is None:
        if not os.path.exists(ORACLE_LIB):
            raise ImportError(f"oracle library missing: {ORACLE_LIB} (make -C oracle)")
        l = ctypes.CDLL(ORACLE_LIB)
        l.oracle_gemv_bias_act.argtypes = [_fp, _fp, _fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        l.oracle_mlp_f32.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp, _fp,
                                     ctypes.c_int]
        l.oracle_mlp_bf16.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(ctypes.POINTER(ctypes.c_uint16)),
                                      ctypes.POINTER(_fp), _fp, _fp, ctypes.c_int]
        l.oracle_mlp_int8.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(ctypes.POINTER(ctypes.c_int8)),
                                      ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp, _fp, ctypes.c_int]
        l.oracle_quantize_int8_rows.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int8), _fp]
        l.oracle_round_bf16_array.argtypes = [_fp, _fp, ctypes.c_size_t]
        l.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        l.oracle_f32_to_bf16.restype = ctypes.c_uint16
        l.oracle_pack_rm_to_kmajor_padded.argtypes = [_fp, ctypes.c_size_t, ctypes.c_size_t, _fp, ctypes.c_size_t]
        l.oracle_percentile_linear.argtypes = [_dp, ctypes.c_size_t, ctypes.c_double]
        l.oracle_percentile_linear.restype = ctypes.c_double
        l.oracle_percentile_nearest.argtypes = [_dp, ctypes.c_size_t, ctypes.c_double]
        l.oracle_percentile_nearest.restype = ctypes.c_double
        l.oracle_bench_mlp_f32.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp,
                                           ctypes.c_int, ctypes.c_long, _dp, _fp]
        l.oracle_bench_mlp_f32.restype = ctypes.c_double
        l.oracle_bench_mlp_f32_mt.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp,
                                              ctypes.c_int, ctypes.c_long, ctypes.c_int, _ip]
        l.oracle_bench_mlp_f32_mt.restype = ctypes.c_double
        l.oracle_fill_uniform.argtypes = [_fp, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]
        l.oracle_fill_normal.argtypes = [_fp, ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_uint32]
        l.oracle_init_params.argtypes = [ctypes.c_int, _ip, ctypes.c_int, ctypes.c_uint32, ctypes.POINTER(_fp),
                                         ctypes.POINTER(_fp)]
        _o = l
    return _o


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def rlib():
    global _r
    if _r is None:
        if not ref_available():
            raise ImportError(f"reference CPU library missing: {REF_LIB} (make -C oracle ref)")
        l = ctypes.CDLL(REF_LIB)
        l.ref_host_init.argtypes = [_fp, ctypes.c_size_t, ctypes.c_float, ctypes.c_uint32]
        l.ref_cpu_gemv_bias_relu.argtypes = [_fp, _fp, _fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        l.ref_mlp_forward.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp, _fp,
                                      ctypes.c_int]
        l.ref_bench_mlp.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp,
                                    ctypes.c_int, ctypes.c_long, _dp, _fp]
        l.ref_bench_mlp.restype = ctypes.c_double
        l.ref_bench_mlp_mt.argtypes = [ctypes.c_int, _ip, _ip, ctypes.POINTER(_fp), ctypes.POINTER(_fp), _fp,
                                       ctypes.c_int, ctypes.c_long, ctypes.c_int, _ip]
        l.ref_bench_mlp_mt.restype = ctypes.c_double
        _r = l
    return _r


def _arrs(dims, acts, Ws, bs):
    n = len(dims) - 1
    d = (ctypes.c_int * (n + 1))(*dims)
    a = (ctypes.c_int * n)(*acts)
    Wk = [np.ascontiguousarray(w, np.float32) for w in Ws]
    bk = [np.ascontiguousarray(b, np.float32) for b in bs]
    Wp = (_fp * n)(*[_f(w) for w in Wk])
    bp = (_fp * n)(*[_f(b) for b in bk])
    return n, d, a, Wp, bp, (Wk, bk)


def gemv_bias_act(W, b, x, act: int) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    m, k = W.shape
    y = np.empty(m, np.float32)
    olib().oracle_gemv_bias_act(_f(W), _f(np.ascontiguousarray(b, np.float32)), _f(np.ascontiguousarray(x, np.float32)),
                                _f(y), m, k, act)
    return y


def mlp_f32(dims, acts, Ws, bs, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, dims[0])
    y = np.empty((x.shape[0], dims[-1]), np.float32)
    n, d, a, Wp, bp, keep = _arrs(dims, acts, Ws, bs)
    olib().oracle_mlp_f32(n, d, a, Wp, bp, _f(x), _f(y), x.shape[0])
    return y


def mlp_bf16(dims, acts, Wbf16: Sequence[np.ndarray], bs, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, dims[0])
    y = np.empty((x.shape[0], dims[-1]), np.float32)
    n = len(dims) - 1
    d = (ctypes.c_int * (n + 1))(*dims)
    a = (ctypes.c_int * n)(*acts)
    Wk = [np.ascontiguousarray(w, np.uint16) for w in Wbf16]
    bk = [np.ascontiguousarray(b, np.float32) for b in bs]
    Wp = (ctypes.POINTER(ctypes.c_uint16) * n)(*[w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)) for w in Wk])
    bp = (_fp * n)(*[_f(b) for b in bk])
    olib().oracle_mlp_bf16(n, d, a, Wp, bp, _f(x), _f(y), x.shape[0])
    return y


def mlp_int8(dims, acts, Qs, Ss, bs, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, dims[0])
    y = np.empty((x.shape[0], dims[-1]), np.float32)
    n = len(dims) - 1
    d = (ctypes.c_int * (n + 1))(*dims)
    a = (ctypes.c_int * n)(*acts)
    Qk = [np.ascontiguousarray(q, np.int8) for q in Qs]
    Sk = [np.ascontiguousarray(s, np.float32) for s in Ss]
    bk = [np.ascontiguousarray(b, np.float32) for b in bs]
    Qp = (ctypes.POINTER(ctypes.c_int8) * n)(*[q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)) for q in Qk])
    Sp = (_fp * n)(*[_f(s) for s in Sk])
    bp = (_fp * n)(*[_f(b) for b in bk])
    olib().oracle_mlp_int8(n, d, a, Qp, Sp, bp, _f(x), _f(y), x.shape[0])
    return y


def quantize_int8_rows(W):
    W = np.ascontiguousarray(W, np.float32)
    m, k = W.shape
    q = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    olib().oracle_quantize_int8_rows(_f(W), m, k, q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)), _f(s))
    return q, s


def f32_to_bf16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32).ravel()
    return np.array([olib().oracle_f32_to_bf16(float(v)) for v in a], np.uint16)


def round_bf16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.empty_like(a)
    olib().oracle_round_bf16_array(_f(a), _f(out), a.size)
    return out


def pack_rm_to_kmajor_padded(W, Mpad):
    W = np.ascontiguousarray(W, np.float32)
    M, K = W.shape
    out = np.empty((K, Mpad), np.float32)
    olib().oracle_pack_rm_to_kmajor_padded(_f(W), M, K, _f(out), Mpad)
    return out


def percentile_linear(xs, p):
    s = np.ascontiguousarray(np.sort(np.asarray(xs, np.float64)))
    return olib().oracle_percentile_linear(s.ctypes.data_as(_dp), s.size, p)


def percentile_nearest(xs, p):
    s = np.ascontiguousarray(np.sort(np.asarray(xs, np.float64)))
    return olib().oracle_percentile_nearest(s.ctypes.data_as(_dp), s.size, p)


# ---- the reference's own code (oracle/_ref) ----
def ref_host_init(n: int, scale: float, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    rlib().ref_host_init(_f(out), n, scale, seed)
    return out


def ref_gemv_bias_relu(W, b, x, relu: bool) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    m, k = W.shape
    y = np.empty(m, np.float32)
    rlib().ref_cpu_gemv_bias_relu(_f(W), _f(np.ascontiguousarray(b, np.float32)),
                                  _f(np.ascontiguousarray(x, np.float32)), _f(y), m, k, 1 if relu else 0)
    return y


def ref_mlp(dims, relu_flags, Ws, bs, x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, dims[0])
    y = np.empty((x.shape[0], dims[-1]), np.float32)
    n, d, a, Wp, bp, keep = _arrs(dims, [1 if r else 0 for r in relu_flags], Ws, bs)
    rlib().ref_mlp_forward(n, d, a, Wp, bp, _f(x), _f(y), x.shape[0])
    return y


def bench_cpu(dims, acts, Ws, bs, xs, n_req: int, kind: str = "port", threads: int = 1, cpus=None):
    """Timed CPU forward.  kind "reference" runs the reference's own chain (oracle/_ref),
    "port" the C restatement.  threads == 1: per-request latencies (ns) and total ns;
    threads > 1: slowest thread's total ns for threads * n_req requests."""
    xs = np.ascontiguousarray(xs, np.float32).reshape(-1, dims[0])
    flags = list(acts)
    if kind == "reference":
        if any(a not in (0, 1) for a in acts):
            raise ValueError("the reference CPU forward has ReLU / identity only")
        l, fn, fn_mt = rlib(), "ref_bench_mlp", "ref_bench_mlp_mt"
    else:
        l, fn, fn_mt = olib(), "oracle_bench_mlp_f32", "oracle_bench_mlp_f32_mt"
    n, d, a, Wp, bp, keep = _arrs(dims, flags, Ws, bs)
    if threads <= 1:
        lat = np.empty(n_req, np.float64)
        y = np.empty(dims[-1], np.float32)
        total = getattr(l, fn)(n, d, a, Wp, bp, _f(xs), xs.shape[0], n_req, lat.ctypes.data_as(_dp), _f(y))
        return total, lat, y
    cp = (ctypes.c_int * threads)(*(cpus if cpus else [-1] * threads))
    total = getattr(l, fn_mt)(n, d, a, Wp, bp, _f(xs), xs.shape[0], n_req, threads, cp)
    return total, None, None


# ---- the benchmark workloads, drawn without the product library (oracle/gen.cpp) ----
ACT_IDENTITY, ACT_RELU, ACT_GELU = 0, 1, 2

# dims, hidden activation, weight init (0 Xavier-uniform, 1 N(0, 1/fan_in)), input distribution and seed
WORKLOADS = {
    0: dict(dims=[64, 256, 256, 16], act=ACT_RELU, normal_fanin=0, x="uniform", x_seed=1),
    1: dict(dims=[128] + [512] * 9 + [32], act=ACT_RELU, normal_fanin=0, x="normal", x_seed=2),
    2: dict(dims=[256] + [1024] * 5 + [64], act=ACT_GELU, normal_fanin=1, x="uniform", x_seed=3),
    3: dict(dims=[1024] + [2048] * 7 + [256], act=ACT_RELU, normal_fanin=1, x="normal", x_seed=4),
}


def fill_uniform(n: int, lo: float, hi: float, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    olib().oracle_fill_uniform(_f(out), n, lo, hi, seed)
    return out


def fill_normal(n: int, mean: float, sd: float, seed: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    olib().oracle_fill_normal(_f(out), n, mean, sd, seed)
    return out


def workload_params(cfg):
    """(dims, acts, fp32 W list [out x in], b list) of a benchmark workload, parameters from seed 0."""
    c = WORKLOADS[cfg]
    dims = c["dims"]
    n = len(dims) - 1
    acts = [c["act"]] * (n - 1) + [ACT_IDENTITY]
    Ws = [np.empty((dims[l + 1], dims[l]), np.float32) for l in range(n)]
    bs = [np.empty(dims[l + 1], np.float32) for l in range(n)]
    d = (ctypes.c_int * (n + 1))(*dims)
    olib().oracle_init_params(n, d, c["normal_fanin"], 0, (_fp * n)(*[_f(w) for w in Ws]),
                              (_fp * n)(*[_f(b) for b in bs]))
    return list(dims), acts, Ws, bs


def workload_inputs(cfg, n_rows: int) -> np.ndarray:
    """The first n_rows inputs of a benchmark workload (request-major)."""
    c = WORKLOADS[cfg]
    n = n_rows * c["dims"][0]
    x = fill_uniform(n, -1.0, 1.0, c["x_seed"]) if c["x"] == "uniform" else fill_normal(n, 0.0, 1.0, c["x_seed"])
    return x.reshape(n_rows, c["dims"][0])
