"""Generate tests/golden/golden.json -- run in a container that has the
reference sources (it builds and calls oracle/_ref, the reference's own CPU
forward compiled from those sources).

  python tests/golden/make_golden.py

Fixtures (float32 values stored as uint32 bit patterns, so comparisons are exact):
  ref_bench : the reference's own MLP 512->256->64->1 with its own seeds
              (host_init: x (1.0, 1), W1 (0.02, 2), b1 (0.01, 3), W2 (0.02, 4),
              b2 (0.01, 5), W3 (0.02, 6), b3 (0.01, 7); src/bench_cublas_mlp.cu:74-85),
              hidden and final outputs of the reference chain.
  cfg0, cfg1: fp32 workloads (Xavier-uniform weights from one mt19937(0) stream),
              outputs of the reference chain on the first requests.
  cfg2, cfg3: bf16 / int8 workloads; the reference has no GELU, bf16 or int8,
              so these outputs come from the oracle restatement (unpinned) --
              they guard against regressions, not against the reference.
Each fixture also records the sha256 of its generated inputs, pinning the
product's generators.
"""
import hashlib
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import low_latency_inference_gpu_b200 as ll  # noqa: E402
import oracle  # noqa: E402


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def bits(a):
    return [int(v) for v in np.ascontiguousarray(a, np.float32).ravel().view(np.uint32)]


def main():
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    out = {}

    # ---- the reference's own bench fixture ----
    dims = [512, 256, 64, 1]
    x = oracle.ref_host_init(512, 1.0, 1)
    Ws, bs = [], []
    for l in range(3):
        Ws.append(oracle.ref_host_init(dims[l] * dims[l + 1], 0.02, 2 + 2 * l).reshape(dims[l + 1], dims[l]))
        bs.append(oracle.ref_host_init(dims[l + 1], 0.01, 3 + 2 * l))
    y1 = oracle.ref_gemv_bias_relu(Ws[0], bs[0], x, True)
    y2 = oracle.ref_gemv_bias_relu(Ws[1], bs[1], y1, True)
    y3 = oracle.ref_gemv_bias_relu(Ws[2], bs[2], y2, False)
    out["ref_bench"] = dict(dims=dims, inputs_sha256=sha(x, *Ws, *bs), y1=bits(y1), y2=bits(y2), y3=bits(y3))

    # ---- fp32 workloads through the reference chain ----
    for cfg, n in ((0, 8), (1, 4)):
        net, Ws, bs = ll.config_params(cfg)
        xs = ll.config_inputs(cfg, n)
        relu = [a == ll.ACT_RELU for a in net.acts]
        y = oracle.ref_mlp(net.dims, relu, Ws, bs, xs)
        out[f"cfg{cfg}"] = dict(dims=net.dims, n=n, inputs_sha256=sha(xs, *Ws, *bs), y=bits(y))

    # ---- bf16 / int8 workloads through the restatement ----
    net, Ws, bs = ll.config_params(2)
    xs = ll.config_inputs(2, 2)
    Wb = [ll.f32_to_bf16(w) for w in Ws]
    y = oracle.mlp_bf16(net.dims, net.acts, Wb, bs, xs)
    out["cfg2"] = dict(dims=net.dims, n=2, inputs_sha256=sha(xs, *Ws, *bs), weights_sha256=sha(*Wb), y=bits(y))

    net, Ws, bs = ll.config_params(3)
    xs = ll.config_inputs(3, 2)
    qs = [ll.quantize_int8_rows(w) for w in Ws]
    y = oracle.mlp_int8(net.dims, net.acts, [q for q, _ in qs], [s for _, s in qs], bs, xs)
    out["cfg3"] = dict(dims=net.dims, n=2, inputs_sha256=sha(xs, *Ws, *bs),
                       weights_sha256=sha(*[q for q, _ in qs], *[s for _, s in qs]), y=bits(y))

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
