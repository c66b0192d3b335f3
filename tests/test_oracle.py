"""The CPU oracle, pinned against the reference's own code and golden vectors (no GPU)."""
import hashlib

import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def unbits(v):
    return np.array(v, np.uint32).view(np.float32)


needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="reference CPU library (oracle/_ref) not built")


@needs_ref
@pytest.mark.parametrize("m,k,relu,seed", [(256, 512, True, 2), (64, 256, True, 4), (1, 64, False, 6),
                                           (33, 597, True, 11), (597, 293, False, 12), (1, 1, True, 13)])
def test_gemv_bit_exact_vs_reference(m, k, relu, seed):
    W = oracle.ref_host_init(m * k, 0.02, seed).reshape(m, k)
    b = oracle.ref_host_init(m, 0.01, seed + 100)
    x = oracle.ref_host_init(k, 1.0, seed + 200)
    y_ref = oracle.ref_gemv_bias_relu(W, b, x, relu)
    y = oracle.gemv_bias_act(W, b, x, ll.ACT_RELU if relu else ll.ACT_IDENTITY)
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))


@needs_ref
def test_mlp_chain_bit_exact_vs_reference():
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 16)
    y_ref = oracle.ref_mlp(net.dims, [a == ll.ACT_RELU for a in net.acts], Ws, bs, xs)
    y = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))


@needs_ref
def test_generator_matches_reference_host_init():
    for n, scale, seed in ((1000, 0.02, 2), (513, 1.0, 1), (7, 0.01, 7)):
        a = ll.fill_normal(n, 0.0, scale, seed)
        b = oracle.ref_host_init(n, scale, seed)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_golden_reference_bench(golden):
    g = golden["ref_bench"]
    dims = g["dims"]
    x = ll.fill_normal(512, 0.0, 1.0, 1)
    Ws = [ll.fill_normal(dims[l] * dims[l + 1], 0.0, 0.02, 2 + 2 * l).reshape(dims[l + 1], dims[l]) for l in range(3)]
    bs = [ll.fill_normal(dims[l + 1], 0.0, 0.01, 3 + 2 * l) for l in range(3)]
    assert sha(x, *Ws, *bs) == g["inputs_sha256"]
    y1 = oracle.gemv_bias_act(Ws[0], bs[0], x, ll.ACT_RELU)
    y2 = oracle.gemv_bias_act(Ws[1], bs[1], y1, ll.ACT_RELU)
    y3 = oracle.gemv_bias_act(Ws[2], bs[2], y2, ll.ACT_IDENTITY)
    assert np.array_equal(y1, unbits(g["y1"]))
    assert np.array_equal(y2, unbits(g["y2"]))
    assert np.array_equal(y3, unbits(g["y3"]))


@pytest.mark.parametrize("cfg", [0, 1])
def test_golden_fp32_configs(golden, cfg):
    g = golden[f"cfg{cfg}"]
    net, Ws, bs = ll.config_params(cfg)
    xs = ll.config_inputs(cfg, g["n"])
    assert sha(xs, *Ws, *bs) == g["inputs_sha256"]
    y = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    assert np.array_equal(y.ravel().view(np.uint32), np.array(g["y"], np.uint32))


def test_golden_bf16_config(golden):
    g = golden["cfg2"]
    net, Ws, bs = ll.config_params(2)
    xs = ll.config_inputs(2, g["n"])
    assert sha(xs, *Ws, *bs) == g["inputs_sha256"]
    Wb = [ll.f32_to_bf16(w) for w in Ws]
    assert sha(*Wb) == g["weights_sha256"]
    y = oracle.mlp_bf16(net.dims, net.acts, Wb, bs, xs)
    assert np.array_equal(y.ravel().view(np.uint32), np.array(g["y"], np.uint32))


def test_golden_int8_config(golden):
    g = golden["cfg3"]
    net, Ws, bs = ll.config_params(3)
    xs = ll.config_inputs(3, g["n"])
    assert sha(xs, *Ws, *bs) == g["inputs_sha256"]
    qs = [ll.quantize_int8_rows(w) for w in Ws]
    assert sha(*[q for q, _ in qs], *[s for _, s in qs]) == g["weights_sha256"]
    y = oracle.mlp_int8(net.dims, net.acts, [q for q, _ in qs], [s for _, s in qs], bs, xs)
    assert np.array_equal(y.ravel().view(np.uint32), np.array(g["y"], np.uint32))


@needs_ref
def test_bf16_int8_linear_part_follows_reference_order():
    """With bf16 / dequantised weights written as fp32, the restatement's pre-activation
    equals the reference's cpu_gemv_bias_relu bit for bit (only GELU / rounding are ours)."""
    rng = np.random.default_rng(5)
    W = rng.standard_normal((48, 96)).astype(np.float32)
    x = oracle.round_bf16(rng.standard_normal(96).astype(np.float32))
    b = np.zeros(48, np.float32)
    Wb = oracle.round_bf16(W)
    y_ref = oracle.ref_gemv_bias_relu(Wb, b, x, False)
    y = oracle.mlp_bf16([96, 48], [ll.ACT_IDENTITY], [ll.f32_to_bf16(W).reshape(48, 96)], [b], x)[0]
    assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    q, s = oracle.quantize_int8_rows(W)
    y_ref = oracle.ref_gemv_bias_relu(q.astype(np.float32), b, x, False) * s
    y = oracle.mlp_int8([96, 48], [ll.ACT_IDENTITY], [q], [s], [b], x)[0]
    assert np.array_equal(y.view(np.uint32), y_ref.astype(np.float32).view(np.uint32))


def test_bf16_rounding_round_to_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.005859375, -2.5e-3, 3.0e38, 1e-40, 0.0, -0.0], np.float32)
    ours = oracle.round_bf16(vals)
    # independent numpy statement of RNE on the top 16 bits
    u = vals.view(np.uint32).astype(np.uint64)
    exp = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(ours.view(np.uint32), exp.view(np.uint32))
    assert np.array_equal(ll.f32_to_bf16(vals), oracle.f32_to_bf16(vals))


def test_int8_quantisation_properties_and_product_agreement():
    rng = np.random.default_rng(7)
    W = (rng.standard_normal((64, 200)) / np.sqrt(200)).astype(np.float32)
    W[3] = 0.0  # all-zero row: scale 1, all q zero
    q, s = oracle.quantize_int8_rows(W)
    assert q.dtype == np.int8 and np.abs(q.astype(int)).max() <= 127
    assert s[3] == 1.0 and not q[3].any()
    rows = [i for i in range(64) if i != 3]
    assert (np.abs(q[rows]).max(axis=1) == 127).all()
    err = np.abs(q.astype(np.float32) * s[:, None] - W)
    assert (err <= s[:, None] * 0.5 + 1e-7).all()
    q2, s2 = ll.quantize_int8_rows(W)
    assert np.array_equal(q, q2) and np.array_equal(s, s2)


def test_gelu_restatement_values():
    x = np.array([-3.0, -1.0, 0.0, 0.5, 2.0], np.float32)
    from math import erf, sqrt

    want = np.array([0.5 * v * (1 + erf(v / sqrt(2))) for v in x], np.float32)
    W = np.eye(5, dtype=np.float32)
    y = oracle.gemv_bias_act(W, np.zeros(5, np.float32), x, ll.ACT_GELU)
    assert np.allclose(y, want, rtol=1e-6, atol=1e-7)


def test_kmajor_packing_matches_reference_layout():
    rng = np.random.default_rng(3)
    W = rng.standard_normal((37, 19)).astype(np.float32)
    a = oracle.pack_rm_to_kmajor_padded(W, 64)
    b = ll.pack_rm_to_kmajor_padded(W, 64)
    assert np.array_equal(a, b)
    assert np.array_equal(a[:, :37], W.T) and not a[:, 37:].any()
    bp = ll.pack_bias_padded(np.arange(37, dtype=np.float32), 64)
    assert np.array_equal(bp[:37], np.arange(37)) and not bp[37:].any()


def test_stats_match_reference_conventions():
    rng = np.random.default_rng(1)
    xs = rng.exponential(3.0, 1001)
    st = ll.compute_stats(xs)
    for p, key in ((0.5, "p50"), (0.9, "p90"), (0.99, "p99")):
        assert st[key] == pytest.approx(oracle.percentile_linear(xs, p), rel=1e-12)
    assert st["min"] == xs.min() and st["max"] == xs.max()
    assert st["sd"] == pytest.approx(np.std(xs), rel=1e-9)
    assert ll.compute_stats([4.0])["p99"] == 4.0
    assert ll.compute_stats([])["p50"] == 0.0


@pytest.mark.parametrize("cfg", [0, 1, 2, 3])
def test_oracle_workload_generators_match_the_product_generators(cfg):
    # bench.py's reference arm draws its weights and inputs from oracle/gen.cpp so that it
    # loads no product library; both generators must give the same bytes
    dims, acts, Wo, bo = oracle.workload_params(cfg)
    net, Wp, bp = ll.config_params(cfg)
    assert dims == net.dims and acts == net.acts
    assert all(np.array_equal(a, b) for a, b in zip(Wo, Wp))
    assert all(np.array_equal(a, b) for a, b in zip(bo, bp))
    assert np.array_equal(oracle.workload_inputs(cfg, 37), ll.config_inputs(cfg, 37))
    assert np.array_equal(oracle.fill_normal(1000, 0.0, 0.02, 2), ll.fill_normal(1000, 0.0, 0.02, 2))
