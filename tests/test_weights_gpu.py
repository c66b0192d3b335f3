"""Engines built from weight files give the oracle's outputs (need a B200).
Tolerances: fp32 1e-5, int8 2e-2 (norm-wise relative error)."""
import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]


def test_resident_engine_from_file(tmp_path):
    net, Ws, bs = ll.config_params(0)
    path = str(tmp_path / "c0.llw")
    ll.save_weights(path, net, Ws, bs)
    net2, W2, b2, _ = ll.load_weights(path)
    xs = ll.config_inputs(0, 16)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with ll.Engine(net2, W2, b2) as e:
        for i in range(16):
            assert rel_err(e.infer(xs[i])[0], ref[i]) <= 1e-5


def test_batched_int8_from_file(tmp_path):
    net, Ws, bs = ll.config_params(3)
    Wd, bd, sd = ll.device_weights(net, Ws, bs)
    path = str(tmp_path / "c3.llw")
    ll.save_weights(path, net, Wd, bd, sd)
    net2, Wq, b2, s2 = ll.load_weights(path)
    xs = ll.config_inputs(3, 8)
    ref = oracle.mlp_int8(net.dims, net.acts, Wq, s2, b2, xs)
    with ll.BatchedMLP(net2, Wq, b2, s2) as m:
        assert rel_err(m.infer(xs), ref) <= 2e-2
