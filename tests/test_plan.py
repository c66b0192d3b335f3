"""Planner and weight-image packing, checked on the CPU by emulating the kernel's
data movement (tests/kernel_emulator.py) against the oracle."""
import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import rel_err
from kernel_emulator import run as emulate


def _opts(**kw):
    o = ll.default_opts()
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def _oracle(net, Ws, bs, xs):
    if net.wtype == ll.W_F32:
        return oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    if net.wtype == ll.W_BF16:
        return oracle.mlp_bf16(net.dims, net.acts, [ll.f32_to_bf16(w) for w in Ws], bs, xs)
    qs = [oracle.quantize_int8_rows(w) for w in Ws]
    return oracle.mlp_int8(net.dims, net.acts, [q for q, _ in qs], [s for _, s in qs], bs, xs)


TOL = {ll.W_F32: 1e-5, ll.W_BF16: 1e-2, ll.W_I8: 2e-2}


def _check(net, Ws, bs, xs, opts=None):
    Wd, bd, sd = ll.device_weights(net, Ws, bs)
    plan, img = ll.plan_net(net, Wd, bd, sd, opts, want_images=True)
    assert plan.smem_bytes <= 227 * 1024 - 4096
    y = emulate(plan, img, xs, net.dims[-1])
    ref = _oracle(net, Ws, bs, xs)
    assert rel_err(y, ref) <= TOL[net.wtype], rel_err(y, ref)
    return plan


def test_config0_plan_single_cluster_one_hop():
    net, Ws, bs = ll.config_params(0)
    plan = _check(net, Ws, bs, ll.config_inputs(0, 1))
    assert plan.n_stages == 1 and plan.cluster_size == 16
    modes = [plan.layers[l].mode for l in range(3)]
    assert modes == [0, 2, 3]  # replicated, row-split local, K-split gather: one DSMEM hop per request


@pytest.mark.parametrize("rep", [0, 1])
@pytest.mark.parametrize("C", [1, 2, 4, 8, 16])
def test_config0_every_cluster_size(C, rep):
    net, Ws, bs = ll.config_params(0)
    if C == 1:  # the 256x256 fp32 layer (256 KB) cannot live in one CTA's shared memory
        with pytest.raises(ll.LLError):
            ll.plan_net(net, opts=_opts(cluster_size=C, replicate_first=rep))
        return
    _check(net, Ws, bs, ll.config_inputs(0, 1), _opts(cluster_size=C, replicate_first=rep))


def test_reference_mlp_plan():
    net, Ws, bs = ll.config_params("ref")
    _check(net, Ws, bs, ll.fill_normal(512, 0.0, 1.0, 1).reshape(1, 512))


def test_config1_pipelines_over_clusters():
    net, Ws, bs = ll.config_params(1)
    plan = _check(net, Ws, bs, ll.config_inputs(1, 1))
    assert plan.n_stages > 1
    assert plan.layers[plan.stage_last[0]].mode == 5  # handoff through global memory


@pytest.mark.parametrize("dims", [[33, 597, 293, 7], [5, 3], [17, 100, 1], [64, 64, 64, 64, 64, 3],
                                  [1, 1, 1], [300, 40]])
@pytest.mark.parametrize("C", [1, 4, 16])
def test_odd_shapes_fp32(dims, C):
    net = ll.mlp(dims, ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 1)
    Ws, bs = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 9)
    xs = ll.fill_uniform(dims[0], -1, 1, 4).reshape(1, -1)
    biggest = max(dims[l] * dims[l + 1] * 4 for l in range(len(dims) - 1))
    if biggest / C > 200 * 1024:  # a layer's slice cannot fit one CTA's shared memory
        with pytest.raises(ll.LLError):
            ll.plan_net(net, opts=_opts(cluster_size=C))
        return
    _check(net, Ws, bs, xs, _opts(cluster_size=C))


@pytest.mark.parametrize("wtype", [ll.W_BF16, ll.W_I8])
@pytest.mark.parametrize("rows", [1, 3, 5])
def test_low_precision_small_nets(wtype, rows):
    net = ll.mlp([40, 96, 72, 10], ll.ACT_GELU if wtype == ll.W_BF16 else ll.ACT_RELU, ll.ACT_IDENTITY, wtype, 5)
    Ws, bs = ll.init_params(net, ll.INIT_NORMAL_FANIN, 3)
    xs = ll.fill_uniform(rows * 40, -1, 1, 8).reshape(rows, 40)
    _check(net, Ws, bs, xs, _opts(cluster_size=4))


@pytest.mark.parametrize("stages", [2, 3])
def test_forced_multi_stage_batch(stages):
    net = ll.mlp([48, 128, 128, 128, 128, 20], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 6)
    Ws, bs = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 1)
    xs = ll.fill_normal(6 * 48, 0, 1, 2).reshape(6, 48)
    plan = _check(net, Ws, bs, xs, _opts(cluster_size=2, min_stages=stages))
    assert plan.n_stages == stages


def test_plan_rejects_too_large():
    net = ll.config_net(2)  # bf16 batch-32 activations do not fit this kernel's shared memory
    with pytest.raises(ll.LLError) as e:
        ll.plan_net(net)
    assert e.value.code == ll.LL_ERR_BAD_DESC


def test_plan_rejects_bad_descriptors():
    for net in (ll.Net([8, 4], [ll.ACT_RELU], ll.W_F32, 0), ll.Net([8, 4], [7], ll.W_F32, 1)):
        with pytest.raises(ll.LLError) as e:
            ll.plan_net(net)
        assert e.value.code == ll.LL_ERR_BAD_DESC
    o = _opts(cluster_size=3)
    with pytest.raises(ll.LLError) as e:
        ll.plan_net(ll.config_net(0), opts=o)
    assert e.value.code == ll.LL_ERR_INVALID_ARG
