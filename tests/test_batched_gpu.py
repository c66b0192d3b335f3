"""Batched dense path on the tensor cores (tcgen05), against the oracle (need a B200).

Tolerances (norm-wise relative error max|y - ref| / max|ref|, per weight type as
stated for the workloads): bf16 1e-2, int8 2e-2.  The oracle rounds the input and
every hidden activation to bf16 like the device path; only the summation order
differs (tensor-core tiles and split-K partials against a sequential sum).  The
device path itself is deterministic: split-K partials are added in a fixed order.
"""
import numpy as np
import pytest
import torch

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import close, rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

TOL = {ll.W_BF16: 1e-2, ll.W_I8: 2e-2}


def params(net, seed=0):
    Ws, bs = ll.init_params(net, ll.INIT_NORMAL_FANIN, seed)
    return Ws, bs


def oracle_out(net, Ws, bs, xs):
    if net.wtype == ll.W_BF16:
        return oracle.mlp_bf16(net.dims, net.acts, [ll.f32_to_bf16(w) for w in Ws], bs, xs)
    qs = [oracle.quantize_int8_rows(w) for w in Ws]
    return oracle.mlp_int8(net.dims, net.acts, [q for q, _ in qs], [s for _, s in qs], bs, xs)


def make(net, Ws, bs, **kw):
    Wd, bd, sd = ll.device_weights(net, Ws, bs)
    return ll.BatchedMLP(net, Wd, bd, sd, device=0, opts=ll.batched_opts(**kw) if kw else None)


def run_device(m, xs):
    dx = torch.from_numpy(np.ascontiguousarray(xs, np.float32)).cuda()
    dy = torch.empty((xs.shape[0], m.out_dim), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    m.forward(dx.data_ptr(), dy.data_ptr(), xs.shape[0], s.cuda_stream)
    m.check(s.cuda_stream)
    return dy.cpu().numpy()


@pytest.mark.parametrize("wtype", [ll.W_BF16, ll.W_I8])
@pytest.mark.parametrize("bn,splits", [(64, 1), (128, 1), (256, 1), (64, 2), (64, 4), (128, 2), (128, 4)])
def test_small_net_every_tile_shape(wtype, bn, splits):
    # 256 -> 256 -> 256, ReLU then identity: every kernel variant, with and without split-K
    net = ll.mlp([256, 256, 256], ll.ACT_RELU, ll.ACT_IDENTITY, wtype, 200)
    Ws, bs = params(net, 11)
    xs = ll.fill_uniform(200 * 256, -1.0, 1.0, 12).reshape(200, 256)
    with make(net, Ws, bs, bn=bn, splits=splits) as m:
        info = m.info()
        assert info["bn"] == [bn, bn] and info["splits"] == [splits, splits]
        y = run_device(m, xs)
    ref = oracle_out(net, Ws, bs, xs)
    assert close(y, ref, TOL[wtype]), (bn, splits)


@pytest.mark.parametrize("rows", [1, 7, 128, 129, 256])
def test_config3_int8_rows(rows):
    # 1024 -> 2048 x 6 -> 256 int8 weights, per-channel scales, bf16 activations; ragged row counts
    net = ll.config_net(3)
    Ws, bs = ll.config_params(3)[1:]
    xs = ll.config_inputs(3, rows)
    with make(net, Ws, bs) as m:
        y = run_device(m, xs)
    check = np.r_[0:min(rows, 12), max(0, rows - 12):rows]
    ref = oracle_out(net, Ws, bs, xs[check])
    assert close(y[check], ref, TOL[ll.W_I8])


def test_config3_repeated_forwards_are_identical():
    # the K splits of a tile add their partials in cluster-rank order through shared
    # memory: no atomics, no workspace, so every forward gives the same bits
    net = ll.config_net(3)
    Ws, bs = ll.config_params(3)[1:]
    xs = ll.config_inputs(3, 256)
    with make(net, Ws, bs) as m:
        ys = [run_device(m, xs) for _ in range(3)]
        y_host = m.infer(xs)
    assert all(np.array_equal(ys[0], y) for y in ys[1:])
    assert np.array_equal(ys[0], y_host)


def test_graph_replay_matches_direct_launches():
    # forwards replayed from the captured CUDA graph (default) against per-layer launches
    # from the host; a new row count or new pointers make the object capture again
    net = ll.config_net(3)
    Ws, bs = ll.config_params(3)[1:]
    xs = ll.config_inputs(3, 256)
    with make(net, Ws, bs) as g, make(net, Ws, bs, graph=0) as d:
        for rows in (256, 100, 256):
            yg = run_device(g, xs[:rows])
            yd = run_device(d, xs[:rows])
            assert np.array_equal(yg, yd), rows
    ref = oracle_out(net, Ws, bs, xs[:8])
    assert rel_err(yg[:8], ref) <= TOL[ll.W_I8]


@pytest.mark.parametrize("rows", [1, 2, 4, 8, 16, 32])
def test_config2_bf16_gelu_batch_sweep(rows):
    net = ll.config_net(2)
    Ws, bs = ll.config_params(2)[1:]
    xs = ll.config_inputs(2, rows)
    with make(net, Ws, bs) as m:
        y = run_device(m, xs)
    ref = oracle_out(net, Ws, bs, xs)
    assert close(y, ref, TOL[ll.W_BF16])


@pytest.mark.parametrize("rows", [1, 3, 5, 13, 31])
def test_small_batch_kernel_ragged_rows(rows):
    # config 2 on the small-batch kernel (one cooperative launch per forward)
    net = ll.config_net(2)
    Ws, bs = ll.config_params(2)[1:]
    xs = ll.config_inputs(2, rows)
    with make(net, Ws, bs) as m:
        assert m.info()["kind"] == [ll.KERNEL_GEMV] * 6
        y = run_device(m, xs)
    assert close(y, oracle_out(net, Ws, bs, xs), TOL[ll.W_BF16])


@pytest.mark.parametrize("rows", [1, 32])
def test_config2_on_split_k_tiles(rows):
    net = ll.config_net(2)
    Ws, bs = ll.config_params(2)[1:]
    xs = ll.config_inputs(2, rows)
    with make(net, Ws, bs, kernel=ll.KERNEL_SPLITK) as m:
        assert m.info()["kind"] == [1] * 6
        y = run_device(m, xs)
    assert rel_err(y, oracle_out(net, Ws, bs, xs)) <= TOL[ll.W_BF16]


@pytest.mark.parametrize("rows", [1, 6, 32])
def test_small_batch_kernel_int8(rows):
    # int8 weights with per-channel scales; 384 and 128 outputs leave CTAs with 3, 2, 1 or 0 rows
    net = ll.mlp([256, 512, 384, 128], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_I8, 32)
    Ws, bs = params(net, 31)
    xs = ll.fill_uniform(rows * 256, -1.0, 1.0, 32).reshape(rows, 256)
    with make(net, Ws, bs) as m:
        assert m.info()["kind"] == [ll.KERNEL_GEMV] * 3
        y = run_device(m, xs)
    assert close(y, oracle_out(net, Ws, bs, xs), TOL[ll.W_I8])


def test_config3_single_row_on_small_batch_kernel():
    net = ll.config_net(3, 1)
    Ws, bs = ll.config_params(3)[1:]
    xs = ll.config_inputs(3, 1)
    with make(net, Ws, bs) as m:
        assert m.info()["kind"] == [ll.KERNEL_GEMV] * 8
        y = run_device(m, xs)
    assert rel_err(y, oracle_out(net, Ws, bs, xs)) <= TOL[ll.W_I8]


def test_small_batch_kernel_repeated_forwards_are_identical():
    # every forward tags its hand-off words anew; 11 000 forwards of 6 layers pass the
    # 16-bit tag range once, so the words are cleared and the tags start over
    net = ll.config_net(2)
    Ws, bs = ll.config_params(2)[1:]
    xs = ll.config_inputs(2, 32)
    with make(net, Ws, bs) as m:
        first = run_device(m, xs)
        dx = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
        dy = torch.empty((32, m.out_dim), dtype=torch.float32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        for i in range(11000):
            rows = (1, 4, 9, 32)[i % 4]
            m.forward(dx.data_ptr(), dy.data_ptr(), rows, s)
        m.check(s)
        last = run_device(m, xs)
        one = run_device(m, xs[:1])
        one_again = run_device(m, xs[:1])
    assert np.array_equal(first, last)
    assert np.array_equal(one, one_again)
    # another row count maps K onto the lanes differently: same values up to summation order
    assert rel_err(one, first[:1]) <= 1e-5


def test_small_batch_wait_runs_out_and_is_reported():
    # a 1 ns bound: the layer barrier waits give up, every CTA lets its weight copies land
    # and returns; the host reads the status, and the object is usable afterwards
    net = ll.config_net(2)
    Ws, bs = ll.config_params(2)[1:]
    xs = ll.config_inputs(2, 4)
    with make(net, Ws, bs, wait_ns=1) as m:
        with pytest.raises(ll.LLError) as e:
            run_device(m, xs)
        assert e.value.code == ll.LL_ERR_DEVICE_FAULT
        m.check(torch.cuda.current_stream().cuda_stream)  # the status was cleared
    with make(net, Ws, bs) as m:
        y = run_device(m, xs)
    assert rel_err(y, oracle_out(net, Ws, bs, xs)) <= TOL[ll.W_BF16]


def test_without_programmatic_launch_matches():
    net = ll.config_net(2)
    Ws, bs = ll.config_params(2)[1:]
    xs = ll.config_inputs(2, 32)
    with make(net, Ws, bs) as a, make(net, Ws, bs, pdl=0) as b:
        assert np.array_equal(run_device(a, xs), run_device(b, xs))


@pytest.mark.parametrize("wtype", [ll.W_BF16, ll.W_I8])
def test_weights_in_tmem_tiles_small_net(wtype):
    # 256 -> 384 -> 256, 512 rows, forced onto the weights-in-TMEM kernel (A operand in TMEM)
    net = ll.mlp([256, 384, 256], ll.ACT_RELU, ll.ACT_IDENTITY, wtype, 512)
    Ws, bs = params(net, 21)
    xs = ll.fill_uniform(512 * 256, -1.0, 1.0, 22).reshape(512, 256)
    with make(net, Ws, bs, kernel=2) as m:
        assert m.info()["kind"] == [2, 2]
        y = run_device(m, xs)
        y300 = run_device(m, xs[:300])  # a ragged row count: the second row block is partial
    ref = oracle_out(net, Ws, bs, xs)
    assert close(y, ref, TOL[wtype])
    assert np.array_equal(y300, y[:300])


@pytest.mark.parametrize("wtype", [ll.W_BF16, ll.W_I8])
def test_weights_in_tmem_tiles_on_sm_pairs(wtype):
    # 256 -> 512 -> 256 over 512 rows: both layers have an even number of 128-channel tiles, so
    # the weights-in-TMEM tiles run on SM pairs (one 2-SM MMA per 256-channel tile); the same
    # net with one CTA per tile is the comparison
    net = ll.mlp([256, 512, 256], ll.ACT_RELU, ll.ACT_IDENTITY, wtype, 512)
    Ws, bs = params(net, 23)
    xs = ll.fill_uniform(512 * 256, -1.0, 1.0, 24).reshape(512, 256)
    with make(net, Ws, bs, kernel=2, sm_pairs=1) as m:
        y = run_device(m, xs)
        y300 = run_device(m, xs[:300])
    with make(net, Ws, bs, kernel=2) as m1:
        y1 = run_device(m1, xs)
    ref = oracle_out(net, Ws, bs, xs)
    assert close(y, ref, TOL[wtype]) and close(y1, ref, TOL[wtype])
    assert np.array_equal(y300, y[:300])
    assert np.array_equal(y, y1)  # the same MMA sums, K step by K step (measured bit-identical)


def test_config3_stacked_batches_auto():
    net = ll.config_net(3, 2048)
    Ws, bs = ll.config_params(3)[1:]
    xs = ll.config_inputs(3, 2048)
    with make(net, Ws, bs) as m:
        assert m.info()["kind"][:7] == [2] * 7
        y = run_device(m, xs)
    check = np.r_[0:8, 1020:1030, 2040:2048]
    ref = oracle_out(net, Ws, bs, xs[check])
    assert close(y[check], ref, TOL[ll.W_I8])
