"""The engine's resident small-batch kernel (kernel variant 3: one CTA per SM, each holding its
row slice of every layer in shared memory for the whole launch) behind the TickBuffer mailbox
(need a B200).  Outputs are checked against the oracle: bf16 1e-2, int8 2e-2 norm-wise relative."""
import time

import numpy as np
import pytest
import torch

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]


def opts(**kw):
    o = ll.default_opts()
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def cfg_net(cfg, rows):
    """A workload's net at max_batch = rows, its weights in the engine's types."""
    net = ll.config_net(cfg, rows)
    Ws, bs = ll.init_params(net, ll.CONFIGS[cfg]["init"], 0)
    Wd, bd, sd = ll.device_weights(net, Ws, bs)
    return net, Wd, bd, sd


def cfg2(rows):
    return cfg_net(2, rows)


def bf16_ref(net, Wd, bd, xs):
    return oracle.mlp_bf16(net.dims, net.acts, Wd, bd, xs)


@pytest.mark.parametrize("max_rows,rows", [(1, [1]), (4, [1, 3, 4]), (8, [8, 5]), (32, [32, 1, 17])])
def test_config2_rows_through_the_mailbox(max_rows, rows):
    net, Wd, bd, sd = cfg2(max_rows)
    with ll.Engine(net, Wd, bd, sd, device=0) as e:
        info = e.info()
        if max_rows == 1:  # batch 1: the deep register-resident kernel, chosen automatically
            assert info.kernel_variant == ll.VARIANT_REGISTER_RESIDENT
        else:  # chosen automatically (9 MB of bf16)
            assert info.kernel_variant == ll.VARIANT_RESIDENT_SMALL_BATCH
            assert info.threads == 256 and info.image_bytes > 0
        for i, r in enumerate(rows * 3):  # the same engine serves every row count up to max_batch
            xs = ll.config_inputs(2, 40)[i:i + r]
            assert rel_err(e.infer(xs), bf16_ref(net, Wd, bd, xs)) <= 1e-2
        assert e.info().status == ll.LL_OK


def test_matches_the_per_forward_small_batch_kernel():
    # same instantiation (8 rows), same lane mapping and summation order: bit-identical outputs
    net, Wd, bd, sd = cfg2(8)
    xs = ll.config_inputs(2, 8)
    with ll.BatchedMLP(net, Wd, bd, sd, device=0) as m:
        ref = m.infer(xs)
    with ll.Engine(net, Wd, bd, sd, device=0) as e:
        assert np.array_equal(e.infer(xs), ref)


def test_int8_config3_single_rows():
    net, Wd, bd, sd = cfg_net(3, 1)
    xs = ll.config_inputs(3, 4)
    ref = oracle.mlp_int8(net.dims, net.acts, Wd, sd, bd, xs)
    with ll.Engine(net, Wd, bd, sd, device=0) as e:
        assert e.info().kernel_variant == ll.VARIANT_RESIDENT_SMALL_BATCH
        ys = np.concatenate([e.infer(xs[i:i + 1]) for i in range(4)])
    assert rel_err(ys, ref) <= 2e-2


@pytest.mark.parametrize("max_rows", [1, 16])
def test_queue_mode_and_tag_budget(max_rows):
    # 1 row hands off in 16-bit tags: 11 000 requests take two launches (65534 / 6 per launch)
    net, Wd, bd, sd = cfg2(max_rows)
    n = 11000 if max_rows == 1 else 600
    xs = ll.config_inputs(2, n * max_rows)
    dx = torch.from_numpy(xs).cuda()
    dy = torch.zeros(n * max_rows, net.dims[-1], device="cuda")
    with ll.Engine(net, Wd, bd, sd, device=0, opts=opts(kernel_variant=3)) as e:
        before = e.info().launches
        ms = e.run_queue(dx.data_ptr(), dy.data_ptr(), n, max_rows)
        inf = e.info()
        assert inf.status == ll.LL_OK and ms > 0
        assert inf.launches - before == (2 if max_rows == 1 else 1)
        assert inf.passes == n and inf.rows == n * max_rows
        # and the mailbox still works after the queue runs
        assert rel_err(e.infer(xs[:max_rows]), bf16_ref(net, Wd, bd, xs[:max_rows])) <= 1e-2
    y = dy.cpu().numpy()
    pick = np.r_[0:64, n * max_rows - 64:n * max_rows]  # both ends of the queue
    assert rel_err(y[pick], bf16_ref(net, Wd, bd, xs[pick])) <= 1e-2


def test_idle_exit_relaunch_and_stop():
    net, Wd, bd, sd = cfg2(4)
    xs = ll.config_inputs(2, 16)
    with ll.Engine(net, Wd, bd, sd, device=0, opts=opts(idle_timeout_ns=30_000_000)) as e:
        for rnd in range(3):
            x = xs[4 * rnd:4 * rnd + 4]
            assert rel_err(e.infer(x), bf16_ref(net, Wd, bd, x)) <= 1e-2
            time.sleep(0.15)  # the kernel leaves after 30 ms idle; the next request relaunches it
        assert e.info().launches >= 3
        e.stop()
        assert e.info().state == 4  # exited
        assert rel_err(e.infer(xs[12:16]), bf16_ref(net, Wd, bd, xs[12:16])) <= 1e-2


def test_forced_variant_is_refused_where_it_cannot_run():
    net, Wd, bd, sd = cfg2(4)
    with pytest.raises(ll.LLError) as e:
        ll.Engine(net, Wd, bd, sd, device=0, opts=opts(kernel_variant=3, mailbox_format=1))
    assert e.value.code == ll.LL_ERR_UNSUPPORTED
    f32 = ll.mlp([64, 256, 16], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 1)
    W, b = ll.init_params(f32, ll.INIT_XAVIER_UNIFORM, 0)
    with pytest.raises(ll.LLError) as e:
        ll.Engine(f32, W, b, device=0, opts=opts(kernel_variant=3))
    assert e.value.code == ll.LL_ERR_UNSUPPORTED
    # a small bf16 net stays on the generic kernel unless forced
    small = ll.mlp([256, 256, 64], ll.ACT_GELU, ll.ACT_IDENTITY, ll.W_BF16, 4)
    W, b = ll.init_params(small, ll.INIT_NORMAL_FANIN, 0)
    Wd, bd, sd = ll.device_weights(small, W, b)
    with ll.Engine(small, Wd, bd, sd, device=0) as eng:
        assert eng.info().kernel_variant == ll.VARIANT_GENERIC
    with ll.Engine(small, Wd, bd, sd, device=0, opts=opts(kernel_variant=3)) as eng:
        x = ll.config_inputs(2, 3)
        assert rel_err(eng.infer(x), oracle.mlp_bf16(small.dims, small.acts, Wd, bd, x)) <= 1e-2


def test_one_row_on_the_tagged_mailbox():
    # x arrives with the doorbell in tagged chunks and y leaves in tagged chunks; an idle exit
    # and relaunch continue the sequence; the replies equal the TickBuffer engine's bit for bit
    net, Wd, bd, sd = cfg2(1)
    xs = ll.config_inputs(2, 12)
    ref = bf16_ref(net, Wd, bd, xs)
    with ll.Engine(net, Wd, bd, sd, device=0,
                   opts=opts(mailbox_format=1, idle_timeout_ns=30_000_000, kernel_variant=3)) as e:
        assert e.info().kernel_variant == ll.VARIANT_RESIDENT_SMALL_BATCH
        ys = [e.infer(xs[i:i + 1]) for i in range(6)]
        time.sleep(0.15)  # the kernel leaves after 30 ms idle; the next request relaunches it
        ys += [e.infer(xs[i:i + 1]) for i in range(6, 12)]
        assert e.info().launches >= 2 and e.info().status == ll.LL_OK
    ys = np.concatenate(ys)
    assert rel_err(ys, ref) <= 1e-2
    with ll.Engine(net, Wd, bd, sd, device=0, opts=opts(kernel_variant=3)) as tick:
        assert np.array_equal(np.concatenate([tick.infer(xs[i:i + 1]) for i in range(12)]), ys)
