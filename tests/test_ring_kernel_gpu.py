"""Pipelined ring kernel (engine kernel variant 4; needs a B200).

An I/O CTA reads the waiting ring slots and writes the replies while the compute CTAs run
the layers of the previous pass, with the weights blocked for many rows per pass.  Every
reply must equal, bit for bit, this kernel's reply to the same request served alone (a pass
of one row), whatever the size of the pass that carried it, and be within 1e-5 of the
oracle; the register-resident kernel's reply (another summation order) is within 1e-5 too."""
import time

import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import close, rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]


def opts(**kw):
    o = ll.default_opts()
    o.mailbox_format = 1
    o.kernel_variant = ll.VARIANT_PIPELINED_RING
    for k, v in kw.items():
        setattr(o, k, v)
    return o


@pytest.fixture(scope="module")
def cfg0():
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 64)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with ll.Engine(net, Ws, bs, opts=opts()) as one:  # this kernel, one request (one row) per pass
        assert one.info().kernel_variant == ll.VARIANT_PIPELINED_RING
        single = np.stack([one.infer(xs[i])[0] for i in range(xs.shape[0])])
    return net, Ws, bs, xs, ref, single


def test_single_requests_against_the_oracle_and_the_register_resident_kernel(cfg0):
    net, Ws, bs, xs, ref, single = cfg0
    o = ll.default_opts()
    o.mailbox_format = 1
    with ll.Engine(net, Ws, bs, opts=o) as e2:
        assert e2.info().kernel_variant == ll.VARIANT_REGISTER_RESIDENT
        y2 = np.stack([e2.infer(xs[i])[0] for i in range(xs.shape[0])])
    with ll.Engine(net, Ws, bs, opts=opts()) as e:
        inf = e.info()
        assert inf.kernel_variant == ll.VARIANT_PIPELINED_RING and inf.cluster_size == 8
        ys = np.stack([e.infer(xs[i])[0] for i in range(xs.shape[0])])
        assert e.info().status == ll.LL_OK
    assert np.array_equal(ys, single)  # deterministic from launch to launch
    assert rel_err(ys, ref) <= 1e-5 and close(ys, ref, 1e-5)
    assert close(ys, y2, 1e-5)


@pytest.mark.parametrize("ring,micro", [(16, 4), (64, 16), (32, 16), (8, 1)])
def test_ring_kept_full(cfg0, ring, micro):
    net, Ws, bs, xs, ref, single = cfg0
    n = 5000
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=ring, micro_batch=micro)) as e:
        lat, el, ys = e.bench_ring(xs, n, ring, keep_outputs=True)
        e.stop()
        inf = e.info()
        assert inf.status == ll.LL_OK
        assert inf.rows == n
    rows = np.arange(n) % xs.shape[0]
    assert np.array_equal(ys, single[rows])
    assert rel_err(ys, ref[rows]) <= 1e-5
    assert np.all(np.isfinite(lat)) and el > 0
    if micro > 1:
        assert inf.passes < inf.rows


@pytest.mark.parametrize("ring,micro", [(64, 16), (16, 4)])
def test_ring_kept_full_from_two_host_threads(cfg0, ring, micro):
    # ll_engine_bench_ring_mt: a poster thread fills the free slots while the caller collects
    net, Ws, bs, xs, ref, single = cfg0
    n = 20000
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=ring, micro_batch=micro)) as e:
        lat, el, ys = e.bench_ring_mt(xs, n, ring, keep_outputs=True)
        lat2, _, ys2 = e.bench_ring(xs, 1000, ring, keep_outputs=True)  # the engine goes on after it
        e.stop()
        inf = e.info()
        assert inf.status == ll.LL_OK and inf.rows == n + 1000
    rows = np.arange(n) % xs.shape[0]
    assert np.array_equal(ys, single[rows])
    assert np.array_equal(ys2, single[np.arange(1000) % xs.shape[0]])
    assert rel_err(ys, ref[rows]) <= 1e-5
    assert np.all(np.isfinite(lat)) and np.all(lat > 0) and el > 0


@pytest.mark.parametrize("n_eng", [2, 4])
def test_several_engines_on_one_gpu(cfg0, n_eng):
    # the e2e throughput leg: several ring engines on one GPU, each kept full by its own host
    # thread (ctypes releases the GIL); every reply equals the one-at-a-time reply
    import threading

    net, Ws, bs, xs, ref, single = cfg0
    n = 4000
    engs = [ll.Engine(net, Ws, bs, opts=opts(ring_slots=64, micro_batch=16)) for _ in range(n_eng)]
    out, errors = [None] * n_eng, []

    def drive(i):
        try:
            out[i] = engs[i].bench_ring(xs[i:] if i else xs, n, 64, keep_outputs=True)[2]
        except Exception as ex:  # noqa: BLE001 - reported below
            errors.append(repr(ex))

    try:
        threads = [threading.Thread(target=drive, args=(i,)) for i in range(n_eng)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(120)
        assert not errors, errors
        for e in engs:
            e.stop()
            assert e.info().status == ll.LL_OK
    finally:
        for e in engs:
            e.close()
    for i in range(n_eng):
        rows = i + np.arange(n) % (xs.shape[0] - i) if i else np.arange(n) % xs.shape[0]
        assert np.array_equal(out[i], single[rows])
        assert rel_err(out[i], ref[rows]) <= 1e-5


def test_bursts_are_taken_several_requests_per_pass(cfg0):
    net, Ws, bs, xs, ref, single = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=32, micro_batch=16)) as e:
        n = 0
        bursts = (16, 1, 7, 16, 3, 12)
        for burst in bursts:
            seqs = e.submit_many(xs[n:n + burst])
            for i in (range(burst) if burst % 2 else reversed(range(burst))):
                assert np.array_equal(e.poll(seqs[i])[0], single[n + i])
            n += burst
        e.stop()
        inf = e.info()
        assert inf.status == ll.LL_OK and inf.rows == n
        assert inf.passes < inf.rows


def test_poisson_replies_at_one_million_per_second(cfg0):
    net, Ws, bs, xs, ref, single = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=64, micro_batch=16)) as e:
        lat, el, ys, idx = e.serve_poisson(xs, 30000, 1_000_000.0, seed=5, keep_outputs=True)
        e.stop()
        assert e.info().status == ll.LL_OK
    assert np.array_equal(idx, np.arange(30000))
    assert np.array_equal(ys, single[idx % xs.shape[0]])
    assert np.all(np.isfinite(lat))


def test_idle_relaunch_and_stop(cfg0):
    net, Ws, bs, xs, ref, single = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=16, micro_batch=16, idle_timeout_ns=30_000_000)) as e:
        n = 0
        for rnd in range(3):
            seqs = e.submit_many(xs[n:n + 9])
            for i, s in enumerate(seqs):
                assert np.array_equal(e.poll(s)[0], single[n + i])
            n += 9
            time.sleep(0.15)  # the kernel leaves after 30 ms idle; the next submit relaunches it
        assert e.info().launches >= 3
        for i in range(n, n + 5):
            assert np.array_equal(e.infer(xs[i])[0], single[i])
        e.stop()
        assert e.info().status == ll.LL_OK


def test_refused_where_it_cannot_run(cfg0):
    net, Ws, bs, xs, ref, single = cfg0
    o = opts()
    o.mailbox_format = 0  # the TickBuffer
    with pytest.raises(ll.LLError) as err:
        ll.Engine(net, Ws, bs, opts=o)
    assert err.value.code == ll.LL_ERR_UNSUPPORTED
    with pytest.raises(ll.LLError) as err:  # 4 CTAs per cluster: no room for multi-row passes
        ll.Engine(net, Ws, bs, opts=opts(cluster_size=4))
    assert err.value.code == ll.LL_ERR_UNSUPPORTED


@pytest.mark.parametrize("n", [1, 16, 37, 3000])
def test_device_queue_on_the_ring_kernel(cfg0, n):
    """A device queue (inputs in HBM) through the pipelined ring kernel: the reader takes up to
    16 queued requests per pass, the gatherer writes the replies to the output queue, and the
    last pass tells every CTA to leave.  Replies are bit-identical to single requests; the
    mailbox works again after the queue launch."""
    torch = pytest.importorskip("torch")
    net, Ws, bs, xs, ref, single = cfg0
    idx = np.arange(n) % xs.shape[0]
    dx = torch.from_numpy(np.ascontiguousarray(xs[idx])).cuda()
    dy = torch.full((n, 16), float("nan"), device="cuda")
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=64, micro_batch=16)) as e:
        ms = e.run_queue(dx.data_ptr(), dy.data_ptr(), n, 1)
        inf = e.info()
        assert inf.status == ll.LL_OK and ms > 0
        assert inf.rows == n and inf.passes == -(-n // 16)  # full passes of 16, the rest in one
        assert np.array_equal(e.infer(xs[5])[0], single[5])
    assert np.array_equal(dy.cpu().numpy(), single[idx])
