"""Request ring on the tagged mailbox and the open-loop Poisson driver (need a B200).

Outputs are checked against the oracle (fp32: 1e-5 norm-wise relative error)."""
import time

import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]


def opts(**kw):
    o = ll.default_opts()
    o.mailbox_format = 1
    for k, v in kw.items():
        setattr(o, k, v)
    return o


@pytest.fixture(scope="module")
def cfg0():
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 64)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    return net, Ws, bs, xs, ref


@pytest.mark.parametrize("variant", [1, 2])
def test_ring_holds_several_requests_in_flight(cfg0, variant):
    net, Ws, bs, xs, ref = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=4, kernel_variant=variant)) as e:
        assert e.info().kernel_variant == variant
        for base in range(0, 24, 4):
            seqs = [e.submit(xs[base + i]) for i in range(4)]
            with pytest.raises(ll.LLError) as busy:
                e.submit(xs[0])
            assert busy.value.code == ll.LL_ERR_BUSY
            order = [0, 1, 2, 3] if base % 8 == 0 else [2, 0, 3, 1]  # replies may be collected in any order
            for i in order:
                y = e.poll(seqs[i])
                assert rel_err(y[0], ref[base + i]) <= 1e-5
        # single requests keep working after the ring has wrapped several times
        for i in range(24, 40):
            assert rel_err(e.infer(xs[i])[0], ref[i]) <= 1e-5
        assert e.info().status == ll.LL_OK


def test_ring_survives_idle_relaunch(cfg0):
    net, Ws, bs, xs, ref = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=3, idle_timeout_ns=30_000_000)) as e:
        n = 0
        for rnd in range(3):
            seqs = [e.submit(xs[n + i]) for i in range(2)]
            for i, s in enumerate(seqs):
                assert rel_err(e.poll(s)[0], ref[n + i]) <= 1e-5
            n += 2
            time.sleep(0.15)  # the kernel leaves after 30 ms idle; the next submit relaunches it
        assert e.info().launches >= 3
        for i in range(n, n + 5):
            assert rel_err(e.infer(xs[i])[0], ref[i]) <= 1e-5


def test_poisson_stream_is_split_across_ranks_and_fully_served(cfg0):
    net, Ws, bs, xs, _ = cfg0
    total = 3000
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=8)) as e:
        lat0, el0 = e.serve_poisson(xs, total, 100_000.0, seed=5, rank=0, world=2)
        lat1, el1 = e.serve_poisson(xs, total, 100_000.0, seed=5, rank=1, world=2)
        lat, el = e.serve_poisson(xs, total, 100_000.0, seed=5)
        assert e.info().status == ll.LL_OK
    assert len(lat0) + len(lat1) == total and abs(len(lat0) - len(lat1)) < 300
    assert len(lat) == total
    for a in (lat0, lat1, lat):
        assert np.all(np.isfinite(a)) and a.min() > 0.5 and np.median(a) < 1000
    # 100k requests/s over 3000 requests is a 30 ms stream
    assert 0.025 < el < 0.5


@pytest.fixture(scope="module")
def single(cfg0):
    """Replies to every input row served alone (one request per pass)."""
    net, Ws, bs, xs, _ = cfg0
    with ll.Engine(net, Ws, bs, opts=opts()) as one:
        return np.stack([one.infer(xs[i])[0] for i in range(xs.shape[0])])


def test_micro_batched_ring_matches_single_requests(cfg0, single):
    # requests taken together from the ring run the same FMA sequence per row as one request
    # alone, so the replies are bit-identical to single requests (and within 1e-5 of the oracle).
    # ll_submit_many writes a whole burst before the device can take its first request, so
    # the device finds the rest of the burst waiting and takes it several rows per pass.
    net, Ws, bs, xs, ref = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=8, micro_batch=4)) as e:
        assert e.info().kernel_variant == 2
        n = 0
        bursts = (8, 1, 5, 3, 8, 7, 2, 6, 8, 8)  # ragged bursts; the ring wraps several times
        for burst in bursts:
            seqs = e.submit_many(xs[n:n + burst])
            assert len(seqs) == burst
            order = range(burst) if burst % 2 else reversed(range(burst))
            for i in order:
                y = e.poll(seqs[i])[0]
                assert np.array_equal(y, single[n + i])
                assert rel_err(y, ref[n + i]) <= 1e-5
            n += burst
        for i in range(n, n + 5):  # single requests on the same engine
            assert np.array_equal(e.infer(xs[i])[0], single[i])
        e.stop()
        inf = e.info()
        assert inf.status == ll.LL_OK
        assert inf.rows == n + 5
        # each burst of 8 takes at most 1 + 1 + 2 passes (the first poll may read a stale
        # seq_in; then one single-slot poll and 4-row reads), so the 8-row bursts alone save
        # at least 4 passes each
        assert inf.passes <= inf.rows - 4 * bursts.count(8)


def test_submit_many_refuses_a_burst_larger_than_the_free_slots(cfg0, single):
    net, Ws, bs, xs, _ = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=4, micro_batch=4)) as e:
        seqs = e.submit_many(xs[:3])
        with pytest.raises(ll.LLError) as busy:
            e.submit_many(xs[3:5])
        assert busy.value.code == ll.LL_ERR_BUSY
        seqs += e.submit_many(xs[3:4])
        for i, s in enumerate(seqs):
            assert np.array_equal(e.poll(s)[0], single[i])
    with ll.Engine(net, Ws, bs) as tb:  # the TickBuffer holds one request
        with pytest.raises(ll.LLError) as bad:
            tb.submit_many(xs[:2])
        assert bad.value.code == ll.LL_ERR_INVALID_ARG
        s = tb.submit_many(xs[:1])[0]
        assert np.array_equal(tb.poll(s)[0], single[0])


@pytest.mark.parametrize("kw", [dict(ring_slots=8, micro_batch=4), dict(ring_slots=8), dict(ring_slots=16, kernel_variant=1)])
def test_ring_kept_full_replies_match_single_requests(cfg0, single, kw):
    # the closed loop with every ring slot in use (bench_ring): replies come back in order and
    # equal, bit for bit, the replies of the same kernel to single requests
    net, Ws, bs, xs, ref = cfg0
    n = 3000
    if "kernel_variant" in kw:
        with ll.Engine(net, Ws, bs, opts=opts(kernel_variant=kw["kernel_variant"])) as one:
            single = np.stack([one.infer(xs[i])[0] for i in range(xs.shape[0])])
    with ll.Engine(net, Ws, bs, opts=opts(**kw)) as e:
        lat, el, ys = e.bench_ring(xs, n, kw["ring_slots"], keep_outputs=True)
        e.stop()
        inf = e.info()
        assert inf.status == ll.LL_OK
    rows = np.arange(n) % xs.shape[0]
    assert np.array_equal(ys, single[rows])
    assert rel_err(ys, ref[rows]) <= 1e-5
    assert np.all(np.isfinite(lat)) and lat.min() > 0.0 and el > 0.0
    if kw.get("micro_batch", 1) > 1:
        assert inf.passes < inf.rows  # a full ring is taken several requests per pass


def test_micro_batched_ring_survives_idle_relaunch(cfg0):
    net, Ws, bs, xs, ref = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=4, micro_batch=4, idle_timeout_ns=30_000_000)) as e:
        n = 0
        for rnd in range(3):
            seqs = [e.submit(xs[n + i]) for i in range(4)]
            for i, s in enumerate(seqs):
                assert rel_err(e.poll(s)[0], ref[n + i]) <= 1e-5
            n += 4
            time.sleep(0.15)  # the kernel leaves after 30 ms idle; the next submit relaunches it
        assert e.info().launches >= 3
        for i in range(n, n + 5):
            assert rel_err(e.infer(xs[i])[0], ref[i]) <= 1e-5


@pytest.mark.parametrize("kw", [dict(ring_slots=2, micro_batch=4),       # more rows than slots
                                dict(ring_slots=32, micro_batch=17),     # more than one pass carries
                                dict(ring_slots=8, micro_batch=4, kernel_variant=1),  # generic kernel
                                dict(ring_slots=8, micro_batch=4, cluster_size=4)])   # 66 weights/thread: 1 row
def test_micro_batch_is_refused_where_it_cannot_run(cfg0, kw):
    net, Ws, bs, _, _ = cfg0
    with pytest.raises(ll.LLError) as e:
        ll.Engine(net, Ws, bs, opts=opts(**kw))
    assert e.value.code == ll.LL_ERR_UNSUPPORTED


def test_micro_batched_poisson_stream_is_fully_served(cfg0, single):
    # 1 M requests/s offered overloads one GPU: the ring stays full and the device takes
    # several requests per pass; every reply is checked against the same request served
    # alone (bit for bit) and against the oracle
    net, Ws, bs, xs, ref = cfg0
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=8, micro_batch=4)) as e:
        lat, el, ys, idx = e.serve_poisson(xs, 20000, 1_000_000.0, seed=5, keep_outputs=True)
        e.stop()
        inf = e.info()
        assert inf.status == ll.LL_OK
    assert len(lat) == 20000 and np.all(np.isfinite(lat)) and lat.min() > 0.5
    assert np.array_equal(idx, np.arange(20000))  # one rank: every request, in arrival order
    rows = idx % xs.shape[0]
    assert np.array_equal(ys, single[rows])
    assert rel_err(ys, ref[rows]) <= 1e-5
    assert inf.passes < inf.rows  # an overloaded stream keeps the ring full: several rows per pass


def test_poisson_replies_of_two_ranks_cover_the_stream(cfg0, single):
    net, Ws, bs, xs, _ = cfg0
    total = 2000
    got = []
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=8, micro_batch=4)) as e:
        for rank in (0, 1):
            _, _, ys, idx = e.serve_poisson(xs, total, 200_000.0, seed=7, rank=rank, world=2, keep_outputs=True)
            assert np.all(np.diff(idx) > 0)
            assert np.array_equal(ys, single[idx % xs.shape[0]])
            got.append(idx)
    assert np.array_equal(np.sort(np.concatenate(got)), np.arange(total))


def test_ring_on_a_multi_cluster_pipeline():
    # requests waiting in the ring of a 4-stage pipeline (config 1): each stage hands off
    # through one buffer, so the first stage takes the next request only after the last stage
    # has published the previous one; every reply must belong to its own request
    net, Ws, bs = ll.config_params(1)
    xs = ll.config_inputs(1, 32)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with ll.Engine(net, Ws, bs, opts=opts(ring_slots=8)) as e:
        assert e.info().n_stages > 1
        for base in range(0, 32, 8):
            seqs = [e.submit(xs[base + i]) for i in range(8)]
            for i, s in enumerate(seqs):
                assert rel_err(e.poll(s)[0], ref[base + i]) <= 1e-5
        assert e.info().status == ll.LL_OK
