"""GPU parity tests through the C ABI (need a B200).

Tolerances (stated per north-star workload, norm-wise relative error
max|y - ref| / max|ref|): fp32 1e-5, bf16 1e-2, int8 2e-2.  The reference is the
CPU oracle (pinned to the reference's own cpu_gemv_bias_relu) and the committed
golden vectors.
"""
import ctypes
import time

import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import close, rel_err

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]

TOL = {ll.W_F32: 1e-5, ll.W_BF16: 1e-2, ll.W_I8: 2e-2}


def unbits(v):
    return np.array(v, np.uint32).view(np.float32)


def opts(**kw):
    o = ll.default_opts()
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def oracle_out(net, Ws, bs, xs):
    if net.wtype == ll.W_F32:
        return oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    if net.wtype == ll.W_BF16:
        return oracle.mlp_bf16(net.dims, net.acts, [ll.f32_to_bf16(w) for w in Ws], bs, xs)
    qs = [oracle.quantize_int8_rows(w) for w in Ws]
    return oracle.mlp_int8(net.dims, net.acts, [q for q, _ in qs], [s for _, s in qs], bs, xs)


def engine_for(net, Ws, bs, **kw):
    Wd, bd, sd = ll.device_weights(net, Ws, bs)
    return ll.Engine(net, Wd, bd, sd, device=0, opts=opts(**kw) if kw else None)


def test_echo_floor_seq_only_and_payload():
    with ll.EchoEngine(0, 0) as e:
        for _ in range(200):
            s = e.submit()
            e.poll(s)
        assert e.info().status == ll.LL_OK
    with ll.EchoEngine(64, 16) as e:
        xs = ll.config_inputs(0, 20)
        for i in range(20):
            y = e.infer(xs[i])
            assert np.array_equal(y[0], xs[i, :16])


def test_config0_parity_oracle_and_golden(golden):
    net, Ws, bs = ll.config_params(0)
    g = golden["cfg0"]
    xs = ll.config_inputs(0, 64)
    with engine_for(net, Ws, bs) as e:
        ys = np.stack([e.infer(xs[i])[0] for i in range(64)])
        info = e.info()
    assert info.kernel_variant == 2 and info.cluster_size == 8  # register-resident kernel by default
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    assert close(ys, ref, 1e-5)
    gy = unbits(g["y"]).reshape(g["n"], -1)
    assert rel_err(ys[: g["n"]], gy) <= 1e-5


def test_reference_own_mlp_matches_reference_golden(golden):
    """The reference's 512->256->64->1 MLP with its own host_init seeds (src/bench_cublas_mlp.cu:74-85)."""
    net, Ws, bs = ll.config_params("ref")
    x = ll.fill_normal(512, 0.0, 1.0, 1)
    with engine_for(net, Ws, bs) as e:
        y = e.infer(x)[0]
    y3 = unbits(golden["ref_bench"]["y3"])
    assert abs(float(y[0]) - float(y3[0])) <= 1e-5 * max(1.0, abs(float(y3[0])))


def test_config1_multi_cluster_parity(golden):
    net, Ws, bs = ll.config_params(1)
    g = golden["cfg1"]
    xs = ll.config_inputs(1, 16)
    with engine_for(net, Ws, bs) as e:
        ys = np.stack([e.infer(xs[i])[0] for i in range(16)])
        assert e.info().n_stages > 1
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    assert close(ys, ref, 1e-5)
    assert rel_err(ys[: g["n"]], unbits(g["y"]).reshape(g["n"], -1)) <= 1e-5


def test_config1_register_resident_deep_kernel_every_request_path():
    """Config 1 runs on the deep register-resident kernel (5 clusters of 16, 64 weights per
    thread): the tagged ring, the TickBuffer and the device queue give bit-identical replies
    (one kernel, one summation order), within 1e-5 of the oracle and of the generic kernel,
    which still serves the net when asked for."""
    torch = pytest.importorskip("torch")
    net, Ws, bs = ll.config_params(1)
    xs = ll.config_inputs(1, 40)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs, mailbox_format=1, ring_slots=8) as e:
        inf = e.info()
        assert inf.kernel_variant == ll.VARIANT_REGISTER_RESIDENT
        assert inf.n_stages == 5 and inf.cluster_size == 16 and inf.weight_regs == 64
        # per stage: rows split + all-gather over DSMEM (1), rows split + L2 hand-off to the next
        # cluster (5); the last stage keeps its rows local (2) for the K-split last layer (3)
        assert list(inf.layer_modes[:10]) == [1, 5] * 4 + [2, 3]
        tagged = np.stack([e.infer(xs[i])[0] for i in range(16)])
        seqs = e.submit_many(xs[16:24])
        tagged = np.concatenate([tagged, np.stack([e.poll(s)[0] for s in seqs])])
        e.stop()
        dx = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
        dy = torch.zeros(40, net.dims[-1], device="cuda")
        e.run_queue(dx.data_ptr(), dy.data_ptr(), 40, 1)
        queued = dy.cpu().numpy()
        assert e.info().status == ll.LL_OK
    with engine_for(net, Ws, bs, mailbox_format=0) as e:
        assert e.info().kernel_variant == ll.VARIANT_REGISTER_RESIDENT
        tick = np.stack([e.infer(xs[i])[0] for i in range(24)])
    with engine_for(net, Ws, bs, kernel_variant=1) as e:
        assert e.info().kernel_variant == ll.VARIANT_GENERIC
        generic = np.stack([e.infer(xs[i])[0] for i in range(24)])
    assert np.array_equal(tagged, tick) and np.array_equal(tagged, queued[:24])
    assert close(queued, ref, 1e-5) and rel_err(queued, ref) <= 1e-5
    assert close(tagged, generic, 1e-5)


def test_config2_batch1_on_the_deep_kernel_with_bf16_weight_pairs():
    """Config 2 at batch 1 (bf16 256 -> 1024 x 5 -> 64, GELU) runs on the deep register-resident
    kernel with two bf16 weights per register (5 clusters, one layer each): x and the hidden
    outputs rounded to bf16 as the oracle does; the tagged ring, the TickBuffer and the device
    queue agree bit for bit; within the bf16 tolerance of the oracle and of the resident
    small-batch kernel (another summation order)."""
    torch = pytest.importorskip("torch")
    net32, Ws, bs = ll.config_params(2)
    net = ll.mlp(net32.dims, ll.ACT_GELU, ll.ACT_IDENTITY, ll.W_BF16, 1)
    xs = ll.config_inputs(2, 24)
    ref = oracle_out(net, Ws, bs, xs)
    with engine_for(net, Ws, bs, mailbox_format=1, ring_slots=8) as e:
        inf = e.info()
        assert inf.kernel_variant == ll.VARIANT_REGISTER_RESIDENT and inf.n_stages == 5
        assert inf.weight_regs == 68  # 64 of the hidden layer + 4 of the last layer's K-split
        assert list(inf.layer_modes[:6]) == [5, 5, 5, 5, 2, 3]
        tagged = np.stack([e.infer(xs[i])[0] for i in range(8)])
        seqs = e.submit_many(xs[8:16])
        tagged = np.concatenate([tagged, np.stack([e.poll(s)[0] for s in seqs])])
        e.stop()
        dx = torch.from_numpy(np.ascontiguousarray(xs)).cuda()
        dy = torch.zeros(24, net.dims[-1], device="cuda")
        e.run_queue(dx.data_ptr(), dy.data_ptr(), 24, 1)
        queued = dy.cpu().numpy()
        assert e.info().status == ll.LL_OK
    with engine_for(net, Ws, bs, mailbox_format=0) as e:
        tick = np.stack([e.infer(xs[i])[0] for i in range(16)])
    with engine_for(net, Ws, bs, kernel_variant=3) as e:
        assert e.info().kernel_variant == ll.VARIANT_RESIDENT_SMALL_BATCH
        small = np.stack([e.infer(xs[i])[0] for i in range(16)])
    assert np.array_equal(tagged, tick) and np.array_equal(tagged, queued[:16])
    assert close(queued, ref, TOL[ll.W_BF16]) and rel_err(queued, ref) <= TOL[ll.W_BF16]
    assert close(tagged, small, TOL[ll.W_BF16])


@pytest.mark.parametrize("C,rep", [(2, 0), (4, 1), (8, 0), (8, 1), (16, 0), (16, 1)])
def test_config0_generic_kernel_cluster_sizes(C, rep):
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 8)
    with engine_for(net, Ws, bs, cluster_size=C, replicate_first=rep, kernel_variant=1) as e:
        ys = np.stack([e.infer(xs[i])[0] for i in range(8)])
        assert e.info().kernel_variant == 1
    assert rel_err(ys, oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)) <= 1e-5


@pytest.mark.parametrize("C", [4, 8])
def test_config0_register_resident_kernel(C):
    torch = pytest.importorskip("torch")
    net, Ws, bs = ll.config_params(0)
    n = 300
    xs = ll.config_inputs(0, n)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs, cluster_size=C, kernel_variant=2) as e:
        info = e.info()
        assert info.kernel_variant == 2 and info.cluster_size == C and info.weight_regs > 0
        lat, ys = e.bench_closed_loop(xs, n, keep_outputs=True)
        dx = torch.from_numpy(xs).cuda()
        dy = torch.zeros((n, 16), device="cuda")
        torch.cuda.synchronize()
        e.run_queue(dx.data_ptr(), dy.data_ptr(), n, 1)
    assert rel_err(ys[:, 0, :], ref) <= 1e-5
    assert rel_err(dy.cpu().numpy(), ref) <= 1e-5


def test_register_resident_kernel_refuses_other_shapes():
    net = ll.mlp([32, 64, 16], ll.ACT_RELU)
    Ws, bs = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 1)
    with pytest.raises(ll.LLError) as e:
        engine_for(net, Ws, bs, kernel_variant=2)
    assert e.value.code == ll.LL_ERR_UNSUPPORTED


@pytest.mark.parametrize("wtype,act,rows", [(ll.W_F32, ll.ACT_RELU, 3), (ll.W_BF16, ll.ACT_GELU, 5),
                                            (ll.W_I8, ll.ACT_RELU, 4), (ll.W_BF16, ll.ACT_GELU, 1)])
def test_small_batches_and_precisions(wtype, act, rows):
    net = ll.mlp([40, 96, 200, 72, 10], act, ll.ACT_IDENTITY, wtype, 8)
    Ws, bs = ll.init_params(net, ll.INIT_NORMAL_FANIN, 3)
    xs = ll.fill_uniform(rows * 40, -1, 1, 8).reshape(rows, 40)
    with engine_for(net, Ws, bs, cluster_size=4, min_stages=2) as e:
        y = e.infer(xs)
    assert close(y, oracle_out(net, Ws, bs, xs), TOL[wtype])


@pytest.mark.parametrize("dims", [[33, 597, 293, 7], [5, 3], [17, 100, 1], [1, 1, 1]])
def test_odd_shapes(dims):
    net = ll.mlp(dims, ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 1)
    Ws, bs = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 9)
    xs = ll.fill_uniform(4 * dims[0], -1, 1, 4).reshape(4, -1)
    with engine_for(net, Ws, bs, cluster_size=8) as e:
        ys = np.stack([e.infer(xs[i])[0] for i in range(4)])
    assert close(ys, oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs), 1e-5)


def test_reference_style_raw_mailbox_host_loop():
    """Drive the engine the way the reference host does (src/bench_persistent_mbyv_mlp.cu:499-509,
    536-557): write x into the mapped TickBuffer, bump seq_in, spin on seq_out, stop with stop + seq bump."""
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 10)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs) as e:
        e.start()
        base = e.mailbox()
        hdr = (ctypes.c_uint32 * 4).from_address(base)
        xbuf = np.ctypeslib.as_array((ctypes.c_float * 64).from_address(base + 16))
        ybuf = np.ctypeslib.as_array((ctypes.c_float * 16).from_address(base + 16 + 64 * 4))
        seq = hdr[1]
        for i in range(10):
            xbuf[:] = xs[i]
            seq += 1
            hdr[0] = seq
            t0 = time.time()
            while hdr[1] != seq:
                assert time.time() - t0 < 2.0
            assert rel_err(ybuf.copy(), ref[i]) <= 1e-5
        hdr[2] = 1  # stop
        hdr[0] = seq + 1  # the reference's stop doorbell
        t0 = time.time()
        while e.info().state != 4:
            assert time.time() - t0 < 5.0
        assert e.info().status == ll.LL_OK
        hdr[2] = 0
        hdr[1] = seq + 1  # host re-arms the doorbell baseline before re-use
        e.stop()


def test_hand_driven_host_may_skip_sequence_numbers_on_a_pipeline():
    """A TickBuffer host that advances seq_in by more than one (any new non-zero number starts
    a request) on the 4-stage config-1 pipeline: the later stages take the number the hand-off
    words carry, so every request is answered with its own output."""
    net, Ws, bs = ll.config_params(1)
    xs = ll.config_inputs(1, 6)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs) as e:
        assert e.info().n_stages > 1
        e.start()
        base = e.mailbox()
        hdr = (ctypes.c_uint32 * 4).from_address(base)
        xbuf = np.ctypeslib.as_array((ctypes.c_float * 128).from_address(base + 16))
        ybuf = np.ctypeslib.as_array((ctypes.c_float * 32).from_address(base + 16 + 128 * 4))
        seq = hdr[1]
        for i, step in enumerate((1, 3, 2, 7, 1, 5)):
            xbuf[:] = xs[i]
            seq += step
            hdr[0] = seq
            t0 = time.time()
            while hdr[1] != seq:
                assert time.time() - t0 < 2.0
            assert rel_err(ybuf.copy(), ref[i]) <= 1e-5
        assert e.info().status == ll.LL_OK
        e.stop()


def test_closed_loop_bench_outputs():
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 32)
    with engine_for(net, Ws, bs) as e:
        lat, ys = e.bench_closed_loop(xs, 500, keep_outputs=True)
    assert (lat > 0).all() and np.isfinite(lat).all()
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    assert rel_err(ys[:, 0, :], ref[np.arange(500) % 32]) <= 1e-5


@pytest.mark.parametrize("variant", [1, 2])
def test_device_resident_queue(variant):
    torch = pytest.importorskip("torch")
    net, Ws, bs = ll.config_params(0)
    n = 256
    xs = ll.config_inputs(0, n)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    dx = torch.from_numpy(xs).to("cuda:0")
    dy = torch.zeros((n, 16), dtype=torch.float32, device="cuda:0")
    st = torch.zeros(n, dtype=torch.int64, device="cuda:0")
    torch.cuda.synchronize()
    with engine_for(net, Ws, bs, kernel_variant=variant) as e:
        ms = e.run_queue(dx.data_ptr(), dy.data_ptr(), n, 1, st.data_ptr())
        # the mailbox path still works after a queue run
        y = e.infer(xs[3])
    assert ms > 0
    assert rel_err(dy.cpu().numpy(), ref) <= 1e-5
    assert rel_err(y[0], ref[3]) <= 1e-5
    stamps = st.cpu().numpy()
    assert (np.diff(stamps) > 0).all()


@pytest.mark.parametrize("variant", [1, 2])
def test_idle_exit_and_relaunch(variant):
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 4)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs, idle_timeout_ns=int(50e6), kernel_variant=variant) as e:
        y0 = e.infer(xs[0])
        time.sleep(0.3)  # longer than the idle bound: the resident kernel leaves on its own
        assert e.info().state == 4
        y1 = e.infer(xs[1])  # relaunched on demand
        info = e.info()
    assert info.launches == 2 and info.status == ll.LL_OK
    assert rel_err(np.stack([y0[0], y1[0]]), ref[:2]) <= 1e-5


@pytest.mark.parametrize("variant", [1, 2])
def test_device_wait_that_runs_out_reports_status_and_context_survives(variant):
    """A device wait on a barrier nothing completes (diag_wait_never) runs out after the
    50 ms step bound: the kernel records LL_ERR_DEVICE_FAULT with its location and leaves
    cleanly -- no trap, no hang -- and the CUDA context stays usable."""
    net, Ws, bs = ll.config_params(0)
    x = ll.config_inputs(0, 1)
    with engine_for(net, Ws, bs, step_timeout_ns=int(50e6), diag_wait_never=1, kernel_variant=variant) as e:
        with pytest.raises(ll.LLError) as err:
            e.infer(x[0], timeout_s=5.0)
        assert err.value.code == ll.LL_ERR_DEVICE_FAULT
        info = e.info()
        assert info.status == ll.LL_ERR_DEVICE_FAULT and info.err_where == 6
    with engine_for(net, Ws, bs) as e:
        assert rel_err(e.infer(x[0]), oracle.mlp_f32(net.dims, net.acts, Ws, bs, x)) <= 1e-5


def test_dense_launch_per_layer_kernels():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2)
    for M, K, act in ((256, 64, ll.ACT_RELU), (16, 256, ll.ACT_IDENTITY), (1, 64, ll.ACT_IDENTITY),
                      (597, 293, ll.ACT_GELU), (33, 5, ll.ACT_RELU)):
        W = (rng.standard_normal((M, K)) / np.sqrt(K)).astype(np.float32)
        b = rng.standard_normal(M).astype(np.float32) * 0.01
        x = rng.standard_normal(K).astype(np.float32)
        ref = oracle.gemv_bias_act(W, b, x, act)
        dW, db, dx = (torch.from_numpy(a).cuda() for a in (W, b, x))
        dy = torch.zeros(M, device="cuda")
        ll.dense_warp_rm(dW.data_ptr(), db.data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, act)
        torch.cuda.synchronize()
        assert rel_err(dy.cpu().numpy(), ref) <= 1e-5
        Mpad = (M + 31) // 32 * 32
        dWcm = torch.from_numpy(ll.pack_rm_to_kmajor_padded(W, Mpad)).cuda()
        dbp = torch.from_numpy(ll.pack_bias_padded(b, Mpad)).cuda()
        dy2 = torch.zeros(M, device="cuda")
        ll.dense_mbyv_packed(dWcm.data_ptr(), dbp.data_ptr(), dx.data_ptr(), dy2.data_ptr(), M, K, act)
        torch.cuda.synchronize()
        # the packed kernel starts from the bias (src/bench_custom_mbyv_packed_graph.cu:31 order)
        assert rel_err(dy2.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("cls", [ll.LayeredMLP, ll.CublasMLP])
@pytest.mark.parametrize("mode", [ll.RUN_DIRECT_KERNEL, ll.RUN_GRAPH_KERNEL, ll.RUN_GRAPH_E2E, ll.RUN_DIRECT_E2E,
                                  ll.RUN_MAILBOX_TICK])
def test_comparison_paths_parity(cls, mode):
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 5)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with cls(net, Ws, bs) as m:
        lat, y = m.bench(mode, xs, 5)
    assert (lat > 0).all()
    assert rel_err(y, ref[4]) <= 1e-5  # the last request used xs[4]


@pytest.mark.parametrize("variant", [1, 2])
def test_tagged_mailbox_config0(variant):
    net, Ws, bs = ll.config_params(0)
    n = 300
    xs = ll.config_inputs(0, n)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs, mailbox_format=1, kernel_variant=variant) as e:
        lat, ys = e.bench_closed_loop(xs, n, keep_outputs=True)
        y1 = e.infer(xs[5])
    assert rel_err(ys[:, 0, :], ref) <= 1e-5
    assert rel_err(y1[0], ref[5]) <= 1e-5


@pytest.mark.parametrize("dims", [[33, 100, 7], [5, 3], [130, 40, 40, 2]])
def test_tagged_mailbox_odd_widths_generic(dims):
    net = ll.mlp(dims, ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 1)
    Ws, bs = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 9)
    xs = ll.fill_uniform(6 * dims[0], -1, 1, 4).reshape(6, -1)
    with engine_for(net, Ws, bs, cluster_size=4, mailbox_format=1) as e:
        ys = np.stack([e.infer(xs[i])[0] for i in range(6)])
    assert rel_err(ys, oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)) <= 1e-5


def test_tagged_echo_floor_copies_x():
    o = opts(mailbox_format=1)
    with ll.EchoEngine(64, 16, opts=o) as e:
        xs = ll.config_inputs(0, 10)
        for i in range(10):
            assert np.array_equal(e.infer(xs[i])[0], xs[i, :16])


def test_tagged_mailbox_rejects_batches():
    net = ll.mlp([8, 16, 4], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 4)
    Ws, bs = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 1)
    with pytest.raises(ll.LLError) as err:
        engine_for(net, Ws, bs, mailbox_format=1)
    assert err.value.code == ll.LL_ERR_UNSUPPORTED


def test_config1_pipeline_hand_offs_across_queue_runs_and_relaunches():
    # the batch-1 pipeline hands off tagged words {seq, value} between its clusters; queue runs
    # number their requests from 1 again, and an idle exit relaunches: no stale word may match
    torch = pytest.importorskip("torch")
    net, Ws, bs = ll.config_params(1)
    xs = ll.config_inputs(1, 268)
    ref = oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs)
    with engine_for(net, Ws, bs, idle_timeout_ns=30_000_000) as e:
        assert e.info().n_stages > 1
        ys = [e.infer(xs[i])[0] for i in range(4)]
        dx = torch.from_numpy(np.ascontiguousarray(xs[4:260])).cuda()
        for _ in range(2):
            dy = torch.zeros(256, net.dims[-1], device="cuda")
            e.run_queue(dx.data_ptr(), dy.data_ptr(), 256, 1)
            assert rel_err(dy.cpu().numpy(), ref[4:260]) <= 1e-5
        ys += [e.infer(xs[i])[0] for i in range(260, 264)]
        launches = e.info().launches
        time.sleep(0.15)  # the kernel leaves after 30 ms idle; the next request relaunches it
        ys += [e.infer(xs[i])[0] for i in range(264, 268)]
        assert e.info().launches > launches and e.info().status == ll.LL_OK
    idx = list(range(4)) + list(range(260, 268))
    assert rel_err(np.stack(ys), ref[idx]) <= 1e-5
