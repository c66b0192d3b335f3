"""The forward entry point that allocates nothing (ll_mlp_forward_noalloc).

It exists for callers that cannot allocate device memory on their request path:
a cudaMalloc may implicitly synchronise the device and take milliseconds, and
some callers' device memory belongs to another allocator.  Its hidden
activations live in a static, library-owned device array instead.

This file sorts last so that a run stopping at the first failure has already run
every other test.  The checks: through the C ABI, two calls in a row on different
inputs give the same outputs as the existing launch-per-layer entry point
(ll_layered_mlp, which allocates its own buffers) and as the CPU oracle, within the
fp32 tolerance used everywhere else (1e-5 norm-wise relative); a bias-less net
with three hidden layers (so both halves of the static array carry activations)
does the same; and a net wider than the static array is refused with a clear
error.
"""
import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll
import oracle
from conftest import rel_err


@pytest.mark.gpu
@pytest.mark.timeout(300)
def test_noalloc_forward_matches_existing_entry_point_twice():
    torch = pytest.importorskip("torch")
    net, Ws, bs = ll.config_params(0)
    xs = ll.config_inputs(0, 2)
    dW = [torch.from_numpy(np.ascontiguousarray(w)).cuda() for w in Ws]
    db = [torch.from_numpy(np.ascontiguousarray(b)).cuda() for b in bs]
    outs = []
    for i in range(2):  # two calls in a row share (and reuse) the static scratch
        dx = torch.from_numpy(np.ascontiguousarray(xs[i])).cuda()
        dy = torch.full((net.dims[-1],), float("nan"), device="cuda")
        torch.cuda.synchronize()
        ll.mlp_forward_noalloc(net, [t.data_ptr() for t in dW], [t.data_ptr() for t in db], dx.data_ptr(),
                               dy.data_ptr())
        torch.cuda.synchronize()
        outs.append(dy.cpu().numpy())
    with ll.LayeredMLP(net, Ws, bs) as m:
        for i in range(2):
            _, y_ref = m.bench(ll.RUN_DIRECT_KERNEL, xs[i:i + 1], 1)
            assert np.isfinite(outs[i]).all()
            assert rel_err(outs[i], y_ref) <= 1e-5
            assert rel_err(outs[i], oracle.mlp_f32(net.dims, net.acts, Ws, bs, xs[i:i + 1])[0]) <= 1e-5
    assert not np.array_equal(outs[0], outs[1])  # two different requests, not one stale result


@pytest.mark.gpu
@pytest.mark.timeout(300)
def test_noalloc_forward_without_biases_through_both_scratch_halves():
    torch = pytest.importorskip("torch")
    net = ll.mlp([64, 96, 200, 48, 16], ll.ACT_RELU)  # hidden layers write halves 0, 1, 0
    Ws, _ = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 11)
    zeros = [np.zeros(d, np.float32) for d in net.dims[1:]]
    xs = ll.fill_uniform(2 * 64, -1.0, 1.0, 12).reshape(2, 64)
    dW = [torch.from_numpy(np.ascontiguousarray(w)).cuda() for w in Ws]
    for i in range(2):
        dx = torch.from_numpy(np.ascontiguousarray(xs[i])).cuda()
        dy = torch.full((net.dims[-1],), float("nan"), device="cuda")
        ll.mlp_forward_noalloc(net, [t.data_ptr() for t in dW], None, dx.data_ptr(), dy.data_ptr())
        torch.cuda.synchronize()
        y = dy.cpu().numpy()
        assert np.isfinite(y).all()
        assert rel_err(y, oracle.mlp_f32(net.dims, net.acts, Ws, zeros, xs[i:i + 1])[0]) <= 1e-5


@pytest.mark.gpu
@pytest.mark.timeout(120)
def test_noalloc_forward_refuses_nets_wider_than_the_static_scratch():
    torch = pytest.importorskip("torch")
    wide = ll.NOALLOC_MAX_WIDTH + 4
    net = ll.mlp([8, wide, 4], ll.ACT_RELU)
    dW = [torch.zeros((wide, 8), device="cuda"), torch.zeros((4, wide), device="cuda")]
    dx = torch.zeros(8, device="cuda")
    dy = torch.zeros(4, device="cuda")
    with pytest.raises(ll.LLError) as e:
        ll.mlp_forward_noalloc(net, [t.data_ptr() for t in dW], None, dx.data_ptr(), dy.data_ptr())
    assert e.value.code == ll.LL_ERR_INVALID_ARG
    assert "LL_NOALLOC_MAX_WIDTH" in str(e.value)
