"""Host-side checks of the batched tensor-core path (no GPU): tiling choices and
descriptor validation."""
import pytest

import low_latency_inference_gpu_b200 as ll


def test_config3_fills_the_gpu():
    p = ll.batched_plan(ll.config_net(3))
    assert p["rows_pad"] == 256
    assert all(c <= 148 for c in p["ctas"])
    assert min(p["ctas"]) >= 128  # every layer uses at least 128 of the 148 SMs
    assert all(s <= 227 * 1024 for s in p["smem_bytes"])
    # the square layers: 128-wide tiles split 4 ways (a split 256-wide tile has no room to exchange)
    assert p["bn"][1:7] == [128] * 6 and p["splits"][1:7] == [4] * 6


def test_config2_batch_sweep_plans():
    for rows in (1, 2, 4, 8, 16, 32):
        # up to 32 rows: the small-batch kernel, one CTA per SM holding 7 rows of each
        # 1024-wide layer (1 of the 64-wide last layer) in shared memory
        p = ll.batched_plan(ll.config_net(2, rows))
        assert p["kind"] == [ll.KERNEL_GEMV] * 6
        assert p["ctas"] == [148] * 6 and p["bn"] == [7] * 5 + [1]
        assert p["smem_bytes"][0] <= 227 * 1024
        # the tensor-core tiles on request
        t = ll.batched_plan(ll.config_net(2, rows), ll.batched_opts(kernel=ll.KERNEL_SPLITK))
        assert t["rows_pad"] == 256 and t["kind"] == [1] * 6
        assert all(1 <= c <= 148 for c in t["ctas"])
    # 33 rows is past the small-batch kernel
    assert ll.batched_plan(ll.config_net(2, 33))["kind"] == [1] * 6
    with pytest.raises(ll.LLError):
        ll.batched_plan(ll.config_net(2, 33), ll.batched_opts(kernel=ll.KERNEL_GEMV))


def test_small_batch_kernel_needs_the_slices_to_fit():
    # config 3 (int8, 2048 wide): one row fits beside the weight slices, eight rows do not
    assert ll.batched_plan(ll.config_net(3, 1))["kind"] == [ll.KERNEL_GEMV] * 8
    assert ll.batched_plan(ll.config_net(3, 8))["kind"] == [1] * 8
    # forcing tile options keeps the tensor-core tiles
    net = ll.mlp([256, 256, 256], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_BF16, 16)
    assert ll.batched_plan(net)["kind"] == [ll.KERNEL_GEMV] * 2
    assert ll.batched_plan(net, ll.batched_opts(bn=64))["kind"] == [1, 1]


def test_forced_tiles_are_honoured_and_checked():
    net = ll.mlp([256, 256, 256], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_I8, 64)
    p = ll.batched_plan(net, ll.batched_opts(bn=128, splits=2))
    assert p["bn"] == [128, 128] and p["splits"] == [2, 2]
    with pytest.raises(ll.LLError):
        ll.batched_plan(net, ll.batched_opts(splits=3))  # 3 does not divide 256/64
    with pytest.raises(ll.LLError):
        ll.batched_plan(net, ll.batched_opts(bn=96))
    with pytest.raises(ll.LLError):
        ll.batched_plan(net, ll.batched_opts(bn=256, splits=2))  # no shared memory for the exchange


@pytest.mark.parametrize("dims,wtype", [([100, 256], ll.W_BF16), ([256, 100], ll.W_I8), ([256, 256], ll.W_F32)])
def test_unsupported_nets_are_rejected(dims, wtype):
    net = ll.mlp(dims, ll.ACT_RELU, ll.ACT_IDENTITY, wtype, 8)
    with pytest.raises(ll.LLError) as e:
        ll.batched_plan(net)
    assert e.value.code == ll.LL_ERR_BAD_DESC


def test_stacked_batches_use_weights_in_tmem_tiles():
    p = ll.batched_plan(ll.config_net(3, 2048))
    # 16 channel tiles x 8 row blocks of 256 for every 2048-wide layer; the 256-wide last
    # layer has only 16 such tiles and keeps the split-K kernel
    assert p["kind"] == [2] * 7 + [1]
    assert p["ctas"][:7] == [128] * 7 and p["splits"][:7] == [1] * 7
    forced = ll.batched_plan(ll.config_net(3, 256), ll.batched_opts(kernel=2))
    assert forced["kind"] == [2] * 8
