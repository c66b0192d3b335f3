"""Weight files: round trips for every weight type and the checks that reject
damaged files (no GPU)."""
import os

import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll


@pytest.mark.parametrize("cfg", [0, 2, 3])
def test_round_trip_keeps_every_byte(tmp_path, cfg):
    net, Ws, bs = ll.config_params(cfg)
    Wd, bd, sd = ll.device_weights(net, Ws, bs)
    path = str(tmp_path / "net.llw")
    ll.save_weights(path, net, Wd, bd, sd)
    net2, W2, b2, s2 = ll.load_weights(path)
    assert net2 == net
    for a, c in zip(Wd, W2):
        assert a.dtype == c.dtype and np.array_equal(a, c)
    for a, c in zip(bd, b2):
        assert np.array_equal(a, c)
    if net.wtype == ll.W_I8:
        for a, c in zip(sd, s2):
            assert np.array_equal(a, c)
    else:
        assert s2 is None


def test_file_without_biases(tmp_path):
    net = ll.mlp([8, 4, 2], ll.ACT_RELU, ll.ACT_IDENTITY, ll.W_F32, 1)
    W = [np.arange(32, dtype=np.float32).reshape(4, 8), np.ones((2, 4), np.float32)]
    path = str(tmp_path / "nob.llw")
    ll.save_weights(path, net, W)
    _, W2, b2, _ = ll.load_weights(path)
    assert b2 is None and np.array_equal(W2[0], W[0])


def _file(tmp_path):
    net, Ws, bs = ll.config_params(0)
    path = str(tmp_path / "c0.llw")
    ll.save_weights(path, net, Ws, bs)
    return path


def test_corrupt_payload_is_rejected(tmp_path):
    path = _file(tmp_path)
    data = bytearray(open(path, "rb").read())
    data[32 + 3 * 16 + 1000] ^= 0x40  # one bit inside the first weight section
    open(path, "wb").write(bytes(data))
    with pytest.raises(ll.LLError) as e:
        ll.load_weights(path)
    assert e.value.code == ll.LL_ERR_BAD_DESC and "checksum" in str(e.value)


def test_truncated_file_is_rejected(tmp_path):
    path = _file(tmp_path)
    data = open(path, "rb").read()
    open(path, "wb").write(data[:-100])
    with pytest.raises(ll.LLError) as e:
        ll.load_weights(path)
    assert "truncated" in str(e.value)


def test_wrong_magic_version_and_missing_file(tmp_path):
    path = _file(tmp_path)
    data = bytearray(open(path, "rb").read())
    bad = tmp_path / "magic.llw"
    bad.write_bytes(b"XXXX" + bytes(data[4:]))
    with pytest.raises(ll.LLError):
        ll.load_weights(str(bad))
    data[4] = 7  # version 7
    ver = tmp_path / "ver.llw"
    ver.write_bytes(bytes(data))
    with pytest.raises(ll.LLError) as e:
        ll.load_weights(str(ver))
    assert e.value.code == ll.LL_ERR_UNSUPPORTED
    with pytest.raises(ll.LLError):
        ll.load_weights(str(tmp_path / "absent.llw"))
    assert os.path.exists(path)


def test_int8_net_needs_scales(tmp_path):
    net, Ws, bs = ll.config_params(3)
    Wd, bd, _ = ll.device_weights(net, Ws, bs)
    with pytest.raises(ll.LLError):
        ll.save_weights(str(tmp_path / "x.llw"), net, Wd, bd, None)
