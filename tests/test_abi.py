"""C ABI surface and the host half of the mailbox protocol (no GPU).

A Python thread plays the device on a plain-memory mailbox, the way the
resident kernel does on host-mapped memory: it waits for seq_in to change,
reads x and n_rows, writes y, then seq_out.  The fault cases (dropped
doorbell, stale seq_out, seq wrap) are made on the host, never on a GPU.
"""
import ctypes
import os
import re
import threading
import time

import numpy as np
import pytest

import low_latency_inference_gpu_b200 as ll

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "ll_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ll_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_function():
    lib = ll.lib()
    declared = header_functions()
    assert len(declared) >= 35
    missing = [f for f in declared if not hasattr(lib, f)]
    assert not missing, missing
    assert set(declared) == set(ll.EXPORTED_SYMBOLS)


def test_version_and_error_string():
    assert b"sm_100a" in ll.lib().ll_version()
    with pytest.raises(ll.LLError) as e:
        ll.plan_net(ll.Net([4, 4], [9], ll.W_F32, 1))
    assert "activation" in str(e.value)


def test_tick_header_layout_matches_reference_tickbuffer():
    # src/bench_persistent_mbyv_mlp.cu:88-95: seq_in, seq_out, stop, pad, then x[IN], y[OUT]
    assert ctypes.sizeof(ll.TickHeader) == 16
    assert [f[0] for f in ll.TickHeader._fields_] == ["seq_in", "seq_out", "stop", "n_rows"]
    assert ll.lib().ll_mailbox_bytes(512, 1, 1) == 16 + 512 * 4 + 4 + 44  # rounded to 64 like alignas(64)
    assert ll.lib().ll_mailbox_bytes(64, 16, 1) % 64 == 0


def test_next_seq_skips_idle_and_stop():
    f = ll.lib().ll_next_seq
    assert f(0) == 1 and f(41) == 42
    assert f(0xFFFFFFFE) == 1  # never LL_STOP_SEQ
    assert f(0xFFFFFFFF) == 1  # never 0


class FakeDevice(threading.Thread):
    """CPU stand-in for the resident kernel: y = 2*x[:out] + seq; optional faults."""

    def __init__(self, buf, in_dim, out_dim, max_batch, drop_every=0, delay_s=0.0):
        super().__init__(daemon=True)
        self.buf, self.in_dim, self.out_dim, self.max_batch = buf, in_dim, out_dim, max_batch
        self.drop_every, self.delay_s = drop_every, delay_s
        self.stop_flag = False
        self.served = 0

    def run(self):
        hdr = np.frombuffer(self.buf, np.uint32, 4, 0)
        x = np.frombuffer(self.buf, np.float32, self.in_dim * self.max_batch, 16)
        y = np.frombuffer(self.buf, np.float32, self.out_dim * self.max_batch, 16 + 4 * self.in_dim * self.max_batch)
        last = 0
        n = 0
        while not self.stop_flag:
            s = int(hdr[0])
            if hdr[2]:
                return
            if s == last or s == 0:
                time.sleep(0)
                continue
            last = s
            n += 1
            if self.drop_every and n % self.drop_every == 0:
                continue  # dropped doorbell: never answer
            if self.delay_s:
                time.sleep(self.delay_s)
            rows = max(1, int(hdr[3]))
            xs = x[: rows * self.in_dim].reshape(rows, self.in_dim)
            y[: rows * self.out_dim] = (2 * xs[:, : self.out_dim] + s).ravel()
            hdr[1] = s
            self.served = s


def _mailbox(in_dim, out_dim, max_batch):
    n = ll.lib().ll_mailbox_bytes(in_dim, out_dim, max_batch)
    return (ctypes.c_uint8 * n)()


def test_mailbox_round_trips_with_fake_device():
    in_dim, out_dim, mb = 8, 3, 4
    buf = _mailbox(in_dim, out_dim, mb)
    dev = FakeDevice(buf, in_dim, out_dim, mb)
    dev.start()
    lib = ll.lib()
    seq = 0
    try:
        for r in range(50):
            rows = 1 + r % mb
            x = np.arange(rows * in_dim, dtype=np.float32) + r
            seq = lib.ll_next_seq(seq)
            lib.ll_mailbox_post(ctypes.addressof(buf), in_dim, x.ctypes.data_as(ll._fp), rows, seq, r % 2)
            y = np.empty(rows * out_dim, np.float32)
            rc = lib.ll_mailbox_wait(ctypes.addressof(buf), in_dim, out_dim, mb, seq, y.ctypes.data_as(ll._fp), rows,
                                     int(2e9))
            assert rc == ll.LL_OK
            want = (2 * x.reshape(rows, in_dim)[:, :out_dim] + seq).ravel()
            assert np.array_equal(y, want)
    finally:
        dev.stop_flag = True
        dev.join(2)


def test_mailbox_dropped_doorbell_times_out_then_recovers():
    in_dim, out_dim = 4, 4
    buf = _mailbox(in_dim, out_dim, 1)
    dev = FakeDevice(buf, in_dim, out_dim, 1, drop_every=3)
    dev.start()
    lib = ll.lib()
    seq, timeouts = 0, 0
    try:
        for r in range(9):
            x = np.full(in_dim, r, np.float32)
            seq = lib.ll_next_seq(seq)
            lib.ll_mailbox_post(ctypes.addressof(buf), in_dim, x.ctypes.data_as(ll._fp), 1, seq, 0)
            rc = lib.ll_mailbox_wait(ctypes.addressof(buf), in_dim, out_dim, 1, seq, None, 1, int(50e6))
            if rc == ll.LL_ERR_TIMEOUT:
                timeouts += 1
                assert b"timed out" in lib.ll_last_error()
            else:
                assert rc == ll.LL_OK
        assert timeouts == 3  # every third doorbell was dropped; later ones still served
    finally:
        dev.stop_flag = True
        dev.join(2)


def test_mailbox_stale_seq_out_is_not_mistaken_for_completion():
    buf = _mailbox(4, 4, 1)
    hdr = np.frombuffer(buf, np.uint32, 4, 0)
    hdr[1] = 7  # seq_out left over from an earlier request
    rc = ll.lib().ll_mailbox_wait(ctypes.addressof(buf), 4, 4, 1, 8, None, 1, int(20e6))
    assert rc == ll.LL_ERR_TIMEOUT
    hdr[1] = 8
    assert ll.lib().ll_mailbox_wait(ctypes.addressof(buf), 4, 4, 1, 8, None, 1, int(20e6)) == ll.LL_OK


def test_stop_flag_ends_fake_device():
    buf = _mailbox(4, 4, 1)
    dev = FakeDevice(buf, 4, 4, 1)
    dev.start()
    hdr = np.frombuffer(buf, np.uint32, 4, 0)
    hdr[2] = 1  # stop, as src/bench_persistent_mlp.cu:409
    dev.join(2)
    assert not dev.is_alive()


def test_generators_and_params_are_deterministic():
    net = ll.config_net(0)
    a = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 0)
    b = ll.init_params(net, ll.INIT_XAVIER_UNIFORM, 0)
    for wa, wb in zip(a[0] + a[1], b[0] + b[1]):
        assert np.array_equal(wa, wb)
    lim = np.sqrt(6.0 / (64 + 256))
    assert np.abs(a[0][0]).max() <= lim and np.abs(a[1][0]).max() <= 0.01
    x = ll.config_inputs(0, 100)
    assert x.shape == (100, 64) and np.abs(x).max() <= 1.0


def test_invalid_arguments_are_rejected_without_gpu():
    lib = ll.lib()
    h = ctypes.c_void_p()
    assert lib.ll_engine_create_ex(None, None, None, None, 0, None, ctypes.byref(h)) == ll.LL_ERR_BAD_DESC
    assert lib.ll_dense_warp_rm(None, None, None, None, 4, 4, 0, None) == ll.LL_ERR_INVALID_ARG
    assert lib.ll_submit(None, None, 1, None) == ll.LL_ERR_INVALID_ARG


class FakeTaggedDevice(threading.Thread):
    """CPU stand-in for the device on the tagged mailbox: takes a request when every x chunk
    carries the same new tag, answers y = 2*x[:out] + seq in tagged chunks (floats, then tag)."""

    def __init__(self, buf, in_dim, out_dim):
        super().__init__(daemon=True)
        self.buf, self.in_dim, self.out_dim = buf, in_dim, out_dim
        self.stop_flag = False

    def run(self):
        xc, yc = (self.in_dim + 2) // 3, (self.out_dim + 2) // 3
        xw = np.frombuffer(self.buf, np.uint32, 4 * xc, 16).reshape(xc, 4)
        yw = np.frombuffer(self.buf, np.uint32, 4 * yc, ll.lib().ll_tagged_y_offset(self.in_dim)).reshape(yc, 4)
        last = 0
        while not self.stop_flag:
            snap = xw.copy()
            tags = snap[:, 3]
            if (tags == tags[0]).all() and tags[0] != last and tags[0] != 0:
                s = int(tags[0])
                x = snap[:, :3].copy().view(np.float32).ravel()[: self.in_dim]
                y = np.zeros(3 * yc, np.float32)
                y[: self.out_dim] = 2 * x[: self.out_dim] + s
                yv = y.view(np.uint32).reshape(yc, 3)
                for c in range(yc):
                    yw[c, :3] = yv[c]
                    yw[c, 3] = s
                last = s
            else:
                time.sleep(0)


@pytest.mark.parametrize("in_dim,out_dim", [(64, 16), (7, 5), (1, 1), (384, 96)])
def test_tagged_mailbox_round_trips_with_fake_device(in_dim, out_dim):
    lib = ll.lib()
    n = lib.ll_tagged_mailbox_bytes(in_dim, out_dim)
    yoff = lib.ll_tagged_y_offset(in_dim)
    assert yoff % 64 == 0 and yoff >= 16 + 16 * ((in_dim + 2) // 3)  # y never shares a line with x
    assert n % 64 == 0 and n >= yoff + 16 * ((out_dim + 2) // 3)
    buf = (ctypes.c_uint8 * n)()
    dev = FakeTaggedDevice(buf, in_dim, out_dim)
    dev.start()
    seq = 0
    try:
        for r in range(20):
            x = (np.arange(in_dim, dtype=np.float32) * 0.5 + r).astype(np.float32)
            seq = lib.ll_next_seq(seq)
            lib.ll_tagged_post(ctypes.addressof(buf), in_dim, x.ctypes.data_as(ll._fp), seq)
            y = np.empty(out_dim, np.float32)
            rc = lib.ll_tagged_wait(ctypes.addressof(buf), in_dim, out_dim, seq, y.ctypes.data_as(ll._fp), int(2e9))
            assert rc == ll.LL_OK
            assert np.array_equal(y, 2 * x[:out_dim] + seq)
        # a reply that never comes times out
        seq2 = lib.ll_next_seq(seq)
        dev.stop_flag = True
        dev.join(2)
        rc = lib.ll_tagged_wait(ctypes.addressof(buf), in_dim, out_dim, seq2, None, int(20e6))
        assert rc == ll.LL_ERR_TIMEOUT
    finally:
        dev.stop_flag = True
        dev.join(2)
