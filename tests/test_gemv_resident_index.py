"""Host restatement of the resident small-batch kernel's request and reply index arithmetic
(low_latency_inference_gpu_b200/csrc/gemv_net.cuh, RES = true) -- test infrastructure.

For every row count and width the engine accepts, each load from the host-mapped mailbox
stays inside its x rows [max_batch][in], each store into the L2 relay / gather buffers
inside [32][in] / [32][out], each store into the mailbox inside its y rows, and every 16-byte
piece of the request is copied exactly once.  Also checked: the host's queue split gives a
launch exactly as many requests as the kernel serves before its 16-bit tags run out."""
import pytest

THREADS = 256        # kGvThreads
TAG_ROWS = 4         # kGvTagRows
MAX_ROWS = 32        # kGvMaxRows
SPEC, REST, YB = 4, 4, 2  # loads a thread keeps in flight: first rows, other rows, y
TAG_LIMIT = 0xFFFF   # kGvTagLimit
TAG_CHUNKS = 4       # chunks a lane of the tagged poll holds


def x_copy(in_dim, max_rows, rows):
    """(mailbox float4 index, relay float4 index) pairs of one TickBuffer request."""
    q = in_dim // 4
    spec = min(min(max_rows, TAG_ROWS) * q, SPEC * THREADS) // q * q
    n4 = rows * q
    reads, writes = [], []
    for tid in range(THREADS):
        for u in range(SPEC):  # speculative loads, before the row count is known
            if tid + u * THREADS < spec:
                reads.append(tid + u * THREADS)
        for u in range(SPEC):
            i = tid + u * THREADS
            if i < min(spec, n4):
                writes.append((i, i))
        i0 = spec + tid
        while i0 < n4:  # the other rows: REST loads in flight, then REST stores
            for u in range(REST):
                i = i0 + u * THREADS
                if i < n4:
                    reads.append(i)
                    writes.append((i, i))
            i0 += REST * THREADS
    return spec, n4, reads, writes


@pytest.mark.parametrize("in_dim", [4, 64, 252, 256, 1024, 2048])
def test_request_rows_are_read_in_bounds_and_relayed_once(in_dim):
    q = in_dim // 4
    for max_rows in range(1, MAX_ROWS + 1):
        # the kernel clamps a request's row count to max_rows
        for rows in sorted(r for r in {1, 2, max_rows // 2, max_rows} if 1 <= r <= max_rows):
            spec, n4, reads, writes = x_copy(in_dim, max_rows, rows)
            assert spec % q == 0 and spec <= max_rows * q
            assert all(0 <= r < max_rows * q for r in reads)         # inside the mailbox's x rows
            dst = [d for _, d in writes]
            assert sorted(dst) == list(range(n4))                    # every piece once
            assert all(s == d for s, d in writes) and n4 <= MAX_ROWS * q  # inside the relay


@pytest.mark.parametrize("out_dim", [4, 16, 64, 96, 256])
def test_reply_rows_are_written_in_bounds_once(out_dim):
    for rows in range(1, MAX_ROWS + 1):
        n4 = rows * out_dim // 4
        seen = []
        for tid in range(THREADS):
            i0 = tid
            while i0 < n4:
                for u in range(YB):
                    i = i0 + u * THREADS
                    if i < n4:
                        seen.append(i)
                i0 += YB * THREADS
        assert sorted(seen) == list(range(n4))  # gather [32][out] read and mailbox y rows written once each


@pytest.mark.parametrize("in_dim,out_dim", [(1, 1), (4, 4), (256, 64), (382, 95), (384, 96)])
def test_tagged_poll_and_reply_chunks(in_dim, out_dim):
    # batch 1: warp 0 holds every x chunk {v0, v1, v2, seq}; the reply is (out + 2) / 3 chunks
    nxc = (in_dim + 2) // 3
    held = [lane + 32 * j for lane in range(32) for j in range(TAG_CHUNKS) if lane + 32 * j < nxc]
    assert sorted(held) == list(range(nxc))
    relay = [3 * ch + e for ch in held for e in range(3) if 3 * ch + e < in_dim]
    assert sorted(relay) == list(range(in_dim))
    nyc = (out_dim + 2) // 3
    gather = [3 * t + e for t in range(nyc) for e in range(3) if 3 * t + e < out_dim]
    assert sorted(gather) == list(range(out_dim))


@pytest.mark.parametrize("layers", range(1, 25))
def test_queue_split_matches_the_tag_budget(layers):
    # the kernel takes request k (tag base 1 + k * layers) while base + layers <= 65535; the
    # last layer is counted, so the highest tag used is base + layers - 2
    served = 0
    while 1 + served * layers + layers <= TAG_LIMIT:
        assert 1 + served * layers + max(layers - 2, 0) <= TAG_LIMIT
        served += 1
    assert served == (TAG_LIMIT - 1) // layers  # the host's per-launch cap in ll_engine_run_queue
