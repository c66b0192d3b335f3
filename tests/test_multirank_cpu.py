"""The N > 1 host path of bench.py on CPU: two gloo ranks exercise the host
collectives (barrier, max over ranks, gather) and the merge of per-rank serving
results that rank 0 reports."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        hg = bench.HostGroup(world)
        hg.barrier()
        top = hg.max(10.0 + rank)
        rng = np.random.default_rng(rank)
        lat = rng.uniform(3.0, 9.0, 1000 + 100 * rank)
        # as bench.py's serving section sends it: latencies, elapsed, requests and kernel passes
        per_rank = hg.gather((lat.tolist(), 0.5 + 0.25 * rank, 1000 + 100 * rank, 500 + 100 * rank))
        merged = bench.merge_serving(per_rank, 200_000.0, 2100)
        q.put((rank, top, merged, lat.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_gloo_ranks_merge_serving_results():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (top, m, lat)) for r, top, m, lat in (q.get(timeout=100) for _ in procs))
    for p in procs:
        p.join(30)
        assert p.exitcode == 0
    for r in (0, 1):
        top, merged, _ = got[r]
        assert top == 11.0  # max over ranks
        assert merged["served"] == 2100 and merged["per_rank_served"] == [1000, 1100]
        assert merged["sustained_per_s"] == pytest.approx(2100 / 0.75)  # the slowest rank's elapsed time
        assert merged["requests_per_pass"] == pytest.approx(2100 / 1100)
    every = np.concatenate([got[0][2], got[1][2]])
    assert got[0][1]["p99_us"] == pytest.approx(float(np.percentile(every, 99)))
    assert got[0][1] == got[1][1]  # every rank computes the same line


def test_single_rank_merge_has_no_collectives():
    hg = bench.HostGroup(1)
    hg.barrier()
    assert hg.max(3.5) == 3.5 and hg.gather("x") == ["x"]
    m = bench.merge_serving([([5.0, 6.0, 7.0], 1.0)], 50_000.0, 3)
    assert m["served"] == 3 and m["p50_us"] == 6.0 and m["sustained_per_s"] == 3.0


def test_merge_reports_requests_per_kernel_pass():
    # per rank: latencies, elapsed, requests taken and passes of the resident kernel
    m = bench.merge_serving([([5.0, 6.0], 1.0, 30, 12), ([7.0], 2.0, 10, 8)], 1_000_000.0, 3)
    assert m["requests_per_pass"] == pytest.approx(40 / 20)
    assert m["served"] == 3 and m["sustained_per_s"] == 1.5
    assert "requests_per_pass" not in bench.merge_serving([([5.0], 1.0)], 50_000.0, 1)


def test_ring_thread_cores_split_the_host_between_ranks():
    # the throughput leg's host threads: distinct cores, half of each rank's share, at most 8
    allowed = list(range(16))
    one = bench.ring_thread_cores(allowed, 0, 1, 0)
    assert len(one) == 8 and len(set(one)) == 8 and set(one) <= set(allowed)
    for world in (2, 4, 8):
        per = [bench.ring_thread_cores(allowed, r, world, r) for r in range(world)]
        assert all(len(c) == max(1, 16 // world // 2) for c in per)
        flat = [c for cs in per for c in cs]
        assert len(set(flat)) == len(flat) and set(flat) <= set(allowed)
    assert bench.ring_thread_cores([3], 0, 1, 0) == [3]
    assert len(bench.ring_thread_cores(list(range(64)), 0, 1, 0)) == bench.RING_ENGINES_MAX
