"""The bench's multi-rank bookkeeping (one process per GPU on a real run) on
two gloo ranks on the CPU: rank set-up from the torchrun environment, the
whole-job throughput = all ranks' tokens over the slowest rank's time, and
the reference arm's non-zero ranks exiting without work."""
import multiprocessing as mp
import os
import socket
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    sys.path.insert(0, REPO)
    try:
        import bench
        import torch.distributed as dist
        w, r, local = bench.dist_setup(world)
        # rank r ran 10 * (r + 1) tokens in (r + 1) * 100 ms of device time, (r + 1) * 0.2 s wall
        value, e2e, max_ms = bench.job_throughput(w, 10 * (r + 1), (r + 1) * 100.0, (r + 1) * 0.2)
        bench.barrier(w)

        class A:
            steps, warmup, workload = 2, 1, "ragged64"
        ref = bench.run_reference(A) if r != 0 else "skipped"
        dist.destroy_process_group()
        q.put((r, w, local, value, e2e, max_ms, ref))
    except Exception as ex:  # reported to the parent
        q.put((rank, "error", repr(ex)))


def test_two_gloo_ranks_whole_job_throughput():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(o[1] != "error" for o in out), out
    tokens = 10 + 20
    for r, w, local, value, e2e, max_ms, ref in out:
        assert w == world and local == r
        assert max_ms == pytest.approx(200.0)  # the slowest rank's device time
        assert value == pytest.approx(tokens / 0.2)
        assert e2e == pytest.approx(tokens / 0.4)
        if r != 0:
            assert ref is None  # only rank 0 times the reference arm
