"""bench.py's multi-rank host logic on CPU: two gloo ranks (127.0.0.1) check that every rank draws its own
utterances (weak scaling) and that the job value is the sum of the ranks' audio over the slowest rank's step."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench

        secs, t_in, _ = bench.workload(rank)
        audio = float(sum(secs))
        ms = 10.0 + 5.0 * rank  # rank 1 is the slow one
        value, ms_max, total = bench.rank_value(audio, ms, dist, "cpu")
        q.put((rank, audio, list(map(int, t_in[:4])), value, ms_max, total))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    (r0, a0, t0, v0, m0, s0), (r1, a1, t1, v1, m1, s1) = res
    assert t0 != t1, "ranks must draw different utterances"
    assert m0 == m1 == 15.0 and s0 == s1 == pytest.approx(a0 + a1)
    assert v0 == v1 == pytest.approx((a0 + a1) / 0.015)
