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


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config5_sharding(world):
    """Config 5's box scheduling (voxrt_b200.box): every utterance lands on exactly one rank, the longest-first
    greedy keeps the ranks' T + T^2/1500 loads within one utterance of each other, and each rank's buckets keep the
    length order and stay inside the frame budget (an utterance longer than the budget gets a bucket of its own)."""
    import numpy as np

    sys.path.insert(0, ROOT)
    from voxrt_b200 import box, synth

    secs = synth.config5_lengths()
    t_in = [synth.mel_frames(s) for s in secs]
    te = np.array([synth.out_frames(t) for t in t_in], np.int64)
    shards = box.lpt_shards(te, world)
    allu = np.sort(np.concatenate([np.array(s, np.int64) for s in shards]))
    np.testing.assert_array_equal(allu, np.arange(len(secs)))
    loads = [box.cost(te[s]).sum() for s in shards]
    assert max(loads) - min(loads) <= box.cost(te).max() + 1e-6
    plans = box.plan(t_in, world, 16384, out_frames=synth.out_frames)
    for s, bks in zip(shards, plans):
        assert all(te[a] >= te[b] for a, b in zip(s, s[1:]))
        assert [u for b in bks for u in b] == list(s)
        for b in bks:
            assert len(b) == 1 or te[b].sum() <= 16384


def test_oversized_utterance_runs_alone():
    import numpy as np

    sys.path.insert(0, ROOT)
    from voxrt_b200 import box

    te = np.array([20000, 10, 9000, 9000, 5])
    order = sorted(range(5), key=lambda u: -te[u])
    assert box.length_buckets(order, te, 16384) == [[0], [2], [3, 1, 4]]


def _plan_rank_main(rank, world, port, q):
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        from voxrt_b200 import box, synth

        secs = synth.config5_lengths()
        t_in = [synth.mel_frames(s) for s in secs]
        mine = [u for b in box.plan(t_in, world, 16384, out_frames=synth.out_frames)[rank] for u in b]
        audio = float(np.sum(secs[mine]))
        # strong scaling: the box's total audio over the slowest rank's pass time
        total = bench.reduce_over_ranks(dist, audio, "sum", "cpu")
        ms_max = bench.reduce_over_ranks(dist, 100.0 + rank, "max", "cpu")
        got = torch.zeros(len(secs), dtype=torch.int64)
        got[mine] = 1
        dist.all_reduce(got)
        q.put((rank, len(mine), total, ms_max, int(got.min()), int(got.max())))
    finally:
        dist.destroy_process_group()


def test_config5_two_gloo_ranks_share_the_box():
    """Two gloo ranks each plan their share of the same 4096 utterances: the shares are disjoint and cover the box,
    and the job value divides the box's audio by the slowest rank's time."""
    import numpy as np
    import torch.multiprocessing as mp

    sys.path.insert(0, ROOT)
    from voxrt_b200 import synth

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_plan_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res[0][1] + res[1][1] == 4096
    assert res[0][2] == res[1][2] == pytest.approx(float(np.sum(synth.config5_lengths())))
    assert res[0][3] == res[1][3] == 101.0
    assert all(r[4] == 1 and r[5] == 1 for r in res)
