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
    """Config 5's box scheduling: every utterance lands on exactly one rank, the longest-first greedy keeps the
    ranks' T + T^2/1500 loads within one utterance of each other, and each rank's buckets keep the length order and
    stay inside the frame budget (an utterance longer than the budget gets a bucket of its own)."""
    import numpy as np

    sys.path.insert(0, ROOT)
    import bench
    from voxrt_b200 import synth

    secs = synth.config5_lengths()
    te = np.array([synth.out_frames(synth.mel_frames(s)) for s in secs], np.int64)
    shards = bench.shard_config5(len(secs), te, world)
    allu = np.sort(np.concatenate([np.array(s, np.int64) for s in shards]))
    np.testing.assert_array_equal(allu, np.arange(len(secs)))
    cost = te + te.astype(np.float64) ** 2 / 1500.0
    loads = [cost[s].sum() for s in shards]
    assert max(loads) - min(loads) <= cost.max() + 1e-6
    for s in shards:
        assert all(te[a] >= te[b] for a, b in zip(s, s[1:]))
        bks = bench.buckets(s, te, 16384)
        assert [u for b in bks for u in b] == list(s)
        for b in bks:
            assert len(b) == 1 or te[b].sum() <= 16384
