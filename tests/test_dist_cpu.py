"""Multi-process host logic on CPU (gloo, world_size 2): utterance partitioning, the
whole-job rate (sum of units over the slowest rank), and re-queueing the utterances of a
rank whose work failed.  No GPU and no data-path collective is involved."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, mode):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from __graft_entry__ import load_package
    load_package()
    import datetime

    import torch.distributed as dist
    from voxcpm_rs_b200 import dist as vxd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        rate = vxd.aggregate_rate(10.0 * (rank + 1), 1.0 + rank)  # units 10, 20; seconds 1, 2 -> 30/2
        items = list(range(9))

        def work(x):
            if mode == "rank1_down" and rank == 1:
                raise RuntimeError("simulated failure of rank 1")
            if mode == "item7_bad" and x == 7:
                raise RuntimeError("simulated failure of item 7")
            return x * x
        if mode.startswith("waves"):
            # 20 utterances in waves of up to 4 per rank; in "waves_bad" the wave holding
            # utterance 13 raises on rank 1, so its 4 utterances are re-queued to rank 0

            def work_batch(xs):
                if mode == "waves_bad" and rank == 1 and 13 in xs:
                    raise RuntimeError("simulated failure of a wave")
                assert len(xs) <= 4
                return [x * x for x in xs]
            done = vxd.run_partitioned(list(range(20)), work_batch, batch=4)
        else:
            done = vxd.run_partitioned(items, work)
        q.put((rank, rate, done))
    finally:
        dist.destroy_process_group()


def test_partition_covers_everything():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from voxcpm_rs_b200 import dist as vxd
    for n, w in ((64, 1), (64, 2), (64, 8), (10, 3), (3, 4)):
        parts = [vxd.partition(n, w, r) for r in range(w)]
        flat = [i for p in parts for i in p]
        assert flat == list(range(n))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1


def test_waves():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from voxcpm_rs_b200 import dist as vxd
    assert vxd.waves(list(range(10)), 4) == [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9]]
    assert vxd.waves([], 8) == []


@pytest.mark.parametrize("mode", ["ok", "rank1_down", "item7_bad", "waves", "waves_bad"])
def test_two_rank_partition_and_requeue(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=90) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rates = {r: rate for r, rate, _ in results}
    assert rates[0] == rates[1] == pytest.approx(15.0)
    merged = {}
    for _, _, done in results:
        for k, v in done.items():
            assert k not in merged
            merged[k] = v
    if mode.startswith("waves"):
        # every utterance completes exactly once; a failed wave is retried by a healthy rank
        assert merged == {i: i * i for i in range(20)}
        return
    if mode == "item7_bad":
        # item 7 fails on every rank: everything else completes exactly once
        assert merged == {i: i * i for i in range(9) if i != 7}
    else:
        # with rank 1 down, rank 0 re-runs rank 1's utterances: all complete exactly once
        assert merged == {i: i * i for i in range(9)}
    if mode == "rank1_down":
        assert all(k in results[[r for r, _, _ in results].index(0)][2] for k in range(9))
