"""bench.py's multi-replica aggregation, on 2 gloo ranks (CPU): the job time is
the slowest rank's, the rate counts every rank's units."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import datetime
    import sys

    from conftest import PKG, REPO

    for p in (str(REPO), str(PKG)):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60))
    import bench

    dev = torch.device("cpu")
    ms_local = 10.0 + 5.0 * rank  # rank 1 is slower
    ms_max, rate = bench.replica_rate(1e9, ms_local, dev, world)
    total = bench.cross_rank(rank + 1, torch.distributed.ReduceOp.SUM, dev, world)
    per = bench.gather_ranks({"rank": rank, "tok_s": 100.0 * (rank + 1)}, world)

    def leg_fails_on_rank_1():
        if rank == 1:
            raise RuntimeError("planted")
        return {"rank": rank}

    failed = bench.opt_in_run(leg_fails_on_rank_1, dev, world)
    ok = bench.opt_in_run(lambda: {"rank": rank}, dev, world)
    q.put((rank, ms_max, rate, total, per, failed, ok))
    torch.distributed.destroy_process_group()


def test_replica_rate_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, ms_max, rate, total, per, failed, ok in got:
        # an opt-in leg that raised on one rank is reported as failed on both,
        # after the same collectives; one that ran everywhere returns its result
        assert failed == (None, "RuntimeError: planted" if rank == 1 else "failed on another rank")
        assert ok == ({"rank": rank}, None)
        assert ms_max == pytest.approx(15.0)           # the slowest rank
        assert rate == pytest.approx(2e9 / 15e-3)      # both ranks' units / job time
        assert total == pytest.approx(3.0)
        # every rank sees every rank's summary, in rank order
        assert per == [{"rank": 0, "tok_s": 100.0}, {"rank": 1, "tok_s": 200.0}]


def test_replica_rate_single_process_is_identity():
    import bench

    ms, rate = bench.replica_rate(2e9, 4.0, torch.device("cpu"), 1)
    assert ms == 4.0 and rate == pytest.approx(2e9 / 4e-3)
