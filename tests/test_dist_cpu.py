"""The multi-process path of bench.py on CPU: two ranks over the gloo backend
(one process per GPU on a B200 box, NCCL there). Checks the rank environment,
the per-rank seeds (every rank compacts its own cache), the max-over-ranks
step time and the whole-job throughput (weak scaling: all ranks' tokens over
the slowest rank's time)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    from kvc_b200 import dist as kdist
    try:
        r, w = kdist.init("gloo", timeout_s=60)
        assert (r, w) == (rank, world)
        kdist.barrier(w)
        step_ms = 10.0 + 5.0 * rank                 # rank 1 is the slow one
        ms_max = kdist.max_over_ranks(step_ms, w)
        value = kdist.job_tokens_per_s(w, 100_000, ms_max)
        seed = kdist.rank_seed(1000, r)
        kdist.finish(w)
        q.put((rank, ms_max, value, seed, None))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, None, None, repr(e)))


def test_two_rank_weak_scaling_reduction():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, ms_max, value, seed, err = q.get(timeout=120)
        assert err is None, err
        out[rank] = (ms_max, value, seed)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][0] == out[1][0] == pytest.approx(15.0)            # the slowest rank's time
    assert out[0][1] == pytest.approx(2 * 100_000 / 15e-3)          # every rank's tokens
    assert out[0][2] != out[1][2]                                   # distinct caches


def test_single_rank_defaults(monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    from kvc_b200 import dist as kdist
    assert kdist.env_ranks() == (0, 1, 0)
    assert kdist.max_over_ranks(3.5, 1) == 3.5
    assert kdist.job_tokens_per_s(1, 100_000, 50.0) == pytest.approx(2e6)
