"""The multi-GPU plumbing of bench.py on CPU: two gloo ranks (world size 2, 127.0.0.1) run bench.Ranks the way
`torchrun --nproc-per-node 2 bench.py` does. Each rank times its own GPU's whole conversations with no collective on
the data path; the only cross-rank steps are the barrier around the timed region and the max of the per-rank times,
and the job value counts every rank's tokens (weak scaling)."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench
    r = bench.Ranks()
    r.barrier()
    ms = 10.0 + 5.0 * rank                      # each rank's own device time
    worst = r.max(ms)
    tokens_per_rank = 2 * 128                   # the riding step: 2 tokens per step, 128 steps
    value = r.world * tokens_per_rank / (worst / 1e3)
    out.put((rank, r.world, r.local, worst, value))
    r.close()


def test_two_gloo_ranks_barrier_and_max():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(k, 2, port, q)) for k in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[0] for r in res] == [0, 1]
    assert all(r[1] == 2 for r in res) and [r[2] for r in res] == [0, 1]
    assert all(r[3] == pytest.approx(15.0) for r in res)          # the slowest rank's time, on every rank
    assert all(r[4] == pytest.approx(2 * 256 / 0.015) for r in res)


def test_single_rank_needs_no_process_group(monkeypatch):
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    sys.path.insert(0, ROOT)
    import bench
    r = bench.Ranks()
    assert (r.rank, r.world, r.local) == (0, 1, 0)
    assert r.max(3.5) == 3.5
    r.barrier()
    r.close()
