"""The multi-process plumbing of bench.py on CPU: two gloo ranks, launched the way
torch.distributed.run launches them (RANK / LOCAL_RANK / WORLD_SIZE / MASTER_* in the
environment). Each rank holds independent sequences, so the only cross-rank steps are the
barriers around the timed region and the maximum of the per-rank times."""
import os
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")
ROOT = Path(__file__).resolve().parent.parent


def _rank(rank: int, world: int, port: int, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import bench
    d = bench.Dist(world)
    try:
        d.barrier()
        got = d.max(10.0 + rank)  # every rank sees the slowest rank's time
        d.barrier()
        q.put((rank, got, d.device))
    finally:
        d.close()


def test_two_rank_max_and_barrier():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=10) for _ in range(2))
    assert [r[1] for r in results] == [11.0, 11.0]
    assert all(r[2] == "cpu" for r in results)


def test_world_size_must_match_gpus(monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setenv("WORLD_SIZE", "1")
    with pytest.raises(SystemExit):
        bench.Dist(2)
