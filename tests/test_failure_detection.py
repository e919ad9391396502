"""Failure detection without a GPU fault.

- On the GPU: a bounded wait that nothing completes (q3_selftest_wait_timeout: the mbarrier wait
  the pipelined kernels use, on a phase no copy will ever complete) gives up after its limit, the
  kernel returns, the wait-timeout flag comes back through q3_device_error, and the context keeps
  working: a kernel launched afterwards produces its normal result.
- On the CPU: the multi-rank plumbing of bench.py (gloo, world size 2) when one rank leaves before
  the timed region. The surviving rank's next collective ends with an error within the process
  group's timeout instead of waiting for ever; nothing of the decode path is involved.
"""
import os
import sys
import time
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(HERE))
import conftest  # noqa: E402,F401

torch = pytest.importorskip("torch")


@pytest.mark.gpu
def test_bounded_wait_times_out_and_context_survives():
    import llm_inference_b200 as q3
    from llm_inference_b200 import _lib
    assert q3.device_error() == 0
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    t0 = time.monotonic()
    _lib.call("q3_selftest_wait_timeout", done.data_ptr(), s)
    flags = q3.device_error()
    elapsed = time.monotonic() - t0
    assert flags == 1, f"device flags {flags}: expected the wait-timeout bit alone"
    assert int(done.item()) == 2
    assert 1.0 < elapsed < 30.0, f"the wait gave up after {elapsed:.1f} s"
    # the context still works: an exact kernel after the timed-out wait
    x = torch.arange(64, dtype=torch.float32, device="cuda").bfloat16()
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    q3.argmax_forward(out, x, 64)
    assert int(out.item()) == 63
    assert q3.device_error() == 0


def _rank(rank: int, world: int, port: int, q):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    os.environ["CUDA_VISIBLE_DEVICES"] = ""  # host-side plumbing only
    sys.path.insert(0, str(ROOT))
    import datetime

    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
    import bench
    d = bench.Dist.__new__(bench.Dist)  # the bench's wrapper over an existing group
    d.world, d.rank, d.local_rank, d.device, d.pg = world, rank, rank, "cpu", dist
    d.barrier()  # both ranks reach the start
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # leaves between steps: no collective of its own in flight
    t0 = time.monotonic()
    try:
        d.max(1.0)  # the next step's collective: its peer is gone
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 -- gloo raises RuntimeError subclasses
        q.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_exit_ends_peer_collective_with_error():
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
    got = dict(q.get(timeout=10) for _ in range(2))
    assert got[1] == "left"
    assert got[0].startswith("error after"), got[0]
    assert float(got[0].split()[2].rstrip("s:")) < 60
