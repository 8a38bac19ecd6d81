"""Host-side failure detection of the head-sharded path, on CPU with gloo ranks.

A rank that leaves between steps, or stays alive but never joins the next
all-gather, must make the surviving rank's next gather end with
DzError(DZ_ENCCL) within the process group's timeout instead of hanging.  No
GPU is involved: the failure is made on the host (the ranks are processes)."""
import multiprocessing as mp
import os
import time

import pytest


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, mode, q, done):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["DZ_PG_TIMEOUT_S"] = "5"
    from daiza_b200 import parallel as P
    from daiza_b200._ffi import DZ_ENCCL, DzError
    P.init_process_group("gloo", rank=rank, world=world)
    x = torch.full((2, 8), float(rank))
    parts = P.all_gather_rows(x)                  # step 1: both ranks take part
    if rank == 1:
        if mode == "exit":
            os._exit(0)                           # leaves between steps, no goodbye
        done.wait(60)                             # "stall": alive, never joins step 2
        os._exit(0)
    ok1 = [float(p[0, 0]) for p in parts] == [0.0, 1.0]
    t0 = time.time()
    try:
        P.all_gather_rows(x)                      # step 2: the peer is gone / absent
        q.put(("no error", ok1, time.time() - t0))
    except DzError as e:
        q.put(("DzError", ok1 and e.status == DZ_ENCCL, time.time() - t0))
    except Exception as e:                        # noqa: BLE001 -- reported to the test
        q.put((type(e).__name__, ok1, time.time() - t0))
    done.set()
    os._exit(0)


@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_surviving_rank_gets_an_error(mode):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        kind, ok, dt = q.get(timeout=300)       # a cold start imports torch in both ranks
    finally:
        done.set()
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert kind == "DzError" and ok, (kind, ok)
    assert dt < 60.0
