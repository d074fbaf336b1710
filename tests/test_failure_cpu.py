"""Failure detection among CPU ranks (gloo): a rank that dies or stalls
between steps is detected by the survivors within a deadline through a short
process-group timeout, and surfaces as a typed error, never a hang."""
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist

    from braidinfer_b200.parallel.health import Heartbeat
    # The rendezvous gets a generous timeout (spawned ranks start at different
    # times); detection itself rests on the 2 s heartbeat deadline.
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    hb = Heartbeat(timeout_s=2.0)
    try:
        for step in range(4):
            if rank == 1 and step == 2:
                if mode == "exit":
                    os._exit(0)           # dies between steps
                time.sleep(6)             # stalls past every deadline
            t0 = time.time()
            hb.check(step)                # host-side liveness check before the step's collectives
            x = torch.ones(4) * (rank + 1)
            dist.all_reduce(x)
        q.put((rank, "finished", 0.0))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__, time.time() - t0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.timeout(120)
@pytest.mark.parametrize("mode", ["exit", "stall"])
def test_survivor_detects_dead_or_stalled_rank(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    [p.start() for p in ps]
    res = {}
    deadline = time.time() + 60
    while time.time() < deadline and 0 not in res:
        try:
            r = q.get(timeout=1)
            res[r[0]] = r
        except Exception:
            pass
    [p.join(timeout=20) for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert 0 in res, "rank 0 never reported"
    assert res[0][1] in ("PeerFailureError", "DistributedError", "RuntimeError", "DistBackendError"), res[0]
    assert res[0][2] < 15.0
