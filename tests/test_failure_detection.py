"""Failure detection on the host with gloo ranks (no GPU is faulted, trapped
or hung): a rank that raises, a rank that exits, and a rank that stalls are
all reported to the survivors as RankFailure within the timeout, before any
collective would block.  The GPU side (a bounded in-kernel wait running out)
is tested in test_gpu_bounded_waits.py."""
import datetime
import multiprocessing as mp
import os
import socket
import time

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q):
    import torch.distributed as dist

    from arc_chain_b200.parallel.health import Heartbeat, RankFailure

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, timeout_s=2.0)
    try:
        for step in range(4):
            if rank == 1 and step == 2:
                if mode == "raise":
                    hb.fail("injected exception in rank 1")
                    q.put((rank, "raised"))
                    return
                if mode == "exit":
                    q.put((rank, "exited"))
                    os._exit(0)
                if mode == "stall":
                    q.put((rank, "stalled"))
                    time.sleep(6)
                    return
            hb.beat(step)
            hb.wait_peers(step)
        q.put((rank, "ok"))
    except RankFailure as e:
        q.put((rank, f"failure:{e.ranks}"))
    finally:
        if mode == "none" or rank == 0:
            try:
                dist.destroy_process_group()
            except Exception:
                pass


@pytest.mark.parametrize("mode", ["none", "raise", "exit", "stall"])
def test_heartbeat_detects_failed_rank(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    t0 = time.time()
    while len(res) < 2 and time.time() - t0 < 60:
        try:
            r, v = q.get(timeout=1)
            res[r] = v
        except Exception:
            pass
    for p in ps:
        p.join(timeout=15)
        if p.is_alive():
            p.kill()
    if mode == "none":
        assert res == {0: "ok", 1: "ok"}
    else:
        assert res.get(0) == "failure:[1]", res


def test_replay_request_needs_exact_prefix():
    from arc_chain_b200.parallel.health import replay_request

    class Fake:
        def generate(self, prompt, n, eos=()):
            return list(range(n)), b""

    assert replay_request(Fake(), [1], [0, 1], 4) == [0, 1, 2, 3]
    with pytest.raises(AssertionError):
        replay_request(Fake(), [1], [5], 4)
