"""Data-parallel replicas on gloo CPU ranks with the C++ oracle as the
backend: request sharding returns every result in order on every rank and
equals one-process generation; cross-replica agreement accepts identical
hashes and names a dissenting replica."""
import datetime
import os
import socket
import time

import torch.multiprocessing as mp

from arc_chain_b200.parallel.dp import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _requests(vocab):
    from arc_chain_b200.formats import gen

    return [(gen.seeded_prompt(3 + i, vocab, 70 + i), 3 + i % 4) for i in range(7)]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from arc_chain_b200.formats import gen
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.oracle import arcref
    from arc_chain_b200.parallel.dp import ReplicaGroup

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        host = gen.random_model(preset("micro"), 0)
        m = arcref.Model(host)
        g = ReplicaGroup(m.generate)
        res = g.run(_requests(host.cfg.vocab))
        ok = g.agree([5, 6, 7], 4)
        # rank 1 is a faulty replica: its backend returns a different hash
        bad = ReplicaGroup(lambda p, n: (m.generate(p, n)[0], b"\x00" * 32 if rank == 1 else m.generate(p, n)[1]))
        dis = bad.agree([5, 6, 7], 4, min_agree=2)
        q.put((rank, [(t, h.hex()) for t, h in res], ok, dis))
    finally:
        dist.destroy_process_group()


def test_shard():
    assert shard(7, 1, 3) == [1, 4] and sorted(sum((shard(7, r, 3) for r in range(3)), [])) == list(range(7))


def test_replicas_shard_and_agree():
    from arc_chain_b200.formats import gen
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.oracle import arcref

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    t0 = time.time()
    while len(out) < 2 and time.time() - t0 < 120:
        try:
            r, *v = q.get(timeout=1)
            out[r] = v
        except Exception:
            pass
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(out) == 2
    host = gen.random_model(preset("micro"), 0)
    m = arcref.Model(host)
    want = [(t, h.hex()) for t, h in (m.generate(p, n) for p, n in _requests(host.cfg.vocab))]
    for r in (0, 1):
        res, ok, dis = out[r]
        assert [(list(t), h) for t, h in res] == want
        assert ok["accepted"] and ok["agree"] == 2 and ok["dissenting_ranks"] == []
        assert not dis["accepted"] and dis["agree"] == 1 and len(dis["dissenting_ranks"]) == 1
