"""Tensor-parallel generate checked against the CPU oracle.

Run one process per GPU:
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m arc_chain_b200.parallel.tp_check --model micro_gqa --comm nccl
Rank 0 prints one JSON line with the tokens' hash, the oracle's hash and
whether they match (they must: integer partial sums are exact, so TP=N is
bit-identical to TP=1 and to the reference CPU engine).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from arc_chain_b200.formats import gen
from arc_chain_b200.models import dense
from arc_chain_b200.models.config import preset
from arc_chain_b200.parallel import tp
from arc_chain_b200.runtime.engine import Engine


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="micro_gqa")
    ap.add_argument("--comm", default="nccl", choices=["nccl", "fused"])
    ap.add_argument("--prompt-len", type=int, default=24)
    ap.add_argument("--gen", type=int, default=24)
    ap.add_argument("--graph", type=int, default=1)
    a = ap.parse_args()
    rank, world = tp.init_distributed()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = preset(a.model)
    host = gen.random_model(cfg, 0)
    dm = dense.from_host(host, dev, tp_rank=rank, tp_size=world)
    if a.comm == "fused":
        from arc_chain_b200.parallel.fused import FusedComm

        comm = FusedComm()
    else:
        comm = tp.NcclComm()
    eng = Engine(dm, comm=comm)
    prompt = gen.seeded_prompt(a.prompt_len, cfg.vocab, 1)
    toks, h = eng.generate(prompt, a.gen, use_graph=bool(a.graph))
    err = eng.check_errors()
    # every rank must agree
    t = torch.tensor(toks, dtype=torch.int64, device=dev)
    g = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(g, t)
    agree = all(torch.equal(x, t) for x in g)
    if rank == 0:
        from arc_chain_b200.oracle import arcref

        ref, rh = arcref.Model(host).generate(prompt, a.gen)
        print(json.dumps({"model": a.model, "tp": world, "comm": a.comm, "graph": a.graph, "match": toks == ref,
                          "ranks_agree": agree, "hash": h.hex(), "oracle_hash": rh.hex(), "kernel_errors": err}))
    eng._graphs.clear()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
