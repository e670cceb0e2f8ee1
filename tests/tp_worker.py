"""Worker of tests/test_gpu_tp.py: one rank of a tensor-parallel dense
decoder run, launched by torch.distributed.run (one process per GPU).  Every
rank checks its tokens against the C++ oracle (single stream, eager and CUDA
graph; continuous batching over up to 40 lanes, so both the one-block and
the 32-slot-block limb layouts run through the reduce) and rank 0 prints one
JSON line."""
import argparse
import dataclasses
import gc
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", default="fused", choices=["nccl", "fused", "fused-nccl-logits", "fused-rsag"])
    a = ap.parse_args()
    import torch
    import torch.distributed as dist

    from arc_chain_b200.formats import gen
    from arc_chain_b200.models import dense
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.oracle import arcref
    from arc_chain_b200.parallel import tp
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    rank, world = tp.init_distributed(timeout_s=60)
    comm = tp.NcclComm()
    if a.comm.startswith("fused"):
        from arc_chain_b200.parallel.fused import FusedComm

        # fused-rsag: the reduce-scatter + all-gather form at every batch size
        # fused-nccl-logits: the fused reduce with the logits gathered over NCCL
        comm = FusedComm(fuse_logits=a.comm != "fused-nccl-logits",
                         rs_ag="on" if a.comm == "fused-rsag" else "auto")
    cfg = preset("tiny")
    if cfg.n_heads % world:  # whole heads per rank: 8 heads of 64 for 8 ranks
        cfg = dataclasses.replace(cfg, d_model=512, n_heads=8, n_kv_heads=8, d_ff=1536)
    if (cfg.d_ff // world) % 16:  # TP shards of the FFN must stay 16-byte rows
        cfg = dataclasses.replace(cfg, d_ff=768)
    host = gen.random_model(cfg, 0)
    oracle = arcref.Model(host)
    eng = Engine(dense.from_host(host, "cuda", rank, world), comm=comm, n_pages=512, max_seq=256)
    res = {"comm": a.comm, "world": world, "ok": True, "checks": 0}
    prompt = gen.seeded_prompt(32, cfg.vocab, 1)
    ref, rh = oracle.generate(prompt, 24)
    for use_graph in (False, True):
        got, gh = eng.generate(prompt, 24, use_graph=use_graph)
        res["ok"] &= got == ref and gh == rh
        res["checks"] += 1
    for n_req, lanes in ((10, 8), (40, 40)):
        sch = Scheduler(eng, max_batch=lanes, prefill_chunk=32, gen_cap=24)
        specs = [(gen.seeded_prompt(3 + (5 * i) % 29, cfg.vocab, 90 + i), 4 + (i % 9)) for i in range(n_req)]
        rids = [sch.submit(p, n) for p, n in specs]
        sch.run()
        for rid, (p, n) in zip(rids, specs):
            res["ok"] &= sch.requests[rid].tokens == oracle.generate(p, n)[0]
            res["checks"] += 1
    res["kernel_errors"] = eng.check_errors()
    res["ok"] &= res["kernel_errors"] == 0
    flag = torch.tensor([0 if res["ok"] else 1], device="cuda")
    dist.all_reduce(flag)
    res["ok_all_ranks"] = int(flag.item()) == 0
    if rank == 0:
        print(json.dumps(res), flush=True)
    eng._graphs.clear()
    gc.collect()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if res["ok_all_ranks"] else 1)


if __name__ == "__main__":
    main()
