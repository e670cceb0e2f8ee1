"""Worker of tests/test_gpu_ep.py: one rank of an expert-parallel MLA + MoE
run, launched by torch.distributed.run (one process per GPU).  Every rank
checks its tokens against the numpy oracle and rank 0 prints one JSON line."""
import argparse
import gc
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--comm", default="fused", choices=["nccl", "fused", "dispatch"])
    a = ap.parse_args()
    import torch
    import torch.distributed as dist

    from arc_chain_b200.formats import gen
    from arc_chain_b200.models import mla_moe, mla_moe_engine as me
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.parallel import tp
    from arc_chain_b200.parallel.ep import EpDispatchComm, EpFusedComm, EpNcclComm
    from arc_chain_b200.runtime.scheduler import Scheduler

    rank, world = tp.init_distributed(timeout_s=60)
    cfg = preset("micro_moe")
    host = gen.random_model(cfg, 4)
    orc = mla_moe.MlaMoeOracle
    comm = {"fused": EpFusedComm, "nccl": EpNcclComm, "dispatch": EpDispatchComm}[a.comm]()
    eng = me.MlaMoeEngine(me.from_host(host, "cuda", rank, world), comm=comm)
    res = {"comm": a.comm, "world": world, "ok": True, "checks": 0}
    if a.comm == "dispatch":
        # token dispatch: every rank decodes its own prompts in lockstep
        # (equal lengths, different tokens) and checks them against the oracle
        prompt = gen.seeded_prompt(9, cfg.vocab, 3 + rank)
        ref, rh = orc(host).generate(prompt, 12)
        for use_graph in (False, True):
            got, gh = eng.generate(prompt, 12, use_graph=use_graph)
            res["ok"] &= got == ref and gh == rh
            res["checks"] += 1
        # three lanes per rank: prefill each (lockstep), then batched decode
        lanes, n_gen = 3, 7
        prompts = [gen.seeded_prompt(5 + 4 * i, cfg.vocab, 50 + 10 * rank + i) for i in range(lanes)]
        rids = []
        for p in prompts:
            rid = eng.new_request(1 + len(p) + n_gen)
            eng.prefill(rid, [1] + p)
            rids.append(rid)
        bb = eng.buffers(lanes, gen_cap=n_gen)
        eng._reset_sampling(bb, rids, [p[-1] for p in prompts], [len(p) + 1 for p in prompts], ())
        g = eng._graph_for(bb)
        for _ in range(n_gen):
            g.replay()
        torch.cuda.synchronize()
        for i, p in enumerate(prompts):
            got = [int(t) for t in bb.gen[i, :int(bb.count[i].item())].tolist()]
            res["ok"] &= got == orc(host).generate(p, n_gen)[0]
            res["checks"] += 1
        g = None
        res["kernel_errors"] = eng.check_errors()
        res["ok"] &= res["kernel_errors"] == 0
        return _finish(res, rank, eng)
    prompt = gen.seeded_prompt(9, cfg.vocab, 3)
    ref, rh = orc(host).generate(prompt, 12)
    for use_graph in (False, True):
        got, gh = eng.generate(prompt, 12, use_graph=use_graph)
        res["ok"] &= got == ref and gh == rh
        res["checks"] += 1
    sch = Scheduler(eng, max_batch=8, prefill_chunk=16, gen_cap=10)
    specs = [(gen.seeded_prompt(3 + 2 * i, cfg.vocab, 90 + i), 5 + (i % 4)) for i in range(10)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        res["ok"] &= sch.requests[rid].tokens == orc(host).generate(p, n)[0]
        res["checks"] += 1
    res["kernel_errors"] = eng.check_errors()
    res["ok"] &= res["kernel_errors"] == 0
    return _finish(res, rank, eng)


def _finish(res, rank, eng):
    import torch
    import torch.distributed as dist

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
