"""The other benchmark workloads (besides the 7B single-stream decode in
bench.py): continuous batching, MLA + MoE batched decode, speculative
decoding.  Each returns a dict for bench.py's JSON line.  All use seeded
random-init weights and seeded prompts; timing is CUDA events around the
device work (max over ranks when distributed)."""
from __future__ import annotations

import os
import time

import torch

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset


def _sync_barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def batched(model: str, n_requests: int, rank: int, world: int, comm, max_batch: int = 128,
            prompt_range=(64, 1024), out_range=(128, 512), seed: int = 2) -> dict:
    """Continuous batching: requests with seeded prompt/output lengths."""
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.kv_paged import PAGE, PagedKV
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset(model)
    plens = gen.seeded_lengths(n_requests, *prompt_range, seed=seed, stream=0xFFFF0001)
    olens = gen.seeded_lengths(n_requests, *out_range, seed=seed, stream=0xFFFF0002)
    cfg.max_seq = (max(p + o for p, o in zip(plens, olens)) + 2 + 15) // 16 * 16
    dev = torch.device("cuda", torch.cuda.current_device())
    m = dense.random_device(cfg, dev, seed=0, tp_rank=rank, tp_size=world)
    lanes = min(max_batch, n_requests)
    need_pages = sum((1 + p + o + PAGE - 1) // PAGE for p, o in zip(plens, olens)) + 2
    free = torch.cuda.mem_get_info()[0]
    per = PagedKV.bytes_per_page(cfg.n_layers, m.n_kv_local, cfg.d_head)
    budget = int(free * 0.75) - 8 * lanes * (1 << 20)
    n_pages = max(4 * ((cfg.max_seq + 15) // 16), min(need_pages, budget // per))
    eng = Engine(m, max_seq=cfg.max_seq, comm=comm, n_pages=n_pages)
    sch = Scheduler(eng, max_batch=lanes, prefill_chunk=1024, gen_cap=max(olens))
    for i in range(n_requests):
        sch.submit(gen.seeded_prompt(plens[i], cfg.vocab, 1000 + i), olens[i])
    sch.phase_events = []  # device time of prefill and decode, separately
    # warm-up: one step builds the decode graph
    _sync_barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    sch.run()
    e1.record()
    _sync_barrier(world)
    wall = time.perf_counter() - t0
    dev_ms = _max_over_ranks(e0.elapsed_time(e1), world)
    gen_tokens = sum(len(r.tokens) for r in sch.requests.values())
    prompt_tokens = sum(plens)
    return {"metric": f"{model} INT8 continuous batching tok/s", "value": round(gen_tokens / (dev_ms / 1000), 2),
            "unit": "generated tokens/s", "higher_is_better": True, "n_requests": n_requests, "lanes": lanes,
            "generated_tokens": gen_tokens, "prompt_tokens": prompt_tokens, "device_ms": round(dev_ms, 2),
            "wall_s": round(wall, 3), "decode_steps": sch.steps, "kv_pages": n_pages,
            "device_ms_by_phase": sch.phase_times_ms(),
            "config": {"model": model, "parallelism": f"tp{world}", "prompt_len": list(prompt_range),
                       "out_len": list(out_range)}}


def moe_decode(model: str, batch: int, prompt_len: int, gen_len: int, steps: int, warmup: int, rank: int = 0,
               world: int = 1, comm=None) -> dict:
    """MLA + MoE batched greedy decode; expert-parallel over `world` ranks
    (weights generated on each device, experts g % world == rank).  With a
    token-dispatch communicator each rank owns batch / world of the
    requests (its own attention, KV cache and dense layers) and the MoE
    layers exchange tokens; otherwise every rank runs all `batch` tokens."""
    from arc_chain_b200.models import mla_moe_engine as me

    cfg = preset(model)
    cfg.max_seq = (prompt_len + gen_len + 2 + 15) // 16 * 16
    m = me.random_device(cfg, torch.device("cuda", torch.cuda.current_device()), 0, rank, world)
    dispatch = world > 1 and getattr(comm, "token_dispatch", False)
    if dispatch and batch % world:
        raise ValueError(f"batch {batch} does not split over {world} ranks")
    local = batch // world if dispatch else batch
    first = rank * local if dispatch else 0
    eng = me.MlaMoeEngine(m, n_pages=local * ((cfg.max_seq + 15) // 16) + 4, comm=comm if world > 1 else None)
    bb = eng.buffers(local, gen_cap=gen_len)
    rids = []
    for i in range(first, first + local):
        p = gen.seeded_prompt(prompt_len, cfg.vocab, 1 + i)
        rid = eng.new_request(1 + prompt_len + gen_len)
        eng.prefill(rid, [1] + p)
        rids.append((rid, p))
    eng._reset_sampling(bb, [r for r, _ in rids], [p[-1] for _, p in rids], [prompt_len + 1] * local, ())
    g = eng._graph_for(bb)
    for _ in range(warmup):
        g.replay()
    _sync_barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = min(steps, gen_len - warmup)
    e0.record()
    for _ in range(n):
        g.replay()
    e1.record()
    _sync_barrier(world)
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    err = eng.check_errors()
    g = None
    eng._graphs.clear()
    return {"metric": f"{model} MLA+MoE INT8 batched decode tok/s", "value": round(batch * n / (ms / 1000), 2),
            "unit": "tokens/s", "higher_is_better": True, "ms_per_step": round(ms / n, 4), "batch": batch,
            "steps": n, "warmup": warmup, "kernel_errors": err,
            "config": {"model": model, "prompt_len": prompt_len, "gen_len": gen_len, "parallelism": f"ep{world}",
                       "slots_per_rank": local,
                       "comm": getattr(comm, "__class__", type(None)).__name__ if world > 1 else "none"}}


def spec_decode(target: str, draft: str, batch: int, prompt_len: int, gen_len: int, k: int, rank: int, world: int,
                comm) -> dict:
    """Speculative decoding: Q4 group-32 target (TP=world), INT8 draft on rank 0."""
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.spec_decode import SpecDecoder

    tc = preset(target)
    tc.max_seq = (prompt_len + gen_len + k + 3 + 15) // 16 * 16
    dev = torch.device("cuda", torch.cuda.current_device())
    tm = dense.to_q4(dense.random_device(tc, dev, seed=0, tp_rank=rank, tp_size=world), "group")
    teng = Engine(tm, max_seq=tc.max_seq, comm=comm, n_pages=batch * ((tc.max_seq + 15) // 16) + 4)
    deng = None
    if rank == 0:
        if draft == "self":
            # the target's own weights (unsharded, Q4 group-32) as the draft:
            # every proposal is accepted, so the run shows the speculative
            # path's best case and its verify cost
            dm = dense.to_q4(dense.random_device(tc, dev, seed=0), "group")
            deng = Engine(dm, max_seq=tc.max_seq, n_pages=batch * ((tc.max_seq + 15) // 16) + 4)
        else:
            dc = preset(draft)
            dc.max_seq = tc.max_seq
            deng = Engine(dense.random_device(dc, dev, seed=1), max_seq=dc.max_seq,
                          n_pages=batch * ((dc.max_seq + 15) // 16) + 4)
    sd = SpecDecoder(teng, deng, k=k, lanes=batch, gen_cap=gen_len)
    prompts = [gen.seeded_prompt(prompt_len, tc.vocab, 1 + i) for i in range(batch)]
    _sync_barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    out = sd.generate(prompts, gen_len)
    e1.record()
    _sync_barrier(world)
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    toks = sum(len(t) for t, _ in out)
    exact = None
    if os.environ.get("ARCB_SPEC_CHECK", "1") != "0":
        # every sequence equals plain greedy decoding of the target
        plain = [teng.generate(p, gen_len)[0] for p in prompts]
        exact = all(list(t) == pl for (t, _), pl in zip(out, plain))
    note = ("the draft is the target itself: every proposal is accepted" if draft == "self" else
            "random-init target and draft are unrelated models, so almost no draft token is accepted")
    return {"metric": f"speculative decoding ({target} Q4 g32 + {draft} draft) tok/s",
            "value": round(toks / (ms / 1000), 2), "unit": "tokens/s", "higher_is_better": True,
            "acceptance": round(sd.acceptance, 4), "rounds": sd.rounds, "tokens": toks, "device_ms": round(ms, 2),
            "config": {"target": target, "draft": draft, "k": k, "batch": batch, "prompt_len": prompt_len,
                       "gen_len": gen_len, "parallelism": f"tp{world}"},
            "equals_plain_greedy": exact, "note": note}
