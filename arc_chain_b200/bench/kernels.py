"""Kernel microbenchmarks with roofline fractions.

Times each hot kernel alone with CUDA events after warm-up, rotating over
enough weight copies that every launch streams from HBM (working set > the
126 MB L2).  Reports achieved bandwidth against the measured HBM copy peak
(MEASURED_PEAKS.json ``hbm_gbs``; 6650 GB/s fallback) as JSON lines.

    python -m arc_chain_b200.bench.kernels [--shape 22016x4096] [--B 1] [--iters 50]
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from arc_chain_b200.ops import int_ops as ops

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
SHAPES_7B = {"qkv": (12288, 4096), "wo": (4096, 4096), "gate_up": (22016, 4096), "down": (4096, 11008),
             "lm_head": (32000, 4096)}
# DeepSeek-V2-Lite architecture: stacked 66-expert gate/up and down, MLA W_o.
SHAPES_MOE = {"moe_gate_up": (185856, 2048), "moe_down": (135168, 1408), "mla_wo": (2048, 2048),
              "mla_q": (3072, 2048)}


def hbm_peak_gbs() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return 6650.0


def bench_fgemm(M, K, B, iters=50, mode="store", pdl=True, sub_box=None, ctas=None, limbs=3, sched=0):
    """One fused GEMM alone.  sub_box: rows per TMA box of the limb operand
    (None = the whole BN tile); ctas: persistent CTA budget (None = the
    split_ctas heuristic, 0 = one per SM); limbs: device limb count; sched:
    work schedule of multi-n-tile launches (0 = round-robin / grouped, 1 =
    plain stream-K)."""
    dev = torch.device("cuda")
    nbytes = M * K
    copies = max(2, -(-300_000_000 // nbytes))
    Ws = [ops.tile_weight(torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev)) for _ in range(copies)]
    maps = [ops.TensorMap(w, 128) for w in Ws]
    S = torch.randint(1, 100, (M,), dtype=torch.int64, device=dev)
    bn = ops.fgemm_bn(B)
    X = torch.randint(-127, 128, (ops.limb_rows(B, bn), K), dtype=torch.int8, device=dev)
    xm = ops.TensorMap(X, bn, min(sub_box, bn) if sub_box else None)
    lmax = torch.tensor([limbs], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    e = ops.epi(ops.STORE if mode == "store" else ops.PARTIAL, S, err, out=out, ldo=M)
    e.max_ctas = ops.split_ctas(M, B, bn) if ctas is None else ctas
    e.sched = sched
    ops.set_pdl(pdl)
    for i in range(5):
        ops.fgemm(maps[i % copies], xm, M, K, B, lmax, P, tiles, e)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(iters):
        ops.fgemm(maps[i % copies], xm, M, K, B, lmax, P, tiles, e)
    t1.record()
    torch.cuda.synchronize()
    us = t0.elapsed_time(t1) * 1000 / iters
    gbs = nbytes / us / 1e3
    assert int(err.item()) == 0
    return {"kernel": "fgemm", "M": M, "K": K, "B": B, "mode": mode, "pdl": pdl, "sub_box": sub_box,
            "ctas": e.max_ctas, "limbs": limbs, "sched": sched, "us": round(us, 2),
            "GB_s": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm_peak_gbs(), 3)}


def bench_attn(T, n_heads=32, dh=128, B=1, iters=50, cluster=None, paged=True, n_kv=None):
    """Decode attention over T cached tokens; paged selects the TMA-fed
    page-ring form (else per-thread loads); n_kv < n_heads is grouped-query
    attention, also timed in the block form (one CTA per slot and KV head)."""
    dev = torch.device("cuda")
    n_kv = n_kv or n_heads
    ops.set_attn_paged(paged)
    pages = (T + 15) // 16
    npg = pages * B
    K = torch.randint(-(1 << 18), 1 << 18, (npg, n_kv, 16, dh), dtype=torch.int64, device=dev)
    V = torch.randint(-(1 << 18), 1 << 18, (npg, n_kv, 16, dh), dtype=torch.int64, device=dev)
    q = torch.randint(-(1 << 18), 1 << 18, (B, n_heads * dh), dtype=torch.int64, device=dev)
    pt = torch.arange(npg, dtype=torch.int32, device=dev).view(B, pages)
    pos = torch.full((B,), T - 1, dtype=torch.int32, device=dev)
    X = torch.zeros(ops.limb_rows(B), n_heads * dh, dtype=torch.int8, device=dev)
    lm = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(3):
        ops.attn(q, K, V, pt, pos, n_heads, n_kv, dh, 5793, B, X, lm, pages * 16, err, cluster=cluster)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(iters):
        ops.attn(q, K, V, pt, pos, n_heads, n_kv, dh, 5793, B, X, lm, pages * 16, err, cluster=cluster)
    t1.record()
    torch.cuda.synchronize()
    us = t0.elapsed_time(t1) * 1000 / iters
    assert int(err.item()) == 0
    nbytes = 2 * B * T * n_kv * dh * 8  # the K and V bytes, each read once
    ops.set_attn_paged(True)
    kind = "attn_paged" if paged else "attn_cluster"
    res = {"kernel": kind, "T": T, "heads": n_heads, "kv_heads": n_kv, "B": B, "us": round(us, 2),
           "frac_of_measured_hbm": round(nbytes / us / 1e3 / hbm_peak_gbs(), 3),
           "GB_s": round(nbytes / us / 1e3, 1), "cluster": cluster or ops.attn_cluster_size(B, n_heads)}
    if n_kv < n_heads and n_heads // n_kv <= 8:
        # the block form: one CTA per (slot, KV head) for its query heads
        X2 = torch.zeros_like(X)
        run = lambda: ops.attn_gqa_block(q, K, V, pt, pos, n_heads, n_kv, dh, 5793, B, X2, lm, pages * 16,
                                         pages * 16, err)
        if run():
            torch.cuda.synchronize()
            t0.record()
            for _ in range(iters):
                run()
            t1.record()
            torch.cuda.synchronize()
            ub = t0.elapsed_time(t1) * 1000 / iters
            res["gqa_block_us"] = round(ub, 2)
            res["gqa_block_frac_of_measured_hbm"] = round(nbytes / ub / 1e3 / hbm_peak_gbs(), 3)
    return res



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=1)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--only", default="")
    ap.add_argument("--model", default="")
    ap.add_argument("--T", type=int, default=800)
    ap.add_argument("--shape", default="", help="one of " + ",".join(SHAPES_7B))
    a = ap.parse_args()
    torch.cuda.set_device(0)
    if a.shape:
        M, K = SHAPES_7B[a.shape]
        r = bench_fgemm(M, K, a.B, a.iters)
        r["name"] = a.shape
        print(json.dumps(r), flush=True)
        return
    if a.only in ("", "gemm"):
        for name, (M, K) in SHAPES_7B.items():
            for pdl in (True, False):
                r = bench_fgemm(M, K, a.B, a.iters, pdl=pdl)
                r["name"] = name
                print(json.dumps(r), flush=True)
    if a.only == "optimeline_batched":
        from arc_chain_b200.utils.clocks import ClockSampler

        with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
            r = op_timeline_batched(a.model or "llama70b", a.B if a.B > 1 else 64, a.T)
        r["clocks"] = clk.summary()
        if r["rank"] == 0:
            print(json.dumps(r), flush=True)
        return
    if a.only == "optimeline":
        # per-op device time of one eager 7B decode step (CUDA events between launches)
        from arc_chain_b200.utils.clocks import ClockSampler

        with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
            r = op_timeline()
        r["clocks"] = clk.summary()
        if r["rank"] == 0:
            print(json.dumps(r), flush=True)
        return
    if a.only == "optimeline_moe":
        # per-op device time of one eager MLA + MoE decode step (expert-parallel under torch.distributed.run)
        from arc_chain_b200.utils.clocks import ClockSampler

        with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
            r = op_timeline_moe(a.model or "dsv2lite", a.B if a.B > 1 else 32, a.T,
                                layout=os.environ.get("ARCB_EP_LAYOUT", "dispatch"))
        r["clocks"] = clk.summary()
        if r["rank"] == 0:
            print(json.dumps(r), flush=True)
        return
    if a.only == "large":
        # 70B-architecture shapes at prefill / batched sizes: time and int8 tensor rate
        shapes = {"70b_qkv": (10240, 8192), "70b_wo": (8192, 8192), "70b_gate_up": (57344, 8192),
                  "70b_down": (8192, 28672)}
        for B in (64, 256, 1024):
            for name, (M, K) in shapes.items():
                for sched in (0, 1):
                    r = bench_fgemm(M, K, B, max(3, a.iters // 5), limbs=4, sched=sched)
                    r["name"] = name
                    r["int8_TOPS"] = round(2 * M * K * 4 * B / (r["us"] * 1e-6) / 1e12, 1)
                    print(json.dumps(r), flush=True)
        return
    if a.only == "attn_batch":
        # attention forms across decode / batched / prefill-like grids
        for B, heads, T in ((1, 32, 386), (8, 32, 386), (32, 32, 386), (64, 8, 512), (256, 8, 512), (512, 8, 256)):
            for paged in (True, False):
                print(json.dumps(bench_attn(T, n_heads=heads, B=B, iters=a.iters, paged=paged)), flush=True)
        return
    if a.only == "attn_gqa":
        # 70B-style grouped-query decode (64 query / 8 KV heads; TP8 shard 8 / 1)
        for B, heads, kv, T in ((1, 64, 8, 1024), (16, 64, 8, 800), (64, 64, 8, 800), (64, 8, 1, 800), (128, 8, 1, 800)):
            for paged in (True, False):
                print(json.dumps(bench_attn(T, n_heads=heads, B=B, iters=a.iters, paged=paged, n_kv=kv)), flush=True)
        return
    if a.only == "attn_cs":
        for T in (130, 386, 1024):
            for cs in (1, 2, 4, 8):
                for paged in (True, False):
                    print(json.dumps(bench_attn(T, B=a.B, iters=a.iters, cluster=cs, paged=paged)), flush=True)
        return
    if a.only == "batch":
        # sub-box limb loads and CTA budget across batch sizes
        shapes = dict(SHAPES_7B, **SHAPES_MOE)
        for B in (1, 8, 32):
            for name in ("qkv", "gate_up", "moe_gate_up", "moe_down", "mla_wo", "mla_q"):
                M, K = shapes[name]
                for sub, ctas in ((None, 0), (32, 0), (32, None)):
                    r = bench_fgemm(M, K, B, a.iters, sub_box=sub, ctas=ctas)
                    r["name"] = name
                    print(json.dumps(r), flush=True)
        return
    if a.only == "timeline":
        for name, (M, K) in SHAPES_7B.items():
            print(json.dumps(timeline_fgemm(M, K, a.B)), flush=True)
        return
    if a.only in ("", "attn"):
        for T in (130, 386, 1024, 2048):
            for paged in (True, False):
                print(json.dumps(bench_attn(T, B=a.B, iters=a.iters, paged=paged)), flush=True)



def timeline_fgemm(M, K, B=1, reps=5):
    """Per-CTA %globaltimer stamps of one fused GEMM (microseconds from the
    earliest CTA entry): entry, after the dependency wait, first stage
    consumed, last MMA issued, epilogue done, exit."""
    dev = torch.device("cuda")
    W = ops.tile_weight(torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev))
    wm = ops.TensorMap(W, 128)
    S = torch.randint(1, 100, (M,), dtype=torch.int64, device=dev)
    bn = ops.fgemm_bn(B)
    X = torch.randint(-127, 128, (ops.limb_rows(B, bn), K), dtype=torch.int8, device=dev)
    xm = ops.TensorMap(X, bn)
    lmax = torch.tensor([3], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    prof = torch.zeros(ops.num_sms() * 8, dtype=torch.int64, device=dev)
    e = ops.epi(ops.STORE, S, err, out=out, ldo=M)
    e.prof = prof.data_ptr()
    flush = torch.empty(256 << 20, dtype=torch.int8, device=dev)
    res = []
    for _ in range(reps):
        flush.zero_()
        prof.zero_()
        ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, e, pdl=False)
        torch.cuda.synchronize()
        t = prof.view(-1, 8).cpu().numpy().astype("float64")
        t0 = t[:, 0][t[:, 0] > 0].min()
        row = {}
        for k, name in ((0, "entry"), (1, "dep_wait"), (2, "first_stage"), (3, "last_mma"), (4, "epi_done"),
                        (6, "exit")):
            v = t[:, k][t[:, k] > 0] - t0
            if len(v):
                row[name] = [round(float(x) / 1000, 2) for x in (v.min(), float(__import__("numpy").median(v)), v.max())]
        res.append(row)
    return {"kernel": "fgemm_timeline", "M": M, "K": K, "B": B, "us_min_med_max": res[-1]}




def op_timeline(prompt_len: int = 128, reps: int = 5) -> dict:
    """Mean device time of each op of one eager decode step of the 7B
    architecture (events recorded between launches; the whole step is queued
    behind a sleep so launch overhead is not timed), one rank per GPU when
    launched under torch.distributed.run (fused in-kernel reduce)."""
    import collections

    import torch.distributed as dist

    from arc_chain_b200.formats import gen
    from arc_chain_b200.models import dense
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.runtime.engine import Comm, Engine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank, comm = 0, Comm()
    if world > 1:
        from arc_chain_b200.parallel import tp
        from arc_chain_b200.parallel.fused import FusedComm

        rank, world = tp.init_distributed()
        comm = FusedComm()
    else:
        torch.cuda.set_device(0)
    cfg = preset("llama7b")
    cfg.max_seq = 400
    m = dense.random_device(cfg, torch.device("cuda", torch.cuda.current_device()), seed=0, tp_rank=rank,
                            tp_size=world)
    eng = Engine(m, max_seq=400, comm=comm, n_pages=64)
    p = gen.seeded_prompt(prompt_len, cfg.vocab, 1)
    rid = eng.new_request(prompt_len + 100)
    eng.prefill(rid, [1] + p)
    bb = eng.buffers(1, gen_cap=64)
    eng._reset_sampling(bb, [rid], [p[-1]], [prompt_len + 1], ())
    for _ in range(3):
        eng.decode_step(bb)
    agg, cnt = collections.defaultdict(float), collections.Counter()
    for _ in range(reps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        eng.op_events = []
        torch.cuda._sleep(80_000_000)
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.decode_step(bb)
        torch.cuda.synchronize()
        prev = e0
        for lab, e in eng.op_events:
            agg[lab] += prev.elapsed_time(e) * 1000 / reps
            cnt[lab] += 1
            prev = e
        eng.op_events = None
    agg = _max_over_ranks(agg, world)
    out = {"world": world, "total_us": round(sum(agg.values()), 1),
           "per_op_us": {k: {"launches": cnt[k] // reps, "total": round(v, 1), "each": round(v / max(1, cnt[k] // reps), 2)}
                         for k, v in agg.items()}, "rank": rank}
    if world > 1:
        import gc

        eng._graphs.clear()
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    return out



def _max_over_ranks(agg: dict, world: int) -> dict:
    """Per-label device times, each the maximum over the ranks (every rank
    records the same labels in the same order)."""
    if world <= 1:
        return dict(agg)
    import torch.distributed as dist

    keys = list(agg)
    t = torch.tensor([agg[k] for k in keys], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return dict(zip(keys, t.tolist()))


def op_timeline_moe(model: str = "dsv2lite", B: int = 32, T: int = 512, reps: int = 3,
                    layout: str = "dispatch") -> dict:
    """Per-op device time of one eager MLA + MoE decode step over B slots in
    total (every slot at position T - 1, distinct pages), expert-parallel over
    the ranks of torch.distributed.run (token dispatch: B / N slots per rank;
    replicated: all B on every rank), each op the maximum over ranks."""
    import collections

    import torch.distributed as dist

    from arc_chain_b200.models import mla_moe_engine as me
    from arc_chain_b200.models.config import preset

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank, comm = 0, None
    if world > 1:
        from arc_chain_b200.parallel import tp
        from arc_chain_b200.parallel.ep import EpDispatchComm, EpFusedComm

        rank, world = tp.init_distributed()
        comm = EpDispatchComm() if layout == "dispatch" else EpFusedComm()
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = preset(model)
    cfg.max_seq = (T + 16 + 15) // 16 * 16
    local = B // world if (world > 1 and layout == "dispatch") else B
    m = me.random_device(cfg, dev, 0, rank, world)
    pps = cfg.max_seq // 16
    eng = me.MlaMoeEngine(m, n_pages=local * pps + 4, comm=comm)
    bb = eng.buffers(local, gen_cap=8)
    bb.tokens.copy_(torch.arange(local, dtype=torch.int32) * 7 + 3 + rank)
    bb.pos.fill_(T - 1)
    bb.pt.copy_(torch.arange(local * pps, dtype=torch.int32).view(local, pps)[:, :bb.pt.shape[1]])
    for _ in range(2):
        eng.forward(bb, local, True)
    agg, cnt = collections.defaultdict(float), collections.Counter()
    for _ in range(reps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        eng.op_events = []
        torch.cuda._sleep(80_000_000)
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.forward(bb, local, True)
        torch.cuda.synchronize()
        prev = e0
        for lab, e in eng.op_events:
            agg[lab] += prev.elapsed_time(e) * 1000 / reps
            cnt[lab] += 1
            prev = e
        eng.op_events = None
    agg = _max_over_ranks(agg, world)
    out = {"model": model, "B": B, "slots_per_rank": local, "T": T, "world": world, "layout": layout,
           "total_us": round(sum(agg.values()), 1), "kernel_errors": eng.check_errors(),
           "per_op_us": {k: {"launches": cnt[k] // reps, "total": round(v, 1),
                             "each": round(v / max(1, cnt[k] // reps), 2)} for k, v in agg.items()}, "rank": rank}
    if world > 1:
        import gc

        eng._graphs.clear()
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    return out


def op_timeline_batched(model: str = "llama70b", B: int = 64, T: int = 800, reps: int = 3) -> dict:
    """Per-op device time of one eager decode step over B slots, every slot at
    position T - 1 (distinct pages): where a batched step's time goes.  Under
    torch.distributed.run: tensor-parallel over the ranks (fused in-kernel
    reduce), each op the maximum over ranks."""
    import collections

    import torch.distributed as dist

    from arc_chain_b200.models import dense
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.runtime.engine import Comm, Engine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank, comm = 0, Comm()
    if world > 1:
        from arc_chain_b200.parallel import tp
        from arc_chain_b200.parallel.fused import FusedComm

        rank, world = tp.init_distributed()
        comm = FusedComm()
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = preset(model)
    cfg.max_seq = (T + 16 + 15) // 16 * 16
    m = dense.random_device(cfg, dev, seed=0, tp_rank=rank, tp_size=world)
    pps = cfg.max_seq // 16
    eng = Engine(m, max_seq=cfg.max_seq, n_pages=B * pps + 4, comm=comm)
    bb = eng.buffers(B, gen_cap=8)
    bb.tokens.copy_(torch.arange(B, dtype=torch.int32) * 7 + 3)
    bb.pos.fill_(T - 1)
    bb.pt.copy_(torch.arange(B * pps, dtype=torch.int32).view(B, pps)[:, :bb.pt.shape[1]])
    for _ in range(2):
        eng.forward(bb, B, True)
    agg, cnt = collections.defaultdict(float), collections.Counter()
    for _ in range(reps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        eng.op_events = []
        torch.cuda._sleep(80_000_000)
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        eng.forward(bb, B, True)
        torch.cuda.synchronize()
        prev = e0
        for lab, e in eng.op_events:
            agg[lab] += prev.elapsed_time(e) * 1000 / reps
            cnt[lab] += 1
            prev = e
        eng.op_events = None
    agg = _max_over_ranks(agg, world)
    out = {"model": model, "B": B, "T": T, "world": world, "total_us": round(sum(agg.values()), 1),
           "kernel_errors": eng.check_errors(), "rank": rank,
           "per_op_us": {k: {"launches": cnt[k] // reps, "total": round(v, 1), "each": round(v / max(1, cnt[k] // reps), 2)}
                         for k, v in agg.items()}}
    if world > 1:
        import gc

        eng._graphs.clear()
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
