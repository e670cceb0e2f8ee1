"""Small launches of single hot kernels, sized for profiler captures: each
target holds at most a few GB on the device and launches its kernel a
handful of times (a warm-up, then the launches to capture).

    python -m arc_chain_b200.bench.profile_targets <target>

targets (kernel name to select, launches before the first timed one):
  attn        k_attn_paged     7B decode attention, T = 386, 32 heads    (3)
  gemm_b1     k_gemm_fused     7B gate/up 22016 x 4096 at B = 1          (5)
  gemm_b256   k_gemm_fused     70B gate/up 57344 x 8192 at B = 256       (5)
  commit      k_batch_commit   BLAKE3 derive-key commit, 1M x 256 B      (1)
  ed25519     k_verify         Ed25519 verify_strict, 65,536 signatures  (1)
  mla_attn    k_attn_cluster   MLA latent attention, 16 heads, T = 512, B = 32 (3)
  moe_route   k_moe_route      top-6 of 64 experts + 2 shared, B = 32    (3)
  q4_gemm     k_gemm_fused     7B gate/up as group-32 Q4 at B = 1        (5)
  sample      k_sample         penalty + argmax, vocab 32000, B = 1      (3)
  norm_limbs  k_norm_limbs     RMSNorm apply + limb split, d = 4096      (3)

Every target prints its CUDA-event time per launch with the SM clocks
sampled while it ran (nvidia-smi, read-only).
"""
from __future__ import annotations

import json
import sys

import torch


def _clocked(run) -> None:
    """Runs run(iters) (a benchmark returning a dict) with the clock sampler
    on: enough iterations for samples on a plain run, two under a profiler
    (PT_SECONDS=0); prints the dict with the clock record."""
    import os

    from arc_chain_b200.utils.clocks import ClockSampler

    import time

    secs = float(os.environ.get("PT_SECONDS", "1.0"))
    with ClockSampler(0, period_ms=50) as clk:
        w0 = time.perf_counter()
        res = run(2 if secs == 0 else 400)
        while time.perf_counter() - w0 < secs:  # repeat so the sampler sees the load
            res = run(400)
    res["clocks"] = clk.summary()
    print(json.dumps(res), flush=True)


def attn():
    from arc_chain_b200.bench.kernels import bench_attn

    _clocked(lambda n: bench_attn(386, iters=n))


def gemm_b1():
    from arc_chain_b200.bench.kernels import bench_fgemm

    _clocked(lambda n: bench_fgemm(22016, 4096, 1, iters=n))


def gemm_b256():
    from arc_chain_b200.bench.kernels import bench_fgemm

    _clocked(lambda n: bench_fgemm(57344, 8192, 256, iters=max(2, n // 8), limbs=4))


def commit():
    from arc_chain_b200.bench.crypto import bench_commit

    _clocked(lambda n: bench_commit(1 << 20, reps=max(2, n // 20)))


def ed25519():
    from arc_chain_b200.bench.crypto import bench_ed25519

    _clocked(lambda n: bench_ed25519(1 << 16, reps=max(2, n // 40)))


def _timed(fn, warm: int, iters: int, extra: dict) -> None:
    """Runs fn `warm` times, then times `iters` launches with CUDA events
    while sampling clocks; prints one JSON line."""
    from arc_chain_b200.utils.clocks import ClockSampler

    import os
    import time

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    # PT_SECONDS: keep launching for this long so the clock sampler sees the
    # timed region (0 under a profiler: only the first launches are captured)
    secs = float(os.environ.get("PT_SECONDS", "1.0"))
    with ClockSampler(0, period_ms=50) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        n, w0 = 0, time.perf_counter()
        while n < iters or time.perf_counter() - w0 < secs:
            for _ in range(iters):
                fn()
            n += iters
            if secs > 0:
                torch.cuda.synchronize()
        t1.record()
        torch.cuda.synchronize()
    iters = n
    us = t0.elapsed_time(t1) * 1000 / iters
    extra.update({"us": round(us, 2), "clocks": clk.summary()})
    if "bytes" in extra:
        from arc_chain_b200.bench.kernels import hbm_peak_gbs

        extra["GB_s"] = round(extra["bytes"] / us / 1e3, 1)
        extra["frac_of_measured_hbm"] = round(extra["GB_s"] / hbm_peak_gbs(), 3)
    print(json.dumps(extra), flush=True)


def mla_attn():
    """MLA latent attention (DeepSeek-V2-Lite, 16 heads, T = 512); B and the
    cluster size from ARCB_PT_B / ARCB_PT_CS (default 32 slots, heuristic)."""
    import os

    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    H, r, dr, T = 16, 512, 64, 512
    B = int(os.environ.get("ARCB_PT_B", "32"))
    cs = int(os.environ.get("ARCB_PT_CS", "0")) or None
    dk = r + dr
    pages = (T + 15) // 16
    cache = torch.randint(-(1 << 18), 1 << 18, (B * pages, 1, 16, dk), dtype=torch.int64, device=dev)
    Q = torch.randint(-(1 << 18), 1 << 18, (B, H, dk), dtype=torch.int64, device=dev)
    oc = torch.zeros(B, H, r, dtype=torch.int64, device=dev)
    pt = torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages)
    pos = torch.full((B,), T - 1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _timed(lambda: ops.attn_mla(Q, cache, pt, pos, H, dk, r, 5793, T, B, oc, err, cluster=cs), 3, 10,
           {"kernel": "attn_mla (k_attn_cluster)", "heads": H, "dk": dk, "dv": r, "T": T, "B": B,
            "cluster": cs or ops.attn_cluster_size(B, H), "bytes": B * T * dk * 8})
    assert int(err.item()) == 0


def moe_route():
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    B, E, S, k = 32, 64, 2, 6
    lg = torch.randint(-(1 << 20), 1 << 20, (B, E), dtype=torch.int64, device=dev)
    route = torch.zeros(B, E + S, dtype=torch.int64, device=dev)
    _timed(lambda: ops.moe_route(lg, E, S, k, B, route), 3, 20,
           {"kernel": "k_moe_route", "B": B, "experts": E, "shared": S, "top_k": k})


def q4_gemm():
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    M, K, B = 22016, 4096, 1
    w = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev)
    q, mult = ops.q4_group_quantize(w)
    packs = [ops.pack_q4(q, mult) for _ in range(3)]
    del w, q
    S = torch.randint(1, 100, (M,), dtype=torch.int64, device=dev)
    bn = ops.fgemm_bn(B)
    X = torch.randint(-127, 128, (ops.limb_rows(B, bn), K), dtype=torch.int8, device=dev)
    xm = ops.TensorMap(X, bn)
    lmax = torch.tensor([3], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    e = ops.epi(ops.STORE, S, err, out=out, ldo=M)
    e.max_ctas = ops.split_ctas(M, B, bn)
    it = [0]

    def run():
        ops.fgemm_q4(packs[it[0] % 3], xm, M, K, B, lmax, P, tiles, e)
        it[0] += 1

    _timed(run, 5, 20, {"kernel": "k_gemm_fused<16,Q4>", "M": M, "K": K, "B": B,
                        "bytes": M * K // 2 + M * (K // 32) // 2})
    assert int(err.item()) == 0


def sample():
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    V, B = 32000, 1
    logits = torch.randint(-(1 << 30), 1 << 30, (B, V), dtype=torch.int64, device=dev)
    hist = torch.randint(0, V, (B, 64), dtype=torch.int32, device=dev)
    count = torch.full((B,), 40, dtype=torch.int32, device=dev)
    gen_ = torch.zeros(B, 1 << 20, dtype=torch.int32, device=dev)
    tok = torch.zeros(B, dtype=torch.int32, device=dev)
    _timed(lambda: ops.sample(logits, V, B, hist, count, gen_, tok), 3, 20,
           {"kernel": "k_sample", "vocab": V, "B": B, "bytes": B * V * 8})


def norm_limbs():
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    d, B = 4096, 1
    h = torch.randint(-(1 << 24), 1 << 24, (B, d), dtype=torch.int64, device=dev)
    ss = torch.full((B,), 1 << 40, dtype=torch.int64, device=dev)
    g = torch.randint(1 << 15, 1 << 17, (d,), dtype=torch.int64, device=dev)
    X = torch.zeros(ops.limb_rows(B), d, dtype=torch.int8, device=dev)
    lm = torch.zeros(1, dtype=torch.int32, device=dev)
    _timed(lambda: ops.norm_limbs(h, ss, g, d, B, X, lm), 3, 20,
           {"kernel": "k_norm_limbs", "d": d, "B": B, "bytes": B * d * (8 + 8) + 8 * d})



def attn_block():
    """Grouped-query block decode attention: 128 slots x 1 KV head (8 query
    heads), T = 800 (the 70B TP8 shape): one wave of 128 CTAs."""
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    B, H, KV, DH, T = 128, 8, 1, 128, 800
    pages = (T + 15) // 16
    K = torch.randint(-(1 << 18), 1 << 18, (B * pages, KV, 16, DH), dtype=torch.int64, device=dev)
    V = torch.randint(-(1 << 18), 1 << 18, (B * pages, KV, 16, DH), dtype=torch.int64, device=dev)
    q = torch.randint(-(1 << 18), 1 << 18, (B, H * DH), dtype=torch.int64, device=dev)
    pt = torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages)
    pos = torch.full((B,), T - 1, dtype=torch.int32, device=dev)
    X = torch.zeros(ops.limb_rows(B), H * DH, dtype=torch.int8, device=dev)
    lm = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _timed(lambda: ops.attn_gqa_block(q, K, V, pt, pos, H, KV, DH, 5793, B, X, lm, T, T, err), 3, 10,
           {"kernel": "k_attn_block<8,128,1>", "B": B, "heads": H, "kv_heads": KV, "T": T,
            "bytes": 2 * B * T * KV * DH * 8})
    assert int(err.item()) == 0


def moe_gemm():
    """Expert GEMMs of one MoE layer, DeepSeek-V2-Lite shapes with 33 local
    experts (expert parallelism over 2 GPUs), 32 gathered slots, 4 limbs:
    gate/up (SwiGLU epilogue writing the down GEMM's limb planes) and down
    (grouped: each expert reads its own 1408 columns; routing-weighted
    combine into the hidden state).  ARCB_PT_MOE=down times the down GEMM."""
    import os

    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    G, F, d, B = 33, 1408, 2048, 32
    which = os.environ.get("ARCB_PT_MOE", "gate_up")
    bn = ops.fgemm_bn(B)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    if which == "gate_up":
        M, K = G * 2 * F, d
    else:
        M, K = G * d, G * F
    W = ops.tile_weight(torch.randint(-127, 128, (M, K if which == "gate_up" else F), dtype=torch.int8, device=dev))
    wm = ops.TensorMap(W, 128)
    S = torch.randint(1, 100, (M,), dtype=torch.int64, device=dev)
    X = torch.randint(-127, 128, (ops.limb_rows(B, bn), K), dtype=torch.int8, device=dev)
    xm = ops.TensorMap(X, bn, min(bn, 32))
    lmax = torch.tensor([4], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    if which == "gate_up":
        Xm = torch.zeros(ops.limb_rows(B, bn), G * F, dtype=torch.int8, device=dev)
        lo = torch.zeros(1, dtype=torch.int32, device=dev)
        e = ops.epi(ops.SWIGLU, S, err, X=Xm, ldx=G * F, lmax_out=lo)
        nbytes = M * K
    else:
        h = torch.zeros(B, d, dtype=torch.int64, device=dev)
        # 8 of the 66 experts per slot carry weight (6 routed + 2 shared)
        route = torch.zeros(B, 66, dtype=torch.int64, device=dev)
        route[:, torch.randperm(66)[:8]] = 8192
        e = ops.epi(ops.MOE_COMBINE, S, err, out=h, ldo=d, route=route, route_ld=66)
        e.grp_rows, e.grp_koff = d, F
        nbytes = M * F
    e.max_ctas = min(ops.num_sms(), ops.split_ctas(M, B, bn))
    _timed(lambda: ops.fgemm(wm, xm, M, K if which == "gate_up" else F, B, lmax, P, tiles, e), 3, 10,
           {"kernel": f"k_gemm_fused<256,0,0> expert {which}", "M": M, "K": K, "B": B, "limbs": 4,
            "bytes": nbytes})
    assert int(err.item()) == 0


TARGETS = {"moe_gemm": moe_gemm, "attn_block": attn_block, "attn": attn, "gemm_b1": gemm_b1, "gemm_b256": gemm_b256, "commit": commit, "ed25519": ed25519,
           "mla_attn": mla_attn, "moe_route": moe_route, "q4_gemm": q4_gemm, "sample": sample,
           "norm_limbs": norm_limbs}


def main():
    torch.cuda.set_device(0)
    TARGETS[sys.argv[1]]()


if __name__ == "__main__":
    main()
