"""Throughput of the chain-side GPU kernels against CPU implementations:
BLAKE3 batch commitments (derive-key mode, 256-byte transactions) and
Ed25519 strict batch verification.  Device time by CUDA events around the
kernel (inputs already on the device), plus the end-to-end time of the
public host API (pinned copies in, results out).  CPU baselines: the
threaded C++ commitment loop, and PyNaCl (libsodium) single-core verify.

    python -m arc_chain_b200.bench.crypto [--items 1000000] [--sigs 65536]
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch


def bench_commit(n: int, item: int = 256, reps: int = 5) -> dict:
    from arc_chain_b200.crypto import commit

    rng = np.random.default_rng(0)
    buf = rng.integers(0, 256, size=n * item, dtype=np.uint8)
    offs = np.arange(n + 1, dtype=np.int64) * item
    dev = torch.device("cuda")
    tb, to = torch.from_numpy(buf).to(dev), torch.from_numpy(offs).to(dev)
    commit.batch_commit_device(tb, to, max_item_len=item)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        out = commit.batch_commit_device(tb, to, max_item_len=item)
    e1.record()
    torch.cuda.synchronize()
    dev_s = e0.elapsed_time(e1) / 1000 / reps
    items = [bytes(buf[i * item:(i + 1) * item]) for i in range(min(n, 200000))]
    t0 = time.perf_counter()
    cpu = commit.batch_commit_cpu(items)
    cpu_s = (time.perf_counter() - t0) * n / len(items)
    t0 = time.perf_counter()
    e2e = commit.batch_commit(items)
    e2e_s = (time.perf_counter() - t0) * n / len(items)
    assert e2e == cpu
    assert bytes(out[0].cpu().numpy()) == cpu[0]
    return {"kernel": "blake3_batch_commit", "items": n, "item_bytes": item, "device_items_per_s": round(n / dev_s),
            "device_GB_s": round(n * item / dev_s / 1e9, 1), "e2e_items_per_s": round(n / e2e_s),
            "cpu_items_per_s": round(n / cpu_s), "cpu_threads": os.cpu_count()}


def bench_ed25519(n: int, reps: int = 3) -> dict:
    import nacl.signing

    from arc_chain_b200.crypto import ed25519 as G

    rng = np.random.default_rng(1)
    keys = [nacl.signing.SigningKey(rng.bytes(32)) for _ in range(64)]
    msgs, sigs, pks = [], [], []
    for i in range(n):
        k = keys[i % 64]
        m = rng.bytes(100)
        msgs.append(m)
        sigs.append(k.sign(m).signature)
        pks.append(bytes(k.verify_key))
    sig, pk, msg, offs = G.pack(msgs, sigs, pks)
    dev = torch.device("cuda")
    t = [torch.from_numpy(a.copy()).to(dev) for a in (sig, pk, msg, offs)]
    G.verify_device(*t)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        codes = G.verify_device(*t)
    e1.record()
    torch.cuda.synchronize()
    dev_s = e0.elapsed_time(e1) / 1000 / reps
    assert int((codes != 0).sum().item()) == 0
    m = min(n, 4000)
    vks = [nacl.signing.VerifyKey(p) for p in pks[:m]]
    t0 = time.perf_counter()
    for i in range(m):
        vks[i].verify(msgs[i], sigs[i])
    cpu_s = (time.perf_counter() - t0) / m
    t0 = time.perf_counter()
    ok = G.verify_batch(msgs, sigs, pks)
    e2e_s = time.perf_counter() - t0
    assert all(ok)
    return {"kernel": "ed25519_verify_strict", "sigs": n, "device_sigs_per_s": round(n / dev_s),
            "e2e_sigs_per_s": round(n / e2e_s), "cpu_1core_sigs_per_s": round(1 / cpu_s)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--items", type=int, default=1 << 20)
    ap.add_argument("--sigs", type=int, default=1 << 16)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    print(json.dumps(bench_commit(a.items)), flush=True)
    print(json.dumps(bench_ed25519(a.sigs)), flush=True)


if __name__ == "__main__":
    main()
