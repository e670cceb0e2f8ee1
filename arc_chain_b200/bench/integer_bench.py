"""Cross-platform determinism benchmark of the small integer transformer
(the reference's ``arc-bench-integer``, crates/arc-bench/src/integer_bench.rs):
three LCG-seeded models, prompt [1, 2, 3, 4, 5], 16 new tokens, EOS 99;
per model the determinism over ``--runs`` runs, the output hash and the
latency distribution.  Prints the same JSON document shape.

    python -m arc_chain_b200.bench.integer_bench [--runs 100]
"""
from __future__ import annotations

import argparse
import json
import platform
import sys
import time

from arc_chain_b200.models.toy_integer import ToyIntegerModel

CONFIGS = [("2-layer tiny (v=50, d=32, h=2, ff=64)", 50, 32, 2, 64, 2),
           ("4-layer small (v=100, d=64, h=2, ff=128)", 100, 64, 2, 128, 4),
           ("4-layer medium (v=200, d=128, h=4, ff=256)", 200, 128, 4, 256, 4)]


def run(runs: int = 100, prompt=(1, 2, 3, 4, 5), max_tokens: int = 16, eos: int = 99) -> dict:
    results = []
    for name, v, d, h, ff, nl in CONFIGS:
        m = ToyIntegerModel(v, d, h, ff, nl)
        m.generate_with_hash(prompt, max_tokens, eos)  # warm-up
        hashes, lat, first = [], [], None
        for i in range(runs):
            t0 = time.perf_counter()
            toks, hh = m.generate_with_hash(prompt, max_tokens, eos)
            lat.append(int((time.perf_counter() - t0) * 1e6))
            hashes.append(hh)
            if i == 0:
                first = toks
        s = sorted(lat)
        results.append({"name": name, "vocab_size": v, "d_model": d, "n_heads": h, "d_ff": ff, "n_layers": nl,
                        "runs": runs, "deterministic": all(x == hashes[0] for x in hashes),
                        "output_hash": hashes[0].hex(), "generated_tokens": first,
                        "avg_us": sum(lat) / len(lat), "p50_us": s[len(s) // 2],
                        "p99_us": s[min(len(s) - 1, (len(s) * 99) // 100)]})
    return {"benchmark": "IntegerEngine", "platform": f"{sys.platform} {platform.machine()}", "models": results}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--runs", type=int, default=100)
    a = ap.parse_args()
    print(json.dumps(run(a.runs), indent=2))


if __name__ == "__main__":
    main()
