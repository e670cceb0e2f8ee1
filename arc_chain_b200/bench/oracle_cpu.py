"""The CPU baseline: the C++ oracle (a bit-exact restatement of the
reference CPU engine) timed on the host, on the same seeded workloads as
bench.py.  Prints ms/token and the BLAKE3 hash of the generated tokens,
which every B200 run of the same workload must reproduce.

    python -m arc_chain_b200.bench.oracle_cpu --model llama7b --prompt-len 128 --gen 256 [--threads N]
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np


def run(model: str, prompt_len: int, gen_len: int, threads: int = 0, seed: int = 0, prompt_seed: int = 1) -> dict:
    from arc_chain_b200.formats import gen
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.oracle import arcref

    if threads:
        arcref.lib().arcref_set_threads(threads)
    cfg = preset(model)
    cfg.max_seq = ((1 + prompt_len + gen_len + 1) + 15) // 16 * 16
    t0 = time.perf_counter()
    host = gen.random_model(cfg, seed, vocab_strings=False)
    t_gen = time.perf_counter() - t0
    om = arcref.Model(host)
    prompt = gen.seeded_prompt(prompt_len, cfg.vocab, prompt_seed)
    t0 = time.perf_counter()
    toks, h = om.generate(prompt, gen_len)
    t = time.perf_counter() - t0
    return {"oracle": "arcref (C++)", "model": model, "prompt_len": prompt_len, "gen_len": len(toks),
            "threads": int(arcref.lib().arcref_num_threads()), "cpu": os.uname().machine,
            "ms_per_token_incl_prefill": round(1000 * t / max(1, len(toks)), 2), "wall_s": round(t, 2),
            "model_gen_s": round(t_gen, 1), "output_hash": h.hex(),
            "tokens_blake3_first": {n: _hash(toks[:n]) for n in (64, 128, 136, 256) if n <= len(toks)},
            "tokens": [int(t) for t in toks]}


def _hash(t):
    from arc_chain_b200.utils.hashing import blake3

    return blake3(np.asarray(t, dtype="<u4").tobytes()).hex()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama7b")
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--threads", type=int, default=0)
    a = ap.parse_args()
    print(json.dumps(run(a.model, a.prompt_len, a.gen, a.threads)))


if __name__ == "__main__":
    main()
