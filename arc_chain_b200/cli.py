"""Command-line tools, the counterparts of the reference's inference
examples and bench binaries (crates/arc-inference/examples/*.rs,
crates/arc-bench/src/*_bench.rs):

    python -m arc_chain_b200.cli info MODEL
    python -m arc_chain_b200.cli bench-int8 MODEL [--tokens 8] [--runs 7] [--save PATH] [--device cpu|cuda]
    python -m arc_chain_b200.cli generate [--preset P] [--config run.toml] [--set k=v ...]
                                          (--prompt TEXT | --prompt-ids 1,2,3) [--max-tokens N] [--oracle]
    python -m arc_chain_b200.cli perplexity MODEL (--tokens-file F | --text-file F | --seeded N) [--device cpu|cuda]
    python -m arc_chain_b200.cli convert SRC DST          # .gguf / .arc-int8 / .arc-int8v3
    python -m arc_chain_b200.cli shard MODEL OUTDIR --tp N
    python -m arc_chain_b200.cli serve [server options]
    python -m arc_chain_b200.cli nn-run FILE (--text T | --tokens 1,2 | --embedding 0.5,1 | --image-file F)
                                          [--integer]   # a NeuralNet / create_model.py file

MODEL is a model preset name (random-init weights, ``--seed``) or a file.
Every command prints one JSON object on stdout.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import math
import sys
import time
from typing import List, Optional

import numpy as np

REF_PROMPT = "[INST] What is 2+2? [/INST]"  # the prompt of the reference's bench_int8


def _host(model: str, seed: int = 0, max_seq: int = 0):
    from arc_chain_b200.config import RunConfig, load_host_model

    return load_host_model(RunConfig(model=model, seed=seed, max_seq=max_seq))


def _prompt_ids(host, text: Optional[str], ids: Optional[str], n_seeded: int = 16) -> List[int]:
    from arc_chain_b200.formats import gen
    from arc_chain_b200.formats.tokenizer import Tokenizer

    if ids:
        return [int(x) for x in ids.split(",") if x.strip()]
    if text is not None and host.vocab:
        return Tokenizer(host.vocab).encode(text)
    return gen.seeded_prompt(n_seeded, host.cfg.vocab, 1)


def _decode(host, toks) -> str:
    from arc_chain_b200.formats.tokenizer import Tokenizer

    return Tokenizer(host.vocab).decode(toks) if host.vocab else ""


def _generator(host, device: str):
    """generate(prompt, n) -> (tokens, output hash) on the CPU oracle or the GPU engine."""
    if device == "cpu":
        from arc_chain_b200.oracle import arcref

        m = arcref.Model(host)
        return m.generate
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    eng = Engine(dense.from_host(host, "cuda"))
    return eng.generate


def cmd_info(a) -> dict:
    from arc_chain_b200.runtime import attest

    host = _host(a.model, a.seed)
    c = host.cfg
    n_params = sum(d.size for _, d, _ in host.matrices())
    return {"model": a.model, "config": json.loads(c.to_json()), "model_id": attest.model_id_string(c),
            "model_hash": attest.hx(attest.model_id(c)), "weight_hash": host.weight_hash().hex(),
            "int8_params": int(n_params), "tier": attest.tier_for_params(n_params), "vocab_entries": len(host.vocab)}


def cmd_bench_int8(a) -> dict:
    """Load (and optionally save) a model, then generate the same prompt
    `runs` times and check every run's output hash (bench_int8.rs)."""
    from arc_chain_b200.formats import arc_int8

    t0 = time.perf_counter()
    host = _host(a.model, a.seed)
    load_s = time.perf_counter() - t0
    res = {"model": a.model, "load_s": round(load_s, 3), "weight_hash": host.weight_hash().hex()}
    if a.save:
        arc_int8.save(host, a.save)
        again = arc_int8.load(a.save)
        res["saved"] = a.save
        res["reload_weight_hash_equal"] = again.weight_hash() == host.weight_hash()
    prompt = _prompt_ids(host, REF_PROMPT, None)
    gen_fn = _generator(host, a.device)
    hashes, times = [], []
    toks = []
    for _ in range(a.runs):
        t0 = time.perf_counter()
        toks, h = gen_fn(prompt, a.tokens)
        times.append(time.perf_counter() - t0)
        hashes.append(h.hex())
    res.update({"device": a.device, "prompt_tokens": len(prompt), "tokens": toks, "output_text": _decode(host, toks),
                "runs": a.runs, "output_hashes": hashes, "deterministic": len(set(hashes)) == 1,
                "ms_per_token_best": round(min(times) * 1000 / max(1, a.tokens), 3)})
    return res


def cmd_generate(a) -> dict:
    from arc_chain_b200.config import RunConfig, load_host_model
    from arc_chain_b200.runtime import attest

    cfg = RunConfig.load(a.config, a.preset, a.set or [])
    host = load_host_model(cfg)
    prompt = _prompt_ids(host, a.prompt, a.prompt_ids)
    text = a.prompt if a.prompt is not None else ",".join(map(str, prompt))
    t0 = time.perf_counter()
    if a.oracle:
        from arc_chain_b200.oracle import arcref

        m = arcref.Model(host)
        if cfg.quant == "q4-row":
            m.enable_q4()
        toks, h = m.generate(prompt, a.max_tokens, eos=cfg.eos)
        engine = "arcref (CPU oracle)"
    else:
        from arc_chain_b200.models import dense
        from arc_chain_b200.runtime.engine import Engine

        q4 = "row" if cfg.quant == "q4-row" else None
        m = dense.from_host(host, "cuda", q4=q4)
        if cfg.quant == "q4-group":
            m = dense.to_q4(m, "group")
        eng = Engine(m, max_seq=cfg.max_seq or None)
        toks, h = eng.generate(prompt, a.max_tokens, eos=cfg.eos, use_graph=cfg.use_graph)
        engine = "arc_chain_b200 (B200)"
    ms = (time.perf_counter() - t0) * 1000
    out = attest.inference_result(host.cfg, text, prompt, toks, _decode(host, toks), ms, 0.0, engine)
    out["output_hash_blake3"] = h.hex()
    att = dataclasses.asdict(attest.attest(host.cfg, text, toks, host.weight_hash()))
    out["attestation"] = {k: (v.hex() if isinstance(v, bytes) else v) for k, v in att.items()}
    return out


def log_softmax_f64(logits_q16: np.ndarray) -> np.ndarray:
    """Log-softmax of Q16 logits in f64 (eval_perplexity.rs:27-38)."""
    x = np.asarray(logits_q16, dtype=np.int64).astype(np.float64) / 65536.0
    mx = x.max()
    return x - (math.log(np.exp(x - mx).sum()) + mx)


def perplexity_from_logits(logit_rows, targets, vocab: int) -> dict:
    """NLL over (logits after token i, token i + 1) pairs; an out-of-vocab
    target adds ln(-vocab), which is NaN, exactly as the reference does."""
    nll, n = 0.0, 0
    for row, t in zip(logit_rows, targets):
        lp = log_softmax_f64(row)
        if 0 <= t < lp.size:
            nll -= lp[t]
        else:
            nll = float("nan")  # the reference subtracts ln(-vocab)
        n += 1
    avg = nll / max(1, n)
    return {"tokens_evaluated": n, "avg_nll": avg, "perplexity": math.exp(avg) if avg == avg else float("nan"),
            "bits_per_token": avg / math.log(2)}


def cmd_perplexity(a) -> dict:
    from arc_chain_b200.formats import gen
    from arc_chain_b200.formats.tokenizer import Tokenizer

    host = _host(a.model, a.seed)
    if a.tokens_file:
        toks = [int(x) for x in open(a.tokens_file).read().split()]
    elif a.text_file:
        toks = Tokenizer(host.vocab).encode(open(a.text_file).read())
    else:
        toks = gen.seeded_prompt(a.seeded, host.cfg.vocab, 7)
    if a.max_tokens:
        toks = toks[:a.max_tokens]
    feed = [1] + toks[:-1]  # BOS, then each token predicts the next
    t0 = time.perf_counter()
    if a.device == "cpu":
        from arc_chain_b200.oracle import arcref

        cache = arcref.Model(host).new_cache()
        rows = [cache.forward(t) for t in feed][1:]
    else:
        from arc_chain_b200.models import dense
        from arc_chain_b200.runtime.engine import Engine

        eng = Engine(dense.from_host(host, "cuda"), max_seq=max(host.cfg.max_seq, len(feed) + 2))
        rows = list(eng.score(feed))[1:]
    res = perplexity_from_logits(rows, toks[1:], host.cfg.vocab)
    res.update({"model": a.model, "device": a.device, "seconds": round(time.perf_counter() - t0, 3)})
    return res


def cmd_convert(a) -> dict:
    from arc_chain_b200.formats import arc_int8

    host = _host(a.src, a.seed)
    if a.dst.endswith(".arc-int8v3"):
        arc_int8.save_v3(host, a.dst)
    else:
        arc_int8.save(host, a.dst)
    return {"src": a.src, "dst": a.dst, "weight_hash": host.weight_hash().hex()}


def cmd_shard(a) -> dict:
    from arc_chain_b200.formats import sharded

    host = _host(a.model, a.seed)
    man = sharded.save_sharded(host, a.outdir, a.tp)
    return {"outdir": a.outdir, "manifest": man}


def cmd_nn_run(a) -> dict:
    """Runs a NeuralNet file (the VM's tagged f32 MLP format, or
    create_model.py's) on the native library, as the VM engine's real
    compute path does (crates/arc-vm/src/inference.rs:676-723).  With
    --integer an embedding input runs through the integer form instead
    (Q16 in and out)."""
    from arc_chain_b200.formats import neuralnet
    from arc_chain_b200.utils.hashing import blake3

    raw = open(a.file, "rb").read()
    net = neuralnet.NativeNet.from_bytes(raw)
    res = {"file": a.file, "file_hash": blake3(raw).hex(), "tag_base": net.tag_base,
           "input_size": net.input_size, "output_size": net.output_size}
    if a.integer:
        if a.embedding is None:
            raise SystemExit("--integer takes an --embedding input")
        x = [neuralnet._q16(float(v)) for v in a.embedding.split(",")]
        res["output_q16"] = [int(v) for v in net.forward_q16(x)]
        return res
    if a.text is not None:
        r = neuralnet.run_request(net, "text", a.text)
    elif a.tokens is not None:
        r = neuralnet.run_request(net, "tokens", [int(t) for t in a.tokens.split(",") if t])
    elif a.embedding is not None:
        r = neuralnet.run_request(net, "embedding", [float(v) for v in a.embedding.split(",") if v])
    elif a.image_file is not None:
        r = neuralnet.run_request(net, "image", open(a.image_file, "rb").read())
    else:
        raise SystemExit("give one of --text, --tokens, --embedding, --image-file")
    out = r.output
    if hasattr(out, "tolist"):
        out = out.tolist()
    res.update({"output": out, "tokens_used": r.tokens_used, "compute_time_ms": r.compute_time_ms, "cost": r.cost})
    return res


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "serve":
        from arc_chain_b200.runtime import server

        sys.argv = ["arc_chain_b200.runtime.server"] + argv[1:]
        server.main()
        return 0
    ap = argparse.ArgumentParser(prog="arc_chain_b200.cli")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("info")
    p.add_argument("model")
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("bench-int8")
    p.add_argument("model")
    p.add_argument("--tokens", type=int, default=8)
    p.add_argument("--runs", type=int, default=7)
    p.add_argument("--save", default=None)
    p.add_argument("--device", default="cuda", choices=["cpu", "cuda"])
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("generate")
    p.add_argument("--preset", default=None)
    p.add_argument("--config", default=None)
    p.add_argument("--set", action="append", help="key=value run config override")
    p.add_argument("--prompt", default=None)
    p.add_argument("--prompt-ids", default=None)
    p.add_argument("--max-tokens", type=int, default=32)
    p.add_argument("--oracle", action="store_true", help="run the CPU oracle instead of the GPU engine")
    p = sub.add_parser("perplexity")
    p.add_argument("model")
    p.add_argument("--tokens-file", default=None)
    p.add_argument("--text-file", default=None)
    p.add_argument("--seeded", type=int, default=128)
    p.add_argument("--max-tokens", type=int, default=0)
    p.add_argument("--device", default="cuda", choices=["cpu", "cuda"])
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("convert")
    p.add_argument("src")
    p.add_argument("dst")
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("shard")
    p.add_argument("model")
    p.add_argument("outdir")
    p.add_argument("--tp", type=int, required=True)
    p.add_argument("--seed", type=int, default=0)
    p = sub.add_parser("nn-run")
    p.add_argument("file")
    p.add_argument("--text", default=None)
    p.add_argument("--tokens", default=None)
    p.add_argument("--embedding", default=None)
    p.add_argument("--image-file", default=None)
    p.add_argument("--integer", action="store_true", help="run the Q16 integer form on an --embedding input")
    a = ap.parse_args(argv)
    fn = {"info": cmd_info, "bench-int8": cmd_bench_int8, "generate": cmd_generate, "perplexity": cmd_perplexity,
          "convert": cmd_convert, "shard": cmd_shard, "nn-run": cmd_nn_run}[a.cmd]
    print(json.dumps(fn(a), default=str))
    return 0


if __name__ == "__main__":
    sys.exit(main())
