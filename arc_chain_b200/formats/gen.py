"""Seeded random-init models and prompts.

The generator is SplitMix64 used as a counter-based stream (definition in
``csrc/common/rng.h``); numpy, the C++ oracle and the CUDA fill kernel produce
identical values, so models of any size can be generated where they are used
(host for files and the oracle, device for the benchmarks) and still be the
same model.

Tensor streams: stream = (tensor_id << 2) | kind, kind 0 = data, 1 = scales /
norm values.  tensor ids: embedding 0, output 1, final_norm 2, then for
layer l: 3 + 9*l + j with j over (wq, wk, wv, wo, gate, up, down, attn_norm,
ffn_norm).  MLA/MoE tensors use ids from ``EXT_BASE`` (see ``ext_tensor_id``).

Value rules (all integer):
* int8 weight = (r % 255) - 127, uniform in [-127, 127];
* per-row Q16 scale = s_base + (r % (s_base // 8 + 1)) with
  s_base = max(1, round(ONE / (73.3 * sqrt(K)))) for a matrix with K input
  columns (so W @ x keeps O(1) magnitudes: 73.3 is the std of the int8 values);
  the embedding uses s_base = 894 (~ONE / 73.3) so rows are O(1) in Q16;
* norm gamma = ONE + (r % 8193) - 4096.
* RoPE tables: the reference's compute_rope_tables
  (cached_integer_model.rs:1622-1635) with Rust's round-half-away-from-zero.
"""
from __future__ import annotations

import math
from typing import List, Optional

import numpy as np

from arc_chain_b200.models.config import ModelConfig
from arc_chain_b200.formats.arc_int8 import Int8Model, LAYER_MATS

ONE = 1 << 16
M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
GAMMA = 0x9E3779B97F4A7C15
EXT_BASE = 1 << 20
EMB_SCALE_BASE = 894


def _fin(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def _fin_int(z: int) -> int:
    m = (1 << 64) - 1
    z &= m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


def stream_key(seed: int, stream: int) -> int:
    return _fin_int((((seed << 32) ^ stream) + GAMMA) & ((1 << 64) - 1))


def rng_u64(seed: int, stream: int, n: int, start: int = 0) -> np.ndarray:
    key = np.uint64(stream_key(seed, stream))
    i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _fin(key + i * np.uint64(GAMMA))


def rng_i8(seed: int, stream: int, n: int) -> np.ndarray:
    """int8 weights in [-127, 127]; uses the C++ filler for big tensors."""
    if n >= (1 << 20):
        from arc_chain_b200.oracle import arcref

        out = np.empty(n, dtype=np.int8)
        arcref.rng_fill_i8(seed, stream, out)
        return out
    out = np.empty(n, dtype=np.int8)
    step = 1 << 22
    for s in range(0, n, step):
        r = rng_u64(seed, stream, min(step, n - s), start=s)
        out[s:s + len(r)] = ((r % np.uint64(255)).astype(np.int16) - 127).astype(np.int8)
    return out


def scale_base(k: int) -> int:
    return max(1, int(round(ONE / (73.3 * math.sqrt(k)))))


def row_scales(seed: int, stream: int, rows: int, base: int) -> np.ndarray:
    r = rng_u64(seed, stream, rows)
    return (np.int64(base) + (r % np.uint64(base // 8 + 1)).astype(np.int64)).astype(np.int64)


def gamma(seed: int, stream: int, n: int) -> np.ndarray:
    r = rng_u64(seed, stream, n)
    return (ONE + (r % np.uint64(8193)).astype(np.int64) - 4096).astype(np.int64)


def layer_tensor_id(layer: int, j: int) -> int:
    return 3 + 9 * layer + j


def ext_tensor_id(layer: int, slot: int) -> int:
    """MLA/MoE tensors: 64 slots per layer above EXT_BASE."""
    return EXT_BASE + layer * 4096 + slot


def rust_round(v: float) -> int:
    t = math.trunc(v)
    f = v - t
    if f >= 0.5:
        t += 1
    elif f <= -0.5:
        t -= 1
    return int(t)


def rope_tables(d_head: int, max_seq: int, base: float = 10000.0):
    half = d_head // 2
    cos = np.empty(max_seq * half, dtype=np.int64)
    sin = np.empty(max_seq * half, dtype=np.int64)
    freqs = [1.0 / base ** (2.0 * i / d_head) for i in range(half)]
    for pos in range(max_seq):
        for i, fq in enumerate(freqs):
            a = pos * fq
            cos[pos * half + i] = rust_round(math.cos(a) * ONE)
            sin[pos * half + i] = rust_round(math.sin(a) * ONE)
    return cos, sin


def matrix(seed: int, tid: int, rows: int, cols: int, base: Optional[int] = None):
    d = rng_i8(seed, tid << 2, rows * cols).reshape(rows, cols)
    s = row_scales(seed, (tid << 2) | 1, rows, scale_base(cols) if base is None else base)
    return d, s


def random_model(cfg: ModelConfig, seed: int = 0, vocab_strings: bool = True) -> Int8Model:
    """Dense MHA/GQA INT8 decoder with seeded weights (host numpy arrays)."""
    if cfg.is_mla or cfg.is_moe:
        from arc_chain_b200.models.mla_moe import random_mla_moe_model

        return random_mla_moe_model(cfg, seed)
    d = cfg.d_model
    emb, emb_s = matrix(seed, 0, cfg.vocab, d, base=EMB_SCALE_BASE)
    out, out_s = matrix(seed, 1, cfg.vocab, d)
    fn = gamma(seed, (2 << 2) | 1, d)
    rc, rs = rope_tables(cfg.d_head, cfg.max_seq, cfg.rope_theta)
    shapes = {"wq": (d, d), "wk": (cfg.d_kv, d), "wv": (cfg.d_kv, d), "wo": (d, d),
              "gate": (cfg.d_ff, d), "up": (cfg.d_ff, d), "down": (d, cfg.d_ff)}
    layers = []
    for l in range(cfg.n_layers):
        L = {}
        for j, n in enumerate(LAYER_MATS):
            L[n], L[n + "_s"] = matrix(seed, layer_tensor_id(l, j), *shapes[n])
        L["attn_norm"] = gamma(seed, (layer_tensor_id(l, 7) << 2) | 1, d)
        L["ffn_norm"] = gamma(seed, (layer_tensor_id(l, 8) << 2) | 1, d)
        layers.append(L)
    vocab = [f"tok_{i}" for i in range(cfg.vocab)] if vocab_strings else []
    return Int8Model(cfg, cfg.resolved_attn_scale(), rc, rs, emb, emb_s, out, out_s, fn, layers, vocab)


def seeded_prompt(n: int, vocab: int, seed: int) -> List[int]:
    """n token ids uniform in [0, vocab) from `seed` (prompt stream 0xFFFF0000)."""
    r = rng_u64(seed, 0xFFFF0000, n)
    return [int(x) for x in (r % np.uint64(vocab))]


def seeded_lengths(n: int, lo: int, hi: int, seed: int, stream: int) -> List[int]:
    """n integers uniform in [lo, hi] (request lengths for batching workloads)."""
    r = rng_u64(seed, stream, n)
    return [lo + int(x) for x in (r % np.uint64(hi - lo + 1))]
