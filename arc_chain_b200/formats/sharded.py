"""Tensor-parallel sharded checkpoints: one file per TP rank plus a JSON
manifest carrying the full model's weight hash (the attestation model hash)
and a BLAKE3 of every shard file.

A rank's file is an ARC-INT8 v3 container (formats/arc_int8.py) of that
rank's slices in the reference's tensor layout: q/k/v and gate/up by output
rows (whole heads / FFN units), W_o and W_down by input columns, the LM head
by its vocab range; embeddings, norms and RoPE tables are replicated.  The
slices are the ones ``dense.from_host`` cuts, so ``load_shard`` +
``from_host(..., presharded=True)`` uploads a rank without reading the
other ranks' weights.  The reference keeps one ARC-INT8 file per model
(cached_integer_model.rs:1560-1595); this container is this framework's
addition for TP deployments.
"""
from __future__ import annotations

import copy
import json
import os
from typing import Dict, Optional

import numpy as np

from arc_chain_b200.formats import arc_int8
from arc_chain_b200.formats.arc_int8 import Int8Model
from arc_chain_b200.utils.hashing import blake3

ROW_SPLIT = ("wq", "wk", "wv", "gate", "up")
COL_SPLIT = ("wo", "down")
MANIFEST = "manifest.json"


def _rows(a, r, n):
    k = a.shape[0] // n
    return np.ascontiguousarray(a[r * k:(r + 1) * k])


def _cols(a, r, n):
    k = a.shape[1] // n
    return np.ascontiguousarray(a[:, r * k:(r + 1) * k])


def vocab_range(V: int, rank: int, size: int):
    per = (V + size - 1) // size
    lo = min(V, rank * per)
    return lo, min(V, lo + per)


def shard_host(m: Int8Model, rank: int, size: int) -> Int8Model:
    """Rank `rank` of `size`: its slices, the configuration unchanged."""
    from arc_chain_b200.models.dense import check_tp

    check_tp(m.cfg, size)
    out = copy.copy(m)
    out.layers = []
    for L in m.layers:
        L2 = dict(L)
        for n in ROW_SPLIT:
            L2[n], L2[n + "_s"] = _rows(L[n], rank, size), _rows(L[n + "_s"], rank, size)
        for n in COL_SPLIT:
            L2[n] = _cols(L[n], rank, size)
        out.layers.append(L2)
    lo, hi = vocab_range(m.cfg.vocab, rank, size)
    out.out, out.out_s = np.ascontiguousarray(m.out[lo:hi]), np.ascontiguousarray(m.out_s[lo:hi])
    return out


def _file_hash(path: str) -> str:
    with open(path, "rb") as f:
        return blake3(f.read()).hex()


def save_sharded(m: Int8Model, outdir: str, tp: int, q4: Optional[str] = None) -> Dict:
    """Write tp shard files and the manifest; q4="row" stores the
    reference's per-row Q4 values (applied to whole rows before slicing)."""
    from arc_chain_b200.models.dense import q4_row_host
    from arc_chain_b200.runtime import attest

    os.makedirs(outdir, exist_ok=True)
    full = q4_row_host(m) if q4 == "row" else m
    files, hashes = [], []
    for r in range(tp):
        name = f"rank{r}.arc-int8v3"
        path = os.path.join(outdir, name)
        arc_int8.save_v3(shard_host(full, r, tp), path)
        files.append(name)
        hashes.append(_file_hash(path))
    man = {"format": "arc-int8-tp", "version": 1, "tp": tp, "q4": q4, "config": json.loads(m.cfg.to_json()),
           "model_id": attest.model_id_string(m.cfg), "weight_hash": m.weight_hash().hex(), "files": files,
           "file_blake3": hashes, "row_split": list(ROW_SPLIT), "col_split": list(COL_SPLIT)}
    with open(os.path.join(outdir, MANIFEST), "w") as f:
        json.dump(man, f, indent=1)
    return man


def load_manifest(outdir: str) -> Dict:
    with open(os.path.join(outdir, MANIFEST)) as f:
        man = json.load(f)
    if man.get("format") != "arc-int8-tp":
        raise ValueError(f"{outdir}: not a sharded ARC-INT8 checkpoint")
    return man


def load_shard(outdir: str, rank: int, verify: bool = True) -> Int8Model:
    man = load_manifest(outdir)
    if not 0 <= rank < man["tp"]:
        raise ValueError(f"rank {rank} outside tp={man['tp']}")
    path = os.path.join(outdir, man["files"][rank])
    if verify and _file_hash(path) != man["file_blake3"][rank]:
        raise ValueError(f"{path}: BLAKE3 does not match the manifest")
    return arc_int8.load(path)


def assemble(outdir: str) -> Int8Model:
    """The full model from all shards; its weight hash is checked against
    the manifest (for q4 checkpoints the hash is of the INT8 source)."""
    man = load_manifest(outdir)
    tp = man["tp"]
    parts = [load_shard(outdir, r) for r in range(tp)]
    out = copy.copy(parts[0])
    out.layers = []
    for li in range(out.cfg.n_layers):
        L = dict(parts[0].layers[li])
        for n in ROW_SPLIT:
            L[n] = np.concatenate([p.layers[li][n] for p in parts])
            L[n + "_s"] = np.concatenate([p.layers[li][n + "_s"] for p in parts])
        for n in COL_SPLIT:
            L[n] = np.concatenate([p.layers[li][n] for p in parts], axis=1)
        out.layers.append(L)
    out.out = np.concatenate([p.out for p in parts])
    out.out_s = np.concatenate([p.out_s for p in parts])
    if man.get("q4") is None and out.weight_hash().hex() != man["weight_hash"]:
        raise ValueError("assembled weights do not match the manifest's weight hash")
    return out
