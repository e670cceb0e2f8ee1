"""ARC-INT8 model files.

v2 is the reference's binary format, byte for byte
(``save_weights`` / ``load_cached_model_binary``,
crates/arc-inference/src/cached_integer_model.rs:1560-1595 and 1783-1864;
``I8Weights::write_to/read_from`` 1260-1292; ``write/read_i64_vec`` 1295-1311):

    b"ARC-INT8\\x02\\x00"
    u64 x 9   n_layers, d_model, n_heads, n_kv_heads, d_ff, d_head, d_kv, vocab, max_seq
    i64       attn_scale
    vec       rope_cos, rope_sin                 (vec = u64 len + LE i64 items)
    I8W       embedding, output                  (I8W = u64 rows, u64 cols,
    vec       final_norm                          i64 scale x rows, i8 data row-major)
    per layer I8W x 7 (wq wk wv wo gate up down), vec attn_norm, vec ffn_norm
    u64 len + vocab JSON (list of strings)

All little-endian.  The reader checks only the first 8 magic bytes, as the
reference does, so the minor byte is free.

v3 (``b"ARC-INT8\\x03\\x00"``) is this framework's extension for tensors the
reference has no slot for (MLA, MoE, Q4 group-32): the v2 header fields, then
a JSON manifest (u64 len + bytes) naming each tensor with dtype and shape,
then the raw tensors in manifest order, each 64-byte aligned.  A v2 reader
rejects nothing it understands: v3 files are only written for models that v2
cannot express.
"""
from __future__ import annotations

import io
import json
import os
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from arc_chain_b200.models.config import ModelConfig

MAGIC_V2 = b"ARC-INT8\x02\x00"
MAGIC_V3 = b"ARC-INT8\x03\x00"
LAYER_MATS = ("wq", "wk", "wv", "wo", "gate", "up", "down")


@dataclass
class Int8Model:
    """Host-side container of a dense INT8 decoder (numpy arrays)."""

    cfg: ModelConfig
    attn_scale: int
    rope_cos: np.ndarray
    rope_sin: np.ndarray
    emb: np.ndarray
    emb_s: np.ndarray
    out: np.ndarray
    out_s: np.ndarray
    final_norm: np.ndarray
    layers: List[Dict[str, np.ndarray]]
    vocab: List[str] = field(default_factory=list)
    extra: Dict[str, np.ndarray] = field(default_factory=dict)
    # Full-precision Q16 embedding [vocab, d] (models imported from GGUF keep
    # one; the ARC-INT8 file stores only emb / emb_s).
    emb_q16: Optional[np.ndarray] = None

    def matrices(self):
        """(name, data, scales) in weight-hash order (1598-1617)."""
        yield "embedding", self.emb, self.emb_s
        yield "output", self.out, self.out_s
        for li, L in enumerate(self.layers):
            for n in LAYER_MATS:
                yield f"layers.{li}.{n}", L[n], L[n + "_s"]

    def weight_hash(self) -> bytes:
        from arc_chain_b200.utils.hashing import Blake3

        h = Blake3()
        for _, d, s in self.matrices():
            h.update(np.ascontiguousarray(d).view(np.uint8))
            h.update(np.ascontiguousarray(s.astype("<i8")).view(np.uint8))
        return h.digest()


def _w_u64(f, v: int):
    f.write(struct.pack("<Q", int(v)))


def _w_vec(f, v: np.ndarray):
    v = np.ascontiguousarray(v, dtype="<i8")
    _w_u64(f, v.size)
    f.write(v.tobytes())


def _w_i8w(f, d: np.ndarray, s: np.ndarray):
    rows, cols = d.shape
    _w_u64(f, rows)
    _w_u64(f, cols)
    f.write(np.ascontiguousarray(s, dtype="<i8").tobytes())
    f.write(np.ascontiguousarray(d, dtype=np.int8).tobytes())


def save(model: Int8Model, path: str) -> None:
    """Write an ARC-INT8 v2 file (same bytes the reference's save_weights writes)."""
    c = model.cfg
    if c.is_mla or c.is_moe:
        raise ValueError("MLA/MoE models need the v3 container: use save_v3")
    with open(path, "wb") as f:
        f.write(MAGIC_V2)
        for v in (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.d_head, c.d_kv,
                  c.vocab, c.max_seq):
            _w_u64(f, v)
        f.write(struct.pack("<q", int(model.attn_scale)))
        _w_vec(f, model.rope_cos)
        _w_vec(f, model.rope_sin)
        _w_i8w(f, model.emb, model.emb_s)
        _w_i8w(f, model.out, model.out_s)
        _w_vec(f, model.final_norm)
        for L in model.layers:
            for n in LAYER_MATS:
                _w_i8w(f, L[n], L[n + "_s"])
            _w_vec(f, L["attn_norm"])
            _w_vec(f, L["ffn_norm"])
        vj = json.dumps(model.vocab, ensure_ascii=False, separators=(",", ":")).encode()
        _w_u64(f, len(vj))
        f.write(vj)


class _Buf:
    def __init__(self, mm):
        self.mm = mm
        self.off = 0

    def u64(self) -> int:
        if self.off + 8 > len(self.mm):
            raise ValueError("truncated ARC-INT8 file")
        v = int(np.frombuffer(self.mm, dtype="<u8", count=1, offset=self.off)[0])
        self.off += 8
        return v

    def i64(self) -> int:
        v = self.u64()
        return v - (1 << 64) if v >> 63 else v

    def arr(self, dtype, count, shape=None):
        nbytes = np.dtype(dtype).itemsize * count
        if self.off + nbytes > len(self.mm):
            raise ValueError("truncated ARC-INT8 file")
        a = np.frombuffer(self.mm, dtype=dtype, count=count, offset=self.off)
        self.off += nbytes
        return a.reshape(shape) if shape is not None else a

    def vec(self):
        n = self.u64()
        return self.arr("<i8", n).astype(np.int64)

    def i8w(self):
        rows, cols = self.u64(), self.u64()
        s = self.arr("<i8", rows).astype(np.int64)
        d = self.arr(np.int8, rows * cols, (rows, cols))
        return d, s


def load(path: str) -> Int8Model:
    """Read an ARC-INT8 v2 (or v3) file.  Matrix data is memory-mapped."""
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    if len(mm) < 10 or bytes(mm[:8]) != b"ARC-INT8":
        raise ValueError("Not an ARC-INT8 file")
    b = _Buf(mm)
    b.off = 10
    hdr = [b.u64() for _ in range(9)]
    n_layers, d_model, n_heads, n_kv_heads, d_ff, d_head, d_kv, vocab, max_seq = hdr
    attn_scale = b.i64()
    if bytes(mm[:10]) == MAGIC_V3:
        return _load_v3(b, hdr, attn_scale)
    cfg = ModelConfig(n_layers=n_layers, d_model=d_model, n_heads=n_heads, n_kv_heads=n_kv_heads,
                      d_ff=d_ff, d_head=d_head, vocab=vocab, max_seq=max_seq, attn_scale=attn_scale)
    if cfg.d_kv != d_kv:
        raise ValueError(f"d_kv {d_kv} != n_kv_heads*d_head {cfg.d_kv}")
    if n_heads < 1 or n_kv_heads < 1 or d_head < 2 or n_heads * d_head != d_model or vocab < 1:
        raise ValueError("inconsistent config (heads x d_head must equal d_model)")
    if n_layers > (len(mm) - b.off) // (7 * 16 + 2 * 8):  # each layer's headers alone
        raise ValueError("layer count exceeds the file")
    rope_cos, rope_sin = b.vec(), b.vec()
    emb, emb_s = b.i8w()
    out, out_s = b.i8w()
    final_norm = b.vec()
    layers = []
    for _ in range(n_layers):
        L = {}
        for n in LAYER_MATS:
            L[n], L[n + "_s"] = b.i8w()
        L["attn_norm"], L["ffn_norm"] = b.vec(), b.vec()
        layers.append(L)
    # the forward indexes every matrix with the config's dimensions
    want = {"embedding": (emb, (vocab, d_model)), "output": (out, (vocab, d_model))}
    shapes = {"wq": (d_model, d_model), "wk": (d_kv, d_model), "wv": (d_kv, d_model), "wo": (d_model, d_model),
              "gate": (d_ff, d_model), "up": (d_ff, d_model), "down": (d_model, d_ff)}
    for li, L in enumerate(layers):
        for n, shp in shapes.items():
            want[f"layers.{li}.{n}"] = (L[n], shp)
    for name, (a, shp) in want.items():
        if tuple(a.shape) != shp:
            raise ValueError(f"{name} is {a.shape[0]} x {a.shape[1]}, the config needs {shp[0]} x {shp[1]}")
    vlen = b.u64()
    try:
        vocab_list = json.loads(bytes(b.arr(np.uint8, vlen)).decode())
    except Exception:  # the reference falls back to an empty vocab
        vocab_list = []
    return Int8Model(cfg, attn_scale, rope_cos, rope_sin, emb, emb_s, out, out_s, final_norm,
                     layers, vocab_list)


# ---------------------------------------------------------------------------
# v3 container (MLA / MoE / Q4 group-32 tensors)
# ---------------------------------------------------------------------------
def save_v3(model: Int8Model, path: str) -> None:
    c = model.cfg
    tensors: Dict[str, np.ndarray] = {
        "rope_cos": model.rope_cos, "rope_sin": model.rope_sin,
        "embedding": model.emb, "embedding_s": model.emb_s,
        "output": model.out, "output_s": model.out_s, "final_norm": model.final_norm,
    }
    for li, L in enumerate(model.layers):
        for k, v in L.items():
            tensors[f"layers.{li}.{k}"] = v
    tensors.update(model.extra)
    manifest = {"config": json.loads(c.to_json()), "attn_scale": int(model.attn_scale),
                "vocab": model.vocab, "tensors": []}
    off = 0
    for k, v in tensors.items():
        v = np.ascontiguousarray(v)
        manifest["tensors"].append({"name": k, "dtype": v.dtype.str, "shape": list(v.shape),
                                    "offset": off})
        off += (v.nbytes + 63) // 64 * 64
    mj = json.dumps(manifest).encode()
    with open(path, "wb") as f:
        f.write(MAGIC_V3)
        for v in (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.d_head, c.d_kv,
                  c.vocab, c.max_seq):
            _w_u64(f, v)
        f.write(struct.pack("<q", int(model.attn_scale)))
        _w_u64(f, len(mj))
        f.write(mj)
        pad = (-f.tell()) % 64
        f.write(b"\0" * pad)
        for k, v in tensors.items():
            v = np.ascontiguousarray(v)
            f.write(v.tobytes())
            f.write(b"\0" * ((-v.nbytes) % 64))


def _load_v3(b: _Buf, hdr, attn_scale) -> Int8Model:
    mlen = b.u64()
    manifest = json.loads(bytes(b.arr(np.uint8, mlen)).decode())
    b.off += (-b.off) % 64
    base = b.off
    t = {}
    for e in manifest["tensors"]:
        dt = np.dtype(e["dtype"])
        cnt = int(np.prod(e["shape"])) if e["shape"] else 1
        t[e["name"]] = np.frombuffer(b.mm, dtype=dt, count=cnt, offset=base + e["offset"]).reshape(e["shape"])
    cfg = ModelConfig(**manifest["config"])
    layers = []
    for li in range(cfg.n_layers):
        pre = f"layers.{li}."
        layers.append({k[len(pre):]: v for k, v in t.items() if k.startswith(pre)})
    known = {"rope_cos", "rope_sin", "embedding", "embedding_s", "output", "output_s", "final_norm"}
    extra = {k: v for k, v in t.items() if k not in known and not k.startswith("layers.")}
    return Int8Model(cfg, manifest["attn_scale"], t["rope_cos"].astype(np.int64),
                     t["rope_sin"].astype(np.int64), t["embedding"], t["embedding_s"].astype(np.int64),
                     t["output"], t["output_s"].astype(np.int64), t["final_norm"].astype(np.int64),
                     layers, manifest.get("vocab", []), extra)
