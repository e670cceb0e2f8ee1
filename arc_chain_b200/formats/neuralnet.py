"""The reference's tagged f32 MLP format ("NeuralNet") and the files
scripts/create_model.py writes.

Layout (little-endian): u32 n_layers, then per layer a u8 tag and payload:
  Dense      u32 rows, u32 cols, f32 W[rows*cols] row-major, f32 bias[rows]
  ReLU / Softmax   (no payload)
  LayerNorm  u32 n, f32 gamma[n], f32 beta[n], f32 eps
  Embedding  u32 vocab, u32 dim, f32 table[vocab*dim]
The VM's reader numbers the tags 0..4 (Dense, ReLU, Softmax, LayerNorm,
Embedding; crates/arc-vm/src/inference.rs:51-55, 132-211) while
create_model.py writes 1..5 (scripts/create_model.py:30-61), and the VM
silently falls back to a mock when parsing fails (inference.rs:566-573).
:func:`parse` accepts both: it parses the file under each numbering and keeps
the one that consumes the bytes exactly (never a mock).

Two executions are provided: :func:`forward_f32` restates the reference's f32
forward (inference.rs:282-381: left-to-right f32 sums, max-subtracted
softmax, mean/variance LayerNorm, embedding lookup), and
:class:`IntegerNet` quantises the model to the integer engine's arithmetic
(per-row INT8 Dense with Q16 bias, softmax_i64, integer LayerNorm), which is
deterministic across platforms.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import List, Optional, Tuple

import numpy as np

from arc_chain_b200 import spec

NAMES = ("dense", "relu", "softmax", "layernorm", "embedding")
ONE = spec.ONE


@dataclass
class Layer:
    kind: str
    W: Optional[np.ndarray] = None
    b: Optional[np.ndarray] = None
    gamma: Optional[np.ndarray] = None
    beta: Optional[np.ndarray] = None
    eps: float = 1e-5
    table: Optional[np.ndarray] = None


def _parse_with(data: bytes, base: int) -> Optional[Tuple[List[Layer], int]]:
    off = 0

    def u32():
        nonlocal off
        if off + 4 > len(data):
            raise ValueError("truncated")
        v = struct.unpack_from("<I", data, off)[0]
        off += 4
        return v

    def f32(n):
        nonlocal off
        if off + 4 * n > len(data):
            raise ValueError("truncated")
        a = np.frombuffer(data, dtype="<f4", count=n, offset=off).astype(np.float32)
        off += 4 * n
        return a

    try:
        n = u32()
        if n > 1 << 20:
            return None
        layers = []
        for _ in range(n):
            if off >= len(data):
                return None
            tag = data[off] - base
            off += 1
            if tag == 0:
                r, c = u32(), u32()
                W = f32(r * c).reshape(r, c)
                layers.append(Layer("dense", W=W, b=f32(r)))
            elif tag == 1:
                layers.append(Layer("relu"))
            elif tag == 2:
                layers.append(Layer("softmax"))
            elif tag == 3:
                k = u32()
                g, bt = f32(k), f32(k)
                layers.append(Layer("layernorm", gamma=g, beta=bt, eps=float(f32(1)[0])))
            elif tag == 4:
                v, dim = u32(), u32()
                layers.append(Layer("embedding", table=f32(v * dim).reshape(v, dim)))
            else:
                return None
        return layers, off
    except ValueError:
        return None


def parse(data: bytes) -> Tuple[List[Layer], int]:
    """Returns (layers, tag_base).  Raises if neither numbering fits exactly."""
    for base in (0, 1):
        r = _parse_with(data, base)
        if r is not None and r[1] == len(data):
            return r[0], base
    raise ValueError("not a NeuralNet file under either tag numbering")


def write(layers: List[Layer], tag_base: int = 0) -> bytes:
    out = [struct.pack("<I", len(layers))]
    for L in layers:
        t = NAMES.index(L.kind) + tag_base
        out.append(bytes([t]))
        if L.kind == "dense":
            out.append(struct.pack("<II", *L.W.shape))
            out += [L.W.astype("<f4").tobytes(), L.b.astype("<f4").tobytes()]
        elif L.kind == "layernorm":
            out.append(struct.pack("<I", len(L.gamma)))
            out += [L.gamma.astype("<f4").tobytes(), L.beta.astype("<f4").tobytes(), struct.pack("<f", L.eps)]
        elif L.kind == "embedding":
            out.append(struct.pack("<II", *L.table.shape))
            out.append(L.table.astype("<f4").tobytes())
    return b"".join(out)


def forward_f32(layers: List[Layer], x: np.ndarray) -> np.ndarray:
    a = np.asarray(x, dtype=np.float32)
    for L in layers:
        if L.kind == "dense":
            acc = L.b.astype(np.float32).copy()
            k = min(L.W.shape[1], len(a))
            for j in range(k):  # strictly left-to-right per output, as the reference
                acc = (acc + L.W[:, j] * a[j]).astype(np.float32)
            a = acc
        elif L.kind == "relu":
            a = np.where(a > 0, a, np.float32(0)).astype(np.float32)
        elif L.kind == "softmax":
            if len(a):
                e = np.exp((a - a.max()).astype(np.float32)).astype(np.float32)
                s = np.float32(0)
                for v in e:
                    s = np.float32(s + v)
                a = (e / s).astype(np.float32) if s != 0 else np.full(len(a), np.float32(1) / len(a), np.float32)
        elif L.kind == "layernorm":
            n = np.float32(len(a))
            s = np.float32(0)
            for v in a:
                s = np.float32(s + v)
            mean = np.float32(s / n)
            d = (a - mean).astype(np.float32)
            vs = np.float32(0)
            for v in d * d:
                vs = np.float32(vs + v)
            inv = np.float32(1) / np.sqrt(np.float32(vs / n) + np.float32(L.eps))
            g = np.ones(len(a), np.float32)
            bt = np.zeros(len(a), np.float32)
            k1, k2 = min(len(a), len(L.gamma)), min(len(a), len(L.beta))
            g[:k1], bt[:k2] = L.gamma[:k1], L.beta[:k2]
            a = (d * inv * g + bt).astype(np.float32)
        elif L.kind == "embedding":
            dim = L.table.shape[1]
            rows = [L.table[int(i)] if 0 <= int(i) < len(L.table) else np.zeros(dim, np.float32) for i in a]
            a = np.concatenate(rows).astype(np.float32) if rows else np.zeros(0, np.float32)
    return a


class IntegerNet:
    """The same network in the integer engine's arithmetic (Q16 activations).

    Dense: per-row INT8 weights (I8Weights::quantize_f32) with the exact
    i8 x i64 linear, plus a Q16 bias (round(b * ONE), half away from zero);
    ReLU: max(0, x); Softmax: softmax_i64; LayerNorm: mean = sum / n
    (truncating), var = sum(((x - mean)^2) >> 16) / n, inv = isqrt(var + eps
    in Q16, at least 1), y = ((((x - mean) * inv) >> 16) * g >> 16) + b;
    Embedding: Q16 table rows."""

    def __init__(self, layers: List[Layer]):
        from arc_chain_b200.formats.quantize import quantize_f32
        from arc_chain_b200.formats.gen import rust_round

        self.ops = []
        q = lambda v: np.array([rust_round(float(x) * ONE) for x in np.asarray(v).reshape(-1)], np.int64)
        for L in layers:
            if L.kind == "dense":
                w, s = quantize_f32(L.W.reshape(-1), *L.W.shape)
                self.ops.append(("dense", w, s, q(L.b)))
            elif L.kind == "layernorm":
                self.ops.append(("layernorm", q(L.gamma), q(L.beta), max(1, rust_round(L.eps * ONE))))
            elif L.kind == "embedding":
                self.ops.append(("embedding", q(L.table).reshape(L.table.shape)))
            else:
                self.ops.append((L.kind,))

    def forward(self, x) -> np.ndarray:
        a = np.asarray(x, dtype=np.int64)
        for op in self.ops:
            k = op[0]
            if k == "dense":
                w, s, b = op[1:]
                a = spec.linear_i8(w[:, :len(a)], s, a[:w.shape[1]]) + b
            elif k == "relu":
                a = np.maximum(a, 0)
            elif k == "softmax":
                a = spec.softmax(a)
            elif k == "layernorm":
                g, bt, eps = op[1:]
                n = len(a)
                mean = spec.tdiv(int(a.sum()), n)
                d = a - mean
                var = spec.tdiv(int(((d * d) >> 16).sum()), n)
                inv = spec.integer_isqrt(max(1, var + eps))
                gg = np.full(n, ONE, np.int64)
                bb = np.zeros(n, np.int64)
                gg[:min(n, len(g))] = g[:n]
                bb[:min(n, len(bt))] = bt[:n]
                a = ((((d * inv) >> 16) * gg) >> 16) + bb
            elif k == "embedding":
                tab = op[1]
                dim = tab.shape[1]
                a = np.concatenate([tab[i] if 0 <= i < len(tab) else np.zeros(dim, np.int64)
                                    for i in (a >> 16).tolist()]) if len(a) else a
        return a
