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
the one that consumes the bytes exactly (the VM's when both do, as for a file
of only ReLU / Softmax layers); failing both, it applies the VM's
own rule (numbering 0..4, bytes after the last layer ignored).  It never
falls back to a mock.

Two executions are provided: :func:`forward_f32` restates the reference's f32
forward (inference.rs:282-381: left-to-right f32 sums folded from -0.0 as
Rust's float ``Sum`` does, NaN-ignoring max-subtracted softmax,
mean/variance LayerNorm, embedding lookup through Rust's saturating
float -> usize cast), and :class:`IntegerNet` quantises the model to the
integer engine's arithmetic (per-row INT8 Dense with Q16 bias, softmax_i64,
integer LayerNorm), which is deterministic across platforms.

:class:`NativeNet` runs both on the native library (``csrc/ref/neuralnet.cpp``,
which calls the C library's ``expf`` as Rust's ``f32::exp`` does on Linux);
:func:`run_request` is the VM engine's real compute path
(``InferenceEngine::run_real_inference``, inference.rs:676-723) on top of it.
The Python functions are an independent restatement used to test the native
one; their softmax computes exp in f64 and rounds, which can differ from
``expf`` in the last bit.
"""
from __future__ import annotations

import ctypes
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
        if n > len(data) - off:  # every layer takes at least its tag byte
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
    """Returns (layers, tag_base).  Raises if the bytes are a NeuralNet file
    under neither numbering."""
    for base in (0, 1):
        r = _parse_with(data, base)
        if r is not None and r[1] == len(data):
            return r[0], base
    r = _parse_with(data, 0)  # the VM's rule: trailing bytes ignored
    if r is not None:
        return r[0], 0
    raise ValueError("not a NeuralNet file under either tag numbering")


def write(layers: List[Layer], tag_base: int = 0) -> bytes:
    """NeuralNet::to_bytes (inference.rs:213-270): an empty Dense or Embedding
    has no first row, so its column count is written as 0."""
    out = [struct.pack("<I", len(layers))]
    for L in layers:
        t = NAMES.index(L.kind) + tag_base
        out.append(bytes([t]))
        if L.kind == "dense":
            r, c = L.W.shape
            out.append(struct.pack("<II", r, c if r else 0))
            out += [L.W.astype("<f4").tobytes(), L.b.astype("<f4").tobytes()]
        elif L.kind == "layernorm":
            out.append(struct.pack("<I", len(L.gamma)))
            out += [L.gamma.astype("<f4").tobytes(), L.beta.astype("<f4").tobytes(), struct.pack("<f", L.eps)]
        elif L.kind == "embedding":
            r, c = L.table.shape
            out.append(struct.pack("<II", r, c if r else 0))
            out.append(L.table.astype("<f4").tobytes())
    return b"".join(out)


def _fold(values) -> np.float32:
    """Left-to-right f32 sum from -0.0 (Rust's ``Sum`` for f32)."""
    s = np.float32(-0.0)
    for v in values:
        s = np.float32(s + v)
    return s


def _emb_dim(table: np.ndarray) -> int:
    return table.shape[1] if table.shape[0] else 0


def _index_f32(v) -> int:
    """Rust's saturating ``f32 as usize``: NaN and negatives give 0."""
    v = float(v)
    if not v >= 0.0:
        return 0
    return int(v) if v < 2.0 ** 64 else (1 << 64) - 1


def softmax_f32(a: np.ndarray) -> np.ndarray:
    """forward_softmax (inference.rs:318-336): NaN-ignoring max, exp, a
    left-to-right sum, uniform 1/n when the sum is 0.  exp is taken in f64
    and rounded to f32."""
    a = np.asarray(a, dtype=np.float32)
    if not len(a):
        return a.copy()
    m = np.float32(-np.inf)
    for v in a:
        if not np.isnan(v):
            m = max(m, v)
    with np.errstate(invalid="ignore"):
        e = np.exp((a - m).astype(np.float32).astype(np.float64)).astype(np.float32)
    s = _fold(e)
    if s == 0:
        return np.full(len(a), np.float32(1) / np.float32(len(a)), np.float32)
    return (e / s).astype(np.float32)


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
            a = softmax_f32(a)
        elif L.kind == "layernorm":
            n = np.float32(len(a))
            mean = np.float32(_fold(a) / n)
            d = (a - mean).astype(np.float32)
            vs = _fold((d * d).astype(np.float32))
            inv = np.float32(1) / np.sqrt(np.float32(vs / n) + np.float32(L.eps))
            g = np.ones(len(a), np.float32)
            bt = np.zeros(len(a), np.float32)
            k1, k2 = min(len(a), len(L.gamma)), min(len(a), len(L.beta))
            g[:k1], bt[:k2] = L.gamma[:k1], L.beta[:k2]
            a = (d * inv * g + bt).astype(np.float32)
        elif L.kind == "embedding":
            dim = _emb_dim(L.table)
            idx = [_index_f32(v) for v in a]
            rows = [L.table[i, :dim] if i < len(L.table) else np.zeros(dim, np.float32) for i in idx]
            a = np.concatenate(rows).astype(np.float32) if rows else np.zeros(0, np.float32)
    return a


class IntegerNet:
    """The same network in the integer engine's arithmetic (Q16 activations).

    Dense: per-row INT8 weights (I8Weights::quantize_f32) with the exact
    i8 x i64 linear, plus a Q16 bias (round(b * ONE), half away from zero);
    ReLU: max(0, x); Softmax: softmax_i64; LayerNorm: mean = sum / n
    (truncating), var = sum(((x - mean)^2) >> 16) / n, inv = isqrt(var + eps
    in Q16, at least 1), y = ((((x - mean) * inv) >> 16) * g >> 16) + b;
    Embedding: Q16 table rows, indexed by the integer part of the input with
    negatives taken as 0 (as the f32 path's saturating cast does).  Float ->
    Q16 conversions round half away from zero and saturate (NaN -> 0)."""

    def __init__(self, layers: List[Layer]):
        from arc_chain_b200.formats.quantize import quantize_f32

        self.ops = []
        q = lambda v: np.array([_q16(x) for x in np.asarray(v).reshape(-1)], np.int64)
        for L in layers:
            if L.kind == "dense":
                w, s = quantize_f32(L.W.reshape(-1), *L.W.shape)
                self.ops.append(("dense", w, s, q(L.b)))
            elif L.kind == "layernorm":
                self.ops.append(("layernorm", q(L.gamma), q(L.beta), max(1, _q16(np.float32(L.eps)))))
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
                if n == 0:
                    continue
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
                dim = _emb_dim(tab)
                a = np.concatenate([tab[i, :dim] if i < len(tab) else np.zeros(dim, np.int64)
                                    for i in np.maximum(a, 0) >> 16]) if len(a) else a
        return a


def _q16(x) -> int:
    """round(x * ONE) half away from zero, saturated to i64 (NaN -> 0)."""
    v = float(x) * ONE
    if v != v:
        return 0
    if v >= 2.0 ** 63:
        return (1 << 63) - 1
    if v <= -(2.0 ** 63):
        return -(1 << 63)
    from arc_chain_b200.formats.gen import rust_round

    return rust_round(v)


_KINDS = {n: i for i, n in enumerate(NAMES)}


class NativeNet:
    """A NeuralNet held by the native library: parse / serialise, the f32
    forward and the integer forward in C++."""

    def __init__(self, handle):
        from arc_chain_b200.oracle import arcref

        self._L = arcref.lib()
        self.h = handle

    @classmethod
    def from_bytes(cls, data: bytes) -> "NativeNet":
        from arc_chain_b200.oracle import arcref

        L = arcref.lib()
        err = ctypes.create_string_buffer(256)
        h = L.arcnn_parse(data, len(data), err, 256)
        if not h:
            raise ValueError(err.value.decode())
        return cls(h)

    @classmethod
    def from_layers(cls, layers: List[Layer]) -> "NativeNet":
        from arc_chain_b200.oracle import arcref

        L = arcref.lib()
        net = cls(L.arcnn_new())
        for ly in layers:
            a = b = None
            rows = cols = 0
            eps = 0.0
            if ly.kind == "dense":
                a, b = np.ascontiguousarray(ly.W, np.float32), np.ascontiguousarray(ly.b, np.float32)
                rows, cols = a.shape
            elif ly.kind == "layernorm":
                a, b = np.ascontiguousarray(ly.gamma, np.float32), np.ascontiguousarray(ly.beta, np.float32)
                rows, eps = len(a), ly.eps
            elif ly.kind == "embedding":
                a = np.ascontiguousarray(ly.table, np.float32)
                rows, cols = a.shape
            rc = L.arcnn_add_layer(net.h, _KINDS[ly.kind], rows, cols,
                                   None if a is None else a.ctypes.data,
                                   None if b is None else b.ctypes.data, eps)
            if rc != 0:
                raise ValueError(f"layer kind {ly.kind!r}")
        return net

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            self._L.arcnn_free(h)
            self.h = None

    @property
    def tag_base(self) -> int:
        return self._L.arcnn_tag_base(self.h)

    @property
    def input_size(self) -> int:
        return self._L.arcnn_input_size(self.h)

    @property
    def output_size(self) -> int:
        return self._L.arcnn_output_size(self.h)

    def layers(self) -> List[Layer]:
        out = []
        for i in range(self._L.arcnn_num_layers(self.h)):
            r, c, e = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_float()
            k = NAMES[self._L.arcnn_layer(self.h, i, ctypes.byref(r), ctypes.byref(c), ctypes.byref(e))]
            arr = []
            for which in (0, 1):
                n = self._L.arcnn_layer_data(self.h, i, which, None, 0)
                v = np.zeros(n, np.float32)
                self._L.arcnn_layer_data(self.h, i, which, v.ctypes.data, n)
                arr.append(v)
            if k == "dense":
                out.append(Layer(k, W=arr[0].reshape(r.value, c.value), b=arr[1]))
            elif k == "layernorm":
                out.append(Layer(k, gamma=arr[0], beta=arr[1], eps=float(e.value)))
            elif k == "embedding":
                out.append(Layer(k, table=arr[0].reshape(r.value, c.value)))
            else:
                out.append(Layer(k))
        return out

    def to_bytes(self, tag_base: Optional[int] = None) -> bytes:
        base = self.tag_base if tag_base is None else tag_base
        n = self._L.arcnn_serialize(self.h, base, None, 0)
        buf = ctypes.create_string_buffer(n)
        self._L.arcnn_serialize(self.h, base, buf, n)
        return buf.raw[:n]

    def forward_f32(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = self._L.arcnn_output_len(self.h, len(x))
        out = np.zeros(n, np.float32)
        self._L.arcnn_forward_f32(self.h, x.ctypes.data, len(x), out.ctypes.data, n)
        return out

    def forward_q16(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.int64)
        n = self._L.arcnn_output_len(self.h, len(x))
        out = np.zeros(n, np.int64)
        self._L.arcnn_forward_q16(self.h, x.ctypes.data, len(x), out.ctypes.data, n)
        return out

    def softmax(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(len(x), np.float32)
        self._L.arcnn_softmax_f32(x.ctypes.data, len(x), out.ctypes.data)
        return out


def _sat_u32(v: float) -> int:
    """Rust's saturating ``f32 as u32``."""
    if not v >= 0.0:
        return 0
    return int(v) if v < 4294967296.0 else 4294967295


def decode_text(output: np.ndarray) -> str:
    """decode_output (inference.rs:729-743): per value
    ((|v| * 100) as u32) % 128, raised by 32 below 32, as one ASCII char."""
    chars = []
    for v in np.asarray(output, dtype=np.float32):
        idx = _sat_u32(float(np.float32(abs(v) * np.float32(100.0)))) % 128
        chars.append(chr(idx + 32 if idx < 32 else idx))
    return "".join(chars)


@dataclass
class Response:
    output: object
    tokens_used: int
    compute_time_ms: int  # the reference's reported formula, tokens * 2 + 10 (not a measurement)
    cost: int


def run_request(net: NativeNet, kind: str, payload) -> Response:
    """The VM engine's real compute path (run_real_inference,
    inference.rs:676-723) over a native net.  ``kind`` is ``text`` (a str:
    each char's code point mod 256 as input), ``tokens`` (ints, output values
    cast to u32 with saturation), ``embedding`` (floats in, floats out) or
    ``image`` (bytes divided by 255 in f32; the output is classified by
    softmax as ``[("class_i", p), ...]``, or ``[("unknown", 1.0)]`` when it
    is empty).  Tokens used: the input length, 10 for an image."""
    if kind == "text":
        x = np.array([ord(c) % 256 for c in payload], np.float32)
        out, used = decode_text(net.forward_f32(x)), len(x)
    elif kind == "tokens":
        y = net.forward_f32(np.array([float(np.float32(t)) for t in payload], np.float32))
        out, used = [_sat_u32(float(v)) for v in y], len(payload)
    elif kind == "embedding":
        out, used = net.forward_f32(np.asarray(payload, np.float32)), len(payload)
    elif kind == "image":
        x = (np.frombuffer(bytes(payload), np.uint8).astype(np.float32) / np.float32(255.0)).astype(np.float32)
        y = net.forward_f32(x)
        out = [("class_%d" % i, float(p)) for i, p in enumerate(net.softmax(y))] if len(y) else [("unknown", 1.0)]
        used = 10
    else:
        raise ValueError(f"unknown input kind {kind!r}")
    return Response(out, used, used * 2 + 10, used * 5)
