"""GGUF import: llama-architecture GGUF files -> the per-row INT8 model the
integer engine runs, with the reference loader's semantics
(crates/arc-inference/src/cached_integer_model.rs:1638-1775,
``load_cached_model``):

* config from ``llama.block_count / embedding_length / attention.head_count /
  attention.head_count_kv (0 -> head_count) / feed_forward_length``; vocab
  size = rows of ``token_embd.weight``; vocabulary strings from
  ``tokenizer.ggml.tokens``;
* every matrix dequantised to f32 and quantised per row with the INT8
  quantiser (``formats.quantize.quantize_f32``, reference quirk kept);
  ``output.weight`` missing -> the embedding's INT8 copy;
* norms: round(x * ONE) computed in f32 (missing -> ONE);
* the embedding is also kept at full precision, round(x * ONE) in f64, and
  that table (not i8 * scale) feeds the forward;
* max_seq = 2048, RoPE tables of d_head at theta 10000,
  attn_scale = integer_isqrt(d_head * ONE).

The container reader (header, typed metadata, tensor infos, aligned data)
and the dequantisers of F32, F16, BF16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K,
Q5_K and Q6_K are written here from the GGUF / GGML block layouts; other
block types are dequantised by the ``gguf`` package when it is installed.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Dict, Tuple

import numpy as np

from arc_chain_b200 import spec
from arc_chain_b200.formats import gen
from arc_chain_b200.formats.arc_int8 import Int8Model
from arc_chain_b200.formats.quantize import quantize_f32
from arc_chain_b200.models.config import ModelConfig

ONE = spec.ONE

# metadata value types
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
STRING, ARRAY = 8, 9

# ggml tensor types: (name, block elements, block bytes)
TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22),
         7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36), 10: ("Q2_K", 256, 84),
         11: ("Q3_K", 256, 110), 12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210),
         15: ("Q8_K", 256, 292), 30: ("BF16", 1, 2)}


@dataclass
class TensorInfo:
    name: str
    shape: Tuple[int, ...]  # numpy order (outermost first): GGUF dims reversed
    type: int
    offset: int             # relative to the data section

    @property
    def n(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @property
    def nbytes(self) -> int:
        _, be, bb = TYPES[self.type]
        return self.n // be * bb


class GGUFFile:
    """Reads the header, metadata and tensor table; tensors on demand."""

    def __init__(self, path: str):
        self.path = path
        self.buf = np.memmap(path, dtype=np.uint8, mode="r")
        self.pos = 0
        magic = bytes(self.buf[:4])
        if magic != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        self.pos = 4
        self.version = self._u("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} not supported")
        n_tensors, n_kv = self._u("<Q"), self._u("<Q")
        self.metadata: Dict[str, object] = {}
        for _ in range(n_kv):
            k = self._str()
            self.metadata[k] = self._value(self._u("<I"))
        self.tensors: Dict[str, TensorInfo] = {}
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u("<I")
            dims = [self._u("<Q") for _ in range(nd)]
            t = self._u("<I")
            off = self._u("<Q")
            self.tensors[name] = TensorInfo(name, tuple(reversed(dims)), t, off)
        align = int(self.metadata.get("general.alignment", 32))
        self.data_start = (self.pos + align - 1) // align * align

    def _u(self, fmt):
        n = struct.calcsize(fmt)
        v = struct.unpack(fmt, bytes(self.buf[self.pos:self.pos + n]))[0]
        self.pos += n
        return v

    def _str(self) -> str:
        n = self._u("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def _value(self, t):
        if t in _SCALARS:
            return self._u(_SCALARS[t])
        if t == STRING:
            return self._str()
        if t == ARRAY:
            et, n = self._u("<I"), self._u("<Q")
            if et in _SCALARS and et != 7:
                dt = np.dtype(_SCALARS[et])
                a = np.frombuffer(bytes(self.buf[self.pos:self.pos + n * dt.itemsize]), dtype=dt)
                self.pos += n * dt.itemsize
                return a.tolist()
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {t}")

    def raw(self, name: str) -> np.ndarray:
        ti = self.tensors[name]
        o = self.data_start + ti.offset
        return np.asarray(self.buf[o:o + ti.nbytes])

    def f32(self, name: str) -> np.ndarray:
        """Dequantised tensor as float32 in numpy shape order."""
        ti = self.tensors[name]
        return dequantize(self.raw(name), ti.type, ti.n).reshape(ti.shape)


# ---------------------------------------------------------------- dequantisation
def _f16(b: np.ndarray) -> np.ndarray:
    return b.view(np.float16).astype(np.float32)


def _f16col(b: np.ndarray) -> np.ndarray:
    """A 2-byte f16 field of every block as a [blocks, 1] float32 column."""
    return np.ascontiguousarray(b).view(np.float16).astype(np.float32).reshape(-1, 1)


def _blocks(raw: np.ndarray, bb: int) -> np.ndarray:
    return np.ascontiguousarray(raw).reshape(-1, bb)


def _scale_min_k4(sc: np.ndarray):
    """6-bit scales and mins of the 8 sub-blocks from the 12 packed bytes."""
    q = sc.astype(np.uint8)
    s = np.empty((q.shape[0], 8), np.uint8)
    m = np.empty((q.shape[0], 8), np.uint8)
    for j in range(8):
        if j < 4:
            s[:, j] = q[:, j] & 63
            m[:, j] = q[:, j + 4] & 63
        else:
            s[:, j] = (q[:, j + 4] & 0xF) | ((q[:, j - 4] >> 6) << 4)
            m[:, j] = (q[:, j + 4] >> 4) | ((q[:, j] >> 6) << 4)
    return s.astype(np.float32), m.astype(np.float32)


def dequantize(raw: np.ndarray, t: int, n: int) -> np.ndarray:
    name, be, bb = TYPES.get(t, (None, 0, 0))
    raw = np.ascontiguousarray(raw)
    if name == "F32":
        return raw.view(np.float32)[:n].copy()
    if name == "F16":
        return _f16(raw)[:n]
    if name == "BF16":
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)[:n]
    if name in ("Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0"):
        B = _blocks(raw, bb)
        d = _f16col(B[:, 0:2])
        if name == "Q8_0":
            return (d * B[:, 2:34].view(np.int8).astype(np.float32)).reshape(-1)[:n]
        off = 4 if name in ("Q4_1", "Q5_1") else 2
        mn = _f16col(B[:, 2:4]) if off == 4 else None
        if name.startswith("Q5"):
            qh = B[:, off:off + 4].copy().view(np.uint32)[:, 0]
            qs = B[:, off + 4:off + 20]
        else:
            qs = B[:, off:off + 16]
        lo, hi = (qs & 0xF).astype(np.int32), (qs >> 4).astype(np.int32)
        q = np.concatenate([lo, hi], axis=1)
        if name.startswith("Q5"):
            bits = ((qh[:, None] >> np.arange(32, dtype=np.uint32)[None, :]) & 1).astype(np.int32)
            q = q | (bits << 4)
        if name == "Q4_0":
            return (d * (q - 8).astype(np.float32)).reshape(-1)[:n]
        if name == "Q5_0":
            return (d * (q - 16).astype(np.float32)).reshape(-1)[:n]
        return (d * q.astype(np.float32) + mn).reshape(-1)[:n]
    if name in ("Q4_K", "Q5_K"):
        B = _blocks(raw, bb)
        d = _f16col(B[:, 0:2])
        dmin = _f16col(B[:, 2:4])
        s, m = _scale_min_k4(B[:, 4:16])
        if name == "Q4_K":
            qs = B[:, 16:144]
        else:
            qh = B[:, 16:48]
            qs = B[:, 48:176]
        out = np.empty((B.shape[0], 256), np.float32)
        for c in range(4):
            q = qs[:, 32 * c:32 * c + 32]
            lo, hi = (q & 0xF).astype(np.float32), (q >> 4).astype(np.float32)
            if name == "Q5_K":
                lo = lo + ((qh >> (2 * c)) & 1).astype(np.float32) * 16
                hi = hi + ((qh >> (2 * c + 1)) & 1).astype(np.float32) * 16
            d1, m1 = d * s[:, 2 * c:2 * c + 1], dmin * m[:, 2 * c:2 * c + 1]
            d2, m2 = d * s[:, 2 * c + 1:2 * c + 2], dmin * m[:, 2 * c + 1:2 * c + 2]
            out[:, 64 * c:64 * c + 32] = d1 * lo - m1
            out[:, 64 * c + 32:64 * c + 64] = d2 * hi - m2
        return out.reshape(-1)[:n]
    if name == "Q6_K":
        B = _blocks(raw, bb)
        ql, qh = B[:, 0:128], B[:, 128:192]
        sc = B[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16col(B[:, 208:210])
        out = np.empty((B.shape[0], 256), np.float32)
        for half in range(2):
            L, H, S = ql[:, 64 * half:64 * half + 64], qh[:, 32 * half:32 * half + 32], sc[:, 8 * half:8 * half + 8]
            a, b = L[:, :32].astype(np.int32), L[:, 32:].astype(np.int32)
            h = H.astype(np.int32)
            q1 = ((a & 0xF) | (((h >> 0) & 3) << 4)) - 32
            q2 = ((b & 0xF) | (((h >> 2) & 3) << 4)) - 32
            q3 = ((a >> 4) | (((h >> 4) & 3) << 4)) - 32
            q4 = ((b >> 4) | (((h >> 6) & 3) << 4)) - 32
            base = 128 * half
            for k, qq in enumerate((q1, q2, q3, q4)):
                for l0 in (0, 16):
                    s_ = S[:, (l0 // 16) + 2 * k][:, None]
                    out[:, base + 32 * k + l0:base + 32 * k + l0 + 16] = (d * s_) * qq[:, l0:l0 + 16].astype(np.float32)
        return out.reshape(-1)[:n]
    try:
        import gguf as _g

        return np.asarray(_g.quants.dequantize(raw, _g.GGMLQuantizationType(t)), dtype=np.float32).reshape(-1)[:n]
    except Exception as e:  # noqa: BLE001
        raise ValueError(f"GGUF tensor type {t} not supported: {e}")


# ---------------------------------------------------------------- import
def _round_half_away(v: np.ndarray) -> np.ndarray:
    """Rust's ``x.round() as i64``: half away from zero, then a saturating
    cast (NaN -> 0, out of range -> i64::MIN / i64::MAX).  Inputs come from
    f32 values, so ``|v| + 0.5`` is exact in f64."""
    v = np.asarray(v, dtype=np.float64)
    with np.errstate(invalid="ignore"):
        r = np.sign(v) * np.floor(np.abs(v) + 0.5)
    out = np.zeros(r.shape, dtype=np.int64)
    hi, lo = r >= 2.0 ** 63, r <= -(2.0 ** 63)
    mid = ~(hi | lo | np.isnan(r))
    out[mid] = r[mid].astype(np.int64)
    out[hi], out[lo] = np.iinfo(np.int64).max, np.iinfo(np.int64).min
    return out


def norm_q16(x: np.ndarray) -> np.ndarray:
    """(x * ONE as f32).round() as i64."""
    return _round_half_away(np.asarray(x, np.float32) * np.float32(ONE))


def load_gguf(path: str, max_seq: int = 2048) -> Int8Model:
    g = GGUFFile(path)
    md = g.metadata

    def u32(k):
        v = md.get(k, 0)
        return int(v) & 0xFFFFFFFF if isinstance(v, (int, np.integer)) else 0

    nl, dm, nh = u32("llama.block_count"), u32("llama.embedding_length"), u32("llama.attention.head_count")
    nkv = u32("llama.attention.head_count_kv") or nh
    dff = u32("llama.feed_forward_length")
    emb_t = g.tensors.get("token_embd.weight")
    V = emb_t.shape[0] if emb_t is not None else 32000
    toks = md.get("tokenizer.ggml.tokens", [])
    vocab = [t for t in toks if isinstance(t, str)] if isinstance(toks, list) else []
    dh = dm // nh
    cfg = ModelConfig(n_layers=nl, d_model=dm, n_heads=nh, n_kv_heads=nkv, d_ff=dff, d_head=dh, vocab=V,
                      max_seq=max_seq, name="gguf")

    def i8(name, rows, cols):
        return quantize_f32(g.f32(name), rows, cols)

    def nrm(name, size):
        return norm_q16(g.f32(name).reshape(-1)) if name in g.tensors else np.full(size, ONE, np.int64)

    emb_f = g.f32("token_embd.weight").reshape(V, dm)
    emb, emb_s = quantize_f32(emb_f, V, dm)
    emb_q16 = _round_half_away(emb_f.astype(np.float64) * float(ONE))
    if "output.weight" in g.tensors:
        out, out_s = i8("output.weight", V, dm)
    else:
        out, out_s = emb.copy(), emb_s.copy()
    dkv = dh * nkv
    layers = []
    for l in range(nl):
        p = f"blk.{l}"
        L = {}
        for n, t, r, c in (("wq", "attn_q", dm, dm), ("wk", "attn_k", dkv, dm), ("wv", "attn_v", dkv, dm),
                           ("wo", "attn_output", dm, dm), ("gate", "ffn_gate", dff, dm), ("up", "ffn_up", dff, dm),
                           ("down", "ffn_down", dm, dff)):
            L[n], L[n + "_s"] = i8(f"{p}.{t}.weight", r, c)
        L["attn_norm"] = nrm(f"{p}.attn_norm.weight", dm)
        L["ffn_norm"] = nrm(f"{p}.ffn_norm.weight", dm)
        layers.append(L)
    rc, rs = gen.rope_tables(dh, max_seq, 10000.0)
    attn_scale = spec.integer_isqrt(dh * ONE)
    m = Int8Model(cfg, attn_scale, rc, rs, emb, emb_s, out, out_s, nrm("output_norm.weight", dm), layers, vocab)
    m.emb_q16 = emb_q16
    return m
