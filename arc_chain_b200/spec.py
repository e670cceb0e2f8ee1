"""Integer semantics of the engine, restated independently in numpy int64.

This module is the second, independent restatement of the reference CPU
engine (the first is the C++ oracle ``csrc/ref/arcref.cpp``).  Tests require
the two to agree byte-for-byte.  Sources of truth in the reference:

* ``crates/arc-inference/src/integer_lut.rs:7-147`` — FRAC_BITS, ONE, the exp
  LUT built by recurrence, integer_exp, softmax_i64, argmax_i64, integer_isqrt.
* ``crates/arc-inference/src/cached_integer_model.rs`` — per-row INT8 linear
  (221-262), Q4 (670-701, 955-978), RMSNorm (985-1000), RoPE (1002-1012),
  SiLU (1016-1027), forward_one_token (1381-1516), generate (1518-1557).

All i64 arithmetic wraps modulo 2^64 (the reference is built without
overflow checks).  numpy int64 array arithmetic wraps the same way; Python
ints are wrapped explicitly with :func:`wrap`.  ``/`` truncates toward zero
(:func:`tdiv`), ``>>`` is arithmetic.

The MLA, MoE, Q4 group-32 and batching semantics that the reference lacks are
defined at the end of this module (``mla_*``, ``moe_*``, ``q4g_*``).
"""
from __future__ import annotations

import numpy as np

FRAC_BITS = 16
ONE = 1 << FRAC_BITS
EXP_RANGE = 8 * ONE
EXP_STEP = ONE // 32
EXP_DECAY = 63521
MASK64 = (1 << 64) - 1


def wrap(x: int) -> int:
    """Python int -> i64 two's-complement value."""
    x &= MASK64
    return x - (1 << 64) if x >> 63 else x


def tdiv(a: int, b: int) -> int:
    """Truncating integer division (Rust/C semantics)."""
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def tdiv_np(a: np.ndarray, b) -> np.ndarray:
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    q = np.abs(a) // np.abs(b)
    return np.where((a >= 0) == (b >= 0), q, -q).astype(np.int64)


def build_exp_lut() -> np.ndarray:
    t = [0] * 257
    t[256] = ONE
    for i in range(255, -1, -1):
        t[i] = (t[i + 1] * EXP_DECAY) >> FRAC_BITS
    return np.array(t, dtype=np.int64)


EXP_LUT = build_exp_lut()
_LUT = [int(v) for v in EXP_LUT]


def integer_exp(x: int) -> int:
    if x >= 0:
        return ONE
    if x <= -EXP_RANGE:
        return 0
    off = x + EXP_RANGE
    idx, frac = off // EXP_STEP, off % EXP_STEP  # off > 0: floor == trunc
    if idx >= 256:
        return ONE
    lo, hi = _LUT[idx], _LUT[idx + 1]
    return lo + tdiv((hi - lo) * frac, EXP_STEP)


def integer_exp_np(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.int64)
    off = np.clip(x + EXP_RANGE, 0, EXP_RANGE)
    idx = off // EXP_STEP
    frac = off % EXP_STEP
    idc = np.minimum(idx, 255)
    lo, hi = EXP_LUT[idc], EXP_LUT[idc + 1]
    val = lo + tdiv_np((hi - lo) * frac, EXP_STEP)
    val = np.where(idx >= 256, ONE, val)
    val = np.where(x <= -EXP_RANGE, 0, val)
    return np.where(x >= 0, ONE, val).astype(np.int64)


def integer_isqrt(x: int) -> int:
    if x <= 0:
        return ONE * 100
    bits = x.bit_length() - 1
    y = tdiv(ONE * 256, 1 << ((bits + 1) // 2))
    if y <= 0:
        y = 1
    for _ in range(3):
        y2 = wrap(y * y) >> FRAC_BITS
        xy2 = wrap(x * y2) >> FRAC_BITS
        tm = wrap(3 * ONE - xy2)
        y = tdiv(wrap(y * tm), 2 * ONE)
        if y <= 0:
            y = 1
    return y


def silu(x: int) -> int:
    if x >= 0:
        e = integer_exp(-x)
        sig = tdiv(ONE * ONE, max(ONE + e, 1))
    else:
        e = integer_exp(x)
        sig = tdiv(e * ONE, max(ONE + e, 1))
    return wrap(x * sig) >> FRAC_BITS


def silu_np(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.int64)
    with np.errstate(over="ignore"):
        neg = -x
    e_pos = integer_exp_np(np.where(x >= 0, neg, 0))
    e_neg = integer_exp_np(np.where(x < 0, x, 0))
    sig_pos = tdiv_np(np.full_like(x, ONE * ONE), np.maximum(ONE + e_pos, 1))
    sig_neg = tdiv_np(e_neg * ONE, np.maximum(ONE + e_neg, 1))
    sig = np.where(x >= 0, sig_pos, sig_neg)
    return (x * sig) >> FRAC_BITS


def softmax(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.int64)
    n = len(v)
    if n == 0:
        return v.copy()
    if n == 1:
        return np.array([ONE], dtype=np.int64)
    m = v.max()
    e = integer_exp_np(v - m)
    s = int(e.sum(dtype=np.int64))
    if s == 0:
        return np.full(n, ONE // n, dtype=np.int64)
    return tdiv_np(e * ONE, s)


def argmax(v: np.ndarray) -> int:
    """First maximum (lowest index on ties), integer_lut.rs:103-113."""
    return int(np.argmax(v))  # numpy returns the first occurrence


def rmsnorm(x: np.ndarray, gamma: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.int64)
    n = len(x)
    ss = int(((x * x) >> FRAC_BITS).sum(dtype=np.int64))
    ss = wrap(ss)
    inv = integer_isqrt(wrap(tdiv(ss, n) + 1))
    g = np.full(n, ONE, dtype=np.int64)
    k = min(n, len(gamma))
    g[:k] = gamma[:k]
    return (((x * inv) >> FRAC_BITS) * g) >> FRAC_BITS


def rope(v: np.ndarray, pos: int, d_head: int, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Half-split RoPE on one head vector (returns a new array)."""
    half = d_head // 2
    c = cos[pos * half:(pos + 1) * half]
    s = sin[pos * half:(pos + 1) * half]
    x0, x1 = v[:half], v[half:2 * half]
    out = v.copy()
    out[:half] = ((x0 * c) >> FRAC_BITS) - ((x1 * s) >> FRAC_BITS)
    out[half:2 * half] = ((x0 * s) >> FRAC_BITS) + ((x1 * c) >> FRAC_BITS)
    return out


def linear_i8(w: np.ndarray, s: np.ndarray, x: np.ndarray) -> np.ndarray:
    """out = ((W_i8 @ x) * s) >> 16 with wrapping i64 (221-262)."""
    acc = w.astype(np.int64) @ np.asarray(x, dtype=np.int64)
    return (acc * s) >> FRAC_BITS


def penalize(v: int) -> int:
    return tdiv(wrap(v * 5), 6) if v > 0 else tdiv(wrap(v * 6), 5)


def apply_repetition_penalty(logits: np.ndarray, generated) -> np.ndarray:
    """Compounding penalty over the last 64 generated ids, newest first."""
    out = logits.copy()
    for t in list(reversed(generated))[:64]:
        if t < len(out):
            out[t] = penalize(int(out[t]))
    return out


# ---------------------------------------------------------------------------
# Q4 (reference per-row variant and the group-32 extension)
# ---------------------------------------------------------------------------
def q4_from_i8(w: np.ndarray, s: np.ndarray):
    """Q4WeightsX86::from_i8 (cached_integer_model.rs:670-701).

    Returns (nibble values in [-8, 7] as int8 [rows, cols], row scales)."""
    am = np.maximum(np.abs(w.astype(np.int16)).max(axis=1), 1).astype(np.int64)
    qpu = np.maximum((am + 6) // 7, 1)
    v = tdiv_np(w.astype(np.int64), qpu[:, None])
    v = np.clip(v, -8, 7).astype(np.int8)
    return v, s * qpu


def q4_pack(v: np.ndarray) -> np.ndarray:
    """bias-8 nibbles, low nibble = even column."""
    lo = (v[:, 0::2].astype(np.int16) + 8) & 0xF
    hi = (v[:, 1::2].astype(np.int16) + 8) & 0xF
    return (lo | (hi << 4)).astype(np.uint8)


# Q4 group-32 (extension): nibble q in [-8, 7]; per 32-column group an
# unsigned 4-bit multiplier m_g in [1, 15]; per-row Q16 scale s.  The
# fixed-point group scale is s * m_g, and
#     out_i = ((sum_g m_g * sum_{j in g} q_j x_j) * s_i) >> 16,
# i.e. the effective int8 weight is m_g * q_j in [-120, 105].
Q4G = 32


def q4g_effective(q: np.ndarray, m: np.ndarray) -> np.ndarray:
    rows, cols = q.shape
    mm = np.repeat(m.astype(np.int16), Q4G, axis=1)[:, :cols]
    return (q.astype(np.int16) * mm).astype(np.int8)


def q4g_from_i8(w: np.ndarray, s: np.ndarray):
    """Group-32 Q4 of an int8 matrix: per 32-column group
    m_g = clamp(ceil(absmax_g / 7), 1, 15) and q = clamp(trunc(w / m_g), -8, 7)
    (the reference's per-row rule, cached_integer_model.rs:682-690, applied per
    group with a 4-bit multiplier); the row scale s is kept.  Returns
    (q int8 [rows, cols], m uint8 [rows, groups], s)."""
    rows, cols = w.shape
    ng = (cols + Q4G - 1) // Q4G
    pad = ng * Q4G - cols
    wp = np.pad(w.astype(np.int64), ((0, 0), (0, pad)))
    g = wp.reshape(rows, ng, Q4G)
    am = np.maximum(np.abs(g).max(axis=2), 1)
    m = np.clip((am + 6) // 7, 1, 15)
    q = np.clip(tdiv_np(g, m[:, :, None]), -8, 7).reshape(rows, ng * Q4G)[:, :cols]
    return q.astype(np.int8), m.astype(np.uint8), s.copy()


def q4g_effective_model(model):
    """The INT8 model whose weights are the effective group-Q4 values m_g * q
    (the oracle for group-32 Q4 runs this model)."""
    import copy

    out = copy.copy(model)

    def eff(w, s):
        q, m, s2 = q4g_from_i8(w, s)
        return q4g_effective(q, m), s2

    out.out, out.out_s = eff(model.out, model.out_s)
    out.layers = []
    for L in model.layers:
        L2 = dict(L)
        for n in ("wq", "wk", "wv", "wo", "gate", "up", "down"):
            L2[n], L2[n + "_s"] = eff(L[n], L[n + "_s"])
        out.layers.append(L2)
    return out


# ---------------------------------------------------------------------------
# Dense decoder forward / generate (numpy restatement)
# ---------------------------------------------------------------------------
class NumpyEngine:
    """Single-stream restatement of CachedIntegerModel over an Int8Model."""

    def __init__(self, model):
        self.m = model
        c = model.cfg
        self.k = [[] for _ in range(c.n_layers)]
        self.v = [[] for _ in range(c.n_layers)]
        self.pos = 0
        self.emb = model.emb.astype(np.int64) * model.emb_s[:, None]
        self.lin = lambda name, layer, x: linear_i8(layer[name], layer[name + "_s"], x)

    def forward(self, tok: int) -> np.ndarray:
        m, c = self.m, self.m.cfg
        dh, half = c.d_head, c.d_head // 2
        pos = self.pos
        h = self.emb[min(tok, c.vocab - 1)].copy()
        for li, L in enumerate(m.layers):
            n = rmsnorm(h, L["attn_norm"])
            q = self.lin("wq", L, n)
            k = self.lin("wk", L, n)
            v = self.lin("wv", L, n)
            for hh in range(c.n_heads):
                q[hh * dh:(hh + 1) * dh] = rope(q[hh * dh:(hh + 1) * dh], pos, dh, m.rope_cos, m.rope_sin)
            for hh in range(c.n_kv_heads):
                k[hh * dh:(hh + 1) * dh] = rope(k[hh * dh:(hh + 1) * dh], pos, dh, m.rope_cos, m.rope_sin)
            self.k[li].append(k)
            self.v[li].append(v)
            K = np.stack(self.k[li])
            V = np.stack(self.v[li])
            ao = np.zeros(c.d_model, dtype=np.int64)
            for hq in range(c.n_heads):
                kvh = hq * c.n_kv_heads // c.n_heads
                qh = q[hq * dh:(hq + 1) * dh]
                Kh = K[:, kvh * dh:(kvh + 1) * dh]
                dots = (Kh * qh).sum(axis=1, dtype=np.int64)
                sc = ((dots >> FRAC_BITS) * m.attn_scale) >> FRAC_BITS
                w = softmax(sc)
                Vh = V[:, kvh * dh:(kvh + 1) * dh]
                ao[hq * dh:(hq + 1) * dh] = ((w[:, None] * Vh) >> FRAC_BITS).sum(axis=0, dtype=np.int64)
            h = h + self.lin("wo", L, ao)
            n2 = rmsnorm(h, L["ffn_norm"])
            g = self.lin("gate", L, n2)
            u = self.lin("up", L, n2)
            gg = (silu_np(g) * u) >> FRAC_BITS
            h = h + self.lin("down", L, gg)
        self.pos = pos + 1
        nf = rmsnorm(h, m.final_norm)
        return linear_i8(m.out, m.out_s, nf)

    def generate(self, prompt, max_tokens: int, eos=()):
        self.forward(1)
        for t in prompt:
            self.forward(int(t))
        gen = []
        for _ in range(max_tokens):
            last = gen[-1] if gen else (int(prompt[-1]) if len(prompt) else 0)
            logits = apply_repetition_penalty(self.forward(last), gen)
            nxt = argmax(logits)
            gen.append(nxt)
            if nxt in eos:
                break
        return gen


def tokens_hash(tokens) -> bytes:
    """output_hash = BLAKE3(concat LE u32 tokens) (cached_integer_model.rs:1553-1555)."""
    from arc_chain_b200.utils.hashing import blake3

    return blake3(np.asarray(list(tokens), dtype="<u4").tobytes())
