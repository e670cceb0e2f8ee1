"""The reference's small full-sequence integer transformer (its determinism
benchmark model; crates/arc-inference/src/integer_engine.rs): native C++
implementation in ``csrc/ref/toy_engine.cpp`` plus a numpy restatement used
to cross-check it.

Model: i64 Q16 weights drawn from an LCG (seed 42, value
((r >> 33) % 13107) - 6553), pre-LayerNorm blocks (mean / variance /
integer inverse sqrt, gamma = ONE, beta = 0), multi-head attention over the
whole sequence with masked scores set to -8 * ONE (they still enter the
softmax), ReLU FFN, final LayerNorm and LM head on the last position.
Generation recomputes the whole sequence per token (masked positions can
contribute, so caching would change results).
"""
from __future__ import annotations

import ctypes as C
from typing import List, Sequence, Tuple

import numpy as np

from arc_chain_b200 import spec

ONE = spec.ONE
M64 = (1 << 64) - 1


def _lib():
    from arc_chain_b200.oracle import arcref

    lib = arcref.lib()
    if not getattr(lib, "_toy_sigs", False):
        vp = C.c_void_p
        lib.arcref_toy_build.restype = vp
        lib.arcref_toy_build.argtypes = [C.c_int] * 5
        lib.arcref_toy_free.restype = None
        lib.arcref_toy_free.argtypes = [vp]
        lib.arcref_toy_forward.restype = None
        lib.arcref_toy_forward.argtypes = [vp, vp, C.c_int, vp]
        lib.arcref_toy_generate.restype = C.c_int
        lib.arcref_toy_generate.argtypes = [vp, vp, C.c_int, C.c_int, C.c_uint32, vp, vp]
        lib._toy_sigs = True
    return lib


class ToyIntegerModel:
    """``build_test_model(vocab, d_model, n_heads, d_ff, n_layers)``."""

    def __init__(self, vocab: int, d_model: int, n_heads: int, d_ff: int, n_layers: int):
        self.vocab, self.d, self.h, self.ff, self.layers = vocab, d_model, n_heads, d_ff, n_layers
        self._lib = _lib()
        self._h = self._lib.arcref_toy_build(vocab, d_model, n_heads, d_ff, n_layers)

    def forward(self, tokens: Sequence[int]) -> np.ndarray:
        t = np.asarray(list(tokens), dtype=np.uint32)
        out = np.zeros(self.vocab, dtype=np.int64)
        self._lib.arcref_toy_forward(self._h, t.ctypes.data_as(C.c_void_p), t.size, out.ctypes.data_as(C.c_void_p))
        return out

    def generate_with_hash(self, prompt: Sequence[int], max_tokens: int, eos: int) -> Tuple[List[int], bytes]:
        p = np.asarray(list(prompt), dtype=np.uint32)
        out = np.zeros(max(1, max_tokens), dtype=np.uint32)
        h = np.zeros(32, dtype=np.uint8)
        n = self._lib.arcref_toy_generate(self._h, p.ctypes.data_as(C.c_void_p), p.size, max_tokens, eos,
                                          out.ctypes.data_as(C.c_void_p), h.ctypes.data_as(C.c_void_p))
        return [int(x) for x in out[:n]], h.tobytes()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.arcref_toy_free(h)
            self._h = None


# ---------------------------------------------------------------- numpy restatement
def _wrap(x: np.ndarray) -> np.ndarray:
    return x.astype(np.int64)


def lcg_weights(n_total: List[int]) -> List[np.ndarray]:
    """The LCG stream cut into consecutive vectors of the given sizes."""
    r = 42
    out = []
    for n in n_total:
        v = np.empty(n, dtype=np.int64)
        for i in range(n):
            r = (r * 6364136223846793005 + 1442695040888963407) & M64
            v[i] = ((r >> 33) % 13107) - 6553
        out.append(v)
    return out


class NumpyToy:
    def __init__(self, vocab, d, h, ff, layers):
        self.vocab, self.d, self.h, self.ff, self.layers = vocab, d, h, ff, layers
        self.dh = d // h
        sizes = [vocab * d, vocab * d] + [d * d, d * d, d * d, d * d, ff * d, d * ff] * layers
        ws = lcg_weights(sizes)
        self.emb = ws[0].reshape(vocab, d)
        self.lm = ws[1].reshape(vocab, d)
        self.blocks = []
        for l in range(layers):
            b = ws[2 + 6 * l: 8 + 6 * l]
            self.blocks.append([b[0].reshape(d, d), b[1].reshape(d, d), b[2].reshape(d, d), b[3].reshape(d, d),
                                b[4].reshape(ff, d), b[5].reshape(d, ff)])
        self.scale = {32: 11585, 64: 8192, 128: 5793}.get(self.dh, ONE // (int(np.sqrt(self.dh)) + 1))

    @staticmethod
    def _mm(W, x):
        with np.errstate(over="ignore"):
            return (W.astype(np.int64) @ x.astype(np.int64)) >> 16

    @staticmethod
    def _ln(x):
        n = len(x)
        with np.errstate(over="ignore"):
            mean = spec.tdiv_np(np.array([x.sum(dtype=np.int64)]), n)[0]
            diff = x - mean
            var = spec.tdiv_np(np.array([((diff * diff) >> 16).sum(dtype=np.int64)]), n)[0]
            inv = spec.integer_isqrt(int(var) + 1)
            nm = (diff * inv) >> 16
            return (nm * ONE) >> 16

    def forward(self, toks):
        d, dh, T = self.d, self.dh, len(toks)
        x = np.stack([self.emb[t] if t < self.vocab else np.zeros(d, np.int64) for t in toks])
        for wq, wk, wv, wo, f1, f2 in self.blocks:
            nx = np.stack([self._ln(x[t]) for t in range(T)])
            q = np.stack([self._mm(wq, nx[t]) for t in range(T)])
            k = np.stack([self._mm(wk, nx[t]) for t in range(T)])
            v = np.stack([self._mm(wv, nx[t]) for t in range(T)])
            att = np.zeros((T, d), np.int64)
            for hh in range(self.h):
                o = hh * dh
                for i in range(T):
                    sc = np.empty(T, np.int64)
                    for j in range(T):
                        if j > i:
                            sc[j] = -8 * ONE
                        else:
                            with np.errstate(over="ignore"):
                                dot = int((q[i, o:o + dh] * k[j, o:o + dh]).sum(dtype=np.int64)) >> 16
                            sc[j] = (dot * self.scale) >> 16
                    p = spec.softmax(sc)
                    with np.errstate(over="ignore"):
                        att[i, o:o + dh] = (p[:, None] * v[:, o:o + dh]).sum(axis=0, dtype=np.int64) >> 16
            r1 = x + np.stack([self._mm(wo, att[t]) for t in range(T)])
            out = np.empty_like(r1)
            for t in range(T):
                hid = np.maximum(self._mm(f1, self._ln(r1[t])), 0)
                out[t] = r1[t] + self._mm(f2, hid)
            x = out
        return self._mm(self.lm, self._ln(x[-1]))
