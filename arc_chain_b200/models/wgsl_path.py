"""The reference's GPU compute-shader decode path, restated.

The reference ships a second, GPU-resident decoder (crates/arc-gpu/src/
transformer.wgsl, dispatched by GpuForward::forward_one_token in
gpu_forward.rs:656-720) that computes a different function from its CPU
integer engine: i32 activations, an abs-max i8 quantisation before every
matmul (`acc * (scale >> 8)`), a mean-subtracting LayerNorm with an f32
square root, an i8 KV cache with per-position scales, a piecewise-linear
exp, `g > 0 ? g : g >> 2` in place of SiLU, and an argmax that breaks ties
by thread order.  As wired there, the hidden state is uploaded as zeros
every token (gpu_forward.rs:664-666) and the KV caches are never written,
so its output is token 0 at every step.  Even with a real embedding, the
matmul's `scale >> 8` is 0 for Q16 per-row scales below 256, which covers
ordinary INT8 weights (max |w| / 127 in Q16), so the projections vanish.

Two restatements run that arithmetic:

* :class:`WgslPathHost` - C++ (csrc/ref/wgsl_forward.cpp), the oracle;
* :class:`WgslPathDevice` - CUDA (csrc/kernels/wgsl_path.cu), the same nine
  kernels with the same workgroup shapes, launched in the reference's order.

``embedding="zero"`` reproduces the reference's upload; ``embedding="q16"``
feeds the CPU engine's Q16 embedding row (truncated to i32, as every
buffer of that path is i32), which with per-row scales of 2^8 or more runs
the arithmetic on non-zero values.  The
exact engine (runtime/engine.py) is the product; this module exists to pin
down what the reference's GPU numbers compute.
"""
from __future__ import annotations

import ctypes as C
from typing import List, Sequence, Tuple

import numpy as np

from arc_chain_b200.formats.arc_int8 import Int8Model

MATS = ("wq", "wk", "wv", "wo", "gate", "up", "down")
ROPE_ROWS = 2048  # the reference uploads its tables for 2048 positions


def _i32(a) -> np.ndarray:
    """`x as i32` of an int64 array (low 32 bits)."""
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64).astype(np.uint64).astype(np.uint32).view(np.int32))


def _words(w: np.ndarray) -> np.ndarray:
    """int8 [rows, cols] -> little-endian packed u32 words (4 per word)."""
    b = np.ascontiguousarray(w, dtype=np.int8).reshape(-1)
    pad = (-b.size) % 4
    if pad:
        b = np.concatenate([b, np.zeros(pad, np.int8)])
    return b.view(np.uint32).copy()


def _rope_tables(model: Int8Model) -> Tuple[np.ndarray, np.ndarray]:
    half = model.cfg.d_head // 2
    n = min(ROPE_ROWS, model.rope_cos.size // half)
    cs = np.zeros(ROPE_ROWS * half, np.int64)
    sn = np.zeros(ROPE_ROWS * half, np.int64)
    cs[:n * half] = np.asarray(model.rope_cos).reshape(-1)[:n * half]
    sn[:n * half] = np.asarray(model.rope_sin).reshape(-1)[:n * half]
    return cs, sn


class _Embed:
    def __init__(self, model: Int8Model, mode: str):
        if mode not in ("zero", "q16"):
            raise ValueError("embedding must be 'zero' (the reference's upload) or 'q16'")
        self.mode, self.d, self.V = mode, model.cfg.d_model, model.cfg.vocab
        if mode == "q16":
            q16 = model.emb_q16 if model.emb_q16 is not None else model.emb.astype(np.int64) * model.emb_s[:, None]
            self.table = _i32(q16)

    def __call__(self, tok: int) -> np.ndarray:
        if self.mode == "zero":
            return np.zeros(self.d, np.int32)
        return self.table[min(int(tok), self.V - 1)].copy()


def _generate(step, emb: _Embed, prompt: Sequence[int], max_tokens: int) -> List[int]:
    """BOS at position 0, the prompt, then greedy tokens fed back."""
    toks = [1] + [int(t) for t in prompt]
    nxt = 0
    for p, t in enumerate(toks):
        nxt = step(emb(t), p)
    out, pos = [], len(toks)
    for _ in range(max_tokens):
        out.append(nxt)
        nxt = step(emb(nxt), pos)
        pos += 1
    return out


class WgslPathHost:
    """C++ restatement (oracle) of the reference's compute-shader path."""

    def __init__(self, model: Int8Model, embedding: str = "zero"):
        from arc_chain_b200.oracle.arcref import lib

        c = model.cfg
        if c.d_model % 4 or c.d_ff % 4:
            raise ValueError("the shader path packs 4 values per word: d_model and d_ff must be multiples of 4")
        self.c, self.L = c, lib()
        self.h = self.L.arcwg_new(c.n_layers, c.d_model, c.d_ff, c.d_head, c.n_heads, c.n_kv_heads, c.vocab,
                                  int(model.attn_scale))
        vp = C.c_void_p
        for li, Ly in enumerate(model.layers):
            ws = [np.ascontiguousarray(Ly[n], dtype=np.int8) for n in MATS]
            ss = [np.ascontiguousarray(Ly[n + "_s"], dtype=np.int64) for n in MATS]
            an = np.ascontiguousarray(Ly["attn_norm"], dtype=np.int64)
            fn = np.ascontiguousarray(Ly["ffn_norm"], dtype=np.int64)
            wp = (vp * 7)(*[a.ctypes.data for a in ws])
            sp = (vp * 7)(*[a.ctypes.data for a in ss])
            if self.L.arcwg_set_layer(self.h, li, wp, sp, an.ctypes.data, fn.ctypes.data) != 0:
                raise ValueError("arcwg_set_layer rejected the layer")
        cs, sn = _rope_tables(model)
        ow = np.ascontiguousarray(model.out, dtype=np.int8)
        os_ = np.ascontiguousarray(model.out_s, dtype=np.int64)
        fnm = np.ascontiguousarray(model.final_norm, dtype=np.int64)
        self.L.arcwg_set_head(self.h, ow.ctypes.data, os_.ctypes.data, fnm.ctypes.data, cs.ctypes.data,
                              sn.ctypes.data, ROPE_ROWS)
        self.emb = _Embed(model, embedding)
        self.logits = np.zeros(c.vocab, np.int32)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.arcwg_free(self.h)
            self.h = None

    def step(self, hidden: np.ndarray, pos: int) -> int:
        hid = np.ascontiguousarray(hidden, dtype=np.int32)
        return int(self.L.arcwg_forward(self.h, hid.ctypes.data, int(pos), self.logits.ctypes.data))

    def generate(self, prompt: Sequence[int], max_tokens: int) -> List[int]:
        return _generate(self.step, self.emb, prompt, max_tokens)


class WgslPathDevice:
    """CUDA restatement of the reference's compute-shader path: one launch
    per reference dispatch (19 per layer + 4), on the current stream."""

    def __init__(self, model: Int8Model, device="cuda", embedding: str = "zero"):
        import torch

        c = model.cfg
        if c.d_model % 4 or c.d_ff % 4:
            raise ValueError("the shader path packs 4 values per word: d_model and d_ff must be multiples of 4")
        self.c, self.dev, self.torch = c, torch.device(device), torch
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(self.dev)
        self.layers = []
        for Ly in model.layers:
            self.layers.append({
                **{n: T(_words(Ly[n]).view(np.int32)) for n in MATS},
                **{n + "_s": T(_i32(Ly[n + "_s"])) for n in MATS},
                "an": T(_i32(Ly["attn_norm"])), "fn": T(_i32(Ly["ffn_norm"])),
            })
        self.lm_w, self.lm_s = T(_words(model.out).view(np.int32)), T(_i32(model.out_s))
        self.fnorm = T(_i32(model.final_norm))
        cs, sn = _rope_tables(model)
        self.cos, self.sin = T(_i32(cs)), T(_i32(sn))
        d, dff, dkv = c.d_model, c.d_ff, c.n_kv_heads * c.d_head
        z = lambda n, dt=torch.int32: torch.zeros(n, dtype=dt, device=self.dev)
        kvw = (2048 * dkv + 3) // 4
        self.kv = [(z(kvw), z(kvw), z(2048), z(2048)) for _ in range(c.n_layers)]  # never written, as in the reference
        self.hidden, self.normed, self.q, self.k, self.v = z(d), z(d), z(d), z(dkv), z(dkv)
        self.attn_out, self.proj, self.gate, self.up, self.ff_out = z(d), z(d), z(dff), z(dff), z(d)
        self.logits, self.packed = z(c.vocab), z((max(d, dff) + 3) // 4)
        self.qscale, self.result = z(1), z(1)
        self.attn_scale = int(np.int64(model.attn_scale).astype(np.uint64).astype(np.uint32).view(np.int32))
        self.emb = _Embed(model, embedding)

    def _launch_token(self, pos: int) -> None:
        from arc_chain_b200.ops import int_ops as ops
        from arc_chain_b200.ops._lib import check, lib

        L, s, c = lib(), ops._s(), self.c
        p = lambda t: t.data_ptr()
        n = lambda t: t.numel()
        d, dff, dh, dkv = c.d_model, c.d_ff, c.d_head, c.n_kv_heads * c.d_head

        def ln(x, g):
            check(L.arcb_wg_layernorm(p(x), n(x), p(self.normed), n(self.normed), p(g), n(g), d, s), "wg_layernorm")

        def qz(x):
            check(L.arcb_wg_quantize(p(x), n(x), p(self.packed), n(self.packed), p(self.qscale), s), "wg_quantize")

        def mm(w, sc, out, k, m):
            check(L.arcb_wg_matmul(p(w), n(w), p(self.packed), n(self.packed), p(out), n(out), k, m, p(sc), n(sc), s),
                  "wg_matmul")

        def rope(x, heads):
            check(L.arcb_wg_rope(p(x), n(x), p(self.cos), p(self.sin), n(self.cos), pos, dh, heads, s), "wg_rope")

        for Ly, (kc, vc, ks, vs) in zip(self.layers, self.kv):
            ln(self.hidden, Ly["an"])
            qz(self.normed)
            mm(Ly["wq"], Ly["wq_s"], self.q, d, d)
            mm(Ly["wk"], Ly["wk_s"], self.k, d, dkv)
            mm(Ly["wv"], Ly["wv_s"], self.v, d, dkv)
            rope(self.q, c.n_heads)
            rope(self.k, c.n_kv_heads)
            check(L.arcb_wg_attention(p(self.q), n(self.q), p(kc), p(vc), n(kc), p(ks), p(vs), n(ks), p(self.attn_out),
                                      n(self.attn_out), dh, c.n_heads, c.n_kv_heads, pos + 1, dkv, self.attn_scale, s),
                  "wg_attention")
            qz(self.attn_out)
            mm(Ly["wo"], Ly["wo_s"], self.proj, d, d)
            check(L.arcb_wg_residual(p(self.hidden), p(self.proj), d, s), "wg_residual")
            ln(self.hidden, Ly["fn"])
            qz(self.normed)
            mm(Ly["gate"], Ly["gate_s"], self.gate, d, dff)
            mm(Ly["up"], Ly["up_s"], self.up, d, dff)
            check(L.arcb_wg_silu(p(self.gate), p(self.up), dff, s), "wg_silu")
            qz(self.gate)
            mm(Ly["down"], Ly["down_s"], self.ff_out, dff, d)
            check(L.arcb_wg_residual(p(self.hidden), p(self.ff_out), d, s), "wg_residual")
        ln(self.hidden, self.fnorm)
        qz(self.normed)
        mm(self.lm_w, self.lm_s, self.logits, d, c.vocab)
        check(L.arcb_wg_argmax(p(self.logits), n(self.logits), p(self.result), s), "wg_argmax")
        ops.LAUNCHES[0] += 19 * c.n_layers + 4

    def step(self, hidden: np.ndarray, pos: int) -> int:
        self.hidden.copy_(self.torch.from_numpy(np.ascontiguousarray(hidden, dtype=np.int32)))
        self._launch_token(pos)
        return int(self.result.item())

    def generate(self, prompt: Sequence[int], max_tokens: int) -> List[int]:
        return _generate(self.step, self.emb, prompt, max_tokens)
