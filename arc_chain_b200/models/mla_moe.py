"""DeepSeek-V2-Lite-style MLA + MoE decoder: integer semantics, seeded
weights and the numpy oracle.

The reference has neither MLA nor MoE; their integer semantics are defined
here from the reference's primitives (Q16 per-row INT8 linear, RMSNorm,
half-split RoPE, softmax_i64, SiLU, repetition penalty; see
:mod:`arc_chain_b200.spec`) and then implemented on the GPU
(:mod:`arc_chain_b200.models.mla_moe_engine`), which must match this oracle
bit for bit.

Per layer, with H heads, dn = qk_nope_dim, dr = qk_rope_dim, dv = v_head_dim,
r = kv_lora_rank:

MLA (absorbed form, cache = latent c_j and shared k_rope_j per position)::

    n      = RMSNorm(h, attn_norm)
    q      = Lin_q(n)                    per head [q_nope (dn) | q_rope (dr)]
    q_rope = RoPE(q_rope, pos)           half split over dr
    kva    = Lin_kva(n)                  [c (r) | k_rope (dr)]
    c      = RMSNorm(c, kv_norm);  k_rope = RoPE(k_rope, pos)
    qa_h   = Lin_uk[h](q_nope_h)         [r]   (per-head INT8 [r x dn])
    s_hj   = attn_score(qa_h . c_j + q_rope_h . k_rope_j)   (wrapping i64 dot)
    w      = softmax_i64(s_h0..s_hpos)
    oc_h   = sum_j (w_j * c_j) >> 16     [r]   (per term)
    o_h    = Lin_uv[h](oc_h)             [dv]  (per-head INT8 [dv x r])
    h     += Lin_o(concat o_h)

FFN: the first ``first_dense_layers`` layers use the dense SwiGLU FFN;
the others are MoE::

    n2   = RMSNorm(h, ffn_norm)
    p    = softmax_i64(Lin_router(n2))                      [E]
    top  = the k experts with the largest p (ties: lower index first)
    h   += sum_{e in top} (p_e * FFN_e(n2)) >> 16  +  sum_s FFN_s(n2)
    FFN_x(v) = Lin_down_x(swiglu(Lin_gate_x(v), Lin_up_x(v)))

(routing weights are not renormalised; shared experts have weight 1).  The
generate loop (BOS, re-fed last prompt token, penalty, argmax, EOS) is the
dense engine's.
"""
from __future__ import annotations

import numpy as np

from arc_chain_b200 import spec
from arc_chain_b200.formats import gen
from arc_chain_b200.formats.arc_int8 import Int8Model
from arc_chain_b200.models.config import ModelConfig

ONE = spec.ONE

# ext tensor slots per layer
SLOTS = {"q": 0, "kva": 1, "uk": 2, "uv": 3, "wo": 4, "gate": 5, "up": 6, "down": 7, "router": 8,
         "attn_norm": 9, "ffn_norm": 10, "kv_norm": 11}
EXPERT_SLOT0 = 64  # slot 64 + 3*e + {0 gate, 1 up, 2 down}; shared experts after the routed ones


def shapes(cfg: ModelConfig, layer: int):
    d, H = cfg.d_model, cfg.n_heads
    dn, dr, dv, r = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
    s = {"q": (H * (dn + dr), d), "kva": (r + dr, d), "uk": (H * r, dn), "uv": (H * dv, r), "wo": (d, H * dv)}
    if layer < cfg.first_dense_layers:
        s.update({"gate": (cfg.d_ff, d), "up": (cfg.d_ff, d), "down": (d, cfg.d_ff)})
    else:
        s["router"] = (cfg.n_experts, d)
    return s


def random_mla_moe_model(cfg: ModelConfig, seed: int = 0) -> Int8Model:
    d, V = cfg.d_model, cfg.vocab
    emb, emb_s = gen.matrix(seed, 0, V, d, base=gen.EMB_SCALE_BASE)
    out, out_s = gen.matrix(seed, 1, V, d)
    fn = gen.gamma(seed, (2 << 2) | 1, d)
    rc, rs = gen.rope_tables(cfg.qk_rope_dim, cfg.max_seq, cfg.rope_theta)
    layers = []
    for l in range(cfg.n_layers):
        L = {}
        for name, (rows, cols) in shapes(cfg, l).items():
            L[name], L[name + "_s"] = gen.matrix(seed, gen.ext_tensor_id(l, SLOTS[name]), rows, cols)
        for name, n in (("attn_norm", d), ("ffn_norm", d), ("kv_norm", cfg.kv_lora_rank)):
            L[name] = gen.gamma(seed, (gen.ext_tensor_id(l, SLOTS[name]) << 2) | 1, n)
        if l >= cfg.first_dense_layers:
            E, S, f = cfg.n_experts, cfg.n_shared_experts, cfg.moe_d_ff
            for kind, count, off in (("e", E, 0), ("s", S, E)):
                g, gs, u, us, dw, ds = [], [], [], [], [], []
                for e in range(count):
                    base = EXPERT_SLOT0 + 3 * (off + e)
                    a, b = gen.matrix(seed, gen.ext_tensor_id(l, base), f, d); g.append(a); gs.append(b)
                    a, b = gen.matrix(seed, gen.ext_tensor_id(l, base + 1), f, d); u.append(a); us.append(b)
                    a, b = gen.matrix(seed, gen.ext_tensor_id(l, base + 2), d, f); dw.append(a); ds.append(b)
                L[kind + "g"], L[kind + "g_s"] = np.stack(g), np.stack(gs)
                L[kind + "u"], L[kind + "u_s"] = np.stack(u), np.stack(us)
                L[kind + "d"], L[kind + "d_s"] = np.stack(dw), np.stack(ds)
        layers.append(L)
    vocab = [f"tok_{i}" for i in range(V)]
    return Int8Model(cfg, cfg.resolved_attn_scale(), rc, rs, emb, emb_s, out, out_s, fn, layers, vocab)


def topk(p: np.ndarray, k: int):
    """Indices of the k largest values, ties to the lower index, ordered by
    (value desc, index asc)."""
    order = sorted(range(len(p)), key=lambda i: (-int(p[i]), i))
    return order[:k]


def ffn(x, g, gs, u, us, dw, ds):
    a = spec.linear_i8(g, gs, x)
    b = spec.linear_i8(u, us, x)
    return spec.linear_i8(dw, ds, (spec.silu_np(a) * b) >> 16)


class MlaMoeOracle:
    """Single-stream numpy oracle of the MLA + MoE decoder."""

    def __init__(self, m: Int8Model):
        self.m = m
        c = m.cfg
        self.c_cache = [[] for _ in range(c.n_layers)]
        self.kr_cache = [[] for _ in range(c.n_layers)]
        self.pos = 0
        self.emb = m.emb.astype(np.int64) * m.emb_s[:, None]

    def forward(self, tok: int) -> np.ndarray:
        m, c = self.m, self.m.cfg
        H, dn, dr, dv, r = c.n_heads, c.qk_nope_dim, c.qk_rope_dim, c.v_head_dim, c.kv_lora_rank
        pos = self.pos
        h = self.emb[min(tok, c.vocab - 1)].copy()
        for li, L in enumerate(m.layers):
            n = spec.rmsnorm(h, L["attn_norm"])
            q = spec.linear_i8(L["q"], L["q_s"], n).reshape(H, dn + dr)
            kva = spec.linear_i8(L["kva"], L["kva_s"], n)
            cj = spec.rmsnorm(kva[:r], L["kv_norm"])
            kr = spec.rope(kva[r:], pos, dr, m.rope_cos, m.rope_sin)
            self.c_cache[li].append(cj)
            self.kr_cache[li].append(kr)
            Cc = np.stack(self.c_cache[li])
            Kr = np.stack(self.kr_cache[li])
            outs = []
            for hh in range(H):
                qn = q[hh, :dn]
                qr = spec.rope(q[hh, dn:].copy(), pos, dr, m.rope_cos, m.rope_sin)
                qa = spec.linear_i8(L["uk"][hh * r:(hh + 1) * r], L["uk_s"][hh * r:(hh + 1) * r], qn)
                dots = (Cc * qa).sum(axis=1, dtype=np.int64) + (Kr * qr).sum(axis=1, dtype=np.int64)
                sc = ((dots >> 16) * m.attn_scale) >> 16
                w = spec.softmax(sc)
                oc = ((w[:, None] * Cc) >> 16).sum(axis=0, dtype=np.int64)
                outs.append(spec.linear_i8(L["uv"][hh * dv:(hh + 1) * dv], L["uv_s"][hh * dv:(hh + 1) * dv], oc))
            h = h + spec.linear_i8(L["wo"], L["wo_s"], np.concatenate(outs))
            n2 = spec.rmsnorm(h, L["ffn_norm"])
            if li < c.first_dense_layers:
                h = h + ffn(n2, L["gate"], L["gate_s"], L["up"], L["up_s"], L["down"], L["down_s"])
            else:
                p = spec.softmax(spec.linear_i8(L["router"], L["router_s"], n2))
                y = np.zeros_like(h)
                for e in topk(p, c.moe_top_k):
                    fe = ffn(n2, L["eg"][e], L["eg_s"][e], L["eu"][e], L["eu_s"][e], L["ed"][e], L["ed_s"][e])
                    y = y + ((int(p[e]) * fe) >> 16)
                for s in range(c.n_shared_experts):
                    y = y + ffn(n2, L["sg"][s], L["sg_s"][s], L["su"][s], L["su_s"][s], L["sd"][s], L["sd_s"][s])
                h = h + y
        self.pos = pos + 1
        return spec.linear_i8(m.out, m.out_s, spec.rmsnorm(h, m.final_norm))

    def generate(self, prompt, max_tokens: int, eos=()):
        self.forward(1)
        for t in prompt:
            self.forward(int(t))
        out = []
        for _ in range(max_tokens):
            last = out[-1] if out else (int(prompt[-1]) if len(prompt) else 0)
            nxt = spec.argmax(spec.apply_repetition_penalty(self.forward(last), out))
            out.append(nxt)
            if nxt in eos:
                break
        return out, spec.tokens_hash(out)
