"""MLA + MoE decoder on B200: device weights and the decode engine.

Semantics: :mod:`arc_chain_b200.models.mla_moe` (the oracle).  Per layer:

    RMSNorm+limbs -> Lin_q (fused GEMM, store) -> Lin_kva (store)
    -> latent KV prep (RMSNorm of c, RoPE of k_rope, paged latent cache)
    -> absorbed queries (per-head W_uk, RoPE of q_rope)
    -> MLA attention over [c | k_rope] (cluster kernel, one shared latent head)
    -> per-head W_uv straight into limb planes -> Lin_o (residual)
    -> RMSNorm+limbs -> dense SwiGLU FFN, or MoE:
         Lin_router (store) -> softmax_i64 + top-k routing table
         -> grouped gate/up GEMM over all routed + shared experts (SwiGLU
            epilogue, each expert's intermediate in its own column block)
         -> grouped down GEMM (each expert reads its own block) whose
            epilogue adds (p_e * y) >> 16 into the hidden state (shared
            experts have p = ONE)

Expert weights stream once per step regardless of how many tokens chose
them; the grouped GEMMs compute every (token, expert) pair and the routing
weight zeroes the unchosen ones, which is exact and costs only idle tensor
cycles in decode.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from arc_chain_b200.formats.arc_int8 import Int8Model
from arc_chain_b200.models.config import ModelConfig
from arc_chain_b200.models.dense import Linear, interleave_pairs
from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.runtime.engine import Comm, Engine, I32, I64, I8
from arc_chain_b200.runtime.kv_paged import PAGE, PagedKV


@dataclass
class MlaLayer:
    q: Linear
    kva: Linear
    kv_norm: torch.Tensor
    uk: torch.Tensor
    uk_s: torch.Tensor
    uv: torch.Tensor
    uv_s: torch.Tensor
    wo: Linear
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor
    gu: Optional[Linear] = None      # dense FFN
    down: Optional[Linear] = None
    router: Optional[Linear] = None  # MoE
    egu: Optional[Linear] = None
    edown: Optional[Linear] = None


@dataclass
class MlaMoeModel:
    cfg: ModelConfig
    attn_scale: int
    emb: torch.Tensor
    emb_s: torch.Tensor
    lm: Linear
    final_norm: torch.Tensor
    rope_cos: torch.Tensor
    rope_sin: torch.Tensor
    layers: List[MlaLayer]
    tp_size: int = 1
    vocab_offset: int = 0

    @property
    def vocab_local(self):
        return self.lm.M


def from_host(m: Int8Model, device) -> MlaMoeModel:
    c = m.cfg
    dev = torch.device(device)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    layers = []
    for li, L in enumerate(m.layers):
        lin = lambda n: Linear(T(L[n]), T(L[n + "_s"])).build_map()
        ly = MlaLayer(lin("q"), lin("kva"), T(L["kv_norm"]), T(L["uk"]), T(L["uk_s"]), T(L["uv"]), T(L["uv_s"]),
                      lin("wo"), T(L["attn_norm"]), T(L["ffn_norm"]))
        if li < c.first_dense_layers:
            ly.gu = Linear(T(interleave_pairs(L["gate"], L["up"])), T(interleave_pairs(L["gate_s"], L["up_s"]))).build_map()
            ly.down = lin("down")
        else:
            ly.router = lin("router")
            gw, gs, dw, ds = [], [], [], []
            for kind, cnt in (("e", c.n_experts), ("s", c.n_shared_experts)):
                for e in range(cnt):
                    gw.append(interleave_pairs(L[kind + "g"][e], L[kind + "u"][e]))
                    gs.append(interleave_pairs(L[kind + "g_s"][e], L[kind + "u_s"][e]))
                    dw.append(L[kind + "d"][e])
                    ds.append(L[kind + "d_s"][e])
            ly.egu = Linear(T(np.concatenate(gw)), T(np.concatenate(gs))).build_map()
            ly.edown = Linear(T(np.concatenate(dw)), T(np.concatenate(ds))).build_map()
        layers.append(ly)
    lm = Linear(T(m.out), T(m.out_s)).build_map()
    return MlaMoeModel(c, int(m.attn_scale), T(m.emb), T(m.emb_s), lm, T(m.final_norm), T(m.rope_cos),
                       T(m.rope_sin), layers)


class MlaBuffers:
    def __init__(self, model: MlaMoeModel, B: int, max_pages: int, gen_cap: int = 0):
        c = model.cfg
        dev = model.emb.device
        self.B = B
        d, H = c.d_model, c.n_heads
        dn, dr, dv, r = c.qk_nope_dim, c.qk_rope_dim, c.v_head_dim, c.kv_lora_rank
        G = c.n_experts + c.n_shared_experts
        self.tokens = torch.zeros(B, dtype=I32, device=dev)
        self.pos = torch.zeros(B, dtype=I32, device=dev)
        self.pt = torch.zeros(B, max_pages, dtype=I32, device=dev)
        self.h = torch.zeros(B, d, dtype=I64, device=dev)
        self.q = torch.zeros(B, H * (dn + dr), dtype=I64, device=dev)
        self.kva = torch.zeros(B, r + dr, dtype=I64, device=dev)
        self.Q = torch.zeros(B, H, r + dr, dtype=I64, device=dev)
        self.oc = torch.zeros(B, H, r, dtype=I64, device=dev)
        self.bn = ops.fgemm_bn(B)
        rows = max(8 * B, self.bn)
        self.Xd = torch.zeros(rows, d, dtype=I8, device=dev)
        self.Xo = torch.zeros(rows, H * dv, dtype=I8, device=dev)
        self.Xf = torch.zeros(rows, max(c.d_ff, 16), dtype=I8, device=dev)
        self.Xm = torch.zeros(rows, max(G * c.moe_d_ff, 16), dtype=I8, device=dev)
        self.mXd, self.mXo = ops.TensorMap(self.Xd, self.bn), ops.TensorMap(self.Xo, self.bn)
        self.mXf, self.mXm = ops.TensorMap(self.Xf, self.bn), ops.TensorMap(self.Xm, self.bn)
        ms = [d, c.vocab, H * (dn + dr), r + dr, 2 * c.d_ff]
        for ly in model.layers:
            for lin in (ly.egu, ly.edown, ly.router):
                if lin is not None:
                    ms.append(lin.M)
        mmax = max(ms)
        self.P = torch.zeros(8 * B * mmax, dtype=torch.int32, device=dev)
        self.tiles = torch.zeros((mmax + 127) // 128 + 1, dtype=I32, device=dev)
        self.cnt = torch.zeros(4 * c.n_layers + 4, dtype=I32, device=dev)
        self.ss = torch.zeros(1, B, dtype=I64, device=dev)
        self.err = torch.zeros(1, dtype=I32, device=dev)
        self.rlog = torch.zeros(B, max(c.n_experts, 1), dtype=I64, device=dev)
        self.route = torch.zeros(B, max(G, 1), dtype=I64, device=dev)
        self.logits = torch.zeros(B, c.vocab, dtype=I64, device=dev)
        self.logits_local = self.logits
        self.hist = torch.zeros(B, 64, dtype=I32, device=dev)
        self.count = torch.zeros(B, dtype=I32, device=dev)
        self.gen = torch.zeros(B, max(1, gen_cap), dtype=I32, device=dev)
        self.done = torch.zeros(B, dtype=I32, device=dev)
        self.eos = torch.zeros(8, dtype=I32, device=dev)
        self.n_eos = 0
        self.epis = None


class MlaMoeEngine(Engine):
    """Engine for the MLA + MoE model (single GPU); reuses the dense engine's
    request, prefill, generate and CUDA-graph machinery."""

    def __init__(self, model: MlaMoeModel, n_pages: Optional[int] = None, max_seq: Optional[int] = None):
        self.m = model
        c = model.cfg
        self.comm = Comm()
        self.max_seq = max_seq or c.max_seq
        self.max_pages = (self.max_seq + PAGE - 1) // PAGE
        if n_pages is None:
            n_pages = 4 * self.max_pages
        self.dk = c.kv_lora_rank + c.qk_rope_dim
        self.kv = PagedKV(c.n_layers, n_pages, 1, self.dk, model.emb.device, self.max_pages, with_v=False)
        self._bufs = {}
        self._graphs = {}
        self._rid = 0

    def buffers(self, B: int, gen_cap: int = 0) -> MlaBuffers:
        key = (B, gen_cap)
        if key not in self._bufs:
            self._bufs[key] = MlaBuffers(self.m, B, self.max_pages, gen_cap)
        return self._bufs[key]

    def _epis(self, bb: MlaBuffers):
        if bb.epis is not None:
            return bb.epis
        m, c = self.m, self.m.cfg
        d = c.d_model
        G = c.n_experts + c.n_shared_experts
        out = []
        for l, ly in enumerate(m.layers):
            e = {"q": ops.epi(ops.STORE, ly.q.s, bb.err, out=bb.q, ldo=ly.q.M),
                 "kva": ops.epi(ops.STORE, ly.kva.s, bb.err, out=bb.kva, ldo=ly.kva.M),
                 "wo": ops.epi(ops.RESID, ly.wo.s, bb.err, out=bb.h, ldo=d)}
            if ly.gu is not None:
                e["gu"] = ops.epi(ops.SWIGLU, ly.gu.s, bb.err, X=bb.Xf, ldx=c.d_ff, lmax_out=bb.cnt[4 * l + 3:4 * l + 4])
                e["down"] = ops.epi(ops.RESID, ly.down.s, bb.err, out=bb.h, ldo=d)
            else:
                e["router"] = ops.epi(ops.STORE, ly.router.s, bb.err, out=bb.rlog, ldo=c.n_experts)
                e["egu"] = ops.epi(ops.SWIGLU, ly.egu.s, bb.err, X=bb.Xm, ldx=G * c.moe_d_ff,
                                   lmax_out=bb.cnt[4 * l + 3:4 * l + 4])
                ed = ops.epi(ops.MOE_COMBINE, ly.edown.s, bb.err, out=bb.h, ldo=d, route=bb.route, route_ld=G)
                ed.grp_rows, ed.grp_koff = d, c.moe_d_ff
                e["edown"] = ed
            out.append(e)
        out.append({"lm": ops.epi(ops.STORE, m.lm.s, bb.err, out=bb.logits, ldo=m.lm.M)})
        bb.epis = out
        return out

    def forward(self, bb: MlaBuffers, B: int, with_logits: bool = True) -> None:
        m, c = self.m, self.m.cfg
        d, H = c.d_model, c.n_heads
        dn, dr, dv, r = c.qk_nope_dim, c.qk_rope_dim, c.v_head_dim, c.kv_lora_rank
        G = c.n_experts + c.n_shared_experts
        E = self._epis(bb)
        T = self.max_pages * PAGE
        ops.embed(bb.tokens, m.emb, m.emb_s, c.vocab, d, B, bb.h, bb.cnt, bb.ss)
        for l, ly in enumerate(m.layers):
            c0, c1, c2, c3 = (bb.cnt[4 * l + i:4 * l + i + 1] for i in range(4))
            e = E[l]
            ops.rmsnorm_limbs(bb.h, ly.attn_norm, d, B, bb.Xd, c0)
            ops.linear_gemm(ly.q, bb.mXd, B, c0, bb.P, bb.tiles, e["q"])
            ops.linear_gemm(ly.kva, bb.mXd, B, c0, bb.P, bb.tiles, e["kva"])
            ops.mla_kv(bb.kva, r, dr, ly.kv_norm, self.kv.K[l], bb.pt, bb.pos, m.rope_cos, m.rope_sin,
                       self.max_seq, B, bb.err)
            ops.mla_q(bb.q, H, dn, dr, r, ly.uk, ly.uk_s, bb.pos, m.rope_cos, m.rope_sin, self.max_seq, B, bb.Q)
            ops.attn_mla(bb.Q, self.kv.K[l], bb.pt, bb.pos, H, self.dk, r, m.attn_scale, T, B, bb.oc, bb.err)
            ops.mla_out(bb.oc, H, r, dv, ly.uv, ly.uv_s, B, bb.Xo, c1)
            ops.linear_gemm(ly.wo, bb.mXo, B, c1, bb.P, bb.tiles, e["wo"])
            ops.rmsnorm_limbs(bb.h, ly.ffn_norm, d, B, bb.Xd, c2)
            if ly.gu is not None:
                ops.linear_gemm(ly.gu, bb.mXd, B, c2, bb.P, bb.tiles, e["gu"])
                ops.linear_gemm(ly.down, bb.mXf, B, c3, bb.P, bb.tiles, e["down"])
            else:
                ops.linear_gemm(ly.router, bb.mXd, B, c2, bb.P, bb.tiles, e["router"])
                ops.moe_route(bb.rlog, c.n_experts, c.n_shared_experts, c.moe_top_k, B, bb.route)
                ops.linear_gemm(ly.egu, bb.mXd, B, c2, bb.P, bb.tiles, e["egu"])
                ops.linear_gemm(ly.edown, bb.mXm, B, c3, bb.P, bb.tiles, e["edown"])
        if with_logits:
            cf = bb.cnt[4 * c.n_layers:4 * c.n_layers + 1]
            ops.rmsnorm_limbs(bb.h, m.final_norm, d, B, bb.Xd, cf)
            ops.linear_gemm(m.lm, bb.mXd, B, cf, bb.P, bb.tiles, E[-1]["lm"])
