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
    ep_rank: int = 0
    ep_size: int = 1

    @property
    def vocab_local(self):
        return self.lm.M


def local_experts(cfg: ModelConfig, ep_rank: int = 0, ep_size: int = 1) -> List[int]:
    """Global expert indices (routed 0..E-1, then shared E..E+S-1) that
    expert-parallel rank `ep_rank` of `ep_size` holds: g % ep_size == ep_rank."""
    G = cfg.n_experts + cfg.n_shared_experts
    return [g for g in range(G) if g % ep_size == ep_rank]


def from_host(m: Int8Model, device, ep_rank: int = 0, ep_size: int = 1) -> MlaMoeModel:
    """Device model from a host model; with ep_size > 1 only this rank's
    experts are kept (all other weights are replicated)."""
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
            for g in local_experts(c, ep_rank, ep_size):
                kind, e = ("e", g) if g < c.n_experts else ("s", g - c.n_experts)
                gw.append(interleave_pairs(L[kind + "g"][e], L[kind + "u"][e]))
                gs.append(interleave_pairs(L[kind + "g_s"][e], L[kind + "u_s"][e]))
                dw.append(L[kind + "d"][e])
                ds.append(L[kind + "d_s"][e])
            ly.egu = Linear(T(np.concatenate(gw)), T(np.concatenate(gs))).build_map()
            ly.edown = Linear(T(np.concatenate(dw)), T(np.concatenate(ds))).build_map()
        layers.append(ly)
    lm = Linear(T(m.out), T(m.out_s)).build_map()
    return MlaMoeModel(c, int(m.attn_scale), T(m.emb), T(m.emb_s), lm, T(m.final_norm), T(m.rope_cos),
                       T(m.rope_sin), layers, ep_rank=ep_rank, ep_size=ep_size)


def random_device(cfg: ModelConfig, device, seed: int = 0, ep_rank: int = 0, ep_size: int = 1) -> MlaMoeModel:
    """Seeded random-init MLA + MoE model generated on the device (the same
    values as :func:`arc_chain_b200.models.mla_moe.random_mla_moe_model`),
    holding only this expert-parallel rank's experts."""
    from arc_chain_b200.formats import gen
    from arc_chain_b200.models.mla_moe import EXPERT_SLOT0, SLOTS, shapes

    dev = torch.device(device)
    d, V, f = cfg.d_model, cfg.vocab, cfg.moe_d_ff

    def mat(tid, rows, cols, base=None):
        w = torch.empty(rows * cols, dtype=I8, device=dev)
        ops.rng_i8(seed, tid << 2, w)
        sc = gen.row_scales(seed, (tid << 2) | 1, rows, gen.scale_base(cols) if base is None else base)
        return w.view(rows, cols), torch.from_numpy(sc).to(dev)

    def gamma(tid, n):
        return torch.from_numpy(gen.gamma(seed, (tid << 2) | 1, n)).to(dev)

    emb, emb_s = mat(0, V, d, base=gen.EMB_SCALE_BASE)
    out, out_s = mat(1, V, d)
    rc, rs = gen.rope_tables(cfg.qk_rope_dim, cfg.max_seq, cfg.rope_theta)
    layers = []
    for l in range(cfg.n_layers):
        ext = lambda slot: gen.ext_tensor_id(l, slot)
        W = {n: mat(ext(SLOTS[n]), *rc_) for n, rc_ in shapes(cfg, l).items()}
        lin = lambda n: Linear(*W[n]).build_map()
        ly = MlaLayer(lin("q"), lin("kva"), gamma(ext(SLOTS["kv_norm"]), cfg.kv_lora_rank), W["uk"][0].contiguous(),
                      W["uk"][1], W["uv"][0].contiguous(), W["uv"][1], lin("wo"),
                      gamma(ext(SLOTS["attn_norm"]), d), gamma(ext(SLOTS["ffn_norm"]), d))
        if l < cfg.first_dense_layers:
            (wg, sg), (wu, su) = W["gate"], W["up"]
            ly.gu = Linear(interleave_pairs(wg, wu).contiguous(), interleave_pairs(sg, su).contiguous()).build_map()
            ly.down = lin("down")
        else:
            ly.router = lin("router")
            gw, gs, dw, ds = [], [], [], []
            for g in local_experts(cfg, ep_rank, ep_size):
                base = EXPERT_SLOT0 + 3 * g
                wg, sg = mat(ext(base), f, d)
                wu, su = mat(ext(base + 1), f, d)
                wd, sd = mat(ext(base + 2), d, f)
                gw.append(interleave_pairs(wg, wu))
                gs.append(interleave_pairs(sg, su))
                dw.append(wd)
                ds.append(sd)
            ly.egu = Linear(torch.cat(gw).contiguous(), torch.cat(gs).contiguous()).build_map()
            ly.edown = Linear(torch.cat(dw).contiguous(), torch.cat(ds).contiguous()).build_map()
            del gw, dw
        layers.append(ly)
        del W
    lm = Linear(out, out_s).build_map()
    return MlaMoeModel(cfg, int(cfg.resolved_attn_scale()), emb.contiguous(), emb_s, lm, gamma(2, d),
                       torch.from_numpy(rc).to(dev), torch.from_numpy(rs).to(dev), layers, ep_rank=ep_rank,
                       ep_size=ep_size)


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
        rows = ops.limb_rows(B, self.bn)
        self.Xd = torch.zeros(rows, d, dtype=I8, device=dev)
        self.Xo = torch.zeros(rows, H * dv, dtype=I8, device=dev)
        self.Xf = torch.zeros(rows, max(c.d_ff, 16), dtype=I8, device=dev)
        self.Xm = torch.zeros(rows, max(G * c.moe_d_ff, 16), dtype=I8, device=dev)
        sub = min(self.bn, 32)
        self.mXd, self.mXo = ops.TensorMap(self.Xd, self.bn, sub), ops.TensorMap(self.Xo, self.bn, sub)
        self.mXf, self.mXm = ops.TensorMap(self.Xf, self.bn, sub), ops.TensorMap(self.Xm, self.bn, sub)
        ms = [d, c.vocab, H * (dn + dr), r + dr, 2 * c.d_ff]
        for ly in model.layers:
            for lin in (ly.egu, ly.edown, ly.router):
                if lin is not None:
                    ms.append(lin.M)
        mmax = max(ms)
        self.P = torch.zeros(8 * B * mmax, dtype=torch.int32, device=dev)
        self.tiles = torch.zeros(ops.tile_counters(mmax, B), dtype=I32, device=dev)
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

    def __init__(self, model: MlaMoeModel, n_pages: Optional[int] = None, max_seq: Optional[int] = None,
                 comm: Optional[Comm] = None):
        self.m = model
        c = model.cfg
        self.comm = comm or Comm()
        self.ep = getattr(self.comm, "ep", False)
        # token dispatch: the trunk runs on this rank's own slots only
        self.dispatch = getattr(self.comm, "token_dispatch", False)
        if self.ep and (self.comm.size != model.ep_size or self.comm.rank != model.ep_rank):
            raise ValueError("model's expert shard does not match the communicator's rank/size")
        if not self.ep and model.ep_size != 1:
            raise ValueError("an expert-sharded model needs an expert-parallel communicator")
        self.n_moe = sum(1 for ly in model.layers if ly.edown is not None)
        self.max_seq = max_seq or c.max_seq
        self.max_pages = (self.max_seq + PAGE - 1) // PAGE
        if n_pages is None:
            n_pages = 4 * self.max_pages
        self.dk = c.kv_lora_rank + c.qk_rope_dim
        self.kv = PagedKV(c.n_layers, n_pages, 1, self.dk, model.emb.device, self.max_pages, with_v=False)
        self._bufs = {}
        self._graphs = {}
        self._rid = 0
        self.op_events = None  # a list: forward records (label, event) after each op

    def _moe_index(self, layer: int) -> int:
        return sum(1 for ly in self.m.layers[:layer] if ly.edown is not None)

    def buffers(self, B: int, gen_cap: int = 0) -> MlaBuffers:
        key = (B, gen_cap)
        if key not in self._bufs:
            self._bufs[key] = MlaBuffers(self.m, B, self.max_pages, gen_cap)
        return self._bufs[key]

    def _gathered(self, bb: MlaBuffers):
        """Expert-GEMM operands over the N * B gathered slots of a token-
        dispatch step: the gathered limb planes (written by every rank's
        dispatch), the SwiGLU planes, split-K scratch and counters."""
        gb = getattr(bb, "gath", None)
        if gb is None:
            c = self.m.cfg
            d = c.d_model
            G = c.n_experts + c.n_shared_experts
            st = self.comm.state(bb, self.n_moe, d)
            gb = type("Gathered", (), {})()
            gb.NB = st.NB
            dev = bb.h.device
            bn = ops.fgemm_bn(gb.NB)
            sub = min(bn, 32)
            gb.Xm = torch.zeros(ops.limb_rows(gb.NB, bn), max(G * c.moe_d_ff, 16), dtype=I8, device=dev)
            gb.mXg, gb.mXm = ops.TensorMap(st.Xg, bn, sub), ops.TensorMap(gb.Xm, bn, sub)
            mmax = max(ly.egu.M for ly in self.m.layers if ly.egu is not None)
            mmax = max(mmax, max(ly.edown.M for ly in self.m.layers if ly.edown is not None))
            gb.P = torch.zeros(8 * gb.NB * mmax, dtype=torch.int32, device=dev)
            gb.tiles = torch.zeros(ops.tile_counters(mmax, gb.NB), dtype=I32, device=dev)
            gb.cnt = torch.zeros(1, dtype=I32, device=dev)
            gb.gcnt = st.gcnt
            gb.route = st.route
            bb.gath = gb
        return gb

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
                gb = self._gathered(bb) if self.dispatch else None
                e["egu"] = ops.epi(ops.SWIGLU, ly.egu.s, bb.err, X=gb.Xm if gb else bb.Xm, ldx=G * c.moe_d_ff,
                                   lmax_out=gb.cnt if gb else bb.cnt[4 * l + 3:4 * l + 4])
                ed = ops.epi(ops.MOE_COMBINE, ly.edown.s, bb.err, out=bb.h, ldo=d,
                             route=gb.route if gb else bb.route, route_ld=G)
                ed.grp_rows, ed.grp_koff = d, c.moe_d_ff
                if self.ep:
                    # local group g is global expert rank + g * size
                    ed.route = (gb.route if gb else bb.route).data_ptr() + 8 * m.ep_rank
                    ed.route_gs = m.ep_size
                    ed = self.comm.combine_epi(ed, bb, self._moe_index(l), self.n_moe, d)
                e["edown"] = ed
            out.append(e)
        out.append({"lm": ops.epi(ops.STORE, m.lm.s, bb.err, out=bb.logits, ldo=m.lm.M)})
        bb.epis = out
        return out

    def forward(self, bb: MlaBuffers, B: int, with_logits: bool = True, span=None) -> None:
        # span (a prefill chunk's extent) selects the dense model's chunk
        # attention; MLA attention runs per position here
        m, c = self.m, self.m.cfg
        d, H = c.d_model, c.n_heads
        dn, dr, dv, r = c.qk_nope_dim, c.qk_rope_dim, c.v_head_dim, c.kv_lora_rank
        G = c.n_experts + c.n_shared_experts
        E = self._epis(bb)
        T = self.max_pages * PAGE
        ev = self.op_events

        def mark(label):
            if ev is not None:
                e_ = torch.cuda.Event(enable_timing=True)
                e_.record()
                ev.append((label, e_))

        ops.embed(bb.tokens, m.emb, m.emb_s, c.vocab, d, B, bb.h, bb.cnt, bb.ss)
        mark("embed")
        for l, ly in enumerate(m.layers):
            c0, c1, c2, c3 = (bb.cnt[4 * l + i:4 * l + i + 1] for i in range(4))
            e = E[l]
            ops.rmsnorm_limbs(bb.h, ly.attn_norm, d, B, bb.Xd, c0)
            mark("norm")
            ops.linear_gemm(ly.q, bb.mXd, B, c0, bb.P, bb.tiles, e["q"])
            ops.linear_gemm(ly.kva, bb.mXd, B, c0, bb.P, bb.tiles, e["kva"])
            mark("q_kva")
            ops.mla_kv(bb.kva, r, dr, ly.kv_norm, self.kv.K[l], bb.pt, bb.pos, m.rope_cos, m.rope_sin,
                       self.max_seq, B, bb.err)
            ops.mla_q(bb.q, H, dn, dr, r, ly.uk, ly.uk_s, bb.pos, m.rope_cos, m.rope_sin, self.max_seq, B, bb.Q)
            mark("mla_kv_q")
            ops.attn_mla(bb.Q, self.kv.K[l], bb.pt, bb.pos, H, self.dk, r, m.attn_scale, T, B, bb.oc, bb.err)
            mark("attn")
            ops.mla_out(bb.oc, H, r, dv, ly.uv, ly.uv_s, B, bb.Xo, c1)
            mark("mla_out")
            ops.linear_gemm(ly.wo, bb.mXo, B, c1, bb.P, bb.tiles, e["wo"])
            mark("wo")
            ops.rmsnorm_limbs(bb.h, ly.ffn_norm, d, B, bb.Xd, c2)
            mark("norm")
            if ly.gu is not None:
                ops.linear_gemm(ly.gu, bb.mXd, B, c2, bb.P, bb.tiles, e["gu"])
                ops.linear_gemm(ly.down, bb.mXf, B, c3, bb.P, bb.tiles, e["down"])
                mark("dense_ffn")
            else:
                ops.linear_gemm(ly.router, bb.mXd, B, c2, bb.P, bb.tiles, e["router"])
                mark("router")
                ops.moe_route(bb.rlog, c.n_experts, c.n_shared_experts, c.moe_top_k, B, bb.route)
                mark("route")
                if self.dispatch:
                    gb = self._gathered(bb)
                    self.comm.dispatch(bb, bb.Xd, c2, self.n_moe, d, gb.cnt)
                    mark("dispatch")
                    ops.linear_gemm(ly.egu, gb.mXg, gb.NB, gb.gcnt, gb.P, gb.tiles, e["egu"])
                    mark("expert_gate_up")
                    ops.linear_gemm(ly.edown, gb.mXm, gb.NB, gb.cnt, gb.P, gb.tiles, e["edown"])
                    mark("expert_down_combine")
                else:
                    ops.linear_gemm(ly.egu, bb.mXd, B, c2, bb.P, bb.tiles, e["egu"])
                    mark("expert_gate_up")
                    ops.linear_gemm(ly.edown, bb.mXm, B, c3, bb.P, bb.tiles, e["edown"])
                    mark("expert_down_combine")
                if self.ep:
                    self.comm.after_combine(bb, self._moe_index(l), self.n_moe, d)
                    mark("combine_wait")
        if with_logits:
            cf = bb.cnt[4 * c.n_layers:4 * c.n_layers + 1]
            ops.rmsnorm_limbs(bb.h, m.final_norm, d, B, bb.Xd, cf)
            ops.linear_gemm(m.lm, bb.mXd, B, cf, bb.P, bb.tiles, E[-1]["lm"])
            mark("lm_head")
