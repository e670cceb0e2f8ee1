"""Host side of the persistent dataflow decode step (``csrc/kernels/decode_flow.cu``).

One decode step of a dense INT8 decoder over 1 or 2 slots (single-stream
decode, a pair of lanes) runs as ONE cooperative kernel: embedding, every
layer's norms, GEMMs and attention, the final norm and the LM head.  The
sampling kernel follows it.  This module builds the step's program (phase
list, per-GEMM records with their TMA maps, norm and attention records, the
monotonic dependency counters, the u64 split-K accumulators and, under
tensor parallelism, the symmetric receive buffers and arrival counters), keeps
it on the device, and launches it.  The program is static for a buffer set,
so the launch is CUDA-graph capturable.

Outputs are bit-identical to the reference CPU engine (and to the per-kernel
path): every reduction is an exact integer sum.  Counterpart in the
reference: the per-token hot loop ``forward_one_token``
(crates/arc-inference/src/cached_integer_model.rs:1381-1516), which runs
rayon 512-row chunks per matmul (247-262) and one task per head (1448-1476).
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional

import torch

from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.ops._lib import check, lib

PH_NORM, PH_GEMM, PH_ATTN = 0, 1, 2
DEP_COUNT, DEP_HEADS, DEP_SWIGLU = 0, 1, 3
FIN_APPLY, FIN_NONE, FIN_PUSH = 0, 1, 2
SRC_EMBED, SRC_ACC, SRC_PEERS = 0, 1, 2

vp, ci, cu, cll = C.c_void_p, C.c_int, C.c_uint, C.c_longlong


class NormD(C.Structure):
    _fields_ = [("src", ci), ("d", ci), ("B", ci), ("npeers", ci), ("tokens", vp), ("emb", vp), ("emb_s", vp),
                ("vocab", ci), ("acc", vp), ("src_cnt", vp), ("src_mul", cu), ("R", vp), ("scales", vp),
                ("gamma", vp), ("ngamma", ci), ("ss", vp), ("cnt1", vp), ("cnt2", vp), ("X", vp),
                ("zero_acc", vp), ("zero_n", ci)]


class AttnD(C.Structure):
    _fields_ = [("qkv_acc", vp), ("qkv_scales", vp), ("qkv_cnt", vp), ("qkv_mul", cu), ("qkv_M", ci),
                ("rcos", vp), ("rsin", vp), ("Kc", vp), ("Vc", vp), ("pt", vp), ("pt_stride", ci), ("pos", vp),
                ("n_heads", ci), ("n_kv", ci), ("dh", ci), ("attn_scale", cll), ("max_T", ci), ("B", ci),
                ("X", vp), ("head_done", vp), ("S", ci), ("xmax", vp), ("xsum", vp), ("xout", vp), ("acnt", vp)]


class Phase(C.Structure):
    _fields_ = [("kind", ci), ("idx", ci)]


class Prog(C.Structure):
    _fields_ = [("n_phases", ci), ("n_gemms", ci), ("B", ci), ("max_T", ci), ("phases", vp), ("norms", vp),
                ("gemms", vp), ("attns", vp), ("epoch", vp), ("exit_cnt", vp), ("err", vp), ("lm_arr", vp),
                ("lm_mul", cu), ("prof", vp), ("stats", vp), ("pf_tiles", ci), ("stages", ci)]


_LAYOUT: Optional[List[int]] = None


def layout() -> List[int]:
    """Device record sizes; raises if a host mirror disagrees."""
    global _LAYOUT
    if _LAYOUT is None:
        out = (C.c_int * 16)()
        check(lib().arcb_flow_layout(out), "flow_layout")
        _LAYOUT = list(out)
        want = {0: C.sizeof(NormD), 1: C.sizeof(AttnD), 3: C.sizeof(Phase), 4: C.sizeof(Prog), 6: C.sizeof(ops.Epi)}
        for i, w in want.items():
            if w != _LAYOUT[i]:
                raise RuntimeError(f"decode-flow record {i}: host layout {w} bytes != device {_LAYOUT[i]}")
    return _LAYOUT


MAX_T = 2048  # attention scores live in shared memory


def eligible(engine, B: int) -> Optional[str]:
    """None if the dataflow step serves this engine at B slots, else why not."""
    m, c = engine.m, engine.m.cfg
    if B > 2:
        return "more than 2 slots"
    if any(getattr(Ly.qkv, "q4", None) is not None for Ly in m.layers) or getattr(m.lm, "q4", None) is not None:
        return "Q4 weights"
    if getattr(m, "emb_q16", None) is not None:
        return "full-precision embedding"
    if c.d_head not in (64, 128) or m.n_heads_local % max(1, m.n_kv_local):
        return "head shape"
    cm = engine.comm
    if cm.size > 1 and not getattr(cm, "fused", False):
        return "NCCL communication"
    G = ops.num_sms()
    if -(-c.d_model // G) * B > 4 * 128:
        return "hidden state too large for the register slices"
    if min(engine.max_seq, engine.max_pages * 16) > MAX_T:
        return "context longer than the shared-memory score buffer"
    return None


def _to_dev(records, dev) -> torch.Tensor:
    raw = b"".join(bytes(r) for r in records) or b"\0"
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).clone().to(dev)


class FlowStep:
    """The dataflow program of one decode step over buffer set `bb` (B <= 2)."""

    # weight tiles (16 KB) each SM keeps requested into L2 beyond its
    # shared-memory ring (0: off; measured slower at 16-48 tiles on the 7B
    # decode: the prefetches delay the latency-bound dependency chain)
    PF_TILES = 0
    # W_down runs in groups of this many K chunks (each group tile-major):
    # a CTA's range then needs the SwiGLU tiles of a few chunks only, and its
    # segments stay several items long
    DOWN_KGROUP = 4

    def __init__(self, engine, bb):
        lay = layout()
        m, c = engine.m, engine.m.cfg
        cm = engine.comm
        dev = bb.h.device
        B = bb.B
        G = ops.num_sms()
        d, dh = c.d_model, c.d_head
        nh, nkv = m.n_heads_local, m.n_kv_local
        dq, dkv, dffl = nh * dh, nkv * dh, m.d_ff_local
        L = c.n_layers
        npeers, rank = cm.size, cm.rank
        tp = npeers > 1
        self.B, self.G, self.npeers = B, G, npeers
        self.max_T = min(engine.max_seq, engine.max_pages * 16)
        I8, I64, U32 = torch.int8, torch.int64, torch.int32
        BMr = ops.BM
        mt = lambda M: (M + BMr - 1) // BMr

        # ---- device state (counters are monotonic: zero once, never reset between steps)
        n_norms = 2 * L + 1
        lin_all = [(Ly.qkv, Ly.wo, Ly.gu, Ly.down) for Ly in m.layers]
        n_tiles = sum(mt(x.M) for ls in lin_all for x in ls) + mt(m.lm.M)
        # attention: S CTAs per (slot, head), exchanging through per-layer scratch
        self.S = max(1, min(8, G // (B * nh)))
        n_bh = B * nh
        NSUB = 8  # a grid-wide count is spread over 8 counters
        n_cnt = 2 + 2 * NSUB * n_norms + n_tiles + L * nh + 3 * L * n_bh
        self.cnt = torch.zeros(n_cnt, dtype=U32, device=dev)
        self._cur = 0

        def take(n):
            v = self.cnt[self._cur:self._cur + n]
            self._cur += n
            return v

        self.epoch, self.exit_cnt = take(1), take(1)
        acc_rows = sum(x.M for ls in lin_all for x in ls) + m.lm.M
        self.acc = torch.zeros(B * acc_rows, dtype=I64, device=dev)
        self._acur = 0

        def acc_of(M):
            v = self.acc[self._acur:self._acur + B * M]
            self._acur += B * M
            return v

        self.ss = torch.zeros(n_norms, 2, G, B, dtype=I64, device=dev)  # per-CTA partial sums of squares
        S = self.S
        self.a_xmax = torch.zeros(L, n_bh, S, dtype=I64, device=dev)
        self.a_xsum = torch.zeros(L, n_bh, S, dtype=I64, device=dev)
        self.a_xout = torch.zeros(L, n_bh, S, dh, dtype=I64, device=dev)
        # limb operands (16 rows: 8 planes x up to 2 slots, row l * B + b)
        self.Xn = [torch.zeros(16, d, dtype=I8, device=dev) for _ in range(n_norms)]
        self.Xo = [torch.zeros(16, dq, dtype=I8, device=dev) for _ in range(L)]
        self.Xf = [torch.zeros(16, dffl, dtype=I8, device=dev) for _ in range(L)]
        self.mXn = [ops.TensorMap(x, 16) for x in self.Xn]
        self.mXo = [ops.TensorMap(x, 16) for x in self.Xo]
        self.mXf = [ops.TensorMap(x, 16) for x in self.Xf]

        # ---- tensor parallelism: symmetric receive buffers and arrival counters
        self._symm = []
        if tp:
            import torch.distributed._symmetric_memory as symm_mem

            gname = cm.group_name
            mtd = mt(d)
            n_sites = 2 * L
            self.R = symm_mem.empty(n_sites * npeers * B * d, dtype=I64, device=dev)
            self.arr = symm_mem.empty(n_sites * mtd + 1, dtype=U32, device=dev)
            V = c.vocab
            self.logits_sym = symm_mem.empty(B * V, dtype=I64, device=dev)
            self.R.zero_()
            self.arr.zero_()
            self.logits_sym.zero_()
            hR = symm_mem.rendezvous(self.R, gname)
            hA = symm_mem.rendezvous(self.arr, gname)
            hL = symm_mem.rendezvous(self.logits_sym, gname)
            self._symm = [hR, hA, hL]
            Rp, Ap, Lp = list(hR.buffer_ptrs), list(hA.buffer_ptrs), list(hL.buffer_ptrs)
            site_R = [[Rp[p] + s * npeers * B * d * 8 for p in range(npeers)] for s in range(n_sites)]
            site_A = [[Ap[p] + s * mtd * 4 for p in range(npeers)] for s in range(n_sites)]
            self.peer_R = torch.tensor(site_R, dtype=I64, device=dev)
            self.peer_A = torch.tensor(site_A, dtype=I64, device=dev)
            self.lm_peer_arr = torch.tensor([Ap[p] + n_sites * mtd * 4 for p in range(npeers)], dtype=I64, device=dev)
            self.lm_peer_h = torch.tensor([Lp[p] + m.vocab_offset * 8 for p in range(npeers)], dtype=I64, device=dev)
            self.logits = self.logits_sym.view(B, V)
            # total LM tiles over all ranks (vocab shards may differ in size)
            per = -(-V // npeers)
            self.lm_total = sum(mt(max(0, min(V, (r + 1) * per) - min(V, r * per))) for r in range(npeers))
            torch.cuda.synchronize(dev)
        else:
            self.logits = bb.logits_local

        # ---- program
        phases, norms, attns, gemms = [], [], [], []
        self._keep = []  # host objects whose addresses the records hold

        def gemm_rec(lin, xmap, dep, dep_dh, dep_n, dep_mul, dep_cnt, acc, tile_cnt, tile_fin, fin, peer_R=None,
                     peer_arr=None, epi=None, src=None, kmajor=0):
            raw = C.create_string_buffer(lay[2] + 64)
            addr = (C.addressof(raw) + 63) & ~63
            check(lib().arcb_flow_gemm(addr, lin.tmap.addr, xmap.addr, lin.M, lin.K, dep, dep_dh, dep_n, dep_mul,
                                       ops._p(dep_cnt), ops._p(acc), ops._p(tile_cnt), ops._p(tile_fin), fin, rank,
                                       npeers, peer_R, peer_arr, None if epi is None else C.addressof(epi), B,
                                       lin.w.data_ptr(), ops._p(src[0]) if src else None,
                                       ops._p(src[1]) if src else None, src[2] if src else 0, kmajor),
                  "flow_gemm")
            gemms.append(C.string_at(addr, lay[2]))
            phases.append(Phase(PH_GEMM, len(gemms) - 1))

        def norm_rec(src, gamma, idx, acc=None, src_cnt=None, src_mul=0, R=None, scales=None, zero=None):
            cnt1, cnt2 = take(NSUB), take(NSUB)
            n = NormD(src, d, B, npeers, bb.tokens.data_ptr(), m.emb.data_ptr(), m.emb_s.data_ptr(), c.vocab,
                      ops._p(acc), ops._p(src_cnt), src_mul, R, ops._p(scales), gamma.data_ptr(), gamma.numel(),
                      self.ss[idx].data_ptr(), cnt1.data_ptr(), cnt2.data_ptr(), self.Xn[idx].data_ptr(),
                      ops._p(zero), 0 if zero is None else zero.numel())
            norms.append(n)
            phases.append(Phase(PH_NORM, len(norms) - 1))
            return cnt2

        E = engine._epis(bb)
        nch = lambda K: (K + 127) // 128
        norm_cnt = norm_rec(SRC_EMBED, m.layers[0].attn_norm, 0)
        for l, Ly in enumerate(m.layers):
            # QKV: accumulate; the attention units finalise their heads' rows
            a_qkv, tc_qkv = acc_of(Ly.qkv.M), take(mt(Ly.qkv.M))
            gemm_rec(Ly.qkv, self.mXn[2 * l], DEP_COUNT, 0, 1, G, norm_cnt, a_qkv, tc_qkv, None, FIN_NONE)
            head_done = take(nh)
            acnt = take(3 * n_bh)
            attns.append(AttnD(a_qkv.data_ptr(), Ly.qkv.s.data_ptr(), tc_qkv.data_ptr(), nch(Ly.qkv.K), Ly.qkv.M,
                               m.rope_cos.data_ptr(), m.rope_sin.data_ptr(), engine.kv.K[l].data_ptr(),
                               engine.kv.V[l].data_ptr(), bb.pt.data_ptr(), bb.pt.shape[1], bb.pos.data_ptr(), nh,
                               nkv, dh, int(m.attn_scale), self.max_T, B, self.Xo[l].data_ptr(),
                               head_done.data_ptr(), self.S, self.a_xmax[l].data_ptr(), self.a_xsum[l].data_ptr(),
                               self.a_xout[l].data_ptr(), acnt.data_ptr()))
            phases.append(Phase(PH_ATTN, len(attns) - 1))
            # W_o: residual, finalised by the FFN norm (summed over ranks under TP)
            a_wo, tc_wo = acc_of(d), take(mt(d))
            if tp:
                s = 2 * l
                gemm_rec(Ly.wo, self.mXo[l], DEP_HEADS, dh, nh, B, head_done, a_wo, tc_wo, None, FIN_PUSH,
                         peer_R=self.peer_R[s].data_ptr(), peer_arr=self.peer_A[s].data_ptr())
                norm_cnt = norm_rec(SRC_PEERS, Ly.ffn_norm, 2 * l + 1, src_cnt=self.arr[s * mt(d):],
                                    src_mul=npeers, R=self.R[s * npeers * B * d:].data_ptr(), scales=Ly.wo.s,
                                    zero=a_qkv)
            else:
                gemm_rec(Ly.wo, self.mXo[l], DEP_HEADS, dh, nh, B, head_done, a_wo, tc_wo, None, FIN_NONE)
                norm_cnt = norm_rec(SRC_ACC, Ly.ffn_norm, 2 * l + 1, acc=a_wo, src_cnt=tc_wo,
                                    src_mul=nch(Ly.wo.K), scales=Ly.wo.s, zero=a_qkv)
            # gate/up: accumulate; W_down's epilogue warps apply SwiGLU into its limb tiles
            a_gu, tc_gu = acc_of(Ly.gu.M), take(mt(Ly.gu.M))
            gemm_rec(Ly.gu, self.mXn[2 * l + 1], DEP_COUNT, 0, 1, G, norm_cnt, a_gu, tc_gu, None, FIN_NONE)
            # W_down: residual, finalised by the next norm
            a_dn, tc_dn = acc_of(d), take(mt(d))
            nxt_gamma = m.layers[l + 1].attn_norm if l + 1 < L else m.final_norm
            src = (a_gu, Ly.gu.s, Ly.gu.M)
            if tp:
                s = 2 * l + 1
                gemm_rec(Ly.down, self.mXf[l], DEP_SWIGLU, 0, mt(Ly.gu.M), nch(Ly.gu.K), tc_gu, a_dn, tc_dn, None,
                         FIN_PUSH, peer_R=self.peer_R[s].data_ptr(), peer_arr=self.peer_A[s].data_ptr(), src=src,
                         kmajor=self.DOWN_KGROUP)
                norm_cnt = norm_rec(SRC_PEERS, nxt_gamma, 2 * l + 2, src_cnt=self.arr[s * mt(d):], src_mul=npeers,
                                    R=self.R[s * npeers * B * d:].data_ptr(), scales=Ly.down.s, zero=a_gu)
            else:
                gemm_rec(Ly.down, self.mXf[l], DEP_SWIGLU, 0, mt(Ly.gu.M), nch(Ly.gu.K), tc_gu, a_dn, tc_dn, None,
                         FIN_NONE, src=src, kmajor=self.DOWN_KGROUP)
                norm_cnt = norm_rec(SRC_ACC, nxt_gamma, 2 * l + 2, acc=a_dn, src_cnt=tc_dn,
                                    src_mul=nch(Ly.down.K), scales=Ly.down.s, zero=a_gu)
        # LM head: logits, into every rank's full-vocab buffer under TP
        a_lm, tc_lm = acc_of(m.lm.M), take(mt(m.lm.M))
        e_lm = ops.Epi.from_buffer_copy(E[-1]["lm"])
        if tp:
            e_lm.mode = ops.STORE_PEERS
            e_lm.ldo = c.vocab
            e_lm.npeers = npeers
            e_lm.peer_h = self.lm_peer_h.data_ptr()
            e_lm.peer_sig = None
            e_lm.max_ctas = 0
            self._keep.append(e_lm)
            gemm_rec(m.lm, self.mXn[2 * L], DEP_COUNT, 0, 1, G, norm_cnt, a_lm, tc_lm, None, FIN_APPLY,
                     peer_arr=self.lm_peer_arr.data_ptr(), epi=e_lm)
        else:
            self._keep.append(e_lm)
            gemm_rec(m.lm, self.mXn[2 * L], DEP_COUNT, 0, 1, G, norm_cnt, a_lm, tc_lm, None, FIN_APPLY, epi=e_lm)
        assert self._cur <= n_cnt and self._acur == self.acc.numel()

        self.t_phases = _to_dev(phases, dev)
        self.t_norms = _to_dev(norms, dev)
        self.t_attns = _to_dev(attns, dev)
        self.t_gemms = _to_dev(gemms, dev)
        assert self.t_gemms.data_ptr() % 64 == 0
        self.kinds = [p.kind for p in phases]
        self.n_gemms = len(gemms)
        self.prog = Prog(len(phases), len(gemms), B, self.max_T, self.t_phases.data_ptr(), self.t_norms.data_ptr(),
                         self.t_gemms.data_ptr(), self.t_attns.data_ptr(), self.epoch.data_ptr(),
                         self.exit_cnt.data_ptr(), bb.err.data_ptr(),
                         self.arr[2 * L * mt(d):].data_ptr() if tp else None, self.lm_total if tp else 0, None, None,
                         self.PF_TILES, 0)
        self.t_prof = None
        self.t_stats = None
        torch.cuda.synchronize(dev)

    # ------------------------------------------------------------------
    def launch(self) -> None:
        ops._count()
        check(lib().arcb_flow_launch(C.addressof(self.prog), ops._s()), "flow_launch")

    def reset(self) -> None:
        """Zero the counters, accumulators and sums (after a kernel error
        left a step incomplete).  Single-GPU only: under tensor parallelism the
        peers' arrival counters would have to be reset together."""
        self.cnt.zero_()
        self.acc.zero_()
        self.ss.zero_()
        self.a_xmax.zero_()
        self.a_xsum.zero_()
        self.a_xout.zero_()

    def set_prefetch(self, tiles: int) -> None:
        """L2 prefetch window of the weight producer, in 16 KB tiles per SM."""
        self.prog.pf_tiles = int(tiles)

    def enable_profile(self, on: bool = True) -> None:
        """Record the %globaltimer timeline of the next steps (see ``profile``)."""
        if on:
            n = self.G * len(self.kinds) * 2 + self.G * self.n_gemms * 4
            self.t_prof = torch.zeros(n, dtype=torch.int64, device=self.cnt.device)
            self.prog.prof = self.t_prof.data_ptr()
        else:
            self.prog.prof = None

    def enable_stats(self, on: bool = True) -> None:
        """Record per-CTA wait totals (ns) of the next steps (see ``stats``)."""
        if on:
            self.t_stats = torch.zeros(self.G, 8, dtype=torch.int64, device=self.cnt.device)
            self.prog.stats = self.t_stats.data_ptr()
        else:
            self.prog.stats = None

    STAT_NAMES = ("weights_wait_free", "limbs_wait_deps", "limbs_wait_free", "mma_wait_full", "epi_wait_acc",
                  "norm_waits", "attention", "kernel")

    def stats(self) -> dict:
        """Per-role wait totals of the last step, in us: mean and max over CTAs."""
        t = self.t_stats.double().cpu() / 1000.0
        return {n: {"mean": round(float(t[:, i].mean()), 1), "max": round(float(t[:, i].max()), 1)}
                for i, n in enumerate(self.STAT_NAMES)}

    def profile(self):
        """Timeline of the last step, in us from its first stamp: (phases
        [G, n_phases, 2] start / end per CTA, gemms [G, n_gemms, 4]: first
        weight tile, first limb tile, first MMA, last MMA per CTA; 0 where a
        CTA had no work)."""
        t = self.t_prof.cpu()
        G, P = self.G, len(self.kinds)
        ph = t[:G * P * 2].view(G, P, 2)
        gm = t[G * P * 2:].view(G, self.n_gemms, 4)
        t0 = ph[:, 0, 0].min()
        ph = torch.where(ph > 0, (ph - t0).double() / 1000, torch.zeros((), dtype=torch.float64))
        gm = torch.where(gm > 0, (gm - t0).double() / 1000, torch.zeros((), dtype=torch.float64))
        return ph, gm

    def release(self) -> None:
        self._symm = []
