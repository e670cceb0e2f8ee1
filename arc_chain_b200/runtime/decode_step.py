"""Host side of the persistent decode-step kernel (``csrc/kernels/decode_step.cu``):
builds the phase program of one single-stream decode step (B <= 2) of a
dense model on one GPU and launches it between the embedding and sampling
kernels.

The program is static for a buffer set (pointers, tensor maps, epilogue
descriptors), so it is built once, copied to the device, and the launch is
CUDA-graph capturable.  Outputs are bit-identical to the per-kernel path
(same GEMM arithmetic and epilogues).
"""
from __future__ import annotations

import ctypes as C
from typing import List

import torch

from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.ops._lib import lib

K_NORM, K_GEMM, K_ATTN = 0, 1, 2
vp, ci, cll = C.c_void_p, C.c_int, C.c_longlong


class NormP(C.Structure):
    _fields_ = [("h", vp), ("ss", vp), ("gamma", vp), ("ngamma", ci), ("d", ci), ("B", ci), ("X", vp), ("lmax", vp)]


class AttnP(C.Structure):
    _fields_ = [("q", vp), ("Kc", vp), ("Vc", vp), ("pt", vp), ("pt_stride", ci), ("pos", vp), ("n_heads", ci),
                ("n_kv", ci), ("dh", ci), ("attn_scale", cll), ("max_T", ci), ("B", ci), ("S", ci), ("X", vp),
                ("lmax", vp), ("gmax", vp), ("gsum", vp), ("gout", vp), ("cnt", vp)]


class Phase(C.Structure):
    _fields_ = [("kind", ci), ("idx", ci)]


class Program(C.Structure):
    _fields_ = [("n_phases", ci), ("n_gemms", ci), ("phases", vp), ("norms", vp), ("attns", vp), ("gemms", vp),
                ("bar", vp), ("P", vp), ("err", vp), ("prof", vp)]


_SIZES = None


def sizes():
    global _SIZES
    if _SIZES is None:
        out = (C.c_int * 8)()
        lib().arcb_ds_sizes(out)
        _SIZES = list(out)
        want = [C.sizeof(NormP), C.sizeof(AttnP), None, C.sizeof(Phase), C.sizeof(Program), None,
                C.sizeof(ops.Epi)]
        for i, w in enumerate(want):
            if w is not None and w != _SIZES[i]:
                raise RuntimeError(f"decode-step record {i}: host layout {w} bytes != device {_SIZES[i]}")
    return _SIZES


def eligible(engine, bb) -> bool:
    m = engine.m
    return (bb.B <= 2 and m.tp_size == 1 and getattr(m, "emb_q16", None) is None and
            all(getattr(Ly.qkv, "q4", None) is None for Ly in m.layers) and m.cfg.d_head <= 128 and
            getattr(engine.comm, "size", 1) == 1)


def _to_dev(structs: List[C.Structure], size: int, dev) -> torch.Tensor:
    raw = bytearray(max(1, len(structs)) * size)
    for i, s in enumerate(structs):
        b = bytes(s) if isinstance(s, C.Structure) else s
        raw[i * size:i * size + len(b)] = b
    return torch.frombuffer(raw, dtype=torch.uint8).clone().to(dev)


class StepProgram:
    """The phase program of a decode step over buffer set `bb` of `engine`."""

    def __init__(self, engine, bb):
        sz = sizes()
        m, c = engine.m, engine.m.cfg
        dev = bb.h.device
        E = engine._epis(bb)
        d, dh, B = c.d_model, c.d_head, bb.B
        nh, nkv = m.n_heads_local, m.n_kv_local
        n_layers = c.n_layers
        n_phases = 7 * n_layers + 2
        # limb counters (4 per layer + final) then one barrier counter per phase; zeroed by the embedding kernel
        self.cnt = torch.zeros(4 * n_layers + 4 + n_phases, dtype=torch.int32, device=dev)
        cnt, bars = self.cnt[:4 * n_layers + 4], self.cnt[4 * n_layers + 4:]
        sms = ops.num_sms()
        S = 4 if sms % 4 == 0 else (2 if sms % 2 == 0 else 1)
        nbh = B * nh
        self.gmax = torch.full((nbh,), -(1 << 63), dtype=torch.int64, device=dev)
        self.gsum = torch.zeros(nbh, dtype=torch.int64, device=dev)
        self.gout = torch.zeros(nbh * dh, dtype=torch.int64, device=dev)
        self.acnt = torch.zeros(3 * nbh, dtype=torch.int32, device=dev)
        phases, norms, attns, gemms = [], [], [], []
        ss = bb.ss
        T = engine.max_pages * 16

        def norm(h, ssv, gamma, lm):
            norms.append(NormP(h.data_ptr(), ssv.data_ptr(), gamma.data_ptr(), gamma.numel(), d, B,
                               bb.Xd.data_ptr(), lm.data_ptr()))
            phases.append(Phase(K_NORM, len(norms) - 1))

        def gemm(lin, xmap, lm, epi):
            raw = C.create_string_buffer(sz[2])
            ops.check(lib().arcb_ds_gemm(raw, lin.tmap.addr, xmap.addr, lin.M, lin.K, B, len(phases) - 1,
                                         lm.data_ptr(), bb.tiles.data_ptr(), C.addressof(epi)), "ds_gemm")
            gemms.append(raw.raw)
            phases.append(Phase(K_GEMM, len(gemms) - 1))

        for l, Ly in enumerate(m.layers):
            c0, c1, c2, c3 = (cnt[4 * l + i:4 * l + i + 1] for i in range(4))
            e = E[l]
            norm(bb.h, ss[2 * l], Ly.attn_norm, c0)
            gemm(Ly.qkv, bb.mXd, c0, e["qkv"])
            attns.append(AttnP(bb.q.data_ptr(), engine.kv.K[l].data_ptr(), engine.kv.V[l].data_ptr(),
                               bb.pt.data_ptr(), bb.pt.shape[1], bb.pos.data_ptr(), nh, nkv, dh, int(m.attn_scale), T,
                               B, S, bb.Xo.data_ptr(), c1.data_ptr(), self.gmax.data_ptr(), self.gsum.data_ptr(),
                               self.gout.data_ptr(), self.acnt.data_ptr()))
            phases.append(Phase(K_ATTN, len(attns) - 1))
            gemm(Ly.wo, bb.mXo, c1, e["wo"])
            norm(bb.h, ss[2 * l + 1], Ly.ffn_norm, c2)
            # the SwiGLU epilogue publishes its output's limb count into this program's counters
            egu = ops.Epi.from_buffer_copy(e["gu"])
            egu.lmax_out = c3.data_ptr()
            gemm(Ly.gu, bb.mXd, c2, egu)
            gemm(Ly.down, bb.mXf, c3, e["down"])
        cf = cnt[4 * n_layers:4 * n_layers + 1]
        norm(bb.h, ss[2 * n_layers], m.final_norm, cf)
        gemm(m.lm, bb.mXd, cf, E[-1]["lm"])
        assert len(phases) == n_phases
        self.t_phases = _to_dev(phases, sz[3], dev)
        self.t_norms = _to_dev(norms, sz[0], dev)
        self.t_attns = _to_dev(attns, sz[1], dev)
        self.t_gemms = _to_dev(gemms, sz[2], dev)
        assert self.t_gemms.data_ptr() % 64 == 0
        self.prog = Program(n_phases, len(gemms), self.t_phases.data_ptr(), self.t_norms.data_ptr(),
                            self.t_attns.data_ptr(), self.t_gemms.data_ptr(), bars.data_ptr(), bb.P.data_ptr(),
                            bb.err.data_ptr(), None)
        self.n_phases = n_phases
        self.kinds = [ph.kind for ph in phases]

    def enable_profile(self, on: bool = True) -> None:
        """Record per-phase %globaltimer stamps of CTA 0 (see ``profile``)."""
        if on:
            self.t_prof = torch.zeros(2 * self.n_phases, dtype=torch.int64, device=self.cnt.device)
            self.prog.prof = self.t_prof.data_ptr()
        else:
            self.prog.prof = None

    def profile(self):
        """(kind, start_us, duration_us) of every phase of the last launch,
        times from the first phase's start."""
        t = self.t_prof.view(-1, 2).cpu().tolist()
        t0 = t[0][0]
        names = {K_NORM: "norm", K_GEMM: "gemm", K_ATTN: "attn"}
        return [(names[k], (a - t0) / 1000, (b - a) / 1000) for k, (a, b) in zip(self.kinds, t)]

    def launch(self) -> None:
        ops._count()
        ops.check(lib().arcb_decode_step(C.addressof(self.prog), ops._s()), "decode_step")
