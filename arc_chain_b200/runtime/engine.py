"""Decode engine for dense INT8 decoders on B200.

One forward over a batch of *slots* (a slot = one token at one position of
one request) runs:

    embed -> per layer [RMSNorm+limbs -> QKV GEMM -> finalize+RoPE+KV append
    -> paged attention (+limbs) -> W_o GEMM -> (TP reduce) -> residual
    -> RMSNorm+limbs -> gate/up GEMM -> SwiGLU+limbs -> down GEMM
    -> (TP reduce) -> residual] -> final RMSNorm -> LM head -> (TP gather)
    -> repetition penalty + argmax

Every output element equals the reference CPU engine's
(crates/arc-inference/src/cached_integer_model.rs:1381-1516): all reductions
are exact integer sums, so batching, prefill of many positions at once, split-K
and tensor-parallel partial sums leave results bit-identical.

``generate`` reproduces the reference's generate loop (1518-1557): BOS=1,
prompt, then the last prompt token is fed again at step 0, compounding
repetition penalty over the newest 64 ids, argmax with lowest-index ties, EOS
kept in the output, output hash = BLAKE3 of the LE u32 ids.  The prompt is
prefilled in one batched forward (its logits are discarded by the reference,
so the LM head is skipped there).  Decode steps replay one CUDA graph.
"""
from __future__ import annotations

import os
import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from arc_chain_b200.models.dense import DenseModel
from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.runtime.kv_paged import PAGE, PagedKV
from arc_chain_b200.utils.hashing import blake3
import numpy as np

I32, I64, I8 = torch.int32, torch.int64, torch.int8


class Comm:
    """Tensor-parallel hooks; the single-GPU instance does nothing."""

    size = 1
    rank = 0

    def reduce_partials(self, P: torch.Tensor, rows: int, M: int, lmax: torch.Tensor) -> None:
        pass

    def gather_logits(self, local: torch.Tensor, full: torch.Tensor, B: int, vocab_offset: int, bb=None) -> None:
        pass

    def fgemm_reduce(self, lin, xmap, B: int, lmax: torch.Tensor, bb: "StepBuffers", epi, site: int = 0) -> None:
        """Row-parallel GEMM whose epilogue sees the full (all-rank) sum; on
        one GPU that is the plain fused GEMM."""
        ops.linear_gemm(lin, xmap, B, lmax, bb.P, bb.tiles, epi)

    @property
    def n_launches(self) -> int:
        return 0


class StepBuffers:
    """Device buffers for a forward over up to B slots."""

    def __init__(self, model: DenseModel, B: int, max_pages: int, gen_cap: int = 0):
        c = model.cfg
        dev = model.emb.device
        self.B = B
        d, dh = c.d_model, c.d_head
        dl = model.n_heads_local * dh
        dffl = model.d_ff_local
        self.tokens = torch.zeros(B, dtype=I32, device=dev)
        self.pos = torch.zeros(B, dtype=I32, device=dev)
        self.pt = torch.zeros(B, max_pages, dtype=I32, device=dev)
        self.h = torch.zeros(B, d, dtype=I64, device=dev)
        self.q = torch.zeros(B, dl, dtype=I64, device=dev)
        self.bn = ops.fgemm_bn(B)
        self.epis = None
        rows = ops.limb_rows(B, self.bn)  # limb_row layout; the TMA box never exceeds the tensor
        self.Xd = torch.zeros(rows, d, dtype=I8, device=dev)
        self.Xo = torch.zeros(rows, dl, dtype=I8, device=dev)
        self.Xf = torch.zeros(rows, dffl, dtype=I8, device=dev)
        self.mXd = ops.TensorMap(self.Xd, self.bn, min(self.bn, 32))
        self.mXo = ops.TensorMap(self.Xo, self.bn, min(self.bn, 32))
        self.mXf = ops.TensorMap(self.Xf, self.bn, min(self.bn, 32))
        L0 = model.layers[0]
        mmax = max(L0.qkv.M, d, L0.gu.M, model.vocab_local)
        self.P = torch.zeros(8 * B * mmax, dtype=I32, device=dev)
        self.cnt = torch.zeros(4 * c.n_layers + 4, dtype=I32, device=dev)
        # per-norm sum of squares: [2 * n_layers + 1, B] (u64 bits in int64)
        self.ss = torch.zeros(2 * c.n_layers + 1, B, dtype=I64, device=dev)
        self.err = torch.zeros(1, dtype=I32, device=dev)
        self.logits_local = torch.zeros(B, model.vocab_local, dtype=I64, device=dev)
        self.logits = self.logits_local if model.tp_size == 1 else torch.zeros(B, c.vocab, dtype=I64, device=dev)
        # sampling state (one sampled slot per row)
        self.hist = torch.zeros(B, 64, dtype=I32, device=dev)
        self.count = torch.zeros(B, dtype=I32, device=dev)
        self.gen = torch.zeros(B, max(1, gen_cap), dtype=I32, device=dev)
        self.done = torch.zeros(B, dtype=I32, device=dev)
        self.eos = torch.zeros(8, dtype=I32, device=dev)
        self.n_eos = 0
        # per-M-tile arrival counters of the fused GEMM (zero between uses)
        self.tiles = torch.zeros(ops.tile_counters(mmax, B), dtype=I32, device=dev)


class Engine:
    def __init__(self, model: DenseModel, n_pages: Optional[int] = None, max_seq: Optional[int] = None,
                 comm: Optional[Comm] = None, kv_bytes: Optional[int] = None):
        self.m = model
        c = model.cfg
        self.comm = comm or Comm()
        self.max_seq = max_seq or c.max_seq
        self.max_pages = (self.max_seq + PAGE - 1) // PAGE
        if n_pages is None:
            per = PagedKV.bytes_per_page(c.n_layers, model.n_kv_local, c.d_head)
            budget = kv_bytes if kv_bytes is not None else 4 * self.max_pages * per
            n_pages = max(self.max_pages, budget // per)
        self.kv = PagedKV(c.n_layers, n_pages, model.n_kv_local, c.d_head, model.emb.device, self.max_pages)
        self._bufs: Dict[Tuple[int, int], StepBuffers] = {}
        self._graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self._rid = 0
        # NVTX ranges per layer and phase (ARCB_NVTX=1), for timeline profilers
        self.nvtx = bool(os.environ.get("ARCB_NVTX"))
        # optional op timeline of eager forwards: list of (label, CUDA event) appended after each op
        self.op_events = None
        # prefill chunks: one chunk-attention launch per layer (each K/V page
        # read once per 16 positions) instead of the per-position decode kernel
        self.prefill_attn = os.environ.get("ARCB_PREFILL_ATTN", "1") != "0"
        # decode steps of 8+ slots with grouped-query heads: one CTA per (slot,
        # KV head) serving its query heads
        self.gqa_block = os.environ.get("ARCB_GQA_BLOCK", "1") != "0"

    # ------------------------------------------------------------------ buffers
    def buffers(self, B: int, gen_cap: int = 0) -> StepBuffers:
        key = (B, gen_cap)
        if key not in self._bufs:
            self._bufs[key] = StepBuffers(self.m, B, self.max_pages, gen_cap)
        return self._bufs[key]

    # ------------------------------------------------------------------ forward
    def forward(self, bb: StepBuffers, B: int, with_logits: bool = True, span=None) -> None:
        """One forward over slots 0..B-1 of `bb` (tokens/pos/pt already set).
        span = (n, p0): slots [0, n) are positions p0.. of one sequence (page
        table row 0) and the rest padding; attention then runs as one
        chunk-attention launch that reads every K/V page once per 16
        positions (the same exact values as the per-position kernel)."""
        m, c, cm = self.m, self.m.cfg, self.comm
        d, dh = c.d_model, c.d_head
        nh, nkv = m.n_heads_local, m.n_kv_local
        dl, dffl = nh * dh, m.d_ff_local
        assert B == bb.B, "a StepBuffers instance serves exactly B slots (tensor maps are sized for it)"
        q16 = getattr(m, "emb_q16", None)
        if q16 is not None:
            ops.embed(bb.tokens, q16, None, c.vocab, d, B, bb.h, bb.cnt, bb.ss)
        else:
            ops.embed(bb.tokens, m.emb, m.emb_s, c.vocab, d, B, bb.h, bb.cnt, bb.ss)
        ss = bb.ss
        E = self._epis(bb)
        reduce_in_kernel = cm.size == 1 or getattr(cm, "fused", False)
        nv = torch.cuda.nvtx if self.nvtx else None
        ev = self.op_events

        def mark(label):
            if ev is not None:
                e_ = torch.cuda.Event(enable_timing=True)
                e_.record()
                ev.append((label, e_))

        mark("embed")
        for l, Ly in enumerate(m.layers):
            c0, c1, c2, c3 = (bb.cnt[4 * l + i:4 * l + i + 1] for i in range(4))
            e = E[l]
            if nv:
                nv.range_push(f"layer {l} attention")
            ops.norm_limbs(bb.h, ss[2 * l], Ly.attn_norm, d, B, bb.Xd, c0)
            mark("norm")
            ops.linear_gemm(Ly.qkv, bb.mXd, B, c0, bb.P, bb.tiles, e["qkv"])
            mark("qkv")
            T_all = self.max_pages * PAGE
            if span is not None:
                done = self.prefill_attn and ops.attn_prefill(bb.q, self.kv.K[l], self.kv.V[l], bb.pt[0], span[0],
                                                              span[1], nh, nkv, dh, m.attn_scale, B, bb.Xo, c1, T_all,
                                                              bb.err)
            else:
                # many decode slots with grouped-query heads: one CTA per (slot,
                # KV head) reads each page once for its query heads
                done = (self.gqa_block and nh // nkv >= 2 and nh // nkv <= 8 and B * nkv >= 64 and
                        ops.attn_gqa_block(bb.q, self.kv.K[l], self.kv.V[l], bb.pt, bb.pos, nh, nkv, dh, m.attn_scale,
                                           B, bb.Xo, c1, T_all, min(T_all, self.max_seq), bb.err))
            if not done:
                ops.attn(bb.q, self.kv.K[l], self.kv.V[l], bb.pt, bb.pos, nh, nkv, dh, m.attn_scale, B, bb.Xo, c1,
                         self.max_pages * PAGE, bb.err)
            mark("attn")
            if reduce_in_kernel:
                cm.fgemm_reduce(Ly.wo, bb.mXo, B, c1, bb, e["wo"], site=0)
            else:
                ops.linear_gemm(Ly.wo, bb.mXo, B, c1, bb.P, bb.tiles, e["partial"])
                cm.reduce_partials(bb.P, 8 * B, d, c1)
                ops.finalize(bb.P, d, B, c1, Ly.wo.s, bb.h, d, 1, ss[2 * l + 1])
            mark("wo")
            if nv:
                nv.range_pop()
                nv.range_push(f"layer {l} ffn")
            ops.norm_limbs(bb.h, ss[2 * l + 1], Ly.ffn_norm, d, B, bb.Xd, c2)
            mark("norm")
            ops.linear_gemm(Ly.gu, bb.mXd, B, c2, bb.P, bb.tiles, e["gu"])
            mark("gate_up")
            if reduce_in_kernel:
                cm.fgemm_reduce(Ly.down, bb.mXf, B, c3, bb, e["down"], site=1)
            else:
                ops.linear_gemm(Ly.down, bb.mXf, B, c3, bb.P, bb.tiles, e["partial"])
                cm.reduce_partials(bb.P, 8 * B, d, c3)
                ops.finalize(bb.P, d, B, c3, Ly.down.s, bb.h, d, 1, ss[2 * l + 2])
            mark("down")
            if nv:
                nv.range_pop()
        if with_logits:
            cf = bb.cnt[4 * c.n_layers:4 * c.n_layers + 1]
            ops.norm_limbs(bb.h, ss[2 * c.n_layers], m.final_norm, d, B, bb.Xd, cf)
            lm_e = cm.lm_epi(E[-1]["lm"], bb, c.vocab, m.vocab_offset) if hasattr(cm, "lm_epi") else E[-1]["lm"]
            ops.linear_gemm(m.lm, bb.mXd, B, cf, bb.P, bb.tiles, lm_e)
            cm.gather_logits(bb.logits_local, bb.logits, B, m.vocab_offset, bb=bb)
            mark("lm_head")

    def _epis(self, bb: StepBuffers):
        """Epilogue descriptors of every fused GEMM of a forward over `bb`."""
        if bb.epis is not None:
            return bb.epis
        m, c = self.m, self.m.cfg
        d, dh = c.d_model, c.d_head
        out = []
        for l, Ly in enumerate(m.layers):
            ss = bb.ss
            out.append({
                "qkv": ops.epi(ops.QKV, Ly.qkv.s, bb.err, n_heads=m.n_heads_local, n_kv=m.n_kv_local, dh=dh,
                               q_out=bb.q, Kc=self.kv.K[l], Vc=self.kv.V[l], pt=bb.pt, pt_stride=bb.pt.shape[1],
                               pos=bb.pos, rcos=m.rope_cos, rsin=m.rope_sin, max_seq=self.max_seq),
                "wo": ops.epi(ops.RESID, Ly.wo.s, bb.err, out=bb.h, ldo=d, ss_out=ss[2 * l + 1]),
                "gu": ops.epi(ops.SWIGLU, Ly.gu.s, bb.err, X=bb.Xf, ldx=m.d_ff_local,
                              lmax_out=bb.cnt[4 * l + 3:4 * l + 4]),
                "down": ops.epi(ops.RESID, Ly.down.s, bb.err, out=bb.h, ldo=d, ss_out=ss[2 * l + 2]),
                "partial": ops.epi(ops.PARTIAL, Ly.wo.s, bb.err),
            })
        out.append({"lm": ops.epi(ops.STORE, m.lm.s, bb.err, out=bb.logits_local, ldo=m.lm.M)})
        bb.epis = out
        return out

    def decode_step(self, bb: StepBuffers) -> None:
        """forward + sample for every slot; slots advance in place."""
        self.forward(bb, bb.B, True)
        ops.sample(bb.logits, self.m.cfg.vocab, bb.B, bb.hist, bb.count, bb.gen, bb.tokens, pos_inc=bb.pos,
                   done=bb.done, eos=bb.eos[:max(1, bb.n_eos)] if bb.n_eos else None)

    def capture(self, bb: StepBuffers) -> torch.cuda.CUDAGraph:
        """Capture one decode step of `bb` into a CUDA graph (after a warm-up
        step has run eagerly, so kernel attributes are already set)."""
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.decode_step(bb)
        torch.cuda.current_stream().wait_stream(s)
        return g

    # ------------------------------------------------------------------ requests
    def new_request(self, n_tokens: int) -> int:
        rid = self._rid
        self._rid += 1
        self.kv.reserve(rid, n_tokens)
        return rid

    @staticmethod
    def bucket(n: int) -> int:
        """Slot-count bucket for a prefill chunk (bounded set of buffers)."""
        b = 16
        while b < n:
            b *= 2
        return b

    @property
    def scratch_rid(self) -> int:
        """A one-page request that padding / idle slots write their KV into."""
        if getattr(self, "_scratch", None) is None:
            self._scratch = self.new_request(1)
        return self._scratch

    def prefill(self, rid: int, tokens: Sequence[int], start_pos: int = 0, chunk: int = 1024,
                logits_sink=None) -> None:
        """Write KV for `tokens` at positions start_pos.. .  Logits are
        discarded unless `logits_sink` is given: it then receives, chunk by
        chunk, the int64 Q16 logits [n, vocab] after each token (host copy).

        Chunks are padded to a power-of-two slot count; padding slots feed
        token 0 at position 0 of the scratch page, which no request reads."""
        row = self.kv.table_row(rid)
        srow = self.kv.table_row(self.scratch_rid)
        self._prefill_chunks(row, srow, tokens, start_pos, chunk, logits_sink)

    def _prefill_chunks(self, row, srow, tokens, start_pos, chunk, logits_sink) -> None:
        s = 0
        for n in self.prefill_chunks(len(tokens), chunk):
            part = [int(t) for t in tokens[s:s + n]]
            B = self.bucket(n)
            bb = self.buffers(B)
            pad = B - n
            bb.tokens.copy_(torch.tensor(part + [0] * pad, dtype=I32))
            bb.pos.copy_(torch.tensor(list(range(start_pos + s, start_pos + s + n)) + [0] * pad, dtype=I32))
            bb.pt.copy_(torch.tensor([row] * n + [srow] * pad, dtype=I32))
            self.forward(bb, B, with_logits=logits_sink is not None, span=(n, start_pos + s))
            if logits_sink is not None:
                logits_sink(bb.logits[:n].cpu().numpy())
            s += n

    @classmethod
    def prefill_chunks(cls, n: int, chunk: int = 1024) -> List[int]:
        """Chunk sizes for prefilling n tokens: full chunks, then the largest
        power of two that fits while more than 64 tokens remain, then the
        rest, so the power-of-two slot buckets pad little (600 tokens run as
        512 + 64 + 24 in buckets of 512, 64 and 32 slots, not as one
        1024-slot forward).  Any split gives the same exact KV."""
        out = []
        while n > 0:
            if n >= chunk:
                take = chunk
            elif n > 64 and cls.bucket(n) != n:
                take = 1 << (n.bit_length() - 1)
            else:
                take = n
            out.append(take)
            n -= take
        return out

    def score(self, tokens: Sequence[int], chunk: int = 256):
        """Q16 logits [len(tokens), vocab] after each of `tokens`, fed from
        position 0 as given (include the BOS yourself), as the reference's
        forward_one_token returns them one by one; for perplexity."""
        import numpy as np

        out = []
        rid = self.new_request(len(tokens) + 1)
        try:
            self.prefill(rid, tokens, chunk=chunk, logits_sink=out.append)
        finally:
            self.kv.release(rid)
        return np.concatenate(out) if out else np.zeros((0, self.m.cfg.vocab), np.int64)

    def generate(self, prompt: Sequence[int], max_tokens: int, eos: Sequence[int] = (),
                 use_graph: bool = True) -> Tuple[List[int], bytes]:
        """Single-stream greedy generate, bit-identical to the reference."""
        prompt = [int(t) for t in prompt]
        n = len(prompt)
        rid = self.new_request(1 + n + max_tokens)
        try:
            self.prefill(rid, [1] + prompt)
            toks = self._decode_loop(rid, prompt[-1] if n else 0, n + 1, max_tokens, eos, use_graph)
        finally:
            self.kv.release(rid)
        return toks, blake3(np.asarray(toks, dtype="<u4").tobytes())

    def stream_generate(self, prompt: Sequence[int], max_tokens: int, eos: Sequence[int] = ()):
        """Streaming generate (public API): yields each token as it is produced.

        Every decode step copies that step's input (token id, position) from
        pinned host memory to the device and reads the sampled id back into
        pinned host memory, so the caller sees tokens one at a time."""
        prompt = [int(t) for t in prompt]
        n = len(prompt)
        rid = self.new_request(1 + n + max_tokens)
        try:
            self.prefill(rid, [1] + prompt)
            bb = self.buffers(1, gen_cap=max(1, max_tokens))
            tok, pos = (prompt[-1] if n else 0), n + 1
            self._reset_sampling(bb, [rid], [tok], [pos], eos)
            g = self._graph_for(bb)
            pin_in = torch.empty(2, dtype=I32, pin_memory=True)
            pin_out = torch.empty(1, dtype=I32, pin_memory=True)
            eos_set = set(int(e) for e in eos)
            st = torch.cuda.current_stream()
            for _ in range(max_tokens):
                pin_in[0], pin_in[1] = tok, pos
                bb.tokens.copy_(pin_in[0:1], non_blocking=True)
                bb.pos.copy_(pin_in[1:2], non_blocking=True)
                g.replay()
                pin_out.copy_(bb.tokens, non_blocking=True)
                st.synchronize()
                tok = int(pin_out[0])
                pos += 1
                yield tok
                if tok in eos_set:
                    break
        finally:
            self.kv.release(rid)

    # bytes moved between host and device by each stream_generate step
    STREAM_H2D_BYTES = 8
    STREAM_D2H_BYTES = 4

    def _decode_loop(self, rid, first_tok, first_pos, max_tokens, eos, use_graph) -> List[int]:
        bb = self.buffers(1, gen_cap=max(1, max_tokens))
        self._reset_sampling(bb, [rid], [first_tok], [first_pos], eos)
        if max_tokens <= 0:
            return []
        if use_graph:
            g = self._graph_for(bb)
            for _ in range(max_tokens):
                g.replay()
        else:
            for _ in range(max_tokens):
                self.decode_step(bb)
        cnt = int(bb.count[0].item())
        return [int(t) for t in bb.gen[0, :cnt].tolist()]

    def _reset_sampling(self, bb: StepBuffers, rids, first_toks, first_pos, eos) -> None:
        B = bb.B
        bb.tokens.copy_(torch.tensor(first_toks, dtype=I32))
        bb.pos.copy_(torch.tensor(first_pos, dtype=I32))
        bb.pt.copy_(torch.tensor([self.kv.table_row(r) for r in rids], dtype=I32))
        bb.hist.zero_()
        bb.count.zero_()
        bb.done.zero_()
        eos = list(eos)[:8]
        bb.n_eos = len(eos)
        if eos:
            bb.eos[:len(eos)].copy_(torch.tensor(eos, dtype=I32))

    def _graph_for(self, bb: StepBuffers) -> torch.cuda.CUDAGraph:
        key = (id(bb), bb.n_eos)
        if key not in self._graphs:
            # warm-up: one eager step on a scratch copy of the state, then restore
            saved = [t.clone() for t in (bb.tokens, bb.pos, bb.hist, bb.count, bb.done, bb.gen)]
            self.decode_step(bb)
            torch.cuda.synchronize()
            for t, s in zip((bb.tokens, bb.pos, bb.hist, bb.count, bb.done, bb.gen), saved):
                t.copy_(s)
            self._graphs[key] = self.capture(bb)
        return self._graphs[key]

    def check_errors(self) -> int:
        e = 0
        for bb in self._bufs.values():
            e |= int(bb.err.item())
        return e
