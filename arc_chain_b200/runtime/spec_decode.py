"""Greedy speculative decoding with a draft model, bit-identical to plain
greedy decoding of the target.

The reference has no speculative decoding; this follows its greedy step
exactly (crates/arc-inference/src/cached_integer_model.rs:1518-1557).  Each
round, per lane (request):

1. the draft model, fed the lane's last confirmed token at its position,
   proposes k tokens greedily, with the repetition penalty over the lane's
   confirmed tokens followed by its own proposals;
2. the target model scores [last, d_1..d_k] at positions pos..pos+k in one
   forward (k+1 slots per lane, exact integer math, so each slot's logits
   equal a sequential decode's), and ``verify_sample`` takes the penalised
   argmax y_i of slot i with history = confirmed + d_1..d_i;
3. the longest prefix with y_i == d_{i+1} is accepted and y_j is appended as
   the correction (or bonus) token, so every emitted token is exactly the
   token plain greedy decoding would emit.  EOS (kept) and max_tokens cut the
   round short.

KV for rejected positions is simply overwritten by later rounds (positions
restart at the first unconfirmed one).  When every draft token is accepted
the draft never consumed d_k, so it is fed d_k first in the next round.
With tensor parallelism the draft runs on rank 0 only and its proposals are
broadcast; every rank verifies.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.runtime.engine import Engine, I32
from arc_chain_b200.utils.hashing import blake3


@dataclass
class _Lane:
    rid_t: int
    rid_d: int
    prompt: List[int]
    max_tokens: int
    gen: List[int] = field(default_factory=list)
    last: int = 0
    pos: int = 0
    pending: List[int] = field(default_factory=list)  # tokens the draft has not consumed
    done: bool = False


class SpecDecoder:
    def __init__(self, target: Engine, draft: Optional[Engine], k: int = 4, lanes: int = 1, gen_cap: int = 1024,
                 use_graph: bool = True):
        self.t, self.d, self.k, self.n = target, draft, k, lanes
        self.use_graph = use_graph
        self.cm = target.comm
        self.runs_draft = draft is not None and self.cm.rank == 0
        dev = target.m.emb.device
        self.tb = target.buffers(lanes * (k + 1))
        self.db = draft.buffers(lanes, gen_cap=gen_cap + k + 2) if self.runs_draft else None
        self.drafts = torch.zeros(lanes, k, dtype=I32, device=dev)
        self.hist = torch.zeros(lanes, 64, dtype=I32, device=dev)
        self.count = torch.zeros(lanes, dtype=I32, device=dev)
        self.y = torch.zeros(lanes * (k + 1), dtype=I32, device=dev)
        self._vgraph = None
        self.rounds = 0
        self.proposed = 0
        self.accepted = 0

    # -------------------------------------------------------------- helpers
    def _ring(self, gen: List[int]):
        ring = [0] * 64
        for i in range(max(0, len(gen) - 64), len(gen)):
            ring[i & 63] = gen[i]
        return ring

    def _verify(self):
        c = self.t.m.cfg
        B = self.tb.B
        self.t.forward(self.tb, B, True)
        ops.verify_sample(self.tb.logits, c.vocab, self.n, self.k, self.drafts, self.hist, self.count, self.y)

    def _verify_graph(self):
        if self._vgraph is None:
            self._verify()  # warm-up (sets kernel attributes); its KV writes are rewritten later
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    self._verify()
            torch.cuda.current_stream().wait_stream(s)
            self._vgraph = g
        return self._vgraph

    # -------------------------------------------------------------- rounds
    def _draft_round(self, lanes: List[_Lane]):
        d, db, k = self.d, self.db, self.k
        for i, ln in enumerate(lanes):
            if not ln.done and ln.pending:
                d.prefill(ln.rid_d, ln.pending, start_pos=ln.pos - len(ln.pending))
                ln.pending = []
        srow = d.kv.table_row(d.scratch_rid)
        db.tokens.copy_(torch.tensor([ln.last if not ln.done else 0 for ln in lanes], dtype=I32))
        db.pos.copy_(torch.tensor([ln.pos if not ln.done else 0 for ln in lanes], dtype=I32))
        db.pt.copy_(torch.tensor([d.kv.table_row(ln.rid_d) if not ln.done else srow for ln in lanes], dtype=I32))
        db.hist.copy_(torch.tensor([self._ring(ln.gen) for ln in lanes], dtype=I32))
        db.count.copy_(torch.tensor([len(ln.gen) for ln in lanes], dtype=I32))
        db.done.copy_(torch.tensor([1 if ln.done else 0 for ln in lanes], dtype=I32))
        g = d._graph_for(db) if self.use_graph else None
        for _ in range(k):
            if g is not None:
                g.replay()
            else:
                d.decode_step(db)
        for i, ln in enumerate(lanes):
            c0 = len(ln.gen)
            self.drafts[i].copy_(db.gen[i, c0:c0 + k])

    def _round(self, lanes: List[_Lane]):
        t, k = self.t, self.k
        if self.runs_draft:
            self._draft_round(lanes)
        if self.cm.size > 1:
            import torch.distributed as dist

            dist.broadcast(self.drafts, src=0)
        drafts = self.drafts.cpu().numpy()
        srow = t.kv.table_row(t.scratch_rid)
        toks, pos, pts = [], [], []
        for i, ln in enumerate(lanes):
            if ln.done:
                toks += [0] * (k + 1)
                pos += [0] * (k + 1)
                pts += [srow] * (k + 1)
            else:
                toks += [ln.last] + [int(x) for x in drafts[i]]
                pos += list(range(ln.pos, ln.pos + k + 1))
                pts += [t.kv.table_row(ln.rid_t)] * (k + 1)
        tb = self.tb
        tb.tokens.copy_(torch.tensor(toks, dtype=I32))
        tb.pos.copy_(torch.tensor(pos, dtype=I32))
        tb.pt.copy_(torch.tensor(pts, dtype=I32))
        self.hist.copy_(torch.tensor([self._ring(ln.gen) for ln in lanes], dtype=I32))
        self.count.copy_(torch.tensor([len(ln.gen) for ln in lanes], dtype=I32))
        if self.use_graph:
            self._verify_graph().replay()
        else:
            self._verify()
        y = self.y.cpu().numpy().reshape(self.n, k + 1)
        self.rounds += 1
        for i, ln in enumerate(lanes):
            if ln.done:
                continue
            j = 0
            while j < k and y[i, j] == drafts[i, j]:
                j += 1
            self.proposed += k
            self.accepted += j
            new = [int(v) for v in y[i, :j + 1]]
            emitted = 0
            for tok in new:
                ln.gen.append(tok)
                emitted += 1
                if tok in self.eos or len(ln.gen) >= ln.max_tokens:
                    ln.done = True
                    break
            if not ln.done:
                ln.pending = [int(drafts[i, k - 1])] if j == k else []
                ln.last = new[-1]
                ln.pos += j + 1

    # -------------------------------------------------------------- API
    def generate(self, prompts: Sequence[Sequence[int]], max_tokens: int, eos: Sequence[int] = ()) \
            -> List[Tuple[List[int], bytes]]:
        assert len(prompts) == self.n, "one prompt per lane"
        self.eos = set(int(e) for e in eos)
        lanes = []
        for p in prompts:
            p = [int(x) for x in p]
            need = 1 + len(p) + max_tokens + self.k + 1
            rid_t = self.t.new_request(need)
            self.t.prefill(rid_t, [1] + p)
            rid_d = -1
            if self.runs_draft:
                rid_d = self.d.new_request(need)
                self.d.prefill(rid_d, [1] + p)
            lanes.append(_Lane(rid_t, rid_d, p, max_tokens, last=p[-1] if p else 0, pos=len(p) + 1))
        try:
            while not all(ln.done for ln in lanes):
                self._round(lanes)
        finally:
            for ln in lanes:
                self.t.kv.release(ln.rid_t)
                if self.runs_draft:
                    self.d.kv.release(ln.rid_d)
        return [(ln.gen, blake3(np.asarray(ln.gen, dtype="<u4").tobytes())) for ln in lanes]

    @property
    def acceptance(self) -> float:
        return self.accepted / max(1, self.proposed)
