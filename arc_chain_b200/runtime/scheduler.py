"""Continuous-batching scheduler over the paged KV cache.

The reference serves one request at a time (single-stream ``generate``,
crates/arc-inference/src/cached_integer_model.rs:1518-1557); batching is an
extension defined so that every request's output is bit-identical to its
own single-stream run: each token's computation reads only its own
request's KV pages, and every reduction is an exact integer sum, so sharing
a GEMM with other requests changes nothing.

Layout: the decode step has ``max_batch`` fixed *lanes* (one CUDA graph per
lane count).  A request holds a lane from the end of its prefill to its last
token; idle lanes are masked (``done`` = 1) and point at a scratch page, so
the graph never changes shape.  Waiting requests are admitted when a lane
and enough KV pages are free; their BOS + prompt is prefilled in chunks of
at most ``prefill_chunk`` tokens between decode steps (logits discarded, as
in the reference), then the lane starts decoding with the last prompt token
fed again at position n + 1.  A request finishes on an EOS id (kept in the
output) or after ``max_tokens`` tokens; its output hash is BLAKE3 of the LE
u32 ids, as the reference computes it.

Resume and recovery are exact.  A request that has produced g tokens is
rebuilt by prefilling BOS + prompt + [last prompt token] + its first g - 1
tokens (exactly the positions its decode steps wrote) and restoring the
penalty history and count, so it continues as if never interrupted.
``snapshot`` / ``from_snapshot`` persist and restore serving state this way
(the KV cache itself is never saved), and a decode step whose kernels raised
an error bit requeues every active request without that step's tokens.
"""
from __future__ import annotations

import collections
import json
import time
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence

import numpy as np
import torch

from arc_chain_b200.runtime.engine import Engine, I32
from arc_chain_b200.runtime.kv_paged import PAGE, PagedKV
from arc_chain_b200.utils.hashing import blake3


@dataclass
class Request:
    rid: int
    prompt: List[int]
    max_tokens: int
    lane: int = -1
    tokens: List[int] = field(default_factory=list)
    output_hash: Optional[bytes] = None
    t_submit: float = 0.0
    t_first: float = 0.0
    t_done: float = 0.0
    resume: List[int] = field(default_factory=list)  # tokens already produced (resumed requests)

    @property
    def done(self) -> bool:
        return self.output_hash is not None


def check_fits(kv: PagedKV, held: int, n_prompt: int, max_tokens: int) -> None:
    """Raises ValueError for a request that no amount of waiting would admit:
    its 1 + prompt + max_tokens positions need more pages than one sequence
    may hold (the engine's max_seq), or more than the pool has besides the
    `held` pages that stay reserved (the idle lanes' scratch page).  Such a
    request would otherwise wait at the head of the queue for good."""
    need = (1 + n_prompt + max_tokens + PAGE - 1) // PAGE
    if need > kv.max_pages_per_seq:
        raise ValueError(f"request of {n_prompt} prompt + {max_tokens} new tokens needs {need} KV pages; "
                         f"a sequence holds at most {kv.max_pages_per_seq}")
    if need > kv.n_pages - held:
        raise ValueError(f"request needs {need} KV pages; the cache has {kv.n_pages - held} besides "
                         f"the {held} it keeps reserved")


class Scheduler:
    def __init__(self, engine: Engine, max_batch: int = 32, prefill_chunk: int = 1024,
                 eos: Sequence[int] = (), gen_cap: Optional[int] = None, use_graph: bool = True,
                 metrics_sink: Optional[Callable[[dict], None]] = None, keep_metrics: int = 10000):
        if getattr(engine, "dispatch", False):
            # token-dispatch expert parallelism needs every rank in lockstep
            raise ValueError("the continuous-batching scheduler needs a replicated-token communicator "
                             "(EpFusedComm / EpNcclComm), not EpDispatchComm")
        self.e = engine
        self.max_batch = max_batch
        self.prefill_chunk = prefill_chunk
        self.eos = [int(x) for x in eos]
        self.gen_cap = gen_cap or engine.max_seq
        self.use_graph = use_graph
        self.waiting: Deque[Request] = collections.deque()
        self.requests: Dict[int, Request] = {}
        self.lanes: List[Optional[Request]] = [None] * max_batch
        self.bb = engine.buffers(max_batch, gen_cap=self.gen_cap)
        self._scratch_rid = engine.scratch_rid  # page for idle lanes
        self._init_lanes()
        self.steps = 0
        self.tokens_out = 0
        # per-step metrics: the last keep_metrics records, and every record
        # to metrics_sink (e.g. a JSON-lines writer) when given
        self.metrics: Deque[dict] = collections.deque(maxlen=keep_metrics)
        self.metrics_sink = metrics_sink
        self.finished = 0
        self._t0 = None
        self.recoveries = 0
        self.max_recoveries = 3

    # ------------------------------------------------------------ lanes
    def _init_lanes(self):
        bb = self.bb
        row = torch.tensor(self.e.kv.table_row(self._scratch_rid), dtype=I32)
        bb.pt.copy_(row.unsqueeze(0).expand(self.max_batch, -1))
        bb.tokens.zero_()
        bb.pos.zero_()
        bb.hist.zero_()
        bb.count.zero_()
        bb.done.fill_(1)
        bb.n_eos = len(self.eos[:8])
        if bb.n_eos:
            bb.eos[:bb.n_eos].copy_(torch.tensor(self.eos[:8], dtype=I32))

    def _open_lane(self, lane: int, r: Request):
        bb = self.bb
        n = len(r.prompt)
        g = len(r.resume)
        bb.pt[lane].copy_(torch.tensor(self.e.kv.table_row(r.rid), dtype=I32))
        bb.hist[lane].zero_()
        if g:
            bb.tokens[lane] = r.resume[-1]
            bb.pos[lane] = n + g + 1
            hist = torch.zeros(64, dtype=I32)
            for j in range(max(0, g - 64), g):
                hist[j & 63] = r.resume[j]
            bb.hist[lane].copy_(hist)
            bb.gen[lane, :g].copy_(torch.tensor(r.resume, dtype=I32))
        else:
            bb.tokens[lane] = r.prompt[-1] if n else 0
            bb.pos[lane] = n + 1
        bb.count[lane] = g
        bb.done[lane] = 0
        r.lane = lane
        self.lanes[lane] = r

    def _close_lane(self, lane: int):
        bb = self.bb
        bb.done[lane] = 1
        bb.pt[lane].copy_(torch.tensor(self.e.kv.table_row(self._scratch_rid), dtype=I32))
        bb.pos[lane] = 0
        bb.tokens[lane] = 0
        self.lanes[lane] = None

    # ------------------------------------------------------------ API
    def _check_fits(self, n_prompt: int, max_tokens: int) -> None:
        if max_tokens > self.gen_cap:
            raise ValueError(f"max_tokens {max_tokens} > gen_cap {self.gen_cap}")
        check_fits(self.e.kv, len(self.e.kv.tables.get(self._scratch_rid, [])), n_prompt, max_tokens)

    def submit(self, prompt: Sequence[int], max_tokens: int) -> int:
        self._check_fits(len(prompt), int(max_tokens))
        rid = self.e._rid
        self.e._rid += 1
        r = Request(rid, [int(t) for t in prompt], int(max_tokens), t_submit=time.perf_counter())
        self.requests[rid] = r
        self.waiting.append(r)
        return rid

    def _admit(self) -> int:
        admitted = 0
        for lane in range(self.max_batch):
            if self.lanes[lane] is not None or not self.waiting:
                continue
            r = self.waiting[0]
            need = 1 + len(r.prompt) + r.max_tokens
            if (need + 15) // 16 > len(self.e.kv.pool.free):
                break
            self.waiting.popleft()
            self.e.kv.reserve(r.rid, need)
            toks = [1] + r.prompt
            if r.resume:
                toks += [r.prompt[-1] if r.prompt else 0] + r.resume[:-1]
            self.e.prefill(r.rid, toks, chunk=self.prefill_chunk)
            self._open_lane(lane, r)
            admitted += 1
        return admitted

    def step(self) -> int:
        """Admit, then one decode step over all lanes; returns active lanes."""
        t0 = time.perf_counter()
        if self._t0 is None:
            self._t0 = t0
        ev = getattr(self, "phase_events", None)
        if ev is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        admitted = self._admit()
        if ev is not None and admitted:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
            ev.append(("prefill", e0, e1))
        active = sum(1 for x in self.lanes if x is not None)
        if active == 0:
            return 0
        fin0 = self.finished
        if ev is not None:
            d0 = torch.cuda.Event(enable_timing=True)
            d0.record()
        try:
            return self._decode(active)
        finally:
            if ev is not None:
                d1 = torch.cuda.Event(enable_timing=True)
                d1.record()
                ev.append(("decode", d0, d1))
            self._record(t0, admitted, active, self.finished - fin0)

    def phase_times_ms(self) -> dict:
        """Device time (CUDA events) spent in prefill (admission) and in decode
        steps, when ``phase_events`` was set to a list before running."""
        out = {"prefill": 0.0, "decode": 0.0}
        torch.cuda.synchronize()
        for kind, a, b in getattr(self, "phase_events", None) or []:
            out[kind] += a.elapsed_time(b)
        return {k: round(v, 2) for k, v in out.items()}

    def _record(self, t0: float, admitted: int, active: int, finished: int) -> None:
        pool = self.e.kv.pool
        m = {"step": self.steps, "active_lanes": active, "admitted": admitted, "finished": finished,
             "waiting": len(self.waiting), "tokens_out": self.tokens_out, "kv_pages_used": pool.used,
             "kv_pages_free": len(pool.free), "step_ms": round((time.perf_counter() - t0) * 1000, 3),
             "recoveries": self.recoveries}
        self.metrics.append(m)
        if self.metrics_sink is not None:
            self.metrics_sink(m)

    def stats(self) -> dict:
        """Totals since the first step (host clock)."""
        el = time.perf_counter() - self._t0 if self._t0 else 0.0
        return {"steps": self.steps, "tokens_out": self.tokens_out, "finished": self.finished,
                "waiting": len(self.waiting), "active_lanes": sum(1 for x in self.lanes if x is not None),
                "kv_pages_used": self.e.kv.pool.used, "recoveries": self.recoveries, "seconds": round(el, 3),
                "tokens_per_s": round(self.tokens_out / el, 2) if el > 0 else 0.0}

    def _decode(self, active: int) -> int:
        before = self.bb.count.cpu().numpy().copy()
        if self.use_graph:
            self.e._graph_for(self.bb).replay()
        else:
            self.e.decode_step(self.bb)
        self.steps += 1
        if int(self.bb.err.item()) != 0:
            self._recover(before)
            return active
        cnt = self.bb.count.cpu().numpy()
        done = self.bb.done.cpu().numpy()
        for lane, r in enumerate(self.lanes):
            if r is None:
                continue
            if r.t_first == 0.0 and cnt[lane] > 0:
                r.t_first = time.perf_counter()
            if done[lane] or cnt[lane] >= r.max_tokens:
                self._finish(lane, r, int(min(cnt[lane], r.max_tokens)))
        self.tokens_out += active
        return active

    def _finish(self, lane: int, r: Request, n: int):
        r.tokens = [int(t) for t in self.bb.gen[lane, :n].tolist()]
        r.output_hash = blake3(np.asarray(r.tokens, dtype="<u4").tobytes())
        r.t_done = time.perf_counter()
        self.e.kv.release(r.rid)
        self._close_lane(lane)
        self.finished += 1

    # ------------------------------------------------------------ recovery and resume
    def _recover(self, counts_before) -> None:
        """A step raised a kernel error bit: requeue every active request with
        the tokens it had before that step, then clear the error."""
        torch.cuda.synchronize()
        if self.recoveries >= self.max_recoveries:
            raise RuntimeError(f"decode step failed again after {self.recoveries} recoveries "
                               f"(error bits {int(self.bb.err.item()):#x})")
        gen = self.bb.gen.cpu()
        requeue = []
        for lane, r in enumerate(self.lanes):
            if r is None:
                continue
            g = int(min(counts_before[lane], r.max_tokens))
            r.resume = [int(t) for t in gen[lane, :g].tolist()]
            self.e.kv.release(r.rid)
            self._close_lane(lane)
            requeue.append(r)
        for r in reversed(requeue):
            self.waiting.appendleft(r)
        for bb in self.e._bufs.values():
            bb.err.zero_()
        self.recoveries += 1

    def snapshot(self) -> str:
        """Serving state as JSON (between steps): every request's prompt,
        budget and tokens so far; finished requests keep their hash."""
        cnt = self.bb.count.cpu().numpy()
        gen = self.bb.gen.cpu()
        reqs = []
        for rid, r in sorted(self.requests.items()):
            if r.done:
                toks = r.tokens
            elif r.lane >= 0 and self.lanes[r.lane] is r:
                toks = [int(t) for t in gen[r.lane, :int(min(cnt[r.lane], r.max_tokens))].tolist()]
            else:
                toks = list(r.resume)
            reqs.append({"rid": rid, "prompt": r.prompt, "max_tokens": r.max_tokens, "tokens": toks,
                         "done": r.done, "output_hash": r.output_hash.hex() if r.done else None})
        return json.dumps({"version": 1, "eos": self.eos, "requests": reqs})

    @classmethod
    def from_snapshot(cls, engine: Engine, snap: str, max_batch: int = 32, prefill_chunk: int = 1024,
                      gen_cap: Optional[int] = None, use_graph: bool = True) -> "Scheduler":
        d = json.loads(snap)
        sch = cls(engine, max_batch, prefill_chunk, eos=d["eos"], gen_cap=gen_cap, use_graph=use_graph)
        for q in d["requests"]:
            rid = engine._rid
            engine._rid += 1
            r = Request(rid, list(q["prompt"]), int(q["max_tokens"]), t_submit=time.perf_counter())
            if q["done"]:
                r.tokens = list(q["tokens"])
                r.output_hash = bytes.fromhex(q["output_hash"])
            else:
                sch._check_fits(len(r.prompt), r.max_tokens)
                r.resume = list(q["tokens"])
                sch.waiting.append(r)
            sch.requests[rid] = r
        return sch

    def run(self, max_steps: Optional[int] = None) -> Dict[int, Request]:
        s = 0
        while self.waiting or any(x is not None for x in self.lanes):
            self.step()
            s += 1
            if max_steps is not None and s >= max_steps:
                break
        return self.requests
