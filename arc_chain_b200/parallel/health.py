"""Failure detection for multi-rank serving, on the host.

The reference detects failures at the protocol level (request timeouts,
rpc.rs:2712-2725; consensus proposer timeouts and view change, arc-consensus
lib.rs:1867-1911; committee disagreement, committee.rs:45-56).  Here the
ranks of one tensor-parallel group each publish a heartbeat (step number
and wall time) to the torch.distributed store between steps; before every
step each rank checks that all peers have advanced within ``timeout_s``.  A
rank that raised, exited or hung is reported as :class:`RankFailure` before
anyone launches a collective or a kernel that would wait on it.  Kernels
that wait on peers have their own bounded waits (they set
ARCB_ERR_COMM_TIMEOUT instead of spinning), and the process group carries a
short timeout as the last bound.

Recovery is request-level and exact: outputs are a pure function of
(weights, prompt), so a failed request is re-queued and re-prefilled from its
prompt and its confirmed tokens (:func:`replay_request`).
"""
from __future__ import annotations

import json
import time
from typing import List, Optional, Sequence


class RankFailure(RuntimeError):
    def __init__(self, ranks: Sequence[int], why: str):
        super().__init__(f"ranks {list(ranks)} failed: {why}")
        self.ranks = list(ranks)
        self.why = why


class Heartbeat:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "arcb_hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = timeout_s
        self.prefix = prefix
        self.step = -1

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int, status: str = "ok") -> None:
        self.step = step
        self.store.set(self._key(self.rank), json.dumps({"step": step, "t": time.time(), "status": status}))

    def fail(self, why: str) -> None:
        """Announce a local failure so peers stop waiting for this rank."""
        self.store.set(self._key(self.rank), json.dumps({"step": self.step, "t": time.time(), "status": "failed",
                                                         "why": why}))

    def read(self, r: int) -> Optional[dict]:
        try:
            if not self.store.check([self._key(r)]):
                return None
            return json.loads(self.store.get(self._key(r)).decode())
        except Exception:
            return None

    def wait_peers(self, step: int, poll_s: float = 0.01) -> None:
        """Block until every rank has published `step` (bounded by timeout_s);
        raise RankFailure naming the ranks that did not."""
        t0 = time.time()
        while True:
            missing, failed = [], []
            for r in range(self.world):
                hb = self.read(r)
                if hb is not None and hb.get("status") == "failed":
                    failed.append((r, hb.get("why", "")))
                elif hb is None or hb["step"] < step:
                    missing.append(r)
            if failed:
                raise RankFailure([r for r, _ in failed], "; ".join(w for _, w in failed))
            if not missing:
                return
            if time.time() - t0 > self.timeout_s:
                raise RankFailure(missing, f"no heartbeat for step {step} within {self.timeout_s}s")
            time.sleep(poll_s)


def replay_request(engine, prompt: Sequence[int], confirmed: Sequence[int], max_tokens: int, eos=()) -> List[int]:
    """Resume a request after a failure: re-prefill BOS + prompt + the last
    prompt token and every confirmed token, then continue decoding.  The
    integer engine is deterministic, so the continuation equals the
    uninterrupted run."""
    toks, _ = engine.generate(list(prompt), max_tokens, eos)
    assert toks[:len(confirmed)] == list(confirmed), "confirmed prefix must reproduce exactly"
    return toks
