"""HTTP serving API with the reference's request/attestation shape.

Routes (the reference's node RPC, crates/arc-node/src/rpc.rs:140-240,
2674-2847): ``POST /inference/run`` {"input": text, "max_tokens": n}
tokenises the text with the model vocab, generates greedily with EOS {2, 0}
(the RPC's choice), and returns ms/token plus the attestation triple (model
id hash, input hash, output hash); ``GET /inference/attestations`` lists the
attestations produced so far; ``GET /health`` and ``GET /stats``.

On a GPU the requests go through the continuous-batching scheduler (one
background thread steps it); ``--cpu-oracle`` serves from the C++ oracle
instead (explicitly, for machines without a GPU).

    python -m arc_chain_b200.runtime.server --model tiny --port 8080
"""
from __future__ import annotations

import argparse
import threading
import time
from typing import List, Optional

from arc_chain_b200.formats.tokenizer import Tokenizer
from arc_chain_b200.runtime import attest

RPC_EOS = (2, 0)


class OracleBackend:
    """Serves from the CPU oracle (no GPU)."""

    name = "INT8 integer, CPU oracle"

    def __init__(self, host_model):
        from arc_chain_b200.oracle import arcref

        self.cfg = host_model.cfg
        self.m = arcref.Model(host_model)

    def generate(self, prompt, max_tokens, eos=RPC_EOS):
        return self.m.generate(prompt, max_tokens, eos)[0]


class BackendError(RuntimeError):
    """The serving backend failed; the request was not completed."""


class SchedulerBackend:
    """Serves from the GPU engine through the continuous-batching scheduler.

    One daemon thread steps the scheduler while requests are queued or
    running; callers wait on a condition variable.  If a step raises (a
    CUDA error, a failure while admitting or decoding), the loop records the
    exception, stops, and wakes every caller: requests in flight and any
    later request raise :class:`BackendError` instead of waiting forever."""

    name = "INT8 integer, B200 (sm_100a), continuous batching"

    def __init__(self, engine=None, max_batch: int = 16, gen_cap: int = 512, sched=None):
        if sched is None:
            from arc_chain_b200.runtime.scheduler import Scheduler

            sched = Scheduler(engine, max_batch=max_batch, eos=RPC_EOS, gen_cap=gen_cap)
        self.cfg = engine.m.cfg if engine is not None else getattr(sched, "cfg", None)
        self.sched = sched
        self.cv = threading.Condition()
        self.stop = False
        self.error: Optional[BaseException] = None
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def _loop(self):
        while not self.stop:
            with self.cv:
                busy = bool(self.sched.waiting) or any(x is not None for x in self.sched.lanes)
                if not busy:
                    self.cv.wait(timeout=0.05)
                    continue
                try:
                    self.sched.step()
                except BaseException as e:  # the thread must not die silently
                    self.error = e
                    self.stop = True
                    self.cv.notify_all()
                    return
                self.cv.notify_all()

    def _raise(self):
        raise BackendError(f"serving backend failed: {self.error!r}") from self.error

    def generate(self, prompt, max_tokens, eos=RPC_EOS):
        with self.cv:
            if self.error is not None:
                self._raise()
            rid = self.sched.submit(prompt, max_tokens)
            self.cv.notify_all()
            while not self.sched.requests[rid].done:
                if self.error is not None:
                    self.sched.requests.pop(rid, None)
                    self._raise()
                self.cv.wait(timeout=0.1)
            return self.sched.requests.pop(rid).tokens

    def close(self):
        with self.cv:
            self.stop = True
            self.cv.notify_all()
        self.t.join(timeout=5)


class Service:
    def __init__(self, backend, vocab: List[str], weight_hash: Optional[bytes] = None):
        self.b = backend
        self.tok = Tokenizer(vocab)
        self.weight_hash = weight_hash
        self.attestations: List[dict] = []
        # the HTTP layer runs requests on a thread pool: the counters and the
        # attestation list are updated under this lock
        self._mu = threading.Lock()
        self.n_requests = 0
        self.total_tokens = 0
        self.total_ms = 0.0

    def run(self, text: str, max_tokens: int = 64) -> dict:
        t0 = time.perf_counter()
        prompt = self.tok.encode(text)
        t1 = time.perf_counter()
        toks = self.b.generate(prompt, int(max_tokens))
        t2 = time.perf_counter()
        out = attest.inference_result(self.b.cfg, text, prompt, toks, self.tok.decode(toks), (t2 - t1) * 1000,
                                      (t1 - t0) * 1000, self.b.name)
        a = attest.attest(self.b.cfg, text, toks, self.weight_hash).body()
        out["attestation"] = a
        with self._mu:
            self.attestations.append(a)
            self.n_requests += 1
            self.total_tokens += len(toks)
            self.total_ms += (t2 - t1) * 1000
        return out

    def stats(self) -> dict:
        with self._mu:
            return {"requests": self.n_requests, "tokens": self.total_tokens,
                    "avg_ms_per_token": self.total_ms / self.total_tokens if self.total_tokens else 0.0,
                    "model": attest.model_id_string(self.b.cfg)}


def make_app(svc: Service):
    from fastapi import FastAPI
    from pydantic import BaseModel

    app = FastAPI(title="arc_chain_b200")

    class RunReq(BaseModel):
        input: str
        max_tokens: int = 64

    @app.post("/inference/run")
    def run(r: RunReq):
        return svc.run(r.input, r.max_tokens)

    @app.get("/inference/attestations")
    def atts():
        return {"attestations": svc.attestations}

    @app.get("/health")
    def health():
        return {"status": "ok"}

    @app.get("/stats")
    def stats():
        return svc.stats()

    return app


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", help="preset name or an .arc-int8 path")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--cpu-oracle", action="store_true")
    a = ap.parse_args()
    from arc_chain_b200.formats import arc_int8, gen
    from arc_chain_b200.models.config import PRESETS

    host = gen.random_model(PRESETS[a.model], a.seed) if a.model in PRESETS else arc_int8.load(a.model)
    if a.cpu_oracle:
        backend = OracleBackend(host)
    else:
        from arc_chain_b200.models import dense
        from arc_chain_b200.runtime.engine import Engine

        backend = SchedulerBackend(Engine(dense.from_host(host, "cuda")))
    svc = Service(backend, host.vocab, host.weight_hash())
    import uvicorn

    uvicorn.run(make_app(svc), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
