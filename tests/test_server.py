"""The serving API's request flow and result shape (CPU oracle backend)."""
from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.runtime import attest, server
from arc_chain_b200 import spec


def test_service_run_and_attestation():
    host = gen.random_model(preset("micro"), 0)
    host.vocab = ["<unk>", "<s>", "</s>", "▁"] + [f"▁w{i}" for i in range(host.cfg.vocab - 4)]
    svc = server.Service(server.OracleBackend(host), host.vocab, host.weight_hash())
    r = svc.run("w5 w7 w9", 6)
    inf = r["inference"]
    assert inf["input_tokens"] == 3 and inf["deterministic"] is True
    assert inf["output_hash"] == "0x" + spec.tokens_hash(inf["output_tokens"]).hex()
    assert inf["input_hash"] == "0x" + attest.input_hash("w5 w7 w9").hex()
    assert r["attestation"]["weight_hash"] == "0x" + host.weight_hash().hex()
    assert svc.stats()["requests"] == 1
    # the same request gives the same attestation (determinism)
    assert svc.run("w5 w7 w9", 6)["attestation"] == r["attestation"]
    app = server.make_app(svc)
    assert {"/inference/run", "/health", "/stats", "/inference/attestations"} <= {x.path for x in app.routes}


def test_concurrent_requests_match_sequential():
    """Requests served at once from several threads (as the HTTP layer's
    worker pool does) give the same attestations as one at a time, and every
    request is counted."""
    import threading

    host = gen.random_model(preset("tiny"), 0)  # large enough for the oracle's worker pool
    host.vocab = ["<unk>", "<s>", "</s>", "▁"] + [f"▁w{i}" for i in range(host.cfg.vocab - 4)]
    svc = server.Service(server.OracleBackend(host), host.vocab, host.weight_hash())
    texts = [f"w{i} w{i + 3} w{2 * i}" for i in range(6)]
    want = {t: svc.run(t, 4)["attestation"] for t in texts}
    got, errs = {}, []

    def work(t):
        try:
            got[t] = svc.run(t, 4)["attestation"]
        except Exception as e:  # pragma: no cover - reported below
            errs.append(e)

    ts = [threading.Thread(target=work, args=(t,)) for t in texts]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs and got == want
    assert svc.stats()["requests"] == 2 * len(texts) and len(svc.attestations) == 2 * len(texts)


class _StubRequest:
    def __init__(self):
        self.done = False
        self.tokens = []


class _FailingScheduler:
    """Scheduler stand-in: accepts requests, then its step raises."""

    cfg = None

    def __init__(self, fail_after: int = 0):
        self.waiting = []
        self.lanes = [None]
        self.requests = {}
        self.steps = 0
        self.fail_after = fail_after

    def submit(self, prompt, max_tokens):
        rid = len(self.requests)
        self.requests[rid] = _StubRequest()
        self.waiting.append(rid)
        return rid

    def step(self):
        self.steps += 1
        if self.steps > self.fail_after:
            raise RuntimeError("CUDA error: an illegal memory access was encountered (injected on the host)")
        rid = self.waiting.pop(0)
        self.requests[rid].done = True
        self.requests[rid].tokens = [7]


def test_scheduler_failure_raises_in_callers():
    """A step that raises ends the loop, wakes the waiting caller with an
    error, and every later request fails at once instead of hanging."""
    import threading

    import pytest

    be = server.SchedulerBackend(sched=_FailingScheduler(fail_after=1))
    try:
        assert be.generate([1, 2], 4) == [7]  # the first step succeeds
        res = {}

        def call(i):
            try:
                res[i] = be.generate([3], 4)
            except server.BackendError as e:
                res[i] = e

        ts = [threading.Thread(target=call, args=(i,)) for i in range(3)]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=10)
        assert not any(t.is_alive() for t in ts), "a caller is still waiting"
        assert all(isinstance(res[i], server.BackendError) for i in range(3))
        assert isinstance(be.error, RuntimeError)
        with pytest.raises(server.BackendError):
            be.generate([4], 1)
        assert not be.t.is_alive()
    finally:
        be.close()
