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
