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
