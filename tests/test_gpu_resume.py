"""Serving snapshot / resume and request-level recovery: a request rebuilt
from (prompt, tokens so far) by re-prefill continues bit-identically, and a
step that raised a kernel error bit is replayed without changing any output."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


def _setup(seed=5):
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, seed)
    specs = [(gen.seeded_prompt(3 + 4 * i, cfg.vocab, 200 + i), 10 + 3 * i) for i in range(6)]
    refs = [arcref.Model(host).generate(p, n)[0] for p, n in specs]
    return host, specs, refs, lambda: Engine(dense.from_host(host, "cuda"))


@pytest.mark.parametrize("steps_before", [1, 4, 9])
def test_snapshot_resume_exact(steps_before):
    from arc_chain_b200.runtime.scheduler import Scheduler

    host, specs, refs, mk = _setup()
    sch = Scheduler(mk(), max_batch=3, prefill_chunk=16, gen_cap=40)
    for p, n in specs:
        sch.submit(p, n)
    sch.run(max_steps=steps_before)
    snap = sch.snapshot()
    sch2 = Scheduler.from_snapshot(mk(), snap, max_batch=3, prefill_chunk=16, gen_cap=40)
    sch2.run()
    got = [r.tokens for _, r in sorted(sch2.requests.items())]
    assert got == refs


def test_recovery_after_error_bit():
    from arc_chain_b200.runtime.scheduler import Scheduler

    host, specs, refs, mk = _setup(6)
    eng = mk()
    sch = Scheduler(eng, max_batch=3, prefill_chunk=16, gen_cap=40)
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run(max_steps=3)
    sch.bb.err.fill_(16)  # as a bounded wait that timed out would leave it
    sch.run()
    assert sch.recoveries == 1
    assert [sch.requests[r].tokens for r in rids] == refs
    assert eng.check_errors() == 0
