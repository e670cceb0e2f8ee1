"""The persistent decode-step kernel (one cooperative launch per token)
against the CPU oracle: single stream (eager and CUDA graph) and two lanes,
exact tokens and hashes."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["micro", "micro_gqa"])
def test_step_kernel_generate_matches_oracle(name):
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    cfg = preset(name)
    host = gen.random_model(cfg, 7)
    eng = Engine(dense.from_host(host, "cuda"))
    eng.use_step_kernel = True
    om = arcref.Model(host)
    for i, n in enumerate((1, 9, 40)):
        p = gen.seeded_prompt(3 + 5 * i, cfg.vocab, 400 + i)
        ref = om.generate(p, n)
        for use_graph in (False, True):
            assert eng.generate(p, n, use_graph=use_graph) == ref
    assert eng.check_errors() == 0
    assert any(v is not None for v in eng._step_progs.values())  # the persistent kernel really ran


def test_step_kernel_two_lanes():
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 8)
    eng = Engine(dense.from_host(host, "cuda"))
    eng.use_step_kernel = True
    sch = Scheduler(eng, max_batch=2, prefill_chunk=16, gen_cap=24)
    specs = [(gen.seeded_prompt(4 + 3 * i, cfg.vocab, 500 + i), 8 + 4 * i) for i in range(4)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == arcref.Model(host).generate(p, n)[0]
    assert eng.check_errors() == 0
