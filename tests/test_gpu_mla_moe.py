"""MLA + MoE decoder on the GPU against its numpy oracle (exact)."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models import mla_moe
from arc_chain_b200.models.config import preset

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("use_graph", [False, True])
def test_mla_moe_generate_matches_oracle(use_graph):
    from arc_chain_b200.models import mla_moe_engine as me

    cfg = preset("micro_moe")
    host = gen.random_model(cfg, 0)
    eng = me.MlaMoeEngine(me.from_host(host, "cuda"))
    prompt = gen.seeded_prompt(11, cfg.vocab, 1)
    ref, rh = mla_moe.MlaMoeOracle(host).generate(prompt, 16)
    got, gh = eng.generate(prompt, 16, use_graph=use_graph)
    assert got == ref and gh == rh
    assert eng.check_errors() == 0


def test_mla_moe_batched_lanes():
    from arc_chain_b200.models import mla_moe_engine as me
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_moe")
    host = gen.random_model(cfg, 1)
    eng = me.MlaMoeEngine(me.from_host(host, "cuda"))
    sch = Scheduler(eng, max_batch=3, prefill_chunk=16, gen_cap=24)
    specs = [(gen.seeded_prompt(4 + 3 * i, cfg.vocab, 30 + i), 6 + 2 * i) for i in range(4)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == mla_moe.MlaMoeOracle(host).generate(p, n)[0]
