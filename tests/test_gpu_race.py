"""Run-to-run hash equality as a race detector.  Every kernel computes exact
integers, so any data race (a missing fence, a stale partial, an early
read of a peer's tile) shows up as a changed token or hash.  The same
generations run under different launch configurations: programmatic
dependent launch on and off, different persistent CTA budgets (tiles split
across many CTAs, one CTA per tile, a few CTAs), eager and CUDA-graph
replay, single-stream and batched lanes; all must equal the oracle."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu

SPLITS = {"default": None, "one_cta_per_tile": [(1 << 30, 1)], "wide_split": [(1 << 30, 64)]}


@pytest.mark.parametrize("pdl", [True, False])
@pytest.mark.parametrize("split", list(SPLITS))
def test_hashes_invariant_under_launch_config(pdl, split):
    from arc_chain_b200.models import dense
    from arc_chain_b200.ops import int_ops as ops
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 11)
    prompts = [(gen.seeded_prompt(5 + 3 * i, cfg.vocab, 300 + i), 12) for i in range(5)]
    refs = [arcref.Model(host).generate(p, n) for p, n in prompts]
    saved = list(ops.SPLIT_TABLE)
    try:
        if SPLITS[split] is not None:
            ops.SPLIT_TABLE[:] = SPLITS[split]
        ops.set_pdl(pdl)
        eng = Engine(dense.from_host(host, "cuda"))
        for (p, n), ref in zip(prompts[:2], refs[:2]):
            for use_graph in (False, True):
                assert eng.generate(p, n, use_graph=use_graph) == ref
        sch = Scheduler(eng, max_batch=4, prefill_chunk=16, gen_cap=16)
        rids = [sch.submit(p, n) for p, n in prompts]
        sch.run()
        assert [(sch.requests[r].tokens, sch.requests[r].output_hash) for r in rids] == refs
        assert eng.check_errors() == 0
    finally:
        ops.SPLIT_TABLE[:] = saved
        ops.set_pdl(True)
