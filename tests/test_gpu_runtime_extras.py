"""Engine.score (per-position logits for perplexity) against the oracle's
forward_one_token logits, the scheduler's per-step metrics, uploading a
pre-sharded checkpoint, and the config-driven engine builder."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen, sharded
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


def test_score_matches_oracle_logits():
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    host = gen.random_model(preset("tiny"), 0)
    toks = [1] + gen.seeded_prompt(40, host.cfg.vocab, 3)
    eng = Engine(dense.from_host(host, "cuda"))
    got = eng.score(toks, chunk=16)  # several chunks
    cache = arcref.Model(host).new_cache()
    want = np.stack([cache.forward(t) for t in toks])
    np.testing.assert_array_equal(got, want)


def test_scheduler_metrics():
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    host = gen.random_model(preset("tiny"), 0)
    eng = Engine(dense.from_host(host, "cuda"))
    sink = []
    sch = Scheduler(eng, max_batch=4, prefill_chunk=16, gen_cap=12, metrics_sink=sink.append)
    free0 = len(eng.kv.pool.free)
    for i in range(7):
        sch.submit(gen.seeded_prompt(3 + i, host.cfg.vocab, 50 + i), 4 + i)
    sch.run()
    assert len(sink) == sch.steps == len(sch.metrics)
    assert sum(m["admitted"] for m in sink) == 7 and sum(m["finished"] for m in sink) == 7
    assert sink[-1]["tokens_out"] == sch.tokens_out == sum(len(r.tokens) for r in sch.requests.values())
    assert all(m["active_lanes"] <= 4 for m in sink) and len(eng.kv.pool.free) == free0
    st = sch.stats()
    assert st["finished"] == 7 and st["tokens_per_s"] > 0


def test_presharded_upload_equals_slicing(tmp_path):
    from arc_chain_b200.models import dense

    host = gen.random_model(preset("micro_gqa"), 4)
    sharded.save_sharded(host, str(tmp_path), 2)
    for r in range(2):
        a = dense.from_host(host, "cuda", r, 2)
        b = dense.from_host(sharded.load_shard(str(tmp_path), r), "cuda", r, 2, presharded=True)
        for la, lb in zip(a.layers, b.layers):
            for n in ("qkv", "wo", "gu", "down"):
                assert torch.equal(getattr(la, n).w, getattr(lb, n).w) and torch.equal(getattr(la, n).s, getattr(lb, n).s)
        assert torch.equal(a.lm.w, b.lm.w) and a.vocab_offset == b.vocab_offset


def test_build_engine_from_config():
    from arc_chain_b200.config import RunConfig, build_engine

    eng = build_engine(RunConfig(model="tiny", max_batch=2))
    host = gen.random_model(preset("tiny"), 0)
    p = gen.seeded_prompt(8, host.cfg.vocab, 1)
    assert eng.generate(p, 6) == arcref.Model(host).generate(p, 6)
