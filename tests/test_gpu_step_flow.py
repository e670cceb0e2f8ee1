"""The persistent dataflow decode step (one cooperative launch per token,
csrc/kernels/decode_flow.cu) against the CPU oracle: single stream (eager
and CUDA graph, MHA and GQA heads, head dims 64 and 128), two lanes through
the scheduler, and the full logits of a step against the per-kernel path,
all exact."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


def _engine(host):
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    eng = Engine(dense.from_host(host, "cuda"))
    eng.use_step_kernel = True
    return eng


def _ran_flow(eng):
    from arc_chain_b200.runtime.step_flow import FlowStep

    return any(isinstance(v, FlowStep) for v in eng._step_progs.values())


@pytest.mark.parametrize("name", ["micro", "micro_gqa", "tiny"])
def test_flow_generate_matches_oracle(name):
    cfg = preset(name)
    host = gen.random_model(cfg, 7)
    eng = _engine(host)
    om = arcref.Model(host)
    for i, n in enumerate((1, 9, 40)):
        p = gen.seeded_prompt(3 + 5 * i, cfg.vocab, 400 + i)
        ref = om.generate(p, n)
        for use_graph in (False, True):
            assert eng.generate(p, n, use_graph=use_graph) == ref, (name, i, use_graph)
    assert eng.check_errors() == 0
    assert _ran_flow(eng)


def test_flow_head_dim_128():
    """Llama-style heads of 128 (the 7B shape) on a small model."""
    from arc_chain_b200.models.config import ModelConfig

    cfg = ModelConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, d_ff=768, d_head=128, vocab=1000,
                      max_seq=256, name="flow128")
    host = gen.random_model(cfg, 3)
    eng = _engine(host)
    p = gen.seeded_prompt(37, cfg.vocab, 9)
    assert eng.generate(p, 24) == arcref.Model(host).generate(p, 24)
    assert eng.check_errors() == 0 and _ran_flow(eng)


def test_flow_logits_equal_per_kernel_path():
    """One decode step: the dataflow kernel's logits equal the per-kernel
    forward's, element for element."""
    cfg = preset("tiny")
    host = gen.random_model(cfg, 5)
    eng = _engine(host)
    p = gen.seeded_prompt(20, cfg.vocab, 3)
    rid = eng.new_request(64)
    eng.prefill(rid, [1] + p)
    bb = eng.buffers(1, gen_cap=4)
    eng._reset_sampling(bb, [rid], [p[-1]], [len(p) + 1], ())
    flow = eng.flow_step(bb)
    assert flow is not None
    flow.launch()
    got = flow.logits[:1].clone()
    eng.forward(bb, 1, True)  # the same step through the per-kernel path (same KV writes)
    torch.cuda.synchronize()
    assert torch.equal(got, bb.logits[:1])
    assert eng.check_errors() == 0


def test_flow_two_lanes():
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 8)
    eng = _engine(host)
    sch = Scheduler(eng, max_batch=2, prefill_chunk=16, gen_cap=24)
    specs = [(gen.seeded_prompt(4 + 3 * i, cfg.vocab, 500 + i), 8 + 4 * i) for i in range(4)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == arcref.Model(host).generate(p, n)[0]
    assert eng.check_errors() == 0
    assert _ran_flow(eng)
