"""Chunk (prefill) attention: one launch per layer for a whole prefill chunk,
every K/V page read once per 16 positions.  Checked element for element
against the per-position decode kernel (random cache, chunks at offsets,
padding slots, MHA and GQA, head dims 64 and 128) and end to end against the
CPU oracle (logits of every prompt position, generated tokens)."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dh,heads,kv,nq,p0,B", [(128, 4, 4, 37, 0, 64), (128, 8, 2, 16, 300, 16),
                                                 (64, 4, 2, 100, 77, 128), (128, 2, 1, 1, 520, 16),
                                                 (64, 2, 2, 1024, 0, 1024)])
def test_prefill_kernel_equals_per_position_kernel(dh, heads, kv, nq, p0, B):
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    T = p0 + nq
    pages = (T + 15) // 16
    n_pages = pages + 3
    g = torch.Generator(device="cpu").manual_seed(dh * 7 + nq)
    K = torch.randint(-(1 << 22), 1 << 22, (n_pages, kv, 16, dh), generator=g, dtype=torch.int64).to(dev)
    V = torch.randint(-(1 << 22), 1 << 22, (n_pages, kv, 16, dh), generator=g, dtype=torch.int64).to(dev)
    q = torch.randint(-(1 << 22), 1 << 22, (B, heads * dh), generator=g, dtype=torch.int64).to(dev)
    perm = torch.randperm(n_pages, generator=g)[:pages].to(torch.int32)
    pt = torch.zeros(B, pages + 4, dtype=torch.int32)
    pt[:, :pages] = perm
    pt = pt.to(dev)
    pos = torch.tensor([p0 + i if i < nq else 0 for i in range(B)], dtype=torch.int32, device=dev)
    rows = ops.limb_rows(B)
    X1 = torch.zeros(rows, heads * dh, dtype=torch.int8, device=dev)
    X2 = torch.zeros_like(X1)
    l1 = torch.zeros(1, dtype=torch.int32, device=dev)
    l2 = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    max_T = (pages + 4) * 16
    assert ops.attn_prefill(q, K, V, pt[0], nq, p0, heads, kv, dh, 5793, B, X1, l1, max_T, err)
    ops.attn(q, K, V, pt, pos, heads, kv, dh, 5793, B, X2, l2, max_T, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    real = [ops.limb_row(l, b, B) for b in range(nq) for l in range(8)]
    assert torch.equal(X1[real], X2[real])
    assert int(l1.item()) == int(l2.item())
    pad = [ops.limb_row(l, b, B) for b in range(nq, B) for l in range(8)]
    if pad:
        assert not X1[pad].any()


@pytest.mark.parametrize("name,chunk", [("micro_gqa", 64), ("tiny", 1024), ("tiny", 48)])
def test_prefill_logits_and_generation_match_oracle(name, chunk):
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    import numpy as np

    cfg = preset(name)
    host = gen.random_model(cfg, 11)
    eng = Engine(dense.from_host(host, "cuda"))
    assert eng.prefill_attn
    om = arcref.Model(host)
    toks = [1] + gen.seeded_prompt(150, cfg.vocab, 5)
    out = []
    rid = eng.new_request(len(toks) + 1)
    eng.prefill(rid, toks, chunk=chunk, logits_sink=out.append)
    eng.kv.release(rid)
    got = np.concatenate(out)
    eng.prefill_attn = False
    ref_gpu = eng.score(toks, chunk=chunk)
    eng.prefill_attn = True
    assert np.array_equal(got, ref_gpu)
    p = gen.seeded_prompt(90, cfg.vocab, 6)
    assert eng.generate(p, 20) == om.generate(p, 20)
    assert eng.check_errors() == 0


@pytest.mark.parametrize("dh,heads,kv,B", [(128, 64, 8, 64), (128, 16, 2, 40), (64, 8, 4, 48), (128, 8, 1, 64)])
def test_gqa_block_decode_equals_per_head_kernel(dh, heads, kv, B):
    """Grouped-query decode attention (one CTA per slot and KV head) against
    the per-query-head kernel, slots at different positions."""
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(heads * 31 + B)
    maxp = 40
    n_pages = B * maxp
    K = torch.randint(-(1 << 22), 1 << 22, (n_pages, kv, 16, dh), generator=g, dtype=torch.int64).to(dev)
    V = torch.randint(-(1 << 22), 1 << 22, (n_pages, kv, 16, dh), generator=g, dtype=torch.int64).to(dev)
    q = torch.randint(-(1 << 22), 1 << 22, (B, heads * dh), generator=g, dtype=torch.int64).to(dev)
    pt = torch.randperm(n_pages, generator=g).to(torch.int32).view(B, maxp).to(dev)
    pos = torch.randint(0, maxp * 16, (B,), generator=g, dtype=torch.int32).to(dev)
    pos[0] = 0
    rows = ops.limb_rows(B)
    X1 = torch.zeros(rows, heads * dh, dtype=torch.int8, device=dev)
    X2 = torch.zeros_like(X1)
    l1 = torch.zeros(1, dtype=torch.int32, device=dev)
    l2 = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    T = maxp * 16
    assert ops.attn_gqa_block(q, K, V, pt, pos, heads, kv, dh, 5793, B, X1, l1, T, T, err)
    ops.attn(q, K, V, pt, pos, heads, kv, dh, 5793, B, X2, l2, T, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(X1, X2) and int(l1.item()) == int(l2.item())


def test_batched_gqa_decode_matches_oracle():
    """Continuous batching over 40 lanes of a grouped-query model (the
    per-(slot, KV head) decode attention runs) equals single-stream oracle
    decoding for every request."""
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 12)
    eng = Engine(dense.from_host(host, "cuda"), n_pages=1200)
    sch = Scheduler(eng, max_batch=40, prefill_chunk=64, gen_cap=24)
    specs = [(gen.seeded_prompt(5 + (7 * i) % 60, cfg.vocab, 300 + i), 6 + (i % 11)) for i in range(44)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    om = arcref.Model(host)
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == om.generate(p, n)[0]
    assert eng.check_errors() == 0
