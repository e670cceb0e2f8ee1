"""Batch-size paths of the fused GEMM and the batched MLA/MoE kernels against
the CPU oracle (exact): limb-operand sub-box loads, persistent CTA budgets
(whole tiles finalised from TMEM in 8-slot batches, or split tiles through
the partial buffer), per-head projections over several slot chunks, and the
warp router."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,mag", [(8, 1 << 17), (16, 1 << 40), (24, 1 << 12), (32, 1 << 20), (40, 1 << 17),
                                   (64, 1 << 23)])
@pytest.mark.parametrize("ctas", ["tiles", "heuristic", 7, 0])
def test_fused_gemm_sub_box_and_cta_budget(B, mag, ctas):
    from arc_chain_b200.ops import int_ops as ops

    M, K = 1280, 768
    rng = np.random.default_rng(B * 7 + mag % 97)
    w = rng.integers(-127, 128, size=(M, K), dtype=np.int64).astype(np.int8)
    s = rng.integers(1, 5000, size=M).astype(np.int64)
    x = rng.integers(-mag, mag, size=(B, K), dtype=np.int64)
    bn = ops.fgemm_bn(B)
    planes, need = ops.limb_planes(x, ops.limb_rows(B, bn))
    dev = torch.device("cuda")
    W, X, S = (torch.from_numpy(a).to(dev) for a in (w, planes, s))
    wm, xm = ops.TensorMap(ops.tile_weight(W), 128), ops.TensorMap(X, bn, min(bn, 32))
    lmax = torch.tensor([need], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    ref = np.stack([arcref.matmul_i8(w, s, x[b]) for b in range(B)])
    e = ops.epi(ops.STORE, S, err, out=out, ldo=M)
    e.max_ctas = {"tiles": (M // 128) * ops.n_tiles(B), "heuristic": ops.split_ctas(M, B, bn)}.get(ctas, ctas)
    for _ in range(2):
        out.zero_()
        ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, e)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
        assert int(P.abs().max().item()) == 0 and int(tiles.abs().max().item()) == 0


def test_dense_batch16_matches_oracle():
    """16 lanes (whole-tile epilogue reads 8 slots per TMEM batch)."""
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 3)
    eng = Engine(dense.from_host(host, "cuda"))
    om = arcref.Model(host)
    sch = Scheduler(eng, max_batch=16, prefill_chunk=16, gen_cap=12)
    specs = [(gen.seeded_prompt(3 + i, cfg.vocab, 50 + i), 6 + (i % 5)) for i in range(16)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == om.generate(p, n)[0], rid
    assert eng.check_errors() == 0


def test_mla_moe_batch24_matches_oracle():
    """24 lanes: per-head projections over two slot chunks, warp router."""
    from arc_chain_b200.models import mla_moe, mla_moe_engine as me
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("micro_moe")
    host = gen.random_model(cfg, 4)
    eng = me.MlaMoeEngine(me.from_host(host, "cuda"))
    sch = Scheduler(eng, max_batch=24, prefill_chunk=16, gen_cap=8)
    specs = [(gen.seeded_prompt(2 + i % 6, cfg.vocab, 70 + i), 4 + (i % 3)) for i in range(24)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == mla_moe.MlaMoeOracle(host).generate(p, n)[0], rid  # fresh oracle state
    assert eng.check_errors() == 0
