"""The fused GEMM's norm converter (decode of one or two slots): the limb
operand is built in shared memory from the hidden state, its sum of squares
and the norm weights, instead of by a separate RMSNorm -> limb-planes
launch.  Checked against RMSNorm then the int8 matmul of the CPU oracle, and
end to end (greedy generation with it on and off against the oracle)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200 import spec
from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,B,mag", [(128, 128, 1, 1 << 17), (4096, 4096, 1, 1 << 18), (1000, 688, 2, 1 << 30),
                                       (256, 4000, 1, 1 << 40), (12288, 4096, 2, 1 << 20)])
def test_norm_converter_gemm_matches_oracle(M, K, B, mag):
    from arc_chain_b200.ops import int_ops as ops

    rng = np.random.default_rng(M + K + B)
    w = rng.integers(-127, 128, size=(M, K), dtype=np.int64).astype(np.int8)
    s = rng.integers(1, 5000, size=M).astype(np.int64)
    h = rng.integers(-mag, mag, size=(B, K), dtype=np.int64)
    gamma = rng.integers(1 << 14, 1 << 17, size=K, dtype=np.int64)
    with np.errstate(over="ignore"):
        ss = np.array([((r * r) >> 16).sum(dtype=np.int64) for r in h], dtype=np.int64)
    ref = np.stack([arcref.matmul_i8(w, s, spec.rmsnorm(h[b], gamma)) for b in range(B)])
    dev = torch.device("cuda")
    W = ops.tile_weight(torch.from_numpy(w).to(dev))
    bn = ops.fgemm_bn(B)
    X = torch.zeros(ops.limb_rows(B, bn), K, dtype=torch.int8, device=dev)  # unread: the converter builds it
    wm, xm = ops.TensorMap(W, 128), ops.TensorMap(X, bn)
    lmax = torch.zeros(1, dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    H, SS, G, S = (torch.from_numpy(a).to(dev) for a in (h, ss, gamma, s))
    e = ops.epi(ops.STORE, S, err, out=out, ldo=M, nc_h=H, nc_ss=SS, nc_gamma=G, nc_ngamma=K)
    for _ in range(2):
        out.zero_()
        ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, e)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
        assert int(P.abs().max().item()) == 0 and int(tiles.abs().max().item()) == 0


@pytest.mark.parametrize("on", [True, False])
def test_generation_with_norm_converter(on):
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.scheduler import Scheduler

    cfg = preset("tiny")
    host = gen.random_model(cfg, 0)
    oracle = arcref.Model(host)
    eng = Engine(dense.from_host(host, "cuda"), n_pages=256, max_seq=256)
    eng.norm_conv = on
    assert eng._norm_conv(1) == on and not eng._norm_conv(3)
    prompt = gen.seeded_prompt(20, cfg.vocab, 5)
    ref, rh = oracle.generate(prompt, 16)
    for use_graph in (False, True):
        got, gh = eng.generate(prompt, 16, use_graph=use_graph)
        assert got == ref and gh == rh
    # two decode lanes (the converter's largest batch)
    sch = Scheduler(eng, max_batch=2, prefill_chunk=16, gen_cap=12)
    specs = [(gen.seeded_prompt(4 + 3 * i, cfg.vocab, 60 + i), 6 + i) for i in range(4)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        assert sch.requests[rid].tokens == oracle.generate(p, n)[0]
    assert eng.check_errors() == 0
