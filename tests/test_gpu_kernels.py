"""sm_100a kernels against the CPU oracle (exact equality)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200 import spec
from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


def _ops():
    from arc_chain_b200.ops import int_ops

    return int_ops


def _limbs(x: np.ndarray, B: int, K: int):
    """Host signed-digit limb planes [8*B, K] and max limb count."""
    planes = np.zeros((8, B, K), dtype=np.int8)
    r = x.astype(np.int64).copy()
    need = 0
    for l in range(8):
        d = (r & 0xFF).astype(np.uint8).view(np.int8)
        planes[l] = d
        r = (r - d.astype(np.int64)) >> 8
        if np.any(r != 0):
            need = l + 2
    need = min(8, need) if np.any(x != 0) else 0
    if np.any(x != 0) and need == 0:
        need = 1
    return planes.reshape(8 * B, K), need


@pytest.mark.parametrize("M,K,B,mag", [(128, 128, 1, 1 << 17), (256, 256, 3, 1 << 20), (384, 688, 2, 1 << 40),
                                       (4096, 4096, 1, 1 << 18), (1000, 512, 5, 1 << 62), (640, 1024, 40, 1 << 17),
                                       (256, 512, 70, 1 << 23)])
def test_gemm_i8_exact(M, K, B, mag):
    ops = _ops()
    rng = np.random.default_rng(M * 7 + K + B)
    w = rng.integers(-127, 128, size=(M, K), dtype=np.int64).astype(np.int8)
    s = rng.integers(1, 5000, size=M).astype(np.int64)
    x = rng.integers(-mag, mag, size=(B, K), dtype=np.int64)
    planes, need = _limbs(x, B, K)
    dev = torch.device("cuda")
    W = torch.from_numpy(w).to(dev)
    bn = ops.gemm_bn(B)
    if planes.shape[0] < bn:
        planes = np.concatenate([planes, np.zeros((bn - planes.shape[0], K), np.int8)])
    X = torch.from_numpy(planes).to(dev)
    wm, xm = ops.TensorMap(W, 128), ops.TensorMap(X, bn)
    lmax = torch.tensor([need], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    S = torch.from_numpy(s).to(dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    for ks in (1, 3):
        ops.gemm_i8(wm, xm, M, K, B, ks, lmax, P, err)
        ops.finalize(P, M, B, lmax, S, out, M, 0)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = out.cpu().numpy()
        for b in range(B):
            ref = arcref.matmul_i8(w, s, x[b])
            np.testing.assert_array_equal(got[b], ref)
        assert int(P.abs().max().item()) == 0  # finalize zeroed the partials


@pytest.mark.parametrize("M,K,B,mag", [(128, 128, 1, 1 << 17), (4096, 4096, 1, 1 << 18), (1000, 688, 3, 1 << 40),
                                       (32000, 256, 2, 1 << 20), (640, 1024, 40, 1 << 17), (384, 512, 33, 1 << 62),
                                       (256, 2048, 130, 1 << 23)])
def test_fused_gemm_store_and_partial(M, K, B, mag):
    """Persistent stream-K GEMM: STORE epilogue (fused finalize) and PARTIAL."""
    ops = _ops()
    rng = np.random.default_rng(M + 3 * K + B)
    w = rng.integers(-127, 128, size=(M, K), dtype=np.int64).astype(np.int8)
    s = rng.integers(1, 5000, size=M).astype(np.int64)
    x = rng.integers(-mag, mag, size=(B, K), dtype=np.int64)
    bn = ops.fgemm_bn(B)
    planes, need = ops.limb_planes(x, ops.limb_rows(B, bn))  # blocked limb layout for B > 32
    dev = torch.device("cuda")
    W, X, S = (torch.from_numpy(a).to(dev) for a in (w, planes, s))
    Wt = ops.tile_weight(W)
    assert torch.equal(ops.untile_weight(Wt, M, K), W)
    wm, xm = ops.TensorMap(Wt, 128), ops.TensorMap(X, bn)
    lmax = torch.tensor([need], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    ref = np.stack([arcref.matmul_i8(w, s, x[b]) for b in range(B)])
    for rep in range(2):
        out.zero_()
        ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, ops.epi(ops.STORE, S, err, out=out, ldo=M))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
        assert int(P.abs().max().item()) == 0 and int(tiles.abs().max().item()) == 0
    ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, ops.epi(ops.PARTIAL, S, err))
    ops.finalize(P, M, B, lmax, S, out, M, 0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_rmsnorm_limbs_exact():
    ops = _ops()
    rng = np.random.default_rng(1)
    B, d = 4, 4096
    h = rng.integers(-(1 << 22), 1 << 22, size=(B, d), dtype=np.int64)
    g = rng.integers(60000, 70000, size=d - 7).astype(np.int64)  # shorter gamma: ONE past the end
    dev = torch.device("cuda")
    H = torch.from_numpy(h).to(dev)
    G = torch.from_numpy(g).to(dev)
    X = torch.zeros(8 * B, d, dtype=torch.int8, device=dev)
    lm = torch.zeros(1, dtype=torch.int32, device=dev)
    Y = torch.zeros(B, d, dtype=torch.int64, device=dev)
    ops.rmsnorm_limbs(H, G, d, B, X, lm, Y)
    torch.cuda.synchronize()
    y = Y.cpu().numpy()
    for b in range(B):
        np.testing.assert_array_equal(y[b], arcref.rmsnorm(h[b], g))
    planes, need = _limbs(y, B, d)
    assert int(lm.item()) == need
    np.testing.assert_array_equal(X.cpu().numpy(), planes)


def _engine_for(cfg_name, seed=0):
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    cfg = preset(cfg_name)
    host = gen.random_model(cfg, seed)
    dm = dense.from_host(host, "cuda")
    return host, Engine(dm)


@pytest.mark.parametrize("name", ["micro", "micro_gqa"])
def test_generate_matches_oracle(name):
    host, eng = _engine_for(name)
    om = arcref.Model(host)
    prompt = gen.seeded_prompt(20, host.cfg.vocab, 1)
    ref, rh = om.generate(prompt, 24)
    for use_graph in (False, True):
        got, gh = eng.generate(prompt, 24, use_graph=use_graph)
        assert got == ref
        assert gh == rh
    assert eng.check_errors() == 0


def test_generate_eos_stops():
    host, eng = _engine_for("micro")
    om = arcref.Model(host)
    prompt = gen.seeded_prompt(8, host.cfg.vocab, 3)
    ref, _ = om.generate(prompt, 12)
    eos = [ref[4]]
    r2, h2 = om.generate(prompt, 12, eos)
    got, gh = eng.generate(prompt, 12, eos)
    assert got == r2 and gh == h2 and len(got) <= 5


def test_tiny_golden_hash():
    """The tiny config: 32-token prompt (seed 1), 64 greedy tokens, weights seed 0."""
    host, eng = _engine_for("tiny")
    prompt = gen.seeded_prompt(32, 32000, 1)
    om = arcref.Model(host)
    ref, rh = om.generate(prompt, 64)
    got, gh = eng.generate(prompt, 64)
    assert got == ref and gh == rh


def test_device_random_init_matches_host():
    from arc_chain_b200.models import dense

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 5)
    dm = dense.random_device(cfg, "cuda", seed=5)
    ref = dense.from_host(host, "cuda")
    assert torch.equal(dm.emb, ref.emb) and torch.equal(dm.emb_s, ref.emb_s)
    assert torch.equal(dm.lm.w, ref.lm.w) and torch.equal(dm.final_norm, ref.final_norm)
    for a, b in zip(dm.layers, ref.layers):
        for n in ("qkv", "wo", "gu", "down"):
            assert torch.equal(getattr(a, n).w, getattr(b, n).w)
            assert torch.equal(getattr(a, n).s, getattr(b, n).s)


def test_continuous_batching_matches_single_stream():
    """Requests of different prompt/output lengths share decode steps; each
    output equals the oracle's single-stream generate."""
    from arc_chain_b200.runtime.scheduler import Scheduler

    host, eng = _engine_for("micro_gqa")
    om = arcref.Model(host)
    sch = Scheduler(eng, max_batch=4, prefill_chunk=16, gen_cap=40)
    specs = [(gen.seeded_prompt(5 + 7 * i, host.cfg.vocab, 10 + i), 8 + 5 * i) for i in range(7)]
    rids = [sch.submit(p, n) for p, n in specs]
    sch.run()
    for rid, (p, n) in zip(rids, specs):
        ref, rh = om.generate(p, n)
        r = sch.requests[rid]
        assert r.tokens == ref, rid
        assert r.output_hash == rh
    assert eng.check_errors() == 0


@pytest.mark.parametrize("M,K,B", [(128, 128, 1), (1000, 688, 3), (4096, 4096, 1), (640, 1024, 40)])
def test_q4_gemm_exact(M, K, B):
    """K2: Q4 group-32 tiles dequantised in shared memory == int8 GEMM of
    the effective weights m_g * q."""
    ops = _ops()
    rng = np.random.default_rng(M + K + 11 * B)
    q = rng.integers(-8, 8, size=(M, K)).astype(np.int8)
    m = rng.integers(1, 16, size=(M, (K + 31) // 32)).astype(np.uint8)
    s = rng.integers(1, 5000, size=M).astype(np.int64)
    x = rng.integers(-(1 << 30), 1 << 30, size=(B, K), dtype=np.int64)
    weff = spec.q4g_effective(q, m)
    bn = ops.fgemm_bn(B)
    planes, need = ops.limb_planes(x, ops.limb_rows(B, bn))
    dev = torch.device("cuda")
    packed = ops.pack_q4(torch.from_numpy(q).to(dev), torch.from_numpy(m).to(dev))
    X, S = torch.from_numpy(planes).to(dev), torch.from_numpy(s).to(dev)
    xm = ops.TensorMap(X, bn)
    lmax = torch.tensor([need], dtype=torch.int32, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    tiles = torch.zeros(ops.tile_counters(M, B), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    ops.fgemm_q4(packed, xm, M, K, B, lmax, P, tiles, ops.epi(ops.STORE, S, err, out=out, ldo=M))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = np.stack([arcref.matmul_i8(weff, s, x[b]) for b in range(B)])
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_q4_reference_row_mode_matches_oracle_enable_q4():
    """The reference's per-row Q4 (enable_q4) end to end."""
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 2)
    eng = Engine(dense.from_host(host, "cuda", q4="row"))
    om = arcref.Model(host)
    om.enable_q4()
    prompt = gen.seeded_prompt(16, cfg.vocab, 4)
    ref, rh = om.generate(prompt, 20)
    got, gh = eng.generate(prompt, 20)
    assert got == ref and gh == rh


def test_q4_group_mode_matches_oracle():
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 3)
    eng = Engine(dense.from_host(host, "cuda", q4="group"))
    om = arcref.Model(spec.q4g_effective_model(host))
    prompt = gen.seeded_prompt(16, cfg.vocab, 5)
    ref, rh = om.generate(prompt, 20)
    got, gh = eng.generate(prompt, 20)
    assert got == ref and gh == rh


@pytest.mark.parametrize("same_draft", [True, False])
def test_speculative_decoding_equals_plain_greedy(same_draft):
    """Accepted output == non-speculative target decoding, whether every draft
    token is accepted (draft == target) or almost none (unrelated draft)."""
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine
    from arc_chain_b200.runtime.spec_decode import SpecDecoder

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 0)
    target = Engine(dense.from_host(host, "cuda"))
    dhost = host if same_draft else gen.random_model(cfg, 9)
    draft = Engine(dense.from_host(dhost, "cuda"))
    sd = SpecDecoder(target, draft, k=4, lanes=2, gen_cap=64)
    prompts = [gen.seeded_prompt(12, cfg.vocab, 21), gen.seeded_prompt(19, cfg.vocab, 22)]
    out = sd.generate(prompts, 30)
    om = arcref.Model(host)
    for p, (toks, h) in zip(prompts, out):
        ref, rh = om.generate(p, 30)
        assert toks == ref and h == rh
    if same_draft:
        assert sd.acceptance == 1.0
    assert target.check_errors() == 0 and draft.check_errors() == 0


def test_sample_penalty_and_argmax_match_reference():
    """k_sample: compounding repetition penalty over the newest 64 ids (with
    repeated ids) then argmax with lowest-index ties, against a direct
    restatement of the reference loop (cached_integer_model.rs:1537-1548)."""
    from arc_chain_b200 import spec
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    rng = np.random.default_rng(3)
    V, S = 5000, 6
    for cnt in (0, 1, 7, 64, 100):
        logits = rng.integers(-(1 << 40), 1 << 40, size=(S, V), dtype=np.int64)
        logits[:, 17] = logits[:, 4000] = logits.max() + 5  # a tie: the lower index wins
        hist = rng.integers(0, 40, size=(S, 64)).astype(np.int32)  # many repeats
        hist[:, ::5] = 17
        want = []
        for s_ in range(S):
            lg = logits[s_].copy()
            for k in range(min(cnt, 64)):
                t = int(hist[s_, (cnt - 1 - k) & 63])
                lg[t] = spec.penalize(int(lg[t]))
            want.append(int(np.argmax(lg)))
        L = torch.from_numpy(logits).to(dev)
        gen_ = torch.zeros(S, 200, dtype=torch.int32, device=dev)
        tok = torch.zeros(S, dtype=torch.int32, device=dev)
        ops.sample(L, V, S, torch.from_numpy(hist).to(dev), torch.full((S,), cnt, dtype=torch.int32, device=dev),
                   gen_, tok)
        torch.cuda.synchronize()
        assert tok.cpu().tolist() == want, cnt


def test_small_quotient_division_is_exact():
    """The kernels' sigmoid and softmax-weight divisions (an estimate from the
    single-precision reciprocal plus one remainder correction) equal the
    64-bit division on every sigmoid divisor and a random softmax sweep."""
    ops = _ops()
    one = 1 << 16
    assert ops.check_udiv(one, 2 * one + 1, 64) == 0
