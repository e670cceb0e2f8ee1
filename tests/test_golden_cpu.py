"""Golden values pinned in the repository: weight hashes of the seeded
random models, the C++ oracle's output hashes (INT8 and the reference's
per-row Q4) for three dense configs, the MLA+MoE oracle's tokens and hash,
and the toy full-sequence engine's.  Any change to the oracle's arithmetic,
the seeded generator, the prompt generator or the hashing shows up here as a
changed hex string.  The reference pins no hash of its own; these are the
oracle's values when they were first recorded."""
import pytest

from arc_chain_b200.formats import gen
from arc_chain_b200.models import mla_moe
from arc_chain_b200.models.config import preset
from arc_chain_b200.models.toy_integer import ToyIntegerModel
from arc_chain_b200.oracle import arcref

# (preset, weight seed, prompt length, prompt seed, generated tokens,
#  weight hash, INT8 output hash, first 8 tokens, Q4 output hash)
DENSE = [
    ("tiny", 0, 32, 1, 64, "be860b1160a08bb7173f8fc390c32c16d933f0aaa1f6da8892f18957fad65b75",
     "a70fd4b54755e0fc34dde75817fa91e7500f23966383edd55e582c6a745bcc90",
     [9327, 31271, 22793, 18384, 27243, 4928, 1310, 30138],
     "c08f097cc55ad807de846dcec3ef8b2437c45dc0e37e62c177e03a8f4f9695e4"),
    ("micro", 3, 16, 2, 48, "422281ead07c72893a2d378b9d08f79eb0c0a3ba6c52b7f5b409cfec0c1912a6",
     "edc4f5b967b71477c84dc1329232905beb933b068ecd8656fca651366666976e",
     [125, 98, 412, 141, 185, 158, 211, 135],
     "e4006c3f6d8164de7d357a73709677d43e702bec5012766fe82ba67c4540ac0d"),
    ("micro_gqa", 5, 24, 7, 40, "907c71b250e74dbc2ce68083053f50a27da52e0001fd57d136e15831025a3d77",
     "3c302bf9acf86262144a301b97ac46f31ae0e5bc4583b4139cbb4c58eb4a0322",
     [667, 260, 13, 776, 479, 217, 437, 666],
     "bf6b4235a9e069e99a9baaccafb4c1aaf5cd6ae3e18ddb78b3cdbdbf7be78669"),
]


@pytest.mark.parametrize("row", DENSE, ids=[r[0] for r in DENSE])
def test_dense_oracle_golden(row):
    name, seed, plen, pseed, n, wh, h8, first, h4 = row
    host = gen.random_model(preset(name), seed)
    assert host.weight_hash().hex() == wh
    prompt = gen.seeded_prompt(plen, host.cfg.vocab, pseed)
    toks, h = arcref.Model(host).generate(prompt, n)
    assert h.hex() == h8 and toks[:8] == first and len(toks) == n
    q = arcref.Model(host)
    q.enable_q4()
    assert q.generate(prompt, n)[1].hex() == h4


def test_oracle_output_independent_of_thread_count():
    name, seed, plen, pseed, n, _, h8, _, _ = DENSE[0]
    host = gen.random_model(preset(name), seed)
    prompt = gen.seeded_prompt(plen, host.cfg.vocab, pseed)
    L = arcref.lib()
    old = L.arcref_num_threads()
    try:
        for t in (1, 3, max(2, old)):
            L.arcref_set_threads(t)
            assert arcref.Model(host).generate(prompt, n)[1].hex() == h8, t
    finally:
        L.arcref_set_threads(old)


def test_mla_moe_oracle_golden():
    m = gen.random_model(preset("micro_moe"), 0)
    toks, h = mla_moe.MlaMoeOracle(m).generate([3, 4, 5], 6)
    assert toks == [752, 230, 117, 779, 247, 275]
    assert h.hex() == "2579cc2b74af110c1558b2f01364fdf6f354b2bd75dc4a17c11a2bf1c7d584bf"


def test_toy_engine_golden():
    toks, h = ToyIntegerModel(100, 64, 2, 128, 2).generate_with_hash([1, 5, 10, 15], 8, 99)
    assert toks == [29, 18, 72, 47, 18, 72, 47, 47]
    assert h.hex() == "eb554f4f8afa13876ac66968b71c0d139eae83d5899a09931d5e65c47172eb1d"


def test_oracle_concurrent_callers():
    """Several host threads (an HTTP server's workers, say) call the oracle
    at once; ctypes releases the GIL, so the native worker pool is shared
    between them.  Every result must still equal the pinned hash."""
    import threading

    name, seed, plen, pseed, n, _, h8, _, _ = DENSE[0]
    host = gen.random_model(preset(name), seed)
    prompt = gen.seeded_prompt(plen, host.cfg.vocab, pseed)
    models = [arcref.Model(host) for _ in range(4)]
    got, errs = [], []

    def work(m):
        try:
            for _ in range(2):
                got.append(m.generate(prompt, n)[1].hex())
        except Exception as e:  # pragma: no cover - reported below
            errs.append(e)

    L = arcref.lib()
    old = L.arcref_num_threads()
    L.arcref_set_threads(max(4, old))
    try:
        ts = [threading.Thread(target=work, args=(m,)) for m in models]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    finally:
        L.arcref_set_threads(old)
    assert not errs and got == [h8] * 8


def test_pinned_7b_output_is_consistent():
    """The pinned 7B tokens hash to the pinned output hash (cheap check of
    the golden table itself)."""
    import numpy as np

    from arc_chain_b200.bench import golden
    from arc_chain_b200.utils.hashing import blake3

    assert len(golden.TOKENS_256) == 256
    assert blake3(np.asarray(golden.TOKENS_256, dtype="<u4").tobytes()).hex() == golden.OUTPUT_HASH_256
    assert golden.prefix_ok(golden.TOKENS_256[:25]) and not golden.prefix_ok(golden.TOKENS_256[1:26])


@pytest.mark.skipif(not __import__("os").environ.get("ARCB_SLOW"), reason="7B on the CPU oracle: ~5 min (ARCB_SLOW=1)")
def test_oracle_reproduces_pinned_7b_output():
    from arc_chain_b200.bench import golden

    cfg = preset(golden.MODEL)
    cfg.max_seq = 400
    host = gen.random_model(cfg, golden.WEIGHT_SEED)
    assert host.weight_hash().hex() == golden.WEIGHT_HASH
    prompt = gen.seeded_prompt(golden.PROMPT_LEN, cfg.vocab, golden.PROMPT_SEED)
    toks, h = arcref.Model(host).generate(prompt, 256)
    assert toks == golden.TOKENS_256 and h.hex() == golden.OUTPUT_HASH_256
