"""CPU: file formats, seeded generator, tokenizer, attestation, committee,
NeuralNet (both tag numberings), Q4 tile packing and the TP decomposition."""
import os
import struct

import numpy as np
import pytest

from arc_chain_b200 import spec
from arc_chain_b200.formats import arc_int8, gen, neuralnet
from arc_chain_b200.formats.tokenizer import Tokenizer
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref
from arc_chain_b200.runtime import attest


def test_arc_int8_v2_layout_and_roundtrip(tmp_path):
    m = gen.random_model(preset("micro"), 0)
    p = str(tmp_path / "m.arc-int8")
    arc_int8.save(m, p)
    raw = open(p, "rb").read()
    assert raw[:10] == b"ARC-INT8\x02\x00"
    hdr = struct.unpack_from("<9Q", raw, 10)
    c = m.cfg
    assert hdr == (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.d_head, c.d_kv, c.vocab, c.max_seq)
    assert struct.unpack_from("<q", raw, 82)[0] == m.attn_scale
    m2 = arc_int8.load(p)
    assert m2.weight_hash() == m.weight_hash()
    np.testing.assert_array_equal(m2.layers[1]["down"], m.layers[1]["down"])
    assert m2.vocab == m.vocab
    # the C++ reader gives the same model (hash + generate)
    a, b = arcref.Model(m), arcref.Model(path=p)
    assert a.weight_hash() == b.weight_hash() == m.weight_hash()
    assert a.generate([5, 6, 7], 6) == b.generate([5, 6, 7], 6)


def test_native_arc_int8_writer(tmp_path):
    """arcref_save_file writes the bytes the Python writer (and the
    reference's save_weights) writes: from a loaded file, keeping its vocab
    verbatim, and from caller arrays with a given vocab."""
    m = gen.random_model(preset("micro"), 4)
    m.vocab = ["<unk>", "<s>", "\u2581h\u00e9", 'q"\\', "\t"]
    src, again, fresh = (str(tmp_path / n) for n in ("a.arc-int8", "b.arc-int8", "c.arc-int8"))
    arc_int8.save(m, src)
    raw = open(src, "rb").read()
    arcref.Model(path=src).save(again)
    assert open(again, "rb").read() == raw
    arcref.Model(m).save(fresh, vocab=m.vocab)
    assert open(fresh, "rb").read() == raw
    # array-built model without a vocab: the empty list, still loadable
    arcref.Model(m).save(fresh)
    m2 = arc_int8.load(fresh)
    assert m2.vocab == [] and m2.weight_hash() == m.weight_hash()
    assert open(fresh, "rb").read()[-10:] == struct.pack("<Q", 2) + b"[]"
    # Q4 mode changes what runs, not what is stored
    q = arcref.Model(path=src)
    q.enable_q4()
    q.save(again)
    assert open(again, "rb").read() == raw
    with pytest.raises(OSError):
        arcref.Model(m).save(str(tmp_path / "missing-dir" / "x.arc-int8"))


def test_arc_int8_minor_version_byte_ignored(tmp_path):
    m = gen.random_model(preset("micro"), 1)
    p = str(tmp_path / "m.arc-int8")
    arc_int8.save(m, p)
    raw = bytearray(open(p, "rb").read())
    raw[9] = 7
    open(p, "wb").write(bytes(raw))
    assert arc_int8.load(p).weight_hash() == m.weight_hash()
    with pytest.raises(ValueError):
        bad = str(tmp_path / "bad")
        open(bad, "wb").write(b"NOPE" + bytes(raw[4:]))
        arc_int8.load(bad)


def test_truncated_file_rejected(tmp_path):
    m = gen.random_model(preset("micro"), 1)
    p = str(tmp_path / "m.arc-int8")
    arc_int8.save(m, p)
    raw = open(p, "rb").read()
    open(p, "wb").write(raw[:len(raw) // 2])
    with pytest.raises(ValueError):
        arc_int8.load(p)
    with pytest.raises(ValueError):
        arcref.Model(path=p)


def test_v3_container_roundtrip(tmp_path):
    m = gen.random_model(preset("micro"), 2)
    m.extra["custom"] = np.arange(10, dtype=np.int64)
    p = str(tmp_path / "m.arc3")
    arc_int8.save_v3(m, p)
    m2 = arc_int8.load(p)
    assert m2.weight_hash() == m.weight_hash()
    np.testing.assert_array_equal(m2.extra["custom"], m.extra["custom"])


def test_rng_numpy_equals_cpp():
    for stream in (0, 5, 1 << 20):
        a = gen.rng_i8(7, stream, 5000)
        b = np.empty(5000, dtype=np.int8)
        arcref.rng_fill_i8(7, stream, b)
        np.testing.assert_array_equal(a, b)
        assert a.min() >= -127 and a.max() <= 127


def test_rope_tables_rust_rounding():
    assert gen.rust_round(2.5) == 3 and gen.rust_round(-2.5) == -3 and gen.rust_round(0.49999999999999994) == 0
    c, s = gen.rope_tables(64, 4)
    assert c[0] == spec.ONE and s[0] == 0 and len(c) == 4 * 32


def test_seeded_prompt_deterministic():
    p = gen.seeded_prompt(32, 32000, 1)
    assert p == gen.seeded_prompt(32, 32000, 1) and all(0 <= t < 32000 for t in p)


def test_tokenizer_longest_match_and_byte_fallback():
    vocab = ["<unk>", "<s>", "</s>", "▁", "▁he", "llo", "▁hello", "l", "o", "h", "e", "<0x21>", "▁w", "orld"]
    t = Tokenizer(vocab)
    ids = t.encode("hello world!")
    assert ids == [6, 12, 13, 11]
    assert t.decode(ids) == " hello world" + "<0x21>"
    assert t.decode([99]) == "[99]"


def test_attestation_triple_and_result_shape():
    cfg = preset("tiny")
    a = attest.attest(cfg, "hi", [3, 4], weight_hash=b"\x01" * 32)
    assert a.model_id == attest.model_id(cfg)
    assert attest.model_id_string(cfg) == "arc-2L-256d-4h-32000v"
    assert a.output_hash == spec.tokens_hash([3, 4])
    r = attest.inference_result(cfg, "hi", [1, 2], [3, 4], "x", 10.0, 1.0, "b200")
    for k in ("model", "model_hash", "input_hash", "output_hash", "tokens_generated", "ms_per_token", "deterministic"):
        assert k in r["inference"]


def test_committee_selection_and_votes():
    vs = [attest.Validator(bytes([i]) * 32, max_tier=1 + i % 4) for i in range(20)]
    c = attest.select_committee(b"\x09" * 32, vs, tier=2, k=7)
    assert len(c.members) == 7 and c.min_agreement == 5
    assert c.members == attest.select_committee(b"\x09" * 32, vs, tier=2, k=7).members
    good, bad = b"\xaa" * 32, b"\xbb" * 32
    votes = [(m, good) for m in c.members[:5]] + [(m, bad) for m in c.members[5:]]
    assert attest.aggregate_votes(c, votes)[0] == "consensus"
    votes = [(m, good) for m in c.members[:4]] + [(m, bad) for m in c.members[4:]]
    assert attest.aggregate_votes(c, votes)[0] == "disagreement"
    assert 0 < attest.corruption_probability(0.2, 7, 5) < 0.01


@pytest.mark.parametrize("base", [0, 1])
def test_neuralnet_both_tag_numberings(base):
    rng = np.random.default_rng(0)
    layers = [neuralnet.Layer("dense", W=rng.standard_normal((8, 6)).astype(np.float32) * 0.5,
                              b=np.zeros(8, np.float32)),
              neuralnet.Layer("relu"),
              neuralnet.Layer("layernorm", gamma=np.ones(8, np.float32), beta=np.zeros(8, np.float32), eps=1e-5),
              neuralnet.Layer("dense", W=rng.standard_normal((4, 8)).astype(np.float32) * 0.5,
                              b=np.zeros(4, np.float32)),
              neuralnet.Layer("softmax")]
    raw = neuralnet.write(layers, tag_base=base)
    parsed, got_base = neuralnet.parse(raw)
    assert got_base == base and [l.kind for l in parsed] == [l.kind for l in layers]
    x = rng.standard_normal(6).astype(np.float32)
    y = neuralnet.forward_f32(parsed, x)
    assert abs(float(y.sum()) - 1.0) < 1e-5
    # the integer engine version is deterministic and close
    net = neuralnet.IntegerNet(parsed)
    xi = np.array([gen.rust_round(float(v) * spec.ONE) for v in x], np.int64)
    yi = net.forward(xi)
    assert np.all(yi == net.forward(xi))
    assert abs(int(yi.sum()) - spec.ONE) < spec.ONE // 50
    with pytest.raises(ValueError):
        neuralnet.parse(raw[:-3])


def test_q4_tile_packing_layout():
    torch = pytest.importorskip("torch")
    from arc_chain_b200.ops import int_ops as ops

    rng = np.random.default_rng(1)
    M, K = 130, 200
    q = rng.integers(-8, 8, size=(M, K)).astype(np.int8)
    m = rng.integers(1, 16, size=(M, (K + 31) // 32)).astype(np.uint8)
    p = ops.pack_q4(torch.from_numpy(q), torch.from_numpy(m)).numpy()
    Mt, nch = 2, 2
    assert p.size == Mt * nch * ops.Q4_TILE
    tiles = p.reshape(Mt * nch, ops.Q4_TILE)
    for (mt, kc, r, col) in [(0, 0, 0, 0), (0, 1, 5, 71), (1, 0, 1, 33), (1, 1, 1, 71), (0, 0, 127, 127)]:
        t = tiles[mt * nch + kc]
        byte = t[r * 64 + col // 2]
        nib = (byte >> 4) if col % 2 else (byte & 15)
        grow, gcol = mt * 128 + r, kc * 128 + col
        want = q[grow, gcol] if grow < M and gcol < K else 0
        assert int(nib) - 8 == want
        mul16 = int(t[128 * 64 + r * 2]) | (int(t[128 * 64 + r * 2 + 1]) << 8)
        g = (col // 32)
        want_m = m[grow, (gcol // 32)] if grow < M and gcol < K else 1
        assert (mul16 >> (4 * g)) & 15 == want_m


def test_tp_decomposition_is_exact():
    """Row-parallel linear: the int32 per-limb partials of K shards summed
    across ranks, then recombined, equal the full reference linear."""
    rng = np.random.default_rng(2)
    M, K, tp = 64, 512, 4
    w = rng.integers(-127, 128, size=(M, K)).astype(np.int8)
    s = rng.integers(1, 1000, size=M)
    x = rng.integers(-(1 << 30), 1 << 30, size=K)
    planes = []
    r = x.copy()
    for _ in range(8):
        d = (r & 0xFF).astype(np.uint8).view(np.int8).astype(np.int64)
        planes.append(d)
        r = (r - d) >> 8
    P = np.zeros((8, M), dtype=np.int64)
    for rank in range(tp):
        sl = slice(rank * K // tp, (rank + 1) * K // tp)
        for l in range(8):
            part = w[:, sl].astype(np.int64) @ planes[l][sl]
            assert np.all(np.abs(part) < (1 << 31))  # fits the int32 exchange
            P[l] += part
    acc = sum((P[l].astype(np.uint64) << np.uint64(8 * l)) for l in range(8)).astype(np.int64)
    np.testing.assert_array_equal((acc * s) >> 16, spec.linear_i8(w, s, x))


def test_interleavings_are_permutations():
    from arc_chain_b200.models.dense import interleave_heads, interleave_pairs

    a = np.arange(2 * 8).reshape(16, 1)
    r = interleave_heads(a, 2, 8).ravel().tolist()
    assert r == [0, 4, 1, 5, 2, 6, 3, 7, 8, 12, 9, 13, 10, 14, 11, 15]
    assert interleave_pairs(np.array([1, 2]), np.array([3, 4])).tolist() == [1, 3, 2, 4]
