"""GGUF import: the container reader and dequantisers against the ``gguf``
package, and the imported model against the reference loader's rules."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

from arc_chain_b200 import spec
from arc_chain_b200.formats import gguf as G
from arc_chain_b200.formats.quantize import quantize_f32

QT = gguf.GGMLQuantizationType
TYPES = [QT.F32, QT.F16, QT.BF16, QT.Q4_0, QT.Q4_1, QT.Q5_0, QT.Q5_1, QT.Q8_0, QT.Q4_K, QT.Q5_K, QT.Q6_K]


# byte offsets of the f16 fields of each block type (set to finite values in random blocks)
F16_FIELDS = {QT.Q4_0: [0], QT.Q4_1: [0, 2], QT.Q5_0: [0], QT.Q5_1: [0, 2], QT.Q8_0: [0], QT.Q4_K: [0, 2],
              QT.Q5_K: [0, 2], QT.Q6_K: [208]}


@pytest.mark.parametrize("qt", TYPES, ids=lambda t: t.name)
def test_dequantize_matches_package(qt):
    rng = np.random.default_rng(int(qt))
    name, be, bb = G.TYPES[int(qt)]
    n = 8 * 512
    if be == 1:
        x = (rng.standard_normal(n) * 0.05).astype(np.float32)
        raw = np.asarray(gguf.quants.quantize(x.reshape(8, 512), qt)).view(np.uint8).reshape(8, -1)
    else:
        raw = rng.integers(0, 256, size=(n // be, bb), dtype=np.uint8)
        for o in F16_FIELDS[qt]:
            raw[:, o:o + 2] = (rng.standard_normal(n // be) * 0.01).astype(np.float16).view(np.uint8).reshape(-1, 2)
        raw = raw.reshape(8, -1)
    want = np.asarray(gguf.quants.dequantize(raw, qt), dtype=np.float32).reshape(-1)
    got = G.dequantize(raw.reshape(-1), int(qt), n)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def _write_llama(path, qt, V=64, d=32, nh=4, nkv=2, ff=64, nl=2, tie=False):
    rng = np.random.default_rng(3)
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(nl)
    w.add_embedding_length(d)
    w.add_head_count(nh)
    w.add_head_count_kv(nkv)
    w.add_feed_forward_length(ff)
    w.add_token_list([f"t{i}" for i in range(V)])
    tensors = {}

    def add(name, shape, quant=True, scale=0.1):
        a = (rng.standard_normal(shape) * scale).astype(np.float32)
        if quant and qt != QT.F32:
            data = gguf.quants.quantize(a, qt)
            w.add_tensor(name, data, raw_shape=data.shape, raw_dtype=qt)
            a = np.asarray(gguf.quants.dequantize(data, qt), dtype=np.float32).reshape(shape)
        else:
            w.add_tensor(name, a)
        tensors[name] = a

    dh = d // nh
    add("token_embd.weight", (V, d))
    if not tie:
        add("output.weight", (V, d))
    add("output_norm.weight", (d,), quant=False, scale=1.0)
    for l in range(nl):
        p = f"blk.{l}"
        add(f"{p}.attn_q.weight", (d, d))
        add(f"{p}.attn_k.weight", (dh * nkv, d))
        add(f"{p}.attn_v.weight", (dh * nkv, d))
        add(f"{p}.attn_output.weight", (d, d))
        add(f"{p}.ffn_gate.weight", (ff, d))
        add(f"{p}.ffn_up.weight", (ff, d))
        add(f"{p}.ffn_down.weight", (d, ff))
        add(f"{p}.attn_norm.weight", (d,), quant=False, scale=1.0)
        add(f"{p}.ffn_norm.weight", (d,), quant=False, scale=1.0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


@pytest.mark.parametrize("qt,tie", [(QT.F32, False), (QT.Q8_0, True), (QT.Q4_0, False)], ids=str)
def test_import_rules(qt, tie, tmp_path):
    path = tmp_path / "m.gguf"
    t = _write_llama(path, qt, tie=tie)
    m = G.load_gguf(str(path))
    c = m.cfg
    assert (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.vocab, c.max_seq) == (2, 32, 4, 2, 64, 64, 2048)
    assert m.vocab == [f"t{i}" for i in range(64)]
    assert m.attn_scale == spec.integer_isqrt(8 * spec.ONE)
    e, es = quantize_f32(t["token_embd.weight"], 64, 32)
    np.testing.assert_array_equal(m.emb, e)
    v = t["token_embd.weight"].astype(np.float64) * 65536  # Rust f64::round: half away from zero
    np.testing.assert_array_equal(m.emb_q16, np.where(v >= 0, np.floor(v + 0.5), np.ceil(v - 0.5)))
    src = t["token_embd.weight"] if tie else t["output.weight"]
    np.testing.assert_array_equal(m.out, quantize_f32(src, 64, 32)[0])
    np.testing.assert_array_equal(m.layers[1]["wk"], quantize_f32(t["blk.1.attn_k.weight"], 16, 32)[0])
    np.testing.assert_array_equal(m.layers[0]["attn_norm"], G.norm_q16(t["blk.0.attn_norm.weight"]))


def test_imported_model_runs_on_oracle(tmp_path):
    from arc_chain_b200.oracle import arcref

    path = tmp_path / "m.gguf"
    _write_llama(path, QT.Q8_0)
    m = G.load_gguf(str(path))
    m.cfg.max_seq = 2048
    om = arcref.Model(m)
    toks, h = om.generate([1, 5, 9], 8)
    assert len(toks) >= 1
    # the Q16 embedding table is what the forward reads: changing it changes the output
    m2 = G.load_gguf(str(path))
    m2.emb_q16 = (m2.emb.astype(np.int64) * m2.emb_s[:, None])
    assert arcref.Model(m2).generate([1, 5, 9], 8)[0] == arcref.Model(_i8_only(m2)).generate([1, 5, 9], 8)[0]


def _i8_only(m):
    m.emb_q16 = None
    return m


def test_q16_rounding_saturates_like_rust():
    v = np.array([np.nan, np.inf, -np.inf, 1e30, -1e30, 2.5, -2.5, 0.49999997, -0.5], np.float32)
    got = G._round_half_away(v)
    i64 = np.iinfo(np.int64)
    assert list(got) == [0, i64.max, i64.min, i64.max, i64.min, 3, -3, 0, -1]


def test_corrupted_gguf_loads_or_raises(tmp_path):
    """Truncations and overwritten 8-byte words of a GGUF file: the importer
    loads a model or raises an ordinary error; it never hangs on a corrupted
    count or length field."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    src = tmp_path / "m.gguf"
    _write_llama(src, QT.Q8_0)
    base = src.read_bytes()

    @hyp.settings(max_examples=60, deadline=None, derandomize=True)
    @hyp.given(st.data())
    def prop(data):
        raw = bytearray(base)
        if data.draw(st.booleans()):
            raw = raw[:data.draw(st.integers(0, len(raw) - 1))]
        else:
            off = data.draw(st.integers(0, len(raw) // 8 - 1)) * 8
            raw[off:off + 8] = data.draw(st.sampled_from([1 << 61, (1 << 64) - 1, 1 << 33, 0, 7])).to_bytes(8, "little")
        p = tmp_path / "c.gguf"
        p.write_bytes(bytes(raw))
        try:
            G.load_gguf(str(p))
        except (ValueError, KeyError, IndexError, TypeError, OverflowError, MemoryError, UnicodeDecodeError,
                AssertionError, ZeroDivisionError, struct_error()):
            pass

    prop()


def struct_error():
    import struct

    return struct.error
