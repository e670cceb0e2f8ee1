"""The native NeuralNet reader / writer / forward passes
(csrc/ref/neuralnet.cpp) against the Python restatement
(arc_chain_b200/formats/neuralnet.py) and against the reference VM's own test
vectors (crates/arc-vm/src/inference.rs:1050-1450, read as text)."""
import struct

import numpy as np
import pytest

from arc_chain_b200 import spec
from arc_chain_b200.formats import neuralnet as nn
from arc_chain_b200.formats.neuralnet import Layer, NativeNet

f32 = np.float32


def dense(W, b):
    return Layer("dense", W=np.asarray(W, f32), b=np.asarray(b, f32))


def lnorm(g, b, eps=1e-5):
    return Layer("layernorm", gamma=np.asarray(g, f32), beta=np.asarray(b, f32), eps=eps)


def emb(t):
    return Layer("embedding", table=np.asarray(t, f32))


def random_net(rng, with_softmax=True, start_emb=False):
    layers = []
    width = 7
    if start_emb:
        layers.append(emb(rng.standard_normal((11, 3)) * 0.7))
        width = 3 * 4  # four token indices in
    dims = [width, 9, 13, 6]
    for i in range(len(dims) - 1):
        layers.append(dense(rng.standard_normal((dims[i + 1], dims[i])) * 0.4, rng.standard_normal(dims[i + 1]) * 0.1))
        layers.append(Layer("relu") if i % 2 == 0 else lnorm(rng.standard_normal(dims[i + 1]) * 0.5 + 1,
                                                            rng.standard_normal(dims[i + 1]) * 0.1))
    if with_softmax:
        layers.append(Layer("softmax"))
    return layers, width


def same_layers(a, b):
    assert [l.kind for l in a] == [l.kind for l in b]
    for x, y in zip(a, b):
        for f in ("W", "b", "gamma", "beta", "table"):
            u, v = getattr(x, f), getattr(y, f)
            if u is not None and v is not None:
                np.testing.assert_array_equal(np.asarray(u, f32).reshape(-1), np.asarray(v, f32).reshape(-1))
        if x.kind == "layernorm":
            assert f32(x.eps) == f32(y.eps)


# ----------------------------------------------------------------- reference vectors
def test_reference_dense_relu_small_network():
    net = NativeNet.from_layers([dense([[1, 0, -1], [0, 1, 2]], [0.5, -0.5])])
    assert list(net.forward_f32([1, 2, 3])) == [-1.5, 7.5]
    net = NativeNet.from_layers([Layer("relu")])
    assert list(net.forward_f32([-3.0, -0.1, 0.0, 0.5, 2.0])) == [0.0, 0.0, 0.0, 0.5, 2.0]
    net = NativeNet.from_layers([dense([[1, -1, 0], [0, 1, 1]], [0, 0]), Layer("relu"), dense([[1, 1]], [0.1])])
    out = net.forward_f32([1, 2, 3])
    assert len(out) == 1 and abs(out[0] - 5.1) < 1e-5


def test_reference_softmax_and_layernorm():
    out = NativeNet.from_layers([Layer("softmax")]).forward_f32([1, 2, 3, 4])
    assert abs(float(nn._fold(out)) - 1.0) < 1e-6 and np.all(out > 0) and np.all(np.diff(out) >= 0)
    out = NativeNet.from_layers([lnorm([1] * 4, [0] * 4)]).forward_f32([2, 4, 6, 8])
    mean = nn._fold(out) / f32(4)
    assert abs(mean) < 1e-5 and abs(nn._fold((out - mean) ** 2) / f32(4) - 1) < 1e-4
    out = NativeNet.from_layers([lnorm([2] * 4, [1] * 4)]).forward_f32([2, 4, 6, 8])
    assert abs(nn._fold(out) / f32(4) - 1) < 1e-4


def test_reference_embedding_and_roundtrip():
    net = NativeNet.from_layers([emb([[10, 20], [30, 40], [50, 60]])])
    assert list(net.forward_f32([2, 0, 1])) == [50, 60, 10, 20, 30, 40]
    assert (net.input_size, net.output_size) == (3, 2)
    layers = [emb([[0.1, 0.2, 0.3], [0.4, 0.5, 0.6], [0.7, 0.8, 0.9]]), lnorm([1] * 3, [0] * 3),
              dense([[1, 0.5, -0.5], [0, 1, 0]], [0.1, -0.1]), Layer("relu"), Layer("softmax")]
    a = NativeNet.from_layers(layers)
    b = NativeNet.from_bytes(a.to_bytes())
    assert (b.input_size, b.output_size) == (3, 2)
    x = [0.0, 1.0, 2.0]
    np.testing.assert_array_equal(a.forward_f32(x), b.forward_f32(x))


def test_reference_classifier_through_run_request():
    layers = [dense([[0.5, -0.3, 0.1, 0.2], [-0.1, 0.4, 0.3, -0.2], [0.2, 0.1, -0.4, 0.5]], [0, 0, 0]),
              Layer("relu"), dense([[1, -1, 0.5], [-0.5, 1, 0.3]], [0, 0]), Layer("softmax")]
    net = NativeNet.from_bytes(nn.write(layers))
    r = nn.run_request(net, "embedding", [1.0, 0.5, -0.5, 0.2])
    assert len(r.output) == 2 and abs(float(nn._fold(r.output)) - 1) < 1e-5
    assert (r.tokens_used, r.compute_time_ms, r.cost) == (4, 18, 20)
    first = net.forward_f32([1.0, -0.5, 0.25, 0.0])
    for _ in range(20):
        np.testing.assert_array_equal(net.forward_f32([1.0, -0.5, 0.25, 0.0]), first)


def test_reference_truncation_errors():
    for raw in (b"", b"\0\0", struct.pack("<I", 1), struct.pack("<I", 1) + bytes([0]) + struct.pack("<II", 2, 2)):
        with pytest.raises(ValueError):
            NativeNet.from_bytes(raw)
        with pytest.raises(ValueError):
            nn.parse(raw)


# ----------------------------------------------------------------- native vs Python
@pytest.mark.parametrize("base", [0, 1])
@pytest.mark.parametrize("start_emb", [False, True])
def test_parse_and_write_agree(base, start_emb):
    rng = np.random.default_rng(3 + base + 2 * start_emb)
    layers, _ = random_net(rng, start_emb=start_emb)
    raw = nn.write(layers, tag_base=base)
    net = NativeNet.from_bytes(raw)
    py_layers, py_base = nn.parse(raw)
    assert net.tag_base == py_base == base
    same_layers(net.layers(), py_layers)
    assert net.to_bytes() == raw
    assert net.to_bytes(1 - base) == nn.write(layers, tag_base=1 - base)
    assert NativeNet.from_layers(layers).to_bytes(base) == raw


@pytest.mark.parametrize("seed", range(4))
def test_forward_f32_bitwise_without_exp(seed):
    rng = np.random.default_rng(seed)
    layers, width = random_net(rng, with_softmax=False, start_emb=seed % 2 == 1)
    net = NativeNet.from_layers(layers)
    for _ in range(5):
        if seed % 2:  # token indices, some fractional, some out of range
            x = rng.integers(-2, 13, size=4).astype(f32) + rng.random(4).astype(f32)
        else:
            x = rng.standard_normal(width).astype(f32) * 2
        np.testing.assert_array_equal(net.forward_f32(x), nn.forward_f32(layers, x))


def test_softmax_within_one_ulp_of_python():
    rng = np.random.default_rng(9)
    net = NativeNet.from_layers([Layer("softmax")])
    for n in (1, 2, 5, 64, 1000):
        x = (rng.standard_normal(n) * 6).astype(f32)
        np.testing.assert_array_max_ulp(net.forward_f32(x), nn.softmax_f32(x), maxulp=1)


@pytest.mark.parametrize("seed", range(4))
def test_forward_q16_matches_integer_net(seed):
    rng = np.random.default_rng(20 + seed)
    layers, width = random_net(rng, with_softmax=True, start_emb=seed % 2 == 1)
    net = NativeNet.from_layers(layers)
    ref = nn.IntegerNet(layers)
    for _ in range(4):
        if seed % 2:
            x = rng.integers(-3, 14, size=4).astype(np.int64) * spec.ONE + rng.integers(0, spec.ONE, size=4)
        else:
            x = rng.integers(-3 * spec.ONE, 3 * spec.ONE, size=width).astype(np.int64)
        np.testing.assert_array_equal(net.forward_q16(x), ref.forward(x))


# ----------------------------------------------------------------- reference semantics at the edges
def test_trailing_bytes_use_the_vm_numbering():
    raw = nn.write([dense([[1, 2]], [0.5]), Layer("relu")], tag_base=0) + b"\x07\x07\x07"
    net = NativeNet.from_bytes(raw)
    layers, base = nn.parse(raw)
    assert net.tag_base == base == 0 and [l.kind for l in layers] == ["dense", "relu"]
    assert list(net.forward_f32([1, 1])) == [3.5]


def test_unknown_tag_and_oversized_layer_count():
    with pytest.raises(ValueError, match="unknown layer tag"):
        NativeNet.from_bytes(struct.pack("<I", 1) + bytes([9]))
    with pytest.raises(ValueError):
        NativeNet.from_bytes(struct.pack("<I", 0xFFFFFFFF) + bytes([1]))


def test_embedding_index_saturates():
    t = [[1, 2], [3, 4], [5, 6]]
    x = np.array([-5.0, -0.5, np.nan, 2.9, 3.0, np.inf, 1e30], f32)
    want = [1, 2, 1, 2, 1, 2, 5, 6, 0, 0, 0, 0, 0, 0]
    assert list(NativeNet.from_layers([emb(t)]).forward_f32(x)) == want
    assert list(nn.forward_f32([emb(t)], x)) == want
    xq = np.array([-5 * spec.ONE, -1, 2 * spec.ONE + 7, 3 * spec.ONE], np.int64)
    q = np.array([[spec.ONE, 2 * spec.ONE], [3 * spec.ONE, 4 * spec.ONE], [5 * spec.ONE, 6 * spec.ONE]], np.int64)
    want_q = [q[0, 0], q[0, 1], q[0, 0], q[0, 1], q[2, 0], q[2, 1], 0, 0]
    assert list(NativeNet.from_layers([emb(t)]).forward_q16(xq)) == want_q
    assert list(nn.IntegerNet([emb(t)]).forward(xq)) == want_q


def test_empty_layers():
    e = Layer("embedding", table=np.zeros((0, 5), f32))
    d = Layer("dense", W=np.zeros((0, 4), f32), b=np.zeros(0, f32))
    raw = nn.write([e])
    assert struct.unpack_from("<II", raw, 5) == (0, 0)
    assert NativeNet.from_layers([e]).to_bytes() == raw
    assert len(NativeNet.from_layers([e]).forward_f32([1.0, 2.0])) == 0
    assert len(nn.forward_f32([e], np.array([1.0, 2.0], f32))) == 0
    assert NativeNet.from_layers([d]).to_bytes() == nn.write([d])
    assert struct.unpack_from("<II", nn.write([d]), 5) == (0, 0)
    ln = lnorm([1.0], [0.0])
    assert len(NativeNet.from_layers([ln]).forward_q16(np.zeros(0, np.int64))) == 0
    assert len(nn.IntegerNet([ln]).forward(np.zeros(0, np.int64))) == 0
    assert len(NativeNet.from_layers([Layer("softmax")]).forward_f32([])) == 0


def test_softmax_nan_and_infinity_propagate():
    # a NaN input makes its exp and so the sum NaN; an all -inf or a +inf
    # input subtracts infinities: every output is NaN, in both restatements
    sm = NativeNet.from_layers([Layer("softmax")])
    for x in ([np.nan, 1.0, 2.0], [-np.inf, -np.inf], [np.inf, 0.0]):
        x = np.array(x, f32)
        assert np.all(np.isnan(sm.forward_f32(x))) and np.all(np.isnan(nn.softmax_f32(x)))
    x = np.array([-np.inf, 0.0, 1.0], f32)  # one -inf is an exact zero weight
    got = sm.forward_f32(x)
    assert got[0] == 0 and np.all(got[1:] > 0)
    np.testing.assert_array_max_ulp(got, nn.softmax_f32(x), maxulp=1)


def test_layernorm_sums_fold_from_negative_zero():
    ln = lnorm([1.0, 1.0], [-0.0, -0.0])
    x = np.array([-0.0, -0.0], f32)
    got = NativeNet.from_layers([ln]).forward_f32(x)
    want = nn.forward_f32([ln], x)
    # from -0.0 the mean of [-0, -0] is -0, x - mean is +0 and the output +0;
    # a fold from +0.0 would give mean +0, x - mean = -0 and outputs -0
    assert np.array_equal(np.signbit(got), np.signbit(want)) and not np.any(np.signbit(got))


def test_q16_conversion_saturates():
    big = dense([[1.0]], [3e38])
    assert list(NativeNet.from_layers([big]).forward_q16(np.zeros(1, np.int64))) == \
        list(nn.IntegerNet([big]).forward(np.zeros(1, np.int64)))
    assert nn._q16(float("nan")) == 0 and nn._q16(1e300) == (1 << 63) - 1 and nn._q16(-1e300) == -(1 << 63)


def test_run_request_kinds():
    layers = [dense(np.eye(3) * 2, [0.5, -0.5, 1.0])]
    net = NativeNet.from_layers(layers)
    r = nn.run_request(net, "text", "AbC")
    y = net.forward_f32(np.array([65, 98, 67], f32))
    assert r.output == nn.decode_text(y) and r.tokens_used == 3 and r.cost == 15
    # outputs 6.5, -0.5 and 6e9 cast to u32 with saturation
    r = nn.run_request(net, "tokens", [3, 0, 3_000_000_000])
    assert r.output == [6, 0, 4294967295] and r.tokens_used == 3
    r = nn.run_request(net, "image", bytes([0, 255, 51]))
    assert [c for c, _ in r.output] == ["class_0", "class_1", "class_2"] and r.tokens_used == 10
    assert abs(sum(p for _, p in r.output) - 1) < 1e-6
    empty = NativeNet.from_layers([Layer("embedding", table=np.zeros((0, 0), f32))])
    assert nn.run_request(empty, "image", b"\x01").output == [("unknown", 1.0)]


def test_decode_text():
    # |v| * 100 in f32, saturating cast to u32, mod 128, +32 below 32
    v = np.array([0.0, -0.33, np.nan, np.inf, 0.5, 1.0, 0.05], f32)
    assert nn.decode_text(v) == " ! \x7f2d%"


# ----------------------------------------------------------------- the VM's model registry
def _mid(seed):
    return bytes([seed]) + bytes(31)


def test_engine_registry_rules():
    from arc_chain_b200.runtime.nn_engine import EngineConfig, ModelInfo, NNEngine

    raw = nn.write([dense([[0.5, -0.3, 0.1, 0.2], [-0.1, 0.4, 0.3, -0.2]], [0, 0]), Layer("relu")], tag_base=1)
    eng = NNEngine(EngineConfig(max_loaded_models=2))
    eng.load_model(_mid(1), ModelInfo("a"), raw)
    with pytest.raises(ValueError, match="already loaded"):
        eng.load_model(_mid(1), ModelInfo("a"), raw)
    eng.load_model(_mid(2), ModelInfo("b"))  # registered without weights
    with pytest.raises(ValueError, match=r"Maximum loaded models \(2\) reached"):
        eng.load_model(_mid(3), ModelInfo("c"), raw)
    with pytest.raises(ValueError, match="without weights"):
        eng.run(_mid(2), "tokens", [1])
    with pytest.raises(ValueError, match="Model not loaded"):
        eng.run(_mid(9), "tokens", [1])
    assert eng.unload_model(_mid(2)) and not eng.unload_model(_mid(2))
    with pytest.raises(ValueError):  # bytes that parse under neither numbering: no mock
        eng.load_model(_mid(4), ModelInfo("bad"), bytes([0xFF, 0xFE, 0xAB]))
    assert eng.loaded_models() == [_mid(1)] and eng.model_status(_mid(1)) == "Ready"


def test_engine_stats_accumulate():
    from arc_chain_b200.runtime.nn_engine import ModelInfo, NNEngine

    eng = NNEngine()
    eng.load_model(_mid(8), ModelInfo("s"), nn.write([dense(np.eye(3), [0, 0, 0])]))
    assert (eng.stats().total_inferences, eng.stats().total_tokens) == (0, 0)
    r = eng.run(_mid(8), "tokens", [1, 2, 3])
    assert r.output == [1, 2, 3] and (r.tokens_used, r.compute_time_ms, r.cost) == (3, 16, 15)
    eng.run(_mid(8), "text", "hello")
    s = eng.stats()
    assert (s.total_inferences, s.total_tokens, s.avg_latency_ms) == (2, 8, (16 + 20) // 2)
    assert eng.model_status(_mid(8)) == "Ready" and eng.models[_mid(8)].last_used == 2


def test_quantiser_nan_and_infinite_rows_match_native():
    """NaN entries are skipped by the row maximum and quantise to 0; an
    infinite maximum saturates the scale's integer cast (both restatements)."""
    W = np.array([[np.nan, 0.5, -2.0], [np.inf, 1.0, 0.0], [-np.inf, np.nan, 3.0], [0.25, -0.75, 0.0]], f32)
    layer = dense(W, [0.0, 0.0, 0.0, 0.0])
    for x in ([spec.ONE, 2 * spec.ONE, -spec.ONE], [0, 0, 0], [7, -3, 65536 * 100]):
        x = np.array(x, np.int64)
        with np.errstate(over="ignore"):
            np.testing.assert_array_equal(NativeNet.from_layers([layer]).forward_q16(x), nn.IntegerNet([layer]).forward(x))
    from arc_chain_b200.formats.quantize import quantize_f32

    q, s = quantize_f32(W.reshape(-1), 4, 3)
    assert list(q[0]) == [0, 32, -127] and s[0] == (2 * spec.ONE + 126) // 127
    # inv = 127 / inf = 0 and inf * 0 is NaN, which quantises to 0; i64::MAX * ONE
    # wraps to -ONE, and (-ONE + 126) / 127 < 1 gives scale 1
    assert list(q[1]) == [0, 0, 0] and s[1] == 1
    # a finite maximum in [2^62, 2^63) keeps its own value: (am * ONE) wraps
    big = np.array([[2.0 ** 62 * 1.5, 1.0]], f32)
    am = int(np.float32(2.0 ** 62 * 1.5))
    num = ((am * spec.ONE + 126 + (1 << 63)) % (1 << 64)) - (1 << 63)
    want = max(1, -(abs(num) // 127) if num < 0 else num // 127)
    assert quantize_f32(big.reshape(-1), 1, 2)[1][0] == want
