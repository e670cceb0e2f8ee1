"""Property-based checks (hypothesis) of the exact-integer building blocks,
over the whole i64 range where the fixed-vector tests only sample: the
signed radix-256 limb decomposition that the tensor-core GEMM relies on,
the C++ oracle's Q16 primitives against the numpy restatement, and random
NeuralNet stacks on the native library against the Python restatement."""
import numpy as np
import pytest

hyp = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

from arc_chain_b200 import spec  # noqa: E402
from arc_chain_b200.formats import neuralnet as nn  # noqa: E402
from arc_chain_b200.ops import int_ops  # noqa: E402
from arc_chain_b200.oracle import arcref  # noqa: E402

I64 = st.integers(min_value=-(1 << 63), max_value=(1 << 63) - 1)
FAST = settings(max_examples=300, deadline=None, derandomize=True)


def _wrap(v: int) -> int:
    return (v + (1 << 63)) % (1 << 64) - (1 << 63)


@FAST
@given(st.lists(st.lists(I64, min_size=3, max_size=3), min_size=1, max_size=5))
def test_limb_planes_represent_every_i64(rows):
    x = np.array(rows, dtype=np.int64)
    B = x.shape[0]
    planes, need = int_ops.limb_planes(x)
    assert 1 <= need <= 8
    for b in range(B):
        for k in range(3):
            digits = [int(planes[int_ops.limb_row(l, b, B), k]) for l in range(8)]
            assert all(-128 <= d <= 127 for d in digits)
            total = sum(d << (8 * l) for l, d in enumerate(digits[:need]))
            assert _wrap(total) == int(x[b, k])  # exact modulo 2^64 with `need` limbs
            assert all(d == 0 for d in digits[need:])


@FAST
@given(I64)
def test_q16_scalars_oracle_equals_spec(x):
    L = arcref.lib()
    assert L.arcref_integer_isqrt(x) == spec.integer_isqrt(x)
    assert L.arcref_integer_exp(x) == spec.integer_exp(x)
    assert L.arcref_silu(x) == spec.silu(x)


@FAST
@given(st.lists(st.one_of(I64, st.integers(-20 * spec.ONE, 20 * spec.ONE)), min_size=0, max_size=40))
def test_softmax_oracle_equals_spec(v):
    x = np.array(v, dtype=np.int64)
    out = np.zeros(len(x), dtype=np.int64)
    if len(x):
        arcref.lib().arcref_softmax(x.ctypes.data, len(x), out.ctypes.data)
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(out, spec.softmax(x))


@FAST
@given(st.integers(1, 6), st.integers(1, 9), st.data())
def test_wrapping_i8_matmul_oracle_equals_spec(rows, cols, data):
    w = np.array(data.draw(st.lists(st.integers(-128, 127), min_size=rows * cols, max_size=rows * cols)),
                 dtype=np.int8).reshape(rows, cols)
    s = np.array(data.draw(st.lists(I64, min_size=rows, max_size=rows)), dtype=np.int64)
    x = np.array(data.draw(st.lists(I64, min_size=cols, max_size=cols)), dtype=np.int64)
    out = np.zeros(rows, dtype=np.int64)
    arcref.lib().arcref_matmul_i8(w.ctypes.data, s.ctypes.data, x.ctypes.data, rows, cols, out.ctypes.data)
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(out, spec.linear_i8(w, s, x))


F32 = st.floats(width=32, allow_nan=True, allow_infinity=True)
SMALL = st.floats(-4, 4, width=32)


@st.composite
def nets(draw):
    """A random stack without softmax (whose exp the two sides compute
    differently) and an input for it."""
    n_in = draw(st.integers(0, 6))
    width, layers = n_in, []
    if draw(st.booleans()):
        vocab, dim = draw(st.integers(0, 5)), draw(st.integers(0, 3))
        tab = np.array(draw(st.lists(SMALL, min_size=vocab * dim, max_size=vocab * dim)), np.float32)
        layers.append(nn.Layer("embedding", table=tab.reshape(vocab, dim)))
        width = n_in * (dim if vocab else 0)
    for _ in range(draw(st.integers(0, 4))):
        kind = draw(st.sampled_from(["dense", "relu", "layernorm"]))
        if kind == "dense":
            r, c = draw(st.integers(0, 5)), draw(st.integers(0, 7))
            W = np.array(draw(st.lists(SMALL, min_size=r * c, max_size=r * c)), np.float32).reshape(r, c)
            b = np.array(draw(st.lists(SMALL, min_size=r, max_size=r)), np.float32)
            layers.append(nn.Layer("dense", W=W, b=b))
            width = r
        elif kind == "relu":
            layers.append(nn.Layer("relu"))
        else:
            k = draw(st.integers(0, 6))
            g = np.array(draw(st.lists(SMALL, min_size=k, max_size=k)), np.float32)
            bt = np.array(draw(st.lists(SMALL, min_size=k, max_size=k)), np.float32)
            layers.append(nn.Layer("layernorm", gamma=g, beta=bt, eps=draw(st.floats(float(np.float32(1e-6)), float(np.float32(1e-2)), width=32))))
    x = np.array(draw(st.lists(st.one_of(F32, st.integers(-2, 7).map(float)), min_size=n_in, max_size=n_in)),
                 np.float32)
    return layers, x


@settings(max_examples=120, deadline=None, derandomize=True)
@given(nets(), st.sampled_from([0, 1]))
def test_native_net_equals_python_restatement(case, base):
    layers, x = case
    raw = nn.write(layers, tag_base=base)
    net = nn.NativeNet.from_bytes(raw)
    parsed, got_base = nn.parse(raw)
    assert net.tag_base == got_base
    assert net.to_bytes() == nn.write(parsed, got_base)
    if got_base != base:
        # the bytes fit both numberings (only ReLU / Softmax layers, or an
        # empty LayerNorm that reads as an empty Embedding): the VM numbering
        # wins, as the VM itself would read the file
        assert got_base == 0 and nn._parse_with(raw, base)[1] == len(raw)
        layers = parsed
    else:
        assert net.to_bytes() == raw or any(
            l.kind in ("dense", "embedding") and (l.W if l.kind == "dense" else l.table).shape[0] == 0
            for l in layers)  # an empty matrix is written with 0 columns
    with np.errstate(all="ignore"):
        want = nn.forward_f32(layers, x)
    got = net.forward_f32(x)
    assert got.shape == want.shape
    nan = np.isnan(got)
    assert np.array_equal(nan, np.isnan(want))  # NaN payloads may differ; positions may not
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    xq = np.array([nn._q16(v) for v in x], np.int64)
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(net.forward_q16(xq), nn.IntegerNet(layers).forward(xq))


_FILE = {}


def _model_file(tmp_dir):
    if "raw" not in _FILE:
        import os
        from arc_chain_b200.formats import arc_int8, gen
        from arc_chain_b200.models.config import preset

        p = os.path.join(tmp_dir, "m.arc-int8")
        arc_int8.save(gen.random_model(preset("micro"), 1), p)
        _FILE["raw"] = open(p, "rb").read()
    return _FILE["raw"]


@settings(max_examples=150, deadline=None, derandomize=True)
@given(st.data())
def test_corrupted_files_load_or_raise(tmp_path_factory, data):
    """Truncations and overwritten 8-byte words anywhere in an ARC-INT8 file:
    the native and Python readers either load a model or raise ValueError;
    a size field that points past the end never reaches an allocation."""
    from arc_chain_b200.formats import arc_int8

    d = tmp_path_factory.mktemp("corrupt")
    raw = bytearray(_model_file(str(d)))
    if data.draw(st.booleans()):
        raw = raw[:data.draw(st.integers(0, len(raw) - 1))]
    else:
        off = data.draw(st.integers(0, len(raw) // 8 - 1)) * 8
        raw[off:off + 8] = data.draw(st.sampled_from([1 << 61, (1 << 64) - 1, 1 << 40, 0, 3])).to_bytes(8, "little")
    p = str(d / "c.arc-int8")
    open(p, "wb").write(bytes(raw))
    ok = []
    for load in (lambda: arcref.Model(path=p), lambda: arc_int8.load(p)):
        try:
            load()
            ok.append(True)
        except (ValueError, MemoryError, OverflowError, struct_error()):
            ok.append(False)
    assert ok[0] == ok[1]  # the two readers accept the same files


def struct_error():
    import struct

    return struct.error


def test_oracle_refuses_positions_past_the_rope_tables():
    from arc_chain_b200.formats import gen
    from arc_chain_b200.models.config import preset

    host = gen.random_model(preset("micro"), 2)  # max_seq 256
    m = arcref.Model(host)
    assert len(m.generate(list(range(3, 203)), 55)[0]) == 55  # positions 0..255
    with pytest.raises(ValueError, match="RoPE"):
        m.generate(list(range(3, 203)), 56)
