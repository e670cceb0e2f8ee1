"""The small full-sequence integer transformer: native C++ against the numpy
restatement, determinism, and the benchmark document shape."""
import numpy as np

from arc_chain_b200.models.toy_integer import NumpyToy, ToyIntegerModel


def test_native_matches_numpy_restatement():
    for cfg in [(50, 32, 2, 64, 2), (100, 64, 2, 128, 1), (30, 48, 3, 40, 1)]:
        m, n = ToyIntegerModel(*cfg), NumpyToy(*cfg)
        for toks in ([1, 2, 3], [1, 2, 3, 4, 5], [7], [cfg[0] - 1, 0, cfg[0] + 5]):
            np.testing.assert_array_equal(m.forward(toks), n.forward(toks))


def test_generate_deterministic_and_full_recompute():
    m = ToyIntegerModel(100, 64, 2, 128, 2)
    a = m.generate_with_hash([1, 5, 10, 15], 8, 99)
    for _ in range(20):
        assert m.generate_with_hash([1, 5, 10, 15], 8, 99) == a
    # each step equals the argmax of a full forward over prompt + generated
    toks = [1, 5, 10, 15]
    for t in a[0]:
        assert int(np.argmax(m.forward(toks))) == t
        toks.append(t)


def test_bench_document():
    from arc_chain_b200.bench import integer_bench

    doc = integer_bench.run(runs=3)
    assert doc["benchmark"] == "IntegerEngine" and len(doc["models"]) == 3
    for r in doc["models"]:
        assert r["deterministic"] and len(r["output_hash"]) == 64 and len(r["generated_tokens"]) >= 1
