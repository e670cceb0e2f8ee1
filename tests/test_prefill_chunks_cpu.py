"""Prefill chunking: the chunks cover the prompt exactly, no chunk exceeds
the chunk limit, and the slot buckets they run in pad far less than one
bucket per chunk limit would."""
import pytest

from arc_chain_b200.runtime.engine import Engine


@pytest.mark.parametrize("chunk", [16, 24, 256, 1024])
def test_chunks_cover_and_fit(chunk):
    for n in list(range(1, 300)) + [600, 1000, 1025, 2049, 4096]:
        cs = Engine.prefill_chunks(n, chunk)
        assert sum(cs) == n and all(0 < c <= chunk for c in cs)


def test_padding_is_small():
    assert Engine.prefill_chunks(600) == [512, 64, 24]
    assert Engine.prefill_chunks(129) == [128, 1]
    assert Engine.prefill_chunks(1024) == [1024]
    for n in range(65, 1025):
        slots = sum(Engine.bucket(c) for c in Engine.prefill_chunks(n))
        assert slots <= max(n + 64, 1.25 * n), (n, slots)
