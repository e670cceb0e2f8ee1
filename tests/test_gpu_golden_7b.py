"""Full-size end-to-end check: the 7B-architecture decoder (seeded random
INT8 weights generated on the device) generates the CPU oracle's pinned
256-token output, bit for bit (CUDA-graph decode steps, chunked prefill
with the chunk attention kernel)."""
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.bench import golden
from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    from arc_chain_b200.models import dense
    from arc_chain_b200.runtime.engine import Engine

    cfg = preset(golden.MODEL)
    cfg.max_seq = 400
    m = dense.random_device(cfg, torch.device("cuda", 0), seed=golden.WEIGHT_SEED)
    eng = Engine(m, max_seq=400, n_pages=64)
    yield eng
    del eng, m
    torch.cuda.empty_cache()


def test_7b_generates_pinned_oracle_tokens(engine):
    from arc_chain_b200.utils.hashing import blake3
    import numpy as np

    prompt = gen.seeded_prompt(golden.PROMPT_LEN, engine.m.cfg.vocab, golden.PROMPT_SEED)
    toks, h = engine.generate(prompt, 256)
    assert toks == golden.TOKENS_256
    assert h.hex() == golden.OUTPUT_HASH_256
    assert blake3(np.asarray(toks, dtype="<u4").tobytes()).hex() == golden.OUTPUT_HASH_256
    assert engine.check_errors() == 0
