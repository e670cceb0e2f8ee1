"""The CUDA restatement of the reference's compute-shader decode path
(csrc/kernels/wgsl_path.cu) against the C++ restatement: every token and
every logit, with the reference's zero embedding and with real embedding
rows and scales large enough for non-zero activations."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.models.wgsl_path import WgslPathDevice, WgslPathHost, _Embed

pytestmark = pytest.mark.gpu


def _loud(host, seed=5):
    rng = np.random.default_rng(seed)
    for Ly in host.layers:
        for n in ("wq", "wk", "wv", "wo", "gate", "up", "down"):
            Ly[n + "_s"] = rng.integers(1 << 12, 1 << 17, size=Ly[n + "_s"].shape, dtype=np.int64)
    host.out_s = rng.integers(1 << 12, 1 << 17, size=host.out_s.shape, dtype=np.int64)
    return host


@pytest.mark.parametrize("name", ["tiny", "micro_gqa"])
@pytest.mark.parametrize("embedding", ["zero", "q16"])
def test_device_matches_host(name, embedding):
    host = _loud(gen.random_model(preset(name), 3))
    h = WgslPathHost(host, embedding=embedding)
    dv = WgslPathDevice(host, "cuda", embedding=embedding)
    emb = _Embed(host, embedding)
    toks = [1] + gen.seeded_prompt(7, host.cfg.vocab, 2)
    nxt = None
    for pos in range(len(toks) + 6):
        tok = toks[pos] if pos < len(toks) else nxt
        a = h.step(emb(tok), pos)
        b = dv.step(emb(tok), pos)
        np.testing.assert_array_equal(dv.logits.cpu().numpy(), h.logits)
        assert a == b
        nxt = a
    if embedding == "zero":
        assert nxt == 0
