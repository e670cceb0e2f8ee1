"""GPU BLAKE3 (chunk-parallel, subtree merge) against the CPU hasher."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("sizes", [[1], [1024], [1025], [3000, 17, 4096], [1 << 20, 5, (1 << 21) + 333],
                                   [8 * 1024 * 1024 + 7]])
def test_device_blake3_matches_cpu(sizes):
    from arc_chain_b200.utils.hashing import DeviceBlake3

    rng = np.random.default_rng(sum(sizes))
    parts = [rng.integers(0, 256, size=n, dtype=np.uint8) for n in sizes]
    dev = torch.device("cuda")
    h = DeviceBlake3(dev, level=4)
    for p in parts:  # one update per segment: carries cross chunk boundaries
        h.update(torch.from_numpy(p).to(dev))
    assert h.digest() == arcref.blake3(np.concatenate(parts).tobytes())


def test_seeded_weight_hash_on_device_equals_host():
    from arc_chain_b200.models import dense

    cfg = preset("micro_gqa")
    host = gen.random_model(cfg, 4)
    assert dense.weight_hash_seeded(cfg, 4, "cuda") == host.weight_hash() == arcref.Model(host).weight_hash()
