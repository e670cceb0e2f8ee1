"""CPU: MLA + MoE semantics (routing rule, determinism, config shapes)."""
import numpy as np

from arc_chain_b200.formats import gen
from arc_chain_b200.models import mla_moe
from arc_chain_b200.models.config import preset


def test_topk_ties_prefer_lower_index():
    p = np.array([5, 9, 9, 1, 9])
    assert mla_moe.topk(p, 3) == [1, 2, 4]
    assert mla_moe.topk(p, 1) == [1]


def test_oracle_deterministic_and_routes_topk():
    cfg = preset("micro_moe")
    m = gen.random_model(cfg, 0)
    a = mla_moe.MlaMoeOracle(m).generate([3, 4, 5], 6)
    b = mla_moe.MlaMoeOracle(m).generate([3, 4, 5], 6)
    assert a == b


def test_dsv2lite_shapes():
    cfg = preset("dsv2lite")
    s = mla_moe.shapes(cfg, 1)
    assert s["q"] == (16 * 192, 2048) and s["kva"] == (576, 2048) and s["uk"] == (16 * 512, 128)
    assert s["router"] == (64, 2048) and "gate" not in s
    assert "gate" in mla_moe.shapes(cfg, 0)
    assert 14e9 < cfg.n_params() < 17e9
