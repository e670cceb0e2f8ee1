"""Run configuration (TOML / JSON / overrides / presets), the command-line
tools on the CPU oracle, sharded checkpoints, the reference's second Q4
format, and the reference's tier and error rules."""
import json
import math
import os

import numpy as np
import pytest

from arc_chain_b200 import cli, spec
from arc_chain_b200.config import RUN_PRESETS, RunConfig
from arc_chain_b200.formats import arc_int8, gen, quantize, sharded
from arc_chain_b200.models.config import preset
from arc_chain_b200.oracle import arcref
from arc_chain_b200.runtime import attest


def _run(capsys, *argv):
    assert cli.main(list(argv)) == 0
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1])


# ------------------------------------------------------------ run config
def test_config_precedence_and_types(tmp_path):
    p = tmp_path / "run.toml"
    p.write_text('[run]\nmodel = "tiny"\nmax_batch = 4\nquant = "q4-group"\n')
    c = RunConfig.load(str(p), preset="llama7b-decode", overrides=["seed=3", "eos=2,0", "use_graph=off"])
    assert (c.model, c.max_batch, c.quant, c.seed, c.eos, c.use_graph) == ("tiny", 4, "q4-group", 3, [2, 0], False)
    assert c.max_seq == RUN_PRESETS["llama7b-decode"].max_seq  # from the preset, not overridden
    j = tmp_path / "run.json"
    j.write_text(json.dumps({"model": "micro", "tp": 2}))
    assert RunConfig.from_file(str(j)).tp == 2
    assert RunConfig.from_dict(json.loads(c.to_json())) == c


@pytest.mark.parametrize("bad", [["quant=fp8"], ["nosuch=1"], ["tp=2", "ep=2"], ["max_batch"]])
def test_config_rejects(bad):
    with pytest.raises((ValueError, KeyError)):
        RunConfig().with_overrides(bad)


def test_presets_name_the_benchmark_configs():
    assert RUN_PRESETS["llama70b-batched-tp8"].tp == 8 and RUN_PRESETS["dsv2lite-ep8"].ep == 8
    s = RUN_PRESETS["spec-q4-tp8"]
    assert (s.quant, s.draft, s.spec_k, s.max_batch) == ("q4-group", "draft1b", 4, 8)


# ------------------------------------------------------------ CLI on the oracle
def test_cli_info(capsys):
    r = _run(capsys, "info", "tiny")
    host = gen.random_model(preset("tiny"), 0)
    assert r["weight_hash"] == host.weight_hash().hex() and r["tier"] == 1
    assert r["model_id"] == attest.model_id_string(host.cfg)


def test_cli_nn_run(capsys, tmp_path):
    from arc_chain_b200.formats import neuralnet as nn

    f = np.float32
    layers = [nn.Layer("dense", W=np.array([[0.5, -0.3, 0.1, 0.2], [-0.1, 0.4, 0.3, -0.2]], f),
                       b=np.zeros(2, f)), nn.Layer("relu"), nn.Layer("softmax")]
    path = tmp_path / "clf.bin"
    path.write_bytes(nn.write(layers, tag_base=1))  # create_model.py numbering
    r = _run(capsys, "nn-run", str(path), "--embedding", "1,0.5,-0.5,0.2")
    assert (r["tag_base"], r["input_size"], r["output_size"], r["tokens_used"]) == (1, 4, 2, 4)
    want = nn.NativeNet.from_layers(layers).forward_f32(np.array([1, 0.5, -0.5, 0.2], f))
    assert r["output"] == [float(v) for v in want]
    r = _run(capsys, "nn-run", str(path), "--embedding", "1,0.5,-0.5,0.2", "--integer")
    assert r["output_q16"] == [int(v) for v in nn.IntegerNet(layers).forward(
        np.array([65536, 32768, -32768, 13107], np.int64))]
    r = _run(capsys, "nn-run", str(path), "--text", "hi")
    assert len(r["output"]) == 2 and r["tokens_used"] == 2


def test_cli_bench_int8_roundtrip_and_determinism(capsys, tmp_path):
    path = str(tmp_path / "tiny.arc-int8")
    r = _run(capsys, "bench-int8", "tiny", "--device", "cpu", "--runs", "3", "--tokens", "4", "--save", path)
    assert r["deterministic"] and r["reload_weight_hash_equal"] and len(r["output_hashes"]) == 3
    r2 = _run(capsys, "bench-int8", path, "--device", "cpu", "--runs", "1", "--tokens", "4")
    assert r2["output_hashes"][0] == r["output_hashes"][0]


def test_cli_generate_oracle_matches_engine_api(capsys):
    r = _run(capsys, "generate", "--preset", "tiny", "--oracle", "--prompt-ids", "5,6,7", "--max-tokens", "6")
    host = gen.random_model(preset("tiny"), 0)
    toks, h = arcref.Model(host).generate([5, 6, 7], 6)
    assert r["output_hash_blake3"] == h.hex()
    assert r["attestation"]["output_hash"] == attest.output_hash(toks).hex()
    assert r["inference"]["output_tokens"] == toks


def test_cli_perplexity_cpu(capsys):
    r = _run(capsys, "perplexity", "tiny", "--device", "cpu", "--seeded", "12")
    host = gen.random_model(preset("tiny"), 0)
    toks = gen.seeded_prompt(12, host.cfg.vocab, 7)
    cache = arcref.Model(host).new_cache()
    rows = [cache.forward(t) for t in [1] + toks[:-1]][1:]
    nll = -sum(cli.log_softmax_f64(row)[t] for row, t in zip(rows, toks[1:]))
    assert r["tokens_evaluated"] == 11 and math.isclose(r["avg_nll"], nll / 11, rel_tol=1e-12)
    assert math.isclose(r["perplexity"], math.exp(nll / 11), rel_tol=1e-12)


def test_perplexity_out_of_vocab_is_nan_like_the_reference():
    r = cli.perplexity_from_logits([np.zeros(8, np.int64)], [99], 8)
    assert math.isnan(r["perplexity"])


def test_cli_convert_v2_v3(capsys, tmp_path):
    v2, v3 = str(tmp_path / "a.arc-int8"), str(tmp_path / "a.arc-int8v3")
    r = _run(capsys, "convert", "micro", v2)
    r3 = _run(capsys, "convert", v2, v3)
    assert r["weight_hash"] == r3["weight_hash"] == arc_int8.load(v3).weight_hash().hex()


# ------------------------------------------------------------ sharded checkpoints
@pytest.mark.parametrize("tp", [1, 2, 4])
def test_sharded_roundtrip(tmp_path, tp):
    cfg = preset("micro_gqa") if tp < 4 else preset("tiny")
    if tp == 4:
        cfg.d_ff = 768
    host = gen.random_model(cfg, 1)
    man = sharded.save_sharded(host, str(tmp_path), tp)
    assert man["tp"] == tp and man["weight_hash"] == host.weight_hash().hex() and len(man["files"]) == tp
    full = sharded.assemble(str(tmp_path))
    assert full.weight_hash() == host.weight_hash()
    s1 = sharded.load_shard(str(tmp_path), tp - 1)
    k = cfg.d_ff // tp
    np.testing.assert_array_equal(s1.layers[0]["down"], host.layers[0]["down"][:, (tp - 1) * k:])
    lo, hi = sharded.vocab_range(cfg.vocab, tp - 1, tp)
    np.testing.assert_array_equal(s1.out, host.out[lo:hi])


def test_sharded_detects_tampering(tmp_path):
    host = gen.random_model(preset("micro"), 0)
    man = sharded.save_sharded(host, str(tmp_path), 2)
    path = os.path.join(str(tmp_path), man["files"][1])
    b = bytearray(open(path, "rb").read())
    b[-100] ^= 1
    open(path, "wb").write(bytes(b))
    with pytest.raises(ValueError):
        sharded.load_shard(str(tmp_path), 1)


def test_cli_shard(capsys, tmp_path):
    r = _run(capsys, "shard", "micro", str(tmp_path / "s"), "--tp", "2")
    assert r["manifest"]["files"] == ["rank0.arc-int8v3", "rank1.arc-int8v3"]


# ------------------------------------------------------------ second Q4 format
def test_q4_engine_format_equals_engine_q4():
    host = gen.random_model(preset("micro"), 2)
    rng = np.random.default_rng(0)
    for n in ("wq", "down"):
        w, s = host.layers[0][n], host.layers[0][n + "_s"]
        packed, s4 = quantize.q4_engine_from_i8(w, s)
        v_ref, s_ref = spec.q4_from_i8(w, s)
        np.testing.assert_array_equal(quantize.q4_engine_values(packed), v_ref)
        np.testing.assert_array_equal(s4, s_ref)
        np.testing.assert_array_equal(packed, spec.q4_pack(v_ref))
        x = rng.integers(-(1 << 20), 1 << 20, size=w.shape[1], dtype=np.int64)
        np.testing.assert_array_equal(quantize.matmul_q4_engine(packed, s4, x), spec.linear_i8(v_ref, s_ref, x))


# ------------------------------------------------------------ tiers and errors
def test_tiers_and_errors():
    assert [attest.tier_min_stake(t) for t in (1, 2, 3, 4)] == [1000, 5000, 10000, 25000]
    assert attest.tier_max_params_b(4) is None and attest.tier_from_u8(5) is None
    attest.check_eligibility(1, 7_000_000_000, 1000)
    with pytest.raises(attest.ModelTooLarge, match="model too large for tier 1"):
        attest.check_eligibility(1, 70_000_000_000, 10**9)
    with pytest.raises(attest.InsufficientStake, match="have 10, need 5000"):
        attest.check_eligibility(2, 7_000_000_000, 10)
    assert str(attest.DeterminismViolation()) == "determinism violation: output mismatch"
