"""Run configuration: one dataclass for a serving or benchmark run (model,
quantisation, TP/EP, paging, batching, speculative decoding, launch
options), loadable from TOML or JSON with ``key=value`` command-line
overrides, plus the named presets of the benchmark configurations.

Precedence follows the reference's node configuration (crates/arc-node/src/
config.rs:48-257, main.rs:133-180): command line over file over defaults.

    cfg = RunConfig.load("run.toml", overrides=["tp=2", "quant=q4-group"])
    eng = build_engine(cfg)
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

QUANTS = ("int8", "q4-row", "q4-group")


@dataclass
class RunConfig:
    model: str = "tiny"          # model preset name, or a .arc-int8 / .arc-int8v3 / .gguf path
    seed: int = 0                # random-init seed of preset weights
    quant: str = "int8"          # int8 | q4-row (the reference's enable_q4) | q4-group
    tp: int = 1                  # tensor-parallel ranks (dense models)
    ep: int = 1                  # expert-parallel ranks (MLA + MoE models)
    comm: str = "fused"          # fused (in-kernel NVLink) | nccl (baseline)
    max_seq: int = 0             # 0: the model's
    kv_pages: int = 0            # 0: sized from free memory
    max_batch: int = 32          # decode lanes of the scheduler
    prefill_chunk: int = 1024
    gen_cap: int = 0             # 0: max_seq
    draft: str = ""              # speculative decoding draft (preset or path); "" = off
    spec_k: int = 4
    eos: List[int] = field(default_factory=list)
    use_graph: bool = True       # CUDA-graph the decode step
    pdl: bool = True             # programmatic dependent launch between kernels
    attn_paged: bool = True      # TMA-fed page-ring attention
    gqa_block: bool = True       # grouped-query decode over 8+ slots: one CTA per (slot, KV head)
    device: str = "cuda"

    def __post_init__(self):
        if self.quant not in QUANTS:
            raise ValueError(f"quant must be one of {QUANTS}, got {self.quant!r}")
        if self.comm not in ("fused", "nccl"):
            raise ValueError("comm must be 'fused' or 'nccl'")
        if self.tp < 1 or self.ep < 1 or (self.tp > 1 and self.ep > 1):
            raise ValueError("tp and ep are >= 1, and at most one of them is > 1")

    # ------------------------------------------------------------ loading
    @classmethod
    def from_dict(cls, d: dict) -> "RunConfig":
        known = {f.name for f in dataclasses.fields(cls)}
        bad = sorted(set(d) - known)
        if bad:
            raise KeyError(f"unknown run config keys {bad}")
        return cls(**d)

    @classmethod
    def from_file(cls, path: str) -> "RunConfig":
        with open(path, "rb") as f:
            raw = f.read()
        if path.endswith(".toml"):
            import tomllib

            d = tomllib.loads(raw.decode())
            d = d.get("run", d)  # a [run] table or top-level keys
        else:
            d = json.loads(raw.decode())
        return cls.from_dict(d)

    def with_overrides(self, overrides: Sequence[str]) -> "RunConfig":
        """``key=value`` strings, typed by the field (lists as a,b,c)."""
        d = dataclasses.asdict(self)
        types = {f.name: f.type for f in dataclasses.fields(self)}
        for o in overrides:
            if "=" not in o:
                raise ValueError(f"override {o!r} is not key=value")
            k, v = o.split("=", 1)
            k = k.strip().replace("-", "_")
            if k not in d:
                raise KeyError(f"unknown run config key {k!r}")
            d[k] = _parse(v.strip(), str(types[k]), d[k])
        return RunConfig.from_dict(d)

    @classmethod
    def load(cls, path: Optional[str] = None, preset: Optional[str] = None,
             overrides: Sequence[str] = ()) -> "RunConfig":
        """Defaults < preset < file < overrides."""
        cfg = RUN_PRESETS[preset] if preset else cls()
        if path:
            base = dataclasses.asdict(cfg)
            with open(path, "rb") as f:
                raw = f.read()
            if path.endswith(".toml"):
                import tomllib

                d = tomllib.loads(raw.decode())
                d = d.get("run", d)
            else:
                d = json.loads(raw.decode())
            base.update(d)
            cfg = cls.from_dict(base)
        return cfg.with_overrides(overrides)

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), sort_keys=True)


def _parse(v: str, typ: str, cur):
    if "bool" in typ:
        if v.lower() in ("1", "true", "yes", "on"):
            return True
        if v.lower() in ("0", "false", "no", "off"):
            return False
        raise ValueError(f"not a bool: {v!r}")
    if "List" in typ or isinstance(cur, list):
        return [int(x) for x in v.split(",") if x.strip()]
    if "int" in typ:
        return int(v)
    return v


# The benchmark configurations as named run presets.
RUN_PRESETS = {
    "tiny": RunConfig(model="tiny", max_batch=8),
    "llama7b-decode": RunConfig(model="llama7b", max_batch=1, max_seq=400),
    "llama7b-decode-tp8": RunConfig(model="llama7b", tp=8, max_batch=1, max_seq=400),
    "llama70b-batched-tp8": RunConfig(model="llama70b", tp=8, max_batch=128, max_seq=1552),
    "dsv2lite-ep8": RunConfig(model="dsv2lite", ep=8, max_batch=32, max_seq=784),
    "spec-q4-tp8": RunConfig(model="llama7b", quant="q4-group", tp=8, draft="draft1b", spec_k=4, max_batch=8,
                             max_seq=528),
}


# ------------------------------------------------------------ construction
def is_file(model: str) -> bool:
    return os.path.sep in model or model.endswith((".arc-int8", ".arc-int8v3", ".gguf", ".bin"))


def load_host_model(cfg: RunConfig):
    """The host (numpy) model named by cfg.model."""
    from arc_chain_b200.formats import arc_int8, gen
    from arc_chain_b200.models.config import preset

    if is_file(cfg.model):
        if cfg.model.endswith(".gguf"):
            from arc_chain_b200.formats import gguf

            return gguf.load_gguf(cfg.model)
        return arc_int8.load(cfg.model)
    mc = preset(cfg.model)
    if cfg.max_seq:
        mc.max_seq = cfg.max_seq
    return gen.random_model(mc, cfg.seed)


def build_engine(cfg: RunConfig, rank: int = 0, world: int = 1, comm=None):
    """The engine for a run: dense models (INT8 / Q4, TP) or MLA + MoE (EP).
    Preset weights are generated on the device; files are uploaded."""
    import torch

    from arc_chain_b200.models import dense
    from arc_chain_b200.models.config import preset
    from arc_chain_b200.ops import int_ops as ops
    from arc_chain_b200.runtime.engine import Engine

    ops.set_pdl(cfg.pdl)
    ops.set_attn_paged(cfg.attn_paged)
    dev = torch.device(cfg.device, torch.cuda.current_device()) if cfg.device == "cuda" else torch.device(cfg.device)
    if not is_file(cfg.model) and preset(cfg.model).n_experts:
        from arc_chain_b200.models import mla_moe_engine as me

        mc = preset(cfg.model)
        if cfg.max_seq:
            mc.max_seq = cfg.max_seq
        m = me.random_device(mc, dev, cfg.seed, rank, world)
        return me.MlaMoeEngine(m, comm=comm if world > 1 else None)
    q4 = {"int8": None, "q4-row": "row", "q4-group": None}[cfg.quant]
    if is_file(cfg.model):
        m = dense.from_host(load_host_model(cfg), dev, rank, world, q4=q4)
    else:
        mc = preset(cfg.model)
        if cfg.max_seq:
            mc.max_seq = cfg.max_seq
        if cfg.quant == "q4-row":
            m = dense.from_host(load_host_model(cfg), dev, rank, world, q4="row")
        else:
            m = dense.random_device(mc, dev, seed=cfg.seed, tp_rank=rank, tp_size=world)
    if cfg.quant == "q4-group":
        m = dense.to_q4(m, "group")
    eng = Engine(m, max_seq=cfg.max_seq or None, comm=comm, n_pages=cfg.kv_pages or None)
    eng.gqa_block = bool(cfg.gqa_block)
    return eng
