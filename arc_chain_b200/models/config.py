"""Model architecture configs and the named presets.

The dense decoder config mirrors the reference's ``ModelConfig``
(crates/arc-inference/src/cached_integer_model.rs:135-148) and the nine u64
header fields of the ARC-INT8 v2 file (cached_integer_model.rs:1565-1569).
The MLA/MoE fields describe a DeepSeek-V2-Lite-style trunk, which the
reference does not have; their integer semantics are defined in
``arc_chain_b200.spec``.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Optional

ONE = 1 << 16


@dataclass
class ModelConfig:
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_ff: int
    d_head: int
    vocab: int
    max_seq: int = 2048
    rope_theta: float = 10000.0
    attn_scale: Optional[int] = None  # Q16; default isqrt(d_head * ONE)
    # --- MLA (DeepSeek-V2 style); 0 = standard MHA/GQA attention
    kv_lora_rank: int = 0
    qk_nope_dim: int = 0
    qk_rope_dim: int = 0
    v_head_dim: int = 0
    # --- MoE; n_experts == 0 = dense FFN in every layer
    n_experts: int = 0
    n_shared_experts: int = 0
    moe_top_k: int = 0
    moe_d_ff: int = 0
    first_dense_layers: int = 0  # leading layers that keep the dense FFN
    name: str = ""

    @property
    def d_kv(self) -> int:
        return self.n_kv_heads * self.d_head

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    def resolved_attn_scale(self) -> int:
        if self.attn_scale is not None:
            return int(self.attn_scale)
        from arc_chain_b200 import spec

        dh = (self.qk_nope_dim + self.qk_rope_dim) if self.is_mla else self.d_head
        # GGUF-loader convention: isqrt(d_head * ONE) = ONE / sqrt(d_head)
        # (cached_integer_model.rs:1759).
        return spec.integer_isqrt(dh * ONE)

    def n_params(self) -> int:
        d = self.d_model
        per = 0
        if self.is_mla:
            qd = self.n_heads * (self.qk_nope_dim + self.qk_rope_dim)
            per += qd * d + (self.kv_lora_rank + self.qk_rope_dim) * d
            per += self.n_heads * (self.qk_nope_dim + self.v_head_dim) * self.kv_lora_rank
            per += d * self.n_heads * self.v_head_dim
        else:
            per += d * d * 2 + 2 * self.d_kv * d
        dense_ffn = 3 * d * self.d_ff
        if self.is_moe:
            moe = (self.n_experts + self.n_shared_experts) * 3 * d * self.moe_d_ff + self.n_experts * d
            ffn = self.first_dense_layers * dense_ffn + (self.n_layers - self.first_dense_layers) * moe
        else:
            ffn = self.n_layers * dense_ffn
        return self.n_layers * per + ffn + 2 * self.vocab * d

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), sort_keys=True)

    @staticmethod
    def from_json(s: str) -> "ModelConfig":
        return ModelConfig(**json.loads(s))


PRESETS = {
    # 2L, d=256, 4 x 64 MHA, SwiGLU 688, vocab 32000
    "tiny": ModelConfig(n_layers=2, d_model=256, n_heads=4, n_kv_heads=4, d_ff=688, d_head=64,
                        vocab=32000, name="tiny"),
    # Llama-2-7B architecture
    "llama7b": ModelConfig(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=32, d_ff=11008,
                           d_head=128, vocab=32000, name="llama7b"),
    # Llama-2-70B architecture (GQA 64/8)
    "llama70b": ModelConfig(n_layers=80, d_model=8192, n_heads=64, n_kv_heads=8, d_ff=28672,
                            d_head=128, vocab=32000, name="llama70b"),
    # 1B Llama-style draft model for speculative decoding
    "draft1b": ModelConfig(n_layers=16, d_model=2048, n_heads=16, n_kv_heads=16, d_ff=5632,
                           d_head=128, vocab=32000, name="draft1b"),
    # DeepSeek-V2-Lite-style MLA + MoE
    "dsv2lite": ModelConfig(n_layers=27, d_model=2048, n_heads=16, n_kv_heads=16, d_ff=10944,
                            d_head=128, vocab=102400, kv_lora_rank=512, qk_nope_dim=128,
                            qk_rope_dim=64, v_head_dim=128, n_experts=64, n_shared_experts=2,
                            moe_top_k=6, moe_d_ff=1408, first_dense_layers=1, name="dsv2lite"),
    # Small test shapes (not benchmark configs)
    "micro": ModelConfig(n_layers=2, d_model=128, n_heads=2, n_kv_heads=2, d_ff=256, d_head=64,
                         vocab=512, max_seq=256, name="micro"),
    "micro_gqa": ModelConfig(n_layers=2, d_model=256, n_heads=4, n_kv_heads=2, d_ff=384,
                             d_head=64, vocab=1024, max_seq=256, name="micro_gqa"),
    "micro_moe": ModelConfig(n_layers=3, d_model=256, n_heads=4, n_kv_heads=4, d_ff=512,
                             d_head=64, vocab=1024, max_seq=256, kv_lora_rank=128,
                             qk_nope_dim=64, qk_rope_dim=32, v_head_dim=64, n_experts=8,
                             n_shared_experts=2, moe_top_k=3, moe_d_ff=128,
                             first_dense_layers=1, name="micro_moe"),
}


def preset(name: str) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; have {sorted(PRESETS)}")
    return dataclasses.replace(PRESETS[name])
