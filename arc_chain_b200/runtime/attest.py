"""InferenceAttestation: the (model hash, input hash, output hash) triple,
the serving API's result shape, replica-committee agreement and tiers.

* model id  = BLAKE3("arc-{n_layers}L-{d_model}d-{n_heads}h-{vocab}v")
  (crates/arc-node/src/rpc.rs:2763-2769); the weight hash
  (cached_integer_model.rs:1598-1617) identifies the exact weights;
* input hash = BLAKE3(input text bytes) (rpc.rs:2774);
* output hash = BLAKE3(generated ids as LE u32) (cached_integer_model.rs:
  1553-1555).
The transaction body fields follow InferenceAttestationBody
(crates/arc-types/src/transaction.rs:541-552).

Committee (crates/arc-inference/src/committee.rs:69-170): members are the
top-k eligible validators by BLAKE3(seed || address); a result is accepted
when at least min(5, k) members report the same output hash.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from arc_chain_b200.utils.hashing import blake3

DEFAULT_COMMITTEE_SIZE = 7
MIN_AGREEMENT = 5


def model_id_string(cfg) -> str:
    return f"arc-{cfg.n_layers}L-{cfg.d_model}d-{cfg.n_heads}h-{cfg.vocab}v"


def model_id(cfg) -> bytes:
    return blake3(model_id_string(cfg).encode())


def input_hash(text: str) -> bytes:
    return blake3(text.encode())


def output_hash(tokens: Sequence[int]) -> bytes:
    return blake3(np.asarray(list(tokens), dtype="<u4").tobytes())


def hx(b: bytes) -> str:
    return "0x" + b.hex()


@dataclass
class InferenceAttestation:
    model_id: bytes
    input_hash: bytes
    output_hash: bytes
    challenge_period: int = 100
    bond: int = 0
    weight_hash: Optional[bytes] = None

    def body(self) -> dict:
        d = {"model_id": hx(self.model_id), "input_hash": hx(self.input_hash),
             "output_hash": hx(self.output_hash), "challenge_period": self.challenge_period, "bond": self.bond}
        if self.weight_hash is not None:
            d["weight_hash"] = hx(self.weight_hash)
        return d


def attest(cfg, text: str, tokens: Sequence[int], weight_hash: Optional[bytes] = None,
           challenge_period: int = 100, bond: int = 0) -> InferenceAttestation:
    return InferenceAttestation(model_id(cfg), input_hash(text), output_hash(tokens), challenge_period, bond,
                                weight_hash)


def inference_result(cfg, text: str, prompt_tokens: Sequence[int], tokens: Sequence[int], output_text: str,
                     inference_ms: float, encode_ms: float, engine: str) -> dict:
    """The JSON the reference's POST /inference/run returns (rpc.rs:2820-2845)."""
    n = len(tokens)
    return {"success": True, "inference": {
        "model": model_id_string(cfg), "model_hash": hx(model_id(cfg)), "input": text,
        "input_tokens": len(prompt_tokens), "input_hash": hx(input_hash(text)), "output": output_text,
        "output_tokens": list(map(int, tokens)), "output_hash": hx(output_hash(tokens)),
        "tokens_generated": n, "inference_ms": int(inference_ms), "ms_per_token": int(inference_ms // n) if n else 0,
        "encode_ms": int(encode_ms), "deterministic": True, "engine": engine}}


# ------------------------------------------------------------------ committee
@dataclass
class Validator:
    address: bytes
    max_tier: int
    stake: int = 0


@dataclass
class Committee:
    members: List[bytes]
    seed: bytes
    tier: int
    min_agreement: int


def select_committee(seed: bytes, eligible: Iterable[Validator], tier: int, k: int = DEFAULT_COMMITTEE_SIZE) -> Committee:
    cands = [(v.address, blake3(seed + v.address)) for v in eligible if v.max_tier >= tier]
    cands.sort(key=lambda x: x[1])
    return Committee([a for a, _ in cands[:k]], seed, tier, min(MIN_AGREEMENT, k))


def aggregate_votes(c: Committee, votes: Sequence[Tuple[bytes, bytes]]):
    """Returns ("consensus", output_hash, agreeing, total) or
    ("disagreement", valid_votes, total)."""
    members = set(c.members)
    valid = [(a, h) for a, h in votes if a in members]
    counts: Dict[bytes, int] = {}
    for _, h in valid:
        counts[h] = counts.get(h, 0) + 1
    for h, n in counts.items():
        if n >= c.min_agreement:
            return ("consensus", h, n, len(c.members))
    return ("disagreement", valid, len(c.members))


def corruption_probability(f: float, k: int, min_agree: int) -> float:
    return sum(math.comb(k, i) * f ** i * (1 - f) ** (k - i) for i in range(min_agree, k + 1))


# ------------------------------------------------------------------ tiers
# Tiers by parameter count (crates/arc-inference/src/lib.rs:24-98): tier 1
# up to 20B, tier 2 up to 50B, tier 3 up to 100B, tier 4 beyond; tiers >= 2
# need a committee.
TIER_LIMITS = ((1, 20e9), (2, 50e9), (3, 100e9), (4, float("inf")))


def tier_for_params(n_params: float) -> int:
    for t, lim in TIER_LIMITS:
        if n_params <= lim:
            return t
    return 4


def needs_committee(tier: int) -> bool:
    return tier >= 2


# Minimum stake per tier in base units (crates/arc-inference/src/lib.rs:61-68).
TIER_MIN_STAKE = {1: 1_000, 2: 5_000, 3: 10_000, 4: 25_000}


def tier_min_stake(tier: int) -> int:
    return TIER_MIN_STAKE[int(tier)]


def tier_max_params_b(tier: int) -> Optional[int]:
    """Largest model (billions of parameters) a tier runs; None = unlimited."""
    return {1: 20, 2: 50, 3: 100, 4: None}[int(tier)]


def tier_from_u8(v: int) -> Optional[int]:
    return int(v) if int(v) in TIER_MIN_STAKE else None


# ------------------------------------------------------------------ errors
# The reference's InferenceError variants (crates/arc-inference/src/lib.rs:22-42),
# as exception classes with the same fields and messages.
class InferenceError(Exception):
    pass


class ModelNotFound(InferenceError):
    def __init__(self, model: str):
        super().__init__(f"model not found: {model}")
        self.model = model


class ModelTooLarge(InferenceError):
    def __init__(self, tier: int, size: int, max: int):
        super().__init__(f"model too large for tier {tier}: {size} params, max {max}")
        self.tier, self.size, self.max = tier, size, max


class InferenceTimeout(InferenceError):
    def __init__(self, elapsed_ms: int, limit_ms: int):
        super().__init__(f"execution timeout: {elapsed_ms}ms > {limit_ms}ms")
        self.elapsed_ms, self.limit_ms = elapsed_ms, limit_ms


class DeterminismViolation(InferenceError):
    def __init__(self):
        super().__init__("determinism violation: output mismatch")


class InsufficientStake(InferenceError):
    def __init__(self, tier: int, have: int, need: int):
        super().__init__(f"insufficient stake for tier {tier}: have {have}, need {need}")
        self.tier, self.have, self.need = tier, have, need


class RuntimeFailure(InferenceError):
    def __init__(self, msg: str):
        super().__init__(f"inference error: {msg}")


def check_eligibility(tier: int, n_params: int, stake: int) -> None:
    """Raises ModelTooLarge / InsufficientStake like the reference's tier checks."""
    mx = tier_max_params_b(tier)
    if mx is not None and n_params > mx * 1_000_000_000:
        raise ModelTooLarge(tier, n_params, mx * 1_000_000_000)
    need = tier_min_stake(tier)
    if stake < need:
        raise InsufficientStake(tier, stake, need)
