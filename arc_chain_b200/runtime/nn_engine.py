"""The VM's model registry for NeuralNet files (``InferenceEngine``,
crates/arc-vm/src/inference.rs:528-811) over the native network library.

Models are keyed by a 32-byte id.  The registry keeps the reference's rules:
a second load of the same id and a load beyond ``max_loaded_models`` fail
with its messages; a request for an id that is not loaded, or whose model is
not Ready, fails; every request adds to the statistics (inferences, tokens,
and the average of the reported latency ``tokens * 2 + 10`` ms, which is the
reference's formula, not a measurement).

One deliberate difference: the reference silently serves a mock (reversed
text, echoed tokens) when a model has no weights or its bytes do not parse.
Here unparsable bytes raise at load time, and a model registered without
weights raises when it is run.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

from arc_chain_b200.formats import neuralnet

READY, BUSY, UNLOADED, LOADING = "Ready", "Busy", "Unloaded", "Loading"


@dataclass
class ModelInfo:
    name: str
    model_type: str = ""
    parameter_count: int = 0
    quantization: str = ""
    max_context: int = 0


@dataclass
class EngineConfig:
    max_loaded_models: int = 4
    default_timeout_ms: int = 5000
    max_tokens: int = 2048
    temperature: float = 0.7


@dataclass
class Stats:
    total_inferences: int = 0
    total_tokens: int = 0
    avg_latency_ms: int = 0
    cache_hits: int = 0


@dataclass
class LoadedModel:
    id: bytes
    info: ModelInfo
    net: Optional[neuralnet.NativeNet]
    status: str = READY
    last_used: int = 0


@dataclass
class Response:
    model_id: bytes
    output: object
    tokens_used: int
    compute_time_ms: int
    cost: int


@dataclass
class NNEngine:
    config: EngineConfig = field(default_factory=EngineConfig)
    models: Dict[bytes, LoadedModel] = field(default_factory=dict)
    _stats: Stats = field(default_factory=Stats)
    _total_latency_ms: int = 0

    def load_model(self, model_id: bytes, info: ModelInfo, model_data: Optional[bytes] = None) -> None:
        """Registers a model; ``model_data`` is a NeuralNet file image
        (either tag numbering).  Raises ValueError when the bytes do not
        parse, or when the id is loaded already or the engine is full."""
        model_id = _check_id(model_id)
        if model_id in self.models:
            raise ValueError("Model is already loaded")
        if len(self.models) >= self.config.max_loaded_models:
            raise ValueError(f"Maximum loaded models ({self.config.max_loaded_models}) reached")
        net = neuralnet.NativeNet.from_bytes(model_data) if model_data else None
        self.models[model_id] = LoadedModel(model_id, info, net)

    def unload_model(self, model_id: bytes) -> bool:
        return self.models.pop(_check_id(model_id), None) is not None

    def model_status(self, model_id: bytes) -> Optional[str]:
        m = self.models.get(_check_id(model_id))
        return None if m is None else m.status

    def loaded_models(self) -> List[bytes]:
        return list(self.models)

    def stats(self) -> Stats:
        return self._stats

    def run(self, model_id: bytes, kind: str, payload) -> Response:
        """One request: ``kind`` is text / tokens / embedding / image, as
        :func:`arc_chain_b200.formats.neuralnet.run_request` takes it."""
        m = self.models.get(_check_id(model_id))
        if m is None:
            raise ValueError("Model not loaded")
        if m.status != READY:
            raise ValueError(f"Model is {m.status.lower()}")
        if m.net is None:
            raise ValueError(f"Model {m.info.name!r} was registered without weights")
        m.status = BUSY
        try:
            r = neuralnet.run_request(m.net, kind, payload)
        finally:
            m.status = READY
        m.last_used += 1
        s = self._stats
        s.total_inferences += 1
        s.total_tokens += r.tokens_used
        self._total_latency_ms += r.compute_time_ms
        s.avg_latency_ms = self._total_latency_ms // s.total_inferences
        return Response(model_id, r.output, r.tokens_used, r.compute_time_ms, r.cost)


def _check_id(model_id: bytes) -> bytes:
    model_id = bytes(model_id)
    if len(model_id) != 32:
        raise ValueError("a model id is 32 bytes")
    return model_id
