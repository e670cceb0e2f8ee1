"""arc_chain_b200: deterministic integer LLM inference on B200 (sm_100a)."""
__version__ = "0.1.0"
