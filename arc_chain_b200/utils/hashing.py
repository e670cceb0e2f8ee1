"""BLAKE3 for the attestation triple, backed by the in-tree C++ implementation
(``csrc/ref/blake3.cpp``).  The reference hashes with BLAKE3 everywhere
(crates/arc-crypto/src/hash.rs:77-80)."""
from __future__ import annotations

import ctypes as C

import numpy as np


def blake3(data) -> bytes:
    from arc_chain_b200.oracle import arcref

    return arcref.blake3(data)


class Blake3:
    """Incremental hasher; accepts bytes or numpy arrays (hashed as raw bytes)."""

    def __init__(self):
        from arc_chain_b200.oracle import arcref

        self._lib = arcref.lib()
        self._h = self._lib.arcref_blake3_new()

    def update(self, data) -> "Blake3":
        if isinstance(data, np.ndarray):
            a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        else:
            a = np.frombuffer(bytes(data), dtype=np.uint8)
        if a.size:
            self._lib.arcref_blake3_update(self._h, a.ctypes.data_as(C.c_void_p), a.size)
        return self

    def push_chunk_cv(self, cv: np.ndarray, total_chunks: int) -> None:
        cv = np.ascontiguousarray(cv, dtype=np.uint32)
        self._lib.arcref_blake3_push_chunk_cv(self._h, cv.ctypes.data_as(C.c_void_p), total_chunks)

    def digest(self) -> bytes:
        out = np.zeros(32, dtype=np.uint8)
        self._lib.arcref_blake3_finalize(self._h, out.ctypes.data_as(C.c_void_p))
        return out.tobytes()

    def hexdigest(self) -> str:
        return self.digest().hex()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.arcref_blake3_free(h)
            self._h = None
