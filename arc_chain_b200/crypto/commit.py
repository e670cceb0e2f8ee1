"""Batch transaction commitments and Merkle roots (BLAKE3 derive-key mode).

Item i is committed as ``derive_key("ARC-chain-tx-v1", [domain_i] ++ data_i)``
(the domain byte only in the domain-separated form), as the reference's
``cpu_batch_commit`` / ``cpu_batch_commit_domain`` / ``gpu_batch_commit``
(crates/arc-gpu/src/lib.rs:70-91, 183-400; kernel crates/arc-gpu/src/blake3.wgsl).
The Merkle root hashes adjacent pairs of 32-byte nodes with the same
commitment, padding an odd layer with a zero hash; no leaves give the zero
hash and one leaf is its own root (lib.rs:414-460).

GPU path: ``csrc/aux/blake3.cu`` (one thread per item; one launch per
Merkle layer).  CPU path: ``csrc/ref/arcref.cpp`` (threaded), the oracle.
"""
from __future__ import annotations

import ctypes as C
from functools import lru_cache
from typing import List, Optional, Sequence

import numpy as np

TX_CONTEXT = "ARC-chain-tx-v1"


def _ref():
    from arc_chain_b200.oracle import arcref

    return arcref.lib()


@lru_cache(maxsize=16)
def context_key(context: str = TX_CONTEXT) -> np.ndarray:
    """Key words of derive_key(context, .) (the material hasher's key)."""
    k = np.zeros(8, dtype=np.uint32)
    c = context.encode()
    _ref().arcref_blake3_context_key(c, len(c), k.ctypes.data_as(C.c_void_p))
    return k


def derive_key(context: str, data: bytes) -> bytes:
    """BLAKE3 derive_key(context, data) (32 bytes), CPU."""
    lib = _ref()
    c = context.encode()
    h = lib.arcref_blake3_new_derive(c, len(c))
    try:
        b = np.frombuffer(bytes(data), dtype=np.uint8)
        if b.size:
            lib.arcref_blake3_update(h, b.ctypes.data_as(C.c_void_p), b.size)
        out = np.zeros(32, dtype=np.uint8)
        lib.arcref_blake3_finalize(h, out.ctypes.data_as(C.c_void_p))
        return out.tobytes()
    finally:
        lib.arcref_blake3_free(h)


def keyed_hash(key: bytes, data: bytes) -> bytes:
    """BLAKE3 keyed_hash(key (32 bytes), data), CPU."""
    assert len(key) == 32
    lib = _ref()
    k = np.frombuffer(key, dtype=np.uint8).copy()
    h = lib.arcref_blake3_new_keyed(k.ctypes.data_as(C.c_void_p))
    try:
        b = np.frombuffer(bytes(data), dtype=np.uint8)
        if b.size:
            lib.arcref_blake3_update(h, b.ctypes.data_as(C.c_void_p), b.size)
        out = np.zeros(32, dtype=np.uint8)
        lib.arcref_blake3_finalize(h, out.ctypes.data_as(C.c_void_p))
        return out.tobytes()
    finally:
        lib.arcref_blake3_free(h)


def pack(items: Sequence[bytes]):
    """Concatenate items into one byte buffer padded to 16 bytes, plus offsets."""
    lens = np.fromiter((len(x) for x in items), dtype=np.int64, count=len(items))
    offs = np.zeros(len(items) + 1, dtype=np.int64)
    np.cumsum(lens, out=offs[1:])
    total = int(offs[-1])
    buf = np.zeros((total + 15) // 16 * 16 or 16, dtype=np.uint8)
    if total:
        buf[:total] = np.frombuffer(b"".join(bytes(x) for x in items), dtype=np.uint8)
    return buf, offs


def batch_commit_cpu(items: Sequence[bytes], domains: Optional[Sequence[int]] = None,
                     context: str = TX_CONTEXT) -> List[bytes]:
    buf, offs = pack(items)
    n = len(items)
    out = np.zeros((max(n, 1), 32), dtype=np.uint8)
    d = None if domains is None else np.asarray(domains, dtype=np.uint8)
    c = context.encode()
    if n:
        _ref().arcref_blake3_batch_commit(buf.ctypes.data_as(C.c_void_p), offs.ctypes.data_as(C.c_void_p), n,
                                          None if d is None else d.ctypes.data_as(C.c_void_p), c, len(c),
                                          out.ctypes.data_as(C.c_void_p))
    return [out[i].tobytes() for i in range(n)]


def merkle_root_cpu(leaves: Sequence[bytes], context: str = TX_CONTEXT) -> bytes:
    n = len(leaves)
    a = np.frombuffer(b"".join(leaves), dtype=np.uint8).copy() if n else np.zeros(32, np.uint8)
    out = np.zeros(32, dtype=np.uint8)
    c = context.encode()
    _ref().arcref_merkle_root(a.ctypes.data_as(C.c_void_p), n, c, len(c), out.ctypes.data_as(C.c_void_p))
    return out.tobytes()


# ---------------------------------------------------------------- GPU
def batch_commit_device(buf, offs, domains=None, context: str = TX_CONTEXT, max_item_len: Optional[int] = None):
    """Commitments of the items packed in device tensors: ``buf`` uint8 (length
    a multiple of 4), ``offs`` int64 [n + 1], ``domains`` uint8 [n] or None.
    Returns a uint8 tensor [n, 32] on the same device."""
    import torch

    from arc_chain_b200.ops import int_ops
    from arc_chain_b200.ops._lib import lib

    n = offs.numel() - 1
    out = torch.empty((max(n, 0), 32), dtype=torch.uint8, device=buf.device)
    if n <= 0:
        return out
    if max_item_len is None:
        max_item_len = int((offs[1:] - offs[:-1]).max().item())
    k = context_key(context)
    int_ops.check(lib().arcb_blake3_batch_commit(buf.data_ptr(), buf.numel(), offs.data_ptr(), n,
                                                 None if domains is None else domains.data_ptr(),
                                                 k.ctypes.data_as(C.c_void_p), max_item_len, out.data_ptr(),
                                                 int_ops._s()), "blake3_batch_commit")
    return out


def batch_commit(items: Sequence[bytes], domains: Optional[Sequence[int]] = None, context: str = TX_CONTEXT,
                 device: str = "cuda") -> List[bytes]:
    """Commitments of host items on the GPU (pinned host -> device copy,
    kernel, device -> host copy)."""
    import torch

    buf, offs = pack(items)
    n = len(items)
    if n == 0:
        return []
    dev = torch.device(device)
    tb = torch.from_numpy(buf).pin_memory().to(dev, non_blocking=True)
    to = torch.from_numpy(offs).pin_memory().to(dev, non_blocking=True)
    td = None
    if domains is not None:
        td = torch.from_numpy(np.asarray(domains, dtype=np.uint8)).to(dev)
    lens = offs[1:] - offs[:-1]
    out = batch_commit_device(tb, to, td, context, int(lens.max()))
    h = out.cpu().numpy()
    return [h[i].tobytes() for i in range(n)]


def merkle_root_device(leaves, context: str = TX_CONTEXT):
    """Merkle root of device leaves (uint8 [n, 32]); returns a uint8 [32] tensor."""
    import torch

    from arc_chain_b200.ops import int_ops
    from arc_chain_b200.ops._lib import lib

    n = leaves.shape[0]
    dev = leaves.device
    out = torch.empty(32, dtype=torch.uint8, device=dev)
    scratch = torch.empty(max(2, 2 * ((n + 1) // 2)) * 32, dtype=torch.uint8, device=dev)
    k = context_key(context)
    int_ops.check(lib().arcb_merkle_root(leaves.contiguous().data_ptr() if n else None, n,
                                         k.ctypes.data_as(C.c_void_p), scratch.data_ptr(), out.data_ptr(),
                                         int_ops._s()), "merkle_root")
    return out


def merkle_root(leaves: Sequence[bytes], context: str = TX_CONTEXT, device: str = "cuda") -> bytes:
    import torch

    n = len(leaves)
    if n == 0:
        return bytes(32)
    t = torch.from_numpy(np.frombuffer(b"".join(leaves), dtype=np.uint8).copy().reshape(n, 32)).to(device)
    return merkle_root_device(t, context).cpu().numpy().tobytes()
