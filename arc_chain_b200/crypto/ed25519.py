"""Ed25519 batch signature verification on the GPU (``csrc/aux/ed25519.cu``).

Strict rule as the reference's batch verifier (``verify_strict``,
crates/arc-gpu/src/lib.rs:470-495; kernel
crates/arc-gpu/src/cuda/ed25519_verify.cu:432-494); the oracle is
``ed25519_ref.verify_strict``.  Result codes per signature: 0 valid,
1 S not canonical, 2 / 3 A / R do not decompress, 4 / 5 A / R of small
order, 6 equation fails.

    ok = verify_batch(messages, signatures, public_keys)   # list of bool
"""
from __future__ import annotations

import ctypes as C
import hashlib
from typing import List, Sequence

import numpy as np

from arc_chain_b200.crypto import ed25519_ref as ref

_INIT = set()
CODES = {0: "valid", 1: "S not canonical", 2: "A invalid", 3: "R invalid", 4: "A small order",
         5: "R small order", 6: "equation mismatch"}


def _words(x: int, n: int) -> np.ndarray:
    return np.array([(x >> (64 * i)) & ((1 << 64) - 1) for i in range(n)], dtype=np.uint64)


def _host_constants():
    K, H = ref.sha512_constants()
    curve = np.array(ref.curve_constants(), dtype=np.int32)
    table = np.array(ref.base_table(), dtype=np.int32).reshape(-1)
    return (curve, np.array(K, dtype=np.uint64), np.array(H, dtype=np.uint64), _words(ref.L, 4),
            _words(ref.barrett_mu(), 5), table)


_CONST = None


def init(device=None) -> None:
    """Upload the curve constants and the base-point table to a device (once)."""
    global _CONST
    import torch

    from arc_chain_b200.ops import int_ops
    from arc_chain_b200.ops._lib import lib

    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx in _INIT:
        return
    if _CONST is None:
        _CONST = _host_constants()
    with torch.cuda.device(idx):
        ptrs = [a.ctypes.data_as(C.c_void_p) for a in _CONST]
        int_ops.check(lib().arcb_ed25519_init(*ptrs), "ed25519_init")
    _INIT.add(idx)


def verify_device(sigs, pks, msgs, offs):
    """Device tensors: sigs uint8 [n, 64], pks uint8 [n, 32], msgs uint8
    (packed messages), offs int64 [n + 1].  Returns int32 codes [n]."""
    import torch

    from arc_chain_b200.ops import int_ops
    from arc_chain_b200.ops._lib import lib

    init(sigs.device)
    n = sigs.shape[0]
    out = torch.empty(n, dtype=torch.int32, device=sigs.device)
    if n:
        int_ops.check(lib().arcb_ed25519_verify(sigs.data_ptr(), pks.data_ptr(), msgs.data_ptr(), offs.data_ptr(), n,
                                                out.data_ptr(), int_ops._s()), "ed25519_verify")
    return out


def verify_prehashed_device(records):
    """records uint8 [n, 128] = [R | S | k | A], k = SHA-512(R || A || M)
    (reduced mod L on the device).  Returns int32 codes [n]."""
    import torch

    from arc_chain_b200.ops import int_ops
    from arc_chain_b200.ops._lib import lib

    init(records.device)
    n = records.shape[0]
    out = torch.empty(n, dtype=torch.int32, device=records.device)
    if n:
        int_ops.check(lib().arcb_ed25519_verify_prehashed(records.data_ptr(), n, out.data_ptr(), int_ops._s()),
                      "ed25519_verify_prehashed")
    return out


def pack(messages: Sequence[bytes], signatures: Sequence[bytes], public_keys: Sequence[bytes]):
    n = len(messages)
    assert len(signatures) == n and len(public_keys) == n
    sig = np.frombuffer(b"".join(bytes(s) for s in signatures), dtype=np.uint8).reshape(n, 64) if n else \
        np.zeros((0, 64), np.uint8)
    pk = np.frombuffer(b"".join(bytes(k) for k in public_keys), dtype=np.uint8).reshape(n, 32) if n else \
        np.zeros((0, 32), np.uint8)
    lens = np.fromiter((len(m) for m in messages), dtype=np.int64, count=n)
    offs = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lens, out=offs[1:])
    msg = np.zeros(max(16, int(offs[-1])), dtype=np.uint8)
    if offs[-1]:
        msg[:offs[-1]] = np.frombuffer(b"".join(bytes(m) for m in messages), dtype=np.uint8)
    return sig, pk, msg, offs


def verify_codes(messages: Sequence[bytes], signatures: Sequence[bytes], public_keys: Sequence[bytes],
                 device: str = "cuda") -> np.ndarray:
    import torch

    if any(len(s) != 64 for s in signatures) or any(len(k) != 32 for k in public_keys):
        raise ValueError("signatures are 64 bytes and public keys 32 bytes")
    sig, pk, msg, offs = pack(messages, signatures, public_keys)
    dev = torch.device(device)
    t = [torch.from_numpy(a.copy()).to(dev) for a in (sig, pk, msg, offs)]
    return verify_device(*t).cpu().numpy()


def verify_batch(messages: Sequence[bytes], signatures: Sequence[bytes], public_keys: Sequence[bytes],
                 device: str = "cuda") -> List[bool]:
    """Per-signature results (the reference's cpu_batch_verify_ed25519 shape)."""
    return [c == 0 for c in verify_codes(messages, signatures, public_keys, device)]


def prehash_records(messages: Sequence[bytes], signatures: Sequence[bytes],
                    public_keys: Sequence[bytes]) -> np.ndarray:
    """[R | S | k | A] records with k = SHA-512(R || A || M) as 32 bytes mod L."""
    out = np.zeros((len(messages), 128), dtype=np.uint8)
    for i, (m, s, a) in enumerate(zip(messages, signatures, public_keys)):
        k = int.from_bytes(hashlib.sha512(bytes(s[:32]) + bytes(a) + bytes(m)).digest(), "little") % ref.L
        out[i] = np.frombuffer(bytes(s) + k.to_bytes(32, "little") + bytes(a), dtype=np.uint8)
    return out


def selftest(op: int, inputs: np.ndarray, device: str = "cuda"):
    """Runs a kernel building block over [n, 64] byte records (test entry)."""
    import torch

    from arc_chain_b200.ops import int_ops
    from arc_chain_b200.ops._lib import lib

    dev = torch.device(device)
    init(dev)
    x = torch.from_numpy(np.ascontiguousarray(inputs, dtype=np.uint8)).to(dev)
    n = x.shape[0]
    out = torch.zeros((n, 32), dtype=torch.uint8, device=dev)
    code = torch.zeros(n, dtype=torch.int32, device=dev)
    int_ops.check(lib().arcb_ed25519_selftest(op, x.data_ptr(), n, out.data_ptr(), code.data_ptr(), int_ops._s()),
                  "ed25519_selftest")
    return out.cpu().numpy(), code.cpu().numpy()
