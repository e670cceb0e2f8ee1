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


class DeviceBlake3:
    """BLAKE3 of a stream of device tensors, hashed on the GPU.

    Complete 1 KiB chunks are hashed by the GPU (one thread per chunk), their
    chaining values merged into aligned subtrees of 2**level chunks on the
    GPU, and the host hasher merges subtree and chunk CVs in stream order.
    Bytes of an incomplete trailing chunk are carried (in a small device
    buffer) into the next update; the final chunk is hashed on the host,
    where it may take the ROOT flag.  Equals blake3(concatenated bytes)."""

    def __init__(self, device=None, level: int = 10):
        import torch

        self.torch = torch
        self.dev = torch.device(device or "cuda")
        self.level = level
        self.h = Blake3()
        self.chunks = 0  # complete chunks already merged
        self.carry = torch.empty(0, dtype=torch.uint8, device=self.dev)

    def update(self, *tensors) -> "DeviceBlake3":
        torch = self.torch
        from arc_chain_b200.ops._lib import lib
        from arc_chain_b200.ops import int_ops

        segs = [self.carry] + [t.contiguous().view(torch.uint8).reshape(-1) for t in tensors]
        segs = [s for s in segs if s.numel()]
        total = sum(s.numel() for s in segs)
        if total == 0:
            return self
        # keep at least one byte back: the final chunk must be finished on the host
        n_full = (total - 1) // 1024
        if n_full > 0:
            offs = [0]
            for s in segs[:-1]:
                offs.append(offs[-1] + s.numel())
            ptrs = torch.tensor([s.data_ptr() for s in segs], dtype=torch.int64, device=self.dev)
            offt = torch.tensor(offs, dtype=torch.int64, device=self.dev)
            cvs = torch.empty(n_full * 8, dtype=torch.int32, device=self.dev)
            int_ops.check(lib().arcb_blake3_chunk_cvs(ptrs.data_ptr(), offt.data_ptr(), len(segs), n_full,
                                                      self.chunks, cvs.data_ptr(), int_ops._s()),
                          "blake3_chunk_cvs")
            self._merge(cvs, n_full)
        # carry the tail bytes [n_full * 1024, total)
        start = n_full * 1024
        parts, pos = [], 0
        for s in segs:
            lo, hi = max(start, pos), min(total, pos + s.numel())
            if hi > lo:
                parts.append(s[lo - pos:hi - pos])
            pos += s.numel()
        self.carry = torch.cat(parts).clone() if parts else self.carry[:0]
        return self

    def _merge(self, cvs, n: int):
        torch = self.torch
        from arc_chain_b200.ops._lib import lib
        from arc_chain_b200.ops import int_ops

        # the stream so far may end mid-subtree; align the GPU subtrees to it
        lvl = self.level
        lead = (-self.chunks) % (1 << lvl)
        lead = min(lead, n)
        host = cvs.view(-1, 8)[:lead].cpu().numpy().astype("<u4")
        for i in range(lead):
            self.chunks += 1
            self.h.push_chunk_cv(host[i], self.chunks)
        rest = n - lead
        nsub = rest >> lvl
        if nsub:
            cur = cvs.view(-1, 8)[lead:lead + (nsub << lvl)].reshape(-1)
            for _ in range(lvl):
                npairs = cur.numel() // 16
                nxt = torch.empty(npairs * 8, dtype=torch.int32, device=self.dev)
                int_ops.check(lib().arcb_blake3_parents(cur.data_ptr(), npairs, nxt.data_ptr(), int_ops._s()),
                              "blake3_parents")
                cur = nxt
            sub = cur.view(-1, 8).cpu().numpy().astype("<u4")
            import ctypes as C

            for i in range(nsub):
                self.chunks += 1 << lvl
                a = np.ascontiguousarray(sub[i])
                self.h._lib.arcref_blake3_push_subtree_cv(self.h._h, a.ctypes.data_as(C.c_void_p), lvl, self.chunks)
        tail = cvs.view(-1, 8)[lead + (nsub << lvl):].cpu().numpy().astype("<u4")
        for i in range(len(tail)):
            self.chunks += 1
            self.h.push_chunk_cv(tail[i], self.chunks)

    def digest(self) -> bytes:
        self.h.update(self.carry.cpu().numpy())
        return self.h.digest()
