"""Fused tensor-parallel communication: GEMM -> int32 limb-partial all-reduce
inside the GEMM kernel, over NVLink peer memory.

For the row-parallel projections (W_o, W_down) every rank holds a K shard,
so each output row needs the sum over ranks of the int32 per-limb partials
before the limb recombination, scale and residual.  Instead of a separate
collective, the fused GEMM (csrc/kernels/gemm_fused.cu, ``rp`` mode) adds
each partial tile straight into every rank's P buffer with ``red.add`` on
peer pointers of a symmetric allocation, then bumps every rank's per-tile
arrival counter.  On each rank a designated CTA per tile waits (bounded; a
timeout sets ARCB_ERR_COMM_TIMEOUT) until all ranks' chunks have arrived and
finalises its own copy (residual add + next norm's sum of squares).  Integer
sums are exact and order free, so every rank ends with the identical,
reference-exact hidden state, and the transfer overlaps the MMA tile by tile.

Two buffer sets (one for W_o, one for W_down) make reuse safe: a rank can be
at most one row-parallel GEMM ahead of a peer.  Multicast is not used (only
plain peer loads/stores/atomics), and no TMA reads peer memory.

Symmetric memory and peer mappings come from torch.distributed's
symmetric-memory allocator; the logits all-gather stays on NCCL.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.parallel.tp import NcclComm

os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")


class _Site:
    def __init__(self, n_p: int, n_cnt: int, device, group_name):
        import torch.distributed._symmetric_memory as symm_mem

        self.P = symm_mem.empty(n_p, dtype=torch.int32, device=device)
        self.cnt = symm_mem.empty(n_cnt, dtype=torch.int32, device=device)
        self.lmax = symm_mem.empty(1, dtype=torch.int32, device=device)
        for t in (self.P, self.cnt, self.lmax):
            t.zero_()
        hp = symm_mem.rendezvous(self.P, group_name)
        hc = symm_mem.rendezvous(self.cnt, group_name)
        hl = symm_mem.rendezvous(self.lmax, group_name)
        self._h = (hp, hc, hl)
        self.peer_P = torch.tensor(list(hp.buffer_ptrs), dtype=torch.int64, device=device)
        self.peer_cnt = torch.tensor(list(hc.buffer_ptrs), dtype=torch.int64, device=device)
        self.peer_lmax = torch.tensor(list(hl.buffer_ptrs), dtype=torch.int64, device=device)


class FusedComm(NcclComm):
    fused = True

    def __init__(self, group=None):
        super().__init__(group)
        self.group_name = (group or dist.group.WORLD).group_name
        self._sites = {}
        self._epis = {}

    def _site(self, bb, site: int, M: int) -> _Site:
        key = (id(bb), site)
        if key not in self._sites:
            self._sites[key] = _Site(8 * bb.B * M, ops.tile_counters(M, bb.B), bb.P.device, self.group_name)
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        return self._sites[key]

    def fgemm_reduce(self, lin, xmap, B, lmax, bb, epi, site: int = 0) -> None:
        s = self._site(bb, site, lin.M)
        key = id(epi)
        e = self._epis.get(key)
        if e is None:
            e = ops.Epi.from_buffer_copy(epi)
            e.rp = 1
            e.npeers = self.size
            e.peer_P = s.peer_P.data_ptr()
            e.peer_cnt = s.peer_cnt.data_ptr()
            e.peer_lmax = s.peer_lmax.data_ptr()
            e.cnt_local = s.cnt.data_ptr()
            e.lmax_fin = s.lmax.data_ptr()
            self._epis[key] = (e, epi)  # keep the source alive: its id is the key
        else:
            e = e[0]
        ops.linear_gemm(lin, xmap, B, lmax, s.P, bb.tiles, e)
