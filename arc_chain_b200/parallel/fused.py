"""Fused tensor-parallel communication: GEMM -> all-reduce inside the GEMM
kernel, over NVLink peer memory.

For the row-parallel projections (W_o, W_down) every rank holds a K shard,
so each output row needs the sum over ranks of the partial dot products
before the scale and residual.  Instead of a separate collective, the fused
GEMM (csrc/kernels/gemm_fused.cu, ``rp`` mode) first sums the split-K limb
partials of a tile in this GPU's own partial buffer, exactly as on one GPU.
The CTA that completes the tile recombines its limbs and stores the wrapping
int64 row sums (128 rows x slots: 1 KB per tile at batch 1) into this rank's
slot of every rank's receive buffer with plain stores to peer memory, fences
and adds 1 to every rank's arrival counter for the tile.  On each rank a
designated CTA per tile waits (bounded; a timeout sets ARCB_ERR_COMM_TIMEOUT)
for all ranks' arrivals, sums the slots and finalises its own copy (residual
add + next norm's sum of squares).  Integer sums are exact and order free,
so every rank ends with the identical, reference-exact hidden state; each
tile crosses NVLink once per peer, as soon as it is complete.

From 4 ranks and 16 slots up the same GEMM runs as a reduce-scatter plus
all-gather instead (``rs_ag``): a completed tile goes only to its owner rank
(m-tile mod N), the owner sums the N slots and stores the total into every
rank, and every rank applies the epilogue; a rank then sends 2 (N - 1) / N
of the output's bytes instead of N - 1 times them (1.75 vs 7 at N = 8).

Two buffer sets (one for W_o, one for W_down) make reuse safe: a rank can be
at most one row-parallel GEMM ahead of a peer.  Multicast is not used (only
plain peer stores and atomics), and no TMA reads peer memory.

Symmetric memory and peer mappings come from torch.distributed's
symmetric-memory allocator.  The LM head GEMM stores its vocab slice into
every rank's logits buffer itself (STORE_PEERS epilogue) and a bounded
arrival wait replaces the all-gather (``fuse_logits``, the default: 2.934 vs
2.957 ms/token with the NCCL all-gather at TP2 on the same box; exact at 2, 4
and 8 ranks).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.parallel.tp import NcclComm

os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")


class _Site:
    def __init__(self, n_slots: int, B: int, M: int, n_cnt: int, device, group_name, rs_ag: bool = False):
        import torch.distributed._symmetric_memory as symm_mem

        self.rs_ag = rs_ag
        self.n_cnt = n_cnt
        self.P = torch.zeros(8 * B * M, dtype=torch.int32, device=device)  # local split-K partials
        # reduce-scatter + all-gather: one more slot (the final area) and a
        # second counter array (the owners' final signals)
        self.R = symm_mem.empty((n_slots + int(rs_ag)) * B * M, dtype=torch.int64, device=device)
        self.cnt = symm_mem.empty(n_cnt * (2 if rs_ag else 1), dtype=torch.int32, device=device)
        self.R.zero_()
        self.cnt.zero_()
        hr = symm_mem.rendezvous(self.R, group_name)
        hc = symm_mem.rendezvous(self.cnt, group_name)
        self._h = (hr, hc)
        self.peer_R = torch.tensor(list(hr.buffer_ptrs), dtype=torch.int64, device=device)
        self.peer_cnt = torch.tensor(list(hc.buffer_ptrs), dtype=torch.int64, device=device)


class _Logits:
    """Symmetric [B, vocab] logits buffer, every rank's pointer offset to
    this rank's vocab columns, and the arrival counter of the gather."""

    def __init__(self, B: int, V: int, lo: int, device, group_name):
        import torch.distributed._symmetric_memory as symm_mem

        self.buf = symm_mem.empty(B * V, dtype=torch.int64, device=device)
        self.cnt = symm_mem.empty(1, dtype=torch.int64, device=device)
        self.buf.zero_()
        self.cnt.zero_()
        hb = symm_mem.rendezvous(self.buf, group_name)
        hc = symm_mem.rendezvous(self.cnt, group_name)
        self._h = (hb, hc)
        self.peer = torch.tensor([p + lo * 8 for p in hb.buffer_ptrs], dtype=torch.int64, device=device)
        self.peer_cnt = torch.tensor(list(hc.buffer_ptrs), dtype=torch.int64, device=device)
        self.epoch = torch.zeros(1, dtype=torch.int64, device=device)
        self.done = torch.zeros(1, dtype=torch.int32, device=device)
        self.view = self.buf.view(B, V)
        self.epi = None


class FusedComm(NcclComm):
    """fuse_logits (default): the LM head GEMM also stores its vocab slice
    into every rank's logits buffer over NVLink (STORE epilogue with peer
    targets) and a bounded arrival wait replaces the NCCL all-gather;
    False gathers the logits with NCCL."""

    fused = True

    def __init__(self, group=None, fuse_logits: bool = True, rs_ag: str = "auto"):
        super().__init__(group)
        # "auto": reduce-scatter + all-gather from 4 ranks and 16 slots up
        # (each rank sends 2 (N - 1) / N of the output instead of N - 1 times
        # it, for one more NVLink hop); "on" / "off" force it
        self.rs_ag = os.environ.get("ARCB_RS_AG", rs_ag)
        self.group_name = (group or dist.group.WORLD).group_name
        self._sites = {}
        self._epis = {}
        self.fuse_logits = fuse_logits
        self._logits = {}

    def _logit_state(self, bb, V: int, lo: int) -> _Logits:
        key = id(bb)
        if key not in self._logits:
            self._logits[key] = _Logits(bb.B, V, lo, bb.P.device, self.group_name)
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
        return self._logits[key]

    def lm_epi(self, epi, bb, V: int, lo: int):
        """The LM head's epilogue descriptor (pushes into every rank when fused)."""
        if not self.fuse_logits:
            return epi
        st = self._logit_state(bb, V, lo)
        if st.epi is None:
            e = ops.Epi.from_buffer_copy(epi)
            e.mode = ops.STORE_PEERS
            e.ldo = V
            e.npeers = self.size
            e.peer_h = st.peer.data_ptr()
            e.peer_sig = st.peer_cnt.data_ptr()
            e.max_ctas = 0
            st.epi = (e, epi)
        return st.epi[0]

    def gather_logits(self, local, full, B, vocab_offset, bb=None):
        if not self.fuse_logits or bb is None or id(bb) not in self._logits:
            return super().gather_logits(local, full, B, vocab_offset)
        st = self._logits[id(bb)]
        ops.ep_wait_apply(st.cnt, st.epoch, self.size * ops.num_sms(), None, None, st.done, bb.err)
        full[:B].copy_(st.view[:B])

    def use_rs_ag(self, B: int) -> bool:
        if self.rs_ag in ("on", "1"):
            return True
        if self.rs_ag in ("off", "0"):
            return False
        return self.size >= 4 and B >= 16

    def _site(self, bb, site: int, M: int) -> _Site:
        key = (id(bb), site)
        if key not in self._sites:
            self._sites[key] = _Site(self.size, bb.B, M, ops.tile_counters(M, bb.B), bb.P.device, self.group_name,
                                     rs_ag=self.use_rs_ag(bb.B))
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
            e.rank = self.rank
            e.peer_R = s.peer_R.data_ptr()
            e.peer_cnt = s.peer_cnt.data_ptr()
            e.cnt_local = s.cnt.data_ptr()
            e.rs_ag = int(s.rs_ag)
            e.rs_cnt_off = s.n_cnt if s.rs_ag else 0
            self._epis[key] = (e, epi)  # keep the source alive: its id is the key
        else:
            e = e[0]
        ops.linear_gemm(lin, xmap, B, lmax, s.P, bb.tiles, e)
