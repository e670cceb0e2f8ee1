"""Expert parallelism for the MLA + MoE decoder (one process per GPU).

Layout: attention, router, dense layers, embedding and LM head are
replicated on every rank (each rank runs them on the same tokens, so all
ranks hold the same hidden state and sampling state); the experts
(routed 0..E-1, then shared) are sharded g % N == rank.  Each rank's grouped
gate/up and down GEMMs cover only its experts, and its combine epilogue
produces a routing-weighted partial of the MoE output.  The partials of all
ranks are summed into every rank's hidden state; integer adds make the sum
exact and order free, so outputs equal the single-GPU run bit for bit.

Two ways of summing:

* ``EpNcclComm`` (baseline): the combine epilogue adds into a local buffer,
  then ``all_reduce(SUM)`` on int64 and a fold kernel h += delta.
* ``EpFusedComm`` (product): the combine epilogue adds straight into every
  rank's per-layer combine buffer over NVLink peer pointers (symmetric
  memory; plain atomics, no multicast, no TMA on peer memory), and each CTA
  bumps every rank's arrival counter once its adds are fenced; a small
  kernel waits (bounded) for all ranks' arrivals and folds h += delta.  One
  buffer per MoE layer keeps reuse safe: a rank can run at most one layer
  ahead of a peer, since it waits for the peer's arrivals every layer.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from arc_chain_b200.ops import int_ops as ops
from arc_chain_b200.runtime.engine import Comm

os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")


class EpComm(Comm):
    """Hooks the MLA + MoE engine calls around each grouped down GEMM."""

    ep = True

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self._state = {}

    def _alloc(self, n: int, dtype, device):
        return torch.zeros(n, dtype=dtype, device=device)

    def state(self, bb, n_moe: int, d: int):
        key = id(bb)
        st = self._state.get(key)
        if st is None:
            st = self._make_state(bb, n_moe, d)
            self._state[key] = st
        return st

    def combine_epi(self, epi, bb, j: int, n_moe: int, d: int):
        raise NotImplementedError

    def after_combine(self, bb, j: int, n_moe: int, d: int) -> None:
        raise NotImplementedError

    @property
    def n_launches(self) -> int:
        return 1


class _State:
    pass


class EpNcclComm(EpComm):
    def _make_state(self, bb, n_moe, d):
        st = _State()
        dev = bb.h.device
        st.delta = self._alloc(n_moe * bb.B * d, torch.int64, dev).view(n_moe, bb.B, d)
        st.epoch = self._alloc(1, torch.int64, dev)
        st.done = self._alloc(1, torch.int32, dev)
        st.cnt = self._alloc(1, torch.int64, dev)
        st.epis = {}
        return st

    def combine_epi(self, epi, bb, j, n_moe, d):
        st = self.state(bb, n_moe, d)
        e = st.epis.get(j)
        if e is None:
            e = ops.Epi.from_buffer_copy(epi)
            e.out = st.delta[j].data_ptr()
            st.epis[j] = e
        return e

    def after_combine(self, bb, j, n_moe, d):
        st = self.state(bb, n_moe, d)
        dist.all_reduce(st.delta[j], op=dist.ReduceOp.SUM, group=self.group)
        ops.ep_wait_apply(st.cnt, st.epoch, 0, bb.h, st.delta[j], st.done, bb.err)


class EpFusedComm(EpComm):
    def _make_state(self, bb, n_moe, d):
        import torch.distributed._symmetric_memory as symm_mem

        st = _State()
        dev = bb.h.device
        gname = (self.group or dist.group.WORLD).group_name
        st.delta = symm_mem.empty(n_moe * bb.B * d, dtype=torch.int64, device=dev)
        st.cnt = symm_mem.empty(1, dtype=torch.int64, device=dev)
        st.delta.zero_()
        st.cnt.zero_()
        hd = symm_mem.rendezvous(st.delta, gname)
        hc = symm_mem.rendezvous(st.cnt, gname)
        st._h = (hd, hc)
        st.delta = st.delta.view(n_moe, bb.B, d)
        layer_bytes = bb.B * d * 8
        st.peer_h = [torch.tensor([p + j * layer_bytes for p in hd.buffer_ptrs], dtype=torch.int64, device=dev)
                     for j in range(n_moe)]
        st.peer_cnt = torch.tensor(list(hc.buffer_ptrs), dtype=torch.int64, device=dev)
        st.epoch = self._alloc(1, torch.int64, dev)
        st.done = self._alloc(1, torch.int32, dev)
        st.epis = {}
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        return st

    def combine_epi(self, epi, bb, j, n_moe, d):
        st = self.state(bb, n_moe, d)
        e = st.epis.get(j)
        if e is None:
            e = ops.Epi.from_buffer_copy(epi)
            e.npeers = self.size
            e.peer_h = st.peer_h[j].data_ptr()
            e.peer_sig = st.peer_cnt.data_ptr()
            e.max_ctas = 0
            st.epis[j] = e
        return e

    def after_combine(self, bb, j, n_moe, d):
        st = self.state(bb, n_moe, d)
        ops.ep_wait_apply(st.cnt, st.epoch, self.size * ops.num_sms(), bb.h, st.delta[j], st.done, bb.err)
