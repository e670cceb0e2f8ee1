"""Expert parallelism for the MLA + MoE decoder (one process per GPU).

Two layouts.  ``EpDispatchComm`` (token dispatch, used for lockstep batched
decode) runs the trunk data-parallel and moves tokens to the experts; it is
described on the class.  The replicated layout (``EpNcclComm``,
``EpFusedComm``, any batching): attention, router, dense layers, embedding and LM head are
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


class EpDispatchComm(EpComm):
    """Token dispatch (data-parallel trunk, expert-parallel MoE).

    Each rank owns its own request slots: embedding, attention, the dense
    layers, the router and the LM head run on those B slots only (each rank
    holds its own KV cache).  Per MoE layer ``dispatch`` stores the slots'
    normalised limb planes and routing weights into every rank's gathered
    buffers (N * B slots, csrc/kernels/ep_ops.cu: k_ep_dispatch); each rank's
    grouped expert GEMMs run its experts over all N * B gathered slots, and
    the combine epilogue adds each slot's routing-weighted output only into
    its owner rank's combine buffer (peer atomics, ``ep_rows`` = B), after
    which ``after_combine`` folds this rank's B rows into its hidden state.

    All ranks must call the engine's forward in lockstep with the same slot
    count (equal prompt lengths and steps), since every MoE layer is a
    collective; the continuous-batching scheduler, which admits requests per
    rank, is not lockstep and uses ``EpFusedComm`` instead."""

    token_dispatch = True

    def _make_state(self, bb, n_moe, d):
        import torch.distributed._symmetric_memory as symm_mem

        st = _State()
        dev = bb.h.device
        N, B = self.size, bb.B
        G = bb.route.shape[1]
        gname = (self.group or dist.group.WORLD).group_name
        NB = N * B
        st.NB = NB
        st.rows = ops.limb_rows(NB, ops.fgemm_bn(NB))

        def sym(n, dtype):
            t = symm_mem.empty(n, dtype=dtype, device=dev)
            t.zero_()
            return t, symm_mem.rendezvous(t, gname)

        st.Xg, hX = sym(st.rows * d, torch.int8)
        st.route, hR = sym(NB * G, torch.int64)
        st.counts, hC = sym(max(N, 4), torch.int32)
        st.dcnt, hD = sym(1, torch.int64)
        st.delta, hd = sym(n_moe * B * d, torch.int64)
        st.cnt, hc = sym(1, torch.int64)
        st._h = (hX, hR, hC, hD, hd, hc)
        ptrs = lambda h, off=0: torch.tensor([p + off for p in h.buffer_ptrs], dtype=torch.int64, device=dev)
        st.pX, st.pR, st.pC, st.pD = ptrs(hX), ptrs(hR), ptrs(hC), ptrs(hD)
        st.Xg = st.Xg.view(st.rows, d)
        st.route = st.route.view(NB, G)
        st.delta = st.delta.view(n_moe, B, d)
        st.peer_h = [ptrs(hd, j * B * d * 8) for j in range(n_moe)]
        st.peer_cnt = ptrs(hc)
        st.d_epoch = self._alloc(1, torch.int64, dev)
        st.c_epoch = self._alloc(1, torch.int64, dev)
        st.gcnt = self._alloc(1, torch.int32, dev)
        st.done = self._alloc(1, torch.int32, dev)
        # dispatch grid: the same on every rank (part of the arrival target)
        chunks = (8 * B * d + B * G * 8) // 16
        st.blocks = max(1, min(32, (chunks + 255) // 256))
        st.epis = {}
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        return st

    def dispatch(self, bb, X, lcnt, n_moe: int, d: int, zero_cnt) -> None:
        st = self.state(bb, n_moe, d)
        G = st.route.shape[1]
        ops.ep_dispatch(X, bb.B, d, bb.route, G, lcnt, self.rank, self.size, st.pX, st.pR, st.pC, st.pD, st.dcnt,
                        st.d_epoch, st.gcnt, zero_cnt, st.blocks, bb.err)

    def combine_epi(self, epi, bb, j, n_moe, d):
        st = self.state(bb, n_moe, d)
        e = st.epis.get(j)
        if e is None:
            e = ops.Epi.from_buffer_copy(epi)
            e.npeers = self.size
            e.peer_h = st.peer_h[j].data_ptr()
            e.peer_sig = st.peer_cnt.data_ptr()
            e.ep_rows = bb.B
            e.max_ctas = 0
            st.epis[j] = e
        return e

    def after_combine(self, bb, j, n_moe, d):
        st = self.state(bb, n_moe, d)
        ops.ep_wait_apply(st.cnt, st.c_epoch, self.size * ops.num_sms(), bb.h, st.delta[j], st.done, bb.err)
