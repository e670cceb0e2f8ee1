"""Tensor-parallel communication for the dense decoder.

``NcclComm`` is the library baseline: after each row-parallel GEMM (W_o,
W_down) the int32 limb partials are summed across ranks with an NCCL
all-reduce (integer sums are exact and order independent, so every rank
then finalizes bit-identical rows), the per-operand limb count is
all-reduced with MAX, and the vocab-sharded logits are all-gathered so each
rank samples the same token.

The fused path (``arc_chain_b200.parallel.fused``) replaces these calls with
kernels that push partials to peers over NVLink from inside the kernel.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from arc_chain_b200.runtime.engine import Comm


def init_distributed(timeout_s: int = 120):
    """torch.distributed over NCCL, one process per GPU (env:// rendezvous)."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s),
                            device_id=torch.device("cuda", local))
    return rank, world


class NcclComm(Comm):
    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self._gbuf = {}

    def reduce_partials(self, P, rows, M, lmax):
        dist.all_reduce(P[:rows * M], op=dist.ReduceOp.SUM, group=self.group)
        dist.all_reduce(lmax, op=dist.ReduceOp.MAX, group=self.group)

    def gather_logits(self, local, full, B, vocab_offset, bb=None):
        Vl = local.shape[1]
        key = (B, Vl)
        if key not in self._gbuf:
            self._gbuf[key] = torch.empty(self.size * B * Vl, dtype=local.dtype, device=local.device)
        g = self._gbuf[key]
        dist.all_gather_into_tensor(g, local[:B].contiguous().view(-1), group=self.group)
        V = full.shape[1]
        full[:B].view(B, -1)[:, :self.size * Vl].view(B, self.size, Vl).copy_(g.view(self.size, B, Vl).transpose(0, 1)) \
            if V == self.size * Vl else _copy_ragged(full, g, B, Vl, self.size)


def _copy_ragged(full, g, B, Vl, size):
    V = full.shape[1]
    gv = g.view(size, B, Vl)
    for r in range(size):
        lo = r * Vl
        hi = min(V, lo + Vl)
        if hi > lo:
            full[:B, lo:hi].copy_(gv[r, :, :hi - lo])
