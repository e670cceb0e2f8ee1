"""Data parallelism: whole-model replicas, one per process (one GPU each, or
a CPU oracle), with requests sharded across them and cross-replica output
agreement.

The reference replicates whole requests across validators and accepts an
output when a committee agrees on its hash (crates/arc-inference/src/
committee.rs:69-170, 5-of-7).  Here the replicas are the ranks of a
torch.distributed group:

* :meth:`ReplicaGroup.run` - request i runs on rank i % world; every rank
  receives all results, in request order;
* :meth:`ReplicaGroup.agree` - every rank runs the same request and the
  output hashes are compared (at least ``min_agree`` equal, the committee
  rule); with exact integer inference every healthy replica agrees.

The backend is any ``generate(prompt, max_tokens) -> (tokens, hash)``: the
GPU engine, a continuous-batching scheduler, or the CPU oracle.
"""
from __future__ import annotations

from collections import Counter
from typing import Callable, List, Optional, Sequence, Tuple

import torch.distributed as dist

Result = Tuple[List[int], bytes]


def shard(n: int, rank: int, world: int) -> List[int]:
    """Request indices of `rank`: i % world == rank."""
    return list(range(rank, n, world))


class ReplicaGroup:
    def __init__(self, generate: Callable[[Sequence[int], int], Result], group=None):
        self.generate = generate
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def _gather(self, obj):
        out = [None] * self.world
        dist.all_gather_object(out, obj, group=self.group)
        return out

    def run(self, requests: Sequence[Tuple[Sequence[int], int]]) -> List[Result]:
        mine = {i: self.generate(list(requests[i][0]), int(requests[i][1]))
                for i in shard(len(requests), self.rank, self.world)}
        merged = {}
        for part in self._gather({i: (list(t), bytes(h)) for i, (t, h) in mine.items()}):
            merged.update(part)
        return [merged[i] for i in range(len(requests))]

    def agree(self, prompt: Sequence[int], max_tokens: int, min_agree: Optional[int] = None) -> dict:
        """Every replica runs the request; returns the majority hash and
        whether at least min_agree replicas produced it (default: all)."""
        toks, h = self.generate(list(prompt), int(max_tokens))
        hashes = self._gather(bytes(h))
        (best, count), = Counter(hashes).most_common(1)
        need = self.world if min_agree is None else min_agree
        return {"output_hash": best.hex(), "agree": count, "replicas": self.world, "accepted": count >= need,
                "dissenting_ranks": [r for r, x in enumerate(hashes) if x != best]}
