"""Tensor-parallel context (forgeserve/parallel.py:7-29): which shard this process is, and the in-place sum of
partial results over the shards (torch.distributed all-reduce on the context's group), with the reference's
counters. ForgeModel(cfg, TPContext(rank, size)) holds one shard of every layer (model.py); pipeline stages run
every layer whole (`SINGLE`, forgeserve/pipeline.py:50)."""

import torch
import torch.distributed as dist


class TPContext:
    """`size` shards; this process is shard `rank`. With size 1 every operation is a no-op."""

    def __init__(self, rank: int = 0, size: int = 1, group=None):
        if not 0 <= rank < size:
            raise ValueError("rank must be in [0, size)")
        self.rank, self.size, self.group = rank, size, group
        self.num_all_reduces = 0
        self.all_reduce_elements = 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sum `t` over all shards in place and return it."""
        if self.size > 1:
            self.num_all_reduces += 1
            self.all_reduce_elements += t.numel()
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t


SINGLE = TPContext()
