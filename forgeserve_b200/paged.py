"""Paged KV cache: block allocator, per-layer block pools and per-step views (forgeserve/paged.py:20-82).

The pool keeps the reference's layout, one (num_blocks, n_kv, block_size, head_dim) tensor per layer in
`pool.k[layer]` / `pool.v[layer]`, and the allocator its LIFO order (block 0 is handed out first). What changes
is the read side: the reference gathers every row's whole block table into a dense (B, n_kv, S, head_dim) copy
before attention (paged.py:80-81). Here the decoder layer hands the block table to the attention kernel, which
reads each key block in place; `PagedLayerView.update` still returns the gathered tensors for callers that use
the view protocol directly (on the GPU, by the fs_kv_store / fs_paged_gather kernels).
"""

from typing import List, Optional, Tuple

import torch

from . import ops
from .config import ModelConfig
from .parallel import SINGLE, TPContext


class OutOfBlocks(RuntimeError):
    pass


class BlockAllocator:
    def __init__(self, num_blocks: int):
        self.num_blocks = num_blocks
        self._free = list(range(num_blocks - 1, -1, -1))   # a stack: block 0 is on top

    @property
    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, n: int) -> List[int]:
        if n > len(self._free):
            raise OutOfBlocks(f"need {n} blocks, {len(self._free)} free")
        out = self._free[len(self._free) - n:][::-1]
        del self._free[len(self._free) - n:]
        return out

    def release(self, blocks: List[int]) -> None:
        self._free.extend(blocks)


class PagedKVPool:
    """The block pool of every layer; shapes (num_blocks, kv_heads_of_this_shard, block_size, head_dim).

    `n_layers` (default cfg.n_layers) lets a pipeline stage hold a pool for its own layers only."""

    def __init__(self, cfg: ModelConfig, num_blocks: int, block_size: int = 16, tp: TPContext = SINGLE,
                 dtype=torch.float32, device="cpu", n_layers: Optional[int] = None):
        shape = (num_blocks, cfg.n_kv_heads // tp.size, block_size, cfg.head_dim)
        layers = cfg.n_layers if n_layers is None else n_layers
        self.k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(layers)]
        self.block_size = block_size
        self.allocator = BlockAllocator(num_blocks)

    @property
    def device(self) -> torch.device:
        return self.k[0].device

    def blocks_for(self, n_tokens: int) -> int:
        return -(-n_tokens // self.block_size)

    def views(self, block_tables: torch.Tensor, positions: torch.Tensor) -> List["PagedLayerView"]:
        """One cache view per layer for a step. block_tables: (B, max_blocks), positions: (B, T)."""
        dev = self.device
        tables = torch.as_tensor(block_tables).to(device=dev, dtype=torch.int64, non_blocking=True).contiguous()
        pos = torch.as_tensor(positions).to(device=dev, dtype=torch.int64, non_blocking=True).contiguous()
        return [PagedLayerView(self, layer, tables, pos) for layer in range(len(self.k))]


class PagedLayerView:
    """What one attention layer sees during one step (same interface as ContiguousKV.update)."""

    def __init__(self, pool: PagedKVPool, layer: int, block_tables: torch.Tensor, positions: torch.Tensor):
        self.pool, self.layer, self.tables, self.positions = pool, layer, block_tables, positions

    @property
    def length(self) -> int:
        raise NotImplementedError("paged views need explicit positions")

    @property
    def n_slots(self) -> int:
        return self.tables.shape[1] * self.pool.block_size

    def descriptor(self):
        return ops.paged_desc(self.pool.k[self.layer], self.pool.v[self.layer], self.tables)

    def update(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Store k, v (B, n_kv, T, head_dim) at their positions; return each row's blocks in table order as
        (B, n_kv, max_blocks * block_size, head_dim)."""
        ops.kv_store(k, v, self.positions, self.descriptor())
        return ops.paged_gather(self.pool.k[self.layer], self.tables), ops.paged_gather(self.pool.v[self.layer],
                                                                                         self.tables)
