"""Continuous batching over a pipeline of stages: the reference's Engine scheduling (forgeserve/engine.py:36-139)
composed with PipelineStage (forgeserve/pipeline.py:44-80), which the reference never combines.

Every stage process builds a PipelineEngine over its own PipelineStage and calls the same add_request / step / run
sequence. The scheduler state is replicated: it depends only on request lengths, the (identical) block allocator
and the sampled tokens, which the last stage broadcasts every step. Each stage holds a paged pool for its own
layers (`PagedKVPool(..., n_layers=len(stage.layers))`), indexed by the same block tables on every stage.

One step (a prefill of one request, or one decode token for every running request) goes through the stages in
`microbatches` groups of rows: stage s runs group i while stage s+1 runs group i-1, and the last stage computes the
head for the last position only and samples.
"""

from typing import List

import torch

from . import ops
from .engine import Request, Scheduler
from .paged import PagedKVPool
from .pipeline import microbatch_sizes


class PipelineEngine(Scheduler):
    def __init__(self, stage, num_blocks: int, block_size: int = 16, max_batch: int = 8, seed: int = 0,
                 microbatches: int = 1):
        self.stage, self.cfg = stage, stage.cfg
        self.pool = PagedKVPool(self.cfg, num_blocks, block_size, dtype=stage.dtype, device=stage.device,
                                n_layers=len(stage.layers))
        self.microbatches = max(1, microbatches)
        self._init_scheduler(max_batch, seed)

    def _forward_rows(self, reqs: List[Request], idx: torch.Tensor, positions: torch.Tensor,
                      tables: torch.Tensor) -> List[int]:
        st = self.stage
        dev = st.device
        R, T = idx.shape
        d = self.cfg.d_model
        sizes = microbatch_sizes(R, min(self.microbatches, R))
        tr = st.transport
        recvs = []
        if not st.is_first:
            for size in sizes:
                buf = torch.empty(size, T, d, dtype=st.dtype, device=dev)
                recvs.append((tr.irecv(buf, st.rank - 1), buf))
        if st.is_first:
            idx_dev = idx.to(device=dev, dtype=torch.int64, non_blocking=True)
        logits = torch.empty(R, 1, self.cfg.vocab_size, dtype=st.dtype, device=dev) if st.is_last else None
        sends, row = [], 0
        for mb, size in enumerate(sizes):
            rows = slice(row, row + size)
            views = self.pool.views(tables[rows], positions[rows])
            pos = views[0].positions if views else positions[rows].to(dev)
            if st.is_first:
                x = st.embed(idx_dev[rows])
            else:
                work, x = recvs[mb]
                work.wait()
            st.run_layers_(x, pos, views)
            if st.is_last:
                st.head(x[:, -1:], out=logits[rows])
            else:
                sends.append(tr.isend(x, st.rank + 1))
            row += size
        for w in sends:
            w.wait()
        if st.is_last:
            tokens = torch.tensor(self._sample_rows(logits[:, -1], reqs), dtype=torch.int64, device=dev)
        else:
            tokens = torch.empty(R, dtype=torch.int64, device=dev)
        tr.broadcast(tokens, src=st.size - 1)
        return tokens.cpu().tolist()
