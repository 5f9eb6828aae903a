"""Continuous batching over a pipeline of stages: the reference's Engine scheduling (forgeserve/engine.py:36-139)
composed with PipelineStage (forgeserve/pipeline.py:44-80), which the reference never combines.

Every stage process builds a PipelineEngine over its own PipelineStage and calls the same add_request / step / run
sequence. The scheduler state is replicated: it depends only on request lengths, the (identical) block allocator
and the sampled tokens, which the last stage broadcasts every step. Each stage holds a paged pool for its own
layers (`PagedKVPool(..., n_layers=len(stage.layers))`), indexed by the same block tables on every stage.

One step (a prefill of one request, or one decode token for every running request) goes through the stages in
`microbatches` groups of rows: stage s runs group i while stage s+1 runs group i-1, and the last stage computes the
head for the last position only and samples.

Decode windows (`run`, one process per stage over torch.distributed): while the running rows are all greedy with
no eos, the scheduler's next steps do not depend on the tokens (Scheduler._window_steps), so every stage plans
them ahead and the rows' groups go round the pipeline without a drain after each step: the last stage sends each
group's new tokens straight to the first (ring_program, as pipeline_generate's overlapped loop), and stage s works
on step t's group j while the first stage already runs step t+1's earlier groups. With at least as many groups as
stages no stage waits for a token. The tokens reach every stage with one broadcast at the end of the window.
"""

from typing import List, Optional

import torch
import torch.distributed as dist

from .engine import Request, Scheduler
from .paged import PagedKVPool
from .pipeline import microbatch_sizes, ring_program, seq_pieces
from .transport import DistTransport, ring_group


class PipelineEngine(Scheduler):
    """overlap (extra): None or True takes decode windows whenever they apply (the tokens, block tables and
    counters are those of stepping one by one); False steps one by one, draining the pipeline every step.

    prefill_chunks (extra): a prefill step pushes the prompt through the stages in up to this many pieces along the
    sequence (pipeline.seq_pieces), so the stages work on different pieces at once instead of taking turns; a
    piece's keys and values of earlier positions are in the pool by the time it reaches a stage. Same tokens."""

    MAX_WINDOW = 64     # decode steps per window: bounds what the host enqueues ahead of the GPUs

    def __init__(self, stage, num_blocks: int, block_size: int = 16, max_batch: int = 8, seed: int = 0,
                 microbatches: int = 1, overlap: Optional[bool] = None, prefill_chunks: int = 1):
        self.stage, self.cfg = stage, stage.cfg
        self.pool = PagedKVPool(self.cfg, num_blocks, block_size, tp=stage.tp, dtype=stage.dtype,
                                device=stage.device, n_layers=len(stage.layers))
        self.microbatches = max(1, microbatches)
        self.overlap = overlap
        self.prefill_chunks = max(1, prefill_chunks)
        self.windows = 0          # decode windows taken by run()
        # decode windows: each step's block tables and positions go to the device in one copy from a pinned slot of
        # its own (a copy from pageable memory would make the host wait for the stream at every group)
        self._ring: Optional[torch.Tensor] = None
        self._ring_dev: Optional[torch.Tensor] = None
        self._init_scheduler(max_batch, seed)

    def _forward_rows(self, reqs: List[Request], idx: torch.Tensor, positions: torch.Tensor,
                      tables: torch.Tensor) -> List[int]:
        st = self.stage
        dev = st.device
        R, T = idx.shape
        d = self.cfg.d_model
        sizes = microbatch_sizes(R, min(self.microbatches, R))
        starts = [sum(sizes[:j]) for j in range(len(sizes))]
        pieces = seq_pieces(T, self.prefill_chunks, min(sizes)) if T > 1 else [(0, T)]
        items = [(j, c0, c1) for j in range(len(sizes)) for c0, c1 in pieces]
        tr = st.transport
        recvs = []
        if not st.is_first:
            for j, c0, c1 in items:
                buf = torch.empty(sizes[j], c1 - c0, d, dtype=st.dtype, device=dev)
                recvs.append((tr.irecv(buf, st.rank - 1), buf))
        if st.is_first:
            idx_dev = idx.to(device=dev, dtype=torch.int64, non_blocking=True)
        logits = torch.empty(R, 1, self.cfg.vocab_size, dtype=st.dtype, device=dev) if st.is_last else None
        sends = []
        for k, (j, c0, c1) in enumerate(items):
            rows = slice(starts[j], starts[j] + sizes[j])
            views = self.pool.views(tables[rows], positions[rows, c0:c1])
            pos = views[0].positions if views else positions[rows, c0:c1].to(dev)
            if st.is_first:
                x = st.embed(idx_dev[rows, c0:c1])
            else:
                work, x = recvs[k]
                work.wait()
            st.run_layers_(x, pos, views)
            if st.is_last:
                if c1 == T:
                    st.head(x[:, -1:], out=logits[rows])
            else:
                sends.append(tr.isend(x, st.rank + 1))
        for w in sends:
            w.wait()
        if st.is_last:
            tokens = torch.tensor(self._sample_rows(logits[:, -1], reqs), dtype=torch.int64, device=dev)
        else:
            tokens = torch.empty(R, dtype=torch.int64, device=dev)
        tr.broadcast(tokens, src=st.size - 1)
        return tokens.cpu().tolist()

    # ---- decode windows ----------------------------------------------------------------------------------
    def _windowed(self) -> bool:
        st = self.stage
        if self.overlap is False or st.size < 2 or min(self.microbatches, len(self.running)) < st.size:
            return False
        if not (isinstance(st.transport, DistTransport) and st.transport.group is None and dist.is_initialized()):
            return False
        backend = dist.get_backend()
        return backend == "nccl" or (backend == "gloo" and st.device.type == "cpu")

    def _window_steps(self) -> int:
        return min(super()._window_steps(), self.MAX_WINDOW)

    def _plan_on_device(self, t: int, tables: torch.Tensor, positions: torch.Tensor):
        """Step t's tables (R, width) and positions (R, 1) on the stage's device, through pinned slot t."""
        if self.stage.device.type != "cuda":
            return tables, positions
        R, width = tables.shape
        cap = -(-self.cfg.max_seq_len // self.pool.block_size) + 1
        n = R * (1 + cap)
        if self._ring is None or self._ring.shape[1] < n:
            self._ring = torch.zeros(self.MAX_WINDOW, n, dtype=torch.int64).pin_memory()
            self._ring_dev = torch.zeros(self.MAX_WINDOW, n, dtype=torch.int64, device=self.stage.device)
        slot = self._ring[t]
        slot[:R].copy_(positions.reshape(-1))
        slot[R : R + R * width].copy_(tables.reshape(-1))
        dst = self._ring_dev[t]
        dst[: R * (1 + width)].copy_(slot[: R * (1 + width)], non_blocking=True)
        return dst[R : R + R * width].view(R, width), dst[:R].view(R, 1)

    @torch.no_grad()
    def _decode_window(self, w: int) -> None:
        """w decode steps of the running rows, in groups, over ring_program's order (item k = step k // m of
        group k % m). Every stage makes each step's block grants, tables and positions (Scheduler._window_step)
        when it first computes a group of that step, in step order on every stage; the first stage takes a
        group's input tokens from the ring (for the first step, the known last tokens, sent by the last stage at
        the start like the prefill's tokens in pipeline_generate)."""
        st = self.stage
        p, r, dev, tr = st.size, st.rank, st.device, st.transport
        rows = list(self.running)
        sizes = microbatch_sizes(len(rows), min(self.microbatches, len(rows)))
        m = len(sizes)
        starts = [sum(sizes[:j]) for j in range(m)]
        cached = [req.cached for req in rows]
        toks = torch.empty(w + 1, len(rows), dtype=torch.int64, device=dev)   # toks[t]: step t's input tokens
        toks[0].copy_(torch.tensor([req.output[-1] for req in rows]))
        ring = ring_group()
        plan, plan_t = None, -1
        tok_in, act_in, act_out, sends = {}, {}, {}, []
        for op, k in ring_program(r, p, m, w * m):
            j, t = k % m, k // m
            grp = slice(starts[j], starts[j] + sizes[j])
            if op == "tok_send":
                buf = toks[t, grp]
                sends.append((dist.isend(buf, dst=0, group=ring), buf))
            elif op == "tok_recv":
                buf = torch.empty(sizes[j], dtype=torch.int64, device=dev)
                tok_in[k] = (dist.irecv(buf, src=p - 1, group=ring), buf)
            elif op == "act_recv":
                buf = torch.empty(sizes[j], 1, self.cfg.d_model, dtype=st.dtype, device=dev)
                act_in[k] = (tr.irecv(buf, r - 1), buf)
            elif op == "act_send":
                sends.append((tr.isend(act_out.pop(k), r + 1), None))
            else:
                if t != plan_t:
                    plan, plan_t = self._plan_on_device(t, *self._window_step(rows, cached, t, last=t == w - 1)), t
                tables, positions = plan
                views = self.pool.views(tables[grp], positions[grp])
                pos = views[0].positions if views else positions[grp].to(dev)
                if st.is_first:
                    work, tb = tok_in.pop(k)
                    work.wait()
                    x = st.embed(tb.view(-1, 1))
                else:
                    work, x = act_in.pop(k)
                    work.wait()
                st.run_layers_(x, pos, views)
                if st.is_last:
                    toks[t + 1, grp].copy_(self._argmax(st.head(x[:, -1:])[:, -1]))
                else:
                    act_out[k] = x
        for work, _ in sends:
            work.wait()
        tr.broadcast(toks, src=p - 1)
        self._window_end(rows, toks[1:].cpu().tolist())
        self.windows += 1
