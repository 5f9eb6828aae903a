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

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from . import ops
from .engine import Request, Scheduler
from .paged import PagedKVPool
from .pipeline import microbatch_sizes, ring_program, seq_pieces
from .transport import DistTransport, ring_group


class _StageDecodeGraph:
    """One decode step of one row group on this stage, captured as a CUDA graph: the embedding (first stage), the
    stage's layers, and the final norm, head of the last position and argmax (last stage), over static device
    buffers for the input (token ids or activations), positions and block tables (tables padded with block 0 to
    max_seq_len / block_size columns, which leaves the decode kernels' sums unchanged). The transfers between stages
    stay outside the graph. The first step of a row count runs eagerly on the graph's own stream (it also sets up
    that stream's GEMM tile counter, split-K and decode workspaces), then the same work is captured; replays run on
    the caller's stream, in order with its transfers."""

    def __init__(self, stage, pool, rows: int):
        self.stage, self.pool, self.rows = stage, pool, rows
        dev = stage.device
        self.width = -(-stage.cfg.max_seq_len // pool.block_size)
        self.pos = torch.zeros(rows, 1, dtype=torch.int64, device=dev)
        self.tab = torch.zeros(rows, self.width, dtype=torch.int64, device=dev)
        if stage.is_first:
            self.inp = torch.zeros(rows, 1, dtype=torch.int64, device=dev)
        else:
            self.inp = torch.zeros(rows, 1, stage.cfg.d_model, dtype=stage.dtype, device=dev)
        self.stream = torch.cuda.Stream(dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.out: Optional[torch.Tensor] = None

    def _step(self) -> torch.Tensor:
        st = self.stage
        x = st.embed(self.inp) if st.is_first else self.inp
        st.run_layers_(x, self.pos, self.pool.views(self.tab, self.pos))
        return ops.argmax(st.head(x[:, -1:])[:, -1]) if st.is_last else x

    def run(self, positions: torch.Tensor, tables: torch.Tensor, inp: torch.Tensor) -> torch.Tensor:
        """The group's step on the current stream: its tokens (last stage) or output activations, in a new
        tensor."""
        self.pos.copy_(positions)
        self.tab.zero_()
        self.tab[:, : tables.shape[1]].copy_(tables)
        self.inp.copy_(inp.view(self.inp.shape))
        if self.graph is not None:
            self.graph.replay()
            return self.out.clone()
        cur = torch.cuda.current_stream(self.stage.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            out = self._step().clone()
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        # thread-local capture: the process group's watchdog thread keeps polling its events meanwhile
        with torch.cuda.graph(g, stream=self.stream, capture_error_mode="thread_local"):
            self.out = self._step()
        self.graph = g
        cur.wait_stream(self.stream)
        return out


class PipelineEngine(Scheduler):
    """overlap (extra): None or True takes decode windows whenever they apply (the tokens, block tables and
    counters are those of stepping one by one); False steps one by one, draining the pipeline every step.

    prefill_chunks (extra): a prefill step pushes the prompt through the stages in up to this many pieces along the
    sequence (pipeline.seq_pieces), so the stages work on different pieces at once instead of taking turns; a
    piece's keys and values of earlier positions are in the pool by the time it reaches a stage. Same tokens.

    cuda_graphs (extra, CUDA stages without tensor parallelism): inside decode windows each row group's step on a
    stage replays a captured CUDA graph (_StageDecodeGraph, one per group size) instead of launching every kernel
    from Python; the same kernels, so the same tokens."""

    MAX_WINDOW = 64     # decode steps per window: bounds what the host enqueues ahead of the GPUs
    MAX_GRAPHS = 4

    def __init__(self, stage, num_blocks: int, block_size: int = 16, max_batch: int = 8, seed: int = 0,
                 microbatches: int = 1, overlap: Optional[bool] = None, prefill_chunks: int = 1,
                 cuda_graphs: bool = True):
        self.stage, self.cfg = stage, stage.cfg
        self.pool = PagedKVPool(self.cfg, num_blocks, block_size, tp=stage.tp, dtype=stage.dtype,
                                device=stage.device, n_layers=len(stage.layers))
        self.microbatches = max(1, microbatches)
        self.overlap = overlap
        self.prefill_chunks = max(1, prefill_chunks)
        self.windows = 0          # decode windows taken by run()
        self.cuda_graphs = cuda_graphs
        self._graphs: Dict[int, _StageDecodeGraph] = {}
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

    def _stage_graph(self, rows: int, tables: torch.Tensor) -> Optional[_StageDecodeGraph]:
        st = self.stage
        if not (self.cuda_graphs and st.device.type == "cuda" and st.tp.size == 1
                and tables.shape[1] * self.pool.block_size <= self.cfg.max_seq_len + self.pool.block_size):
            return None
        g = self._graphs.pop(rows, None)
        if g is None:
            if len(self._graphs) >= self.MAX_GRAPHS:
                self._graphs.pop(next(iter(self._graphs)))
            g = _StageDecodeGraph(st, self.pool, rows)
        self._graphs[rows] = g
        return g

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
                work, inp = (tok_in if st.is_first else act_in).pop(k)
                work.wait()
                g = self._stage_graph(sizes[j], tables)
                if g is not None:
                    out = g.run(positions[grp], tables[grp], inp)
                else:
                    views = self.pool.views(tables[grp], positions[grp])
                    pos = views[0].positions if views else positions[grp].to(dev)
                    x = st.embed(inp.view(-1, 1)) if st.is_first else inp
                    st.run_layers_(x, pos, views)
                    out = self._argmax(st.head(x[:, -1:])[:, -1]) if st.is_last else x
                if st.is_last:
                    toks[t + 1, grp].copy_(out)
                else:
                    act_out[k] = out
        for work, _ in sends:
            work.wait()
        tr.broadcast(toks, src=p - 1)
        self._window_end(rows, toks[1:].cpu().tolist())
        self.windows += 1
