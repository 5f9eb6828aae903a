"""Continuous batching over a paged KV cache (forgeserve/engine.py:23-139), on the GPU.

Scheduling is the reference's, step for step: a step prefills the head of the queue (whole prompt, batch 1)
when a slot and its blocks are free, otherwise decodes one token for every running request; blocks are taken
on demand; when the pool runs dry the most recently started request is preempted (its blocks freed, its
output kept, re-prefilled later from prompt + output); requests finish on max_new_tokens, eos or max_seq_len.

What runs differently: the pool lives on the model's device in the model's dtype; the model computes the head
for the last position only; greedy rows are sampled together by one argmax kernel and read back with one copy,
and temperature rows draw from the engine's seeded CPU generator in row order (the order of the reference's
per-row `sample` calls, so the generator stream is consumed identically).

`Scheduler` holds the scheduling; `Engine` runs it over one model, `PipelineEngine` (pipeline_engine.py) over the
stages of a pipeline.
"""

from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional

import torch
import torch.nn.functional as F

from . import ops
from .paged import PagedKVPool


@dataclass
class Request:
    """One submitted sequence. The field names are the reference's (callers read `output`, `blocks`, `finished`).

    blocks: the physical cache blocks this request owns, in sequence order; empty while it waits (never started,
            or preempted and stripped of its blocks).
    cached: how many of its tokens (prompt, then generated) already have their keys and values stored in those
            blocks; the next token written goes to position `cached`."""
    id: int
    prompt: List[int]
    max_new_tokens: int
    eos_id: Optional[int] = None
    temperature: float = 0.0
    output: List[int] = field(default_factory=list)
    blocks: List[int] = field(default_factory=list)
    cached: int = 0
    finished: bool = False


class Scheduler:
    """The reference's continuous-batching scheduler (engine.py:36-139) over an abstract forward step.

    Subclasses provide `self.pool` (a PagedKVPool), `self.cfg` and `_forward_rows(reqs, idx, positions, tables)`,
    which runs one model step for the given rows and returns one sampled token per row."""

    def _init_scheduler(self, max_batch: int, seed: int) -> None:
        self.max_batch = max_batch
        self.generator = torch.Generator().manual_seed(seed)
        self.waiting: Deque[Request] = deque()
        self.running: List[Request] = []
        self.requests: Dict[int, Request] = {}
        self.steps = self.preemptions = self.peak_running = self.peak_blocks = 0

    # ---- public API ------------------------------------------------------------------------------------
    def add_request(self, prompt: List[int], max_new_tokens: int, eos_id: Optional[int] = None,
                    temperature: float = 0.0) -> int:
        if not 0 < len(prompt) < self.cfg.max_seq_len:
            raise ValueError(f"prompt length must be in 1..{self.cfg.max_seq_len - 1}")
        if self.pool.blocks_for(len(prompt) + 1) > self.pool.allocator.num_blocks:
            raise ValueError("prompt does not fit in the block pool")
        req = Request(len(self.requests), list(prompt), max_new_tokens, eos_id, temperature)
        self.requests[req.id] = req
        self.waiting.append(req)
        return req.id

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def run(self) -> Dict[int, List[int]]:
        """Step until every request is finished. Returns the generated tokens of each request.

        A subclass that can run several decode steps without waiting for each step's tokens (`_windowed`,
        `_decode_window`: PipelineEngine over NCCL ranks) takes them a window at a time; the outputs, block
        tables and counters are those of stepping one by one."""
        while self.has_work():
            w = self._window_steps() if self._windowed() else 0
            if w >= 2:
                self._decode_window(w)
            else:
                self.step()
        return {rid: r.output for rid, r in self.requests.items()}

    def step(self) -> None:
        self.steps += 1
        if self.waiting and len(self.running) < self.max_batch and self._try_prefill():
            pass
        elif self.running:
            self._decode()
        elif self.waiting:
            raise RuntimeError("the head request cannot be scheduled: the block pool is too small")
        self._record_peaks()

    # ---- scheduling ------------------------------------------------------------------------------------
    def _try_prefill(self) -> bool:
        req = self.waiting[0]
        # a preempted request comes back with the tokens it already generated: they are re-encoded with the prompt
        tokens = req.prompt + req.output
        need = self.pool.blocks_for(len(tokens))
        if need > self.pool.allocator.num_free:
            return False
        self.waiting.popleft()
        req.blocks = self.pool.allocator.allocate(need)
        positions = torch.arange(len(tokens))[None]
        token = self._forward_rows([req], torch.tensor([tokens]), positions, torch.tensor([req.blocks]))[0]
        req.cached = len(tokens)
        self._append(req, token)
        if not req.finished:
            self.running.append(req)
        return True

    def _grant_blocks(self) -> None:
        """Every running request writes one token at position `cached`; give a block to those that need one,
        preempting the most recently started request while the pool is empty (engine.py:100-120)."""
        bs = self.pool.block_size
        i = 0
        while i < len(self.running):
            req = self.running[i]
            if req.cached % bs == 0 and req.cached // bs == len(req.blocks):
                if self.pool.allocator.num_free == 0:
                    if len(self.running) == 1:
                        raise RuntimeError("the block pool is too small to hold even one sequence of this length")
                    victim = self.running.pop()
                    self.pool.allocator.release(victim.blocks)
                    victim.blocks, victim.cached = [], 0
                    self.waiting.appendleft(victim)
                    self.preemptions += 1
                    if victim is not req and not self.running:
                        return
                    continue                             # retry: a block is free now (or req itself left)
                req.blocks += self.pool.allocator.allocate(1)
            i += 1

    def _decode(self) -> None:
        self._grant_blocks()
        if not self.running:
            return
        width = max(len(r.blocks) for r in self.running)
        tables = torch.tensor([r.blocks + [0] * (width - len(r.blocks)) for r in self.running])
        positions = torch.tensor([[r.cached] for r in self.running])
        idx = torch.tensor([[r.output[-1]] for r in self.running])
        rows = list(self.running)
        tokens = self._forward_rows(rows, idx, positions, tables)
        for req, tok in zip(rows, tokens):
            req.cached += 1
            self._append(req, tok)
            if req.finished:
                self.running.remove(req)

    def _forward_rows(self, reqs: List[Request], idx: torch.Tensor, positions: torch.Tensor,
                      tables: torch.Tensor) -> List[int]:
        raise NotImplementedError

    # ---- decode windows ----------------------------------------------------------------------------------
    def _windowed(self) -> bool:
        """Whether `_decode_window` can run now (the subclass's execution conditions)."""
        return False

    def _decode_window(self, w: int) -> None:
        raise NotImplementedError

    def _window_steps(self) -> int:
        """How many decode steps, from the next one on, the scheduler takes over the current running rows whatever
        tokens they sample; 0 if the next step is not a decode of rows that are all greedy with no eos.

        Without eos, a row finishes when its length says so (max_new_tokens, max_seq_len), and the block grants
        (_grant_blocks) depend on lengths only; a prefill that cannot get its blocks now cannot later in the window,
        since grants only take blocks. The window ends at the first step where a row finishes, or before the first
        step whose grants would find the pool empty (the step-by-step scheduler preempts there)."""
        if not self.running or any(r.temperature != 0 or r.eos_id is not None for r in self.running):
            return 0
        if self.waiting and len(self.running) < self.max_batch:
            head = self.waiting[0]
            if self.pool.blocks_for(len(head.prompt) + len(head.output)) <= self.pool.allocator.num_free:
                return 0                                 # the next step prefills
        w = min(min(r.max_new_tokens - len(r.output), self.cfg.max_seq_len - len(r.prompt) - len(r.output))
                for r in self.running)
        bs, free = self.pool.block_size, self.pool.allocator.num_free
        nblocks = [len(r.blocks) for r in self.running]
        for t in range(w):
            for i, r in enumerate(self.running):
                pos = r.cached + t
                if pos % bs == 0 and pos // bs == nblocks[i]:
                    if free == 0:
                        return t
                    free -= 1
                    nblocks[i] += 1
        return w

    def _window_step(self, rows: List[Request], cached: List[int], t: int, last: bool):
        """Step t of a decode window over `rows` (their cache lengths `cached` at the window's start): the step's
        block grants in row order, as _grant_blocks makes them (none preempts inside a window), its counters, and
        the (block tables, positions) that _decode would pass for it."""
        self.steps += 1
        bs = self.pool.block_size
        for req, c in zip(rows, cached):
            if (c + t) % bs == 0 and (c + t) // bs == len(req.blocks):
                req.blocks += self.pool.allocator.allocate(1)
        if not last:                                     # as step() records them after a decode with no finish
            self._record_peaks()
        width = max(len(r.blocks) for r in rows)
        tables = torch.tensor([r.blocks + [0] * (width - len(r.blocks)) for r in rows])
        positions = torch.tensor([[c + t] for c in cached])
        return tables, positions

    def _window_end(self, rows: List[Request], tokens: List[List[int]]) -> None:
        """Append a window's tokens (tokens[t][i]: step t, row i) as _decode appends them step by step."""
        for t, step_tokens in enumerate(tokens):
            for req, tok in zip(rows, step_tokens):
                req.cached += 1
                self._append(req, tok)
                if req.finished:
                    if t != len(tokens) - 1:
                        raise RuntimeError("a row finished inside a decode window")
                    self.running.remove(req)
        self._record_peaks()

    def _record_peaks(self) -> None:
        used = self.pool.allocator.num_blocks - self.pool.allocator.num_free
        self.peak_running = max(self.peak_running, len(self.running))
        self.peak_blocks = max(self.peak_blocks, used)

    def _argmax(self, logits: torch.Tensor) -> torch.Tensor:
        return ops.argmax(logits)

    def _sample_rows(self, logits: torch.Tensor, reqs: List[Request]) -> List[int]:
        """One token per row of logits (R, V): greedy rows by one argmax kernel, the others from the engine's
        generator in row order."""
        greedy = self._argmax(logits).cpu().tolist()
        out = []
        for r, req in enumerate(reqs):
            if req.temperature == 0:
                out.append(int(greedy[r]))
            else:
                probs = F.softmax(logits[r].float() / req.temperature, dim=-1).cpu()
                out.append(int(torch.multinomial(probs[None], 1, generator=self.generator)[0, 0]))
        return out

    def _append(self, req: Request, token: int) -> None:
        req.output.append(token)
        total = len(req.prompt) + len(req.output)
        if len(req.output) >= req.max_new_tokens or token == req.eos_id or total >= self.cfg.max_seq_len:
            req.finished = True
            self.pool.allocator.release(req.blocks)
            req.blocks = []


class _DecodeGraph:
    """One decode step of `rows` greedy rows (one new token each) captured as a CUDA graph: embedding, every layer,
    final norm, head of the last position and argmax, over static device buffers for the token ids, positions and
    block tables (tables padded with block 0 to max_seq_len / block_size columns, as the reference pads them,
    engine.py:122). The kernels read positions from device memory, so one graph serves every step with that
    many rows; a step costs one host-to-device copy, one replay and one 8-byte-per-row copy back.

    The first step runs eagerly on the graph's stream (it is a real step, and it sets up that stream's GEMM tile
    counter and split-K workspace), then the same work is captured without running it."""

    def __init__(self, model, pool: PagedKVPool, rows: int):
        self.model, self.pool, self.rows = model, pool, rows
        self.width = -(-model.cfg.max_seq_len // pool.block_size)
        dev = model.device
        n = rows * (2 + self.width)
        self.host = torch.zeros(n, dtype=torch.int64).pin_memory()
        self.inp = torch.zeros(n, dtype=torch.int64, device=dev)
        self.idx = self.inp[:rows].view(rows, 1)
        self.pos = self.inp[rows : 2 * rows].view(rows, 1)
        self.tab = self.inp[2 * rows :].view(rows, self.width)
        self.out_host = torch.empty(rows, dtype=torch.int64).pin_memory()
        self.stream = torch.cuda.Stream(dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.tokens: Optional[torch.Tensor] = None
        # decode windows: per step of a window, its positions and block table (pinned, one slot per step, so that no
        # slot is rewritten while its copy may still be pending) and its tokens on the device
        self.ring: Optional[torch.Tensor] = None
        self.wtok: Optional[torch.Tensor] = None
        self.wtok_host: Optional[torch.Tensor] = None
        self._w = 0

    def _step(self) -> torch.Tensor:
        from .model import layer_forward_
        m = self.model
        cos, sin = m._rope.on(m.device)
        x = ops.embed(self.idx, m.tok_emb.weight)
        for layer, view in zip(m.layers, self.pool.views(self.tab, self.pos)):
            layer_forward_(layer, x, self.pos, view, cos, sin)
        return ops.argmax(m.head(x)[:, -1])

    def _capture(self) -> torch.Tensor:
        """First step of this row count: run it eagerly on the graph's stream, then capture the same work."""
        out = self._step()
        self.stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.tokens = self._step()
        self.graph = g
        return out

    # ---- decode windows: several steps in a row with no host synchronisation between them
    def begin_window(self, idx0: torch.Tensor, w: int) -> None:
        """Start a window of w steps; idx0 (rows,) are the first step's token ids. Each later step takes its ids
        from the previous step's argmax on the device."""
        r, dev = self.rows, self.model.device
        if self.ring is None or self.ring.shape[0] < w:
            n = max(w, Engine.MAX_WINDOW)
            self.ring = torch.zeros(n, r * (1 + self.width), dtype=torch.int64).pin_memory()
            self.wtok = torch.empty(n, r, dtype=torch.int64, device=dev)
            self.wtok_host = torch.empty(n, r, dtype=torch.int64).pin_memory()
        self._w = w
        self.host[:r].copy_(idx0.reshape(-1))
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            self.idx.copy_(self.host[:r].view(r, 1), non_blocking=True)

    def window_step(self, t: int, positions: torch.Tensor, tables: torch.Tensor) -> None:
        """Enqueue step t of the window (its positions and block tables planned on the host)."""
        r = self.rows
        slot = self.ring[t]
        slot.zero_()
        slot[:r].copy_(positions.reshape(-1))
        slot[r:].view(r, self.width)[:, : tables.shape[1]].copy_(tables)
        with torch.cuda.stream(self.stream):
            self.inp[r:].copy_(slot, non_blocking=True)
            if t > 0:
                self.idx.copy_(self.wtok[t - 1].view(r, 1))
            if self.graph is None:
                out = self._capture()
            else:
                self.graph.replay()
                out = self.tokens
            self.wtok[t].copy_(out)

    def end_window(self) -> List[List[int]]:
        """Wait for the window's steps; their tokens, step by step."""
        w = self._w
        with torch.cuda.stream(self.stream):
            self.wtok_host[:w].copy_(self.wtok[:w], non_blocking=True)
        self.stream.synchronize()
        torch.cuda.current_stream(self.model.device).wait_stream(self.stream)
        return self.wtok_host[:w].tolist()

    def run(self, idx: torch.Tensor, positions: torch.Tensor, tables: torch.Tensor) -> List[int]:
        r = self.rows
        self.host.zero_()
        self.host[:r].copy_(idx.reshape(-1))
        self.host[r : 2 * r].copy_(positions.reshape(-1))
        self.host[2 * r :].view(r, self.width)[:, : tables.shape[1]].copy_(tables)
        cur = torch.cuda.current_stream(self.model.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self.inp.copy_(self.host, non_blocking=True)
            if self.graph is None:
                out = self._capture()
            else:
                self.graph.replay()
                out = self.tokens
            self.out_host.copy_(out, non_blocking=True)
        self.stream.synchronize()
        cur.wait_stream(self.stream)
        return self.out_host.tolist()


class Engine(Scheduler):
    """Continuous batching of one model on one GPU (forgeserve/engine.py:36-45).

    cuda_graphs=True (extra): decode steps whose rows are all greedy replay a captured CUDA graph per row count
    (_DecodeGraph) instead of launching every kernel from Python; the tokens are the same. run() then also takes
    decode windows (_decode_window): runs of greedy steps that the scheduler can plan ahead go to the GPU back to
    back, without a host synchronisation per step. A tensor-parallel model (its all-reduces run through
    torch.distributed) always launches eagerly and steps one at a time.

    Under tensor parallelism every shard runs the same Engine over its own model shard (model.tp): the pool holds
    the shard's KV heads, the logits are replicated, so every shard samples the same tokens (engine.py:36-45 with
    the TP model of model.py:112)."""

    MAX_GRAPHS = 4
    MAX_WINDOW = 64     # decode steps per window: bounds what the host enqueues ahead of the GPU

    def __init__(self, model, num_blocks: int, block_size: int = 16, max_batch: int = 8, seed: int = 0,
                 cuda_graphs: bool = True):
        self.model, self.cfg = model, model.cfg
        self.pool = PagedKVPool(self.cfg, num_blocks, block_size, tp=model.tp, dtype=model.dtype, device=model.device)
        self.cuda_graphs = cuda_graphs
        self._graphs: Dict[int, _DecodeGraph] = {}
        self.windows = 0    # decode windows run (see _decode_window)
        self._init_scheduler(max_batch, seed)

    def _graph(self, rows: int) -> "_DecodeGraph":
        g = self._graphs.pop(rows, None)
        if g is None:
            if len(self._graphs) >= self.MAX_GRAPHS:
                self._graphs.pop(next(iter(self._graphs)))
            g = _DecodeGraph(self.model, self.pool, rows)
        self._graphs[rows] = g
        return g

    def _forward_rows(self, reqs, idx, positions, tables):
        if (self.cuda_graphs and self.pool.device.type == "cuda" and idx.shape[1] == 1 and self.model.tp.size == 1
                and all(r.temperature == 0 for r in reqs)
                and tables.shape[1] * self.pool.block_size <= self.cfg.max_seq_len + self.pool.block_size):
            return self._graph(idx.shape[0]).run(idx, positions, tables)
        logits = self.model(idx, positions, self.pool.views(tables, positions), last_only=True)
        return self._sample_rows(logits[:, -1], reqs)

    # ---- decode windows (extra): greedy steps planned ahead and replayed back to back ---------------------------
    def _windowed(self) -> bool:
        return self.cuda_graphs and self.pool.device.type == "cuda" and self.model.tp.size == 1

    def _window_steps(self) -> int:
        return min(super()._window_steps(), self.MAX_WINDOW)

    def _decode_window(self, w: int) -> None:
        """w decode steps of the running rows (all greedy, no eos: the scheduler's window, Scheduler._window_steps)
        with no host synchronisation between them: the host plans step t + 1 (block grants, tables, positions)
        while the GPU runs step t, each step's token ids come from the previous step's argmax on the device, and
        the window's tokens are read back once at its end. Same outputs, tables and counters as stepping."""
        self.windows += 1
        rows = list(self.running)
        cached = [r.cached for r in rows]
        g = self._graph(len(rows))
        g.begin_window(torch.tensor([r.output[-1] for r in rows]), w)
        for t in range(w):
            tables, positions = self._window_step(rows, cached, t, t == w - 1)
            g.window_step(t, positions, tables)
        self._window_end(rows, g.end_window())
