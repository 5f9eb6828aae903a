"""Pipeline parallelism (forgeserve/pipeline.py:26-137): consecutive layer ranges per stage, one process (one
GPU) per stage, GPipe micro-batches flowing stage to stage.

Kept from the reference: the stage split, which stage holds the embedding and the head, the micro-batch rows
(torch.tensor_split of the batch), one KV cache per (micro-batch, local layer), positions
state.length + arange(t) for every row, logits for every position on the last stage, and the generation loop
(last stage samples, tokens broadcast from it).

B200 specifics: a stage's layers run as sm_100a kernels on its GPU; activations move by NCCL send/recv over
NVLink (see transport.py) with every receive posted up front, so micro-batch i+1's compute is enqueued while
micro-batch i is in flight; the last stage writes each micro-batch's logits into one preallocated output
instead of concatenating at the end; optional CUDA events per micro-batch measure the real bubble.

Extras, all with the same results: the output head split over the stages by vocab range (split_head_);
micro-batches pushed through in pieces along the sequence (pipeline_forward's seq_chunks), which shrinks the
pipeline's fill and drain; greedy generation without a drain after every token (a token ring from the last stage
to the first); and tensor parallelism inside the stages (PipelineStage's tp, transport.make_grid).
"""

from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn

from . import ops
from .config import ModelConfig
from .kv import ContiguousKV
from .model import Block, RMSNorm, RopeTables, layer_forward_
from .parallel import SINGLE, TPContext
from .sampling import sample
from .tensor_parallel import shard_state_dict
from .transport import default_transport
from .weights import open_state_dict


def stage_layers(n_layers: int, size: int) -> List[Tuple[int, int]]:
    """Consecutive layer ranges [lo, hi), as even as possible (earlier stages take the extra layers)."""
    if size > n_layers:
        raise ValueError("more pipeline stages than layers")
    base, extra = divmod(n_layers, size)
    bounds = [0]
    for r in range(size):
        bounds.append(bounds[-1] + base + (r < extra))
    return list(zip(bounds[:-1], bounds[1:]))


def bubble_fraction(stages: int, microbatches: int) -> float:
    """Share of stage time spent waiting while the pipeline fills and drains: (p - 1) / (m + p - 1)."""
    return (stages - 1) / (microbatches + stages - 1)


HEAD_TILE = 256   # output columns of one GEMM tile: head slices start and end on tile edges


def head_bounds(vocab: int, size: int) -> List[Tuple[int, int]]:
    """Vocab range [lo, hi) of each stage's slice of a split output head: whole 256-column GEMM tiles, as even as
    possible (earlier stages take the extra tiles); the ranges cover [0, vocab) in order."""
    tiles = -(-vocab // HEAD_TILE)
    base, extra = divmod(tiles, size)
    bounds, at = [], 0
    for r in range(size):
        n = base + (r < extra)
        bounds.append((min(at * HEAD_TILE, vocab), min((at + n) * HEAD_TILE, vocab)))
        at += n
    return bounds


def split_head_program(rank: int, size: int, microbatches: int) -> List[Tuple[str, int]]:
    """Host order of one stage's work in pipeline_forward when the output head is split over the stages.

    ("recv", i) / ("send", i): post the receive of micro-batch i's activation from the previous stage / its send
    to the next; ("bcast", j): post the broadcast of micro-batch j's normalised hidden state (the last stage
    sends, the others receive); ("layers", i): the stage's layers on micro-batch i (the last stage then applies
    the final norm); ("head", j): this stage's vocab slice of micro-batch j's logits.

    Stage s runs micro-batch i in slot i + s of the GPipe schedule, so the last stage's broadcast of j (after its
    layers on j, slot j + p - 1) arrives while stage s runs micro-batch j + p - 1 - s: stage s posts it before
    that micro-batch and takes j's head slice after it; slices whose input comes after the stage's last
    micro-batch run at the end, in the drain. Every rank posts its communication in one global order (a
    stage's send of micro-batch i and the last stage's broadcast, ends of slots, ordered by slot and then by
    stage from last to first), which NCCL needs when several communicators share a GPU: their kernels are not
    guaranteed to run at the same time, so a rank that posted them in another order could wait forever."""
    m, p, s = microbatches, size, rank
    out: List[Tuple[str, int]] = []
    for i in range(m):
        if s > 0:
            out.append(("recv", i))
        j = i + s + 1 - p
        if s < p - 1 and j >= 0:
            out.append(("bcast", j))
        out.append(("layers", i))
        if s < p - 1:
            out.append(("send", i))
            if j >= 0:
                out.append(("head", j))
        else:
            out += [("bcast", i), ("head", i)]
    if s < p - 1:
        for j in range(max(0, m + s + 1 - p), m):
            out += [("bcast", j), ("head", j)]
    return out


def ring_program(rank: int, size: int, microbatches: int, items: int) -> List[Tuple[str, int]]:
    """Host order of one stage's work in overlapped greedy decoding (pipeline_generate with overlap).

    Item k = (t - 1) * m + j feeds token t-1 of micro-batch j through the stages and yields token t. Ops:
    ("tok_recv", k) on stage 0 / ("tok_send", k) on the last stage: token k (item k's input) over the ring
    link last -> first; ("act_recv", k) / ("act_send", k): item k's activation from / to the neighbour;
    ("compute", k): the stage's part of item k (stage 0 embeds, the last stage applies the head and takes the
    argmax). With m >= p micro-batches, stage s runs item k in slot k + s: token k is ready at the end of the last
    stage's slot k - m + p - 1 <= k - 1, so stage 0 never waits for it. Every rank posts its communication in one
    global order (the slot boundary, then the sending stage), which NCCL needs across communicators."""
    m, p, s = microbatches, size, rank
    if m < p:
        raise ValueError("overlapped decoding needs at least as many micro-batches as stages")
    ops: List[Tuple[int, int, str, int]] = []   # (time, sending stage, op, item)
    if s == p - 1:
        for k in range(min(m, items)):             # the prefill's tokens start the ring
            ops.append((0, p - 1, "tok_send", k))
    for k in range(items):
        if s == 0:
            ops.append((0 if k < m else k - m + p, p - 1, "tok_recv", k))
        else:
            ops.append((k + s, s - 1, "act_recv", k))
        ops.append((k + s, p + 1, "compute", k))     # after the slot's receives, before its sends
        if s < p - 1:
            ops.append((k + s + 1, s, "act_send", k))
        elif k + m < items:
            ops.append((k + s + 1, p - 1, "tok_send", k + m))
    ops.sort()
    return [(op, k) for _, _, op, k in ops]


def microbatch_sizes(batch: int, microbatches: int) -> List[int]:
    """Row counts of torch.arange(batch).tensor_split(microbatches): the first batch % m parts get one extra."""
    base, extra = divmod(batch, microbatches)
    return [base + (i < extra) for i in range(microbatches)]


class PipelineStage(nn.Module):
    """Stage `rank` of `size`: layers stage_layers(cfg.n_layers, size)[rank], the embedding on the first stage, the
    final norm and an untied copy of the output head on the last (pipeline.py:44-58).

    `device` / `dtype` build the stage in place (default: the current CUDA device if there is one, fp32).
    `transport` defaults to the torch.distributed default group (or the thread's hub in run_in_threads).

    tp (extra): tensor parallelism inside the stage (the reference runs stages whole, SINGLE, pipeline.py:50):
    this process holds shard tp.rank of the stage's layers, and load_from_full cuts the weights to it. Build the
    stage's tp and transport with transport.make_grid (a stages x shards grid of processes)."""

    def __init__(self, cfg: ModelConfig, rank: int, size: int, device=None, dtype=None, transport=None,
                 tp: TPContext = SINGLE):
        super().__init__()
        self.cfg, self.rank, self.size, self.tp = cfg, rank, size, tp
        self.lo, self.hi = stage_layers(cfg.n_layers, size)[rank]
        self.is_first, self.is_last = rank == 0, rank == size - 1
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        f = dict(device=device, dtype=dtype)
        self.layers = nn.ModuleList(Block(cfg, tp, **f) for _ in range(self.hi - self.lo))
        if self.is_first:
            self.tok_emb = nn.Embedding(cfg.vocab_size, cfg.d_model, **f)
        if self.is_last:
            self.norm = RMSNorm(cfg.d_model, cfg.norm_eps, **f)
            self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False, **f)
        self._rope = RopeTables(cfg)
        self.register_buffer("rope_cos", self._rope.cos.to(device), persistent=False)
        self.register_buffer("rope_sin", self._rope.sin.to(device), persistent=False)
        if tp.size > 1 and transport is None:
            raise ValueError("a tensor-parallel stage needs the transport of its grid (transport.make_grid): the "
                             "default one pairs neighbouring world ranks, not the same shard of neighbouring stages")
        self.transport = transport if transport is not None else default_transport()
        self.trace: Optional[List] = None   # set to a list to record (mb, start, end) CUDA events per micro-batch
        self.head_split: Optional[_HeadSplit] = None   # see split_head_

    @property
    def device(self) -> torch.device:
        return self.rope_cos.device

    @property
    def dtype(self) -> torch.dtype:
        return next(self.parameters()).dtype

    def load_from_full(self, full: Dict[str, torch.Tensor]) -> None:
        """Take this stage's weights out of a full model's state dict, renumbering layers.i -> layers.(i - lo)."""
        own = {}
        for name, w in full.items():
            if name.startswith("layers."):
                i = int(name.split(".")[1])
                if self.lo <= i < self.hi:
                    own[name.replace(f"layers.{i}.", f"layers.{i - self.lo}.", 1)] = w
            elif (name == "tok_emb.weight" and self.is_first) or (name in ("norm.weight", "lm_head.weight")
                                                                  and self.is_last):
                own[name] = w
        if self.tp.size > 1:
            own = shard_state_dict(own, self.cfg, self.tp.rank, self.tp.size)
        self.load_state_dict(own)
        hs = self.head_split
        if hs is not None and not self.is_last and "lm_head.weight" in full:
            hs.weight.copy_(full["lm_head.weight"][hs.lo : hs.hi])

    def load_from_file(self, path) -> None:
        """load_from_full on a state dict saved with torch.save, memory-mapped (weights.open_state_dict): only
        this stage's tensors are read from the file, so no process holds the whole model in host memory."""
        self.load_from_full(open_state_dict(path))

    def split_head_(self, transfer: str = "copy") -> None:
        """Spread the output head over all stages. Collective: every stage calls it once its weights are set.

        Each stage then keeps the lm_head rows of its vocab range (head_bounds). In pipeline_forward with logits
        for every position, the last stage broadcasts each micro-batch's normalised hidden state and every stage
        computes its slice of the logits into the last stage's output over NVLink. The logits are the same (bit
        for bit) as with the whole head on the last stage; they are still returned on the last stage only. This
        evens out the stages: with the whole head, the last stage carries the head GEMM (2 * d_model * vocab FLOP
        per token) on top of its layers and sets the pace of the pipeline.

        transfer="copy": a stage computes its slice locally and the copy engine moves it (rows of the slice are
        contiguous runs of the output) on a side stream, overlapped with the stage's next work. "store": the GEMM
        epilogue stores the slice straight into the last stage's memory (fewer HBM bytes, but the SMs wait on
        NVLink: every thread stores 64-byte pieces of different rows). Needs one process per GPU with an NCCL
        process group."""
        if transfer not in ("copy", "store"):
            raise ValueError("transfer must be 'copy' or 'store'")
        import torch.distributed as dist
        from .transport import DistTransport
        if not (isinstance(self.transport, DistTransport) and dist.is_initialized()
                and dist.get_backend() == "nccl" and self.size > 1):
            raise RuntimeError("split_head_ needs one process per GPU and an NCCL process group of 2 or more ranks")
        hs = _HeadSplit(self)
        cfg = self.cfg
        full = self.lm_head.weight.data if self.is_last else torch.empty(
            cfg.vocab_size, cfg.d_model, dtype=self.dtype, device=self.device)
        dist.broadcast(full, src=self.size - 1, group=hs.group)
        hs.weight = full[hs.lo : hs.hi] if self.is_last else full[hs.lo : hs.hi].clone()
        hs.peer_store = transfer == "store"
        self.head_split = hs

    def _rope_tables(self):
        return self._rope.on(self.device)

    def run_layers_(self, x: torch.Tensor, positions: torch.Tensor, caches: List) -> torch.Tensor:
        """The stage's layers on x (b, t, d) in place; positions (b, t) int64 on the stage's device."""
        cos, sin = self._rope_tables()
        for layer, kv in zip(self.layers, caches):
            layer_forward_(layer, x, positions, kv, cos, sin)
        return x

    @torch.no_grad()
    def run_layers(self, x, positions, caches: List[ContiguousKV]):
        ops.require_cuda(x)
        pos = torch.as_tensor(positions).to(device=x.device, dtype=torch.int64).contiguous()
        return self.run_layers_(x.contiguous().clone(), pos, caches)

    def embed(self, idx: torch.Tensor) -> torch.Tensor:
        return ops.embed(idx, self.tok_emb.weight)

    def head(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return ops.linear(ops.rmsnorm(x, self.norm.weight, self.norm.eps), self.lm_head.weight, out=out)


class _HeadSplit:
    """A stage's part of the split output head: its vocab range and lm_head rows, the communicator the last stage
    broadcasts on, and this process's mappings of the last stage's logits buffers."""

    MAX_MAPS = 4

    def __init__(self, stage: "PipelineStage"):
        from .transport import head_group
        self.group = head_group()
        self.lo, self.hi = head_bounds(stage.cfg.vocab_size, stage.size)[stage.rank]
        self.weight: Optional[torch.Tensor] = None
        self.peer_store = False
        self.side = torch.cuda.Stream(stage.device)
        self.copy = torch.cuda.Stream(stage.device)
        self.maps: Dict[bytes, int] = {}   # IPC handle -> mapped base address, oldest first

    def logits_address(self, handle: bytes) -> int:
        key = bytes(handle[: ops.L.FS_IPC_HANDLE_BYTES])
        base = self.maps.pop(key, None)
        if base is None:
            if len(self.maps) >= self.MAX_MAPS:   # drop the oldest mapping once no queued work can still use it
                torch.cuda.synchronize(self.side.device)
                old = next(iter(self.maps))
                ops.ipc_close(self.maps.pop(old))
            base = ops.ipc_open(key)
        self.maps[key] = base
        return base + int.from_bytes(bytes(handle[ops.L.FS_IPC_HANDLE_BYTES :]), "little", signed=True)


class PipelineState:
    """One KV cache per local layer for each micro-batch (each micro-batch is a fixed set of batch rows)."""

    def __init__(self, stage: PipelineStage, batch: int, microbatches: int):
        self.sizes = microbatch_sizes(batch, microbatches)
        self.caches = [[ContiguousKV(stage.cfg.max_seq_len) for _ in stage.layers] for _ in self.sizes]
        self._length = 0

    @property
    def length(self) -> int:
        return self.caches[0][0].length if self.caches[0] else self._length


_POS_CACHE: Dict[Tuple, torch.Tensor] = {}


def _positions(start: int, t: int, rows: int, device) -> torch.Tensor:
    """Positions start .. start + t - 1 for every row, made on the device (a copy from pageable host memory would
    make the host wait for the stream, once per new decode step)."""
    key = (str(device), start, t, rows)
    p = _POS_CACHE.get(key)
    if p is None:
        if len(_POS_CACHE) > 256:
            _POS_CACHE.clear()
        p = torch.arange(start, start + t, dtype=torch.int64, device=device)[None, :].expand(rows, t).contiguous()
        _POS_CACHE[key] = p
    return p


# Sequence pieces start at multiples of this many tokens: the attention kernels tile queries in blocks of 128 from
# the first new token, so pieces aligned to it see the same query blocks (and key tiles) as the whole sequence.
SEQ_PIECE_QUANTUM = 128
# ... and give the projection GEMMs more than 128 rows (rows x piece length): from 129 rows on they always take the
# 2-SM kernel with whole-K accumulation, as the whole sequence does (128 rows or fewer take the 1-SM kernel and may
# split K, which sums in another order).
PIECE_MIN_ROWS = 129


def seq_pieces(t: int, pieces: int, rows: int = 1) -> List[Tuple[int, int]]:
    """[c0, c1) ranges splitting t new tokens of `rows` rows into at most `pieces` parts whose starts are multiples
    of SEQ_PIECE_QUANTUM and each of which has at least PIECE_MIN_ROWS rows x tokens (a short last part joins the
    one before it); one part if t is too short."""
    q = SEQ_PIECE_QUANTUM
    min_len = -(-PIECE_MIN_ROWS // max(rows, 1))    # tokens per piece for enough GEMM rows
    min_len = -(-min_len // q) * q                   # ... as a whole number of quanta
    n = max(1, min(pieces, t // min_len))
    if n == 1:
        return [(0, t)]
    per = -(-t // n)                                  # ceil(t / n)
    step = -(-per // q) * q                           # rounded up to the quantum (>= min_len, as n <= t // min_len)
    bounds, c0 = [], 0
    while c0 < t:
        bounds.append((c0, min(c0 + step, t)))
        c0 += step
    if len(bounds) > 1 and rows * (bounds[-1][1] - bounds[-1][0]) < PIECE_MIN_ROWS:
        bounds[-2:] = [(bounds[-2][0], t)]
    return bounds


def _reserve_caches(stage: PipelineStage, caches: List, rows: int, t: int) -> None:
    """Give a micro-batch's contiguous caches room for all t new tokens before its first piece, so that later
    pieces never grow (and copy) them."""
    cfg = stage.cfg
    for kv in caches:
        if isinstance(kv, ContiguousKV):     # the stage's own KV heads (all of them, or its tensor-parallel share)
            kv.reserve(rows, cfg.n_kv_heads // stage.tp.size, cfg.head_dim, t, stage.dtype, stage.device)


@torch.no_grad()
def pipeline_forward(stage: PipelineStage, state: PipelineState, idx: Optional[torch.Tensor], t: int,
                     last_only: bool = False, seq_chunks: int = 1):
    """Push t new tokens per row through the pipeline. `idx` (B, t) is needed on stage 0 only.

    Returns the logits (B, t, vocab) on the last stage (on its device) and None elsewhere.
    last_only=True computes the head for the last position only and returns (B, 1, vocab).

    seq_chunks (extra): every stage calls with the same value. Each micro-batch goes through the pipeline in up to
    this many pieces along the sequence (seq_pieces). A piece needs the keys and values of the earlier pieces of its
    rows, which the stage's caches hold by the time it arrives, so the schedule carries m * pieces items instead of
    m and its fill and drain, (p - 1) / (m * pieces + p - 1) of the time, shrink. Every kernel on the path treats
    rows independently and the pieces keep the attention tiles aligned, so the logits are the same."""
    cfg = stage.cfg
    start = state.length
    if start + t > cfg.max_seq_len:
        raise IndexError(f"positions up to {start + t - 1} exceed the rotary table of max_seq_len {cfg.max_seq_len}")
    dev = stage.device
    tr = stage.transport
    batch = sum(state.sizes)
    d = cfg.d_model
    act_dtype = stage.dtype
    recvs = {}
    split = stage.head_split is not None and not last_only
    pieces = seq_pieces(t, seq_chunks, min(state.sizes) if state.sizes else 1)
    items = [(mb, c0, c1) for mb in range(len(state.sizes)) for c0, c1 in pieces]
    if not stage.is_first and all(state.sizes) and not split:
        for k, (mb, c0, c1) in enumerate(items):
            buf = torch.empty(state.sizes[mb], c1 - c0, d, dtype=act_dtype, device=dev)
            recvs[k] = (tr.irecv(buf, stage.rank - 1), buf)
    if stage.is_first:
        idx = torch.as_tensor(idx)
        if idx.shape != (batch, t):
            raise ValueError(f"idx must have shape ({batch}, {t})")
        if idx.device.type == "cpu" and idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= cfg.vocab_size):
            raise IndexError("token id out of range for the embedding")
        idx = idx.to(device=dev, dtype=torch.int64, non_blocking=True)
    out = None
    if stage.is_last:
        out = torch.empty(batch, 1 if last_only else t, cfg.vocab_size, dtype=act_dtype, device=dev)
    stream = torch.cuda.current_stream(dev) if stage.trace is not None else None
    if any(size == 0 for size in state.sizes):
        # The reference fails on a zero-row micro-batch (its attention reshapes an empty tensor,
        # forgeserve/model.py:77); refuse up front, on every stage, instead of part-way through.
        raise RuntimeError(f"more micro-batches ({len(state.sizes)}) than batch rows ({batch})")
    if split:
        _forward_split_head(stage, state, idx, t, start, out, items)
        if not state.caches[0]:
            state._length = start + t
        return out
    sends = []
    rows0 = [sum(state.sizes[:j]) for j in range(len(state.sizes))]
    for k, (mb, c0, c1) in enumerate(items):
        size, row = state.sizes[mb], rows0[mb]
        if stage.is_first:
            x = stage.embed(idx[row : row + size, c0:c1])
        else:
            work, x = recvs.pop(k)
            work.wait()
        if stage.trace is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        if len(pieces) > 1 and c0 == 0:
            _reserve_caches(stage, state.caches[mb], size, t)
        stage.run_layers_(x, _positions(start + c0, c1 - c0, size, dev), state.caches[mb])
        if stage.is_last:
            if last_only:
                if c1 == t:
                    stage.head(x[:, -1:], out=out[row : row + size])
            elif len(pieces) == 1:
                stage.head(x, out=out[row : row + size])
            else:                                    # a piece's positions of each row are contiguous in `out`
                for b in range(size):
                    stage.head(x[b : b + 1], out=out[row + b : row + b + 1, c0:c1])
        else:
            sends.append(tr.isend(x, stage.rank + 1))
        if stage.trace is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record(stream)
            stage.trace.append((mb, e0, e1))
    for work in sends:
        work.wait()
    if not state.caches[0]:
        state._length = start + t
    return out


def _forward_split_head(stage: PipelineStage, state: PipelineState, idx: Optional[torch.Tensor], t: int,
                        start: int, out: Optional[torch.Tensor], items: List[Tuple[int, int, int]]) -> None:
    """pipeline_forward with the output head split over the stages (PipelineStage.split_head_), in the host order
    of split_head_program over `items` (micro-batch, first and end position of a sequence piece)."""
    import torch.distributed as dist
    cfg, hs, tr = stage.cfg, stage.head_split, stage.transport
    dev, p, r = stage.device, stage.size, stage.rank
    sizes = state.sizes
    rows0 = [sum(sizes[:j]) for j in range(len(sizes))]
    V, elt = cfg.vocab_size, torch.tensor([], dtype=stage.dtype).element_size()
    stream = torch.cuda.current_stream(dev)
    # Where the last stage's logits are: its IPC handle, broadcast on a side stream so that no queued compute is
    # waited for (the receivers block on the host until it arrives).
    with torch.cuda.stream(hs.side):
        if stage.is_last:
            hb = torch.frombuffer(bytearray(ops.ipc_handle(out)), dtype=torch.uint8).to(dev)
        else:
            hb = torch.empty(ops.L.FS_IPC_HANDLE_BYTES + 8, dtype=torch.uint8, device=dev)
        dist.broadcast(hb, src=p - 1, group=hs.group)
        logits_at = None if stage.is_last else hs.logits_address(bytes(hb.cpu().tolist()))
    acts: Dict[int, Tuple] = {}
    xn: Dict[int, Tuple] = {}
    sends, keep = [], []

    def mark():
        if stage.trace is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    whole = len(items) == len(sizes)          # one piece per micro-batch: a slice's rows are evenly spaced in out
    for kind, k in split_head_program(r, p, len(items)):
        j, c0, c1 = items[k]
        rows, tc = slice(rows0[j], rows0[j] + sizes[j]), c1 - c0
        if kind == "recv":
            # Posted from the side stream (the transfer does not wait for queued compute); the buffer comes from
            # that stream's pool and is marked as used by the compute stream.
            with torch.cuda.stream(hs.side):
                buf = torch.empty(sizes[j], tc, cfg.d_model, dtype=stage.dtype, device=dev)
                acts[k] = (tr.irecv(buf, r - 1), buf)
            buf.record_stream(stream)
        elif kind == "layers":
            if stage.is_first:
                x = stage.embed(idx[rows, c0:c1])
            else:
                work, x = acts.pop(k)
                work.wait()
            e0 = mark()
            if not whole and c0 == 0:
                _reserve_caches(stage, state.caches[j], sizes[j], t)
            stage.run_layers_(x, _positions(start + c0, tc, sizes[j], dev), state.caches[j])
            if stage.is_last:
                xn[k] = (None, ops.rmsnorm(x, stage.norm.weight, stage.norm.eps))
            else:
                acts[k] = (None, x)
            if e0 is not None:
                stage.trace.append((j, e0, mark()))
        elif kind == "send":
            sends.append(tr.isend(acts.pop(k)[1], r + 1))
        elif kind == "bcast":
            if stage.is_last:
                h = xn[k][1]
            else:
                h = torch.empty(sizes[j], tc, cfg.d_model, dtype=stage.dtype, device=dev)
            xn[k] = (dist.broadcast(h, src=p - 1, group=hs.group, async_op=True), h)
        else:
            work, h = xn.pop(k)
            if not stage.is_last:
                work.wait()
            keep.append(h)
            if hs.hi > hs.lo:
                e0 = mark()
                # this stage's columns of the logits of row b of micro-batch j, positions c0.. (rows of V elements)
                base = (out.data_ptr() if stage.is_last else logits_at) + hs.lo * elt
                at = [base + ((rows0[j] + b) * t + c0) * V * elt for b in range(sizes[j])]
                if whole and stage.is_last:
                    ops.linear(h, hs.weight, out=out[rows, :, hs.lo : hs.hi])
                elif hs.peer_store and not stage.is_last:
                    if whole:
                        ops.linear_to(h, hs.weight, at[0], V, system_fence=True)
                    else:
                        for b in range(sizes[j]):
                            ops.linear_to(h[b], hs.weight, at[b], V, system_fence=True)
                else:
                    part = ops.linear(h, hs.weight)
                    hs.copy.wait_stream(stream)
                    with torch.cuda.stream(hs.copy):
                        if whole:                  # the micro-batch's rows follow one another in out
                            ops.copy_2d_to(at[0], V * elt, part)
                        else:
                            for b in range(sizes[j]):
                                ops.copy_2d_to(at[b], V * elt, part[b])
                    part.record_stream(hs.copy)
                if e0 is not None:
                    stage.trace.append((j, e0, mark()))
    # Every stage reports once its slices are written (copies included); the last stage's stream waits for all of
    # them before the logits are used.
    stream.wait_stream(hs.copy)
    done = torch.zeros(1, dtype=torch.float32, device=dev)
    work = dist.all_reduce(done, group=hs.group, async_op=True)
    if stage.is_last:
        work.wait()
    for w in sends:
        w.wait()


def _overlap_possible(stage: PipelineStage, microbatches: int, temperature: float) -> bool:
    import torch.distributed as dist
    from .transport import DistTransport
    return (temperature == 0 and stage.size > 1 and microbatches >= stage.size
            and isinstance(stage.transport, DistTransport) and dist.is_initialized()
            and dist.get_backend() == "nccl")


@torch.no_grad()
def _generate_overlapped(stage: PipelineStage, prompt: torch.Tensor, n: int, microbatches: int,
                         seq_chunks: int = 1) -> torch.Tensor:
    """Greedy generation without draining the pipeline after every token (ring_program): after the prefill, the
    last stage sends each micro-batch's new tokens straight to the first stage, which starts that micro-batch's
    next step while the other stages still work on the other micro-batches. Same tokens as the step-by-step
    loop; the full token matrix is broadcast from the last stage once, at the end."""
    import torch.distributed as dist
    from .transport import ring_group
    p, r = stage.size, stage.rank
    b, T = prompt.shape
    dev, tr = stage.device, stage.transport
    state = PipelineState(stage, b, microbatches)
    sizes = state.sizes
    m = len(sizes)
    rows0 = [sum(sizes[:j]) for j in range(m)]
    toks = torch.zeros(b, T + n, dtype=torch.int64, device=dev)
    toks[:, :T].copy_(prompt.to(dev))
    logits = pipeline_forward(stage, state, toks[:, :T] if stage.is_first else None, T, last_only=True,
                              seq_chunks=seq_chunks)
    if stage.is_last:
        toks[:, T].copy_(ops.argmax(logits[:, -1]))
    del logits
    items = (n - 1) * m   # item k feeds token k // m of micro-batch k % m and yields the next one
    ring = ring_group()
    tok_in, act_in, act_out, sends = {}, {}, {}, []
    for op, k in ring_program(r, p, m, items):
        j, t = k % m, k // m
        rows = slice(rows0[j], rows0[j] + sizes[j])
        if op == "tok_send":
            buf = toks[rows, T + t].contiguous()
            sends.append((dist.isend(buf, dst=0, group=ring), buf))
        elif op == "tok_recv":
            buf = torch.empty(sizes[j], dtype=torch.int64, device=dev)
            tok_in[k] = (dist.irecv(buf, src=p - 1, group=ring), buf)
        elif op == "act_recv":
            buf = torch.empty(sizes[j], 1, stage.cfg.d_model, dtype=stage.dtype, device=dev)
            act_in[k] = (tr.irecv(buf, r - 1), buf)
        elif op == "act_send":
            sends.append((tr.isend(act_out.pop(k), r + 1), None))
        else:
            if stage.is_first:
                work, tb = tok_in.pop(k)
                work.wait()
                x = stage.embed(tb.view(-1, 1))
            else:
                work, x = act_in.pop(k)
                work.wait()
            if stage.trace is not None:
                e0 = torch.cuda.Event(enable_timing=True)
                e0.record(torch.cuda.current_stream(dev))
            stage.run_layers_(x, _positions(T + t, 1, sizes[j], dev), state.caches[j])
            if stage.is_last:
                toks[rows, T + t + 1].copy_(ops.argmax(stage.head(x)[:, -1]))
            else:
                act_out[k] = x
            if stage.trace is not None:
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record(torch.cuda.current_stream(dev))
                stage.trace.append((j, e0, e1))
    for work, _ in sends:
        work.wait()
    tr.broadcast(toks, src=p - 1)
    return toks


@torch.no_grad()
def pipeline_generate(stage: PipelineStage, prompt: torch.Tensor, max_new_tokens: int, microbatches: int = 1,
                      temperature: float = 0.0, generator=None, overlap: Optional[bool] = None,
                      seq_chunks: int = 1) -> torch.Tensor:
    """Generate with the pipeline. Every stage calls this with the same `prompt` (B, T) and gets the same result
    (on the prompt's device). The last stage samples; the tokens are broadcast from it (pipeline.py:121-137).

    overlap (extra): greedy decoding with at least as many micro-batches as stages, one process per GPU over
    NCCL, can overlap successive steps (_generate_overlapped) instead of draining the pipeline after every token;
    None picks it whenever it applies. The tokens are the same either way.
    seq_chunks (extra): the prompt's forward goes through the pipeline in pieces along the sequence
    (pipeline_forward's seq_chunks); the tokens are the same."""
    b, t = prompt.shape
    max_new_tokens = min(max_new_tokens, stage.cfg.max_seq_len - t)
    possible = _overlap_possible(stage, microbatches, temperature)
    if overlap and not possible:
        raise ValueError("overlapped decoding needs temperature 0, micro-batches >= stages >= 2, and NCCL ranks")
    if (overlap is None or overlap) and possible and max_new_tokens > 0:
        return _generate_overlapped(stage, prompt, max_new_tokens, microbatches, seq_chunks).to(prompt.device)
    state = PipelineState(stage, b, microbatches)
    dev = stage.device
    toks = torch.empty(b, t + max(max_new_tokens, 0), dtype=torch.int64, device=dev)
    toks[:, :t].copy_(prompt.to(dev))
    idx, new = toks[:, :t], t
    for i in range(max_new_tokens):
        logits = pipeline_forward(stage, state, idx if stage.is_first else None, new, last_only=True,
                                  seq_chunks=seq_chunks if i == 0 else 1)
        if stage.is_last:
            nxt = sample(logits[:, -1], temperature, generator).to(torch.int64)
        else:
            nxt = torch.empty(b, dtype=torch.int64, device=dev)
        stage.transport.broadcast(nxt, src=stage.size - 1)
        toks[:, t + i].copy_(nxt)
        idx, new = toks[:, t + i : t + i + 1], 1
    return toks.to(prompt.device)
