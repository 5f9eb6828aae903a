"""How pipeline stages exchange activations and sampled tokens.

`DistTransport` is the multi-process path: torch.distributed point-to-point over NCCL (GPU tensors, NVLink
through NVSwitch on a B200 node) or gloo (CPU tensors; a CUDA tensor is staged through host memory). With
NCCL, `isend`/`irecv` run on the process group's internal stream for that pair of ranks and `wait()` only makes
the caller's current stream wait, so the host keeps enqueueing the next micro-batch while an activation is
in flight (forgeserve/pipeline.py:107-117 does the same with blocking gloo calls).

`LocalTransport` runs all stages as threads of one process on one device (`run_in_threads`): activations are
handed over by reference through queues, and every stage thread uses the same CUDA stream, so the order in
which the threads enqueue work is the order in which it runs.
"""

import os
import queue
import threading
from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist


class _Done:
    def wait(self, timeout=None):
        return True

    def is_completed(self):
        return True


class _HostStagedRecv:
    def __init__(self, work, host: torch.Tensor, dst: torch.Tensor):
        self.work, self.host, self.dst = work, host, dst

    def wait(self, timeout=None):
        self.work.wait()
        self.dst.copy_(self.host)
        return True


# One process group per pair of neighbouring ranks, shared by every DistTransport of the process. With one
# communicator (and NCCL stream) per pair, a stage's receives from rank-1 and its sends to rank+1 never queue
# behind each other; on a single group NCCL serialises all point-to-point ops of a rank on one stream.
_PAIR_GROUPS: Dict[int, list] = {}

# NCCL kernels stay resident on the SMs they run on while a receive waits for its data. Pipeline stages keep a
# few SMs out of the persistent GEMM grid for them, and cap NCCL's point-to-point channels to match.
COMM_SMS = int(os.environ.get("FORGESERVE_COMM_SMS", "12"))
PAIR_GEMM = os.environ.get("FORGESERVE_PAIR_GEMM", "1") != "0"


# The split output head (pipeline.py) uses one more communicator over all ranks: the last stage broadcasts each
# micro-batch's normalised hidden state on it, and every stage reports there when its logits slices are written.
# Its kernels are kept to a few CTAs, like the point-to-point ones, so they fit beside the persistent GEMM.
_HEAD_GROUPS: Dict[int, object] = {}
HEAD_CTAS = int(os.environ.get("FORGESERVE_HEAD_CTAS", "8"))


def head_group():
    world = dist.get_world_size()
    if world not in _HEAD_GROUPS:
        opts = None
        if dist.get_backend() == "nccl":
            opts = dist.ProcessGroupNCCL.Options()
            opts.config.max_ctas = HEAD_CTAS
        _HEAD_GROUPS[world] = dist.new_group(list(range(world)), pg_options=opts)
    return _HEAD_GROUPS[world]


# Overlapped greedy decoding (pipeline.py) sends each new token from the last stage straight to the first over a
# communicator of its own (with two stages this is a second communicator between the same two ranks).
_RING_GROUPS: Dict[int, object] = {}


def ring_group():
    world = dist.get_world_size()
    if world not in _RING_GROUPS:
        _RING_GROUPS[world] = dist.new_group([0, world - 1])
    return _RING_GROUPS[world]


def _pair_groups():
    world = dist.get_world_size()
    if world not in _PAIR_GROUPS:
        # One channel per point-to-point pair: a middle stage both receives and sends every item, and with two
        # channels each its GEMMs ran 12 % slower than the end stages' (4 GPUs, 4 sequence pieces: 238.7k tokens/s;
        # one channel: all stages equal, 248.6k). One channel still moves an item far faster than a stage computes it.
        os.environ.setdefault("NCCL_MAX_P2P_NCHANNELS", "1")
        # every rank creates every pair group, in the same order (new_group is collective over the world)
        _PAIR_GROUPS[world] = [dist.new_group([i, i + 1]) for i in range(world - 1)]
    return _PAIR_GROUPS[world]


class DistTransport:
    def __init__(self, group=None):
        self.group = group
        self.pairs = None
        if group is None and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            self.pairs = _pair_groups()
            if dist.get_backend() == "nccl" and torch.cuda.is_available():
                # A CTA pair needs two free SMs of one GPC, and NCCL kernels resident on scattered SMs delay some
                # pairs; the GEMMs claim their tiles at run time, so a late pair just takes fewer tiles.
                # FORGESERVE_PAIR_GEMM=0 keeps stages on single-CTA tiles.
                _reserve_sms_for_nccl()

    def _group_with(self, peer: int):
        if self.pairs is None:
            return self.group
        me = dist.get_rank()
        lo = min(me, peer)
        if abs(me - peer) != 1:
            return self.group
        return self.pairs[lo]

    def isend(self, t: torch.Tensor, dst: int):
        return _isend(t, dst, self._group_with(dst))

    def irecv(self, buf: torch.Tensor, src: int):
        return _irecv(buf, src, self._group_with(src))

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        if not dist.is_initialized():      # a one-stage pipeline in a process without a group: t is already here
            return
        _broadcast(t, src, self.group)


# Point-to-point and broadcast on one group. gloo moves host tensors only: a CUDA tensor is staged through host
# memory (the send keeps its host copy alive until it completes; the receive copies into the CUDA buffer on wait).
def _isend(t: torch.Tensor, dst: int, group):
    if t.is_cuda and dist.get_backend(group) == "gloo":
        t = t.to("cpu")
    return _KeepAlive(dist.isend(t, dst=dst, group=group), t)


def _irecv(buf: torch.Tensor, src: int, group):
    if buf.is_cuda and dist.get_backend(group) == "gloo":
        host = torch.empty(buf.shape, dtype=buf.dtype)
        return _HostStagedRecv(dist.irecv(host, src=src, group=group), host, buf)
    return dist.irecv(buf, src=src, group=group)


def _broadcast(t: torch.Tensor, src: int, group) -> None:
    if t.is_cuda and dist.get_backend(group) == "gloo":
        host = t.to("cpu")
        dist.broadcast(host, src=src, group=group)
        t.copy_(host)
    else:
        dist.broadcast(t, src=src, group=group)


def _reserve_sms_for_nccl() -> None:
    """Keep SMs out of the persistent GEMM grid for resident NCCL kernels (see COMM_SMS)."""
    from . import ops
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    ops.set_persistent_sms(max(sms - COMM_SMS, 1))
    ops.set_gemm_pair_mode(PAIR_GEMM)


class GridTransport:
    """Pipeline transport for `stages` x `shards` processes, tensor parallelism inside every stage: global rank =
    stage * shards + shard. After its all-reduces every shard of a stage holds the whole activation, so shard r of
    stage s sends to shard r of stage s + 1, over a process group of those two ranks; broadcasts (sampled tokens)
    go down the shard's column of stages. Built by `make_grid`, which also gives the stage's TPContext.
    Peers are stage indices, as PipelineStage uses them."""

    def __init__(self, stage: int, shard: int, stages: int, shards: int, pairs: Dict[int, object], column):
        self.stage, self.shard, self.stages, self.shards = stage, shard, stages, shards
        self.pairs, self.column = pairs, column      # pairs[s]: this shard's group of stages s and s + 1
        self.group = column

    def _rank(self, stage: int) -> int:
        return stage * self.shards + self.shard

    def _pair(self, peer: int):
        if abs(peer - self.stage) != 1:
            raise ValueError("a stage exchanges activations with its neighbours only")
        return self.pairs[min(peer, self.stage)]

    def isend(self, t: torch.Tensor, dst: int):
        return _isend(t, self._rank(dst), self._pair(dst))

    def irecv(self, buf: torch.Tensor, src: int):
        return _irecv(buf, self._rank(src), self._pair(src))

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        _broadcast(t, self._rank(src), self.column)


def make_grid(stages: int, shards: int):
    """Process groups of a stages x shards grid over the whole torch.distributed world, created collectively (every
    rank calls this, in the same order). Returns this rank's (stage, TPContext of its stage's shards,
    GridTransport): build the stage as PipelineStage(cfg, stage, stages, tp=tp, transport=transport)."""
    from .parallel import TPContext
    world, me = dist.get_world_size(), dist.get_rank()
    if world != stages * shards:
        raise ValueError(f"a {stages} x {shards} grid needs {stages * shards} ranks, the world has {world}")
    stage, shard = divmod(me, shards)
    os.environ.setdefault("NCCL_MAX_P2P_NCHANNELS", "1")     # as for the pair groups of one rank per stage
    tp_groups = [dist.new_group(list(range(s * shards, (s + 1) * shards))) for s in range(stages)]
    columns = [dist.new_group([s * shards + r for s in range(stages)]) for r in range(shards)]
    pairs = {}
    for s in range(stages - 1):
        for r in range(shards):
            g = dist.new_group([s * shards + r, (s + 1) * shards + r])
            if r == shard:
                pairs[s] = g
    if dist.get_backend() == "nccl" and torch.cuda.is_available():
        _reserve_sms_for_nccl()
    return stage, TPContext(shard, shards, group=tp_groups[stage]), GridTransport(stage, shard, stages, shards, pairs,
                                                                                  columns[shard])


class _KeepAlive:
    """Holds the sent tensor until the send completes (forgeserve/pipeline.py:114 keeps x alive the same way)."""

    def __init__(self, work, t):
        self.work, self.t = work, t

    def wait(self, timeout=None):
        self.work.wait()
        self.t = None
        return True


class LocalHub:
    """Mailboxes shared by the stage threads of one process."""

    def __init__(self, size: int, timeout: float = 120.0):
        self.size = size
        self.timeout = timeout
        self._boxes: Dict[Tuple, "queue.Queue"] = {}
        self._lock = threading.Lock()

    def box(self, key) -> "queue.Queue":
        with self._lock:
            q = self._boxes.get(key)
            if q is None:
                q = self._boxes[key] = queue.Queue()
            return q

    def get(self, key):
        try:
            return self.box(key).get(timeout=self.timeout)
        except queue.Empty:
            raise RuntimeError(f"no message {key} within {self.timeout}s (a stage thread failed or is stuck)") from None


class _LocalRecv:
    def __init__(self, hub: LocalHub, key, buf: torch.Tensor):
        self.hub, self.key, self.buf = hub, key, buf

    def wait(self, timeout=None):
        self.buf.copy_(self.hub.get(self.key))
        return True


class LocalTransport:
    def __init__(self, hub: LocalHub, rank: int):
        self.hub, self.rank = hub, rank

    def isend(self, t: torch.Tensor, dst: int):
        self.hub.box(("p2p", self.rank, dst)).put(t)
        return _Done()

    def irecv(self, buf: torch.Tensor, src: int):
        return _LocalRecv(self.hub, ("p2p", src, self.rank), buf)

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        if self.rank == src:
            for r in range(self.hub.size):
                if r != src:
                    self.hub.box(("bcast", src, r)).put(t.clone())
        else:
            t.copy_(self.hub.get(("bcast", src, self.rank)))


_local = threading.local()


def set_thread_transport(t: Optional[LocalTransport]) -> None:
    _local.transport = t


def default_transport():
    """The transport a new PipelineStage uses: the thread's LocalTransport inside `run_in_threads`, else the
    default torch.distributed process group."""
    t = getattr(_local, "transport", None)
    return t if t is not None else DistTransport()
