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


class DistTransport:
    def __init__(self, group=None):
        self.group = group

    @property
    def host_staged(self) -> bool:
        return dist.get_backend(self.group) == "gloo"

    def isend(self, t: torch.Tensor, dst: int):
        if t.is_cuda and self.host_staged:
            host = t.to("cpu")
            work = dist.isend(host, dst=dst, group=self.group)
            return _KeepAlive(work, host)
        return _KeepAlive(dist.isend(t, dst=dst, group=self.group), t)

    def irecv(self, buf: torch.Tensor, src: int):
        if buf.is_cuda and self.host_staged:
            host = torch.empty(buf.shape, dtype=buf.dtype)
            return _HostStagedRecv(dist.irecv(host, src=src, group=self.group), host, buf)
        return dist.irecv(buf, src=src, group=self.group)

    def broadcast(self, t: torch.Tensor, src: int) -> None:
        if t.is_cuda and self.host_staged:
            host = t.to("cpu")
            dist.broadcast(host, src=src, group=self.group)
            t.copy_(host)
        else:
            dist.broadcast(t, src=src, group=self.group)


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
