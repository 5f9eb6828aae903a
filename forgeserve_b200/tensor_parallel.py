"""Process launchers for the pipeline (the reference keeps `run_distributed` here, forgeserve/tensor_parallel.py:43-88).

`run_distributed(fn, size, *args, timeout)` keeps the reference's contract: fn(rank, size, *args) runs in `size`
spawned processes, results come back ordered by rank, and a rank that raises or a run that times out is
reported as RuntimeError (naming the rank) after the other ranks are terminated. The backend is NCCL with one
GPU per rank when the machine has at least `size` GPUs, else gloo on the CPU (the reference's only backend);
`backend=` overrides. NCCL process groups get a short timeout so a missing peer ends a collective with an
error instead of a hang.

`run_in_threads(fn, size, *args)` runs the ranks as threads of this process on the current GPU, exchanging
activations through a LocalHub (transport.py): a way to run a multi-stage pipeline on a single GPU.

`shard_state_dict(full, cfg, rank, size)` cuts a full model's weights into one tensor-parallel shard
(forgeserve/tensor_parallel.py:25-39), for `ForgeModel(cfg, TPContext(rank, size))`.
"""

import datetime
import os
import pickle
import socket
import threading
import traceback
from typing import Callable, Dict, List, Optional

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from .config import ModelConfig
from .transport import LocalHub, LocalTransport, set_thread_transport

# Weights split by output feature (rows of an nn.Linear weight: whole heads for q/k/v) and by input feature
# (columns: the matching slice of the attention output and of the SwiGLU hidden features).
_BY_ROWS = ("attn.wq.weight", "attn.wk.weight", "attn.wv.weight", "mlp.w_gate.weight", "mlp.w_up.weight")
_BY_COLUMNS = ("attn.wo.weight", "mlp.w_down.weight")


def shard_state_dict(full: Dict[str, torch.Tensor], cfg: ModelConfig, rank: int, size: int) -> Dict[str, torch.Tensor]:
    """Shard `rank` of `size` of a full state dict: q/k/v/gate/up keep rows [rank * n / size, (rank + 1) * n / size)
    of their n output features, wo/w_down the same range of their input columns, and the embedding, norms and head
    are replicated. Every tensor is a contiguous copy. ValueError when a head count or ffn_dim does not divide."""
    cfg.check_tensor_parallel(size)
    if not 0 <= rank < size:
        raise ValueError("rank must be in [0, size)")
    out = {}
    for name, w in full.items():
        if name.endswith(_BY_ROWS):
            n = w.shape[0] // size
            out[name] = w[rank * n : (rank + 1) * n].contiguous().clone()
        elif name.endswith(_BY_COLUMNS):
            n = w.shape[1] // size
            out[name] = w[:, rank * n : (rank + 1) * n].contiguous().clone()
        else:
            out[name] = w.clone()
    return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def pick_backend(size: int) -> str:
    return "nccl" if torch.cuda.is_available() and torch.cuda.device_count() >= size else "gloo"


def _worker(rank: int, size: int, port: int, backend: str, pg_timeout: float, fn: Callable, args: tuple,
            queue) -> None:
    torch.set_num_threads(1)     # the reference's default: one host thread per rank (tensor_parallel.py:50)
    kwargs = dict(init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=size,
                  timeout=datetime.timedelta(seconds=pg_timeout))
    if backend == "nccl":
        torch.cuda.set_device(rank % torch.cuda.device_count())
        kwargs["device_id"] = torch.device("cuda", torch.cuda.current_device())
    try:
        dist.init_process_group(backend, **kwargs)
        # pickled to bytes here: a tensor put on the queue as-is is shared through a file descriptor that the
        # parent can only fetch while this process is still alive
        queue.put((rank, pickle.dumps(fn(rank, size, *args)), None))
    except BaseException:
        queue.put((rank, None, traceback.format_exc()))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_distributed(fn: Callable, size: int, *args, timeout: float = 180.0, backend: Optional[str] = None,
                    pg_timeout: float = 60.0) -> List:
    """Run fn(rank, size, *args) in `size` processes; return their results ordered by rank.

    `fn` must be a module-level function; args and results must be picklable (CUDA results are returned as
    CPU tensors only if fn moves them)."""
    backend = backend or pick_backend(size)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, size, port, backend, pg_timeout, fn, args, queue))
             for r in range(size)]
    for p in procs:
        p.start()
    results, error = {}, None
    try:
        for _ in range(size):
            rank, res, err = queue.get(timeout=timeout)
            if err is not None:
                error = f"rank {rank} failed:\n{err}"
                break
            results[rank] = pickle.loads(res)
    except Exception as e:       # timeout: some rank is stuck, usually waiting for a peer
        error = f"no result within {timeout}s ({type(e).__name__})"
    finally:
        for p in procs:
            if error is not None and p.is_alive():
                p.terminate()
            p.join(timeout=10)
    if error is not None:
        raise RuntimeError(error)
    return [results[r] for r in range(size)]


def run_in_threads(fn: Callable, size: int, *args, timeout: float = 180.0) -> List:
    """Run fn(rank, size, *args) for every rank as threads of this process (one GPU, one CUDA stream)."""
    hub = LocalHub(size, timeout=timeout)
    results: List = [None] * size
    errors: List = [None] * size
    device = torch.cuda.current_device() if torch.cuda.is_available() else None

    def body(rank):
        if device is not None:
            torch.cuda.set_device(device)
        set_thread_transport(LocalTransport(hub, rank))
        try:
            results[rank] = fn(rank, size, *args)
        except BaseException:
            errors[rank] = traceback.format_exc()
        finally:
            set_thread_transport(None)

    threads = [threading.Thread(target=body, args=(r,), daemon=True) for r in range(size)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout)
    for r, t in enumerate(threads):
        if t.is_alive():
            raise RuntimeError(f"rank {r} did not finish within {timeout}s")
        if errors[r] is not None:
            raise RuntimeError(f"rank {r} failed:\n{errors[r]}")
    return results
