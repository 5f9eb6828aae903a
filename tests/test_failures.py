"""Failure detection without a GPU fault: a rank that raises, a rank that never joins its peer, on gloo."""

import time

import pytest


def raising_worker(rank, size):
    if rank == 1:
        raise ValueError("boom on rank 1")
    return rank


def stuck_worker(rank, size):
    import torch
    import torch.distributed as dist
    if rank == 0:
        t = torch.zeros(4)
        dist.recv(t, src=1)            # rank 1 never sends: the process-group timeout ends this with an error
    else:
        time.sleep(30)
    return rank


def ok_worker(rank, size):
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(rank + 1)])
    dist.all_reduce(t)
    return float(t)


def test_results_ordered_by_rank():
    from forgeserve_b200.tensor_parallel import run_distributed
    assert run_distributed(ok_worker, 3, backend="gloo") == [6.0, 6.0, 6.0]


def test_a_failing_rank_is_reported_not_hung():
    from forgeserve_b200.tensor_parallel import run_distributed
    with pytest.raises(RuntimeError, match="rank 1 failed"):
        run_distributed(raising_worker, 2, backend="gloo", timeout=60)


def test_a_missing_peer_ends_with_an_error():
    from forgeserve_b200.tensor_parallel import run_distributed
    t0 = time.time()
    with pytest.raises(RuntimeError, match="rank 0 failed|no result"):
        run_distributed(stuck_worker, 2, backend="gloo", timeout=60, pg_timeout=3)
    assert time.time() - t0 < 60


def test_thread_ranks_report_failures():
    from forgeserve_b200.tensor_parallel import run_in_threads
    with pytest.raises(RuntimeError, match="rank 1 failed"):
        run_in_threads(raising_worker, 2, timeout=10)


def test_wait_selftest_rejects_limits_outside_its_range_on_the_host():
    """Argument checks of the bounded-wait self-test answer before anything touches a GPU."""
    import ctypes
    from forgeserve_b200 import _lib as L
    lib = L.load()
    out = ctypes.c_void_p(16)
    assert lib.fs_wait_selftest(10, out, None) == -1
    assert b"limit_ns" in lib.fs_last_error()
    assert lib.fs_wait_selftest(3_000_000_000, out, None) == -1
    assert lib.fs_wait_selftest(1_000_000, None, None) == -1
    assert b"NULL" in lib.fs_last_error()
