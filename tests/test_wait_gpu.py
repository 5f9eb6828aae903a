"""A bounded device wait that runs out: the kernel gives up, flags FS_ERR_WAIT_TIMEOUT and returns, and the GPU
keeps working. fs_wait_selftest waits, through the same bounded mbarrier wait the tensor-core kernels use, on a
barrier that never completes, with a limit of a few milliseconds instead of the kernels' 2 s. No fault, no trap:
the failure is a wait that nothing satisfies."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import _lib as L
from forgeserve_b200 import ops


def selftest(limit_ns):
    out = torch.full((2,), -1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    L.check(L.load().fs_wait_selftest(limit_ns, ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(stream.cuda_stream)), "fs_wait_selftest")
    e1.record(stream)
    e1.synchronize()
    return out.cpu().tolist(), e0.elapsed_time(e1)


@pytest.mark.parametrize("limit_ms", [2, 20])
def test_a_wait_that_runs_out_flags_the_timeout_and_returns(limit_ms):
    assert L.device_error(clear=True) == 0
    (waited_ns, completed), ms = selftest(limit_ms * 1_000_000)
    assert completed == 0
    assert waited_ns >= limit_ms * 1_000_000                 # it waited the whole limit ...
    assert ms < limit_ms + 500                                # ... and then returned, far inside the kernels' 2 s
    assert L.device_error(clear=True) == L.FS_ERR_WAIT_TIMEOUT
    assert L.device_error(clear=True) == 0                    # cleared


def test_the_gpu_keeps_working_after_a_timed_out_wait():
    selftest(5_000_000)
    assert L.device_error(clear=True) == L.FS_ERR_WAIT_TIMEOUT
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randn(300, 512, device="cuda", generator=g).bfloat16()
    w = (torch.randn(768, 512, device="cuda", generator=g) * 0.05).bfloat16()
    got = ops.linear(a, w).float()                            # the tcgen05 GEMM, right after the timed-out kernel
    want = a.double() @ w.double().t()
    assert (got.double() - want).abs().max().item() < 2e-2 * want.abs().max().item()
    assert L.device_error(clear=True) == 0
